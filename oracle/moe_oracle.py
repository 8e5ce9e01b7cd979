"""CPU oracle for the MoE layer forward -- TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA path is compared against.  Only the test
suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it; the product path (``linuxnightmaresuite_b200``) never does.

It restates, in numpy, the reference algorithm of
NightmareDesigns/Linuxnightmaresuite for this path:

* block decoders ``dequant_fast.py:44-66`` (Q8_0) and ``:69-100`` (Q4_0);
* ``rms_norm`` / ``silu`` / ``softmax`` ``moe_forward.py:34-52``;
* router ``MoERouter.route`` ``moe_forward.py:91-109`` (top-k, then softmax
  over the k logits, descending order) and the production variant
  ``nightmare_stream.py:3227-3238`` (softmax over all experts, top-k,
  renormalise; ascending order);
* ``ExpertFFN.forward`` ``moe_forward.py:129-133``;
* ``MoELayer.forward`` ``moe_forward.py:154-174`` (weighted sum in router
  order, unweighted shared expert).

Per-token functions use the same numpy calls in the same order as the
reference, so on the same host they reproduce it bit for bit; this is pinned
by ``tests/test_oracle_golden.py`` against fixtures made by running the
reference itself (``tests/golden/make_golden.py``).

Tie rule.  The reference sorts with ``np.argsort`` (default quicksort, which
numpy may run as an unstable SIMD sort).  The oracle implements the stable
rule -- descending value, ties broken by the higher expert index first, i.e.
``argsort(kind='stable')[-k:][::-1]`` -- and reports tokens where numpy's
default sort would pick differently so tests can treat them separately.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import numpy as np

QTYPE_Q4_0 = 2
QTYPE_Q8_0 = 8
# dequant_fast.py:723-754, rows for Q4_0 and Q8_0
BLOCK_SIZES = {QTYPE_Q4_0: (32, 18), QTYPE_Q8_0: (32, 34)}


# --------------------------------------------------------------------------
# block decoders
# --------------------------------------------------------------------------

def dequantize_q8_0(data, n_elements: int) -> np.ndarray:
    """dequant_fast.py:44-66: f32 = fp16 scale * int8 quant, 34-byte blocks."""
    n_blocks = n_elements // 32
    raw = np.frombuffer(bytes(data) if not isinstance(data, np.ndarray) else data.tobytes(),
                        dtype=np.uint8).reshape(n_blocks, 34)
    scales = raw[:, :2].copy().view(np.float16).astype(np.float32).reshape(n_blocks, 1)
    quants = raw[:, 2:].copy().view(np.int8).astype(np.float32)
    return (scales * quants).reshape(-1)


def dequantize_q4_0(data, n_elements: int) -> np.ndarray:
    """dequant_fast.py:69-100: low nibbles -> weights 0-15, high nibbles ->
    16-31, value (nibble - 8) * fp16 scale, 18-byte blocks."""
    n_blocks = n_elements // 32
    raw = np.frombuffer(bytes(data) if not isinstance(data, np.ndarray) else data.tobytes(),
                        dtype=np.uint8).reshape(n_blocks, 18)
    scales = raw[:, :2].copy().view(np.float16).astype(np.float32).reshape(n_blocks, 1)
    packed = raw[:, 2:]
    low = (packed & 0x0F).astype(np.float32) - 8.0
    high = ((packed >> 4) & 0x0F).astype(np.float32) - 8.0
    quants = np.empty((n_blocks, 32), dtype=np.float32)
    quants[:, 0:16] = low
    quants[:, 16:32] = high
    return (scales * quants).reshape(-1)


QTYPE_F32 = 0
QTYPE_Q5_1 = 7
QTYPE_Q4_K = 12
QTYPE_Q6_K = 14
# dequant_fast.py:723-754 rows of the other types the layer takes
BLOCK_SIZES.update({QTYPE_F32: (1, 4), QTYPE_Q5_1: (32, 24), QTYPE_Q4_K: (256, 144),
                    QTYPE_Q6_K: (256, 210)})


def _raw_blocks(data, n_blocks, block_bytes):
    buf = data.tobytes() if isinstance(data, np.ndarray) else bytes(data)
    return np.frombuffer(buf, dtype=np.uint8).reshape(n_blocks, block_bytes)


def dequantize_f32(data, n_elements: int) -> np.ndarray:
    buf = data.tobytes() if isinstance(data, np.ndarray) else bytes(data)
    return np.frombuffer(buf, dtype=np.float32)[:n_elements].copy()


def dequantize_q5_1(data, n_elements: int) -> np.ndarray:
    """dequant_fast.py:169-201: 24-byte blocks [fp16 d][fp16 m][u32 qh][16 B];
    q = nibble (low: weights 0-15, high: 16-31) | qh bit of the weight << 4;
    value d * q + m."""
    nb = n_elements // 32
    raw = _raw_blocks(data, nb, 24)
    scales = raw[:, :2].copy().view(np.float16).astype(np.float32).reshape(nb, 1)
    mins = raw[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(nb, 1)
    qh = raw[:, 4:8].copy().view(np.uint32).reshape(nb)
    packed = raw[:, 8:]
    quants = np.empty((nb, 32), dtype=np.uint32)
    quants[:, 0:16] = (packed & 0x0F).astype(np.uint32)
    quants[:, 16:32] = ((packed >> 4) & 0x0F).astype(np.uint32)
    bits = (qh[:, None] >> np.arange(32, dtype=np.uint32)[None, :]) & 1
    quants |= (bits.astype(np.uint32) << 4)
    return (scales * quants.astype(np.float32) + mins).reshape(-1)


def _k4_scales(raw_scales, d, dmin):
    """6-bit sub-block scales / mins of a Q4_K super-block (dequant_fast.py:256-266,
    llama.cpp's get_scale_min_k4 packing), times d / dmin."""
    n = raw_scales.shape[0]
    scales = np.zeros((n, 8), dtype=np.float32)
    mins = np.zeros((n, 8), dtype=np.float32)
    for j in range(4):
        scales[:, j] = d * (raw_scales[:, j] & 0x3F).astype(np.float32)
        mins[:, j] = dmin * (raw_scales[:, j + 4] & 0x3F).astype(np.float32)
    for j in range(4):
        scales[:, 4 + j] = d * (((raw_scales[:, j + 8] & 0x0F)
                                 | ((raw_scales[:, j] >> 6) << 4)).astype(np.float32))
        mins[:, 4 + j] = dmin * (((raw_scales[:, j + 8] >> 4)
                                  | ((raw_scales[:, j + 4] >> 6) << 4)).astype(np.float32))
    return scales, mins


def dequantize_q4_k(data, n_elements: int) -> np.ndarray:
    """dequant_fast.py:237-289: 144-byte super-blocks of 256 [fp16 d][fp16 dmin]
    [12 scale bytes][128 quant bytes]; sub-block s: low (s even) / high (s
    odd) nibbles of quant bytes 32 (s // 2) ..; value scale_s * q - min_s."""
    nb = n_elements // 256
    raw = _raw_blocks(data, nb, 144)
    d = raw[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(nb)
    dmin = raw[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(nb)
    scales, mins = _k4_scales(raw[:, 4:16], d, dmin)
    qs = raw[:, 16:]
    out = np.zeros((nb, 256), dtype=np.float32)
    for g in range(4):
        sl = qs[:, g * 32:(g + 1) * 32]
        low = (sl & 0x0F).astype(np.float32)
        high = ((sl >> 4) & 0x0F).astype(np.float32)
        out[:, 64 * g:64 * g + 32] = scales[:, 2 * g, None] * low - mins[:, 2 * g, None]
        out[:, 64 * g + 32:64 * g + 64] = scales[:, 2 * g + 1, None] * high - mins[:, 2 * g + 1, None]
    return out.reshape(-1)


def dequantize_q6_k(data, n_elements: int) -> np.ndarray:
    """dequant_fast.py:343-378: 210-byte super-blocks [ql x 128][qh x 64]
    [int8 scales x 16][fp16 d]; per half of 128 weights four streams of 32
    from ql bytes l / l + 32 (low then high nibbles) and two qh bits each;
    value d * scale[p // 16] * (q - 32)."""
    nb = n_elements // 256
    raw = _raw_blocks(data, nb, 210)
    ql, qh = raw[:, :128], raw[:, 128:192]
    scales = raw[:, 192:208].view(np.int8).astype(np.float32)
    d = raw[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(nb, 1)
    out = np.zeros((nb, 256), dtype=np.float32)
    for half in range(2):
        qlh, qhh = ql[:, half * 64:(half + 1) * 64], qh[:, half * 32:(half + 1) * 32]
        sch = scales[:, half * 8:(half + 1) * 8]
        l = np.arange(32)
        q1 = ((qlh[:, l] & 0x0F) | ((qhh[:, l] >> 0) & 0x03) << 4).astype(np.float32) - 32
        q2 = ((qlh[:, l + 32] & 0x0F) | ((qhh[:, l] >> 2) & 0x03) << 4).astype(np.float32) - 32
        q3 = ((qlh[:, l] >> 4) | ((qhh[:, l] >> 4) & 0x03) << 4).astype(np.float32) - 32
        q4 = ((qlh[:, l + 32] >> 4) | ((qhh[:, l] >> 6) & 0x03) << 4).astype(np.float32) - 32
        q_all = np.concatenate([q1, q2, q3, q4], axis=1)
        out[:, half * 128:(half + 1) * 128] = d * np.repeat(sch, 16, axis=1) * q_all
    return out.reshape(-1)


DEQUANT = {QTYPE_Q4_0: dequantize_q4_0, QTYPE_Q8_0: dequantize_q8_0, QTYPE_F32: dequantize_f32,
           QTYPE_Q5_1: dequantize_q5_1, QTYPE_Q4_K: dequantize_q4_k, QTYPE_Q6_K: dequantize_q6_k}


def dequantize_matrix(raw: np.ndarray, qtype: int, rows: int, cols: int) -> np.ndarray:
    """Raw blocks of one (rows, cols) matrix -> f32 (rows, cols), the reshape
    ``gguf_parser.load_tensor`` applies (gguf_parser.py:478-487)."""
    return DEQUANT[qtype](np.ascontiguousarray(raw), rows * cols).reshape(rows, cols)


# --------------------------------------------------------------------------
# math primitives, moe_forward.py:34-52
# --------------------------------------------------------------------------

def rms_norm(x, weight, eps=1e-6, gemma_style=False):
    """moe_forward.py:34-40; gemma_style scales by (1 + weight)."""
    ms = np.mean(x * x) + eps
    normed = x / np.sqrt(ms)
    if gemma_style:
        return normed * (1.0 + weight)
    return normed * weight


def silu(x):
    return x / (1.0 + np.exp(-np.clip(x, -88, 88)))


def softmax(x):
    m = np.max(x)
    e = np.exp(x - m)
    return e / np.sum(e)


def geglu_tanh(g, u):
    """gemma4's expert activation, nightmare_stream.py:3256-3271 (the
    GPUStreamEngine._expert_act GeGLU branch): 0.5 g (1 + tanh(sqrt(2/pi)
    (g + 0.044715 g^3))) u."""
    a = np.sqrt(2.0 / np.pi) * (g + 0.044715 * g ** 3)
    return 0.5 * g * (1.0 + np.tanh(a)) * u


def gemma4_router_input(x, scale, dim, eps):
    """nightmare_stream.py:4662-4667: rms of x without weight, times
    f32(1/sqrt(dim)), times ffn_gate_inp.scale."""
    r = x.astype(np.float32)
    r = r / np.sqrt(np.mean(r * r) + eps)
    r = r * np.float32(1.0 / np.sqrt(float(dim)))
    if scale is not None:
        r = r * np.asarray(scale, dtype=np.float32)
    return r


# --------------------------------------------------------------------------
# router
# --------------------------------------------------------------------------

def stable_topk_desc(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values, descending; ties -> higher index first.
    NaN sorts above every number, as numpy's argsort places it last."""
    return np.argsort(values, kind="stable")[-k:][::-1]


def route_topk_softmax(x: np.ndarray, gate_w: np.ndarray, k: int,
                       bias: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray, bool]:
    """MoERouter.route, moe_forward.py:99-109 (mode 0).

    Returns (ids descending, weights, tie_flag).  ``tie_flag`` is True when
    numpy's default argsort would select or order differently from the stable
    rule (only possible with exactly equal logits)."""
    logits = x @ gate_w
    if bias is not None:
        logits = logits + bias
    ids = stable_topk_desc(logits, k)
    default_ids = np.argsort(logits)[-k:][::-1]
    weights = softmax(logits[ids])
    return ids.astype(np.int64), weights.astype(np.float32), bool(np.any(default_ids != ids))


def route_softmax_topk_renorm(x: np.ndarray, gate_w: np.ndarray, k: int,
                              bias: Optional[np.ndarray] = None):
    """Production routing, nightmare_stream.py:3227-3238 (mode 1): softmax over
    all experts, top-k by probability (ascending order, as argsort yields it),
    renormalise the k probabilities."""
    logits = x @ gate_w
    if bias is not None:
        logits = logits + bias
    gl_max = np.max(logits)
    exp_gl = np.exp(logits - gl_max)
    probs = exp_gl / np.sum(exp_gl)
    ids = np.argsort(probs, kind="stable")[-k:]
    default_ids = np.argsort(probs)[-k:]
    w = probs[ids]
    w = w / np.sum(w)
    return ids.astype(np.int64), w.astype(np.float32), bool(np.any(default_ids != ids))


def route(x, gate_w, k, mode=0, bias=None):
    if mode == 0:
        return route_topk_softmax(x, gate_w, k, bias)
    if mode == 1:
        return route_softmax_topk_renorm(x, gate_w, k, bias)
    raise ValueError(f"unknown routing mode {mode}")


def router_logits(x: np.ndarray, gate_w: np.ndarray, bias: Optional[np.ndarray] = None) -> np.ndarray:
    lg = x @ gate_w
    return lg if bias is None else lg + bias


# --------------------------------------------------------------------------
# experts and layer
# --------------------------------------------------------------------------

class DenseExpert:
    """ExpertFFN, moe_forward.py:116-133, on dequantised f32 weights."""

    def __init__(self, w_gate, w_up, w_down):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down

    def forward(self, x):
        gate = x @ self.w_gate.T
        up = x @ self.w_up.T
        return (silu(gate) * up) @ self.w_down.T


def expert_from_blocks(raw_gate, raw_up, raw_down, qtype, d, F, down_qtype=None) -> DenseExpert:
    return DenseExpert(dequantize_matrix(raw_gate, qtype, F, d),
                       dequantize_matrix(raw_up, qtype, F, d),
                       dequantize_matrix(raw_down, qtype if down_qtype is None else down_qtype,
                                         d, F))


class GeGLUExpert:
    """A gemma4 expert on dequantised f32 weights: down @ geglu(gate @ x, up @ x)
    (nightmare_stream.py:4686-4690), with the down matrix already multiplied
    by the expert's ffn_down_exps.scale as _load_expert_fast does
    (nightmare_stream.py:3430-3438)."""

    def __init__(self, w_gate, w_up, w_down):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down

    def forward(self, x):
        return self.w_down @ geglu_tanh(self.w_gate @ x, self.w_up @ x)


def gemma4_expert_from_blocks(raw_gate_up, gu_qtype, raw_down, down_qtype, d, F, down_scale=None):
    """nightmare_stream.py:3361-3441 (_load_expert_fast): the fused gate_up
    slice (2F, d) splits into gate = rows [0, F), up = rows [F, 2F); the down
    slice (d, F) is multiplied by the expert's scale."""
    gu = dequantize_matrix(raw_gate_up, gu_qtype, 2 * F, d)
    down = dequantize_matrix(raw_down, down_qtype, d, F)
    if down_scale is not None:
        down = down * float(down_scale)
    return GeGLUExpert(np.ascontiguousarray(gu[:F]), np.ascontiguousarray(gu[F:]), down)


def gemma4_routed(attn_out, moe_in, router, gate_inp_scale, experts, n_used, eps):
    """gemma4's routed experts for one token (nightmare_stream.py:4343-4370 and
    the expert loop of :4681-4690): router input from attn_out, softmax over
    all experts, top-k, renormalised, sum of w * expert(moe_in).  Returns
    (cur_moe, ids ascending, weights)."""
    dim = attn_out.shape[0]
    r = gemma4_router_input(attn_out, gate_inp_scale, dim, eps)
    logits = np.asarray(router, dtype=np.float32) @ r
    probs = np.exp(logits - logits.max())
    probs /= probs.sum()
    k = min(int(n_used), probs.shape[0])
    top = np.argsort(probs, kind="stable")[-k:]
    tw = probs[top]
    tw = tw / tw.sum()
    cur_moe = np.zeros(dim, dtype=np.float32)
    for e, wt in zip(top, tw):
        cur_moe += float(wt) * experts[int(e)].forward(np.asarray(moe_in, dtype=np.float32))
    return cur_moe, top, tw


def engine_moe_ffn(xn, router, experts, n_used):
    """GPUStreamEngine._moe_ffn, nightmare_stream.py:3220-3253: logits =
    router (E, d) @ xn, softmax over all experts, top-k ascending,
    renormalised, sum of w * SwiGLU expert; returns (1, dim)."""
    x = np.asarray(xn, dtype=np.float32).reshape(-1)
    logits = np.asarray(router, dtype=np.float32) @ x
    probs = np.exp(logits - np.max(logits))
    probs = probs / np.sum(probs)
    k = min(int(n_used), probs.shape[0])
    top = np.argsort(probs, kind="stable")[-k:]
    tw = probs[top] / np.sum(probs[top])
    out = np.zeros(x.shape[0], dtype=np.float32)
    for e, wt in zip(top, tw):
        out += float(wt) * experts[int(e)].forward(x)
    return out.reshape(1, -1), top, tw


def gemma4_moe_block(attn_out, w, experts, n_used, eps):
    """The MoE feed-forward of a gemma4 layer, nightmare_stream.py:4655-4693
    (CPU branch): shared GeGLU MLP on rms(attn_out, ffn_norm) with its post
    norm, plus the routed experts on rms(attn_out, pre_ffw_norm_2) with
    softmax -> top-k -> renormalised weights from the router input, and their
    post norm.  ``w``: dict with moe_router (E, d), moe_gate_inp_scale,
    ffn_norm, wg / wu (Fs, d), wd (d, Fs), post_ffw_norm_1, pre_ffw_norm_2,
    post_ffw_norm_2 (f32).  ``experts[e]`` has forward(x)."""
    dim = attn_out.shape[0]

    def rms(v, weight):
        return v / np.sqrt(np.mean(v * v) + eps) * weight

    mlp_in = rms(attn_out, w["ffn_norm"])
    g_ = (mlp_in.reshape(1, -1) @ w["wg"].T)[0]
    u_ = (mlp_in.reshape(1, -1) @ w["wu"].T)[0]
    cur_mlp = ((geglu_tanh(g_, 1.0) * u_).reshape(1, -1) @ w["wd"].T)[0]
    if w.get("post_ffw_norm_1") is not None:
        cur_mlp = rms(cur_mlp, w["post_ffw_norm_1"])
    moe_in = rms(attn_out, w["pre_ffw_norm_2"])
    cur_moe, top, tw = gemma4_routed(attn_out, moe_in, w["moe_router"],
                                     w.get("moe_gate_inp_scale"), experts, n_used, eps)
    if w.get("post_ffw_norm_2") is not None:
        cur_moe = rms(cur_moe, w["post_ffw_norm_2"])
    return cur_mlp + cur_moe, top, tw


class LazyExperts:
    """Dequantises an expert the first time a token routes to it."""

    def __init__(self, w_gate, w_up, w_down, qtype, d, F):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down
        self.qtype, self.d, self.F = qtype, d, F
        self.cache = {}

    def __getitem__(self, e) -> DenseExpert:
        e = int(e)
        if e not in self.cache:
            self.cache[e] = expert_from_blocks(self.w_gate[e], self.w_up[e], self.w_down[e],
                                               self.qtype, self.d, self.F)
        return self.cache[e]

    def __len__(self):
        return self.w_gate.shape[0]


def moe_layer_token(x, gate_w, experts, k, mode=0, shared=None, bias=None):
    """MoELayer.forward for one token, moe_forward.py:154-174.

    Returns (output, ids, weights, tie_flag)."""
    ids, weights, tie = route(x, gate_w, k, mode, bias)
    output = np.zeros_like(x)
    for eid, w in zip(ids, weights):
        expert_out = experts[eid].forward(x)
        output += w * expert_out
    if shared is not None:
        output += shared.forward(x)
    return output, ids, weights, tie


def moe_layer(xs, gate_w, experts, k, mode=0, shared=None, bias=None, tokens=None):
    """Token loop over moe_layer_token (how MoETransformerModel batches,
    moe_forward.py:261-281).  ``tokens`` selects a subset of rows."""
    rows = range(xs.shape[0]) if tokens is None else tokens
    outs, all_ids, all_w, ties = [], [], [], []
    for t in rows:
        o, ids, w, tie = moe_layer_token(xs[t], gate_w, experts, k, mode, shared, bias)
        outs.append(o)
        all_ids.append(ids)
        all_w.append(w)
        ties.append(tie)
    return (np.stack(outs), np.stack(all_ids).astype(np.int32), np.stack(all_w),
            np.array(ties, dtype=bool))


def moe_layer_with_ids(xs, experts, ids, weights, shared=None):
    """Layer output for given routing decisions (used where a near-tie lets
    the device legitimately pick a different k-th expert)."""
    out = np.zeros_like(xs)
    for t in range(xs.shape[0]):
        acc = np.zeros_like(xs[t])
        for eid, w in zip(ids[t], weights[t]):
            acc += np.float32(w) * experts[int(eid)].forward(xs[t])
        if shared is not None:
            acc += shared.forward(xs[t])
        out[t] = acc
    return out


def dispatch(ids: np.ndarray, n_experts: int):
    """Stable counting sort of (token, slot) pairs by expert.

    Returns (expert_offsets[E+1], perm_rows[P], inv_perm[P]): row r of the
    expert-sorted order holds pair perm_rows[r] = t*k + slot, and pair p sits
    at row inv_perm[p].  Within an expert, pairs keep ascending (t, slot)."""
    flat = ids.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.zeros(n_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size)
    return offsets, order.astype(np.int32), inv.astype(np.int32)


def stacked_forward(x, layers, k, mode=0):
    """Stacked decode: per layer ``x = x + moe(rms_norm(x, w))`` with the
    residual and RMSNorm of MoETransformerModel._layer_forward
    (moe_forward.py:348-359).  ``layers`` is a list of
    (gate_w, experts, shared, norm_w, bias)."""
    out = x.copy()
    for gate_w, experts, shared, norm_w, bias in layers:
        nxt = np.empty_like(out)
        for t in range(out.shape[0]):
            xn = rms_norm(out[t], norm_w).astype(np.float32)
            o, _, _, _ = moe_layer_token(xn, gate_w, experts, k, mode, shared, bias)
            nxt[t] = out[t] + o
        out = nxt
    return out


def compare(actual: np.ndarray, expected: np.ndarray) -> Tuple[float, float]:
    """(max-abs, rel-L2) of actual against expected."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    diff = a - e
    denom = np.linalg.norm(e)
    return float(np.max(np.abs(diff))) if diff.size else 0.0, \
        float(np.linalg.norm(diff) / denom) if denom > 0 else float(np.linalg.norm(diff))
