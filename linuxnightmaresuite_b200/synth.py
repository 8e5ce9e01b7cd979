"""Seeded synthetic MoE workloads, emitted as raw GGUF block bytes.

Every weight tensor is produced exactly as a GGUF file stores it and as the
reference decoders read it (``dequant_fast.py:44-100``):

* Q8_0 (GGML type 8): 34-byte blocks of 32 weights, ``[fp16 d][int8 q x 32]``,
  value ``d * q``.
* Q4_0 (GGML type 2): 18-byte blocks of 32 weights, ``[fp16 d][16 bytes]``;
  byte ``j`` holds weight ``j`` in its low nibble and weight ``j + 16`` in its
  high nibble, value ``(nibble - 8) * d``.

A 2-D weight of logical shape ``(rows, cols)`` (the reference's ``(out, in)``
orientation, ``gguf_parser.py:478-487``) is ``rows`` consecutive rows of
``cols / 32`` blocks.  An expert stack is ``E`` such matrices back to back,
which is the byte layout of a GGUF ``ffn_*_exps`` tensor with ``ne = [cols,
rows, E]`` (``nightmare_stream.py:3361-3441``).

The workload shapes follow the MoE-layer benchmark configurations: a
CPU-sized single layer, decode, ragged prefill, the expert-parallel layer and
the stacked decode step.  Inputs are deterministic functions of the seed.
"""
from __future__ import annotations

import dataclasses
import hashlib
from typing import Dict, Optional

import numpy as np

QTYPE_Q4_0 = 2
QTYPE_Q8_0 = 8

# GGML type id -> (weights per block, bytes per block); the Q4_0 / Q8_0 rows
# of dequant_fast.py:723-754.
BLOCK_GEOMETRY = {QTYPE_Q4_0: (32, 18), QTYPE_Q8_0: (32, 34)}


def block_bytes(qtype: int) -> int:
    return BLOCK_GEOMETRY[qtype][1]


def row_bytes(qtype: int, cols: int) -> int:
    if cols % 32:
        raise ValueError(f"row length {cols} is not a multiple of 32")
    return cols // 32 * block_bytes(qtype)


def _fp16_scales(rng: np.random.Generator, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n, dtype=np.float32)) * np.float32(scale)).astype(np.float16)


def q8_0_blocks(rng: np.random.Generator, n_blocks: int, scale: float) -> np.ndarray:
    """``n_blocks`` Q8_0 blocks: q ~ U[-127, 127], d = fp16(|N(0,1)| * scale)."""
    out = np.empty((n_blocks, 34), dtype=np.uint8)
    out[:, :2] = _fp16_scales(rng, n_blocks, scale).view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:] = rng.integers(-127, 128, size=(n_blocks, 32), dtype=np.int8).view(np.uint8)
    return out


def q4_0_blocks(rng: np.random.Generator, n_blocks: int, scale: float) -> np.ndarray:
    """``n_blocks`` Q4_0 blocks: nibbles ~ U[0, 15], d = fp16(|N(0,1)| * scale)."""
    out = np.empty((n_blocks, 18), dtype=np.uint8)
    out[:, :2] = _fp16_scales(rng, n_blocks, scale).view(np.uint8).reshape(n_blocks, 2)
    # A uniform byte is two independent uniform nibbles.
    out[:, 2:] = np.frombuffer(rng.bytes(n_blocks * 16), dtype=np.uint8).reshape(n_blocks, 16)
    return out


def quant_matrix(rng: np.random.Generator, qtype: int, n_mats: int, rows: int, cols: int,
                 scale: float) -> np.ndarray:
    """Raw block bytes of ``n_mats`` stacked ``(rows, cols)`` matrices, shape
    ``(n_mats, rows, cols/32 * block_bytes)``."""
    nb = n_mats * rows * (cols // 32)
    if qtype == QTYPE_Q8_0:
        blocks = q8_0_blocks(rng, nb, scale)
    elif qtype == QTYPE_Q4_0:
        blocks = q4_0_blocks(rng, nb, scale)
    else:
        raise ValueError(f"unsupported qtype {qtype}")
    return blocks.reshape(n_mats, rows, row_bytes(qtype, cols))


@dataclasses.dataclass(frozen=True)
class MoEConfig:
    """Shape and value distribution of one MoE layer workload."""
    name: str
    d_model: int
    n_experts: int
    top_k: int
    ffn: int
    tokens: int
    qtype: int
    qscale: float
    router_std: float = 0.02
    route_mode: int = 0          # 0: top-k then softmax; 1: softmax, top-k, renormalise
    zipf_s: float = 0.0          # >0: add a Zipf per-expert bias to the router logits
    zipf_max_rows: int = 1500    # bias tuned so the busiest expert gets about this many rows
    shared_ffn: int = 0
    shared_qtype: int = QTYPE_Q8_0
    shared_qscale: float = 0.002
    n_layers: int = 1


CONFIGS: Dict[str, MoEConfig] = {
    # single MoE FFN layer small enough for the CPU reference
    "cpu_layer": MoEConfig("cpu_layer", 1024, 8, 2, 2816, 4, QTYPE_Q8_0, 0.002, route_mode=1),
    # decode: HBM-bound grouped GEMV, T in {1, 8, 64}
    "decode_t1": MoEConfig("decode_t1", 2816, 128, 8, 704, 1, QTYPE_Q4_0, 0.01),
    "decode_t8": MoEConfig("decode_t8", 2816, 128, 8, 704, 8, QTYPE_Q4_0, 0.01),
    "decode_t64": MoEConfig("decode_t64", 2816, 128, 8, 704, 64, QTYPE_Q4_0, 0.01),
    # prefill: ragged groups from a Zipf(1.1) expert bias
    "prefill": MoEConfig("prefill", 2816, 128, 8, 704, 4096, QTYPE_Q8_0, 0.002, zipf_s=1.1),
    # expert-parallel layer, uniform routing
    "ep": MoEConfig("ep", 4096, 128, 8, 1536, 8192, QTYPE_Q8_0, 0.002),
    # stacked decode: 30 layers, routed Q4_0 + always-on Q8_0 shared expert
    "stacked": MoEConfig("stacked", 2816, 128, 8, 704, 256, QTYPE_Q4_0, 0.01,
                         shared_ffn=2112, n_layers=30),
}


def q5_1_blocks(rng: np.random.Generator, n_blocks: int, scale: float) -> np.ndarray:
    """Q5_1 blocks ``[fp16 d][fp16 m][u32 qh][16 B]``: uniform quants, d =
    fp16(|N(0,1)| * scale), m = fp16(-16 * d * U[0.5, 1.5])."""
    out = np.empty((n_blocks, 24), dtype=np.uint8)
    d = _fp16_scales(rng, n_blocks, scale)
    m = (-16.0 * d.astype(np.float32) * rng.uniform(0.5, 1.5, n_blocks).astype(np.float32))
    out[:, :2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = m.astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
    out[:, 4:] = np.frombuffer(rng.bytes(n_blocks * 20), dtype=np.uint8).reshape(n_blocks, 20)
    return out


def q4_k_blocks(rng: np.random.Generator, n_blocks: int, scale: float) -> np.ndarray:
    """Q4_K super-blocks ``[fp16 d][fp16 dmin][12 scale bytes][128 quant bytes]``:
    uniform 6-bit scales / mins and nibbles, d = fp16(|N| * scale / 32), dmin =
    fp16(|N| * scale / 64), so weights span about +-scale * 15."""
    out = np.empty((n_blocks, 144), dtype=np.uint8)
    out[:, :2] = _fp16_scales(rng, n_blocks, scale / 32).view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = _fp16_scales(rng, n_blocks, scale / 64).view(np.uint8).reshape(n_blocks, 2)
    out[:, 4:] = np.frombuffer(rng.bytes(n_blocks * 140), dtype=np.uint8).reshape(n_blocks, 140)
    return out


def q6_k_blocks(rng: np.random.Generator, n_blocks: int, scale: float) -> np.ndarray:
    """Q6_K super-blocks ``[ql x 128][qh x 64][int8 scales x 16][fp16 d]``:
    uniform quants, int8 scales in [-64, 63], d = fp16(|N| * scale / 64)."""
    out = np.empty((n_blocks, 210), dtype=np.uint8)
    out[:, :192] = np.frombuffer(rng.bytes(n_blocks * 192), dtype=np.uint8).reshape(n_blocks, 192)
    out[:, 192:208] = rng.integers(-64, 64, size=(n_blocks, 16), dtype=np.int8).view(np.uint8)
    out[:, 208:] = _fp16_scales(rng, n_blocks, scale / 64).view(np.uint8).reshape(n_blocks, 2)
    return out


# GGML type -> (weights per block, bytes per block) of every type the layer takes
ALL_GEOMETRY = {0: (1, 4), QTYPE_Q4_0: (32, 18), 7: (32, 24), QTYPE_Q8_0: (32, 34),
                12: (256, 144), 14: (256, 210)}


def blocks_of(rng: np.random.Generator, qtype: int, n_mats: int, rows: int, cols: int,
              scale: float) -> np.ndarray:
    """Raw blocks of ``n_mats`` stacked (rows, cols) matrices in any type the
    layer takes, shape (n_mats, rows, row bytes)."""
    be, bb = ALL_GEOMETRY[qtype]
    if cols % be:
        raise ValueError(f"{cols} columns are not whole blocks of type {qtype}")
    nb = n_mats * rows * (cols // be)
    if qtype in (QTYPE_Q4_0, QTYPE_Q8_0):
        return quant_matrix(rng, qtype, n_mats, rows, cols, scale)
    if qtype == 0:
        w = rng.standard_normal(nb, dtype=np.float32) * np.float32(scale * 40)
        return w.view(np.uint8).reshape(n_mats, rows, cols * 4)
    gen = {7: q5_1_blocks, 12: q4_k_blocks, 14: q6_k_blocks}[qtype]
    return gen(rng, nb, scale).reshape(n_mats, rows, cols // be * bb)


@dataclasses.dataclass
class Gemma4LayerData:
    """Inputs of a gemma4 MoE feed-forward block (host numpy arrays)."""
    x: np.ndarray              # (T, d) attention output
    router: np.ndarray         # (E, d) f32 moe_router
    gate_inp_scale: np.ndarray  # (d,) ffn_gate_inp.scale
    gate_up: np.ndarray        # (E, 2F, row bytes) fused Q4_K ffn_gate_up_exps
    down: np.ndarray           # (E, d, row bytes) Q5_1 ffn_down_exps
    down_scale: np.ndarray     # (E,) ffn_down_exps.scale
    s_gate: np.ndarray         # (Fs, row bytes) Q8_0 dense shared MLP
    s_up: np.ndarray
    s_down: np.ndarray
    ffn_norm: np.ndarray
    post_norm_1: np.ndarray
    pre_norm_2: np.ndarray
    post_norm_2: np.ndarray

    def digest(self) -> str:
        h = hashlib.sha256()
        for a in dataclasses.astuple(self):
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


def make_gemma4_layer(d: int, E: int, F: int, Fs: int, T: int, seed: int = 0,
                      gu_qtype: int = 12, down_qtype: int = 7) -> Gemma4LayerData:
    """A gemma4-style MoE block in the layout gemma4 GGUFs ship
    (nightmare_stream.py:3366-3370): fused gate_up Q4_K, down Q5_1 with a
    per-expert scale, a Q8_0 dense shared MLP."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((T, d), dtype=np.float32) * np.float32(4.0))
    router = rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.5)
    gis = (1.0 + 0.2 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
    gate_up = blocks_of(rng, gu_qtype, E, 2 * F, d, 0.01)
    down = blocks_of(rng, down_qtype, E, d, F, 0.01)
    down_scale = (0.5 + rng.uniform(0, 1, E)).astype(np.float32)
    s_gate = quant_matrix(rng, QTYPE_Q8_0, 1, Fs, d, 0.002)[0]
    s_up = quant_matrix(rng, QTYPE_Q8_0, 1, Fs, d, 0.002)[0]
    s_down = quant_matrix(rng, QTYPE_Q8_0, 1, d, Fs, 0.002)[0]
    norms = [(1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
             for _ in range(4)]
    return Gemma4LayerData(x, router, gis, gate_up, down, down_scale, s_gate, s_up, s_down,
                           *norms)


def zipf_bias(rng: np.random.Generator, n_experts: int, s: float, c: float) -> np.ndarray:
    """Per-expert logit bias ``c * log(rank^-s)`` over a seeded permutation of
    experts: adding the log of Zipf(s) probabilities to the logits skews the
    routing towards low ranks and starves the tail."""
    ranks = rng.permutation(n_experts).astype(np.float64) + 1.0
    return (c * (-s) * np.log(ranks)).astype(np.float32)


@dataclasses.dataclass
class MoELayerData:
    """One layer's synthetic inputs (host numpy arrays)."""
    cfg: MoEConfig
    x: np.ndarray                 # (T, d) f32
    gate_w: np.ndarray            # (d, E) f32, the reference router layout (x @ gate_w)
    bias: Optional[np.ndarray]    # (E,) f32 or None
    w_gate: np.ndarray            # (E, F, row_bytes(d)) u8
    w_up: np.ndarray              # (E, F, row_bytes(d)) u8
    w_down: np.ndarray            # (E, d, row_bytes(F)) u8
    s_gate: Optional[np.ndarray] = None   # (1, Fs, row_bytes(d)) u8 shared expert
    s_up: Optional[np.ndarray] = None
    s_down: Optional[np.ndarray] = None
    norm_w: Optional[np.ndarray] = None   # (d,) f32 RMSNorm weight (stacked layers)

    def digest(self) -> str:
        """sha256 over every input array: pins generator output in fixtures."""
        h = hashlib.sha256()
        for a in (self.x, self.gate_w, self.bias, self.w_gate, self.w_up, self.w_down,
                  self.s_gate, self.s_up, self.s_down, self.norm_w):
            if a is not None:
                h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


def make_layer(cfg: MoEConfig, seed: int = 0, tokens: Optional[int] = None,
               n_experts_built: Optional[int] = None, zipf_c: Optional[float] = None) -> MoELayerData:
    """Generate one layer.  Arrays are drawn in a fixed order so a given
    (cfg, seed) always yields the same bytes.  ``n_experts_built`` limits how
    many expert matrices are materialised (the rest are not needed by a test
    whose tokens never route there); the router still spans all experts."""
    rng = np.random.default_rng(seed)
    T = cfg.tokens if tokens is None else tokens
    d, E, F = cfg.d_model, cfg.n_experts, cfg.ffn
    gate_w = (rng.standard_normal((d, E), dtype=np.float32) * np.float32(cfg.router_std))
    x = rng.standard_normal((T, d), dtype=np.float32)
    bias = None
    if cfg.zipf_s > 0:
        c = zipf_c if zipf_c is not None else 0.0
        bias = zipf_bias(rng, E, cfg.zipf_s, 1.0)
        if zipf_c is None:
            c = tune_zipf_scale(x, gate_w, bias, cfg.top_k, cfg.zipf_max_rows)
        bias = (bias * np.float32(c)).astype(np.float32)
    Eb = E if n_experts_built is None else n_experts_built
    w_gate = quant_matrix(rng, cfg.qtype, Eb, F, d, cfg.qscale)
    w_up = quant_matrix(rng, cfg.qtype, Eb, F, d, cfg.qscale)
    w_down = quant_matrix(rng, cfg.qtype, Eb, d, F, cfg.qscale)
    data = MoELayerData(cfg, x, gate_w, bias, w_gate, w_up, w_down)
    if cfg.shared_ffn:
        Fs = cfg.shared_ffn
        data.s_gate = quant_matrix(rng, cfg.shared_qtype, 1, Fs, d, cfg.shared_qscale)
        data.s_up = quant_matrix(rng, cfg.shared_qtype, 1, Fs, d, cfg.shared_qscale)
        data.s_down = quant_matrix(rng, cfg.shared_qtype, 1, d, Fs, cfg.shared_qscale)
    if cfg.n_layers > 1:
        data.norm_w = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
    return data


def make_layer_slice(cfg: MoEConfig, seed: int, tokens: int, e0: int, e1: int) -> MoELayerData:
    """One layer whose experts are drawn from per-expert generators (seed, e),
    so a rank can build just its experts [e0, e1) and every rank agrees on
    them; the router, tokens, shared expert and norm come from (seed, E) and
    are the same on every rank.  w_* hold experts e0..e1-1 only."""
    d, E, F = cfg.d_model, cfg.n_experts, cfg.ffn
    rng = np.random.default_rng([seed, E])
    gate_w = (rng.standard_normal((d, E), dtype=np.float32) * np.float32(cfg.router_std))
    x = rng.standard_normal((tokens, d), dtype=np.float32)
    mats = [slice_expert(cfg, seed, e) for e in range(e0, e1)]
    def stack(j, rows, cols):
        if not mats:
            return np.zeros((0, rows, row_bytes(cfg.qtype, cols)), np.uint8)
        return np.concatenate([m[j] for m in mats])

    data = MoELayerData(cfg, x, gate_w, None, stack(0, F, d), stack(1, F, d), stack(2, d, F))
    if cfg.shared_ffn:
        Fs = cfg.shared_ffn
        data.s_gate = quant_matrix(rng, cfg.shared_qtype, 1, Fs, d, cfg.shared_qscale)
        data.s_up = quant_matrix(rng, cfg.shared_qtype, 1, Fs, d, cfg.shared_qscale)
        data.s_down = quant_matrix(rng, cfg.shared_qtype, 1, d, Fs, cfg.shared_qscale)
    data.norm_w = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
    return data


def slice_expert(cfg: MoEConfig, seed: int, e: int):
    """Raw (gate, up, down) blocks of expert ``e`` of a ``make_layer_slice``
    layer, each shaped (1, rows, row bytes); drawn from its own generator
    (seed, e), so any expert can be rebuilt alone."""
    d, F = cfg.d_model, cfg.ffn
    re = np.random.default_rng([seed, e, 7])
    return (quant_matrix(re, cfg.qtype, 1, F, d, cfg.qscale),
            quant_matrix(re, cfg.qtype, 1, F, d, cfg.qscale),
            quant_matrix(re, cfg.qtype, 1, d, F, cfg.qscale))


def tune_zipf_scale(x: np.ndarray, gate_w: np.ndarray, unit_bias: np.ndarray, k: int,
                    target_max: int) -> float:
    """Bisection on the bias scale so the busiest expert receives about
    ``target_max`` (token, slot) rows.  Uses a float64 top-k count; the exact
    split does not matter, only the skew."""
    logits = x.astype(np.float64) @ gate_w.astype(np.float64)
    E = gate_w.shape[1]
    target = min(target_max, x.shape[0])

    def busiest(c: float) -> int:
        lg = logits + c * unit_bias.astype(np.float64)
        top = np.argpartition(-lg, k - 1, axis=1)[:, :k]
        return int(np.bincount(top.ravel(), minlength=E).max())

    lo, hi = 0.0, 1.0
    while busiest(hi) < target and hi < 1e4:
        hi *= 2.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if busiest(mid) < target:
            lo = mid
        else:
            hi = mid
    return float(hi)


# ----------------------------------------------------------------------------
# device-side generation (benchmark workloads)
#
# The benchmark's large workloads (gigabytes of expert blocks) are drawn on the
# GPU with torch's seeded generator: same block layout and value distribution
# as above, a different random stream.  Every expert comes from its own
# generator (seed, layer, expert), so a rank builds only its experts and any
# expert can be rebuilt alone (``device_expert``) to check results on the host.
# ----------------------------------------------------------------------------

def _mix(*vals: int) -> int:
    h = 0x9E3779B97F4A7C15
    for v in vals:
        h = (h ^ (int(v) & 0xFFFFFFFFFFFFFFFF)) * 0x100000001B3 & 0xFFFFFFFFFFFFFFFF
    return h & 0x7FFFFFFFFFFFFFFF


def _device_quant(gen, qtype: int, rows: int, cols: int, scale: float, out):
    import torch
    nb = rows * (cols // 32)
    dev = out.device
    sc = (torch.randn(nb, generator=gen, device=dev).abs_() * scale).to(torch.float16)
    blk = out.view(nb, block_bytes(qtype))
    blk[:, :2] = sc.view(torch.uint8).view(nb, 2)
    if qtype == QTYPE_Q8_0:
        blk[:, 2:] = torch.randint(-127, 128, (nb, 32), generator=gen, device=dev,
                                   dtype=torch.int8).view(torch.uint8)
    elif qtype == QTYPE_Q4_0:
        blk[:, 2:] = torch.randint(0, 256, (nb, 16), generator=gen, device=dev,
                                   dtype=torch.uint8)
    else:
        raise ValueError(f"unsupported qtype {qtype}")


def _device_expert_into(cfg: MoEConfig, seed: int, layer: int, e: int, g_out, u_out, d_out):
    import torch
    gen = torch.Generator(device=g_out.device)
    gen.manual_seed(_mix(seed, layer, e))
    d, F = cfg.d_model, cfg.ffn
    _device_quant(gen, cfg.qtype, F, d, cfg.qscale, g_out)
    _device_quant(gen, cfg.qtype, F, d, cfg.qscale, u_out)
    _device_quant(gen, cfg.qtype, d, F, cfg.qscale, d_out)


def device_expert(cfg: MoEConfig, seed: int, layer: int, e: int, device):
    """Raw (gate, up, down) blocks of expert e of a device-generated layer,
    each (rows, row bytes) uint8 on ``device``."""
    import torch
    d, F = cfg.d_model, cfg.ffn
    g = torch.empty((F, row_bytes(cfg.qtype, d)), dtype=torch.uint8, device=device)
    u = torch.empty_like(g)
    dn = torch.empty((d, row_bytes(cfg.qtype, F)), dtype=torch.uint8, device=device)
    _device_expert_into(cfg, seed, layer, e, g, u, dn)
    return g, u, dn


def make_layer_device(cfg: MoEConfig, seed: int, tokens: int, e0: int, e1: int, device,
                      layer: int = 0) -> MoELayerData:
    """One layer whose experts e0..e1-1 are drawn on ``device`` (torch uint8
    tensors in w_gate / w_up / w_down / s_*); the tokens, router weights, Zipf
    bias and RMSNorm weight are host numpy arrays from (seed, layer) and are the
    same on every rank."""
    import torch
    d, E, F = cfg.d_model, cfg.n_experts, cfg.ffn
    rng = np.random.default_rng([seed, layer, E, 11])
    gate_w = (rng.standard_normal((d, E), dtype=np.float32) * np.float32(cfg.router_std))
    x = rng.standard_normal((tokens, d), dtype=np.float32)
    bias = None
    if cfg.zipf_s > 0:
        unit = zipf_bias(rng, E, cfg.zipf_s, 1.0)
        c = tune_zipf_scale(x, gate_w, unit, cfg.top_k, cfg.zipf_max_rows)
        bias = (unit * np.float32(c)).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
    El = e1 - e0
    wg = torch.empty((El, F, row_bytes(cfg.qtype, d)), dtype=torch.uint8, device=device)
    wu = torch.empty_like(wg)
    wd = torch.empty((El, d, row_bytes(cfg.qtype, F)), dtype=torch.uint8, device=device)
    for i, e in enumerate(range(e0, e1)):
        _device_expert_into(cfg, seed, layer, e, wg[i], wu[i], wd[i])
    data = MoELayerData(cfg, x, gate_w, bias, wg, wu, wd, norm_w=norm_w)
    if cfg.shared_ffn:
        Fs = cfg.shared_ffn
        gen = torch.Generator(device=device)
        gen.manual_seed(_mix(seed, layer, 1 << 20))
        sg = torch.empty((1, Fs, row_bytes(cfg.shared_qtype, d)), dtype=torch.uint8,
                         device=device)
        su = torch.empty_like(sg)
        sd = torch.empty((1, d, row_bytes(cfg.shared_qtype, Fs)), dtype=torch.uint8,
                         device=device)
        _device_quant(gen, cfg.shared_qtype, Fs, d, cfg.shared_qscale, sg[0])
        _device_quant(gen, cfg.shared_qtype, Fs, d, cfg.shared_qscale, su[0])
        _device_quant(gen, cfg.shared_qtype, d, Fs, cfg.shared_qscale, sd[0])
        data.s_gate, data.s_up, data.s_down = sg, su, sd
    return data


# ----------------------------------------------------------------------------
# synthetic GGUF models (one MoE block)
# ----------------------------------------------------------------------------

def moe_gguf_tensors(kind: str = "swiglu", seed: int = 0, d: int = 512, E: int = 16, F: int = 256,
                     Fs: int = 192, k: int = 4, block: int = 0):
    """(metadata, tensors) of a one-block MoE model in llama.cpp's tensor
    naming, for ``gguf.write_gguf``.  Shapes are ggml order (contiguous first):
    a logical (out, in) matrix is ``[in, out]``, an expert stack ``[in, out, E]``.

    kind "swiglu": ffn_gate_inp (F32), ffn_gate_exps / ffn_up_exps (Q4_0),
    ffn_down_exps (Q8_0), shared expert ffn_*_shexp (Q8_0).
    kind "gemma4": fused ffn_gate_up_exps (Q4_K), ffn_down_exps (Q5_1) with
    ffn_down_exps.scale, ffn_gate_inp.scale, dense ffn_gate/up/down (Q8_0) and
    the four norms -- the layout nightmare_stream.py:3366-3370 describes."""
    rng = np.random.default_rng([seed, 101])
    p = f"blk.{block}."
    arch = "gemma4" if kind == "gemma4" else "qwen3moe"
    meta = {"general.architecture": arch, "general.name": f"synthetic-{kind}",
            f"{arch}.embedding_length": d, f"{arch}.expert_count": E,
            f"{arch}.expert_used_count": k, f"{arch}.expert_feed_forward_length": F,
            f"{arch}.block_count": 1, f"{arch}.attention.layer_norm_rms_epsilon": 1e-6,
            "general.tags": ["synthetic", "moe"], "general.flag": True,
            "general.scale_hint": 0.5}
    router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.05))
    t = [(p + "ffn_gate_inp.weight", (d, E), 0, router.tobytes())]
    if kind == "gemma4":
        gu = blocks_of(rng, 12, E, 2 * F, d, 0.01)
        dn = blocks_of(rng, 7, E, d, F, 0.01)
        ds = (0.5 + rng.uniform(0, 1, E)).astype(np.float32)
        gis = (1.0 + 0.2 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
        t += [(p + "ffn_gate_up_exps.weight", (d, 2 * F, E), 12, gu.tobytes()),
              (p + "ffn_down_exps.weight", (F, d, E), 7, dn.tobytes()),
              (p + "ffn_down_exps.scale", (E,), 0, ds.tobytes()),
              (p + "ffn_gate_inp.scale", (d,), 0, gis.tobytes())]
        for m, (r, c) in (("gate", (Fs, d)), ("up", (Fs, d)), ("down", (d, Fs))):
            t.append((p + f"ffn_{m}.weight", (c, r), 8,
                      quant_matrix(rng, QTYPE_Q8_0, 1, r, c, 0.002).tobytes()))
        for n in ("ffn_norm", "post_ffw_norm_1", "pre_ffw_norm_2", "post_ffw_norm_2"):
            w = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
            t.append((p + f"{n}.weight", (d,), 0, w.tobytes()))
    else:
        for m in ("gate", "up"):
            t.append((p + f"ffn_{m}_exps.weight", (d, F, E), 2,
                      quant_matrix(rng, QTYPE_Q4_0, E, F, d, 0.01).tobytes()))
        t.append((p + "ffn_down_exps.weight", (F, d, E), 8,
                  quant_matrix(rng, QTYPE_Q8_0, E, d, F, 0.002).tobytes()))
        for m, (r, c) in (("gate", (Fs, d)), ("up", (Fs, d)), ("down", (d, Fs))):
            t.append((p + f"ffn_{m}_shexp.weight", (c, r), 8,
                      quant_matrix(rng, QTYPE_Q8_0, 1, r, c, 0.002).tobytes()))
    t.append(("token_embd.weight", (d, 8), 0,
              rng.standard_normal((8, d), dtype=np.float32).tobytes()))
    return meta, t
