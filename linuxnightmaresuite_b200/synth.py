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
    mats = []
    for e in range(e0, e1):
        re = np.random.default_rng([seed, e, 7])
        mats.append((quant_matrix(re, cfg.qtype, 1, F, d, cfg.qscale),
                     quant_matrix(re, cfg.qtype, 1, F, d, cfg.qscale),
                     quant_matrix(re, cfg.qtype, 1, d, F, cfg.qscale)))
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
