"""Helpers shared by the GPU parity tests."""
import os

import numpy as np

from linuxnightmaresuite_b200 import synth
from oracle import moe_oracle as orc

# Output tolerance of the MoE layer against the reference (f32 accumulate).
TOL_MAX_ABS = 1e-2
TOL_REL_L2 = 2e-3
# Router weights: logits differ from numpy's BLAS order at the f32 rounding
# level and expf differs from numpy's SIMD exp by a few ulp.
TOL_W_RTOL = 1e-5
TOL_W_ATOL = 1e-7
# relative k-boundary gap below which a differing k-th expert is a near-tie
NEAR_TIE = 1e-5

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def oracle_parts(data):
    cfg = data.cfg
    experts = orc.LazyExperts(data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.d_model, cfg.ffn)
    shared = None
    if cfg.shared_ffn:
        shared = orc.expert_from_blocks(data.s_gate[0], data.s_up[0], data.s_down[0],
                                        cfg.shared_qtype, cfg.d_model, cfg.shared_ffn)
    return experts, shared


def near_tie(logits: np.ndarray, k: int) -> bool:
    s = np.sort(logits.astype(np.float64))[::-1]
    if k >= s.size:
        return False
    gap = abs(s[k - 1] - s[k])
    return gap <= NEAR_TIE * max(1.0, abs(s[k - 1]))


def check_layer(x, gate_w, bias, k, mode, experts, shared, out_dev, ids_dev, w_dev,
                tokens=None, exp_out=None, exp_ids=None, exp_w=None):
    """Compare device results with the oracle on the given token rows.

    Returns the number of near-tie tokens.  Ids must match exactly except on
    near-ties, where the expected output is recomputed with the device's ids."""
    rows = list(range(x.shape[0])) if tokens is None else list(tokens)
    if exp_out is None:
        exp_out, exp_ids, exp_w, _ = orc.moe_layer(x, gate_w, experts, k, mode, shared, bias, rows)
    ties = 0
    expected = np.array(exp_out, dtype=np.float32, copy=True)
    for i, t in enumerate(rows):
        if not np.array_equal(ids_dev[t], exp_ids[i]):
            lg = orc.router_logits(x[t], gate_w, bias)
            if mode == 1:
                lg = np.exp(lg - lg.max())
            assert near_tie(lg, k), (t, ids_dev[t], exp_ids[i])
            ties += 1
            sel = ids_dev[t].astype(np.int64)
            lgt = orc.router_logits(x[t], gate_w, bias)
            if mode == 0:
                w = orc.softmax(lgt[sel])
            else:
                p = orc.softmax(lgt)
                w = p[sel] / np.sum(p[sel])
            expected[i] = orc.moe_layer_with_ids(x[t:t + 1], experts, sel[None], w[None],
                                                 shared)[0]
        else:
            np.testing.assert_allclose(w_dev[t], exp_w[i], rtol=TOL_W_RTOL, atol=TOL_W_ATOL)
    got = out_dev[rows]
    mx, rel = orc.compare(got, expected)
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)
    return ties


def make(cfg_name, seed=0, tokens=None, **kw):
    return synth.make_layer(synth.CONFIGS[cfg_name], seed, tokens=tokens, **kw)


class SliceExperts:
    """Experts of a ``synth.make_layer_slice`` layer for the oracle: each is
    generated from its own seed and dequantised the first time it is used."""

    def __init__(self, cfg, seed):
        self.cfg, self.seed = cfg, seed
        self.cache = {}

    def __getitem__(self, e):
        e = int(e)
        if e not in self.cache:
            g, u, d = synth.slice_expert(self.cfg, self.seed, e)
            self.cache[e] = orc.expert_from_blocks(g[0], u[0], d[0], self.cfg.qtype,
                                                   self.cfg.d_model, self.cfg.ffn)
        return self.cache[e]


def slice_layers(cfg, seed, tokens, n_layers):
    """Oracle layers (gate_w, experts, shared, norm_w, bias) of a stack built
    from ``make_layer_slice(cfg, seed + l, tokens, ...)``, yielded one at a
    time so that a layer's dequantised experts are freed once it is done."""
    for li in range(n_layers):
        base = synth.make_layer_slice(cfg, seed + li, tokens, 0, 0)
        shared = None
        if cfg.shared_ffn:
            shared = orc.expert_from_blocks(base.s_gate[0], base.s_up[0], base.s_down[0],
                                            cfg.shared_qtype, cfg.d_model, cfg.shared_ffn)
        yield base.gate_w, SliceExperts(cfg, seed + li), shared, base.norm_w, None


def sample_tokens(ids: np.ndarray, extra=(), per_expert: int = 1):
    """Token rows to check: ``extra`` plus, for the busiest and the rarest
    routed expert, the first ``per_expert`` tokens that route there."""
    E = int(ids.max()) + 1
    counts = np.bincount(ids.reshape(-1), minlength=E)
    busiest = int(np.argmax(counts))
    rare = int(np.argmin(np.where(counts > 0, counts, 1 << 30)))
    toks = set(int(t) for t in extra)
    for e in (busiest, rare):
        toks |= set(np.nonzero((ids == e).any(1))[0][:per_expert].tolist())
    return sorted(toks), busiest, rare, counts
