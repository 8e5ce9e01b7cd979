"""Generate the golden fixtures by running the reference implementation.

Run from the repository root, with the directory of a reference checkout as
the argument (or in ``MOE_REFERENCE_DIR``); ``--only NAME`` regenerates just
the named fixture groups:

    python tests/golden/make_golden.py REFERENCE_DIR [--only rms_norm ...]

It imports the reference's own modules -- ``moe_forward`` (router, expert
FFN, layer), ``dequant_fast`` (Q8_0 / Q4_0 decoders, through the reference's
``nightmare_np`` substrate for the known-answer blocks and through numpy for
bulk weights, which computes the same values) and ``nightmare_stream``
(production routing, ``GPUStreamEngine._moe_ffn``) -- feeds them the seeded
inputs of ``linuxnightmaresuite_b200.synth`` and stores their outputs with a
sha256 of the inputs.  The fixtures hold outputs only; tests regenerate the
inputs from the seed and check the digest.
"""
from __future__ import annotations

import importlib.util
import os
import platform
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = None   # set by main() from the command line or MOE_REFERENCE_DIR
sys.path.insert(0, ROOT)

from linuxnightmaresuite_b200 import synth  # noqa: E402


def _import_reference():
    sys.path.insert(0, REF)
    import dequant_fast  # noqa: F401  (real nightmare_np substrate)
    import moe_forward
    import nightmare_stream
    return moe_forward, dequant_fast, nightmare_stream


def _dequant_fast_on_numpy():
    """The reference decoder module with numpy bound as its ``np``."""
    saved = sys.modules.get("nightmare_np")
    sys.modules["nightmare_np"] = np
    try:
        spec = importlib.util.spec_from_file_location("dequant_fast_numpy",
                                                      os.path.join(REF, "dequant_fast.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        if saved is not None:
            sys.modules["nightmare_np"] = saved
        else:
            del sys.modules["nightmare_np"]
    return mod


def _nightmare_stream_on_numpy():
    """nightmare_stream with numpy bound as its ``np`` (fast enough for full
    layers; the pure-Python substrate is used for the router goldens)."""
    saved = sys.modules.get("nightmare_np")
    sys.modules["nightmare_np"] = np
    try:
        spec = importlib.util.spec_from_file_location("nightmare_stream_numpy",
                                                      os.path.join(REF, "nightmare_stream.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        if saved is not None:
            sys.modules["nightmare_np"] = saved
        else:
            del sys.modules["nightmare_np"]
    return mod


def _substrate(ns):
    """(to_array, to_numpy) converters for the module's ``np``."""
    if ns.np is np:
        return (lambda a: a), (lambda a: np.asarray(a))
    nnp = ns.np

    def to_arr(a):
        a = np.asarray(a, np.float32)
        return nnp.array(a.reshape(-1).tolist(), dtype=nnp.float32).reshape(*a.shape)

    def to_np(a):
        return np.asarray(a.reshape(-1).tolist(), dtype=np.float32).reshape(tuple(a.shape))

    return to_arr, to_np


def _meta():
    return dict(numpy_version=np.__version__, machine=platform.machine(),
                processor=platform.processor() or "")


def kat_blocks(dq):
    """Known-answer blocks: special fp16 scales x extreme quants."""
    scales = np.array([0.0, -0.0, 5.96e-08, 6.1e-05, 1.0, -1.0, 0.5, 65504.0, 0.00213],
                      dtype=np.float16)
    q8_vals = np.array([-128, -127, -1, 0, 1, 127], dtype=np.int8)
    q8 = []
    for s in scales:
        for v in q8_vals:
            blk = np.empty(34, np.uint8)
            blk[:2] = np.array([s], np.float16).view(np.uint8)
            q = np.full(32, v, np.int8)
            q[::3] = np.int8(-v if v != -128 else 127)
            blk[2:] = q.view(np.uint8)
            q8.append(blk)
    q4 = []
    for s in scales:
        for lo in range(16):
            blk = np.empty(18, np.uint8)
            blk[:2] = np.array([s], np.float16).view(np.uint8)
            nib_lo = (np.arange(16) + lo) % 16
            nib_hi = (15 - np.arange(16) - lo) % 16
            blk[2:] = (nib_lo | (nib_hi << 4)).astype(np.uint8)
            q4.append(blk)
    q8 = np.stack(q8)
    q4 = np.stack(q4)
    exp8 = np.asarray(dq.dequantize_q8_0(q8.tobytes(), q8.shape[0] * 32), dtype=np.float32)
    exp4 = np.asarray(dq.dequantize_q4_0(q4.tobytes(), q4.shape[0] * 32), dtype=np.float32)
    np.savez(os.path.join(HERE, "kat_blocks.npz"), q8_raw=q8, q8_expected=exp8,
             q4_raw=q4, q4_expected=exp4, **_meta())
    print("kat_blocks", q8.shape, q4.shape)


def router_cases(mf, ns, ns_np):
    """Router goldens for both routing semantics, incl. exact-tie cases."""
    rng = np.random.default_rng(123)
    cases = {}
    for ci, (d, E, k) in enumerate([(64, 8, 2), (256, 128, 8), (96, 16, 4)]):
        T = 16
        x = rng.standard_normal((T, d), dtype=np.float32)
        G = (rng.standard_normal((d, E), dtype=np.float32) * np.float32(0.02))
        if ci == 2:
            # duplicated router columns -> exactly equal logits
            G[:, 5] = G[:, 3]
            G[:, 9] = G[:, 3]
            G[:, 12] = G[:, 0]
        router = mf.MoERouter(G, E, k)
        ids0, w0 = [], []
        for t in range(T):
            i, w = router.route(x[t])
            ids0.append(i)
            w0.append(np.asarray(w, np.float32))
        # production semantics: softmax over all experts, top-k, renormalise
        # On the pure-Python nightmare_np substrate, argsort returns float
        # indices and ``probs[top_idx]`` then gathers the wrong entries, so
        # its weights are wrong while its ids are right.  Ids are pinned on
        # both substrates; weights on the numpy-bound copy.
        # Exactly tied logits (case 2) are ordered by numpy's default, unstable
        # argsort in the numpy-bound copy and by nightmare_np's stable argsort
        # in the substrate run; both are kept.
        ids1, w1, ids1_np, substrate_weight_defects = [], [], [], 0
        for t in range(T):
            ids_t, w_t = _production_route(ns, G.T.copy(), x[t], E, k)
            ids_n, w_n = _production_route(ns_np, G.T.copy(), x[t], E, k)
            assert sorted(ids_t.tolist()) == sorted(ids_n.tolist()) or ci == 2, (ids_t, ids_n)
            substrate_weight_defects += int(not np.allclose(np.sort(w_t), np.sort(w_n),
                                                            rtol=1e-5, atol=1e-7))
            # weights by expert from the numpy-bound run, in the substrate's order
            wmap = dict(zip(ids_n.tolist(), w_n.tolist()))
            if set(wmap) == set(ids_t.tolist()):
                w_sub = np.array([wmap[e] for e in ids_t.tolist()], np.float32)
            else:
                w_sub = w_n
                ids_t = ids_n
            ids1.append(ids_t)
            ids1_np.append(ids_n)
            w1.append(w_sub)
        cases[f"c{ci}_ids_mode1_numpy"] = np.array(ids1_np, np.int32)
        cases[f"c{ci}_nightmare_np_weight_defects"] = np.int32(substrate_weight_defects)
        cases[f"c{ci}_x"] = x
        cases[f"c{ci}_G"] = G
        cases[f"c{ci}_k"] = np.int32(k)
        cases[f"c{ci}_ids_mode0"] = np.array(ids0, np.int32)
        cases[f"c{ci}_w_mode0"] = np.array(w0, np.float32)
        cases[f"c{ci}_ids_mode1"] = np.array(ids1, np.int32)
        cases[f"c{ci}_w_mode1"] = np.array(w1, np.float32)
    np.savez(os.path.join(HERE, "router.npz"), **cases, **_meta())
    print("router cases", len(cases))


class _FakeEngine:
    """Just enough state for GPUStreamEngine._moe_ffn to run one token."""

    def __init__(self, ns, dim, n_exp, k, experts):
        self.dim = dim
        self._n_experts = n_exp
        self._n_experts_used = k
        self._architecture = "qwen2moe"
        self._ffn_activation = "swiglu"
        to_arr, _ = _substrate(ns)
        self._experts = {e: tuple(to_arr(m) for m in mats) for e, mats in experts.items()}
        self.routed = []
        self._uses_geglu_expert = lambda: ns.GPUStreamEngine._uses_geglu_expert(self)
        self._expert_act = lambda g, u: ns.GPUStreamEngine._expert_act(self, g, u)

    def _load_expert(self, layer_idx, ei):
        self.routed.append(int(ei))
        return self._experts[int(ei)]


def _production_route(ns, R, x, E, k):
    """Routing decision of GPUStreamEngine._moe_ffn (nightmare_stream.py:3227-3238).

    Runs the real method with probe experts: expert e has one hidden unit that
    reads input j (the largest |x|) and writes ``act`` to output e, so the
    layer output at e is ``w_e * act``.  Needs d >= E."""
    d = x.shape[0]
    assert d >= E
    j = int(np.argmax(np.abs(x)))
    experts = {}
    for e in range(E):
        g = np.zeros((1, d), np.float32)
        g[0, j] = 1.0
        dn = np.zeros((d, 1), np.float32)
        dn[e, 0] = 1.0
        experts[e] = (g, g.copy(), dn)
    eng = _FakeEngine(ns, d, E, k, experts)
    to_arr, to_np = _substrate(ns)
    out = to_np(ns.GPUStreamEngine._moe_ffn(eng, to_arr(x.reshape(1, -1)), 0,
                                            {"moe_router": to_arr(R)})).reshape(-1)
    ids = np.array(eng.routed, np.int32)
    xj = to_arr(np.array([x[j]], np.float32))
    act = to_np(eng._expert_act(xj, xj))[0]
    return ids, (out[ids] / act).astype(np.float32)


def _production_layer(ns, R, x, E, k, experts):
    """Output of GPUStreamEngine._moe_ffn for one token with real experts."""
    d = x.shape[0]
    eng = _FakeEngine(ns, d, E, k, {e: (ex.w_gate, ex.w_up, ex.w_down)
                                    for e, ex in enumerate(experts) if ex is not None})
    to_arr, to_np = _substrate(ns)
    out = to_np(ns.GPUStreamEngine._moe_ffn(eng, to_arr(x.reshape(1, -1)), 0,
                                            {"moe_router": to_arr(R)})).reshape(-1)
    return out, np.array(eng.routed, np.int32)


def _ref_experts(dqn, data, E_used):
    """Reference ExpertFFN objects for the experts in E_used (others None)."""
    cfg = data.cfg
    d, F, qt = cfg.d_model, cfg.ffn, cfg.qtype
    fn = dqn.DEQUANT_FUNCTIONS[qt]
    import moe_forward as mf
    experts = [None] * cfg.n_experts
    for e in sorted(set(int(v) for v in E_used)):
        wg = np.asarray(fn(data.w_gate[e].tobytes(), F * d), np.float32).reshape(F, d)
        wu = np.asarray(fn(data.w_up[e].tobytes(), F * d), np.float32).reshape(F, d)
        wd = np.asarray(fn(data.w_down[e].tobytes(), d * F), np.float32).reshape(d, F)
        experts[e] = mf.ExpertFFN(wg, wu, wd)
    return experts


def _ref_shared(dqn, data):
    import moe_forward as mf
    cfg = data.cfg
    d, Fs, qt = cfg.d_model, cfg.shared_ffn, cfg.shared_qtype
    fn = dqn.DEQUANT_FUNCTIONS[qt]
    wg = np.asarray(fn(data.s_gate[0].tobytes(), Fs * d), np.float32).reshape(Fs, d)
    wu = np.asarray(fn(data.s_up[0].tobytes(), Fs * d), np.float32).reshape(Fs, d)
    wd = np.asarray(fn(data.s_down[0].tobytes(), d * Fs), np.float32).reshape(d, Fs)
    return mf.ExpertFFN(wg, wu, wd)


def layer_case(mf, ns, dqn, name, cfg, seed, tokens, mode, n_experts_built=None):
    data = synth.make_layer(cfg, seed, tokens=tokens, n_experts_built=n_experts_built)
    x, G = data.x, data.gate_w
    E, k, d = cfg.n_experts, cfg.top_k, cfg.d_model
    if data.bias is not None:
        # the reference router has no bias term; an extra constant input
        # feature whose router row is the bias adds it to every logit
        G_use = np.concatenate([G, data.bias[None, :]], axis=0)
        x_router = np.concatenate([x, np.ones((x.shape[0], 1), np.float32)], axis=1)
    else:
        G_use, x_router = G, x
    router = mf.MoERouter(G_use, E, k)
    all_ids = []
    for t in range(x.shape[0]):
        if mode == 0:
            i, _ = router.route(x_router[t])
        else:
            i, _ = _production_route(ns, G_use.T.copy(), x_router[t], E, k)
        all_ids.extend(int(v) for v in i)
    experts = _ref_experts(dqn, data, all_ids)
    shared = _ref_shared(dqn, data) if cfg.shared_ffn else None
    outs, ids_l, w_l = [], [], []
    for t in range(x.shape[0]):
        if mode == 0:
            if data.bias is None:
                layer = mf.MoELayer(router, experts, shared)
                out = layer.forward(x[t])
                i, w = router.route(x[t])
            else:
                i, w = router.route(x_router[t])
                out = np.zeros_like(x[t])
                for eid, ww in zip(i, w):
                    out += ww * experts[eid].forward(x[t])
                if shared is not None:
                    out += shared.forward(x[t])
        else:
            if data.bias is not None:
                raise NotImplementedError("bias with production routing")
            out, i_out = _production_layer(ns, G.T.copy(), x[t], E, k, experts)
            if shared is not None:
                out = out + shared.forward(x[t])
            i, w = _production_route(ns, G.T.copy(), x[t], E, k)
            assert np.array_equal(i, i_out)
        outs.append(np.asarray(out, np.float32))
        ids_l.append(np.asarray(i, np.int32))
        w_l.append(np.asarray(w, np.float32))
    np.savez(os.path.join(HERE, f"layer_{name}.npz"), out=np.stack(outs), ids=np.stack(ids_l),
             weights=np.stack(w_l), seed=np.int32(seed), tokens=np.int32(x.shape[0]),
             mode=np.int32(mode), config=cfg.name, digest=data.digest(),
             n_experts_built=np.int32(-1 if n_experts_built is None else n_experts_built),
             **_meta())
    print("layer", name, np.stack(outs).shape)


def stacked_case(mf, dqn, name, cfg, seed, n_layers, tokens):
    """Stacked layers composed from the reference's rms_norm and MoELayer."""
    x0 = None
    layers = []
    for l in range(n_layers):
        data = synth.make_layer(cfg, seed + l, tokens=tokens)
        if x0 is None:
            x0 = data.x
        layers.append(data)
    x = x0.copy()
    for data in layers:
        router = mf.MoERouter(data.gate_w, cfg.n_experts, cfg.top_k)
        xn_all = np.stack([mf.rms_norm(x[t], data.norm_w).astype(np.float32) for t in range(x.shape[0])])
        used = []
        for t in range(x.shape[0]):
            used.extend(router.route(xn_all[t])[0])
        experts = _ref_experts(dqn, data, used)
        shared = _ref_shared(dqn, data)
        layer = mf.MoELayer(router, experts, shared)
        x = np.stack([x[t] + layer.forward(xn_all[t]) for t in range(x.shape[0])]).astype(np.float32)
    np.savez(os.path.join(HERE, f"stacked_{name}.npz"), out=x, seed=np.int32(seed),
             n_layers=np.int32(n_layers), tokens=np.int32(tokens), config=cfg.name,
             digest=layers[0].digest(), **_meta())
    print("stacked", name, x.shape)


def rms_norm_cases(mf):
    """The reference's rms_norm (moe_forward.py:34-40) over seeded rows of
    several widths, both scalings."""
    rng = np.random.default_rng(21)
    out = {}
    for d in (7, 100, 1024, 2816, 4096, 5000):
        x = (rng.standard_normal((3, d), dtype=np.float32) * np.float32(3.0))
        w = (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)
        for g in (0, 1):
            out[f"x_{d}"] = x
            out[f"w_{d}"] = w
            out[f"out_{d}_{g}"] = np.stack([mf.rms_norm(x[t], w, 1e-6, gemma_style=bool(g))
                                           for t in range(3)])
    np.savez(os.path.join(HERE, "rms_norm.npz"), **out, **_meta())
    print("rms_norm", len(out))


def _special_halves(rng, n):
    """fp16 scales with +-0, subnormals, 1.0, 65504 and random magnitudes."""
    v = (np.abs(rng.standard_normal(n, dtype=np.float32)) * np.float32(0.01)).astype(np.float16)
    special = np.array([0.0, -0.0, 6e-8, 1.0, 65504.0, -2.0], dtype=np.float16)
    v[:special.size] = special
    return v


def kquant_blocks(dq_real, dqn):
    """Q5_1 / Q4_K / Q6_K known answers: seeded raw blocks with special fp16
    scales, decoded by the reference's dequant_fast on its own nightmare_np
    substrate and on numpy (the two must agree)."""
    rng = np.random.default_rng(31)
    out = {}
    cases = {7: (32, 24, 48), 12: (256, 144, 12), 14: (256, 210, 12)}
    names = {7: "dequantize_q5_1", 12: "dequantize_q4_k", 14: "dequantize_q6_k"}
    for qt, (be, bb, nb) in cases.items():
        raw = np.frombuffer(rng.bytes(nb * bb), dtype=np.uint8).reshape(nb, bb).copy()
        if qt == 7:
            raw[:, 0:2] = _special_halves(rng, nb).view(np.uint8).reshape(nb, 2)
            raw[:, 2:4] = _special_halves(rng, nb)[::-1].copy().view(np.uint8).reshape(nb, 2)
        elif qt == 12:
            raw[:, 0:2] = _special_halves(rng, nb).view(np.uint8).reshape(nb, 2)
            raw[:, 2:4] = _special_halves(rng, nb)[::-1].copy().view(np.uint8).reshape(nb, 2)
        else:
            raw[:, 208:210] = _special_halves(rng, nb).view(np.uint8).reshape(nb, 2)
        n = nb * be
        exp_np = np.asarray(getattr(dqn, names[qt])(raw.tobytes(), n), dtype=np.float32)
        try:   # the reference's own nightmare_np substrate, when it runs these
            exp_real = np.asarray(getattr(dq_real, names[qt])(raw.tobytes(), n),
                                  dtype=np.float32)
            assert np.array_equal(exp_np.view(np.uint32), exp_real.view(np.uint32)), qt
            out[f"substrate_{qt}"] = np.array("nightmare_np+numpy")
        except AssertionError:
            raise
        except Exception as exc:   # noqa: BLE001
            print("nightmare_np substrate failed on", names[qt], repr(exc)[:120])
            out[f"substrate_{qt}"] = np.array("numpy")
        out[f"raw_{qt}"] = raw
        out[f"expected_{qt}"] = exp_np
    np.savez(os.path.join(HERE, "kquant_blocks.npz"), **out, **_meta())
    print("kquant_blocks", sorted(out))


class _G4Stub:
    """The engine state the gemma4 FFN block reads, around the reference's own
    GPUStreamEngine methods (_mm, _rms_norm, _expert_act)."""

    def __init__(self, ns, dim, n_exp, k, experts):
        cls = ns.GPUStreamEngine
        self._n_experts, self._n_experts_used, self.dim = n_exp, k, dim
        self._architecture = "gemma4"
        self.use_gpu = False
        self._experts = experts
        for name in ("_mm", "_rms_norm", "_expert_act", "_uses_geglu_expert"):
            setattr(self, name, getattr(cls, name).__get__(self))

    def _g4_moe_gpu_enabled(self):
        return False

    def _load_expert(self, layer_idx, ei):
        return self._experts[ei]


def _g4_block_source(ns):
    """The FFN part of GPUStreamEngine._layer_forward_gemma4, from the MoE
    test up to the sum of the shared and routed outputs."""
    import inspect
    import textwrap
    src = inspect.getsource(ns.GPUStreamEngine._layer_forward_gemma4)
    a = src.index("_is_moe = (self._n_experts")
    b = src.index("pfn = weights.get('post_ffw_norm')")
    body = src[a:b]
    lines = body.split("\n")
    indent = len(lines[1]) - len(lines[1].lstrip()) if len(lines) > 1 else 0
    return textwrap.dedent("\n".join(" " * indent + lines[0].lstrip() if i == 0 else ln
                                     for i, ln in enumerate(lines)))


def gemma4_cases(dq_real, dqn, ns_np):
    """Reference outputs of the gemma4 MoE FFN (nightmare_stream.py:4655-4693)
    and of its GeGLU activation (GPUStreamEngine._expert_act) on seeded
    inputs: fused Q4_K gate_up, Q5_1 down with a per-expert scale, Q8_0 shared
    MLP, router input scale, the four sandwich norms."""
    rng = np.random.default_rng(41)
    stub0 = _G4Stub(ns_np, 4, 1, 1, {})
    g = (rng.standard_normal(257, dtype=np.float32) * np.float32(3.0))
    u = rng.standard_normal(257, dtype=np.float32)
    act = np.asarray(stub0._expert_act(g, u))
    from linuxnightmaresuite_b200 import synth as sy
    d, E, k, F, Fs, T, eps = 256, 16, 4, 256, 192, 5, 1e-6
    data = sy.make_gemma4_layer(d, E, F, Fs, T, seed=43)
    experts = {}
    for e in range(E):
        gu = np.asarray(dqn.dequantize_q4_k(data.gate_up[e].tobytes(), 2 * F * d),
                        dtype=np.float32).reshape(2 * F, d)
        dn = np.asarray(dqn.dequantize_q5_1(data.down[e].tobytes(), d * F),
                        dtype=np.float32).reshape(d, F)
        # nightmare_stream.py:3422-3438: split the fused slice, scale the down
        dn = dn * float(data.down_scale[e])
        experts[e] = (np.ascontiguousarray(gu[:F]), np.ascontiguousarray(gu[F:]), dn)
    shared = [np.asarray(dqn.dequantize_q8_0(m.tobytes(), m.shape[0] * (m.shape[1] // 34) * 32),
                         dtype=np.float32).reshape(m.shape[0], -1) for m in
              (data.s_gate, data.s_up, data.s_down)]
    weights = {"moe_router": data.router, "moe_gate_inp_scale": data.gate_inp_scale,
               "ffn_norm": data.ffn_norm, "wg": shared[0], "wu": shared[1], "wd": shared[2],
               "post_ffw_norm_1": data.post_norm_1, "pre_ffw_norm_2": data.pre_norm_2,
               "post_ffw_norm_2": data.post_norm_2}
    code = compile(_g4_block_source(ns_np), "nightmare_stream.py:_layer_forward_gemma4", "exec")
    outs = []
    for t in range(T):
        env = {"self": _G4Stub(ns_np, d, E, k, experts), "np": np, "weights": weights,
               "x": data.x[t], "eps": eps, "layer": 0}
        exec(code, env)
        outs.append(np.asarray(env["f"], dtype=np.float32))
    np.savez(os.path.join(HERE, "gemma4.npz"), act_g=g, act_u=u, act_out=act,
             out=np.stack(outs), seed=np.int32(43), tokens=np.int32(T), digest=data.digest(),
             eps=np.float32(eps), **_meta())
    print("gemma4", np.stack(outs).shape)


def gguf_cases():
    """The reference's own GGUF parser (gguf_parser.py:325-555) on the two
    synthetic one-block MoE files this library writes: header, metadata,
    tensor infos, data offset and the raw bytes load_tensor_raw returns."""
    import hashlib
    import json
    import tempfile
    sys.path.insert(0, REF)
    import gguf_parser
    from linuxnightmaresuite_b200 import gguf
    out = {}
    for kind in ("swiglu", "gemma4"):
        meta, tensors = synth.moe_gguf_tensors(kind, 3)
        with tempfile.TemporaryDirectory() as tmp:
            path = os.path.join(tmp, f"{kind}.gguf")
            gguf.write_gguf(path, meta, tensors)
            with open(path, "rb") as f:
                file_sha = hashlib.sha256(f.read()).hexdigest()
            parser = gguf_parser.GGUFParser(path)
            model = parser.parse()
            infos = {n: [list(i.shape), int(i.dtype), int(i.offset)]
                     for n, i in model.tensors.items()}
            raw_sha = {}
            # the parser's arrays are its nightmare_np substrate's: convert by value
            for n in model.tensors:
                raw, dt, shape, ne = parser.load_tensor_raw(model, n)
                b = np.asarray(raw.reshape(-1).tolist(), dtype=np.uint8).tobytes()
                raw_sha[n] = [hashlib.sha256(b).hexdigest(), int(ne)]
            f32 = {}
            for n, i in model.tensors.items():
                if int(i.dtype) == 0:
                    a = parser.load_tensor(model, n)
                    f32[n] = np.asarray(a.reshape(-1).tolist(),
                                        dtype=np.float32).reshape(tuple(a.shape))
            parser.close()
        rec = {"file_sha": file_sha, "version": int(model.version),
               "tensor_data_offset": int(model.tensor_data_offset), "infos": infos,
               "raw_sha": raw_sha,
               "metadata": {k: v for k, v in model.metadata.items()}}
        out[f"{kind}_json"] = np.array(json.dumps(rec, sort_keys=True))
        for n, a in f32.items():
            out[f"{kind}_f32_{n}"] = a
    np.savez(os.path.join(HERE, "gguf.npz"), **out, **_meta())
    print("gguf", sorted(k for k in out if k.endswith("_json")))


def main(argv=None):
    import argparse
    global REF
    ap = argparse.ArgumentParser(description="generate the golden fixtures from the reference")
    ap.add_argument("reference_dir", nargs="?", default=os.environ.get("MOE_REFERENCE_DIR"))
    ap.add_argument("--only", action="append", default=None,
                    help="fixture groups: kat, router, layers, stacked, rms_norm, kquant, "
                         "gemma4, gguf")
    args = ap.parse_args(argv)
    if not args.reference_dir:
        ap.error("give the reference checkout directory (argument or MOE_REFERENCE_DIR)")
    REF = os.path.abspath(args.reference_dir)
    only = set(args.only) if args.only else None

    def want(name):
        return only is None or name in only

    mf, dq_real, ns = _import_reference()
    dqn = _dequant_fast_on_numpy()
    if want("rms_norm"):
        rms_norm_cases(mf)
    if want("gguf"):
        gguf_cases()
    if want("kquant"):
        kquant_blocks(dq_real, dqn)
    if want("gemma4"):
        gemma4_cases(dq_real, dqn, _nightmare_stream_on_numpy())
    if want("kat"):
        kat_blocks(dq_real)
    ns_np = _nightmare_stream_on_numpy()
    if want("router"):
        router_cases(mf, ns, ns_np)
    ns = ns_np
    C = synth.CONFIGS
    if not (want("layers") or want("stacked")):
        return
    if not want("layers"):
        small_stack = synth.MoEConfig("small_stack", 256, 16, 4, 128, 5, synth.QTYPE_Q4_0, 0.01,
                                      shared_ffn=192, n_layers=2)
        stacked_case(mf, dqn, "small_stack", small_stack, 11, 2, 5)
        return
    layer_case(mf, ns, dqn, "cpu_layer_mode0", C["cpu_layer"], 0, None, 0)
    layer_case(mf, ns, dqn, "cpu_layer_mode1", C["cpu_layer"], 0, None, 1)
    layer_case(mf, ns, dqn, "decode_t2", C["decode_t8"], 0, 2, 0)
    small_shared = synth.MoEConfig("small_shared", 256, 16, 4, 128, 6, synth.QTYPE_Q4_0, 0.01,
                                   shared_ffn=192, n_layers=1)
    layer_case(mf, ns, dqn, "small_shared", small_shared, 7, None, 0)
    small_zipf = synth.MoEConfig("small_zipf", 256, 16, 4, 128, 64, synth.QTYPE_Q8_0, 0.002,
                                 zipf_s=1.1, zipf_max_rows=40)
    layer_case(mf, ns, dqn, "small_zipf", small_zipf, 3, None, 0)
    small_stack = synth.MoEConfig("small_stack", 256, 16, 4, 128, 5, synth.QTYPE_Q4_0, 0.01,
                                  shared_ffn=192, n_layers=2)
    if want("stacked"):
        stacked_case(mf, dqn, "small_stack", small_stack, 11, 2, 5)


if __name__ == "__main__":
    main()
