"""Expert variants and the other block formats on the GPU.

* Q5_1 / Q4_K / Q6_K decode bit for bit as the reference's dequant_fast
  (known answers made by the reference) -- moe_dequantize;
* layers whose experts are stored in those formats (and a Q4_K gate/up with a
  Q5_1 down, as gemma4 ships them) on the raw-block path, against the oracle;
* the gemma4 variant -- GeGLU-tanh, a fused ffn_gate_up_exps stack, a
  per-expert down scale -- on the packed Q8_0 kernels (GEMV and tensor-core
  paths) and on the raw path;
* gemma4's router input and the whole gemma4 MoE block against the outputs of
  the reference's own block code (nightmare_stream.py:4655-4693).
"""
import os

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import _lib, kernels as K, moe_forward as M, synth
from linuxnightmaresuite_b200.gemma4 import Gemma4MoEBlock
from oracle import moe_oracle as orc

from ._util import GOLD, TOL_MAX_ABS, TOL_REL_L2, check_layer

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("qt", [7, 12, 14])
def test_dequantize_kquant_known_answers_bit_exact(qt):
    z = np.load(os.path.join(GOLD, "kquant_blocks.npz"))
    raw, exp = z[f"raw_{qt}"], z[f"expected_{qt}"]
    got = K.dequantize(cuda(raw.reshape(-1)), qt, exp.size).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("qt", [7, 12, 14])
def test_dequantize_kquant_large_matches_oracle(qt):
    rng = np.random.default_rng(qt)
    raw = synth.blocks_of(rng, qt, 3, 256, 1024, 0.01)
    n = 3 * 256 * 1024
    got = K.dequantize(cuda(raw.reshape(-1)), qt, n).cpu().numpy()
    exp = orc.DEQUANT[qt](raw, n)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def _layer_case(gu_qt, dn_qt, T, E=16, k=4, d=512, F=256, seed=0, act=0, scale=False,
                fused=False, mode=0):
    rng = np.random.default_rng(seed)
    gate_w = rng.standard_normal((d, E), dtype=np.float32) * np.float32(0.05)
    x = rng.standard_normal((T, d), dtype=np.float32)
    wg = synth.blocks_of(rng, gu_qt, E, F, d, 0.01)
    wu = synth.blocks_of(rng, gu_qt, E, F, d, 0.01)
    wd = synth.blocks_of(rng, dn_qt, E, d, F, 0.01)
    ds = (0.5 + rng.uniform(0, 1, E)).astype(np.float32) if scale else None
    experts = []
    for e in range(E):
        g = orc.dequantize_matrix(wg[e], gu_qt, F, d)
        u = orc.dequantize_matrix(wu[e], gu_qt, F, d)
        dn = orc.dequantize_matrix(wd[e], dn_qt, d, F)
        if ds is not None:
            dn = dn * float(ds[e])
        experts.append(orc.GeGLUExpert(g, u, dn) if act else orc.DenseExpert(g, u, dn))
    kw = dict(act=act, down_qtype=dn_qt, down_scale=ds)
    if fused:
        gu = np.concatenate([wg, wu], axis=1)   # (E, 2F, row bytes): gate rows, then up rows
        layer = M.MoELayer.from_blocks(gate_w, None, None, wd, gu_qt, k, mode=mode, gate_up=gu,
                                       **kw)
    else:
        layer = M.MoELayer.from_blocks(gate_w, wg, wu, wd, gu_qt, k, mode=mode, **kw)
    return layer, x, gate_w, experts


def _run_check(layer, x, gate_w, experts, k, mode=0, tokens=None):
    out, ids, w = layer.forward_batch(cuda(x), return_routing=True)
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    check_layer(x, gate_w, None, k, mode, experts, None, out.cpu().numpy(), ids.cpu().numpy(),
                w.cpu().numpy(), tokens=tokens)


@pytest.mark.parametrize("gu_qt,dn_qt", [(12, 12), (14, 14), (7, 7), (12, 7), (0, 0), (8, 7),
                                          (2, 14)])
@pytest.mark.parametrize("T", [3, 200])
def test_raw_format_layers_match_oracle(gu_qt, dn_qt, T):
    layer, x, gate_w, experts = _layer_case(gu_qt, dn_qt, T, seed=gu_qt * 31 + dn_qt)
    _run_check(layer, x, gate_w, experts, 4)


@pytest.mark.parametrize("T", [3, 40])
def test_gemma4_variant_on_packed_gemv(T):
    """Q8_0 everywhere -> packed GEMV kernels with GeGLU, fused stack, down scale."""
    layer, x, gate_w, experts = _layer_case(8, 8, T, act=1, scale=True, fused=True, seed=5,
                                            mode=1)
    _run_check(layer, x, gate_w, experts, 4, mode=1)


def test_gemma4_variant_on_tensor_cores():
    """Enough rows per expert for the tcgen05 path, same variant."""
    layer, x, gate_w, experts = _layer_case(8, 8, 1024, E=8, k=2, d=512, F=256, act=1,
                                            scale=True, fused=True, seed=6, mode=1)
    _run_check(layer, x, gate_w, experts, 2, mode=1, tokens=list(range(0, 1024, 37)))


def test_gemma4_variant_on_raw_path():
    """Fused Q4_K gate/up + Q5_1 down with scale and GeGLU (the gemma4 GGUF layout)."""
    layer, x, gate_w, experts = _layer_case(12, 7, 64, act=1, scale=True, fused=True, seed=7,
                                            mode=1)
    _run_check(layer, x, gate_w, experts, 4, mode=1)


def test_router_input_matches_oracle():
    rng = np.random.default_rng(3)
    for d in (256, 2816, 1000):
        x = rng.standard_normal((7, d), dtype=np.float32) * np.float32(5)
        s = (1 + 0.2 * rng.standard_normal(d)).astype(np.float32)
        got = K.router_input(cuda(x), cuda(s), 1e-6).cpu().numpy()
        exp = np.stack([orc.gemma4_router_input(x[t], s, d, 1e-6) for t in range(7)])
        np.testing.assert_allclose(got, exp, rtol=2e-6, atol=1e-7)
        got0 = K.router_input(cuda(x), None, 1e-6).cpu().numpy()
        exp0 = np.stack([orc.gemma4_router_input(x[t], None, d, 1e-6) for t in range(7)])
        np.testing.assert_allclose(got0, exp0, rtol=2e-6, atol=1e-7)


def _gemma4_block(data, F, top_k, eps):
    return Gemma4MoEBlock(data.router, data.gate_inp_scale, data.gate_up, 12, data.down, 7,
                          data.down_scale, top_k, (data.s_gate, data.s_up, data.s_down), 8,
                          data.s_gate.shape[0], data.ffn_norm, data.post_norm_1, data.pre_norm_2,
                          data.post_norm_2, eps=eps)


def test_gemma4_block_matches_reference_golden():
    z = np.load(os.path.join(GOLD, "gemma4.npz"))
    data = synth.make_gemma4_layer(256, 16, 256, 192, int(z["tokens"]), seed=int(z["seed"]))
    assert data.digest() == str(z["digest"])
    block = _gemma4_block(data, 256, 4, float(z["eps"]))
    got = block.forward(data.x)
    assert block.device_status() == 0
    assert isinstance(got, np.ndarray) and got.shape == z["out"].shape
    mx, rel = orc.compare(got, z["out"])
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)
    one = block.forward(data.x[1])
    mx, rel = orc.compare(one, z["out"][1])
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)


def test_gemma4_block_batch_matches_oracle():
    """A batch at gemma4-26B-A4B's expert shape (d 2816, expert ffn 704,
    128 experts, top-8) through the block, against the oracle on sampled rows."""
    T, d, E, F, Fs, k, eps = 48, 2816, 128, 704, 2112, 8, 1e-6
    data = synth.make_gemma4_layer(d, E, F, Fs, T, seed=9)
    block = _gemma4_block(data, F, k, eps)
    got, ids, w = block.forward(cuda(data.x), return_routing=True)
    got = got.cpu().numpy()
    assert block.device_status() == 0
    rows = [0, 5, 17, 47]
    experts = {}
    Fs_ = data.s_gate.shape[0]
    wts = {"moe_router": data.router, "moe_gate_inp_scale": data.gate_inp_scale,
           "ffn_norm": data.ffn_norm, "wg": orc.dequantize_matrix(data.s_gate, 8, Fs_, d),
           "wu": orc.dequantize_matrix(data.s_up, 8, Fs_, d),
           "wd": orc.dequantize_matrix(data.s_down, 8, d, Fs_),
           "post_ffw_norm_1": data.post_norm_1, "pre_ffw_norm_2": data.pre_norm_2,
           "post_ffw_norm_2": data.post_norm_2}

    class Lazy:
        def __getitem__(self, e):
            if e not in experts:
                experts[e] = orc.gemma4_expert_from_blocks(data.gate_up[e], 12, data.down[e], 7,
                                                           d, F, data.down_scale[e])
            return experts[e]
    ids = ids.cpu().numpy()
    for t in rows:
        exp, top, _ = orc.gemma4_moe_block(data.x[t], wts, Lazy(), k, eps)
        assert np.array_equal(np.sort(top), np.sort(ids[t])), t
        mx, rel = orc.compare(got[t], exp)
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (t, mx, rel)
