"""The reference's own constructor forms on the GPU.

``ExpertFFN(w_gate, w_up, w_down)`` with the dequantised f32 matrices of
moe_forward.py:119-133 (GGML type 0 path, 4 bytes per weight, no CPU
fallback) and ``rms_norm(x, weight, eps, gemma_style)`` of
moe_forward.py:34-40, against the oracle and the reference goldens."""
import os

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import moe_forward as M, synth
from oracle import moe_oracle as orc

from ._util import GOLD, TOL_MAX_ABS, TOL_REL_L2, check_layer

pytestmark = pytest.mark.gpu


def _f32_experts(data, n=None):
    cfg = data.cfg
    n = cfg.n_experts if n is None else n
    return [orc.expert_from_blocks(data.w_gate[e], data.w_up[e], data.w_down[e], cfg.qtype,
                                   cfg.d_model, cfg.ffn) for e in range(n)]


def test_f32_expert_single_token_matches_reference_golden():
    """The reference's MoERouter / ExpertFFN / MoELayer calls with f32 matrices,
    one token at a time, against the outputs of the reference itself."""
    z = np.load(os.path.join(GOLD, "layer_cpu_layer_mode0.npz"))
    data = synth.make_layer(synth.CONFIGS["cpu_layer"], 0)
    assert data.digest() == str(z["digest"])
    cfg = data.cfg
    dense = _f32_experts(data)
    router = M.MoERouter(data.gate_w, cfg.n_experts, cfg.top_k)
    experts = [M.ExpertFFN(e.w_gate, e.w_up, e.w_down) for e in dense]
    assert experts[0].qtype == M.QTYPE_F32 and experts[0].dim == cfg.d_model
    layer = M.MoELayer(router, experts)
    for t in range(data.x.shape[0]):
        out = layer.forward(data.x[t])
        assert isinstance(out, np.ndarray) and out.dtype == np.float32
        mx, rel = orc.compare(out, z["out"][t])
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (t, mx, rel)
        ids, _ = router.route(data.x[t])
        e0 = experts[ids[0]].forward(data.x[t])
        mx, rel = orc.compare(e0, dense[ids[0]].forward(data.x[t]))
        assert mx <= 1e-3 and rel <= 1e-5, (mx, rel)


@pytest.mark.parametrize("T", [1, 5, 300])
def test_f32_layer_batch_with_shared_expert(T):
    """A batch through the f32 layer: ragged groups, several 8-row work items
    per expert at T=300, an f32 shared expert."""
    cfg = synth.MoEConfig("f32_small", 512, 16, 4, 384, T, synth.QTYPE_Q8_0, 0.002,
                          shared_ffn=256)
    data = synth.make_layer(cfg, 5, tokens=T)
    dense = _f32_experts(data)
    sh = orc.expert_from_blocks(data.s_gate[0], data.s_up[0], data.s_down[0], cfg.shared_qtype,
                                cfg.d_model, cfg.shared_ffn)
    router = M.MoERouter(data.gate_w, cfg.n_experts, cfg.top_k)
    layer = M.MoELayer(router, [M.ExpertFFN(e.w_gate, e.w_up, e.w_down) for e in dense],
                       M.ExpertFFN(sh.w_gate, sh.w_up, sh.w_down))
    out, ids, w = layer.forward_batch(torch.from_numpy(data.x).cuda(), return_routing=True)
    torch.cuda.synchronize()
    assert layer.device_status() == 0
    check_layer(data.x, data.gate_w, None, cfg.top_k, 0, dense, sh, out.cpu().numpy(),
                ids.cpu().numpy(), w.cpu().numpy())


def test_f32_constructor_rejects_block_bytes_without_qtype():
    data = synth.make_layer(synth.CONFIGS["cpu_layer"], 0)
    with pytest.raises(TypeError):
        M.ExpertFFN(data.w_gate[0], data.w_up[0], data.w_down[0])


@pytest.mark.parametrize("d", [7, 100, 1024, 2816, 4096, 5000])
@pytest.mark.parametrize("gemma", [False, True])
def test_rms_norm_gemma_style_matches_reference(d, gemma):
    z = np.load(os.path.join(GOLD, "rms_norm.npz"))
    x, w = z[f"x_{d}"], z[f"w_{d}"]
    exp = z[f"out_{d}_{int(gemma)}"]
    got = M.rms_norm(x, w, 1e-6, gemma_style=gemma)
    np.testing.assert_allclose(got, exp, rtol=2e-6, atol=1e-6)
    one = M.rms_norm(x[0], w, 1e-6, gemma)
    assert one.shape == (d,)
    np.testing.assert_allclose(one, exp[0], rtol=2e-6, atol=1e-6)
