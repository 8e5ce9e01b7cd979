"""GPU parity of the whole MoE layer against the reference goldens and the
oracle, at the parity tolerance (max-abs <= 1e-2, rel-L2 <= 2e-3)."""
import os

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import moe_forward as M, synth
from oracle import moe_oracle as orc

from ._util import GOLD, TOL_MAX_ABS, TOL_REL_L2, check_layer, oracle_parts

pytestmark = pytest.mark.gpu


def build_layer(data, mode=0):
    cfg = data.cfg
    shared = None
    if cfg.shared_ffn:
        shared = (data.s_gate[0], data.s_up[0], data.s_down[0])
    return M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                                  cfg.top_k, shared=shared, shared_qtype=cfg.shared_qtype,
                                  shared_hidden=cfg.shared_ffn, mode=mode, bias=data.bias)


def run(layer, x):
    out, ids, w = layer.forward_batch(torch.from_numpy(x).cuda(), return_routing=True)
    assert layer.device_status() == 0
    return out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()


GOLDEN_LAYERS = {
    "cpu_layer_mode0": synth.CONFIGS["cpu_layer"],
    "cpu_layer_mode1": synth.CONFIGS["cpu_layer"],
    "decode_t2": synth.CONFIGS["decode_t8"],
    "small_shared": synth.MoEConfig("small_shared", 256, 16, 4, 128, 6, synth.QTYPE_Q4_0, 0.01,
                                    shared_ffn=192, n_layers=1),
    "small_zipf": synth.MoEConfig("small_zipf", 256, 16, 4, 128, 64, synth.QTYPE_Q8_0, 0.002,
                                  zipf_s=1.1, zipf_max_rows=40),
}


@pytest.mark.parametrize("name", sorted(GOLDEN_LAYERS))
def test_layer_matches_reference_golden(name):
    z = np.load(os.path.join(GOLD, f"layer_{name}.npz"))
    nb = int(z["n_experts_built"])
    data = synth.make_layer(GOLDEN_LAYERS[name], int(z["seed"]), tokens=int(z["tokens"]),
                            n_experts_built=None if nb < 0 else nb)
    assert data.digest() == str(z["digest"])
    mode = int(z["mode"])
    out, ids, w = run(build_layer(data, mode), data.x)
    experts, shared = oracle_parts(data)
    check_layer(data.x, data.gate_w, data.bias, data.cfg.top_k, mode, experts, shared, out, ids,
                w, exp_out=z["out"], exp_ids=z["ids"], exp_w=z["weights"])


def test_drop_in_surface_single_token():
    """MoERouter / ExpertFFN / MoELayer used exactly as moe_forward.py's."""
    z = np.load(os.path.join(GOLD, "layer_cpu_layer_mode0.npz"))
    data = synth.make_layer(synth.CONFIGS["cpu_layer"], 0)
    cfg = data.cfg
    router = M.MoERouter(data.gate_w, cfg.n_experts, cfg.top_k)
    experts = [M.ExpertFFN(data.w_gate[e], data.w_up[e], data.w_down[e], cfg.qtype, cfg.d_model,
                           cfg.ffn) for e in range(cfg.n_experts)]
    layer = M.MoELayer(router, experts)
    for t in range(data.x.shape[0]):
        ids, w = router.route(data.x[t])
        assert isinstance(ids, list) and ids == z["ids"][t].tolist()
        assert isinstance(w, np.ndarray) and w.dtype == np.float32
        out = layer.forward(data.x[t])
        assert isinstance(out, np.ndarray) and out.shape == (cfg.d_model,)
        mx, rel = orc.compare(out, z["out"][t])
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2
        e0 = experts[ids[0]].forward(data.x[t])
        ref = orc.expert_from_blocks(data.w_gate[ids[0]], data.w_up[ids[0]], data.w_down[ids[0]],
                                     cfg.qtype, cfg.d_model, cfg.ffn).forward(data.x[t])
        mx, rel = orc.compare(e0, ref)
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2


@pytest.fixture(scope="module", params=[1, 8, 64])
def decode_data(request):
    return synth.make_layer(synth.CONFIGS["decode_t8"], 0, tokens=request.param)


def test_decode_layer_full_size(decode_data):
    data = decode_data
    out, ids, w = run(build_layer(data), data.x)
    experts, shared = oracle_parts(data)
    check_layer(data.x, data.gate_w, None, 8, 0, experts, shared, out, ids, w)


def test_decode_layer_deterministic_and_batch_consistent(decode_data):
    data = decode_data
    layer = build_layer(data)
    a, ids_a, _ = run(layer, data.x)
    b, ids_b, _ = run(layer, data.x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # a token alone gives the batch row within tolerance
    t = data.x.shape[0] - 1
    c, ids_c, _ = run(layer, data.x[t:t + 1])
    if np.array_equal(ids_c[0], ids_a[t]):
        mx, rel = orc.compare(c[0], a[t])
        assert mx <= 1e-3 and rel <= 1e-5


def test_prefill_layer_sampled_tokens():
    """4096 tokens with Zipf-skewed routing: the whole batch runs, a sample of
    tokens (busiest and rarest experts included) is checked against the oracle."""
    data = synth.make_layer(synth.CONFIGS["prefill"], 0)
    out, ids, w = run(build_layer(data), data.x)
    counts = np.bincount(ids.reshape(-1), minlength=128)
    # Zipf-skewed: the busiest expert takes ~1500 of 32768 rows, the tail a
    # fraction of the 256-row mean
    assert counts.max() > 1000 and counts.min() < 128
    assert np.isfinite(out).all()
    rng = np.random.default_rng(0)
    busiest = int(np.argmax(counts))
    rare = int(np.argmin(np.where(counts > 0, counts, 1 << 30)))
    toks = set(rng.choice(4096, 24, replace=False).tolist())
    toks |= set(np.nonzero((ids == busiest).any(1))[0][:4].tolist())
    toks |= set(np.nonzero((ids == rare).any(1))[0][:4].tolist())
    experts, shared = oracle_parts(data)
    check_layer(data.x, data.gate_w, data.bias, 8, 0, experts, shared, out, ids, w,
                tokens=sorted(toks))


def test_long_reduction_layer_precision():
    """d_model 4096 / ffn 1536 (the expert-parallel layer's shapes) with 256
    rows per expert, so the tensor-core path runs with the longest reductions;
    top-2 keeps each token's output close to a single expert's, where the
    accumulation error would show."""
    cfg = synth.MoEConfig("long_k", 4096, 8, 2, 1536, 1024, synth.QTYPE_Q8_0, 0.002)
    data = synth.make_layer(cfg, 0)
    out, ids, w = run(build_layer(data), data.x)
    experts, shared = oracle_parts(data)
    check_layer(data.x, data.gate_w, None, 2, 0, experts, shared, out, ids, w,
                tokens=list(range(0, 1024, 32)))


def test_shared_expert_layer_sampled_tokens():
    """Stacked-decode layer shape: routed Q4_0 + always-on Q8_0 shared expert."""
    data = synth.make_layer(synth.CONFIGS["stacked"], 0)
    out, ids, w = run(build_layer(data), data.x)
    experts, shared = oracle_parts(data)
    check_layer(data.x, data.gate_w, None, 8, 0, experts, shared, out, ids, w,
                tokens=list(range(0, 256, 17)))


def test_stacked_matches_reference_golden():
    from linuxnightmaresuite_b200 import stacked
    z = np.load(os.path.join(GOLD, "stacked_small_stack.npz"))
    cfg = synth.MoEConfig("small_stack", 256, 16, 4, 128, 5, synth.QTYPE_Q4_0, 0.01,
                          shared_ffn=192, n_layers=2)
    layers = [synth.make_layer(cfg, int(z["seed"]) + l, tokens=int(z["tokens"]))
              for l in range(int(z["n_layers"]))]
    assert layers[0].digest() == str(z["digest"])
    model = stacked.StackedMoE.from_layers(layers)
    out = model.forward(torch.from_numpy(layers[0].x).cuda()).cpu().numpy()
    mx, rel = orc.compare(out, z["out"])
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)
