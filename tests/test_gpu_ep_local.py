"""Expert-parallel layer with all ranks on one GPU, against the oracle.

``EPLocalRanks`` drives W ranks of the expert-parallel layer from one process:
W exchange windows, workspaces and expert shards on cuda:0, the same device
code as one process per GPU (``moe_ep_forward_phases``).  Each phase runs for
every rank before the next phase starts, so every wait finds its flag raised by
work already completed in stream order.  The rows, counts, positions, owner
order and return path of the exchange are thus checked on one GPU, and every
rank's output is compared with the oracle (the reference's MoELayer.forward
restated), not with the single-GPU layer.
"""
import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import synth
from linuxnightmaresuite_b200.ep import EPLocalRanks
from oracle import moe_oracle as orc

from ._util import check_layer, make, oracle_parts

pytestmark = pytest.mark.gpu

TOKENS = 64   # tokens over all ranks


@pytest.fixture(scope="module")
def decode_case():
    data = make("decode_t8", seed=5, tokens=TOKENS)
    experts, shared = oracle_parts(data)
    cfg = data.cfg
    exp = orc.moe_layer(data.x, data.gate_w, experts, cfg.top_k, cfg.route_mode, shared,
                        data.bias)
    return data, experts, exp


@pytest.mark.parametrize("world", [2, 4, 8])
def test_local_ranks_match_oracle(decode_case, world):
    data, experts, (exp_out, exp_ids, exp_w, _) = decode_case
    cfg = data.cfg
    dev = torch.device("cuda", 0)
    layer = EPLocalRanks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.top_k,
                         world, cfg.route_mode, data.bias, device=dev)
    T = TOKENS // world
    xs = [torch.from_numpy(np.ascontiguousarray(data.x[r * T:(r + 1) * T])).to(dev)
          for r in range(world)]
    outs = [o.clone() for o in layer.forward(xs)]
    outs2 = layer.forward(xs)           # a second step (next epoch) on the same windows
    torch.cuda.synchronize()
    assert layer.device_status() == [0] * world
    got = torch.cat(outs).cpu().numpy()
    assert np.array_equal(got, torch.cat(outs2).cpu().numpy()), "second step differs"
    from linuxnightmaresuite_b200 import kernels as K
    ids, w = K.router(torch.from_numpy(data.x).to(dev), layer.gate_w, cfg.top_k, cfg.route_mode,
                      layer.bias)
    check_layer(data.x, data.gate_w, data.bias, cfg.top_k, cfg.route_mode, experts, None, got,
                ids.cpu().numpy(), w.cpu().numpy(), exp_out=exp_out, exp_ids=exp_ids,
                exp_w=exp_w)


def test_local_ranks_shared_expert_and_residual():
    """A stacked-decode layer (routed Q4_0 experts + always-on Q8_0 shared
    expert) on 4 ranks, with the residual added in the combine."""
    cfg = synth.CONFIGS["stacked"]
    world, T = 4, 6
    data = synth.make_layer(cfg, 11, tokens=world * T)
    experts, shared = oracle_parts(data)
    dev = torch.device("cuda", 0)
    layer = EPLocalRanks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.top_k,
                         world, cfg.route_mode, data.bias, device=dev,
                         shared=(data.s_gate, data.s_up, data.s_down),
                         shared_qtype=cfg.shared_qtype)
    xs = [torch.from_numpy(np.ascontiguousarray(data.x[r * T:(r + 1) * T])).to(dev)
          for r in range(world)]
    res = [torch.full_like(x, 0.5) for x in xs]
    outs = layer.forward(xs, residuals=res)
    torch.cuda.synchronize()
    assert layer.device_status() == [0] * world
    got = torch.cat(outs).cpu().numpy() - np.float32(0.5)
    from linuxnightmaresuite_b200 import kernels as K
    ids, w = K.router(torch.from_numpy(data.x).to(dev), layer.gate_w, cfg.top_k, cfg.route_mode,
                      layer.bias)
    check_layer(data.x, data.gate_w, data.bias, cfg.top_k, cfg.route_mode, experts, shared, got,
                ids.cpu().numpy(), w.cpu().numpy())
