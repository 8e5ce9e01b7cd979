"""The layer with its tokens and output in pinned host memory: the router's
first pass reads x over the bus and leaves the device copy the experts read,
the combine writes the output in place -- the same result, bit for bit, as
with device tensors."""
import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import moe_forward as M
from linuxnightmaresuite_b200 import synth
from linuxnightmaresuite_b200.ep import EPLocalRanks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 8, 64, 200])
def test_host_tokens_match_device_tokens(T):
    dev = torch.device("cuda:0")
    cfg = synth.MoEConfig("host_io", 512, 16, 4, 256, T, synth.QTYPE_Q4_0, 0.01)
    data = synth.make_layer_device(cfg, 7, T, 0, cfg.n_experts, dev)
    layer = M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                                   cfg.top_k, mode=cfg.route_mode, bias=data.bias, device=dev)
    x = np.ascontiguousarray(data.x[:T])
    ref = layer.forward_batch(torch.from_numpy(x).to(dev)).cpu().numpy()
    x_host = torch.from_numpy(x).pin_memory()
    out_host = torch.empty(x_host.shape, dtype=torch.float32).pin_memory()
    got = layer.forward_batch(x_host, out=out_host)
    torch.cuda.synchronize()
    assert got.data_ptr() == out_host.data_ptr()
    np.testing.assert_array_equal(out_host.numpy(), ref)
    # device output from host tokens
    got_dev = layer.forward_batch(x_host, out=torch.empty((T, 512), device=dev)).cpu().numpy()
    np.testing.assert_array_equal(got_dev, ref)
    assert layer.device_status() == 0


def test_pageable_host_tokens_rejected():
    dev = torch.device("cuda:0")
    cfg = synth.MoEConfig("host_io", 256, 8, 2, 128, 4, synth.QTYPE_Q8_0, 0.002)
    data = synth.make_layer_device(cfg, 3, 4, 0, cfg.n_experts, dev)
    layer = M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                                   cfg.top_k, mode=cfg.route_mode, device=dev)
    with pytest.raises(TypeError):
        layer.forward_batch(torch.from_numpy(np.ascontiguousarray(data.x[:4])))


def test_expert_parallel_host_tokens_match_device_tokens():
    """The expert-parallel layer (its ranks emulated on one GPU): pinned host
    tokens and outputs give the device tensors' result bit for bit."""
    dev = torch.device("cuda:0")
    W, T = 2, 16
    cfg = synth.MoEConfig("host_io_ep", 512, 16, 4, 256, T * W, synth.QTYPE_Q8_0, 0.002)
    data = synth.make_layer_device(cfg, 5, T * W, 0, cfg.n_experts, dev)
    ep = EPLocalRanks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.top_k, W,
                      mode=cfg.route_mode, bias=data.bias, device=dev)
    xs = [np.ascontiguousarray(data.x[r * T:(r + 1) * T]) for r in range(W)]
    ref = [o.cpu().numpy() for o in ep.forward([torch.from_numpy(x).to(dev) for x in xs])]
    got = ep.forward([torch.from_numpy(x).pin_memory() for x in xs])
    torch.cuda.synchronize()
    for g, r in zip(got, ref):
        assert not g.is_cuda
        np.testing.assert_array_equal(g.numpy(), r)
    assert ep.device_status() == [0] * W
