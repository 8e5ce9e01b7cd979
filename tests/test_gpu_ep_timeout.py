"""Failure detection of the expert-parallel exchange, on one GPU and without a
GPU fault: rank 0 of a two-rank layer runs against a stand-in window for rank 1
that no process ever writes.  Both of rank 0's waits on rank 1 (its rows, its
returned outputs) must give up after their bound, set MOE_STATUS_TIMEOUT in the
status word and leave the device usable."""
import ctypes
import time

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import _lib, kernels as K, synth

pytestmark = pytest.mark.gpu


def _ipc_alloc(nbytes):
    p = ctypes.c_void_p(0)
    _lib.call("moe_ipc_alloc", nbytes, ctypes.byref(p))
    return p.value


def test_ep_wait_on_a_silent_rank_times_out():
    cfg = synth.CONFIGS["decode_t8"]
    W, rank, T = 2, 0, 8
    data = synth.make_layer(cfg, 5, tokens=T)
    E, k, d, F = cfg.n_experts, cfg.top_k, cfg.d_model, cfg.ffn
    El = E // W
    dev = torch.device("cuda", 0)
    gate_w = torch.from_numpy(np.ascontiguousarray(data.gate_w, dtype=np.float32)).to(dev)
    packed = []
    for raw, rows, cols in ((data.w_gate, F, d), (data.w_up, F, d), (data.w_down, d, F)):
        r = torch.from_numpy(np.ascontiguousarray(raw[:El]).reshape(-1).view(np.uint8)).to(dev)
        packed.append(K.pack_weights(r, cfg.qtype, El, rows, cols))
    lw = K.LayerWeights(gate_w, packed[0], packed[1], packed[2], cfg.qtype, E, k, d, F)
    nbytes = ctypes.c_size_t(0)
    _lib.call("moe_ep_window_bytes", W, E, T, k, d, ctypes.byref(nbytes))
    own, silent = _ipc_alloc(nbytes.value), _ipc_alloc(nbytes.value)
    try:
        peers = torch.tensor([own, silent], dtype=torch.int64, device=dev)
        wsb = ctypes.c_size_t(0)
        _lib.call("moe_ep_workspace_bytes", ctypes.byref(lw.c), W, T, ctypes.byref(wsb))
        ws = K.workspace(wsb.value, dev)
        ws[:256].zero_()
        x = torch.from_numpy(data.x).to(dev)
        out = torch.empty_like(x)
        t0 = time.time()
        _lib.call("moe_ep_forward", ctypes.byref(lw.c), W, rank,
                  ctypes.c_void_p(peers.data_ptr()), ctypes.c_void_p(own), K._ptr(x), T,
                  K._ptr(out), K._ptr(None), 1, K._ptr(ws), ws.numel(), K._stream())
        torch.cuda.synchronize()
        waited = time.time() - t0
        st = K.read_status(ws)
        assert st & _lib.MOE_STATUS_TIMEOUT, st
        assert 1.0 <= waited < 30.0, waited
        # the device is still usable: a normal single-GPU layer runs and agrees
        # with itself
        y = torch.ones(1024, device=dev).sum().item()
        assert y == 1024.0
    finally:
        torch.cuda.synchronize()
        _lib.call("moe_ipc_free", ctypes.c_void_p(own))
        _lib.call("moe_ipc_free", ctypes.c_void_p(silent))
