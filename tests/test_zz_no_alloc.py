"""The allocation-free router entry point, moe_router_noalloc.

It exists for callers that cannot allocate device memory and cannot let the
library allocate either (their device memory is already owned by their own
pool, or they must keep a fixed footprint).  It keeps its scratch in a fixed
array inside the library instead of a caller workspace.  These tests call it
through the C ABI and check it against moe_router, the workspace-taking entry
point, on two calls in a row (the second smaller, so stale contents from the
first call would show), plus the size limit.  This file is collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import _lib, kernels as K

from ._util import TOL_W_ATOL, TOL_W_RTOL

pytestmark = pytest.mark.gpu


def _noalloc(x, G, bias, k, mode, layout=_lib.MOE_ROUTER_D_E):
    T, d = x.shape
    E = G.shape[1] if layout == _lib.MOE_ROUTER_D_E else G.shape[0]
    ids = torch.empty((T, k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, k), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    rc = lib.moe_router_noalloc(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(G.data_ptr()),
                                ctypes.c_void_p(0 if bias is None else bias.data_ptr()),
                                T, d, E, k, layout, mode, ctypes.c_void_p(ids.data_ptr()),
                                ctypes.c_void_p(w.data_ptr()),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return ids, w


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_router_matches_workspace_router_twice(mode):
    rng = np.random.default_rng(42 + mode)
    d, E, k = 2816, 128, 8
    G = torch.from_numpy(rng.standard_normal((d, E), dtype=np.float32) * np.float32(0.02)).cuda()
    bias = torch.from_numpy(rng.standard_normal(E).astype(np.float32) * np.float32(0.1)).cuda()
    for T in (300, 64, 7):       # each call smaller than the one before; 300 takes the tiled pass
        x = torch.from_numpy(rng.standard_normal((T, d), dtype=np.float32)).cuda()
        ids_n, w_n = _noalloc(x, G, bias, k, mode)
        ids_r, w_r = K.router(x, G, k, mode, bias)
        torch.cuda.synchronize()
        assert torch.equal(ids_n, ids_r)
        np.testing.assert_allclose(w_n.cpu().numpy(), w_r.cpu().numpy(),
                                   rtol=TOL_W_RTOL, atol=TOL_W_ATOL)


def test_noalloc_router_rejects_oversized_calls():
    # any slice plan keeps at least T x E partial logits: 16384 x 128 is twice
    # the fixed scratch
    d, E, k, T = 2816, 128, 8, 16384
    x = torch.zeros((T, d), dtype=torch.float32, device="cuda")
    G = torch.zeros((d, E), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.MoEError) as err:
        _noalloc(x, G, None, k, 0)
    assert err.value.status == _lib.MOE_ERR_WORKSPACE
    assert "fixed scratch" in str(err.value)
