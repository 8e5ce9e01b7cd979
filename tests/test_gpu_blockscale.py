"""The block-scale tcgen05 expert kernels (exact integer weights, one tensor-
memory accumulator per 32-wide block, scale applied in registers) against the
oracle through the C ABI: every chunk size, ragged groups (empty experts, a
partial chunk, experts spanning several chunks), gather / scatter row maps, a
partial last output tile (d not a multiple of 128) and an odd number of 64-wide
k tiles, the expert variant options, and the same inputs through each kernel
family."""
import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import kernels as K, synth
from oracle import moe_oracle as orc

from ._util import TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(qt, d, F, counts, seed, act=0, scale=False):
    rng = np.random.default_rng(seed)
    E = len(counts)
    s = 0.002 if qt == 8 else 0.01
    wg = synth.quant_matrix(rng, qt, E, F, d, s)
    wu = synth.quant_matrix(rng, qt, E, F, d, s)
    wd = synth.quant_matrix(rng, qt, E, d, F, s)
    ds = (0.5 + rng.uniform(0, 1, E)).astype(np.float32) if scale else None
    experts = []
    for e in range(E):
        g = orc.dequantize_matrix(wg[e], qt, F, d)
        u = orc.dequantize_matrix(wu[e], qt, F, d)
        dn = orc.dequantize_matrix(wd[e], qt, d, F)
        if ds is not None:
            dn = dn * float(ds[e])
        experts.append(orc.GeGLUExpert(g, u, dn) if act else orc.DenseExpert(g, u, dn))
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return rng, wg, wu, wd, ds, experts, off


def _check(y, x, x_rows, y_rows, off, experts):
    for e, ex in enumerate(experts):
        for r in range(off[e], off[e + 1]):
            exp = ex.forward(x[x_rows[r]] if x_rows is not None else x[r])
            got = y[y_rows[r]] if y_rows is not None else y[r]
            mx, rel = orc.compare(got, exp)
            assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (e, r, mx, rel)


@pytest.mark.parametrize("qt", [2, 8])
@pytest.mark.parametrize("rb", [8, 16, 32, 64])
@pytest.mark.parametrize("d,F", [(256, 128), (320, 192)])
def test_blockscale_chunks_and_row_maps(qt, rb, d, F):
    counts = [3, 0, rb + 5, 1, 2 * rb]
    rng, wg, wu, wd, _, experts, off = _case(qt, d, F, counts, seed=qt * 100 + rb + d)
    rows = int(off[-1])
    n_tok = rows + 7
    x = rng.standard_normal((n_tok, d), dtype=np.float32)
    x_rows = rng.permutation(n_tok)[:rows].astype(np.int32)
    y_rows = rng.permutation(rows).astype(np.int32)
    E = len(counts)
    pk = [K.pack_weights(cuda(w.reshape(-1)), qt, E, *sh)
          for w, sh in ((wg, (F, d)), (wu, (F, d)), (wd, (d, F)))]
    ws = K.workspace(K._size_out("moe_experts_workspace_bytes", rows, E, d, F), "cuda")
    ws[:256].zero_()
    opts = K.ExpertOpts(kernels=K.KERNELS_BLOCKSCALE, chunk_rows=rb)
    y = K.experts(pk[0], pk[1], pk[2], qt, cuda(off), cuda(x), d, F, x_rows=cuda(x_rows),
                  y_rows=cuda(y_rows), rows=rows, ws=ws, opts=opts)
    torch.cuda.synchronize()
    assert K.read_status(ws) == 0
    _check(y.cpu().numpy(), x, x_rows, y_rows, off, experts)


@pytest.mark.parametrize("family", [1, 2, 3])
def test_families_agree_at_full_width(family):
    """Decode width (d=2816, F=704: an odd number of 64-wide k tiles in the
    down projection), ragged Poisson groups of mean 6: the GEMV, block-scale and
    split-GEMM families each match the oracle."""
    qt, d, F = 2, 2816, 704
    counts = list(np.random.default_rng(5).poisson(6, 12))
    rng, wg, wu, wd, _, experts, off = _case(qt, d, F, counts, seed=77)
    rows = int(off[-1])
    x = rng.standard_normal((rows, d), dtype=np.float32)
    E = len(counts)
    pk = [K.pack_weights(cuda(w.reshape(-1)), qt, E, *sh)
          for w, sh in ((wg, (F, d)), (wu, (F, d)), (wd, (d, F)))]
    ws = K.workspace(K._size_out("moe_experts_workspace_bytes", rows, E, d, F), "cuda")
    ws[:256].zero_()
    y = K.experts(pk[0], pk[1], pk[2], qt, cuda(off), cuda(x), d, F, rows=rows, ws=ws,
                  opts=K.ExpertOpts(kernels=family))
    torch.cuda.synchronize()
    assert K.read_status(ws) == 0
    _check(y.cpu().numpy(), x, None, None, off, experts)


@pytest.mark.parametrize("rb", [8, 32])
def test_blockscale_expert_variant(rb):
    """GeGLU-tanh, a per-expert down scale and a fused gate_up stack."""
    qt, d, F = 8, 512, 256
    counts = [5, rb + 3, 0, 2]
    rng, wg, wu, wd, ds, experts, off = _case(qt, d, F, counts, seed=rb, act=1, scale=True)
    rows = int(off[-1])
    x = rng.standard_normal((rows, d), dtype=np.float32)
    E = len(counts)
    gu = np.concatenate([wg, wu], axis=1)    # (E, 2F, row bytes): gate rows, then up rows
    pgu = K.pack_weights(cuda(gu.reshape(-1)), qt, E, 2 * F, d)
    pd = K.pack_weights(cuda(wd.reshape(-1)), qt, E, d, F)
    mat = F * (d // 32) * K.BLOCK_BYTES[qt]
    opts = K.ExpertOpts(act=K.ACT_GEGLU_TANH, gate_up_stride=2 * mat, down_scale=cuda(ds),
                        kernels=K.KERNELS_BLOCKSCALE, chunk_rows=rb)
    y = K.experts(pgu, pgu[mat:], pd, qt, cuda(off), cuda(x), d, F, rows=rows, opts=opts)
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), x, None, None, off, experts)
