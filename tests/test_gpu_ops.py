"""GPU parity of the individual stages through the C ABI, against the oracle."""
import os

import numpy as np
import pytest
import torch

from linuxnightmaresuite_b200 import _lib, kernels as K, synth
from oracle import moe_oracle as orc

from ._util import GOLD, TOL_MAX_ABS, TOL_REL_L2, TOL_W_ATOL, TOL_W_RTOL

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_dequantize_known_answers_bit_exact():
    z = np.load(os.path.join(GOLD, "kat_blocks.npz"))
    for raw, exp, qt in ((z["q8_raw"], z["q8_expected"], 8), (z["q4_raw"], z["q4_expected"], 2)):
        got = K.dequantize(cuda(raw.reshape(-1)), qt, raw.shape[0] * 32).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("qt", [2, 8])
def test_dequantize_random_blocks_bit_exact(qt):
    rng = np.random.default_rng(3)
    raw = synth.quant_matrix(rng, qt, 3, 64, 256, 0.05)
    exp = orc.DEQUANT[qt](raw.reshape(-1), raw.size // synth.block_bytes(qt) * 32)
    got = K.dequantize(cuda(raw.reshape(-1)), qt, exp.size).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("qt", [2, 8])
def test_pack_unpack_round_trip(qt):
    rng = np.random.default_rng(4)
    raw = synth.quant_matrix(rng, qt, 5, 48, 192, 0.01)
    t = cuda(raw.reshape(-1))
    packed = K.pack_weights(t, qt, 5, 48, 192)
    assert packed.numel() == raw.size
    assert not torch.equal(packed, t)
    back = K.unpack_weights(packed, qt, 5, 48, 192)
    assert torch.equal(back, t)


@pytest.mark.parametrize("case", [0, 1, 2])
@pytest.mark.parametrize("mode", [0, 1])
def test_router_matches_reference_goldens(case, mode):
    z = np.load(os.path.join(GOLD, "router.npz"))
    x, G, k = z[f"c{case}_x"], z[f"c{case}_G"], int(z[f"c{case}_k"])
    ids, w = K.router(cuda(x), cuda(G), k, mode)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    for t in range(x.shape[0]):
        exp_ids, exp_w, tie = orc.route(x[t], G, k, mode)
        assert np.array_equal(ids[t], exp_ids), (t, ids[t], exp_ids)
        np.testing.assert_allclose(w[t], exp_w, rtol=TOL_W_RTOL, atol=TOL_W_ATOL)
        if mode == 1 or not tie:
            # the reference's own decision (production ids were made on the
            # stable-sorting substrate, so they hold on tie tokens too)
            assert np.array_equal(ids[t], z[f"c{case}_ids_mode{mode}"][t])


@pytest.mark.parametrize("layout", [_lib.MOE_ROUTER_D_E, _lib.MOE_ROUTER_E_D])
@pytest.mark.parametrize("T,d,E,k", [(1, 2816, 128, 8), (64, 2816, 128, 8), (300, 1024, 8, 2),
                                     (33, 4096, 128, 8), (5, 64, 4, 4), (17, 128, 256, 32),
                                     (512, 2816, 128, 8), (200, 4096, 256, 8), (130, 2816, 132, 4)])
def test_router_shapes_and_layouts(layout, T, d, E, k):
    rng = np.random.default_rng(T * 7 + d)
    x = rng.standard_normal((T, d), dtype=np.float32)
    G = rng.standard_normal((d, E), dtype=np.float32) * np.float32(0.02)
    bias = rng.standard_normal(E).astype(np.float32) * np.float32(0.1)
    Gd = cuda(G if layout == _lib.MOE_ROUTER_D_E else G.T.copy())
    for mode in (0, 1):
        ids, w = K.router(cuda(x), Gd, k, mode, cuda(bias), layout)
        ids, w = ids.cpu().numpy(), w.cpu().numpy()
        for t in range(T):
            exp_ids, exp_w, _ = orc.route(x[t], G, k, mode, bias)
            if not np.array_equal(ids[t], exp_ids):
                from ._util import near_tie
                lg = orc.router_logits(x[t], G, bias)
                assert near_tie(lg if mode == 0 else np.exp(lg - lg.max()), k)
                continue
            np.testing.assert_allclose(w[t], exp_w, rtol=TOL_W_RTOL, atol=TOL_W_ATOL)


def test_router_exact_ties_take_higher_index_first():
    d, E, k = 32, 16, 5
    x = np.ones((3, d), np.float32)
    G = np.zeros((d, E), np.float32)     # all logits equal
    ids, w = K.router(cuda(x), cuda(G), k, 0)
    assert ids.cpu().numpy().tolist() == [[15, 14, 13, 12, 11]] * 3
    np.testing.assert_allclose(w.cpu().numpy(), 0.2, rtol=1e-6)
    ids, w = K.router(cuda(x), cuda(G), k, 1)
    assert ids.cpu().numpy().tolist() == [[11, 12, 13, 14, 15]] * 3


@pytest.mark.parametrize("T,k,E,skew", [(1, 8, 128, 0), (64, 8, 128, 0), (4096, 8, 128, 1),
                                        (777, 2, 8, 1), (3, 4, 1024, 0), (5000, 1, 16, 2),
                                        # >= 4096 pairs: the chunked (multi-CTA) dispatch
                                        (1024, 4, 1024, 0), (8192, 8, 128, 0), (4099, 1, 8, 1)])
def test_dispatch_matches_stable_counting_sort(T, k, E, skew):
    rng = np.random.default_rng(T + E)
    if skew == 1:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        ids = rng.choice(E, size=(T, k), p=p / p.sum())
    elif skew == 2:
        ids = np.full((T, k), E - 1)            # every pair to one expert
    else:
        ids = rng.integers(0, E, size=(T, k))
    ids = ids.astype(np.int32)
    off, perm, inv = K.dispatch(cuda(ids), E)
    e_off, e_perm, e_inv = orc.dispatch(ids, E)
    assert np.array_equal(off.cpu().numpy(), e_off)
    assert np.array_equal(perm.cpu().numpy(), e_perm)
    assert np.array_equal(inv.cpu().numpy(), e_inv)


def test_chunked_dispatch_flags_bad_expert_ids():
    rng = np.random.default_rng(11)
    T, k, E = 2048, 4, 64
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ids[5, 1], ids[1000, 3], ids[2047, 0] = E, -3, 99
    nbytes = K._size_out("moe_dispatch_workspace_bytes", T, k, E)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    off, perm, inv = K.dispatch(cuda(ids), E, ws)
    assert K.read_status(ws) & _lib.MOE_STATUS_BAD_EXPERT_ID
    good = (ids >= 0) & (ids < E)
    inv = inv.cpu().numpy()
    assert (inv[~good.reshape(-1)] == -1).all()
    # the valid pairs keep the stable order of the valid ids
    flat = ids.reshape(-1)
    order = np.argsort(np.where(good.reshape(-1), flat, E), kind="stable")[:good.sum()]
    assert np.array_equal(perm.cpu().numpy()[:good.sum()], order)
    assert off.cpu().numpy()[-1] == good.sum()


def test_dispatch_flags_bad_expert_ids():
    ids = np.array([[0, 3], [9, 1], [-1, 2]], np.int32)
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    off, perm, inv = K.dispatch(cuda(ids), 4, ws)
    assert K.read_status(ws) & _lib.MOE_STATUS_BAD_EXPERT_ID
    inv = inv.cpu().numpy()
    assert inv[2] == -1 and inv[4] == -1
    assert off.cpu().numpy().tolist() == [0, 1, 2, 3, 4]
    assert K.read_status(ws) == 0            # reading clears it


@pytest.mark.parametrize("qt", [2, 8])
@pytest.mark.parametrize("d,F,n", [(256, 128, 1), (256, 128, 3), (1024, 2816, 4), (2816, 704, 5),
                                   (512, 192, 17), (2816, 704, 40), (128, 64, 2),
                                   # >= 64 rows: the tcgen05 GEMM path
                                   (256, 128, 64), (2816, 704, 300), (1024, 2816, 130),
                                   (512, 192, 257)])
def test_single_expert_matches_oracle(qt, d, F, n):
    rng = np.random.default_rng(d + F + n + qt)
    s = 0.002 if qt == 8 else 0.01
    wg = synth.quant_matrix(rng, qt, 1, F, d, s)
    wu = synth.quant_matrix(rng, qt, 1, F, d, s)
    wd = synth.quant_matrix(rng, qt, 1, d, F, s)
    x = rng.standard_normal((n, d), dtype=np.float32)
    ex = orc.expert_from_blocks(wg[0], wu[0], wd[0], qt, d, F)
    exp = np.stack([ex.forward(x[i]) for i in range(n)])
    pg = K.pack_weights(cuda(wg.reshape(-1)), qt, 1, F, d)
    pu = K.pack_weights(cuda(wu.reshape(-1)), qt, 1, F, d)
    pd = K.pack_weights(cuda(wd.reshape(-1)), qt, 1, d, F)
    off = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    y = K.experts(pg, pu, pd, qt, off, cuda(x), d, F, rows=n).cpu().numpy()
    mx, rel = orc.compare(y, exp)
    assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (mx, rel)


def test_experts_row_maps_and_empty_experts():
    """Gather/scatter maps, experts with no rows, and the (E_local+1) offsets."""
    rng = np.random.default_rng(11)
    qt, d, F, E = 8, 256, 128, 6
    wg = synth.quant_matrix(rng, qt, E, F, d, 0.002)
    wu = synth.quant_matrix(rng, qt, E, F, d, 0.002)
    wd = synth.quant_matrix(rng, qt, E, d, F, 0.002)
    counts = [3, 0, 7, 0, 0, 1]
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(off[-1])
    x = rng.standard_normal((20, d), dtype=np.float32)
    x_rows = rng.permutation(20)[:rows].astype(np.int32)
    y_rows = rng.permutation(rows).astype(np.int32)
    pk = [K.pack_weights(cuda(w.reshape(-1)), qt, E, *sh)
          for w, sh in ((wg, (F, d)), (wu, (F, d)), (wd, (d, F)))]
    y = K.experts(pk[0], pk[1], pk[2], qt, cuda(off), cuda(x), d, F, x_rows=cuda(x_rows),
                  y_rows=cuda(y_rows), rows=rows).cpu().numpy()
    for e in range(E):
        ex = orc.expert_from_blocks(wg[e], wu[e], wd[e], qt, d, F)
        for r in range(off[e], off[e + 1]):
            exp = ex.forward(x[x_rows[r]])
            mx, rel = orc.compare(y[y_rows[r]], exp)
            assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2


def test_combine_and_rms_norm():
    rng = np.random.default_rng(12)
    T, k, d = 9, 3, 128
    y = rng.standard_normal((T * k, d), dtype=np.float32)
    inv = rng.permutation(T * k).astype(np.int32)
    w = rng.random((T, k), dtype=np.float32)
    sh = rng.standard_normal((T, d), dtype=np.float32)
    res = rng.standard_normal((T, d), dtype=np.float32)
    out = K.combine(cuda(y), cuda(inv), cuda(w), cuda(sh), cuda(res)).cpu().numpy()
    for t in range(T):
        acc = np.zeros(d, np.float32)
        for s in range(k):
            acc += w[t, s] * y[inv[t * k + s]]
        acc += sh[t]
        assert np.array_equal(out[t], res[t] + acc)
    x = rng.standard_normal((T, 2816), dtype=np.float32)
    nw = (1 + 0.1 * rng.standard_normal(2816)).astype(np.float32)
    got = K.rms_norm(cuda(x), cuda(nw)).cpu().numpy()
    exp = np.stack([orc.rms_norm(x[t], nw) for t in range(T)])
    np.testing.assert_allclose(got, exp, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("d", [100, 128, 1000, 2816, 4096, 8192])
def test_rms_norm_widths(d):
    """Warp-per-row path (perfect pairwise trees: 128, 2816, 4096) and the
    CTA path (100, 1000, 8192), odd row counts."""
    rng = np.random.default_rng(d)
    T = 37
    x = (rng.standard_normal((T, d)) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    got = K.rms_norm(cuda(x), cuda(nw)).cpu().numpy()
    exp = np.stack([orc.rms_norm(x[t], nw) for t in range(T)])
    np.testing.assert_allclose(got, exp, rtol=2e-6, atol=1e-6)
    again = K.rms_norm(cuda(x), cuda(nw)).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))


def test_gather_rows_and_ep_local_order():
    from linuxnightmaresuite_b200 import ep
    rng = np.random.default_rng(21)
    x = rng.standard_normal((40, 96), dtype=np.float32)
    rows = rng.integers(0, 40 * 3, size=77).astype(np.int32)
    got = K.gather_rows(cuda(x), cuda(rows), 3).cpu().numpy()
    assert np.array_equal(got, x[rows // 3])
    for W, El in ((2, 64), (4, 32), (8, 16), (3, 5)):
        rc = rng.integers(0, 6, size=(W, El)).astype(np.int32)
        rc[rng.random((W, El)) < 0.3] = 0
        R = int(rc.sum())
        ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
        loff, rmap = K.ep_local_order(cuda(rc), R, ws)
        e_loff, e_map = ep.local_order(rc)
        assert np.array_equal(loff.cpu().numpy(), e_loff)
        assert np.array_equal(rmap.cpu().numpy()[:R], e_map)
        assert K.read_status(ws) == 0
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    K.ep_local_order(cuda(np.full((2, 4), 3, np.int32)), 10, ws)   # 24 rows > 10
    assert K.read_status(ws) & _lib.MOE_STATUS_ROW_OVERFLOW
