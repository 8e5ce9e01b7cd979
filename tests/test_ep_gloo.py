"""Expert-parallel exchange on CPU ranks (gloo, world size 2 and 4).

Each rank routes its own tokens with the oracle, sorts its (token, slot)
pairs by expert, and runs the product's ``ep_exchange`` (count all-to-all,
row all-to-all, owner-side expert order, reverse all-to-all) with the oracle
standing in for the device experts.  The combined outputs must equal the
single-process oracle layer exactly: every row is computed by the same oracle
expert on the same input, only moved between ranks.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from linuxnightmaresuite_b200 import ep, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    return synth.MoEConfig("ep_small", 128, 8, 2, 64, 24, synth.QTYPE_Q8_0, 0.01)


def _worker(rank, world, port, out_q):
    sys.path.insert(0, ROOT)
    from oracle import moe_oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        data = synth.make_layer(cfg, 5)               # same weights on every rank
        E, k, d = cfg.n_experts, cfg.top_k, cfg.d_model
        T = data.x.shape[0]
        mine = np.arange(rank, T, world)              # this rank's tokens
        x = data.x[mine]
        ids = np.zeros((len(mine), k), np.int32)
        wts = np.zeros((len(mine), k), np.float32)
        for i in range(len(mine)):
            ids[i], wts[i], _ = orc.route(x[i], data.gate_w, k)
        off, perm, inv = orc.dispatch(ids, E)
        send = torch.from_numpy(x[perm // k].copy())
        counts = torch.from_numpy(np.diff(off).astype(np.int32).reshape(world, -1).copy())
        e0, e1 = ep.expert_range(rank, world, E)
        experts = orc.LazyExperts(data.w_gate, data.w_up, data.w_down, cfg.qtype, d, cfg.ffn)

        def expert_fn(recv, loff, row_map):
            y = np.zeros((recv.shape[0], d), np.float32)
            r = recv.numpy()
            for el in range(e1 - e0):
                for row in row_map[loff[el]:loff[el + 1]]:
                    y[row] = experts[e0 + el].forward(r[row])
            return torch.from_numpy(y)

        y_sorted = ep.ep_exchange(send, counts, expert_fn).numpy()
        out = np.zeros_like(x)
        for i in range(len(mine)):
            acc = np.zeros(d, np.float32)
            for s in range(k):
                acc += wts[i, s] * y_sorted[inv[i * k + s]]
            out[i] = acc
        out_q.put((rank, mine, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_matches_single_process(world):
    from oracle import moe_oracle as orc
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = _cfg()
    data = synth.make_layer(cfg, 5)
    experts = orc.LazyExperts(data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.d_model, cfg.ffn)
    ref, _, _, _ = orc.moe_layer(data.x, data.gate_w, experts, cfg.top_k)
    for rank, mine, out in results:
        assert np.array_equal(out, ref[mine]), rank


def test_local_order_and_plan():
    rc = np.array([[2, 0, 1], [1, 3, 0]])          # 2 sources x 3 local experts
    loff, row_map = ep.local_order(rc)
    assert loff.tolist() == [0, 3, 6, 7]
    # source 0 block: rows 0,1 (e0) 2 (e2); source 1 block: 3 (e0) 4,5,6 (e1)
    assert row_map.tolist() == [0, 1, 3, 4, 5, 6, 2]
    rows, counts = ep.exchange_plan(np.array([0, 2, 2, 5, 9, 9, 10]), 2)
    assert rows.tolist() == [5, 5] and counts.tolist() == [[2, 0, 3], [4, 0, 1]]
    assert ep.expert_range(1, 4, 128) == (32, 64)
    with pytest.raises(ValueError):
        ep.expert_range(0, 3, 128)
