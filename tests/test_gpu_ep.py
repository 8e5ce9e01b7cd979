"""Expert-parallel layer on 2 GPUs (NVLink peer-memory exchange) against the
single-GPU layer.

Runs as child processes (one per GPU); skipped when fewer than 2 GPUs are
visible.  NVLink multicast (NVLS) is off so a failing rank cannot leave a
multicast object bound on its peer.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist

    from linuxnightmaresuite_b200 import synth
    from linuxnightmaresuite_b200.ep import EPMoELayer
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = synth.CONFIGS["decode_t8"]
        T = 32
        data = synth.make_layer(cfg, 3, tokens=T * world)
        layer = EPMoELayer(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.top_k,
                           device=dev)
        x = torch.from_numpy(np.ascontiguousarray(data.x[rank * T:(rank + 1) * T])).to(dev)
        out = layer.forward(x).cpu().numpy()
        out2 = layer.forward(x).cpu().numpy()
        out_q.put((rank, out, out2, layer.device_status()))
        layer.close()
        dist.barrier()
    except Exception as exc:          # report at once instead of leaving the parent waiting
        out_q.put((rank, None, None, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from linuxnightmaresuite_b200 import moe_forward as M, synth
    from oracle import moe_oracle as orc

    from ._util import TOL_MAX_ABS, TOL_REL_L2
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, out2, st = q.get(timeout=300)
        assert out is not None and st == 0, (r, st)
        res[r] = (out, out2)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = synth.CONFIGS["decode_t8"]
    T = 32
    data = synth.make_layer(cfg, 3, tokens=T * world)
    layer = M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                                   cfg.top_k)
    ref = layer.forward_batch(torch.from_numpy(data.x).cuda()).cpu().numpy()
    for r in range(world):
        out, out2 = res[r]
        assert np.array_equal(out, out2)              # run-to-run deterministic
        mx, rel = orc.compare(out, ref[r * T:(r + 1) * T])
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (r, mx, rel)


def _stacked_worker(rank, world, port, out_q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist

    from linuxnightmaresuite_b200 import synth
    from linuxnightmaresuite_b200.stacked import StackedEP
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = synth.CONFIGS["stacked"]
        T = 16
        model = StackedEP.build(cfg, 21, T, device=dev, layers=2)
        x_all = synth.make_layer_slice(cfg, 21, T * world, 0, 0).x
        x = torch.from_numpy(np.ascontiguousarray(x_all[rank * T:(rank + 1) * T])).to(dev)
        out = model.forward(x).cpu().numpy()
        st = max(layer.device_status() for layer in model.layers)
        out_q.put((rank, out, st))
        model.close()
        dist.barrier()
    except Exception as exc:          # report at once instead of leaving the parent waiting
        out_q.put((rank, None, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def test_stacked_ep_with_shared_expert_matches_single_gpu():
    """Two stacked layers (shared expert, RMSNorm, residual) expert-parallel on
    2 GPUs, sharing one exchange window, against the same stack on one GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from linuxnightmaresuite_b200 import synth
    from linuxnightmaresuite_b200.stacked import StackedMoE
    from oracle import moe_oracle as orc

    from ._util import TOL_MAX_ABS, TOL_REL_L2
    world, T = 2, 16
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stacked_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, st = q.get(timeout=300)
        assert out is not None and st == 0, (r, st)
        res[r] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = synth.CONFIGS["stacked"]
    E = cfg.n_experts
    ref_model = StackedMoE.from_layers(
        [synth.make_layer_slice(cfg, 21 + li, T * world, 0, E) for li in range(2)])
    x_all = synth.make_layer_slice(cfg, 21, T * world, 0, 0).x
    ref = ref_model.forward(torch.from_numpy(x_all).cuda()).cpu().numpy()
    for r in range(world):
        mx, rel = orc.compare(res[r], ref[r * T:(r + 1) * T])
        assert mx <= TOL_MAX_ABS and rel <= TOL_REL_L2, (r, mx, rel)
