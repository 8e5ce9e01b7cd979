#!/usr/bin/env python
"""MoE layer forward benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200|reference]

A step is one MoE layer forward (router -> dispatch -> grouped SwiGLU experts
-> combine) over one batch of synthetic tokens whose weights are GGUF Q4_0 /
Q8_0 blocks resident in HBM.  The default workload is the decode layer
(d_model 2816, 128 experts, top-8, expert ffn 704, 64 tokens, Q4_0).

Timing: W untimed warm-up steps; then K steps, each preceded by a 512 MiB
write that flushes the 126 MB L2 (the flush is outside each step's CUDA-event
pair), bracketed by a barrier and a device synchronise; the step time is the
mean of the per-step event durations, max over ranks.  ``e2e`` repeats the
steps through the public API with the tokens in pinned host memory: the
host->device copy of the inputs and the device->host read of the output are
inside each timed step.

Per-kernel device times come from the library's own event profiler during the
timed steps; the roofline reports the dominant kernel.  With ``--gpus N`` the
script runs under torchrun, one process per GPU.

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle, a restatement of moe_forward.MoELayer.forward on numpy/OpenBLAS) on
the host cores for the same workload, on a bounded token sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

# the CPU legs use every host core through OpenBLAS; set before numpy loads
os.environ.setdefault("OPENBLAS_NUM_THREADS", str(os.cpu_count() or 1))

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from linuxnightmaresuite_b200 import synth  # noqa: E402

METRIC = "MoE layer tokens/s"
UNIT = "tokens/s"
FLUSH_BYTES = 512 << 20

# name -> (config, tokens, tokens split over the ranks?, layers)
#   split False: each rank routes `tokens` of its own (weak scaling);
#   split True:  the step's `tokens` are divided over the ranks (strong scaling)
WORKLOADS = {
    "decode_t64": ("decode_t64", 64, False, 1),
    "decode_t8": ("decode_t8", 8, False, 1),
    "decode_t1": ("decode_t1", 1, False, 1),
    "prefill": ("prefill", 4096, False, 1),
    "ep": ("ep", 8192, True, 1),
    "stacked_layer": ("stacked", 256, False, 1),
    "stacked": ("stacked", 256, True, 30),
}


def parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode_t64", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_desc(cfg: synth.MoEConfig, T: int) -> str:
    q = {2: "Q4_0", 8: "Q8_0"}[cfg.qtype]
    s = (f"{cfg.name}: d_model={cfg.d_model} E={cfg.n_experts} top-{cfg.top_k} "
         f"ffn={cfg.ffn} T={T} {q}")
    if cfg.shared_ffn:
        s += f" + shared ffn={cfg.shared_ffn} Q8_0"
    if cfg.zipf_s:
        s += f" zipf({cfg.zipf_s}) expert bias"
    return s


# ----------------------------------------------------------------------------- CPU

def cpu_layer_timing(data, sample_tokens: int, repeats: int, warmup: int):
    """Times the oracle's per-token MoE layer (moe_forward.MoELayer.forward
    restated) on the first ``sample_tokens`` tokens.  Weights are dequantised
    beforehand (outside the timing), as the reference engines cache them."""
    from oracle import moe_oracle as orc
    cfg = data.cfg
    xs = data.x[:sample_tokens]
    experts = orc.LazyExperts(data.w_gate, data.w_up, data.w_down, cfg.qtype, cfg.d_model,
                              cfg.ffn)
    shared = None
    if cfg.shared_ffn:
        shared = orc.expert_from_blocks(data.s_gate[0], data.s_up[0], data.s_down[0],
                                        cfg.shared_qtype, cfg.d_model, cfg.shared_ffn)
    t0 = time.perf_counter()
    for t in range(xs.shape[0]):  # dequantise every expert the sample touches
        ids, _, _ = orc.route(xs[t], data.gate_w, cfg.top_k, cfg.route_mode, data.bias)
        for e in ids:
            experts[e]
    dequant_s = time.perf_counter() - t0
    times = []
    for i in range(warmup + repeats):
        t0 = time.perf_counter()
        orc.moe_layer(xs, data.gate_w, experts, cfg.top_k, cfg.route_mode, shared, data.bias)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times, dequant_s


def cpu_threads() -> int:
    return int(os.environ.get("OPENBLAS_NUM_THREADS", os.cpu_count() or 1))


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    name, T, _, n_layers = WORKLOADS[args.workload]
    cfg = synth.CONFIGS[name]
    data = synth.make_layer(cfg, args.seed, tokens=T)
    sample = min(T, 16)
    times, dq = cpu_layer_timing(data, sample, args.steps, args.warmup)
    ms = 1e3 * float(np.mean(times)) * n_layers   # a stacked step: one layer's time per layer
    value = sample / (ms / 1e3)
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload_desc(cfg, T) + (f" x {n_layers} layers" if n_layers > 1 else ""),
                   "sample_tokens_per_step": sample,
                   "path": "oracle restatement of moe_forward.MoELayer.forward (numpy/OpenBLAS)",
                   "dequant_s_untimed": dq},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"first {sample} of {T} tokens per step, weights pre-dequantised"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- clocks

REASONS = [(0x1, "gpu_idle"), (0x2, "applications_clocks_setting"), (0x4, "sw_power_cap"),
           (0x8, "hw_slowdown"), (0x10, "sync_boost"), (0x20, "sw_thermal_slowdown"),
           (0x40, "hw_thermal_slowdown"), (0x80, "hw_power_brake_slowdown"),
           (0x100, "display_clock_setting")]


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self.period = period_s

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= int(r)
        names = [n for b, n in REASONS if bits & b and n != "gpu_idle"]
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(mhz)}


# ----------------------------------------------------------------------------- GPU

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def ncu_traffic(workload: str, kernel: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload, {}).get(kernel)
    except Exception:
        return None


def build_layer(data, device):
    from linuxnightmaresuite_b200 import moe_forward as M
    cfg = data.cfg
    shared = None
    if cfg.shared_ffn:
        shared = (data.s_gate[0], data.s_up[0], data.s_down[0])
    return M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                                  cfg.top_k, shared=shared, shared_qtype=cfg.shared_qtype,
                                  shared_hidden=cfg.shared_ffn, mode=cfg.route_mode,
                                  bias=data.bias, device=device)


def run_b200(args):
    import torch
    import torch.distributed as dist
    from linuxnightmaresuite_b200 import _lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    name, T_step, split, n_layers = WORKLOADS[args.workload]
    cfg = synth.CONFIGS[name]
    if split and T_step % world:
        raise SystemExit(f"{T_step} tokens do not split over {world} ranks")
    T = T_step // world if split else T_step        # tokens per rank
    stacked = n_layers > 1
    model = None
    if stacked:
        # 30 layers, seed + layer index; every layer has a shared expert,
        # RMSNorm and the residual in between
        from linuxnightmaresuite_b200.stacked import StackedEP, StackedMoE
        if world == 1:
            E = cfg.n_experts
            model = StackedMoE.from_layers(
                (synth.make_layer_slice(cfg, args.seed + li, T, 0, E) for li in range(n_layers)),
                device=dev)
            layer = model.layers[0]
        else:
            model = StackedEP.build(cfg, args.seed, T, device=dev)
            layer = model.layers[0]
        x_np = np.ascontiguousarray(
            synth.make_layer_slice(cfg, args.seed, T * world, 0, 0).x[rank * T:(rank + 1) * T])
        data = None
    elif world == 1:
        data = synth.make_layer(cfg, args.seed, tokens=T)
        layer = build_layer(data, dev)
        x_np = data.x
    else:
        # expert parallelism: the same layer on every rank (experts sharded),
        # T tokens per rank
        from linuxnightmaresuite_b200.ep import EPMoELayer
        data = synth.make_layer(cfg, args.seed, tokens=T * world)
        layer = EPMoELayer(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                           cfg.top_k, cfg.route_mode, data.bias, device=dev)
        x_np = np.ascontiguousarray(data.x[rank * T:(rank + 1) * T])
    x = torch.from_numpy(x_np).to(dev)
    out = torch.empty_like(x)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(inp=x):
        if model is not None:
            return model.forward(inp, out=out)
        if world == 1:
            return layer.forward_batch(inp, out=out)
        return layer.forward(inp)

    for _ in range(max(args.warmup, 0)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if world == 1 and layer.device_status() != 0:
        raise RuntimeError("device status error during warm-up")

    # routing statistics of this batch (unique experts -> algorithmic bytes);
    # for the stacked step, those of its first layer
    if world == 1 and stacked:
        ids, _ = layer.router.route_batch(x)
        ids = ids.cpu().numpy()
        uniq = int(np.unique(ids).size)
        rows = int(ids.size)
    elif world == 1:
        _, ids, _ = layer.forward_batch(x, out=out, return_routing=True)
        ids = ids.cpu().numpy()
        uniq = int(np.unique(ids).size)
        rows = int(ids.size)
    else:
        uniq, rows = layer.routing_stats(x)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
        # per-kernel device times: the same steps again with an event pair
        # around every library launch (kept out of the timed steps above,
        # because events between two kernels stop the second one from
        # starting early as a programmatic dependent launch)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        _lib.profile_collect()
        _lib.profile_enable(True)
        for i in range(args.steps):
            flush.zero_()
            step()
        torch.cuda.synchronize()
        _lib.profile_enable(False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = float(np.mean(step_ms))
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = T * world / (ms / 1e3)    # tokens of the whole job per second
    launches = sum(c for _, c in prof.values())

    # end to end through the public API with host buffers
    x_host = torch.from_numpy(x_np).pin_memory()
    out_host = torch.empty(x_host.shape, dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for _ in range(2):
        x_dev.copy_(x_host, non_blocking=True)
        res = step(x_dev)
        out_host.copy_(res, non_blocking=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()
        e_starts[i].record()
        x_dev.copy_(x_host, non_blocking=True)
        res = step(x_dev)
        out_host.copy_(res, non_blocking=True)
        e_ends[i].record()
    torch.cuda.synchronize()
    e2e_ms = float(np.mean([s.elapsed_time(e) for s, e in zip(e_starts, e_ends)]))
    e_t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e_t.item())
    if world == 1 and layer.device_status() != 0:
        raise RuntimeError("device status error during the timed steps")

    hbm_peak, tc_peak, peak_kind = peaks()
    bb = synth.block_bytes(cfg.qtype)
    d, F = cfg.d_model, cfg.ffn
    mat = F * d // 32 * bb
    gu_ms, gu_n = prof["gateup"]
    dn_ms, dn_n = prof["down"]
    kernels = {k: {"ms_total": v[0], "launches": v[1]} for k, v in prof.items() if v[1]}
    gu_launch_ms = gu_ms / gu_n if gu_n else None
    dn_launch_ms = dn_ms / dn_n if dn_n else None
    layer_bytes = uniq * 3 * mat + d * cfg.n_experts * 4 + T * d * 8  # this rank's share
    if cfg.shared_ffn:
        layer_bytes += 3 * cfg.shared_ffn * d // 32 * synth.block_bytes(cfg.shared_qtype)
    layer_bytes *= n_layers
    tensor_bound = rows / max(1, uniq) >= 64      # the tcgen05 GEMM path
    if tensor_bound:
        # gate/up GEMM: 2 * rows * d * 2F algorithmic flops (the three split-operand
        # MMAs that keep f32 accuracy are implementation work, not counted)
        gu_work = 2.0 * rows * d * 2 * F
        dn_work = 2.0 * rows * F * d
        achieved = gu_work / (gu_launch_ms / 1e3) / 1e12 if gu_launch_ms else None
        roofline = {
            "kernel": "tc_gateup_kernel (persistent tcgen05 grouped GEMM + SiLU*up)",
            "bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
            "frac": (achieved / tc_peak) if achieved else None,
            "traffic": ncu_traffic(args.workload, "gateup"),
            "peak_kind": f"{peak_kind} bf16_tflops (dense)",
            "algorithmic_flops_per_launch": gu_work, "launch_ms": gu_launch_ms,
            "executed_tensor_flops_per_launch": 3 * gu_work,
            "layer": {"algorithmic_flops": gu_work + dn_work, "ms": ms,
                      "achieved_tflops": (gu_work + dn_work) / (ms / 1e3) / 1e12},
        }
        if dn_n:
            roofline["down"] = {"algorithmic_flops_per_launch": dn_work, "launch_ms": dn_launch_ms,
                                "achieved_tflops": dn_work / (dn_launch_ms / 1e3) / 1e12}
    else:
        # gate/up GEMV: both matrices of every routed expert, the activation rows
        # it reads and the hidden rows it writes
        gu_bytes = uniq * 2 * mat + rows * d * 4 + rows * F * 4
        dn_bytes = uniq * mat + rows * F * 4 + rows * d * 4
        achieved = gu_bytes / (gu_launch_ms / 1e3) / 1e9 if gu_launch_ms else None
        roofline = {
            "kernel": "gateup (grouped gate/up GEMV + SiLU*up)",
            "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": (achieved / hbm_peak) if achieved else None,
            "traffic": ncu_traffic(args.workload, "gateup"),
            "peak_kind": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu_launch_ms,
            "layer": {"algorithmic_bytes": layer_bytes, "ms": ms,
                      "achieved_gbs": layer_bytes / (ms / 1e3) / 1e9,
                      "frac": layer_bytes / (ms / 1e3) / 1e9 / hbm_peak},
        }
        if dn_n:
            roofline["down"] = {"algorithmic_bytes_per_launch": dn_bytes,
                                "launch_ms": dn_launch_ms,
                                "achieved": dn_bytes / (dn_launch_ms / 1e3) / 1e9}

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and data is not None:
        sample = min(T, 16)
        times, dq = cpu_layer_timing(data, sample, 3, 1)
        cms = float(np.median(times))
        cpu_base = {"value": sample / cms, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                    "sample": f"first {sample} of {T} tokens, median of 3 runs, weights "
                              f"pre-dequantised ({dq:.1f} s, untimed)"}

    if world > 1:
        (model if model is not None else layer).close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if split else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_desc(cfg, T_step) + (f" x {n_layers} layers" if stacked else ""),
                   "tokens_per_rank": T, "layers": n_layers,
                   "unique_experts": uniq, "routed_rows": rows,
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "experts_per_rank": cfg.n_experts // world,
                   "l2": f"flushed by a {FLUSH_BYTES >> 20} MiB write before every step "
                         "(outside the step events)",
                   "weights_bytes_resident": 3 * cfg.n_experts * mat},
        "roofline": roofline,
        "kernels": kernels,
        "kernels_timing": "event pair per launch, in a second pass of the same steps",
        "cpu_baseline": cpu_base,
        "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(x_host.numel() * 4),
                "d2h_bytes_per_step": int(out_host.numel() * 4)},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
