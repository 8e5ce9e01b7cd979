#!/usr/bin/env python
"""MoE layer forward benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl b200|reference] [--no-workloads] [--no-cpu-baseline]

A step is one MoE layer forward (router -> dispatch -> grouped SwiGLU experts
-> combine) over one batch of synthetic tokens whose expert weights are GGUF
Q4_0 / Q8_0 blocks resident in HBM.  The headline workload is the decode layer
(d_model 2816, 128 experts, top-8, expert ffn 704, 64 tokens, Q4_0).  After it,
in the same process and JSON line (``workloads``), come the prefill layer
(4096 tokens, Q8_0, Zipf-skewed routing; one GPU only), the expert-parallel
layer (d_model 4096, ffn 1536, 8192 tokens per step split over the ranks,
Q8_0) and the stacked decode step (30 layers with a shared expert, 256 tokens
split over the ranks).  With N GPUs (torchrun, one process per GPU) the decode
and stacked workloads are expert-parallel too.

Timing: W untimed warm-up steps; then K steps, each preceded by a 512 MiB write
that flushes the 126 MB L2 and (N > 1) a one-element all-reduce that lines the
ranks up, both outside the step's CUDA-event pair; the step time is the mean of
the per-step event durations, max over ranks.  ``e2e`` repeats the steps
through the public API with the tokens in pinned host memory: the host->device
copy of the inputs and the device->host read of the output are inside each
timed step.  Per-kernel device times come from the library's own event
profiler in a second pass of the same steps.  Every rank reads its device
status word after each workload and checks two of its tokens against the
oracle (outside the timed region); a non-zero status fails the run.

Weights are drawn on the GPU by a seeded generator (per expert, so a rank
builds only its experts); tokens and router weights come from numpy.

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle, a restatement of moe_forward.MoELayer.forward on numpy/OpenBLAS) on
the host cores for the headline workload.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time


def _physical_cores() -> int:
    try:
        import psutil
        n = psutil.cpu_count(logical=False)
        if n:
            return int(n)
    except Exception:
        pass
    return os.cpu_count() or 1


# the CPU legs use every physical core through OpenBLAS; set before numpy loads
os.environ.setdefault("OPENBLAS_NUM_THREADS", str(_physical_cores()))

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from linuxnightmaresuite_b200 import synth  # noqa: E402

METRIC = "MoE layer tokens/s"
UNIT = "tokens/s"
FLUSH_BYTES = 512 << 20


class Workload:
    """name, configuration, tokens per step, tokens split over ranks (strong
    scaling) or per rank (weak), layers per step, tokens of the CPU sample."""

    def __init__(self, name, cfg, tokens, split, layers, cpu_tokens, single_gpu=False):
        self.name, self.cfg, self.tokens, self.split = name, cfg, tokens, split
        self.layers, self.cpu_tokens, self.single_gpu = layers, cpu_tokens, single_gpu


C = synth.CONFIGS
WORKLOADS = {
    "decode_t64": Workload("decode_t64", C["decode_t64"], 64, False, 1, 64),
    "decode_t8": Workload("decode_t8", C["decode_t8"], 8, False, 1, 8),
    "decode_t1": Workload("decode_t1", C["decode_t1"], 1, False, 1, 1),
    "prefill": Workload("prefill", C["prefill"], 4096, False, 1, 64, single_gpu=True),
    "ep": Workload("ep", C["ep"], 8192, True, 1, 4),
    "stacked_layer": Workload("stacked_layer", C["stacked"], 256, False, 1, 16),
    "stacked": Workload("stacked", C["stacked"], 256, True, 30, 16),
}
EXTRA = ("prefill", "ep", "stacked")   # measured after the headline


def parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode_t64", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-workloads", action="store_true",
                    help="measure only --workload (no prefill / ep / stacked record)")
    ap.add_argument("--extra-steps", type=int, default=10,
                    help="timed steps of each extra workload (at most --steps)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_desc(wl: Workload) -> str:
    cfg = wl.cfg
    q = {2: "Q4_0", 8: "Q8_0"}[cfg.qtype]
    s = (f"{wl.name}: d_model={cfg.d_model} E={cfg.n_experts} top-{cfg.top_k} "
         f"ffn={cfg.ffn} T={wl.tokens} {q}")
    if cfg.shared_ffn:
        s += f" + shared ffn={cfg.shared_ffn} Q8_0"
    if cfg.zipf_s:
        s += f" zipf({cfg.zipf_s}) expert bias"
    if wl.layers > 1:
        s += f" x {wl.layers} layers (RMSNorm + residual between layers)"
    return s


# ----------------------------------------------------------------------------- data

def gen_device():
    import torch
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
        else torch.device("cpu")


class HostExperts:
    """Oracle experts of a device-generated layer: each expert's blocks are
    regenerated on the generating device, copied to the host and dequantised
    the first time a token routes to it."""

    def __init__(self, cfg, seed, layer, device):
        self.cfg, self.seed, self.layer, self.device = cfg, seed, layer, device
        self.cache = {}

    def __getitem__(self, e):
        from oracle import moe_oracle as orc
        e = int(e)
        if e not in self.cache:
            g, u, d = synth.device_expert(self.cfg, self.seed, self.layer, e, self.device)
            cfg = self.cfg
            self.cache[e] = orc.expert_from_blocks(g.cpu().numpy(), u.cpu().numpy(),
                                                   d.cpu().numpy(), cfg.qtype, cfg.d_model,
                                                   cfg.ffn)
        return self.cache[e]


def host_shared(data):
    from oracle import moe_oracle as orc
    cfg = data.cfg
    if not cfg.shared_ffn:
        return None
    return orc.expert_from_blocks(data.s_gate[0].cpu().numpy(), data.s_up[0].cpu().numpy(),
                                  data.s_down[0].cpu().numpy(), cfg.shared_qtype, cfg.d_model,
                                  cfg.shared_ffn)


def oracle_tokens(wl: Workload, seed: int, xs: np.ndarray, dev, datas=None):
    """Expected outputs of the rows xs (from the step's input) by the oracle,
    every layer of the workload in turn."""
    from oracle import moe_oracle as orc
    cfg = wl.cfg
    T_total = wl.tokens
    if wl.layers == 1:
        data = datas[0] if datas else synth.make_layer_device(cfg, seed, T_total, 0, 0, dev)
        out, _, _, _ = orc.moe_layer(xs, data.gate_w, HostExperts(cfg, seed, 0, dev), cfg.top_k,
                                     cfg.route_mode, host_shared(data), data.bias)
        return out

    def layers():
        for li in range(wl.layers):
            data = synth.make_layer_device(cfg, seed, T_total, 0, 0, dev, layer=li)
            yield (data.gate_w, HostExperts(cfg, seed, li, dev), host_shared(data), data.norm_w,
                   data.bias)
    return orc.stacked_forward(xs, layers(), cfg.top_k, cfg.route_mode)


# ----------------------------------------------------------------------------- CPU

def cpu_layer_timing(wl: Workload, seed: int, n_tokens: int, repeats: int, warmup: int):
    """Times the oracle's per-token MoE layer (moe_forward.MoELayer.forward
    restated) on the first ``n_tokens`` tokens of the workload's first layer.
    Experts are dequantised beforehand (outside the timing), as the reference
    holds them.  Returns (seconds per run, dequantisation seconds)."""
    from oracle import moe_oracle as orc
    cfg = wl.cfg
    dev = gen_device()
    data = synth.make_layer_device(cfg, seed, wl.tokens, 0, 0, dev)
    xs = np.ascontiguousarray(data.x[:n_tokens])
    if wl.layers > 1:   # the layer's input is the normalised residual stream
        xs = np.stack([orc.rms_norm(xs[t], data.norm_w).astype(np.float32)
                       for t in range(n_tokens)])
    experts = HostExperts(cfg, seed, 0, dev)
    shared = host_shared(data)
    t0 = time.perf_counter()
    for t in range(n_tokens):  # dequantise every expert the sample touches
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
    return int(os.environ.get("OPENBLAS_NUM_THREADS", _physical_cores()))


def cpu_baseline(wl: Workload, seed: int, n_tokens=None, repeats=5, warmup=2):
    n = wl.cpu_tokens if n_tokens is None else n_tokens
    times, dq = cpu_layer_timing(wl, seed, n, repeats, warmup)
    sec = float(np.median(times)) * wl.layers     # a stacked step: one layer's time per layer
    layers = f", scaled x{wl.layers} layers" if wl.layers > 1 else ""
    return {"value": n / sec, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": f"first {n} of {wl.tokens} tokens of layer 0{layers}; median of "
                      f"{repeats} runs after {warmup} warm-up; experts pre-dequantised "
                      f"({dq:.1f} s, untimed); OPENBLAS_NUM_THREADS={cpu_threads()} "
                      f"(physical cores)",
            "ms_per_run": 1e3 * float(np.median(times))}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    n = min(wl.tokens, wl.cpu_tokens)
    # at least 2 warm-up runs and the median of at least 5
    times, dq = cpu_layer_timing(wl, args.seed, n, max(args.steps, 5), max(args.warmup, 2))
    ms = 1e3 * float(np.median(times)) * wl.layers
    value = n / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload_desc(wl), "sample_tokens_per_step": n,
                   "path": "oracle restatement of moe_forward.MoELayer.forward (numpy/OpenBLAS)",
                   "dequant_s_untimed": dq},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                         "sample": f"first {n} of {wl.tokens} tokens per step, weights "
                                   f"pre-dequantised, physical cores, median of "
                                   f"{max(args.steps, 5)} runs after {max(args.warmup, 2)} "
                                   f"warm-up"},
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

    def _sample(self):
        nv = self._nv
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.samples.append((mhz, rs))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
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
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any
    (captured on one GPU; not used for expert-parallel runs)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload, {}).get(kernel)
    except Exception:
        return None


class Built:
    """A workload ready to step on this rank.  host_io: the step takes pinned
    host tensors itself (its kernels read x and write the output over the bus)."""

    def __init__(self, wl, step, x_np, T, datas, status, close, routing_stats, host_io=False):
        self.wl, self.step, self.x_np, self.T, self.datas = wl, step, x_np, T, datas
        self.status, self.close, self.routing_stats = status, close, routing_stats
        self.host_io = host_io


def build(wl: Workload, seed: int, rank: int, world: int, dev) -> Built:
    import torch
    from linuxnightmaresuite_b200 import moe_forward as M
    from linuxnightmaresuite_b200.ep import EPMoELayer, expert_range
    from linuxnightmaresuite_b200.stacked import StackedEP, StackedMoE
    cfg = wl.cfg
    T = wl.tokens // world if wl.split else wl.tokens          # tokens per rank
    T_gen = wl.tokens if wl.split else wl.tokens * world       # tokens of all ranks
    e0, e1 = expert_range(rank, world, cfg.n_experts)

    def shared_of(data):
        return (data.s_gate[0], data.s_up[0], data.s_down[0]) if cfg.shared_ffn else None

    if wl.layers > 1:
        datas = []

        def layers():
            # one layer's raw blocks at a time: once the model has packed them,
            # only the host parts (router, norm, tokens) are kept
            for li in range(wl.layers):
                dt = synth.make_layer_device(cfg, seed, T_gen, e0, e1, dev, layer=li)
                yield dt
                dt.w_gate = dt.w_up = dt.w_down = None
                datas.append(dt)
        if world == 1:
            model = StackedMoE.from_layers(layers(), device=dev)
        else:
            model = StackedEP.from_layers(layers(), device=dev)
        x_np = np.ascontiguousarray(datas[0].x[rank * T:(rank + 1) * T])
        first = model.layers[0]

        def status():
            return max(int(layer.device_status()) for layer in model.layers)

        def routing_stats(x):
            if world == 1:
                ids, _ = first.router.route_batch(x)
                ids = ids.cpu().numpy()
                return int(np.unique(ids).size), int(ids.size)
            return first.routing_stats(x)
        return Built(wl, lambda inp, out: model.forward(inp, out=out), x_np, T, datas, status,
                     (model.close if world > 1 else (lambda: None)), routing_stats)

    data = synth.make_layer_device(cfg, seed, T_gen, e0, e1, dev)
    x_np = np.ascontiguousarray(data.x[rank * T:(rank + 1) * T])
    if world == 1:
        layer = M.MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down,
                                       cfg.qtype, cfg.top_k, shared=shared_of(data),
                                       shared_qtype=cfg.shared_qtype,
                                       shared_hidden=cfg.shared_ffn, mode=cfg.route_mode,
                                       bias=data.bias, device=dev)

        def routing_stats(x):
            _, ids, _ = layer.forward_batch(x, return_routing=True)
            ids = ids.cpu().numpy()
            return int(np.unique(ids).size), int(ids.size)
        step = lambda inp, out: layer.forward_batch(inp, out=out)  # noqa: E731
        close = lambda: None  # noqa: E731
    else:
        shared = (data.s_gate, data.s_up, data.s_down) if cfg.shared_ffn else None
        layer = EPMoELayer(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                           cfg.top_k, cfg.route_mode, data.bias, device=dev, shared=shared,
                           shared_qtype=cfg.shared_qtype, local=True)
        routing_stats = layer.routing_stats
        step = lambda inp, out: layer.forward(inp, out=out)  # noqa: E731
        close = layer.close
    data.w_gate = data.w_up = data.w_down = None
    torch.cuda.synchronize()
    return Built(wl, step, x_np, T, [data], lambda: int(layer.device_status()), close,
                 routing_stats, host_io=True)


def measure(wl: Workload, args, steps: int, warmup: int, rank: int, world: int, local: int,
            dev, cpu: bool):
    """Builds the workload, times it and returns its JSON record (on every
    rank; rank 0's is printed)."""
    import torch
    import torch.distributed as dist
    from linuxnightmaresuite_b200 import _lib
    from oracle import moe_oracle as orc

    b = build(wl, args.seed, rank, world, dev)
    cfg, T = wl.cfg, b.T
    x = torch.from_numpy(b.x_np).to(dev)
    out = torch.empty_like(x)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    line_up = torch.zeros(1, dtype=torch.float32, device=dev)

    def pre_step():
        flush.zero_()
        if world > 1:   # every rank starts its step together
            dist.all_reduce(line_up)

    for _ in range(max(warmup, 0)):
        pre_step()
        b.step(x, out)
    torch.cuda.synchronize()
    uniq, rows = b.routing_stats(x)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(steps):
            pre_step()
            starts[i].record()
            b.step(x, out)
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
        for i in range(steps):
            pre_step()
            b.step(x, out)
        torch.cuda.synchronize()
        _lib.profile_enable(False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    ms = float(np.mean([s.elapsed_time(e) for s, e in zip(starts, ends)]))
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = T * world / (ms / 1e3)    # tokens of the whole job per second
    launches = sum(c for _, c in prof.values())

    # end to end through the public API with host buffers
    x_host = torch.from_numpy(b.x_np).pin_memory()
    out_host = torch.empty(x_host.shape, dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    def e2e_step():
        if b.host_io:   # the layer reads x and writes out in host memory itself
            b.step(x_host, out_host)
        else:
            x_dev.copy_(x_host, non_blocking=True)
            out_host.copy_(b.step(x_dev, out), non_blocking=True)

    for _ in range(2):
        pre_step()
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as e_clocks:
        for i in range(steps):
            pre_step()
            e_starts[i].record()
            e2e_step()
            e_ends[i].record()
        torch.cuda.synchronize()
    e2e_ms = float(np.mean([s.elapsed_time(e) for s, e in zip(e_starts, e_ends)]))
    e_t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e2e_ms = float(e_t.item())

    # device status of every rank, and two of this rank's tokens against the oracle
    st = torch.tensor([b.status()], dtype=torch.int64, device=dev)
    sts = [torch.zeros_like(st) for _ in range(world)]
    if world > 1:
        dist.all_gather(sts, st)
    else:
        sts = [st]
    statuses = [int(s_.item()) for s_ in sts]
    got = out_host.numpy()
    check_rows = sorted({0, T - 1})
    if wl.layers > 1 and rank != 0:
        check = None          # a token through every layer: rank 0 checks one
    else:
        rows_chk = check_rows[:1] if wl.layers > 1 else check_rows
        exp = oracle_tokens(wl, args.seed, b.x_np[rows_chk], dev, b.datas)
        mx, rel = orc.compare(got[rows_chk], exp)
        # layer tolerance; through a stack the layers' errors add (the residual
        # stream reaches ~1e4, where the reference's own f32 rounding is ~2e-2)
        bound = 1e-2 * wl.layers
        check = {"tokens": [rank * T + r for r in rows_chk], "max_abs": mx, "rel_l2": rel,
                 "max_abs_bound": bound, "ok": bool(mx <= bound and rel <= 2e-3)}
    chk_t = torch.tensor([0 if (check is None or check["ok"]) else 1], dtype=torch.int64,
                         device=dev)
    if world > 1:
        dist.all_reduce(chk_t, op=dist.ReduceOp.MAX)
    checks_ok = int(chk_t.item()) == 0

    hbm_peak, tc_peak, peak_kind = peaks()
    bb = synth.block_bytes(cfg.qtype)
    d, F = cfg.d_model, cfg.ffn
    mat = F * d // 32 * bb
    gu_ms, gu_n = prof["gateup"]
    dn_ms, dn_n = prof["down"]
    kernels = {k: {"ms_total": v[0], "launches": v[1], "ms_per_launch": v[0] / v[1]}
               for k, v in prof.items() if v[1]}
    gu_launch_ms = gu_ms / gu_n if gu_n else None
    dn_launch_ms = dn_ms / dn_n if dn_n else None
    traffic_gu = ncu_traffic(wl.name, "gateup") if world == 1 else None
    tensor_bound = rows / max(1, uniq) >= 64      # the tcgen05 GEMM path
    if tensor_bound:
        # gate/up GEMM: 2 * rows * d * 2F algorithmic flops (the three
        # split-operand MMAs that keep f32 accuracy are implementation work)
        gu_work = 2.0 * rows * d * 2 * F
        dn_work = 2.0 * rows * F * d
        achieved = gu_work / (gu_launch_ms / 1e3) / 1e12 if gu_launch_ms else None
        roofline = {
            "kernel": "tc_gateup_kernel (persistent tcgen05 grouped GEMM + SiLU*up)",
            "bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
            "frac": (achieved / tc_peak) if achieved else None, "traffic": traffic_gu,
            "peak_kind": f"{peak_kind} bf16_tflops (dense)",
            "algorithmic_flops_per_launch": gu_work, "launch_ms": gu_launch_ms,
            "executed_tensor_flops_per_launch": 3 * gu_work,
            "executed_frac": (3 * achieved / tc_peak) if achieved else None,
            "layer": {"algorithmic_flops": (gu_work + dn_work) * wl.layers, "ms": ms,
                      "achieved_tflops": (gu_work + dn_work) * wl.layers / (ms / 1e3) / 1e12},
        }
        if dn_n:
            roofline["down"] = {"algorithmic_flops_per_launch": dn_work, "launch_ms": dn_launch_ms,
                                "achieved_tflops": dn_work / (dn_launch_ms / 1e3) / 1e12}
    else:
        # gate/up GEMV: both matrices of every routed expert, the activation
        # rows it reads and the hidden rows it writes
        gu_bytes = uniq * 2 * mat + rows * d * 4 + rows * F * 4
        dn_bytes = uniq * mat + rows * F * 4 + rows * d * 4
        layer_bytes = uniq * 3 * mat + d * cfg.n_experts * 4 + T * d * 8  # this rank's share
        if cfg.shared_ffn:
            layer_bytes += 3 * cfg.shared_ffn * d // 32 * synth.block_bytes(cfg.shared_qtype)
        layer_bytes *= wl.layers
        achieved = gu_bytes / (gu_launch_ms / 1e3) / 1e9 if gu_launch_ms else None
        roofline = {
            "kernel": "gateup (grouped gate/up GEMV + SiLU*up)",
            "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": (achieved / hbm_peak) if achieved else None, "traffic": traffic_gu,
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
    if world > 1:
        # rows of this rank's tokens that cross NVLink, out and back, per layer
        off = rows * (world - 1) / world
        roofline["exchange"] = {
            "bytes_per_rank_per_layer": off * d * 4 * 2,
            "nvlink_floor_ms": off * d * 4 * 2 / 770e9 * 1e3,
            "note": "rows sent to other ranks' experts and their results returned, f32; "
                    "floor at the measured 770 GB/s per direction"}

    rec = {
        "workload": workload_desc(wl), "value": value, "unit": UNIT, "ms_per_step": ms,
        "scaling": "strong" if wl.split else "weak", "tokens_per_rank": T,
        "layers": wl.layers, "unique_experts_rank": uniq, "routed_rows_rank": rows,
        "parallelism": f"ep{world}" if world > 1 else "single",
        "roofline": roofline, "kernels": kernels,
        "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(x_host.numel() * 4),
                "d2h_bytes_per_step": int(out_host.numel() * 4)},
        "gpu_launches": launches, "clocks": clocks.summary(), "e2e_clocks": e_clocks.summary(),
        "device_status": statuses, "oracle_check": check, "oracle_checks_all_ranks_ok": checks_ok,
    }
    b.close()
    del b, x, out, flush, x_dev
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    if cpu and rank == 0 and world == 1:
        rec["cpu_baseline"] = cpu_baseline(wl, args.seed)
    return rec


def run_b200(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    wl = WORKLOADS[args.workload]
    if wl.split and wl.tokens % world:
        raise SystemExit(f"{wl.tokens} tokens do not split over {world} ranks")
    if wl.single_gpu and world > 1:
        raise SystemExit(f"{wl.name} is a single-GPU workload")
    head = measure(wl, args, args.steps, args.warmup, rank, world, local, dev,
                   cpu=not args.no_cpu_baseline)
    extra = {}
    if not args.no_workloads and args.workload == "decode_t64":
        for name in EXTRA:
            w2 = WORKLOADS[name]
            if w2.single_gpu and world > 1:
                extra[name] = {"workload": workload_desc(w2), "skipped": "single-GPU workload"}
                continue
            extra[name] = measure(w2, args, min(args.steps, args.extra_steps), 3, rank, world,
                                  local, dev, cpu=not args.no_cpu_baseline)

    bad = [k for k, r in [("headline", head)] + list(extra.items())
           if "device_status" in r and (any(r["device_status"]) or
                                         not r["oracle_checks_all_ranks_ok"])]
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": head["workload"], "tokens_per_rank": head["tokens_per_rank"],
                       "layers": head["layers"], "unique_experts": head["unique_experts_rank"],
                       "routed_rows": head["routed_rows_rank"],
                       "parallelism": head["parallelism"],
                       "experts_per_rank": wl.cfg.n_experts // world,
                       "l2": f"flushed by a {FLUSH_BYTES >> 20} MiB write before every step "
                             "(outside the step events)",
                       "weights": "GGUF blocks drawn on the GPU by a seeded generator, "
                                  "per expert"},
            "roofline": head["roofline"], "kernels": head["kernels"],
            "kernels_timing": "event pair per launch, in a second pass of the same steps",
            "cpu_baseline": head.get("cpu_baseline"), "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "device_status": head["device_status"], "oracle_check": head["oracle_check"],
            "workloads": extra,
        }
        print(json.dumps(line), flush=True)
    if bad:
        sys.stderr.write(f"device status or oracle check failed in: {bad}\n")
        sys.exit(1)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
