"""Benchmark of the fused MLP block (and the other fused workloads) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One step = one pass of the hot path over one batch: for the default workload,
the fused MLP block y = X + GELU(RMSNorm(X) @ W1 + b1) @ W2 at 8192 tokens x
d=4096 x hidden=16384, bf16 I/O, fp32 accumulation, tanh GELU, eps 1e-5. Under
torchrun the 8192 token rows are split into N contiguous blocks, one per rank,
with the weights replicated and no collective (strong scaling: the job's work
is fixed, `value` is the whole job's TFLOP/s); `--scaling weak` gives every
rank its own 8192 rows instead. `--shard-of N` times, on one GPU, the share
one rank has in an N-way split. Timing: W untimed warm-up steps,
then exactly K steps between barrier + synchronize pairs, CUDA events on the
launching stream, max over ranks; the K timed steps are recorded in a CUDA
graph and replayed (`--eager`: the public call per step). `e2e` always runs the
public call with host buffers. Inputs (W1 + W2 + X = 320 MiB) exceed the
126 MB L2, so no flush is needed between steps.

``--impl reference`` times the reference's CPU algorithm instead (the oracle's
restatement of the reference golden, numpy/OpenBLAS on all host cores, exact-erf
GELU through libm per element as the reference does), on a bounded row sample
per step; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "tt-flow_b200")]

import numpy as np  # noqa: E402

METRIC = "fused RMSNorm+MatMul / MLP TFLOP/s & % bf16 tensor peak at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes moved by the dominant kernel per launch (dram__bytes_read.sum +
# dram__bytes_write.sum, averaged over the kernel's launches in one step), from the
# ncu captures summarised in profiles/k_gemm_mlp_8192x4096x16384.md,
# profiles/k_gemm_pair_qkv_8192x4096x6144.md and
# profiles/k_stream_decode_mlp_32x8192x28672.md.
TRAFFIC_BYTES_PER_LAUNCH: dict[str, float | None] = {
    "mlp_8192x4096x16384": (433.472e6 + 252.322e6 + 1319.072e6 + 61.671e6) / 2,
    "qkv_8192x4096x6144": 209.118e6 + 86.456e6,
    "decode_mlp_32x8192x28672": (524.275e6 + 4.995e6 + 472.344e6 + 3.566e6) / 2,
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# ------------------------------------------------------------------ clock sampler


class NvmlClockSampler:
    """Reads the SM clock, power and active clock-event reasons through NVML every
    `period_s` from a background thread, so that a timed region of a few tens of
    milliseconds still gets many samples (nvidia-smi's loop samples every 100 ms at
    best). Read-only: no GPU setting is touched."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_id: str, period_s: float = 0.005):
        import threading

        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        try:
            self.h = pynvml.nvmlDeviceGetHandleByUUID(gpu_id)
        except pynvml.NVMLError:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(int(gpu_id) if gpu_id.isdigit() else 0)
        self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        self._reasons = get
        self.rows: list[tuple[float, float, float, int]] = []
        self.period = period_s
        self.halt = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv, h = self.nv, self.h
        while not self.halt.is_set():
            try:
                self.rows.append((time.time(), float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                  nv.nvmlDeviceGetPowerUsage(h) / 1000.0, int(self._reasons(h))))
            except nv.NVMLError:
                pass
            self.halt.wait(self.period)

    def stop(self, t0: float, t1: float) -> dict | None:
        self.halt.set()
        self.thread.join(timeout=5)
        try:
            self.nv.nvmlShutdown()
        except self.nv.NVMLError:
            pass
        inside = [r for r in self.rows if t0 <= r[0] <= t1]
        if not inside:
            return None
        reasons = sorted({n for r in inside for n, bit in self.REASONS if r[3] & bit})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": self.sm_max,
                "power_w_max": max(r[2] for r in inside), "reasons": reasons, "samples": len(inside),
                "window": "timed", "source": f"NVML every {self.period * 1e3:.0f} ms"}


def make_clock_sampler(gpu_id: str | None):
    if gpu_id is None:
        return None
    try:
        return NvmlClockSampler(gpu_id)
    except Exception:
        return ClockSampler(gpu_id)


class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.proc = None
        self.path = None
        if gpu_id is None or shutil.which("nvidia-smi") is None:
            return
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        self.f = os.fdopen(fd, "w")
        self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      "-lms", "100", "-i", gpu_id], stdout=self.f, stderr=subprocess.DEVNULL)

    def stop(self, t0: float, t1: float) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                rows.append((ts, float(parts[2]), float(parts[3]), float(parts[4]), parts[6:10]))
            except (ValueError, IndexError):
                continue
        os.unlink(self.path)
        if not rows:
            return None
        inside = [r for r in rows if t0 - 0.15 <= r[0] <= t1 + 0.15]
        window = "timed"
        if not inside:
            inside = [r for r in rows if r[3] > 250.0] or rows
            window = "warmup+timed (timed region shorter than the 100 ms sample period)"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in rows),
                "power_w_max": max(r[3] for r in inside), "reasons": reasons, "samples": len(inside),
                "window": window}


def gpu_id_for_smi(dev: int) -> str | None:
    import torch

    try:
        u = torch.cuda.get_device_properties(dev).uuid
        s = str(u)
        return s if s.startswith("GPU-") else f"GPU-{s}"
    except Exception:
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
        if cvd:
            return cvd.split(",")[dev]
        return str(dev)


# -------------------------------------------------------------------- CPU leg


_WORKLOAD_CACHE: dict = {}


def cpu_port_tflops(name: str, rows: int, reps: int = 1) -> tuple[float, float, dict]:
    """Time the oracle's restatement of the reference golden on `rows` rows."""
    from oracle import golden as O
    from tfb200 import workloads as W

    wl = W.WORKLOADS[name]
    d = wl.dims
    if name not in _WORKLOAD_CACHE:
        _WORKLOAD_CACHE[name] = W.generate(name)
    t = _WORKLOAD_CACHE[name]
    f = W.bf16_to_f32
    rows = min(rows, d["M"])
    times = []
    if wl.kind == "fused_mlp":
        x = f(t["x"][:rows])
        args = (x, f(t["gamma"]), f(t["w1"]), f(t["b1"]), f(t["w2"]), x, wl.eps)
        fl = 2 * rows * d["K"] * d["H"] + 2 * rows * d["H"] * d["N"]
        for _ in range(reps):
            s = time.perf_counter()
            O.fused_mlp(*args, gelu_mode="erf")
            times.append(time.perf_counter() - s)
    elif wl.kind == "fused_rmsnorm_matmul":
        x = f(t["x"][:rows])
        fl = 2 * rows * d["K"] * d["N"]
        for _ in range(reps):
            s = time.perf_counter()
            O.fused_rmsnorm_matmul(x, f(t["gamma"]), f(t["w"]), wl.eps)
            times.append(time.perf_counter() - s)
    else:
        a = f(t["a"][:rows])
        fl = 2 * rows * d["K"] * d["N"]
        for _ in range(reps):
            s = time.perf_counter()
            O.matmul(a, f(t["b"]))
            times.append(time.perf_counter() - s)
    sec = statistics.median(times)
    try:
        from threadpoolctl import threadpool_info

        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        cores = os.cpu_count() or 1
    info = {"rows": rows, "seconds": sec, "cores": cores}
    return fl / sec / 1e12, sec, info


def _all_host_threads():
    """torchrun sets OMP_NUM_THREADS=1 for every rank; the CPU legs use all host cores."""
    try:
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=os.cpu_count() or 1)
    except Exception:
        return None


def run_reference(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from tfb200 import workloads as W

    _limits = _all_host_threads()  # noqa: F841 (kept alive for the run)

    name = args.workload
    rows = args.ref_rows
    for _ in range(args.warmup):
        cpu_port_tflops(name, rows)
    vals, secs = [], []
    info = {}
    for _ in range(args.steps):
        v, s, info = cpu_port_tflops(name, rows)
        vals.append(v)
        secs.append(s)
    value = float(np.median(vals))
    wl = W.WORKLOADS[name]
    d = wl.dims
    unit = "TFLOP/s"
    if wl.kind == "fused_mlp" and d["M"] <= 64:  # the decode workload is reported in workload bytes per second
        value = value * 1e12 / W.flops(name) * W.algorithmic_bytes(name) / 1e9
        unit = "GB/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": float(np.median(secs)) * 1e3,
        "higher_is_better": True, "scaling": "strong" if (unit == "GB/s" or args.scaling == "strong") else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded numpy, bf16-rounded inputs)",
        "config": {"workload": name, **d, "gelu": "erf (the reference golden's only form)", "eps": 1e-5,
                   "sample_rows_per_step": info["rows"]},
        "cpu_baseline": {"value": value, "unit": unit, "cores": info["cores"], "kind": "port",
                         "sample": f"{info['rows']} of {d['M']} rows per step, numpy/OpenBLAS fp32 matmuls, "
                                   f"libm erf per element; the sampled rows' rate extrapolated to the workload "
                                   f"(a row sample runs OpenBLAS below its full-M rate)"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# -------------------------------------------------------------------- GPU leg


def _e2e_pipelined(torch, step, x, y, steps: int, warmup: int, barrier) -> float:
    """ms per step of the public call with host input and output: copy-in, compute, copy-out on three streams,
    device tensors double-buffered, events ordering each buffer's reuse. Timed with CUDA events that span all
    three streams."""
    cur = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    xh = x.cpu().pin_memory()
    yh = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x) for _ in range(2)]
    yd = [torch.empty_like(y) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e in ev_comp + ev_out:
        e.record(cur)

    def one(i):
        b = i % 2
        s_in.wait_event(ev_comp[b])          # the compute that last read xd[b] is done
        with torch.cuda.stream(s_in):
            xd[b].copy_(xh, non_blocking=True)
            ev_in[b].record(s_in)
        cur.wait_event(ev_in[b])
        cur.wait_event(ev_out[b])            # the copy-out that last read yd[b] is done
        out = step(xd[b], yd[b])
        if out is not yd[b]:                 # the fused tensor-parallel call returns its own buffer
            yd[b].copy_(out.view(yd[b].shape), non_blocking=True)
        ev_comp[b].record(cur)
        s_out.wait_event(ev_comp[b])
        with torch.cuda.stream(s_out):
            yh[b].copy_(yd[b], non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(warmup):
        one(i)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(steps):
        one(i)
    cur.wait_event(ev_out[(steps - 1) % 2])
    cur.wait_event(ev_out[steps % 2])
    e1.record(cur)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from tfb200 import _lib, ops
    from tfb200 import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    lib = _lib.lib()

    name = args.workload
    wl = W.WORKLOADS[name]
    d = wl.dims
    tp_shape = wl.kind == "fused_mlp" and d["M"] <= 64
    # Row sharding of the prefill workloads: rank r of `parts` owns rows [lo, hi) of the workload's rows.
    parts = world if args.shard_of <= 0 else args.shard_of
    strong = not tp_shape and args.scaling == "strong" and parts > 1
    if strong:
        r = rank if args.shard_of <= 0 else 0
        lo, hi = d["M"] * r // parts, d["M"] * (r + 1) // parts
        t = W.generate(name, rows=(lo, hi))
    else:
        lo, hi = 0, d["M"]
        t = W.generate(name)
    rows_here = hi - lo

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.bfloat16)

    tp = wl.kind == "fused_mlp" and d["M"] <= 64
    fused_tp = tp and args.tp_reduce == "fused" and world > 1
    if tp and world > 1:
        # Decode-shaped MLP: tensor parallel over the ranks (W1 by columns, W2 by
        # rows). "fused": the down-projection kernel reduces across GPUs over
        # NVLink peer memory and finishes the rows; "nccl": fp32 partial sum, one
        # NCCL all-reduce, then the residual add.
        from tfb200.tp import TPDecodeMLP, TPDecodeMLPFused

        x, g, w1, b1, w2 = (dev(t[k]) for k in ("x", "gamma", "w1", "b1", "w2"))
        if fused_tp:
            mlp = TPDecodeMLPFused(w1, b1, w2, g, rank, world, max_rows=d["M"], eps=wl.eps, gelu=wl.gelu)
        else:
            mlp = TPDecodeMLP(w1, b1, w2, g, rank, world, eps=wl.eps, gelu=wl.gelu)
        del w1, w2
        torch.cuda.empty_cache()
        y = torch.empty(d["M"], d["N"], dtype=torch.bfloat16, device="cuda")

        def step(xin=None, yout=None):
            xx = x if xin is None else xin
            return mlp(xx, xx) if fused_tp else mlp(xx, xx, out=y if yout is None else yout)
        in_bytes = x.numel() * 2
    elif wl.kind == "fused_mlp":
        # One GPU (the decode shape included: the C ABI picks the weight-streaming kernels for few rows).
        x, g, w1, b1, w2 = (dev(t[k]) for k in ("x", "gamma", "w1", "b1", "w2"))
        y = torch.empty(rows_here, d["N"], dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(ops.mlp_workspace_bytes(rows_here, d["K"], d["H"], d["N"]), dtype=torch.uint8,
                         device="cuda")

        def step(xin=None, yout=None):
            xx = x if xin is None else xin
            return ops.fused_mlp(xx, g, w1, b1, w2, xx, wl.eps, gelu=wl.gelu, out=y if yout is None else yout,
                                 workspace=ws)
        in_bytes = x.numel() * 2
    elif wl.kind == "fused_rmsnorm_matmul":
        x, g, w = (dev(t[k]) for k in ("x", "gamma", "w"))
        y = torch.empty(rows_here, d["N"], dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(ops.rmsnorm_matmul_workspace_bytes(rows_here, d["K"], d["N"]), dtype=torch.uint8,
                         device="cuda")

        def step(xin=None, yout=None):
            return ops.fused_rmsnorm_matmul(x if xin is None else xin, g, w, wl.eps, out=y if yout is None else yout,
                                            workspace=ws)
        in_bytes = x.numel() * 2
    else:
        x, b = dev(t["a"]), dev(t["b"])
        y = torch.empty(x.shape[0], d["N"], dtype=torch.bfloat16, device="cuda")

        def step(xin=None, yout=None):
            return ops.matmul(x if xin is None else xin, b, out=y if yout is None else yout)
        in_bytes = x.numel() * 2
    flops_step = W.flops(name)  # the whole workload (all ranks together)
    flops_here = flops_step * rows_here // d["M"] if not tp_shape else flops_step

    def barrier():
        if world > 1:
            dist.barrier()

    sampler = make_clock_sampler(gpu_id_for_smi(local)) if rank == 0 else None
    for _ in range(args.warmup):
        step()
    barrier()
    torch.cuda.synchronize()
    # The K timed steps are recorded once in a CUDA graph and replayed, as a serving loop runs fixed-shape steps:
    # the same kernels and arguments as K eager calls (the programmatic-launch chaining between consecutive steps
    # included), without the host's per-call work (argument checks, tensor maps, launches: about 54 us per call,
    # which eight ranks sharing the host's cores do not all hide behind a 200 us step). `--eager` times the
    # public call itself. The path with an NCCL all-reduce stays eager.
    graph = None
    launches_in_graph = 0
    if not args.eager and not (tp and world > 1 and not fused_tp):
        graph = torch.cuda.CUDAGraph()
        lc = lib.tfb200_launch_count()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                step()
        launches_in_graph = lib.tfb200_launch_count() - lc
        graph.replay()  # untimed: the graph's first replay uploads it
        torch.cuda.synchronize()
        barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    l0 = lib.tfb200_launch_count()
    w0 = time.time()
    e0.record()
    if graph is not None:
        graph.replay()
    else:
        for _ in range(args.steps):
            step()
    e1.record()
    torch.cuda.synchronize()
    w1t = time.time()
    barrier()
    launches = lib.tfb200_launch_count() - l0 + launches_in_graph
    ms = e0.elapsed_time(e1)
    ms_by_rank = [ms]
    if world > 1:
        allms = [torch.zeros(1, dtype=torch.float64, device="cuda") for _ in range(world)]
        dist.all_gather(allms, torch.tensor([ms], dtype=torch.float64, device="cuda"))
        ms_by_rank = [float(t.item()) for t in allms]
        ms = max(ms_by_rank)
    clocks = sampler.stop(w0, w1t) if sampler else None
    ms_step = ms / args.steps
    if tp:
        # strong scaling: all ranks together stream the workload's bytes once per step
        bytes_step = W.algorithmic_bytes(name)
        value = bytes_step / (ms_step * 1e-3) / 1e9
    elif args.shard_of > 0:
        value = flops_here / (ms_step * 1e-3) / 1e12  # one rank's share, timed alone
    elif strong:
        value = flops_step / (ms_step * 1e-3) / 1e12  # the whole job's rows over the slowest rank's time
    else:
        value = flops_step * world / (ms_step * 1e-3) / 1e12

    # End to end through the public API with host buffers: every step copies its X in from pinned host memory
    # and its Y out to pinned host memory. As a serving loop does, the copies run on their own streams with
    # double-buffered device tensors, so step i's compute overlaps the copy-in of step i+1 and the copy-out of
    # step i-1; the timed region spans all three streams.
    e2e_ms = _e2e_pipelined(torch, step, x, y, args.steps, max(3, args.warmup), barrier)
    ems = e2e_ms * args.steps
    if world > 1:
        tt = torch.tensor([ems], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ems = float(tt.item())
    e2e_value = (W.algorithmic_bytes(name) / (ems / args.steps * 1e-3) / 1e9 if tp
                 else flops_here / (ems / args.steps * 1e-3) / 1e12 if args.shard_of > 0
                 else flops_step / (ems / args.steps * 1e-3) / 1e12 if strong
                 else flops_step * world / (ems / args.steps * 1e-3) / 1e12)

    pk, pk_src = peaks()
    sustained = ms > 1000.0
    launches_per_step = max(1, launches // max(1, args.steps))
    if tp:
        unit = "GB/s"
        per_gpu = W.algorithmic_bytes(name) / world / (ms_step * 1e-3) / 1e9
        peak = pk["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                "traffic": TRAFFIC_BYTES_PER_LAUNCH.get(name), "kernel": "k_stream (weight-streaming tcgen05 GEMM)",
                "launches_per_step": launches_per_step,
                "peak_source": f"{pk_src} HBM copy bandwidth (MEASURED_PEAKS.json)" if pk_src == "measured"
                else "fallback"}
        scaling = "strong"
        if world == 1:
            parallelism = "1 GPU, weights whole"
        elif fused_tp:
            parallelism = (f"tensor parallel over {world} GPUs: W1 by columns, W2 by rows, the reduction fused into "
                           f"the down-projection kernel over NVLink peer memory")
        else:
            parallelism = f"tensor parallel over {world} GPUs: W1 by columns, W2 by rows, one NCCL all-reduce"
    else:
        unit = "TFLOP/s"
        peak = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
        per_gpu = flops_here / (ms_step * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu / peak,
                "traffic": TRAFFIC_BYTES_PER_LAUNCH.get(name) if rows_here == d["M"] else None,
                "kernel": "k_gemm_pair (persistent cta_group::2 tcgen05 GEMM)",
                "launches_per_step": launches_per_step,
                "peak_source": f"{pk_src} {'sustained' if sustained else 'burst'} bf16 (MEASURED_PEAKS.json)"
                if pk_src == "measured" else "fallback"}
        if args.shard_of > 0:
            scaling = "strong"
            parallelism = (f"one GPU timing rank 0's share ({rows_here} of {d['M']} rows) of a {parts}-way row split, "
                           f"weights replicated")
        elif strong:
            scaling = "strong"
            parallelism = (f"{d['M']} rows split over {world} GPUs ({rows_here} per GPU), weights replicated, "
                           f"no collective")
        else:
            scaling = "weak"
            parallelism = f"{d['M']} rows per GPU on {world} GPU(s), weights replicated, no collective"
    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded numpy normal/uniform, bf16)",
        "config": {"workload": name, **d, "gelu": wl.gelu, "eps": wl.eps,
                   "rows_per_gpu": rows_here,
                   "global_rows": d["M"] * world if (not tp and not strong and args.shard_of <= 0) else d["M"],
                   "parallelism": parallelism,
                   "l2": "weights and activations larger than L2 (no flush)" if rows_here * d["K"] * 2 > 126e6
                   else "weights larger than L2 (no flush); activations of the share fit"},
        "roofline": roof,
        "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": in_bytes * (world if strong else 1),
                "d2h_bytes_per_step": y.numel() * 2 * (world if strong else 1),
                "note": "public call with host buffers: X copied in from pinned host memory and Y copied back every "
                        "step, on copy streams overlapping the neighbouring steps' compute (double-buffered); "
                        "weights resident"},
        "gpu_launches": launches,
        "launch": f"CUDA graph of the {args.steps} timed steps, replayed once" if graph is not None
        else "eager public call per step",
        "ms_per_step_by_rank": [round(v / args.steps, 5) for v in ms_by_rank],
        "clocks": clocks,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        _limits = _all_host_threads()  # noqa: F841
        rows = args.cpu_rows
        if rows <= 0:  # size the sample for about 10 s of CPU work
            _, probe, _ = cpu_port_tflops(name, 64)
            rows = int(min(d["M"], max(64, 64 * 10.0 / max(probe, 1e-3))))
        v, sec, info = cpu_port_tflops(name, rows)
        if tp:  # express the CPU rate in the same unit: workload bytes per second
            v = v * 1e12 / flops_step * W.algorithmic_bytes(name) / 1e9
        line["cpu_baseline"] = {"value": v, "unit": unit, "cores": info["cores"], "kind": "port",
                                "sample": f"{info['rows']} of {d['M']} rows in {sec:.1f} s: the reference golden "
                                          f"restated (numpy/OpenBLAS fp32, libm erf per element); the sampled "
                                          f"rows' rate extrapolated to the workload"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if fused_tp:
        barrier()
        mlp.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="mlp_8192x4096x16384")
    ap.add_argument("--cpu-rows", type=int, default=0, help="rows of the CPU baseline sample (0: about 10 s)")
    ap.add_argument("--ref-rows", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp-reduce", choices=["fused", "nccl"], default="fused",
                    help="decode workloads: cross-GPU reduction inside the kernel, or an NCCL all-reduce")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="prefill workloads under torchrun: split the workload's rows over the ranks (strong) or "
                         "give every rank all of them (weak)")
    ap.add_argument("--eager", action="store_true",
                    help="time the public call per step instead of a CUDA-graph replay of one step")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="time rank 0's share of an N-way row split on this one GPU (prefill workloads)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())
