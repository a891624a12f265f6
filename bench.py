#!/usr/bin/env python
"""Benchmark of the fused softplus MLP on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mlpk|reference]

Headline workload (top of its batch sweep): the 3-layer
D=H=OUT=128 softplus MLP forward on M = 4,194,304 rows per GPU, fp16 operands
and fp32 accumulation, seeded synthetic inputs (x ~ N(0,1), W ~ U(+-1/sqrt(in))).
A step is one forward over the whole batch.  With N > 1 (torchrun, one process
per GPU) every rank runs its own M rows: the path shards by rows with no
collective, so the scaling is weak and ``value`` = N*M*K / max-over-ranks time.

Timing: W untimed warm-up steps, then K steps between CUDA events on the
launching stream, bracketed by a barrier and a device synchronize; inputs
(1 GiB x, 1 GiB out) are larger than L2, so no flush is needed.  SM clocks and
throttle reasons are sampled through NVML during the timed region.  ``e2e``
is the same forward from pinned host rows to pinned host results through
``fused_mlp_fwd_host`` (chunked; the copies in and out overlap each other and
the forward), all bytes crossing the host link every step.

The same JSON line carries the training steps (forward + backward through
the C ABI on preallocated buffers, replayed as one CUDA graph per step, dW
summed over the ranks by the library's NVLink peer-memory kernel when N > 1):
``fwd_bwd`` (3L128 with weight norm and fp32 activation
storage, 262,144 rows per GPU), ``fwd_bwd_h16`` (the same saving fp16
activations, with its gradients' difference from the fp32-storage step),
``fwd_bwd_small`` (config 3's small-batch regime: 16,384 rows per GPU),
``fwd_bwd_5l`` (config 4: 5-layer with weight norm, 1,048,576 rows in total,
strong scaling), ``fwd_bwd_5l_weak`` (N > 1 only: the same with 1,048,576 rows
per GPU) and ``fwd_bwd_w256`` (config 5: D = H = OUT = 256, 1,048,576 rows in
total).  Each has its own roofline (tensor-bound) and e2e figure.

``--impl reference`` times the reference's own PyTorch path (kernel.py:163-171,
restated in oracle/cpu_baseline.py because the reference tree does not exist
on the GPU box) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_METRIC = "fused MLP fwd rows/s & fwd+bwd rows/s vs roofline at M=1M-4M, 1-8 B200"
DIMS = (128, 128, 128, 128)
ROWS = 4 * 1024 * 1024
BYTES_PER_ROW = 2 * (DIMS[0] + DIMS[-1])                     # x in + out out, fp16
FLOP_PER_ROW = 2 * sum(a * b for a, b in zip(DIMS[:-1], DIMS[1:]))
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
FWD_KERNEL = "mlp_fwd_kernel"
TRAIN_ROWS = 262144                                           # BASELINE config 3 (split-K regime)
TRAIN_SMALL_ROWS = 16384                                      # BASELINE config 3 (small-batch regime)
TRAIN5_ROWS = 1024 * 1024                                     # BASELINE config 4 (global)
TRAIN256_ROWS = 1024 * 1024                                   # BASELINE config 5 (global)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="mlpk", choices=["mlpk", "reference"])
    ap.add_argument("--rows", type=int, default=ROWS, help="rows per GPU")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--train-rows", type=int, default=TRAIN_ROWS, help="training rows per GPU")
    ap.add_argument("--train5-rows", type=int, default=TRAIN5_ROWS,
                    help="global rows of the 5-layer training step (split over the GPUs)")
    ap.add_argument("--train256-rows", type=int, default=TRAIN256_ROWS,
                    help="global rows of the wide (256) training step (split over the GPUs)")
    ap.add_argument("--train-steps", type=int, default=50)
    ap.add_argument("--no-train", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time training steps as eager launches")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-2 batch sweep")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 0)) or None,
                "source": "measured"}
    except Exception:
        return dict(FALLBACK_PEAKS)


def load_traffic(name: str):
    """dram bytes per launch recorded from an ncu capture in profiles/<name>.md
    (a line `dram_bytes_per_launch: <int>`), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------- clocks
REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


def _clock_sample_loop(bus: str, index: int, period: float, conn, stop) -> None:
    """Body of ClockSampler's child process: NVML samples of the SM clock and
    the clock-event reasons every `period` seconds until `stop` is set, then
    the list goes back through `conn`.  A separate process, not a thread: the
    main process holds the interpreter lock while it waits in a CUDA
    synchronize, which starved a sampler thread of all samples in a ~10 ms
    timed region."""
    try:
        import pynvml as nv

        nv.nvmlInit()
        try:
            h = nv.nvmlDeviceGetHandleByPciBusId_v2(bus) if bus else nv.nvmlDeviceGetHandleByIndex(index)
        except Exception:
            h = nv.nvmlDeviceGetHandleByIndex(index)
        reasons = None
        for fn in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
            if hasattr(nv, fn):
                reasons = getattr(nv, fn)
                break
        max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
    except Exception as e:  # no NVML: the parent reports it
        conn.send(("error", repr(e)[:200]))
        return
    conn.send(("ready", max_mhz))
    samples = []
    while not stop.is_set():
        try:
            samples.append((time.monotonic(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                            reasons(h) if reasons else 0))
        except Exception:
            pass
        time.sleep(period)
    conn.send(("samples", samples))


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a child
    process (spawned, so it shares no CUDA state and no interpreter lock with
    the timing loop).

    Samples are timestamped on the system's monotonic clock; ``mark_start`` /
    ``mark_stop`` bracket the timed region and ``summary`` reports the samples
    inside it (plus the ones taken under load in the warm-up just before it
    when the timed region is shorter than a few sample periods)."""

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.samples = []
        self.period = period_s
        self.index = device_index
        self.ok = False
        self.note = None
        self.max_mhz = None
        self.t_start = self.t_stop = None
        self.bus = ""
        try:
            import pynvml  # noqa: F401  (present: the child can sample)
            import torch

            props = torch.cuda.get_device_properties(device_index)
            try:
                self.bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            except Exception:
                self.bus = ""
            self.ok = True
        except Exception as e:
            self.note = f"NVML unavailable: {type(e).__name__}"

    def mark_start(self):
        self.t_start = time.monotonic()

    def mark_stop(self):
        self.t_stop = time.monotonic()

    def __enter__(self):
        if not self.ok:
            return self
        import multiprocessing as mp

        ctx = mp.get_context("spawn")
        self._conn, child = ctx.Pipe()
        self._stop = ctx.Event()
        self.proc = ctx.Process(target=_clock_sample_loop,
                                args=(self.bus, self.index, self.period, child, self._stop), daemon=True)
        self.proc.start()
        deadline = time.monotonic() + 60
        while not self._conn.poll(0.05) and self.proc.is_alive() and time.monotonic() < deadline:
            pass
        if self._conn.poll(0):
            kind, val = self._conn.recv()
            if kind == "ready":
                self.max_mhz = val
                time.sleep(5 * self.period)  # first samples before the caller's work starts
                return self
            self.note = f"sampler: {val}"
        else:
            self.note = "sampler process did not start"
        self.ok = False
        self._stop.set()
        self.proc.join(5)
        if self.proc.is_alive():
            self.proc.terminate()
        return self

    def __exit__(self, *a):
        if not self.ok:
            return
        time.sleep(2 * self.period)
        self._stop.set()
        if self._conn.poll(30):
            kind, val = self._conn.recv()
            if kind == "samples":
                self.samples = val
        self.proc.join(10)
        if self.proc.is_alive():
            self.proc.terminate()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.note or "no samples"}
        t0 = self.t_start if self.t_start is not None else -1e30
        t1 = self.t_stop if self.t_stop is not None else 1e30
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        used, window = inside, "timed region"
        if len(inside) < 5:
            # a short timed region: add the samples of the warm-up steps just
            # before it (the same kernels under load) and the first after it
            near = [s for s in self.samples if t0 - 0.05 <= s[0] <= t1 + 0.002]
            used, window = near, "timed region and the 50 ms of warm-up before it"
        if not used:
            used, window = self.samples, "whole sampler run"
        mhz = [s[1] for s in used]
        bits = 0
        for s in used:
            bits |= int(s[2])
        reasons = [n for b, n in REASON_BITS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_min_mhz": min(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz), "samples_in_timed_region": len(inside),
                "window": window, "period_ms": 1e3 * self.period}


# ---------------------------------------------------------------------- CPU legs
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU arm runs on rank 0 only
    import torch

    from oracle.cpu_baseline import model_forward, set_all_threads
    from mlp_megakernel_b200.synthetic import make_weights, make_x

    cores = set_all_threads()
    sample = 65536
    x = make_x(sample, DIMS[0], "normal", 0).float()
    ws = [w.float() for w in make_weights(DIMS)]
    with torch.no_grad():
        for _ in range(max(args.warmup, 1)):
            model_forward(x, ws)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model_forward(x, ws)
        dt = time.perf_counter() - t0
    rps = sample * args.steps / dt
    desc = (f"{sample} rows of the 3L128 forward per step (bounded sample of M={args.rows}), "
            f"fp32 torch CPU, {cores} threads")
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": rps, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "3L128 fwd (kernel.py:163-171 Model on host CPU)",
                   "dims": list(DIMS), "rows_per_step": sample, "device": "cpu"},
        "cpu_baseline": {"value": rps, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": rps, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_model_name() -> str:
    """The host CPU model (the `model name` line of /proc/cpuinfo)."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_forward_full(rows: int, reps: int = 3):
    """The reference's PyTorch forward (kernel.py:163-171) in fp32 on all host
    threads at the bench's full row count: median of `reps` timed passes
    (after one warm-up pass)."""
    import torch

    from oracle.cpu_baseline import model_forward, set_all_threads
    from mlp_megakernel_b200.synthetic import make_weights, make_x

    cores = set_all_threads()
    x = make_x(rows, DIMS[0], "normal", 0).float()
    ws = [w.float() for w in make_weights(DIMS)]
    times = []
    with torch.no_grad():
        model_forward(x, ws)
        for _ in range(reps):
            t0 = time.perf_counter()
            model_forward(x, ws)
            times.append(time.perf_counter() - t0)
    return rows / statistics.median(times), cores, times


def cpu_train_full(rows: int, reps: int = 3):
    """The reference's PyTorch training step for BASELINE config 3 in fp32 on
    all host threads: weight norm W = g v / ||v|| per output column, the
    forward of kernel.py:163-171 and torch.autograd back to (dv, dg) and dx.
    Median of `reps` timed steps after one warm-up step."""
    from oracle.cpu_baseline import set_all_threads, train_step_wn
    from mlp_megakernel_b200.synthetic import make_grad, make_weights, make_x

    cores = set_all_threads()
    x = make_x(rows, DIMS[0], "normal", 0).float()
    g = make_grad(rows, DIMS[-1]).float()
    ws = [w.float() for w in make_weights(DIMS)]
    vs = [w.clone() for w in ws]
    gs = [w.norm(dim=0) for w in ws]
    train_step_wn(x, vs, gs, g)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        train_step_wn(x, vs, gs, g)
        times.append(time.perf_counter() - t0)
    return rows / statistics.median(times), cores, times


# ---------------------------------------------------------------------- batch sweep
SWEEP_MIN_LOG2, SWEEP_MAX_LOG2 = 6, 22  # M = 64 .. 4,194,304


def _load_reference_kernel():
    """The reference's own Triton forward (kernel.py, unmodified) from
    baseline/_ref, or None when it is not present (the reference tree has no
    package metadata, so it is placed there as files)."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "kernel.py")):
        return None, "baseline/_ref/kernel.py not present"
    try:
        import importlib.util

        spec = importlib.util.spec_from_file_location("mlpk_bench_ref_kernel", os.path.join(ref_dir, "kernel.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # e.g. triton missing on the box
        return None, f"import failed: {type(e).__name__}: {e}"[:200]


def _graph_us_per_call(fn, calls: int, reps: int = 5) -> float:
    """Device time per call: `calls` calls captured in one CUDA graph,
    replayed `reps` times between CUDA events (the graph-replay method of
    profile.py:230-260)."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = 1e3 * e0.elapsed_time(e1) / (reps * calls)
    del g
    return us


def _eager_us_per_call(fn, calls: int) -> float:
    """Host wall time per call of back-to-back eager calls (synchronised
    before and after): the per-call latency a Python caller sees, the
    reference's "non-graph" figure (README.md:240-249)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(calls):
        fn()
    torch.cuda.synchronize()
    return 1e6 * (time.perf_counter() - t0) / calls


def run_sweep(x_full, ws, peaks):
    """the 3L128 forward at M = 64 .. 4,194,304 (powers of
    2), per call: device time replayed from a CUDA graph, host per-call time
    of eager calls through ``fused_mlp_fwd`` (the drop-in API), rows/s and the
    fraction of the HBM roofline; the reference's Triton kernel beside it when
    baseline/_ref holds it."""
    import torch

    from mlp_megakernel_b200 import fused_mlp_fwd

    ref, why = _load_reference_kernel()
    out_full = torch.empty((x_full.shape[0], DIMS[-1]), dtype=torch.float16, device=x_full.device)
    rows_out = []
    for lg in range(SWEEP_MIN_LOG2, SWEEP_MAX_LOG2 + 1):
        M = 1 << lg
        if M > x_full.shape[0]:
            break
        x, out = x_full[:M], out_full[:M]
        ours = lambda: fused_mlp_fwd(x, *ws, out=out)  # noqa: E731
        calls = max(1, min(64, (1 << 20) // M))
        n_eager = max(20, min(500, (1 << 24) // M))
        g_us = _graph_us_per_call(ours, calls)
        e_us = _eager_us_per_call(ours, n_eager)
        gbs = BYTES_PER_ROW * M / (g_us * 1e-6) / 1e9
        row = {"M": M, "graph_us": g_us, "eager_us": e_us, "rows_per_s": M / (g_us * 1e-6),
               "eager_rows_per_s": M / (e_us * 1e-6), "hbm_frac": gbs / peaks["hbm_gbs"],
               "l2_resident": BYTES_PER_ROW * M < 100e6}
        if ref is not None:
            try:
                rfn = lambda: ref._fused_mlp_fwd(x, *ws)  # noqa: E731
                rg = _graph_us_per_call(rfn, calls)
                re_ = _eager_us_per_call(rfn, n_eager)
                row.update({"triton_ref_graph_us": rg, "triton_ref_eager_us": re_,
                            "speedup_graph": rg / g_us, "speedup_eager": re_ / e_us})
            except Exception as e:
                why = f"reference Triton kernel failed at M={M}: {type(e).__name__}: {e}"[:200]
                ref = None
        rows_out.append(row)
    res = {
        "workload": "BASELINE config 2: 3L128 forward, M = 64 .. 4,194,304 (powers of 2), x ~ N(0,1) "
                    "seed 0, W ~ U(+-1/sqrt(in)) seed 1, one GPU; rows with l2_resident = true have "
                    "inputs and outputs that fit in L2 (no flush: the small-batch serving regime)",
        "graph_us": "device time per call, calls replayed from a CUDA graph (profile.py:230-260 method)",
        "eager_us": "host time per call of back-to-back fused_mlp_fwd calls (Python + ctypes + launch)",
        "rows": rows_out,
    }
    if ref is not None:
        res["triton_reference"] = ("the reference's unmodified kernel.py _fused_mlp_fwd (kernel.py:130-156), "
                                   "Triton JIT for this GPU, same inputs, timed the same two ways")
    else:
        res["triton_reference_unavailable"] = why
    return res


# ---------------------------------------------------------------------- GPU arm
def run_mlpk(args):
    import torch

    from mlp_megakernel_b200 import _lib, fused_mlp_fwd, fused_mlp_fwd_host
    from mlp_megakernel_b200.synthetic import make_weights, make_x

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    M = args.rows
    x = make_x(M, DIMS[0], "normal", rank, device="cuda")
    ws = make_weights(DIMS, device="cuda")
    _lib.device_status(clear=True)

    out = torch.empty((M, DIMS[-1]), dtype=torch.float16, device="cuda")
    step = lambda: fused_mlp_fwd(x, *ws, out=out)  # noqa: E731
    stream = torch.cuda.current_stream()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_stop()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = _lib.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} after the timed region")

    # e2e through the public API for host-resident rows: pinned host x ->
    # fused_mlp_fwd_host (chunks copied in, run and copied out, the copies of
    # neighbouring chunks overlapping) -> pinned host out
    xh = x.cpu().pin_memory()
    oh = torch.empty((M, DIMS[-1]), dtype=torch.float16, pin_memory=True)

    def e2e_step():
        fused_mlp_fwd_host(xh, *ws, out=oh)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    sweep = None
    if world == 1 and not args.no_sweep:
        sweep = run_sweep(x, ws, load_peaks())

    train = train16 = train_small = train5 = train256 = train5w = None
    if not args.no_train:
        from mlp_megakernel_b200.dp import shard_rows

        train = run_training(args, world, rank, dist, barrier, "3L128", args.train_rows)
        train16 = run_training(args, world, rank, dist, barrier, "3L128_h16", args.train_rows)
        # the fp16-storage step against the fp32-storage step (same inputs):
        # relative L2 difference of the gradients the step returns
        g32, g16 = train.pop("_grads"), train16.pop("_grads")
        train16["grad_diff_vs_fp32_storage"] = {
            name: float((a16.double() - a32.double()).norm() / a32.double().norm().clamp_min(1e-30))
            for name, a32, a16 in zip(("dx", "dv", "dg"), g32, g16)}
        # BASELINE config 3's small-batch regime (M = 16,384 per GPU)
        train_small = run_training(args, world, rank, dist, barrier, "3L128", TRAIN_SMALL_ROWS)
        train_small.pop("_grads")
        a, b = shard_rows(args.train5_rows, rank, world)
        train5 = run_training(args, world, rank, dist, barrier, "5L", b - a)
        a, b = shard_rows(args.train256_rows, rank, world)
        train256 = run_training(args, world, rank, dist, barrier, "W256", b - a)
        train5w = (run_training(args, world, rank, dist, barrier, "5L_weak", args.train5_rows)
                   if world > 1 else None)  # at N = 1 it is the fwd_bwd_5l run
        for t in (train5, train256, train5w):
            if t is not None:
                t.pop("_grads")

    clocks = clk.summary()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = load_peaks()
    per_launch_s = ms / 1e3 / args.steps
    achieved_gbs = BYTES_PER_ROW * M / per_launch_s / 1e9
    traffic = load_traffic("fwd_3L128_M4M")
    value = world * M * args.steps / (ms / 1e3)
    line = {
        "metric": BASELINE_METRIC,
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 operands, f32 accumulate",
        "data": "synthetic (seeded x~N(0,1), W~U(+-1/sqrt(in)))",
        "config": {
            "workload": "3L128 fwd: 3-layer softplus MLP D=H=OUT=128, M=4,194,304 rows per GPU "
                        "(BASELINE config 2, top of the batch sweep)",
            "dims": list(DIMS), "rows_per_gpu": M, "global_rows": world * M,
            "parallelism": f"dp{world} (row-sharded, no collective)",
            "l2": "inputs larger than L2 (x 1 GiB + out 1 GiB per GPU); no flush needed",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved_gbs,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved_gbs / peaks["hbm_gbs"],
            "traffic": traffic,
            "peak_source": peaks["source"],
            "algorithmic_bytes_per_row": BYTES_PER_ROW,
            "kernel": FWD_KERNEL,
            "tensor_tflops": FLOP_PER_ROW * M / per_launch_s / 1e12,
            "tensor_frac_of_bf16_peak": FLOP_PER_ROW * M / per_launch_s / 1e12 / peaks["bf16_tflops"],
        },
        "e2e": {
            "value": world * M * args.e2e_steps / (e2e_ms / 1e3),
            "unit": "rows/s",
            "h2d_bytes_per_step": M * DIMS[0] * 2,
            "d2h_bytes_per_step": M * DIMS[-1] * 2,
            "steps": args.e2e_steps,
            "api": "mlp_megakernel_b200.fused_mlp_fwd_host: pinned host rows streamed through the "
                   "GPU in 131,072-row chunks (copy in, forward, copy out of neighbouring chunks "
                   "overlap); every byte of x crosses to the device and every byte of out back, "
                   "each step",
        },
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if train is not None:
        line["fwd_bwd"] = train
    if train16 is not None:
        line["fwd_bwd_h16"] = train16
    if train_small is not None:
        line["fwd_bwd_small"] = train_small
    if train5 is not None:
        line["fwd_bwd_5l"] = train5
    if train256 is not None:
        line["fwd_bwd_w256"] = train256
    if train5w is not None:
        line["fwd_bwd_5l_weak"] = train5w
    if sweep is not None:
        line["sweep"] = sweep
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_model_name()
        rps, cores, times = cpu_forward_full(M)
        line["cpu_baseline"] = {
            "value": rps, "unit": "rows/s", "cores": cores, "kind": "port", "cpu_model": cpu,
            "sample": f"the full M={M} rows of the 3L128 forward, median of {len(times)} passes "
                      f"({', '.join(f'{t:.2f}' for t in times)} s), reference PyTorch formula "
                      f"(kernel.py:163-171) in fp32 on {cores} threads",
        }
        if train is not None:
            trows = args.train_rows
            trps, tcores, ttimes = cpu_train_full(trows)
            train["cpu_baseline"] = {
                "value": trps, "unit": "rows/s", "cores": tcores, "kind": "port", "cpu_model": cpu,
                "sample": f"BASELINE config 3 training step at M={trows} (weight norm, forward, "
                          f"torch.autograd backward to dx, dv, dg), median of {len(ttimes)} steps "
                          f"({', '.join(f'{t:.2f}' for t in ttimes)} s), fp32 on {tcores} threads",
            }
    print(json.dumps(line), flush=True)


TRAIN_SPECS = {
    # 3L128 with weight norm, split-K regime, rows per GPU fixed
    "3L128": {"dims": (128, 128, 128, 128), "x_dist": "normal", "x_seed": 0, "strong": False, "h32": True,
              "metric": "fused MLP fwd+bwd rows/s (3L128 with weight norm)",
              "workload": "BASELINE config 3: 3L D=H=OUT=128 training step with weight norm, "
                          "fp32 activation storage, M={M} rows per GPU"},
    # the same step saving the fp16 operand copy of h (half the saved-activation traffic)
    "3L128_h16": {"dims": (128, 128, 128, 128), "x_dist": "normal", "x_seed": 0, "strong": False,
                  "metric": "fused MLP fwd+bwd rows/s (3L128 with weight norm)",
                  "workload": "BASELINE config 3 shape with fp16 activation storage (not the config as "
                              "written): 3L D=H=OUT=128 training step with weight norm, M={M} rows per GPU"},
    # 5L 32-64-64-64-64-16 with weight norm, global M = 1,048,576
    # split over the ranks (strong scaling, dW summed over the ranks)
    "5L": {"dims": (32, 64, 64, 64, 64, 16), "x_dist": "uniform", "x_seed": 3, "strong": True,
           "metric": "fused MLP fwd+bwd rows/s (5L 32-64-64-64-64-16 with weight norm)",
           "workload": "BASELINE config 4: 5L D=32 H=64 OUT=16 training step with weight norm, "
                       "fp16 activation storage, global M={G} rows, {M} per GPU"},
    # the same 5-layer step with the rows per GPU fixed (1,048,576 each): weak scaling
    "5L_weak": {"dims": (32, 64, 64, 64, 64, 16), "x_dist": "uniform", "x_seed": 3, "strong": False,
                "metric": "fused MLP fwd+bwd rows/s (5L 32-64-64-64-64-16 with weight norm)",
                "workload": "BASELINE config 4 shape, rows per GPU fixed: 5L D=32 H=64 OUT=16 training "
                            "step with weight norm, fp16 activation storage, M={M} rows per GPU"},
    # wide 3L D=H=OUT=256 (weights streamed), plain weights,
    # global M = 1,048,576 split over the ranks
    "W256": {"dims": (256, 256, 256, 256), "x_dist": "normal", "x_seed": 4, "strong": True, "wn": False,
             "metric": "fused MLP fwd+bwd rows/s (wide 3L D=H=OUT=256)",
             "workload": "BASELINE config 5: 3L D=H=OUT=256 training step (streamed weights), plain "
                         "weights (config 5 has no weight norm), fp16 activation storage, global M={G} rows, "
                         "{M} per GPU"},
}


# Per-kernel DRAM bytes of one launch, from the ncu captures summarised in
# profiles/ (name, rows of the captured launch); a step's traffic is their
# sum scaled to the step's rows (the traffic of these kernels grows with the
# rows: activations in and out; weights come from L2).
TRAIN_TRAFFIC = {
    "3L128": [("trainfwd_f32h_3L128_M262K", 262144), ("bwd_f32h_3L128_M262K", 262144)],
    "3L128_h16": [("trainfwd_3L128_M262K", 262144), ("bwd_3L128_M262K", 262144)],
    "5L": [("trainfwd_5L_M262K", 262144), ("bwd_5L_M262K", 262144)],
    "5L_weak": [("trainfwd_5L_M262K", 262144), ("bwd_5L_M262K", 262144)],
    "W256": [("trainfwd_W256_M131K", 131072), ("dgrad_W256_M131K", 131072), ("wgrad_W256_M131K", 131072)],
}


def step_traffic(name: str, rows: int):
    parts = TRAIN_TRAFFIC.get(name)
    if not parts:
        return None, None
    total = 0.0
    for prof, cap_rows in parts:
        b = load_traffic(prof)
        if b is None:
            return None, None
        total += b * rows / cap_rows
    return int(total), "sum of " + ", ".join(f"profiles/{p}.md" for p, _ in parts) + " scaled to the step's rows"


def run_training(args, world, rank, dist, barrier, name, rows):
    """One training step with weight norm per GPU through the C ABI on
    preallocated buffers: weight-norm forward, training forward, fused backward
    + fixed-order dW reduction, (N > 1: dW summed over the ranks by the
    library's NVLink peer-memory kernel), weight-norm backward.  `rows` is the
    per-GPU batch."""
    import ctypes

    import torch

    from mlp_megakernel_b200 import _lib
    from mlp_megakernel_b200.synthetic import make_grad, make_weights, make_x

    spec = TRAIN_SPECS[name]
    dims = spec["dims"]
    flop_per_row = 3 * 2 * sum(a * b for a, b in zip(dims[:-1], dims[1:]))  # fwd, dgrad, wgrad
    bytes_per_row = 2 * (2 * dims[0] + 2 * dims[-1])                       # x, out, grad_out, dx
    M = rows
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = _lib.lib()
    shape = ctypes.byref(_lib.shape_struct(dims))
    st = torch.cuda.current_stream().cuda_stream
    x = make_x(M, dims[0], spec["x_dist"], spec["x_seed"] + rank, device=dev)
    g = make_grad(M, dims[-1], seed=2 + rank, device=dev)
    ws0 = make_weights(dims, device=dev)
    v_all = torch.cat([w.float().reshape(-1) for w in ws0]).contiguous()
    g_all = torch.cat([w.float().norm(dim=0) for w in ws0]).contiguous()
    W = [torch.empty_like(w) for w in ws0]
    inv = torch.empty_like(g_all)
    out = torch.empty((M, dims[-1]), dtype=torch.float16, device=dev)
    h32 = spec.get("h32", False)
    h_code = _lib.H_F32 if h32 else _lib.H_F16
    hs = [torch.empty((M, d), dtype=torch.float32 if h32 else torch.float16, device=dev) for d in dims[1:-1]]
    dx = torch.empty_like(x)
    dw = torch.empty_like(v_all)
    dv = torch.empty_like(v_all)
    dg = torch.empty_like(g_all)
    work = torch.empty(int(lib.mlpk_bwd_workspace_size(shape, M)), dtype=torch.uint8, device=dev)
    Wp = _lib.ptr_array([w.data_ptr() for w in W])
    Hp = _lib.ptr_array([h.data_ptr() for h in hs])
    red = None
    if dist is not None:  # dW sum over the ranks: NVLink peer-memory kernel on one node
        from mlp_megakernel_b200.dp import make_grad_reducer

        red = make_grad_reducer(dw.numel())

    wn = spec.get("wn", True)
    if not wn:  # plain weights: the step is training forward + backward (+ all-reduce)
        for w, w0 in zip(W, ws0):
            w.copy_(w0)

    def step():
        st = torch.cuda.current_stream().cuda_stream  # the capture stream inside a graph capture
        if wn:
            _lib.check("wn_fwd", lib.mlpk_wn_fwd(shape, v_all.data_ptr(), g_all.data_ptr(), Wp,
                                                 inv.data_ptr(), st))
        _lib.check("train_fwd", lib.mlpk_train_fwd_ex(shape, M, x.data_ptr(), Wp, out.data_ptr(), Hp, h_code, st))
        local = red.local_buffer(dw) if red is not None else dw
        _lib.check("bwd", lib.mlpk_bwd_ex(shape, M, x.data_ptr(), Wp, Hp, h_code, g.data_ptr(), dx.data_ptr(),
                                          work.data_ptr(), work.numel(), local.data_ptr(), st))
        if red is not None:
            red.reduce(local, dw)
        if wn:
            _lib.check("wn_bwd", lib.mlpk_wn_bwd(shape, dw.data_ptr(), v_all.data_ptr(), g_all.data_ptr(),
                                                 inv.data_ptr(), dv.data_ptr(), dg.data_ptr(), st))

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # the timed steps replay the whole step (all kernels, and the dW sum across
    # ranks) as one CUDA graph: no host launch gaps between the kernels
    run = step
    if not args.no_graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        run = graph.replay
        run()
        torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.train_steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if _lib.device_status() != 0:
        raise RuntimeError("device status set during the training timing")

    # e2e: x and grad_out from pinned host memory, gradients (dv, dg) back to host
    xh, gh = x.cpu().pin_memory(), g.cpu().pin_memory()
    dvh = torch.empty(dv.shape, dtype=dv.dtype, pin_memory=True)
    dgh = torch.empty(dg.shape, dtype=dg.dtype, pin_memory=True)

    dwh = torch.empty(dw.shape, dtype=dw.dtype, pin_memory=True)

    def e2e_step():
        x.copy_(xh, non_blocking=True)
        g.copy_(gh, non_blocking=True)
        step()
        if wn:
            dvh.copy_(dv, non_blocking=True)
            dgh.copy_(dg, non_blocking=True)
        else:
            dwh.copy_(dw, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    n_e2e = 5
    e2.record()
    for _ in range(n_e2e):
        e2e_step()
    e3.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e2.elapsed_time(e3)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # kernels of ours per step: [wn_fwd], train_fwd, backward (fused kernel + reduce, or for the
    # streamed network data-gradient chain + weight-gradient kernel + reduce), [peer dW sum], [wn_bwd]
    peer = red is not None and type(red).__name__ == "PeerGradReducer"
    launches_per_step = ((2 if wn else 0) + 1 + (3 if dims == (256, 256, 256, 256) else 2)
                         + (1 if peer else 0))
    if red is not None:
        red.close()
    peaks = load_peaks()
    l2_resident = M * dims[1] * 2 * (len(dims) - 2) <= 126e6
    traffic, traffic_src = (step_traffic(name, M) if not l2_resident else
                            (None, "not scaled: the step's working set stays in L2, so the DRAM bytes "
                                   "of the full-size captures do not carry over"))
    per_step = ms / 1e3 / args.train_steps
    tflops = flop_per_row * M / per_step / 1e12
    gbs = bytes_per_row * M / per_step / 1e9
    tensor_rows = peaks["bf16_tflops"] * 1e12 / flop_per_row
    hbm_rows = peaks["hbm_gbs"] * 1e9 / bytes_per_row
    roof_rows = min(tensor_rows, hbm_rows)
    return {
        "_grads": (dx.detach().clone(), dv.detach().clone(), dg.detach().clone()),
        "metric": spec["metric"],
        "value": world * M * args.train_steps / (ms / 1e3),
        "unit": "rows/s",
        "steps": args.train_steps,
        "ms_per_step": ms / args.train_steps,
        "scaling": "strong" if spec["strong"] else "weak",
        "config": {"workload": spec["workload"].format(M=M, G=world * M),
                   "dims": list(dims), "rows_per_gpu": M, "global_rows": world * M,
                   "activation_storage": "fp32" if h32 else "fp16",
                   "parallelism": f"dp{world}" + ((" (fp32 dW summed by the NVLink peer-memory kernel)" if peer
                                                   else " (NCCL all-reduce of fp32 dW)") if world > 1 else ""),
                   "launch": "eager" if args.no_graph else "CUDA graph of the whole step",
                   "l2": "per-step inputs and saved activations larger than L2" if not l2_resident else
                         "working set partly L2-resident (no flush between steps)"},
        "roofline": {"bound": "tensor" if tensor_rows <= hbm_rows else "hbm",
                     "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / peaks["bf16_tflops"],
                     "rows_frac_of_roofline": (M / per_step) / roof_rows,
                     "achieved_algorithmic_gbs": gbs, "traffic": traffic, "traffic_source": traffic_src,
                     "traffic_unit": "DRAM bytes per step (all of the step's kernels)",
                     "flop_per_row": flop_per_row, "algorithmic_bytes_per_row": bytes_per_row},
        "e2e": {"value": world * M * n_e2e / (e2e_ms / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": M * (dims[0] + dims[-1]) * 2,
                "d2h_bytes_per_step": ((dv.numel() + dg.numel()) if wn else dw.numel()) * 4,
                "api": "C ABI (" + ("mlpk_wn_fwd, " if wn else "") + "mlpk_train_fwd_ex, mlpk_bwd_ex"
                       + (", mlpk_wn_bwd" if wn else "") + ") with pinned host buffers"},
        "gpu_launches": launches_per_step * args.train_steps,
    }


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mlpk(args)


if __name__ == "__main__":
    main()
