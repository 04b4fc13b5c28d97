#!/usr/bin/env python
"""Benchmark of the Mantle graph hot path on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload all|scatter|chain|fft|gemm|cnn|showcase]
                    [--impl ours|reference]

A step is one replay (`run`) of a workload's recorded graph over its synthetic
inputs. With no flags (`--workload all`) every config of the benchmark runs in
turn, K timed steps each, and ONE line is printed:

* the headline is the two-scatters-plus-three-updates graph: two scatter-adds
  of 2^24 Float32 values by uniform Int32 index into 2^16 bins (an Int32
  histogram fused into the first), then three in-place updates with
  read-after-write hazards on a Float32[2^20] buffer. `value` is whole-job
  algorithmic GB/s: (16 B per scattered element + 36 B per updated element) x
  ranks / max-over-ranks time per step. Inputs (256 MiB per replay) exceed
  the 126 MB L2, so steps replay back to back;
* `workloads` holds one record per other config, each with its own
  `value`, `ms_per_step`, `roofline`, `cpu_baseline`, `e2e` and `clocks`:
  the eight-kernel elementwise chain (N = 2^22), the batched FFT (16384 x
  4096 ComplexF32, forward then inverse), the dense GEMM (8 x 8192^3 bf16 ->
  fp32), the CNN forward (batch 256, 3 x 224 x 224), and the reference's own
  replayed-graph comparison (bench/independent.jl: 8 chains x 6 stir! stages,
  derived against :backend barriers, in alternating rounds).

Multi-GPU (torchrun, one process per GPU): the scatter and chain graphs are
independent per rank ("scaling": "weak"); the GEMM batch, the FFT transforms
and the CNN images are split across the ranks (`shard_range`, "scaling":
"strong"), and only the CNN all-gathers its logits over NCCL, every step. The
barrier and the max-over-ranks reduction of the device-timed steps go through
torch.distributed.

`--impl reference` times the CPU restatement of the same workloads (the
oracle, C + OpenMP on all host cores) — the reference itself is Julia on
Vulkan and cannot run here. Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "mantle.jl_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "replayed-graph GB/s & TFLOP/s vs roofline; DNN images/sec at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20  # written between steps whose inputs could stay in the 126 MB L2


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return FALLBACK_PEAKS, "fallback"


def traffic_of(name: str):
    """DRAM bytes per launch of a kernel from its committed ncu summary."""
    tp = ROOT / "profiles" / f"{name}_traffic.json"
    if tp.exists():
        try:
            return json.loads(tp.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


# ── clocks during the timed region (NVML, read only) ────────────────────────
class ClockSampler:
    """Samples SM clock and throttle reasons every few ms while running."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int):
        self.index = index
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: clocks are reported as unavailable
            self.err = str(e)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.005)

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._t:
            self._stop.set()
            self._t.join()
            self._sample()
        return False

    def summary(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ── distributed plumbing ────────────────────────────────────────────────────
def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, x: float) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    # NCCL reduces device tensors; gloo (the CPU tests of this plumbing) host ones
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finish(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def release_device_memory(local: int) -> None:
    """Between workloads: drop the last one's buffers and plans (their
    finalizers free the device memory) and torch's cached blocks."""
    import torch
    torch.cuda.synchronize(local)
    gc.collect()
    torch.cuda.synchronize(local)
    torch.cuda.empty_cache()


# ── timing helpers ──────────────────────────────────────────────────────────
def device_time_ms(stream_ptr: int, fn, steps: int) -> float:
    """CUDA events on the stream the work is launched on; sync on both sides.
    A ~100 us spin kernel runs on the stream before the start event, so the
    host has queued the first steps by the time the GPU reaches it: the timed
    region holds the steps, not the host's latency to issue the first ones
    (without it, 20 replays of the 13.4 us chain measured 14.8 us a step)."""
    import torch
    s = torch.cuda.ExternalStream(stream_ptr)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        torch.cuda._sleep(200_000)
    a.record(s)
    for _ in range(steps):
        fn()
    b.record(s)
    b.synchronize()
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def device_time_flushed_ms(stream_ptr: int, fn, steps: int, local: int) -> float:
    """Sum of per-step CUDA-event durations, with the L2 flushed between
    steps on the same stream, outside the event pairs: a 256 MiB buffer is
    written, then a second one read, so a step finds none of its inputs in
    the 126 MB L2 and no dirty line of the flush left to write back inside
    its own timed region."""
    import torch
    s = torch.cuda.ExternalStream(stream_ptr)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{local}")
    clean = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{local}")
    sink = torch.zeros(1, dtype=torch.float32, device=f"cuda:{local}")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for i in range(steps):
            flush.fill_(float(i))
            torch.sum(clean, dim=0, keepdim=True, out=sink)
            ev[i][0].record(s)
            fn()
            ev[i][1].record(s)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev)


_PINNED: list = []


def pinned_like(a: np.ndarray) -> np.ndarray:
    """A copy of `a` in page-locked host memory (kept alive for the process)."""
    import torch
    t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
    _PINNED.append(t)
    out = t.numpy()
    out[...] = a
    return out


def e2e_time(dev, ws, steps: int, uploads, run, downloads) -> dict:
    """End-to-end seconds per step through the public API: every step uploads
    `uploads` ((Buffer, pinned host array) pairs) from host memory, calls
    `run()`, and downloads `downloads` ((Buffer, host array) pairs); wall
    clock over the steps (max over ranks), after two untimed steps."""
    import mantle_cuda as M

    def one():
        for buf, host in uploads:
            M.check(M.lib().mtl_buffer_upload(buf.handle, host.ctypes.data, 0, host.nbytes))
        run()
        for buf, host in downloads:
            M.check(M.lib().mtl_buffer_download(buf.handle, host.ctypes.data, 0, host.nbytes))

    for _ in range(2):
        one()
    dev.synchronize()
    barrier(ws)
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dev.synchronize()
    sec = max_over_ranks(ws, (time.perf_counter() - t0) / steps)
    return {"seconds": sec, "h2d_bytes_per_step": int(sum(h.nbytes for _, h in uploads)),
            "d2h_bytes_per_step": int(sum(h.nbytes for _, h in downloads))}


# ── CPU timing (the oracle: the reference arm and every cpu_baseline leg) ───
def cpu_timed(one, steps: int, budget_s: float, warm_s: float = 2.0) -> dict:
    """Time `steps` steps of CPU work, each step `reps` calls of `one()` (which
    returns the algorithmic units it processed), with `reps` chosen so the
    steps take about `budget_s` together. Before timing, `one()` runs for
    about `warm_s` untimed (threads spun up, pages touched, clocks settled).
    The reference arm and the cpu_baseline leg of the GPU arm both time
    through here, so the two figures are taken the same way."""
    t0 = time.perf_counter()
    one()
    calls = 1
    while time.perf_counter() - t0 < warm_s:
        one()
        calls += 1
    per_call = max((time.perf_counter() - t0) / calls, 1e-9)
    # a call slower than budget / steps (an image of the CNN, a band of the
    # GEMM) makes each step one call and takes fewer steps
    steps = max(1, steps)
    if steps * per_call > budget_s:
        steps, reps = max(1, int(budget_s / per_call)), 1
    else:
        reps = max(1, math.ceil(budget_s / (steps * per_call)))
    units = 0
    t0 = time.perf_counter()
    for _ in range(steps):
        for _ in range(reps):
            units += one()
    dt = time.perf_counter() - t0
    return {"units_per_s": units / dt, "seconds": dt, "steps": steps, "reps_per_step": reps,
            "calls": steps * reps}


def scatter_inputs(rank: int = 0, n: int = 1 << 24, nbins: int = 1 << 16, nupd: int = 1 << 20) -> dict:
    """The scatter workload's host inputs, as build_scatter draws them."""
    from mantle_cuda.workloads import seeded_integers, seeded_uniform
    s = 10 * rank
    return {"va": seeded_uniform(0, n, 0, 1, s + 0), "ia": seeded_integers(0, n, nbins, s + 1),
            "vb": seeded_uniform(0, n, 0, 1, s + 2), "ib": seeded_integers(0, n, nbins, s + 3),
            "b": seeded_uniform(0, nupd, -1, 1, s + 4), "c": seeded_uniform(0, nupd, -1, 1, s + 5),
            "d": seeded_uniform(0, nupd, -1, 1, s + 6)}


def cpu_scatter_step(inp: dict, nbins: int, threads: int) -> int:
    """One step of the workload on the CPU: two scatters + histogram + three
    updates, float32 with private per-thread bins (oracle/mantle_oracle.c).
    Returns the algorithmic bytes."""
    import ctypes as C

    from oracle import oracle as O
    lib = O.lib()
    n = int(inp["ia"].size)
    nu = int(inp["b"].size)
    st = cpu_scatter_step.__dict__.setdefault("scratch", {})
    key = (threads, nbins)
    if key not in st:
        st[key] = (np.zeros(threads * nbins, np.float32), np.zeros(threads * nbins, np.uint32),
                   np.zeros(nbins, np.float32), np.zeros(nbins, np.float32), np.zeros(nbins, np.uint32))
    sf, su, acc_a, acc_b, hist = st[key]
    if "b_work" not in inp:
        inp["b_work"] = inp["b"].copy()
    f32p, i32p, u32p = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.POINTER(C.c_uint32)
    P = lambda a, t: a.ctypes.data_as(t)  # noqa: E731
    lib.oracle_scatter_f32(P(inp["va"], f32p), P(inp["ia"], i32p), n, nbins, P(acc_a, f32p), P(hist, u32p),
                           P(sf, f32p), P(su, u32p), threads)
    lib.oracle_scatter_f32(P(inp["vb"], f32p), P(inp["ib"], i32p), n, nbins, P(acc_b, f32p), None,
                           P(sf, f32p), P(su, u32p), threads)
    lib.oracle_touch3(P(inp["b_work"], f32p), P(inp["c"], f32p), P(inp["d"], f32p), nu, threads)
    return 16 * n + 36 * nu


def cpu_scatter(inp: dict, nbins: int, steps: int, budget_s: float) -> dict:
    from oracle import oracle as O
    threads = O.max_threads()
    r = cpu_timed(lambda: cpu_scatter_step(inp, nbins, threads), steps, budget_s)
    return {"value": round(r["units_per_s"] / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{r['steps']} steps x {r['reps_per_step']} full replays (2x 2^{int(np.log2(inp['ia'].size))} "
                      f"scatter + histogram + 3 updates on 2^{int(np.log2(inp['b'].size))}), oracle C + OpenMP, "
                      f"{r['seconds']:.1f} s after a 2 s warm-up"}


def cpu_chain(inp: dict, steps: int, budget_s: float) -> dict:
    """The eight kernels as eight OpenMP passes (oracle chain8_passes)."""
    from oracle import oracle as O
    threads = O.max_threads()
    n = inp["x"].size

    def one():
        O.chain8_passes(inp["x"], inp["y"], inp["z"], threads=threads)
        return 16 * n

    r = cpu_timed(one, steps, budget_s)
    return {"value": round(r["units_per_s"] / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{r['calls']} replays of the 8 kernels over 2^{int(np.log2(n))} elements (one OpenMP pass "
                      f"per kernel), {r['seconds']:.1f} s; GB/s of the 16 compulsory bytes per element"}


def cpu_fft(x: np.ndarray, steps: int, budget_s: float) -> dict:
    """Forward + inverse of a sample of 1024 transforms (oracle, float, OpenMP)."""
    from oracle import oracle as O
    threads = O.max_threads()
    sample = np.ascontiguousarray(x[:1024])

    def one():
        O.fft(O.fft(sample, f32=True), inverse=True, f32=True)
        return 2 * 2 * 8 * sample.size

    r = cpu_timed(one, steps, budget_s)
    return {"value": round(r["units_per_s"] / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{r['calls']} x (forward + inverse of 1024 transforms of {x.shape[1]}), oracle radix-2 in "
                      f"float, OpenMP, {r['seconds']:.1f} s"}


def cpu_gemm(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int, steps: int, budget_s: float) -> dict:
    """Bands of 16 rows of one 8192^3 GEMM (oracle, double, OpenMP)."""
    from oracle import oracle as O
    threads = O.max_threads()
    rows = 16
    done = [0]

    def one():
        O.gemm_bf16(A[:1], B[:1], M, N, K, 1, row0=(done[0] * rows) % M, rows=rows)
        done[0] += 1
        return 2 * rows * N * K

    r = cpu_timed(one, steps, budget_s)
    return {"value": round(r["units_per_s"] / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{r['calls'] * rows} rows of one {M}x{N}x{K} GEMM (oracle, double accumulation, OpenMP), "
                      f"{r['seconds']:.1f} s"}


def cpu_cnn(x, wts, fc, steps: int, budget_s: float) -> dict:
    """Whole images through the oracle forward pass (double, OpenMP)."""
    from mantle_cuda.workloads import CNN_LAYERS, STEM_CPAD
    from oracle import oracle as O
    threads = O.max_threads()
    done = [0]
    nimg = x.shape[0]

    def one():
        i = done[0] % nimg
        O.cnn_forward(x[i:i + 1], wts, fc, CNN_LAYERS, STEM_CPAD)
        done[0] += 1
        return 1

    r = cpu_timed(one, steps, budget_s, warm_s=0.0)
    return {"value": round(r["units_per_s"], 3), "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"{r['calls']} images through the oracle forward pass (double, OpenMP), {r['seconds']:.1f} s"}


# ── configs shared by both arms ─────────────────────────────────────────────
def scatter_config(ws: int, n: int = 1 << 24, nbins: int = 1 << 16, nupd: int = 1 << 20) -> dict:
    return {"workload": "two scatters + int32 histogram + three RAW updates (bench/two_scatters.jl, "
                        "bench/three_updates.jl shape)",
            "scatter_elements": n, "bins": nbins, "update_elements": nupd,
            "graph": "5 passes, replayed as one CUDA graph", "parallelism": f"{ws} independent graphs",
            "l2": "inputs (256 MiB/step) exceed the 126 MB L2; no flush"}


SCATTER_DATA = "synthetic: seeded PCG64, values U[0,1], indices U{0..65535}, update buffers U[-1,1]"


def chain_config(ws: int, n: int, unfused: bool, copies: int = 4) -> dict:
    return {"workload": "elementwise chain, 8 dependent kernels (axpy a=0.5, mul, add, fma, abs, sqrt(abs), "
                        "scale 2, sub)" + (" (unfused)" if unfused else " (fused, compiled)"),
            "n": n, "bytes_per_step": 16 * n, "parallelism": f"{ws} independent graphs",
            "l2": f"{copies} copies of the graph (4 x 64 MiB) replayed in turn: inputs larger than the L2"}


def fft_config(ws: int, batch: int, n: int) -> dict:
    return {"workload": "batched 1-D complex FFT, forward then inverse", "transforms": batch, "length": n,
            "bytes_per_step": 2 * 2 * 8 * batch * n,
            "parallelism": f"{batch // ws} transforms per GPU on {ws} GPU(s), no collective",
            "l2": "L2 flushed between steps (256 MiB written, then 256 MiB read, outside the timed events)"}


def gemm_config(ws: int, batch: int, M: int, N: int, K: int) -> dict:
    return {"workload": "dense GEMM C = A.B, bf16 in, fp32 accumulate and out", "M": M, "N": N, "K": K,
            "batch": batch, "parallelism": f"{batch // ws} GEMM(s) per GPU on {ws} GPU(s), no collective",
            "l2": "A and B 128 MiB each per GEMM, C 256 MiB, above the 126 MB L2; no flush"}


def cnn_config(ws: int, total: int) -> dict:
    return {"workload": "CNN inference: 7x7/2 stem, 4 stages of two 3x3 convs (64-512), ReLU, GAP, FC 1000",
            "global_batch": total, "image": [3, 224, 224], "parallelism": f"batch split over {ws} GPUs"
            + (", NCCL all-gather of the logits every step" if ws > 1 else ""),
            "l2": "L2 flushed between steps (256 MiB written, then 256 MiB read, outside the timed events)"}


# ── workloads ───────────────────────────────────────────────────────────────
def bench_scatter(args, ws, rank, local, peaks, peak_kind):
    import torch

    import mantle_cuda as M
    from mantle_cuda.workloads import build_scatter

    dev = M.Device(local)
    w = build_scatter(dev, rank=rank)
    plan = w.plan
    stream = dev.stream

    for _ in range(args.warmup):
        M.run(plan)
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_ms(stream, lambda: M.run(plan), args.steps)
    ms_step = max_over_ranks(ws, ms / args.steps)
    value = ws * w.bytes_step / (ms_step * 1e-3) / 1e9

    # The dominant kernel, timed alone on the same stream: scatter a (value +
    # index per element; histogram fused).
    B = w.bufs
    kargs = (B["acc_a"], B["hist"], B["va"], B["ia"], w.nbins, 0)
    wsb = M.workspace_bytes(M.kernels.scatter_add, kargs, w.n)
    scratch = torch.empty(max(wsb, 16), dtype=torch.uint8, device=f"cuda:{local}")
    launch = lambda: M.launch(M.kernels.scatter_add, kargs, w.n, stream=stream, workspace=scratch)  # noqa: E731
    for _ in range(3):
        launch()
    kreps = max(10, min(args.steps, 200))
    k_ms = device_time_ms(stream, launch, kreps) / kreps
    algo_bytes = 8 * w.n
    achieved = algo_bytes / (k_ms * 1e-3) / 1e9
    # What bounds it in practice: the shared-memory atomics. The same call with
    # 2^12 bins (one CTA holds every bin: no cluster, no redundant streaming)
    # over the same 2^24 values and uniform indices is the atomic floor.
    gen = torch.Generator(device=f"cuda:{local}").manual_seed(1234)
    idx_small = torch.randint(0, 1 << 12, (w.n,), generator=gen, device=f"cuda:{local}", dtype=torch.int32)
    acc_small = torch.zeros(1 << 12, device=f"cuda:{local}")
    hist_small = torch.zeros(1 << 12, dtype=torch.int32, device=f"cuda:{local}")
    fargs = (acc_small, hist_small, B["va"], idx_small, 1 << 12, 0)
    fws = torch.empty(max(M.workspace_bytes(M.kernels.scatter_add, fargs, w.n), 16), dtype=torch.uint8,
                      device=f"cuda:{local}")
    flaunch = lambda: M.launch(M.kernels.scatter_add, fargs, w.n, stream=stream, workspace=fws)  # noqa: E731
    for _ in range(3):
        flaunch()
    floor_ms = device_time_ms(stream, flaunch, kreps) / kreps
    # The same call on piled-up bins, the splat-like case: 90 % of the indices
    # in 64 bins, and all in one bin, through both scatter families.
    rng = np.random.Generator(np.random.PCG64([4321, 9]))
    hot = torch.from_numpy(rng.choice(w.nbins, 64, replace=False).astype(np.int32)).to(f"cuda:{local}")
    gs = torch.Generator(device=f"cuda:{local}").manual_seed(4321)
    idx_skew = torch.randint(0, w.nbins, (w.n,), generator=gs, device=f"cuda:{local}", dtype=torch.int32)
    pick = torch.rand(w.n, generator=gs, device=f"cuda:{local}") < 0.9
    idx_skew[pick] = hot[torch.randint(0, 64, (int(pick.sum()),), generator=gs, device=f"cuda:{local}")]
    idx_one = torch.full((w.n,), 40000, dtype=torch.int32, device=f"cuda:{local}")
    pile = {}
    for shape, ix in (("skewed", idx_skew), ("one_bin", idx_one)):
        for fam in ("scatter_add", "scatter_add_dense"):
            sargs = (B["acc_a"], B["hist"], B["va"], ix, w.nbins, 0)
            kern = getattr(M.kernels, fam)
            slaunch = lambda: M.launch(kern, sargs, w.n, stream=stream, workspace=scratch)  # noqa: E731
            for _ in range(2):
                slaunch()
            reps = 5 if shape == "one_bin" else kreps
            pile[f"{shape}_{fam}_ms"] = round(device_time_ms(stream, slaunch, reps) / reps, 4)
    roofline = {"bound": "hbm", "kernel": "scatter_add (scatter a: 2^24 values -> 2^16 bins + histogram)",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic_of("scatter_add"),
                "algorithmic_bytes": algo_bytes, "peak_kind": f"{peak_kind} (burst copy)",
                "kernel_ms": round(k_ms, 4),
                "atomic_floor_ms": round(floor_ms, 4),
                "frac_of_atomic_floor": round(floor_ms / k_ms, 4),
                "atomic_floor": "the same call with 2^12 bins (all bins in one CTA's shared memory), measured here",
                "piled_bins": dict(pile, note="the same call with 90 % of the indices in 64 of the 2^16 bins "
                                              "(skewed) and with every index in one bin (one_bin), through "
                                              "scatter_add and scatter_add_dense (warp-aggregated atomics)")}
    del scratch, fws, idx_small, acc_small, hist_small, idx_skew, idx_one

    # End to end through the public API: each step the four input arrays go
    # from pinned host memory through Update, the graph replays, and the bins
    # come back to the host.
    w2 = build_scatter(dev, rank=rank, with_updates_from_host=True)
    host = {k: pinned_like(w2.inputs[k]) for k in ("va", "ia", "vb", "ib")}
    h2d = sum(v.nbytes for v in host.values())
    outs = {k: np.empty(w2.nbins, np.float32 if k != "hist" else np.int32) for k in ("acc_a", "acc_b", "hist")}
    d2h = sum(v.nbytes for v in outs.values())

    def e2e_step():
        for k, v in host.items():
            w2.refs[k](v)
        M.run(w2.plan)
        for k, o in outs.items():
            M.lib().mtl_buffer_download(w2.bufs[k].handle, o.ctypes.data, 0, o.nbytes)

    for _ in range(2):
        e2e_step()
    dev.synchronize()
    barrier(ws)
    e2e_steps = max(3, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    dev.synchronize()
    e2e_s = max_over_ranks(ws, (time.perf_counter() - t0) / e2e_steps)
    e2e = {"value": round(ws * w2.bytes_step / e2e_s / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_s * 1e3, 3)}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_scatter(dict(w.inputs), w.nbins, args.steps, args.cpu_seconds)

    nk = plan.nkernels()
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+i32",
        "data": SCATTER_DATA, "config": scatter_config(ws, w.n, w.nbins, w.nupd),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": nk * args.steps, "kernels_per_step": nk, "clocks": clk.summary(),
    }


def bench_chain(args, ws, rank, local, peaks, peak_kind):
    import mantle_cuda as M
    from mantle_cuda.workloads import build_chain

    dev = M.Device(local)
    # The chain's 64 MiB fit in the 126 MB L2, so four copies of the graph on
    # their own buffers (256 MiB) are replayed in turn: a replay finds its
    # inputs evicted by the three before it and reads them from HBM.
    copies = 4
    ws_ = [build_chain(dev, seed=4 * rank + k, fuse=not args.unfused) for k in range(copies)]
    turn = [0]

    def step():
        M.run(ws_[turn[0] % copies].plan)
        turn[0] += 1

    for _ in range(max(args.warmup, copies)):
        step()
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_ms(dev.stream, step, args.steps)
    ms_step = max_over_ranks(ws, ms / args.steps)
    w = ws_[0]
    nbytes = w.bytes_unfused if args.unfused else w.bytes_compulsory
    value = ws * nbytes / (ms_step * 1e-3) / 1e9
    nk = w.plan.nkernels()
    # end to end: x, y, z from pinned host memory, one replay, out back to the host
    ups = [(getattr(w, k), pinned_like(w.inputs[k])) for k in ("x", "y", "z")]
    out_host = np.empty(w.n, np.float32)
    t = e2e_time(dev, ws, max(3, min(args.steps, 20)), ups, lambda: M.run(w.plan), [(w.out, out_host)])
    e2e = {"value": round(ws * w.bytes_compulsory / t["seconds"] / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": t["h2d_bytes_per_step"], "d2h_bytes_per_step": t["d2h_bytes_per_step"],
           "ms_per_step": round(t["seconds"] * 1e3, 3)}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_chain(w.inputs, args.steps, args.cpu_seconds)
    achieved = w.bytes_compulsory / (ms_step * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded PCG64, x,y,z U[-1,1]",
        "config": chain_config(ws, w.n, args.unfused, copies),
        "roofline": {"bound": "hbm", "kernel": "the fused chain kernel (one launch a step)" if not args.unfused
                     else "8 elementwise kernels", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic_of("chain_fused") if not args.unfused else None,
                     "algorithmic_bytes": w.bytes_compulsory, "peak_kind": f"{peak_kind} (burst copy)",
                     "timed": "the whole run per step (one kernel launch a step, the gaps between steps included)"},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": nk * args.steps, "clocks": clk.summary(),
    }


def bench_fft(args, ws, rank, local, peaks, peak_kind):
    """16384 ComplexF32 transforms of 4096 points, forward then inverse, as a
    two-pass graph; the transforms are split across the ranks (strong scaling,
    no collective)."""
    import mantle_cuda as M
    from mantle_cuda.workloads import build_fft

    total = 16384
    dev = M.Device(local)
    w = build_fft(dev, batch=total, rank=rank, world=ws)
    for _ in range(args.warmup):
        M.run(w.plan)
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_flushed_ms(dev.stream, lambda: M.run(w.plan), args.steps, local)
    ms_step = max_over_ranks(ws, ms / args.steps)
    value = ws * w.bytes_step / (ms_step * 1e-3) / 1e9

    # The forward kernel alone on the same stream (16 B per point), L2 flushed
    # between launches.
    launch = lambda: M.launch(M.kernels.fft_c2c, (w.spectrum, w.x, w.n, 0), w.batch, stream=dev.stream)  # noqa: E731
    for _ in range(3):
        launch()
    kreps = max(10, min(args.steps, 100))
    k_ms = device_time_flushed_ms(dev.stream, launch, kreps, local) / kreps
    algo = 16 * w.batch * w.n
    achieved = algo / (k_ms * 1e-3) / 1e9
    # end to end: the input from pinned host memory, forward + inverse, the
    # round trip back to the host
    back_host = np.empty(w.inputs["x"].shape, w.inputs["x"].dtype)
    t = e2e_time(dev, ws, 3, [(w.x, pinned_like(w.inputs["x"]))], lambda: M.run(w.plan), [(w.back, back_host)])
    e2e = {"value": round(ws * w.bytes_step / t["seconds"] / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": t["h2d_bytes_per_step"], "d2h_bytes_per_step": t["d2h_bytes_per_step"],
           "ms_per_step": round(t["seconds"] * 1e3, 3)}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_fft(w.inputs["x"], args.steps, args.cpu_seconds)
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "c64",
        "data": "synthetic: seeded PCG64, re/im U[-1,1]",
        "config": fft_config(ws, total, w.n),
        "roofline": {"bound": "hbm", "kernel": f"fft_pipe_kernel (forward, {w.batch} x {w.n})",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic_of("fft_forward"),
                     "algorithmic_bytes": algo, "peak_kind": f"{peak_kind} (burst copy)", "kernel_ms": round(k_ms, 4)},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": w.plan.nkernels() * args.steps, "clocks": clk.summary(),
    }


def bench_gemm(args, ws, rank, local, peaks, peak_kind):
    """8 GEMMs of 8192^3 (bf16 in, fp32 accumulate and out) as one graph pass;
    the batch is split across the ranks (strong scaling, no collective)."""
    import mantle_cuda as M
    from mantle_cuda.workloads import build_gemm

    total = 8
    dev = M.Device(local)
    w = build_gemm(dev, batch=total, rank=rank, world=ws)
    for _ in range(args.warmup):
        M.run(w.plan)
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_ms(dev.stream, lambda: M.run(w.plan), args.steps)
    ms_step = max_over_ranks(ws, ms / args.steps)
    tflops = ws * w.flops_step / (ms_step * 1e-3) / 1e12
    per_gpu = w.flops_step / (ms_step * 1e-3) / 1e12
    # The timed region is back-to-back GEMMs under the power cap: the sustained
    # peak is the denominator; the burst figure is reported beside it.
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    roofline = {"bound": "tensor", "kernel": f"gemm_bf16_kernel ({w.batch} x 8192^3 per launch)",
                "achieved": round(per_gpu, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(per_gpu / peak, 4),
                "traffic": traffic_of("gemm"), "algorithmic_flops": w.flops_step,
                "peak_kind": f"{peak_kind} (sustained cuBLAS bf16)",
                "frac_of_burst_peak": round(per_gpu / peaks["bf16_tflops"], 4), "kernel_ms": round(ms_step, 4)}
    # end to end: A and B (bf16 bits) from pinned host memory, the batch of
    # GEMMs, C back to the host
    A_host, B_host = w.host_operands()
    C_host = np.empty(w.batch * w.M * w.N, np.float32)
    t = e2e_time(dev, ws, 3, [(w.A, pinned_like(A_host.view(np.int16))), (w.B, pinned_like(B_host.view(np.int16)))],
                 lambda: M.run(w.plan), [(w.C, C_host)])
    e2e = {"value": round(ws * w.flops_step / t["seconds"] / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": t["h2d_bytes_per_step"], "d2h_bytes_per_step": t["d2h_bytes_per_step"],
           "ms_per_step": round(t["seconds"] * 1e3, 3)}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_gemm(A_host, B_host, w.M, w.N, w.K, args.steps, args.cpu_seconds)
    return {
        "metric": METRIC, "value": round(tflops, 1), "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: torch Philox seed 1, normal(0,1)/sqrt(K) rounded to bf16",
        "config": gemm_config(ws, total, w.M, w.N, w.K),
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": w.plan.nkernels() * args.steps,
        "clocks": clk.summary(),
    }


def bench_cnn(args, ws, rank, local, peaks, peak_kind):
    """CNN inference at batch 256: the batch is split across the ranks ("scaling":
    "strong"), each rank replays its forward graph on its images, and the
    logits are all-gathered over NCCL every step (N > 1)."""
    import mantle_cuda as M
    from mantle_cuda.workloads import CNN_CLASSES, build_cnn

    total = 256
    dev = M.Device(local)
    w = build_cnn(dev, batch=total, rank=rank, world=ws)
    comm = gathered = None
    if ws > 1:
        import torch.distributed as dist
        obj = [M.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = M.Comm(dev, ws, rank, obj[0])
        gathered = M.Buffer(dev, np.float32, total * CNN_CLASSES)

    def step():
        M.run(w.plan)
        if comm is not None:
            comm.allgather(w.logits, gathered)

    for _ in range(args.warmup):
        step()
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_flushed_ms(dev.stream, step, args.steps, local)
    ms_step = max_over_ranks(ws, ms / args.steps)
    images_s = total / (ms_step * 1e-3)
    flops = 2 * total * (w.flops_step // (2 * w.batch))

    # End to end through the public API: each step this rank's images (NCHW
    # bf16) go from pinned host memory into the input buffer, the graph
    # replays (and the logits are all-gathered when N > 1), and this rank's
    # logits come back to the host.
    x_bits, wts, fc = w.host_params()
    x_host = pinned_like(x_bits.view(np.int16))
    logits_host = np.empty(w.batch * CNN_CLASSES, np.float32)

    def e2e_step():
        M.check(M.lib().mtl_buffer_upload(w.x.handle, x_host.ctypes.data, 0, x_host.nbytes))
        step()
        M.check(M.lib().mtl_buffer_download(w.logits.handle, logits_host.ctypes.data, 0, logits_host.nbytes))

    for _ in range(2):
        e2e_step()
    dev.synchronize()
    barrier(ws)
    e2e_steps = max(3, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    dev.synchronize()
    e2e_s = max_over_ranks(ws, (time.perf_counter() - t0) / e2e_steps)
    e2e = {"value": round(total / e2e_s, 1), "unit": "images/s", "h2d_bytes_per_step": int(x_host.nbytes),
           "d2h_bytes_per_step": int(logits_host.nbytes), "ms_per_step": round(e2e_s * 1e3, 3)}
    tflops = flops / (ms_step * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    per_gpu = tflops / ws
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_cnn(x_bits, wts, fc, args.steps, args.cpu_seconds)
    if comm is not None:
        dev.synchronize()
        comm.release()
    return {
        "metric": METRIC, "value": round(images_s, 1), "unit": "images/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: torch Philox, input U[0,1) seed 4, He-normal weights seed 3",
        "config": dict(cnn_config(ws, total), tflops=round(tflops, 1)),
        "roofline": {"bound": "tensor", "kernel": "the whole forward graph (conv2d_nchw_bf16 + 8 conv2d_bf16 + "
                                                  "gap + fc)",
                     "achieved": round(per_gpu, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(per_gpu / peak, 4),
                     "traffic": traffic_of("cnn_forward"), "algorithmic_flops": flops // ws,
                     "peak_kind": f"{peak_kind} (sustained cuBLAS bf16)",
                     "frac_of_burst_peak": round(per_gpu / peaks["bf16_tflops"], 4)},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": w.plan.nkernels() * args.steps, "clocks": clk.summary(),
    }


def bench_showcase(args, ws, rank, local, peaks, peak_kind):
    """The showcase frame at the reference's size (1600 x 900, 5000 crystals +
    44 light crystals, 44 lights, a 2048^2 shadow map) as one replayed graph of
    fifteen passes: the thirteen compute passes and the shadow and g-buffer
    raster passes; each rank renders its own frame (weak scaling)."""
    import mantle_cuda as M
    from mantle_cuda.workloads import build_showcase, crystal_scene
    from oracle import oracle as O

    dev = M.Device(local)
    sc = crystal_scene(1600, 900, seed=9 + rank, smap_res=2048)
    w = build_showcase(dev, sc)
    for _ in range(args.warmup):
        M.run(w.plan)
    dev.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        ms = device_time_ms(dev.stream, lambda: M.run(w.plan), args.steps)
    ms_step = max_over_ranks(ws, ms / args.steps)
    npx = sc.w * sc.h
    # compulsory image bytes of a frame: the raster passes' writes (depth and
    # three g-buffer channels, the shadow map); depth for the tiles; depth +
    # normal at the occlusion samples' centres and its half-resolution output,
    # read and blurred; the four g-buffer channels, the occlusion map and the
    # HDR write of lighting; the four bright taps per bloom pixel and the bloom
    # chain; HDR + bloom read and the output write of the composite
    bw, bh = -(-sc.w // sc.shift), -(-sc.h // sc.shift)
    aon = -(-sc.w // 2) * -(-sc.h // 2)
    algo = (16 * npx + 4 * sc.smap_res ** 2
            + 4 * npx + 8 * aon + 8 * aon + 12 * aon + (16 + 4 + 4 * aon / npx) * npx + 16 * npx
            + 4 * 16 * bw * bh + 16 * bw * bh + 4 * 32 * bw * bh + 32 * npx)
    achieved = algo / (ms_step * 1e-3) / 1e9
    # end to end: the frame's scene constants in, the composited image out
    out_host = np.empty(4 * npx, np.float32)
    t = e2e_time(dev, ws, max(3, min(args.steps, 20)), [(w.bufs["P"], pinned_like(sc.P))], lambda: M.run(w.plan),
                 [(w.bufs["out"], out_host)])
    e2e = {"value": round(ws / t["seconds"], 1), "unit": "frames/s", "h2d_bytes_per_step": t["h2d_bytes_per_step"],
           "d2h_bytes_per_step": t["d2h_bytes_per_step"], "ms_per_step": round(t["seconds"] * 1e3, 3)}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        threads = O.max_threads()

        def one():
            lpos, cen, par = O.sc_move_lights(sc.centers, sc.params, sc.home, sc.lcol, sc.P, sc.first)
            vis = (np.nonzero(O.sc_cull(cen, sc.P[0:16]))[0] + 1).astype(np.uint32)
            svis = (np.nonzero(O.sc_cull(cen, sc.P[32:48]))[0] + 1).astype(np.uint32)
            smap, _, _ = O.raster_instances(sc.ppos, None, svis, svis.size, cen, sc.sizes, None, None, sc.P[32:48],
                                            1, sc.smap_res, sc.smap_res)
            dep, (alb, mat, nrm), _ = O.raster_instances(sc.ppos, sc.pnrm, vis, vis.size, cen, sc.sizes, sc.colors,
                                                         par, sc.P[0:16], 0, sc.w, sc.h)
            tl, tc = O.sc_tile_lights(dep, lpos, sc.P, sc.tile, sc.pertile)
            ao = O.sc_ao_blur(O.sc_ssao(dep, nrm, sc.P, sc.nsample), sc.P)
            hdr = O.sc_shade(alb, mat, nrm, dep, lpos, sc.lcol, tl, tc, smap, ao, sc.P, sc.tile, sc.pertile)
            bloom = O.sc_blur(O.sc_blur(O.sc_bright(hdr, sc.P, sc.shift), 1, 0), 0, 1)
            O.sc_composite(hdr, bloom, sc.P, sc.shift)
            return 1

        r = cpu_timed(one, args.steps, args.cpu_seconds, warm_s=0.0)
        cpu = {"value": round(r["units_per_s"], 3), "unit": "frames/s", "cores": threads, "kind": "port",
               "sample": f"{r['calls']} frames of the fifteen passes through the oracle (shading and occlusion on "
                         f"OpenMP, rasterisation and the rest one thread) in {r['seconds']:.1f} s"}
    return {
        "metric": METRIC, "value": round(ws * 1e3 / ms_step, 1), "unit": "frames/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded crystal field (bench/showcase.jl's generator restated, numpy PCG64)",
        "config": {"workload": "showcase frame (bench/showcase.jl): lights, cull x2, draw count, shadow and g-buffer "
                               "rasterisation, tiles, SSAO, AO blur, GGX lighting, bright, blur x/y, composite",
                   "resolution": [sc.w, sc.h], "lights": sc.home.shape[0], "instances": sc.centers.shape[0],
                   "shadow_map": sc.smap_res, "parallelism": f"{ws} independent frames",
                   "l2": "a frame's images (~70 MB) fit the L2; frames replay back to back (no flush)"},
        "roofline": {"bound": "hbm", "kernel": "the whole frame (15 passes)", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": None, "algorithmic_bytes": int(algo), "peak_kind": f"{peak_kind} (burst copy)"},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": w.plan.nkernels() * args.steps, "clocks": clk.summary(),
    }


def bench_independent(args, ws, rank, local, peaks, peak_kind):
    """bench/independent.jl: 8 independent chains of 6 stir! stages over 1 << 20
    floats, declared interleaved, replayed with derived barriers (per-resource
    graph edges: the chains run concurrently) and with :backend barriers (every
    pass chained, as Lava's per-dispatch barrier). The arms alternate in rounds
    after both are warm, as the reference measures them; each rank replays its
    own graph (weak scaling)."""
    import mantle_cuda as M
    from mantle_cuda.workloads import build_independent

    dev = M.Device(local)
    w = build_independent(dev)
    for mode in ("derived", "backend"):
        for _ in range(args.warmup):
            M.run(w.plan, barriers=mode)
    dev.synchronize()
    barrier(ws)
    rounds = 4
    per = max(1, args.steps // rounds)
    tot = {"derived": 0.0, "backend": 0.0}
    with ClockSampler(local) as clk:
        for _ in range(rounds):
            for mode in ("derived", "backend"):
                tot[mode] += device_time_flushed_ms(dev.stream, lambda m=mode: M.run(w.plan, barriers=m), per, local)
    ms = {m: max_over_ranks(ws, v / (rounds * per)) for m, v in tot.items()}
    value = ws * w.bytes_step / (ms["derived"] * 1e-3) / 1e9
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        from oracle import oracle as O
        srcs = w.inputs["sources"]

        def one():
            for c in range(w.chains):
                x = srcs[c]
                for _ in range(w.stages):
                    x = O.stir(x, w.k)
            return w.bytes_step

        r = cpu_timed(one, args.steps, args.cpu_seconds, warm_s=0.5)
        cpu = {"value": round(r["units_per_s"] / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{r['calls']} replays of the 48 stir! stages (oracle, one thread), {r['seconds']:.1f} s"}
    achieved = w.bytes_step / (ms["derived"] * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
        "steps": rounds * per, "warmup": args.warmup, "ms_per_step": round(ms["derived"], 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded PCG64, chain inputs U[-2,2]",
        "config": {"workload": "independent chains (bench/independent.jl): 8 chains x 6 stir! stages, 1 << 20 "
                               "floats, interleaved declaration", "n": w.n, "chains": w.chains, "stages": w.stages,
                   "ms_derived": round(ms["derived"], 5), "ms_backend": round(ms["backend"], 5),
                   "backend_over_derived": round(ms["backend"] / ms["derived"], 4),
                   "edges_derived": w.plan.nedges("derived"), "edges_backend": w.plan.nedges("backend"),
                   "l2": "L2 flushed between steps; the aliased intermediates (peak "
                         f"{M.peakbytes(w.plan) >> 20} MiB) stay in the L2 within a step"},
        "roofline": {"bound": "hbm", "kernel": "48 stir! launches in one graph (derived edges)",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "algorithmic_bytes": w.bytes_step, "peak_kind": f"{peak_kind} (burst copy)",
                     "note": "intermediates are L2-resident within a step, so the HBM fraction can exceed what "
                             "DRAM alone would allow"},
        "cpu_baseline": cpu,
        "e2e": None, "gpu_launches": w.plan.nkernels() * rounds * per * 2, "clocks": clk.summary(),
    }


SUB_KEYS = ("value", "unit", "ms_per_step", "scaling", "dtype", "data", "config", "roofline", "cpu_baseline",
            "e2e", "gpu_launches", "clocks")
WORKLOADS = {"scatter": bench_scatter, "chain": bench_chain, "fft": bench_fft, "gemm": bench_gemm,
             "cnn": bench_cnn, "showcase": bench_showcase, "independent": bench_independent}
ALL_ORDER = ("chain", "fft", "gemm", "cnn", "independent")


def profile_case(args, local):
    """Only the dominant kernel of a workload, three launches, for an ncu capture
    (`-k regex:<kernel> -c 3`); prints nothing but "ok"."""
    import torch

    import mantle_cuda as M
    dev = M.Device(local)
    s = dev.stream
    if args.profile == "scatter":
        from mantle_cuda.workloads import build_scatter
        w = build_scatter(dev)
        B = w.bufs
        for kargs in ((B["acc_a"], B["hist"], B["va"], B["ia"], w.nbins, 0),
                      (B["acc_b"], None, B["vb"], B["ib"], w.nbins, 0)):
            wsb = M.workspace_bytes(M.kernels.scatter_add, kargs, w.n)
            scratch = torch.empty(max(wsb, 16), dtype=torch.uint8, device=f"cuda:{local}")
            for _ in range(3):
                M.launch(M.kernels.scatter_add, kargs, w.n, stream=s, workspace=scratch)
    elif args.profile == "chain":
        from mantle_cuda.workloads import build_chain
        ws_ = [build_chain(dev, seed=k, fuse=True) for k in range(4)]
        for k in range(6):
            M.run(ws_[k % 4].plan)
    elif args.profile == "gemm":
        from mantle_cuda.workloads import build_gemm
        w = build_gemm(dev, batch=1)
        for _ in range(3):
            M.run(w.plan)
    elif args.profile == "cnn":
        from mantle_cuda.workloads import build_cnn
        w = build_cnn(dev, batch=args.profile_batch)
        for _ in range(3):
            M.run(w.plan)
    elif args.profile == "showcase":
        from mantle_cuda.workloads import build_showcase, crystal_scene
        w = build_showcase(dev, crystal_scene(1600, 900, seed=9, smap_res=2048))
        for _ in range(3):
            M.run(w.plan)
    elif args.profile == "fft":
        from mantle_cuda.workloads import build_fft
        w = build_fft(dev, batch=8192)
        for _ in range(3):
            M.launch(M.kernels.fft_c2c, (w.spectrum, w.x, w.n, 0), w.batch, stream=s)
    dev.synchronize()
    print("ok")


def reference_arm(args, ws, rank):
    """The CPU restatement of the same workloads on all host cores, timed the
    way the GPU arm's cpu_baseline legs are (`cpu_timed`)."""
    if rank != 0:
        return None
    n, nbins, nupd = 1 << 24, 1 << 16, 1 << 20
    inp = scatter_inputs(0, n, nbins, nupd)
    cpu = cpu_scatter(inp, nbins, args.steps, args.cpu_seconds)
    v = cpu["value"]
    line = {
        "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round((16 * n + 36 * nupd) / (v * 1e9) * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+i32", "impl": "reference",
        "data": SCATTER_DATA, "config": scatter_config(ws, n, nbins, nupd),
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


def run_workload(name, args, ws, rank, local, peaks, peak_kind):
    rec = WORKLOADS[name](args, ws, rank, local, peaks, peak_kind)
    release_device_memory(local)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", *WORKLOADS], default="all",
                    help="all (default): the scatter headline plus chain, fft, gemm and cnn records")
    ap.add_argument("--unfused", action="store_true", help="chain: time the unfused eight-kernel graph")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--profile-batch", type=int, default=64, help="--profile cnn: the batch (default 64)")
    ap.add_argument("--profile", choices=["scatter", "chain", "fft", "gemm", "cnn", "showcase"], default=None,
                    help="launch only the workload's dominant kernel three times (for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = reference_arm(args, ws, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if args.profile:
        profile_case(args, int(os.environ.get("LOCAL_RANK", "0")))
        return
    ws, rank, local = dist_init()
    peaks, peak_kind = load_peaks()
    try:
        if args.workload == "all":
            line = run_workload("scatter", args, ws, rank, local, peaks, peak_kind)
            subs = {}
            for name in ALL_ORDER:
                rec = run_workload(name, args, ws, rank, local, peaks, peak_kind)
                subs[name] = {k: rec[k] for k in SUB_KEYS if k in rec}
            line["workloads"] = subs
        else:
            line = run_workload(args.workload, args, ws, rank, local, peaks, peak_kind)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        finish(ws)


if __name__ == "__main__":
    main()
