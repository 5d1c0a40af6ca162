"""Benchmark of the B200 FFT path (batched 1D C2C, HBM GB/s).

Workload (the sweep config at its N=4096 point): batched 1D complex64
C2C FFT, N = 4096, batch = 65536 per GPU (2 GiB), re/im i.i.d. uniform[-1, 1)
from a seeded generator. ``--log-n L`` runs another point of the sweep
(single-pass sizes 2 <= L <= 14, batch = 2 GiB / N unless --batch is given). One step = one forward pass (x -> y) and one
inverse pass with 1/N (y -> z) through the C ABI on device-resident buffers.
The metric counts 16 bytes per complex element per pass (8 B read + 8 B
write): GB/s = 2 * 16 * N * batch * ranks / step time. Every buffer (2 GiB)
is larger than the 126 MB L2, so no L2 flush runs between steps.

Multi-GPU (torchrun): one process per GPU, each transforming its own batch
(weak scaling, no data-path collective); the timed region is bracketed by a
barrier and device syncs and the time is the max over ranks.

Arms:
  default            this build's sm_100a kernels
  --impl reference   the reference's CPU Stockham path, as restated in
                     oracle/ (the Rust reference cannot be built here), on
                     all host cores; rank 0 only.

Extra keys on the JSON line: roofline (dominant kernel, per-launch CUDA
events in the timed region vs the measured HBM copy bandwidth), cpu_baseline
(the oracle on a bounded sample), e2e (the public host-pointer API with
pinned buffers, copies inside the timed region), clocks (nvidia-smi sampled
during the timed region) and gpu_launches.
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "ferrum-gpu_b200"))
sys.path.insert(0, REPO)

METRIC = "batched 1D C2C FFT HBM GB/s"
METRIC_2D = "batched 2D C2C FFT HBM GB/s"
UNIT = "GB/s"
LOG_N = 12
BATCH = 65536
TOTAL_ELEMS = 1 << 28  # 2 GiB of complex64 per GPU
BYTES_PER_ELEM_PASS = 16
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=700)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the secondary measurements (other configs, 2D 16384^2)")
    ap.add_argument("--log-n", type=int, default=LOG_N, choices=range(2, 27),
                    help="log2 of the transform length (default 12: the headline N=4096; "
                         "15..26 run the multi-pass 1D path, 2D allows up to 14)")
    ap.add_argument("--kind", choices=["1d", "2d"], default="1d",
                    help="2d: the step is a forward + inverse 2D transform of --batch N x N "
                         "images (the 2D config); GB/s count 2 passes per transform")
    ap.add_argument("--batch", type=int, default=None,
                    help="transforms per GPU (default 2 GiB / N; smaller only for profiling)")
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the bench step: every 1D length 2^2..2^26 and every 2D size "
                         "64^2..16384^2 on 2 GiB, forward and inverse (1/N), min of 3 rounds of 10 "
                         "calls, with cuFFT on the same buffers and the error of one transform "
                         "against complex128; one GPU, one JSON line")
    args = ap.parse_args()
    if args.kind == "2d" and args.log_n > 14:
        ap.error("--kind 2d needs --log-n <= 14")
    if args.batch is None:
        args.batch = TOTAL_ELEMS >> (args.log_n * (2 if args.kind == "2d" else 1))
    return args


def elems_per_item(log_n: int, kind: str) -> int:
    return 1 << (log_n * (2 if kind == "2d" else 1))


def passes_counted(kind: str, log_n: int = 0) -> int:
    """Passes the metric counts per transform: 1 for single-pass 1D (N <= 2^14),
    2 for the multi-pass 1D lengths and for 2D, whatever the plan runs."""
    return 2 if (kind == "2d" or log_n > 14) else 1


def workload_config(log_n: int, batch: int, kind: str = "1d") -> dict:
    mib = batch * elems_per_item(log_n, kind) * 8 / 2**20
    n = 1 << log_n
    what = (f"batched 1D C2C forward+inverse(1/N), N={n}, batch={batch} per GPU"
            if kind == "1d" else
            f"batched 2D C2C forward+inverse(1/N^2), {n}x{n}, {batch} images per GPU")
    return {
        "workload": f"{what} ({mib / 1024:g} GiB complex64), one step = forward + inverse",
        "n": n,
        "batch_per_gpu": batch,
        "inputs": "re/im i.i.d. uniform[-1,1), seeded",
        "l2": (f"no flush: every buffer is {mib:g} MiB > 126 MB L2" if mib > 126 else
               f"L2-resident: buffers of {mib:g} MiB fit the 126 MB L2"),
        "bytes_counted": f"16 B per complex element per pass, {passes_counted(kind, log_n)} "
                         f"pass(es) per transform",
    }


def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(log_n: int, batch: int):
    """Per-launch DRAM bytes (read + write) of the dominant kernel, measured by
    ncu on the full-size launch (profiles/fft_rows_kernel_4096x65536_launches.md);
    None for workloads without such a capture."""
    if (log_n, batch) != (LOG_N, BATCH):
        return None
    path = os.path.join(REPO, "profiles", "fft_rows_kernel_4096x65536_launches.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except Exception:
        pass
    return None


# --------------------------------------------------------------------------
# CPU side (oracle) — test/baseline infrastructure only.

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def time_oracle(transforms: int, threads: int, log_n: int, seed: int = 0, kind: str = "1d"):
    """Forward + inverse (normalized) of `transforms` lanes (1D) or images (2D)
    with the oracle; returns (seconds, bytes counted)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(seed)
    n = 1 << log_n
    e = transforms * elems_per_item(log_n, kind)
    x = (rng.uniform(-1, 1, e) + 1j * rng.uniform(-1, 1, e)).astype(np.complex64)
    t0 = time.perf_counter()
    if kind == "1d":
        y = oracle.fft_1d(x, log_n, "forward", False, threads=threads)
        oracle.fft_1d(y, log_n, "inverse", True, threads=threads)
    else:
        x = x.reshape(transforms, n, n)
        y = oracle.fft_2d(x, log_n, "forward", False, threads=threads)
        oracle.fft_2d(y, log_n, "inverse", True, threads=threads)
    dt = time.perf_counter() - t0
    return dt, 2 * BYTES_PER_ELEM_PASS * passes_counted(kind, log_n) * e


def calibrate_oracle(threads: int, log_n: int, kind: str = "1d") -> float:
    """Seconds per transform (fwd + inv) of the oracle on `threads` threads."""
    probe = max(threads * 4, 64) if kind == "1d" else 1
    dt, _ = time_oracle(probe, threads, log_n, seed=1, kind=kind)
    return dt / probe


def cpu_baseline_leg(target_seconds: float, log_n: int, batch: int, kind: str = "1d") -> dict:
    threads = host_cores()
    per = calibrate_oracle(threads, log_n, kind)
    sample = max(threads if kind == "1d" else 1, int(target_seconds / max(per, 1e-9)))
    sample = min(sample, batch)
    dt, nbytes = time_oracle(sample, threads, log_n, seed=2, kind=kind)
    # Single-threaded, as the reference's CPU path runs (crates/ferrum-gpu-fft/src/cpu.rs:101):
    # a short sample of about a tenth of the target time.
    per1 = calibrate_oracle(1, log_n, kind) if kind == "1d" else per * threads
    sample1 = max(1, min(batch, int(0.1 * target_seconds / max(per1, 1e-9))))
    dt1, nbytes1 = time_oracle(sample1, 1, log_n, seed=3, kind=kind)
    return {
        "value": round(nbytes / dt / 1e9, 3),
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{sample} of the {batch} {kind} transforms (N={1 << log_n}), forward+inverse, "
                  f"lane-parallel oracle (C restatement of crates/ferrum-gpu-fft/src/cpu.rs) "
                  f"on {threads} threads, {cpu_model()}; {dt:.1f} s",
        "single_thread": {"value": round(nbytes1 / dt1 / 1e9, 3), "unit": UNIT, "cores": 1,
                          "sample": f"{sample1} transforms, forward+inverse, {dt1:.1f} s"},
    }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = host_cores()
    per = calibrate_oracle(threads, args.log_n, args.kind)
    budget = 90.0
    sample = int(budget / max(per, 1e-9) / max(1, args.steps + args.warmup))
    sample = max(threads if args.kind == "1d" else 1, min(sample, args.batch))
    for w in range(args.warmup):
        time_oracle(sample, threads, args.log_n, seed=100 + w, kind=args.kind)
    total_t = 0.0
    total_b = 0
    for k in range(args.steps):
        dt, nb = time_oracle(sample, threads, args.log_n, seed=200 + k, kind=args.kind)
        total_t += dt
        total_b += nb
    value = total_b / total_t / 1e9
    sample_desc = (f"{sample} of the {args.batch} {args.kind} transforms per step "
                   f"(N={1 << args.log_n}), "
                   f"forward+inverse(1/N), lane-parallel oracle port of "
                   f"crates/ferrum-gpu-fft/src/cpu.rs on {threads} threads, {cpu_model()}")
    line = {
        "impl": "reference",
        "metric": METRIC if args.kind == "1d" else METRIC_2D,
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_t / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args.log_n, args.batch, args.kind),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": sample_desc},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the Rust/cuda-oxide reference cannot be built in this image (no cargo, no "
                "network); its CPU Stockham path is timed through the C restatement in oracle/",
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU side.

class ClockSampler:
    """nvidia-smi samples every 50 ms; stop() keeps the samples whose
    timestamps fall inside [t_begin, t_end] (the timed region)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,"
             "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.t_begin = None
        self.t_end = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def mark_begin(self):
        self.t_begin = datetime.datetime.now()

    def mark_end(self):
        self.t_end = datetime.datetime.now()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for r in csv.reader(io.StringIO(out)):
            if len(r) < 11:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f")
                rows.append((ts, float(r[2]), float(r[3]), r))
            except ValueError:
                continue
        inside = [x for x in rows if self.t_begin and self.t_end and
                  self.t_begin <= x[0] <= self.t_end]
        use = inside or rows
        reasons = set()
        for _, _, _, r in use:
            for name, v in zip(self.REASONS, r[7:11]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(x[1] for x in use) if use else None,
                "sm_max_mhz": use[-1][2] if use else None,
                "reasons": sorted(reasons),
                "samples": len(rows), "samples_in_timed_region": len(inside),
                "window": "timed region" if inside else "whole run (timed region shorter than "
                                                         "one sample)"}


def _time_ms(fn, stream, reps: int = 5, warm: int = 2) -> float:
    """Mean CUDA-event time of `fn` on `stream` over `reps` calls."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b) / reps


def _cufft_fns(x, y, batch: int, log_n: int, kind: str):
    """Forward and inverse (1/N) cuFFT calls through torch.fft on the same
    device buffers: the reference's yardstick (its bench states every result
    as a ratio to cuFFT on identical buffers), never part of the product."""
    import torch

    n = 1 << log_n
    if kind == "1d":
        xv = x[: batch * n].view(batch, n)
        yv = y[: batch * n].view(batch, n)
        return (lambda: torch.fft.fft(xv, dim=-1, out=yv),
                lambda: torch.fft.ifft(yv, dim=-1, out=xv))
    xv = x[: batch * n * n].view(batch, n, n)
    yv = y[: batch * n * n].view(batch, n, n)
    return (lambda: torch.fft.fft2(xv, out=yv), lambda: torch.fft.ifft2(yv, out=xv))


def measure_extras(capi, dev, x, y, world, rank, barrier, max_over_ranks) -> dict:
    """Secondary measurements on the same device buffers (2^28 complex each):
    BASELINE config 1 (N=1024 x 256, L2-resident), the sweep sizes, the
    large-N multi-pass sizes, 2D 4096^2 x 16 and the 16384^2 2D transform
    (single GPU at N=1, distributed at N>1), each forward and inverse (1/N),
    with cuFFT on the same buffers as a yardstick (`cufft_*_ms`,
    `vs_cufft` = cuFFT time / ours, > 1 when ours is faster). GB/s count 16 B
    per element per pass (1 pass for N <= 2^14, 2 for the multi-pass 1D and
    2D). The inputs of every timed config except config 1 exceed the L2."""
    import torch

    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    total = x.numel()
    out = {}

    def gbs(passes, elems, ms):
        return round(world * passes * 16 * elems / (ms * 1e-3) / 1e9, 1)

    def one(key, log_n, batch, kind, reps=5, cufft=True):
        fft = capi.fft_1d if kind == "1d" else capi.fft_2d
        elems = batch << (log_n * (2 if kind == "2d" else 1))
        passes = passes_counted(kind, log_n)
        ms_f = max_over_ranks(_time_ms(lambda: fft(dev, x.data_ptr(), y.data_ptr(), log_n, batch,
                                                   "forward", False, sp), stream, reps))
        ms_i = max_over_ranks(_time_ms(lambda: fft(dev, y.data_ptr(), x.data_ptr(), log_n, batch,
                                                   "inverse", True, sp), stream, reps))
        rec = {"ms": round(ms_f, 4), "GB/s": gbs(passes, elems, ms_f),
               "inverse_ms": round(ms_i, 4), "inverse_GB/s": gbs(passes, elems, ms_i)}
        if cufft:
            cf, ci = _cufft_fns(x, y, batch, log_n, kind)
            try:
                c_f = max_over_ranks(_time_ms(cf, stream, reps))
                c_i = max_over_ranks(_time_ms(ci, stream, reps))
                rec.update({"cufft_ms": round(c_f, 4), "cufft_inverse_ms": round(c_i, 4),
                            "vs_cufft": round(c_f / ms_f, 3),
                            "vs_cufft_inverse": round(c_i / ms_i, 3)})
            except Exception as e:  # yardstick only: never fail the bench over it
                rec["cufft"] = f"unavailable: {type(e).__name__}: {e}"
            # cuFFT's inverse wrote x: restore a well-scaled input for the next config
            torch.cuda.synchronize()
        out[key] = rec

    one("config1_1d_N1024_x256_L2_resident", 10, 256, "1d", reps=200)
    for log_n in (8, 10, 12, 14):
        one(f"1d_N{1 << log_n}_x{total >> log_n}", log_n, total >> log_n, "1d")
    for log_n, batch in ((20, 64), (24, 4)):
        one(f"1d_N2^{log_n}_x{batch}", log_n, batch, "1d")
    one("2d_4096^2_x16", 12, 16, "2d")

    n = 1 << 14
    if world == 1:
        one("2d_16384^2", 14, 1, "2d")
        capi.fft_2d(dev, x.data_ptr(), y.data_ptr(), 14, 1, "forward", False, sp)
        z = torch.empty(n * n, dtype=x.dtype, device=x.device)
        capi.fft_2d(dev, y.data_ptr(), z.data_ptr(), 14, 1, "inverse", True, sp)
        torch.cuda.synchronize()
        xs = x[: n * n]
        out["2d_16384^2"]["path"] = "single GPU (column passes + row pass)"
        out["2d_16384^2"]["roundtrip_max_rel_err"] = float((z - xs).abs().max() / xs.abs().max())
        del z
    else:
        from ferrum_gpu.dist import Dist2D

        # Set-up (slab allocation, IPC mapping) happens in the first call,
        # under a generous bound; the timed calls' peer barriers then give up
        # after 5 s instead of spinning on a lost peer.
        ctx = Dist2D(dev, timeout_ms=60000)
        rows = n // world
        xs = x[: rows * n]
        ys = y[: rows * n]
        zs = torch.empty_like(xs)
        barrier()
        ctx.fft_2d(xs.data_ptr(), ys.data_ptr(), 14, "forward", False, sp, "rows", "cols")
        ctx.sync(sp)
        ctx.set_timeout(5000)
        barrier()
        # Forward: row slabs -> column slabs (row FFTs, one all-to-all
        # exchange, column FFTs); inverse: column slabs -> row slabs.
        ms_f = max_over_ranks(_time_ms(lambda: ctx.fft_2d(xs.data_ptr(), ys.data_ptr(), 14,
                                                          "forward", False, sp, "rows", "cols"),
                                       stream, 20))
        ms_i = max_over_ranks(_time_ms(lambda: ctx.fft_2d(ys.data_ptr(), zs.data_ptr(), 14,
                                                          "inverse", True, sp, "cols", "rows"),
                                       stream, 20))
        ms_rr = max_over_ranks(_time_ms(lambda: ctx.fft_2d(xs.data_ptr(), ys.data_ptr(), 14,
                                                           "forward", False, sp, "rows", "rows"),
                                        stream, 20))
        ctx.fft_2d(xs.data_ptr(), ys.data_ptr(), 14, "forward", False, sp, "rows", "cols")
        ctx.fft_2d(ys.data_ptr(), zs.data_ptr(), 14, "inverse", True, sp, "cols", "rows")
        ctx.sync(sp)
        err = max_over_ranks(float((zs - xs).abs().max() / xs.abs().max()))
        barrier()
        peer = ctx.peer_path == 1
        ctx.close()
        slab_bytes = rows * n * 8
        out["2d_16384^2"] = {"ms": round(ms_f, 4), "inverse_ms": round(ms_i, 4),
                             "GB/s": gbs(2, n * n // world, ms_f),
                             "rows_to_rows_fwd_ms": round(ms_rr, 4),
                             "data_path": "peer memory (exchange fused into the FFT kernels)"
                             if peer else "NCCL send/recv",
                             "nvlink_bytes_per_rank_each_way": (world - 1) * slab_bytes // world,
                             "path": f"distributed over {world} GPUs: row slabs -> column "
                                     f"slabs (one all-to-all exchange); inverse column -> "
                                     f"row slabs",
                             "roundtrip_max_rel_err": err}
    return out


def measure_sustained(capi, dev, x, y, z, log_n, batch, local, seconds=1.2) -> dict:
    """The headline step (forward + inverse) repeated for about `seconds` of
    GPU time with its own clock samples: the throughput a caller running
    FFTs for seconds sees under the 1 kW power cap."""
    import torch

    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step():
        capi.fft_1d(dev, x.data_ptr(), y.data_ptr(), log_n, batch, "forward", False, sp)
        capi.fft_1d(dev, y.data_ptr(), z.data_ptr(), log_n, batch, "inverse", True, sp)

    per = _time_ms(step, stream, reps=5, warm=2)
    steps = max(10, int(seconds * 1e3 / max(per, 1e-3)))
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    sampler.mark_begin()
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    b.synchronize()
    sampler.mark_end()
    clocks = sampler.stop()
    ms = a.elapsed_time(b)
    elems = batch << log_n
    return {"steps": steps, "ms_per_step": round(ms / steps, 4), "seconds": round(ms * 1e-3, 3),
            "GB/s": round(steps * 2 * 16 * elems / (ms * 1e-3) / 1e9, 1), "clocks": clocks}


def rows_kernel_name(log_n: int) -> str:
    """The single-pass kernel the library launches for length 2^log_n (the
    radix plan gives 32 values per thread from N = 8192, 16 below)."""
    lp = log_n if log_n < 4 else (5 if log_n >= 13 else 4)
    name = "fft_rows_pf_kernel" if log_n == 14 else "fft_rows_kernel"
    return f"{name}<{log_n},{lp},*,*,*> (single-pass N={1 << log_n})"


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from ferrum_gpu import capi

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    B_ = args.batch
    L = args.log_n
    kind = args.kind
    dev = capi.DeviceHandle(local)
    n = 1 << L
    per_item = elems_per_item(L, kind)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    x = torch.complex(torch.rand(B_, per_item, device="cuda", generator=g) * 2 - 1,
                      torch.rand(B_, per_item, device="cuda", generator=g) * 2 - 1)
    y = torch.empty_like(x)
    z = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    launches_per_step = 2 * capi.launch_count(L, B_, 1 if kind == "1d" else 2)
    fft = capi.fft_1d if kind == "1d" else capi.fft_2d
    fft_host = capi.fft_1d_host if kind == "1d" else capi.fft_2d_host

    def step(events=None):
        if events is not None:
            events[0].record(stream)
        fft(dev, x.data_ptr(), y.data_ptr(), L, B_, "forward", False, sp)
        if events is not None:
            events[1].record(stream)
            events[2].record(stream)
        fft(dev, y.data_ptr(), z.data_ptr(), L, B_, "inverse", True, sp)
        if events is not None:
            events[3].record(stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # correctness gate on the measured buffers: inverse(forward(x)) == x
    err = float((z - x).abs().max() / x.abs().max())
    if err > 1e-4:
        raise SystemExit(f"round-trip error {err} exceeds 1e-4; refusing to report")

    per_launch = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
                  for _ in range(args.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    barrier()
    torch.cuda.synchronize()
    sampler.mark_begin()
    start.record(stream)
    for k in range(args.steps):
        step(per_launch[k])
    end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    barrier()
    clocks = sampler.stop()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    launch_ms = [ev[0].elapsed_time(ev[1]) for ev in per_launch] + \
                [ev[2].elapsed_time(ev[3]) for ev in per_launch]
    avg_launch_ms = max_over_ranks(sum(launch_ms) / len(launch_ms))

    # Algorithmic bytes of one transform (forward or inverse): 16 B per element
    # per counted pass.
    bytes_per_pass = BYTES_PER_ELEM_PASS * per_item * B_ * passes_counted(kind, L)
    value = world * args.steps * 2 * bytes_per_pass / (elapsed_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    achieved = bytes_per_pass / (avg_launch_ms * 1e-3) / 1e9
    traffic = profiled_traffic(L, B_) if kind == "1d" else None

    # End to end through the public host-pointer API with pinned buffers.
    e2e = None
    if not args.no_e2e:
        hx = x.cpu().pin_memory()
        hy = torch.empty_like(hx).pin_memory()
        hz = torch.empty_like(hx).pin_memory()
        fft_host(dev, hx.data_ptr(), hy.data_ptr(), L, B_, "forward", False)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            fft_host(dev, hx.data_ptr(), hy.data_ptr(), L, B_, "forward", False)
            fft_host(dev, hy.data_ptr(), hz.data_ptr(), L, B_, "inverse", True)
        t_e2e = max_over_ranks(time.perf_counter() - t0)
        barrier()
        e2e_err = float((hz - hx).abs().max() / hx.abs().max())
        if e2e_err > 1e-4:
            raise SystemExit(f"e2e round-trip error {e2e_err} exceeds 1e-4")
        e2e = {"value": round(world * args.e2e_steps * 2 * bytes_per_pass / t_e2e / 1e9, 3),
               "unit": UNIT,
               "h2d_bytes_per_step": 2 * 8 * per_item * B_,
               "d2h_bytes_per_step": 2 * 8 * per_item * B_,
               "steps": args.e2e_steps,
               "path": f"ferrum_fft_{kind}_c2c_pow2_host (C ABI), pinned host buffers, "
                       f"forward + inverse"}

    extras = None
    if not args.no_extras and (kind, L, B_) == ("1d", LOG_N, BATCH):
        sustained = measure_sustained(capi, dev, x, y, z, L, B_, local)
        extras = measure_extras(capi, dev, x.view(-1), y.view(-1), world, rank, barrier,
                                max_over_ranks)
        extras["sustained"] = sustained

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(args.cpu_seconds, L, B_, kind)

    if rank == 0:
        line = {
            "metric": METRIC if kind == "1d" else METRIC_2D,
            "value": round(value, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": workload_config(L, B_, kind),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 2),
            "transforms_per_s": round(world * args.steps * 2 * B_ / (elapsed_ms * 1e-3), 1),
            "nominal_gflops": round(world * args.steps * 2 * 5 * per_item * L
                                    * (2 if kind == "2d" else 1) * B_ / (elapsed_ms * 1e-3) / 1e9,
                                    1),
            "roofline": {
                "bound": "hbm",
                "kernel": rows_kernel_name(L) if (kind == "1d" and L <= 14) else
                f"whole {kind.upper()} N=2^{L} transform ({launches_per_step // 2} kernels), "
                f"timed per transform",
                "achieved": round(achieved, 2),
                "peak": peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind ==
                "measured" else "fallback 6.65 TB/s",
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": traffic,
                "algorithmic_bytes_per_launch": bytes_per_pass,
                "avg_launch_ms": round(avg_launch_ms, 5),
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks,
            "gpu_launches": args.steps * launches_per_step,
            "secondary": extras,
            "roundtrip_max_rel_err": err,
        }
        print(json.dumps(line), flush=True)
    dev.close()
    if world > 1:
        dist.destroy_process_group()


def run_sweep(args) -> None:
    """The full-range table: one GPU, 2^28 complex values per buffer. GB/s count
    16 B per element per pass, 1 pass up to 2^14 and 2 beyond and for 2D."""
    import torch

    from ferrum_gpu import capi

    torch.cuda.set_device(0)
    dev = capi.DeviceHandle(0)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.complex(torch.rand(TOTAL_ELEMS, device="cuda", generator=g) * 2 - 1,
                      torch.rand(TOTAL_ELEMS, device="cuda", generator=g) * 2 - 1)
    y = torch.empty_like(x)
    out = {}
    for kind, sizes in (("1d", range(2, 27)), ("2d", range(6, 15))):
        fft = capi.fft_1d if kind == "1d" else capi.fft_2d
        for log_n in sizes:
            n = 1 << log_n
            batch = TOTAL_ELEMS // elems_per_item(log_n, kind)
            fwd = lambda: fft(dev, x.data_ptr(), y.data_ptr(), log_n, batch, "forward", False, sp)
            inv = lambda: fft(dev, y.data_ptr(), x.data_ptr(), log_n, batch, "inverse", True, sp)
            f = min(_time_ms(fwd, stream, 10, 3) for _ in range(3))
            i = min(_time_ms(inv, stream, 10, 3) for _ in range(3))
            fwd()
            m = n * n if kind == "2d" else n
            xs = x[:m].to(torch.complex128)
            ref = torch.fft.fft2(xs.view(n, n)).reshape(-1) if kind == "2d" else torch.fft.fft(xs)
            err = float((y[:m].to(torch.complex128) - ref).abs().max() / ref.abs().max())
            del xs, ref
            cf, ci = _cufft_fns(x, y, batch, log_n, kind)
            c_f = _time_ms(cf, stream, 10, 3)
            c_i = _time_ms(ci, stream, 10, 3)  # wrote x: a well-scaled input for the next size
            passes = passes_counted(kind, log_n)
            gbs = lambda ms: round(passes * 16 * TOTAL_ELEMS / (ms * 1e-3) / 1e9, 1)
            rec = {"batch": batch, "ms": round(f, 4), "inverse_ms": round(i, 4), "GB/s": gbs(f),
                   "inverse_GB/s": gbs(i), "cufft_ms": round(c_f, 4), "cufft_inverse_ms": round(c_i, 4),
                   "vs_cufft": round(c_f / f, 3), "vs_cufft_inverse": round(c_i / i, 3),
                   "max_rel_err_vs_complex128": err}
            out[f"{kind}_2^{log_n}"] = rec
            print(f"{kind} 2^{log_n:2d} x{batch:<9d} {f:.4f} / {i:.4f} ms  {rec['GB/s']:7.1f} / "
                  f"{rec['inverse_GB/s']:7.1f} GB/s  vs cuFFT {rec['vs_cufft']:.2f} / "
                  f"{rec['vs_cufft_inverse']:.2f}  err {err:.1e}", file=sys.stderr, flush=True)
    print(json.dumps({"sweep": out, "unit": "GB/s", "data": "synthetic uniform[-1,1)",
                      "bytes_per_buffer": TOTAL_ELEMS * 8}))


def main():
    args = parse_args()
    if args.sweep:
        run_sweep(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
