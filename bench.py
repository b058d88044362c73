"""Benchmark of the FP32 attention hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload (the headline): the 32-wide flash forward,
B=8 H=3 S=1024 d=32 per GPU, no mask, global attention, synthetic N(0,1) inputs from a seeded
torch generator. A step is one call of ``attention_fp32_forward_flash`` through the C ABI.
With N GPUs (torchrun) every rank runs its own B=8 batch slice of a global batch of 8N
sequences (weak scaling; (batch, head) slices are independent, so there is no collective on
the data path) and the reported value is all ranks' FLOPs over the slowest rank's time.

Timing: W untimed steps, then K steps; before each step a 256 MiB buffer is written to flush
the 126 MB L2, and the step itself is bracketed by CUDA events on the launching stream (the
flush is outside the events). Device time is summed over the K steps; the max over ranks is
taken with an all-reduce. FLOPs follow the reference's convention (4*B*H*Q*K*d forward,
AttentionBenchmarks.cpp:141-142).

Also reported: ``e2e`` (the same step through the public C entry point with pinned host
buffers: H2D of q/k/v/mask and D2H of O/lse inside the timed region), ``roofline`` of the
flash kernel, ``cpu_baseline`` (rank 0, N=1: the CPU oracle timed on this box's host cores),
``clocks`` sampled with nvidia-smi during the timed region, and ``gpu_launches``.

``--impl reference`` times the reference's own CPU attention (ReferenceAttention compiled from
its source into oracle/_ref, else the C restatement) on rank 0 with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

WORKLOADS = {
    # name: (batch per GPU, heads, seq, head_dim, description)
    "flash_fwd_b8h3s1024d32": (8, 3, 1024, 32, "BASELINE configs[1]: 32-wide flash forward B8 H3 S1024 d32, no mask, global"),
}
DEFAULT_WORKLOAD = "flash_fwd_b8h3s1024d32"
PUBLISHED_TFLOPS = 3.36  # flash fwd d32, same FLOPs (B2 H12 L1024), RX 6700 (README.md:63)
METRIC = "FP32 attention TFLOP/s (repo FLOP convention: 4*B*H*Q*K*d forward, 8*B*H*Q*K*d backward)"


def workload_config(name: str, world: int) -> dict:
    batch, heads, seq, dim, description = WORKLOADS[name]
    return {"workload": name, "description": description, "batch_per_gpu": batch, "global_batch": batch * world,
            "heads": heads, "seq_len": seq, "head_dim": dim, "mask": "all visible", "radius": -1,
            "parallelism": f"batch-sharded x{world}, no collective", "l2": "flushed (256 MiB write) before every step"}
FLUSH_BYTES = 256 << 20


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.process = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.TemporaryFile(mode="w+")
            self.process = subprocess.Popen(["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.QUERY}",
                                             "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.file,
                                            stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.process = None

    def stop(self) -> dict:
        if self.process is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.process.terminate()
        try:
            self.process.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
        self.file.seek(0)
        rows = [[c.strip() for c in line.split(",")] for line in self.file.read().splitlines() if line.strip()]
        sm, sm_max, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in rows:
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                sm_max.append(float(row[2]))
            except ValueError:
                continue
            for name, flag in zip(names, row[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(workload) -> dict:
    """The oracle (C restatement, forward only) on this host's cores over the full workload."""
    from oracle import oracle

    batch, heads, seq, dim, _ = workload
    threads = oracle.cpu_count()
    q = oracle.normal(batch * heads * seq * dim, 101).reshape(batch, heads, seq, dim)
    k = oracle.normal(batch * heads * seq * dim, 102).reshape(batch, heads, seq, dim)
    v = oracle.normal(batch * heads * seq * dim, 103).reshape(batch, heads, seq, dim)
    mask = __import__("numpy").ones((batch, seq), dtype="uint8")
    flops = 4.0 * batch * heads * seq * seq * dim
    reps, elapsed = 0, 0.0
    while elapsed < 10.0 and reps < 50:
        start = time.perf_counter()
        oracle.attention(q, k, v, mask, None, -1, threads=threads, forward_only=True)
        elapsed += time.perf_counter() - start
        reps += 1
    return {"value": flops * reps / elapsed / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"oracle/attention_oracle.c forward (double accumulation, as ReferenceAttention) over the full "
                      f"workload x{reps}, {elapsed:.1f} s on {threads} threads"}


def run_reference(args, rank: int) -> None:
    """--impl reference: the reference's CPU attention on rank 0; other ranks exit without work."""
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle

    batch, heads, seq, dim, description = WORKLOADS[args.workload]
    threads = oracle.cpu_count()
    use_ref = oracle.reference_available()
    q = oracle.normal(threads * seq * dim, 101).reshape(threads, 1, seq, dim)
    k = oracle.normal(threads * seq * dim, 102).reshape(threads, 1, seq, dim)
    v = oracle.normal(threads * seq * dim, 103).reshape(threads, 1, seq, dim)
    u = oracle.normal(threads * seq * dim, 104).reshape(threads, 1, seq, dim)
    mask = np.ones((1, seq), np.uint8)

    def one_slice(i):
        if use_ref:
            oracle.reference_attention(q[i:i + 1], k[i:i + 1], v[i:i + 1], mask, u[i:i + 1], -1)
        else:
            oracle.attention(q[i:i + 1], k[i:i + 1], v[i:i + 1], mask, u[i:i + 1], -1, threads=1)

    def step():
        workers = [threading.Thread(target=one_slice, args=(i,)) for i in range(threads)]
        for w in workers:
            w.start()
        for w in workers:
            w.join()

    for _ in range(args.warmup):
        step()
    start = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - start
    flops = 12.0 * threads * seq * seq * dim * args.steps  # forward (4) + backward (8) per pair: it computes both
    value = flops / elapsed / 1e12
    kind = "reference" if use_ref else "port"
    sample = (f"{'ReferenceAttention (AttentionTests.cpp:28-125, compiled from the reference source)' if use_ref else 'oracle port'}"
              f" forward+backward of {threads} (batch, head) slices S={seq} d={dim} per step, one slice per thread;"
              f" FLOPs counted as 12*S*S*d per slice (the function always computes forward and backward)")
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64-accumulate/f32-storage", "data": "synthetic N(0,1), seeded",
            "config": workload_config(args.workload, args.gpus), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def traffic_from_profiles(kernel_tag: str):
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    entry = data.get(kernel_tag)
    return None if entry is None else entry.get("dram_bytes_per_launch")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    parser.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle leg")
    args = parser.parse_args()

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    import rocmkernels_b200.attention as api

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    batch, heads, seq, dim, description = WORKLOADS[args.workload]
    generator = torch.Generator(device=device)
    generator.manual_seed(101 + rank)
    q = torch.randn(batch, heads, seq, dim, device=device, generator=generator)
    k = torch.randn(batch, heads, seq, dim, device=device, generator=generator)
    v = torch.randn(batch, heads, seq, dim, device=device, generator=generator)
    mask = torch.ones(batch, seq, dtype=torch.uint8, device=device)
    out = torch.empty_like(q)
    lse = torch.empty(batch, heads, seq, 2, device=device)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    qs, ks, vs, os_ = (api.strides_of(t) for t in (q, k, v, out))
    flops_per_step = 4.0 * batch * heads * seq * seq * dim

    def step_device():
        status = api.attention_fp32_forward_flash(q, k, v, mask, out, lse, batch, heads, seq, seq, -1, qs, ks, vs, os_, stream)
        if status != 0:
            raise api.HipError(status, "attention_fp32_forward_flash")

    # Host-buffer leg: pinned inputs copied in and outputs copied out every step.
    host_q, host_k, host_v = (t.cpu().pin_memory() for t in (q, k, v))
    host_mask = mask.cpu().pin_memory()
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    host_lse = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()
    h2d_bytes = sum(t.numel() * t.element_size() for t in (host_q, host_k, host_v, host_mask))
    d2h_bytes = host_out.numel() * 4 + host_lse.numel() * 4

    def step_e2e():
        q.copy_(host_q, non_blocking=True)
        k.copy_(host_k, non_blocking=True)
        v.copy_(host_v, non_blocking=True)
        mask.copy_(host_mask, non_blocking=True)
        step_device()
        host_out.copy_(out, non_blocking=True)
        host_lse.copy_(lse, non_blocking=True)

    def timed(fn, steps):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        for i in range(steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            fn()
            ends[i].record(stream)
        torch.cuda.synchronize(device)
        return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3  # seconds

    for _ in range(args.warmup):
        flush.fill_(0.0)
        step_device()
    torch.cuda.synchronize(device)

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    sampler = ClockSampler(visible.split(",")[local_rank].strip() if visible else str(local_rank))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    device_seconds = timed(step_device, args.steps)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if rank == 0 else None

    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    torch.cuda.synchronize(device)
    e2e_steps = max(1, min(args.steps, 50))
    e2e_seconds = timed(step_e2e, e2e_steps)

    times = torch.tensor([device_seconds, e2e_seconds], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    device_seconds, e2e_seconds = times.tolist()

    value = world * flops_per_step * args.steps / device_seconds / 1e12
    e2e_value = world * flops_per_step * e2e_steps / e2e_seconds / 1e12
    kernel_seconds = device_seconds / args.steps
    achieved = flops_per_step / kernel_seconds / 1e12
    peaks, peak_source = measured_peaks()
    path = api.flash_kernel_name(batch, heads, seq, seq, dim)
    if path.startswith("tcgen05"):
        peak = float(peaks["bf16_tflops"])
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic_from_profiles(path),
                    "peak_source": f"{peak_source} bf16_tflops (burst); the TF32 dense rate is half of it",
                    "frac_of_tf32_dense": achieved / (peak / 2), "kernel": path}
    else:
        sm_mhz = (clocks or {}).get("sm_mhz") or float(peaks.get("sm_max_mhz", 1965.0))
        peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        roofline = {"bound": "fp32-fma", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic_from_profiles(path),
                    "peak_source": "148 SMs x 128 FP32 lanes x 2 FLOP x median SM clock under load",
                    "kernel": path}

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": device_seconds / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": value / PUBLISHED_TFLOPS,
        "dtype": "f32",
        "data": "synthetic N(0,1) from a seeded torch generator (rank-dependent seed)",
        "config": workload_config(args.workload, world),
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                "steps": e2e_steps},
        "roofline": roofline,
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(WORKLOADS[args.workload])
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
