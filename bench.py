"""Benchmark of the FP32 attention hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload (the headline): the 32-wide flash forward,
B=8 H=3 S=1024 d=32 per GPU, no mask, global attention, synthetic N(0,1) inputs from a seeded
torch generator. A step is one call of ``attention_fp32_forward_flash`` through the C ABI.
With N GPUs (torchrun) every rank runs its own B=8 batch slice of a global batch of 8N
sequences (weak scaling; (batch, head) slices are independent, so there is no collective on
the data path) and the reported value is all ranks' FLOPs over the slowest rank's time.

The other BASELINE configs are opt-in workloads (``--workload``): forward + backward steps
(``attention_fp32_forward_flash`` or ``attention64_fp32_forward``, then the matching backward)
on a fixed global problem whose batch is split over the ranks (strong scaling), with the
BASELINE key-padding lengths (seed 105) and radius. They report the repo-convention TFLOP/s
(12*B*H*Q*K*d per step) as ``value``, the effective TFLOP/s over active (query, key) pairs, and
the forward and backward times separately. The ``generic_*`` workloads are the reference's
AttentionGeneric benchmark cases (AttentionGenericBenchmarks.cpp:14-18, 100-110: B2 H8 L512,
d = 16/32/64, fp32 or fp16 storage): a step is one ``attention_generic_forward`` call, per GPU
(weak scaling), 4*B*H*Q*K*d FLOPs (the reference's operation count, :96). ``rotary_*`` are the
reference's Rotary benchmark cases (RotaryBenchmarks.cpp:75-76: B2 H12 L1024, token-major q and
k, 0.5-valued inputs): one ``rotary_fp32`` call per step, GB/s over the reference's byte count
(4 x elements x 4 B, :68). ``flash_rotary_fwd_b8h3s1024d32`` is the headline forward with the
rotary prologue fused in (``attention_fp32_forward_flash_rotary``); its line also carries the
time of the unfused sequence (``rotary_fp32`` then ``attention_fp32_forward_flash``).

Timing: W untimed steps, then K steps. Forward-only workloads use inputs larger than L2: the
steps rotate through copies of the input set totalling at least twice the 126 MB L2 (each step's
inputs were last touched a whole rotation earlier), run back to back on the launching stream, and
one CUDA event pair brackets the K steps; the line also carries the per-step-flushed figure
(``flushed``: a 256 MiB write before every step, events around each step, summed). Forward +
backward workloads flush before every step and bracket each phase with events. The max over ranks
is taken with an all-reduce. FLOPs follow the reference's convention (4*B*H*Q*K*d forward,
8*B*H*Q*K*d backward, AttentionBenchmarks.cpp:141-142).

Also reported: ``e2e`` (the same step through the public C entry points with pinned host
buffers: every step copies all its inputs in and all its outputs back inside the timed region,
pipelined as a serving loop runs it -- step i's H2D copies, kernels and D2H copies on a copy-in,
a compute and a copy-out stream, overlapping the neighbouring steps, with two device buffer sets
alternating; the time runs from the first H2D to the last D2H), ``roofline`` of the
dominant kernel, ``cpu_baseline`` (rank 0, N=1: the CPU oracle timed on this box's host cores),
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
    # batch: per GPU (weak scaling) for the forward headline, global (split over ranks) for the
    # forward + backward configs; lengths: per-sequence visible keys drawn U[lo, hi] (seed 105),
    # or "c1" (batch 1 keys 112..127 masked), or None (all visible).
    "flash_fwd_b8h3s1024d32": dict(batch=8, heads=3, seq=1024, dim=32, radius=-1, lengths=None, backward=False,
                                   description="BASELINE configs[1]: 32-wide flash forward B8 H3 S1024 d32, no mask, global"),
    "c1_fwd_bwd_b2h12s128d32": dict(batch=2, heads=12, seq=128, dim=32, radius=-1, lengths="c1", backward=True,
                                    description="BASELINE configs[0]: forward+backward B2 H12 S128 d32, batch 1 keys 112..127 masked"),
    "c3_fwd_bwd_b8h6s1024d64": dict(batch=8, heads=6, seq=1024, dim=64, radius=-1, lengths=(512, 1024), backward=True,
                                    description="BASELINE configs[2]: 64-wide forward+backward B8 H6 S1024 d64, lengths U[512,1024]"),
    "c4_fwd_bwd_b16h12s2048d32r128": dict(batch=16, heads=12, seq=2048, dim=32, radius=128, lengths=(1024, 2048), backward=True,
                                          description="BASELINE configs[3]: local radius 128 forward+backward B16 H12 S2048 d32, "
                                                      "lengths U[1024,2048]"),
    "c5_fwd_bwd_b64h12s4096d32": dict(batch=64, heads=12, seq=4096, dim=32, radius=-1, lengths=None, backward=True,
                                      description="BASELINE configs[4]: forward+backward B64 H12 S4096 d32, full attention"),
    "simt_fwd_b8h3s1024d32": dict(batch=8, heads=3, seq=1024, dim=32, radius=-1, lengths=None, backward=False,
                                  entry="attention_fp32_forward",
                                  description="the headline shape through attention_fp32_forward: the exact-FP32 SIMT kernel "
                                              "(for the tensor-core vs SIMT comparison)"),
    "fwd_bwd_b4h12s4096d32": dict(batch=4, heads=12, seq=4096, dim=32, radius=-1, lengths=None, backward=True,
                                  description="profiling case: C5's shape at B=4 (inputs above L2, a few hundred MB)"),
    "c5_fused_fwd_bwd_b64h12s4096d32": dict(batch=64, heads=12, seq=4096, dim=32, radius=-1, lengths=None, backward=True,
                                            backward_entry="attention_fp32_backward_fused",
                                            description="BASELINE configs[4] with the fused single-pass backward "
                                                        "(attention_fp32_backward_fused)"),
    "fused_fwd_bwd_b4h12s4096d32": dict(batch=4, heads=12, seq=4096, dim=32, radius=-1, lengths=None, backward=True,
                                        backward_entry="attention_fp32_backward_fused",
                                        description="profiling case of the fused single-pass backward: C5's shape at B=4"),
}
WORKLOADS["flash_rotary_fwd_b8h3s1024d32"] = dict(
        batch=8, heads=3, seq=1024, dim=32, radius=-1, lengths=None, backward=False, rotary=True,
        description="headline flash forward B8 H3 S1024 d32 with the rotary prologue fused (attention_fp32_forward_flash_rotary)")
for _direction in ("fwd", "bwd"):
    WORKLOADS[f"rotary_{_direction}_b2h12l1024"] = dict(
            batch=2, heads=12, seq=1024, dim=32, radius=-1, lengths=None, backward=_direction == "bwd", kind="rotary",
            description=f"Rotary {'backward' if _direction == 'bwd' else 'forward'} b2 h12 l1024 (RotaryBenchmarks.cpp:75-76), "
                        f"rotary_fp32")
for _width in (16, 32, 64):
    for _storage in ("fp32", "fp16"):
        WORKLOADS[f"generic_fwd_b2h8s512d{_width}_{_storage}"] = dict(
                batch=2, heads=8, seq=512, dim=_width, radius=-1, lengths=None, backward=False, generic=_storage,
                description=f"AttentionGeneric{_width} {_storage} b2 h8 l512 (AttentionGenericBenchmarks.cpp:79-110), "
                            f"attention_generic_forward")
DEFAULT_WORKLOAD = "flash_fwd_b8h3s1024d32"
PUBLISHED_TFLOPS = 3.36  # the reference's published flash fwd d32 figure, same FLOPs (B2 H12 L1024), RX 6700 (README.md:63)
METRIC = "FP32 attention TFLOP/s (repo FLOP convention: 4*B*H*Q*K*d forward, 8*B*H*Q*K*d backward)"


def key_lengths(spec: dict) -> list[int]:
    """Visible keys per sequence of the global batch (keys [0, length) visible): BASELINE's
    lengths U[lo, hi] drawn from MT19937 seed 105 (oracle.lengths, the same draws the parity tests
    use); without the oracle library, numpy's generator (other values) stands in."""
    import numpy as np

    batch, seq, lengths = spec["batch"], spec["seq"], spec["lengths"]
    if lengths is None:
        return [seq] * batch
    if lengths == "c1":
        return [seq if b != 1 else seq - 16 for b in range(batch)]
    low, high = lengths
    try:
        from oracle import oracle

        return [int(x) for x in oracle.lengths(batch, 105, low, high)]
    except (ImportError, OSError, subprocess.CalledProcessError):
        return [int(x) for x in np.random.default_rng(105).integers(low, high + 1, size=batch)]


def active_pairs(seq: int, radius: int, length: int) -> int:
    """(query, key) pairs a sequence with `length` visible keys and the radius window computes."""
    if radius < 0:
        return seq * length
    total = 0
    for i in range(seq):
        lo, hi = max(0, i - radius), min(length - 1, i + radius)
        total += max(0, hi - lo + 1)
    return total


def workload_config(name: str, world: int) -> dict:
    spec = WORKLOADS[name]
    l2 = ("inputs larger than L2: the steps rotate through input sets totalling >= 2 x the 126 MB L2 and run back to back "
          "(one event pair around the K steps); the per-step-flushed protocol is reported beside it"
          if not spec["backward"] else "flushed (256 MiB write) before every step")
    config = {"workload": name, "description": spec["description"], "heads": spec["heads"], "seq_len": spec["seq"],
              "head_dim": spec["dim"], "radius": spec["radius"], "l2": l2}
    if spec.get("generic"):
        config["storage"] = spec["generic"]
    if spec["backward"]:
        lengths = key_lengths(spec)
        config.update({"global_batch": spec["batch"], "batch_per_gpu": spec["batch"] // world, "step": "forward + backward",
                       "mask": "all visible" if spec["lengths"] is None else f"key lengths {lengths}",
                       "parallelism": f"batch-sharded x{world} (strong scaling), no collective"})
    else:
        config.update({"batch_per_gpu": spec["batch"], "global_batch": spec["batch"] * world, "mask": "all visible",
                       "parallelism": f"batch-sharded x{world}, no collective"})
    return config
FLUSH_BYTES = 256 << 20
L2_BYTES = 126 * 10**6  # B200 L2; rotating input sets total at least twice this


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


def cpu_baseline(spec: dict) -> dict:
    """The oracle (C restatement) on this host's cores: the full forward workload for the headline,
    a bounded sample of (batch, head) slices for the forward + backward configs."""
    import numpy as np
    from oracle import oracle

    threads = oracle.cpu_count()
    seq, dim, radius = spec["seq"], spec["dim"], spec["radius"]
    if spec["backward"]:
        batch, heads, length = 1, threads, key_lengths(spec)[0]
        forward_only, upstream = False, oracle.normal(heads * seq * dim, 104).reshape(1, heads, seq, dim)
        flops = 12.0 * heads * seq * seq * dim
        what = (f"forward+backward of {heads} (batch, head) slices (S={seq}, d={dim}, {length} visible keys, radius {radius}),"
                f" one slice per thread; repo-convention FLOPs")
    else:
        batch, heads, length = spec["batch"], spec["heads"], seq
        forward_only, upstream = True, None
        flops = 4.0 * batch * heads * seq * seq * dim
        what = "forward over the full workload"
    q = oracle.normal(batch * heads * seq * dim, 101).reshape(batch, heads, seq, dim)
    k = oracle.normal(batch * heads * seq * dim, 102).reshape(batch, heads, seq, dim)
    v = oracle.normal(batch * heads * seq * dim, 103).reshape(batch, heads, seq, dim)
    if spec.get("generic") == "fp16":  # the values FP16 storage holds, widened (AttentionGenericTests.cpp:118-119)
        q, k, v = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    mask = np.zeros((batch, seq), dtype="uint8")
    mask[:, :length] = 1
    reps, elapsed = 0, 0.0
    while elapsed < 10.0 and reps < 50:
        start = time.perf_counter()
        oracle.attention(q, k, v, mask, upstream, radius, threads=threads, forward_only=forward_only)
        elapsed += time.perf_counter() - start
        reps += 1
    return {"value": flops * reps / elapsed / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"oracle/attention_oracle.c (double accumulation, as ReferenceAttention) {what} x{reps},"
                      f" {elapsed:.1f} s on {threads} threads"}


def run_reference(args, rank: int) -> None:
    """--impl reference: the reference's CPU attention on rank 0; other ranks exit without work.

    The reference's own ReferenceAttention (AttentionTests.cpp:28-125), compiled from its source
    into oracle/_ref/libref_attention.so (a self-contained library: it maps neither this
    repository's CUDA library nor a CUDA runtime), else the oracle's restatement of it. A step is
    the workload's own (batch, head) slices on its seeded inputs -- all of them for the forward
    workloads (the headline: B8 H3 S1024, 24 slices), a bounded sample of one slice per host
    thread for the forward + backward configs -- spread over every host thread. The function always
    computes forward and backward, so its FLOPs are counted as 12*S*S*d per slice."""
    if rank != 0:
        return
    import concurrent.futures

    import numpy as np
    from oracle import oracle

    spec = WORKLOADS[args.workload]
    if spec.get("generic"):
        run_reference_generic(args, spec)
        return
    if spec.get("kind") == "rotary":
        base = rotary_cpu_baseline(spec)
        print(json.dumps({"metric": "rotary GB/s (4 x elements x 4 B per step: q, k read, oq, ok written; RotaryBenchmarks.cpp:68)",
                          "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
                          "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32", "data": "seeded uniform", "config": workload_config(args.workload, args.gpus),
                          "impl": "reference", "cpu_baseline": base,
                          "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    seq, dim, radius, heads = spec["seq"], spec["dim"], spec["radius"], spec["heads"]
    threads = oracle.cpu_count()
    use_ref = oracle.reference_available()
    lengths = key_lengths(spec)
    if spec["backward"]:  # a bounded sample: one slice per thread, spread over the global batch
        batch = min(spec["batch"], threads)
        slice_list = [(b, b % heads) for b in range(batch)]
        what = f"a sample of {batch} of the workload's {spec['batch'] * heads} (batch, head) slices"
    else:
        batch = spec["batch"]
        slice_list = [(b, h) for b in range(batch) for h in range(heads)]
        what = f"all {batch * heads} (batch, head) slices of the workload (B{batch} H{heads})"
    count = batch * heads * seq * dim
    q, k, v, u = (oracle.normal(count, seed).reshape(batch, heads, seq, dim) for seed in (101, 102, 103, 104))
    mask = np.zeros((batch, seq), np.uint8)
    for b in range(batch):
        mask[b, :lengths[b]] = 1

    def one_slice(bh):
        b, h = bh
        cut = lambda x: np.ascontiguousarray(x[b:b + 1, h:h + 1])  # noqa: E731
        if use_ref:
            oracle.reference_attention(cut(q), cut(k), cut(v), mask[b:b + 1], cut(u), radius)
        else:
            oracle.attention(cut(q), cut(k), cut(v), mask[b:b + 1], cut(u), radius, threads=1)

    pool = concurrent.futures.ThreadPoolExecutor(threads)  # the library calls release the GIL

    def step():
        list(pool.map(one_slice, slice_list))

    for _ in range(args.warmup):
        step()
    start = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - start
    pool.shutdown()
    flops = 12.0 * len(slice_list) * seq * seq * dim * args.steps  # forward (4) + backward (8): it computes both
    value = flops / elapsed / 1e12
    kind = "reference" if use_ref else "port"
    sample = (f"{'ReferenceAttention (AttentionTests.cpp:28-125, compiled from the reference source)' if use_ref else 'oracle port'}"
              f" forward+backward of {what} per step, S={seq} d={dim}, radius {radius}, on {threads} threads;"
              f" FLOPs counted as 12*S*S*d per slice (the function always computes forward and backward)")
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak" if not spec["backward"] else "strong", "vs_baseline": None,
            "dtype": "f64-accumulate/f32-storage",
            "data": "synthetic N(0,1), seeds 101-104 (std::mt19937 + libstdc++ normal_distribution, the reference's generator)",
            "config": workload_config(args.workload, args.gpus), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def rotary_cpu_baseline(spec: dict) -> dict:
    """The rotary oracle (ReferenceRotary restated, one thread) over the full workload."""
    from oracle import oracle

    batch, heads, length = spec["batch"], spec["heads"], spec["seq"]
    x = oracle.uniform(batch * length * heads * 32, 21, -2, 2).reshape(batch, length, heads, 32)
    cos = oracle.uniform(batch * length * 32, 23).reshape(batch, length, 32)
    sin = oracle.uniform(batch * length * 32, 24).reshape(batch, length, 32)
    reps, elapsed = 0, 0.0
    while elapsed < 5.0 and reps < 200:
        start = time.perf_counter()
        oracle.rotary(x, cos, sin, spec["backward"])
        oracle.rotary(x, cos, sin, spec["backward"])  # q and k
        elapsed += time.perf_counter() - start
        reps += 1
    moved = 4.0 * batch * heads * length * 32 * 4
    return {"value": moved * reps / elapsed / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"oracle_rotary (ReferenceRotary, PositionalTests.cpp:18-50) on q and k of the full workload x{reps},"
                      f" {elapsed:.1f} s on 1 thread"}


def run_rotary(args, spec: dict, device, world: int, rank: int, dist) -> None:
    """Rotary workloads: rotary_fp32 on token-major q, k (the reference's benchmark layout)."""
    import torch

    import rocmkernels_b200.attention as api

    batch, heads, length = spec["batch"], spec["heads"], spec["seq"]
    backward = 1 if spec["backward"] else 0
    generator = torch.Generator(device=device)
    generator.manual_seed(301 + rank)
    q = torch.randn(batch, length, heads, 32, device=device, generator=generator)
    k = torch.randn(batch, length, heads, 32, device=device, generator=generator)
    cos = torch.randn(batch, length, 32, device=device, generator=generator)
    sin = torch.randn(batch, length, 32, device=device, generator=generator)
    oq, ok = torch.empty_like(q), torch.empty_like(k)
    qk_strides = api.Strides(length * heads * 32, 32, heads * 32)  # RotaryBenchmarks.cpp:55
    table_strides = api.Strides(length * 32, 0, 32)                 # :56
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def run(tensors, st):
        tq, tk, tcos, tsin, toq, tok = tensors
        status = api.rotary_fp32(tq, tk, tcos, tsin, toq, tok, batch, heads, length, backward, qk_strides, qk_strides,
                                 table_strides, table_strides, st)
        if status != 0:
            raise api.HipError(status, "rotary_fp32")

    def step():
        run((q, k, cos, sin, oq, ok), stream)

    inputs, outputs = [q, k, cos, sin], [oq, ok]
    host_inputs = [t.cpu().pin_memory() for t in inputs]
    host_outputs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outputs]
    e2e_sets = [(inputs, outputs), ([torch.empty_like(t) for t in inputs], [torch.empty_like(t) for t in outputs])]

    def launch_set(index, st):
        set_inputs, set_outputs = e2e_sets[index]
        run((*set_inputs, *set_outputs), st)

    def timed(fn, steps):
        marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.fill_(float(i))
            marks[i][0].record(stream)
            fn()
            marks[i][1].record(stream)
        torch.cuda.synchronize(device)
        return sum(a.elapsed_time(b) for a, b in marks) / 1e3

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    sampler = ClockSampler(visible.split(",")[int(os.environ.get("LOCAL_RANK", 0))].strip() if visible else str(rank))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    seconds = timed(step, args.steps)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if rank == 0 else None
    pipelined_e2e(device, e2e_sets, host_inputs, host_outputs, launch_set, 2)
    e2e_steps = max(1, min(args.steps, 50))
    e2e_seconds = pipelined_e2e(device, e2e_sets, host_inputs, host_outputs, launch_set, e2e_steps)
    times = torch.tensor([seconds, e2e_seconds], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    seconds, e2e_seconds = times.tolist()

    moved = 4.0 * batch * heads * length * 32 * 4  # q, k read; oq, ok written (RotaryBenchmarks.cpp:68)
    touched = moved + 2.0 * batch * length * 32 * 4  # plus the two tables
    peaks, peak_source = measured_peaks()
    achieved = touched / (seconds / args.steps) / 1e9
    line = {
        "metric": "rotary GB/s (4 x elements x 4 B per step: q, k read, oq, ok written; RotaryBenchmarks.cpp:68)",
        "value": world * moved * args.steps / seconds / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": seconds / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) from a seeded torch generator",
        "config": workload_config(args.workload, world),
        "e2e": {"value": world * moved * e2e_steps / e2e_seconds / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_inputs),
                "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in host_outputs), "steps": e2e_steps},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                     "frac": achieved / float(peaks["hbm_gbs"]), "traffic": traffic_from_profiles("rotary", args.workload),
                     "peak_source": f"{peak_source} hbm_gbs", "kernel": f"rotary_kernel<{'backward' if backward else 'forward'}>",
                     "bytes": "q, k, oq, ok and both tables once"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = rotary_cpu_baseline(spec)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_generic(args, spec: dict) -> None:
    """--impl reference for the generic workloads: the reference has no CPU implementation of the
    generic forward besides its test's double-precision ComputeReference
    (AttentionGenericTests.cpp:45-104), which the oracle's forward restates; it runs on the full
    workload with all host threads."""
    base = cpu_baseline(spec)
    elapsed_per_step = 4.0 * spec["batch"] * spec["heads"] * spec["seq"] ** 2 * spec["dim"] / (base["value"] * 1e12)
    line = {"metric": METRIC, "value": base["value"], "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_per_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64-accumulate", "data": "synthetic N(0,1), seeded",
            "config": workload_config(args.workload, args.gpus), "impl": "reference",
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def pipelined_e2e(device, sets, host_inputs, host_outputs, launch, steps: int) -> float:
    """Seconds for `steps` end-to-end steps: step i copies `host_inputs` (pinned) into the device
    inputs of buffer set i % 2 (copy-in stream), runs `launch(set, stream)` on the compute stream
    and copies the set's outputs back into `host_outputs` (pinned, copy-out stream). A set's inputs
    are refilled only after the kernels that read them finished, and its outputs rewritten only
    after their read-back, so step i's copies overlap steps i - 1 and i + 1. Timed with events
    from the first H2D to the last D2H."""
    import torch

    copy_in, compute, copy_out = (torch.cuda.Stream(device=device) for _ in range(3))
    loaded, computed, unloaded = ([torch.cuda.Event() for _ in sets] for _ in range(3))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record(copy_in)
    for i in range(steps):
        s = i % len(sets)
        device_inputs, device_outputs = sets[s]
        if i >= len(sets):
            copy_in.wait_event(computed[s])
        with torch.cuda.stream(copy_in):
            for device_tensor, host_tensor in zip(device_inputs, host_inputs):
                device_tensor.copy_(host_tensor, non_blocking=True)
        loaded[s].record(copy_in)
        compute.wait_event(loaded[s])
        if i >= len(sets):
            compute.wait_event(unloaded[s])
        launch(s, compute)
        computed[s].record(compute)
        copy_out.wait_event(computed[s])
        with torch.cuda.stream(copy_out):
            for host_tensor, device_tensor in zip(host_outputs, device_outputs):
                host_tensor.copy_(device_tensor, non_blocking=True)
        unloaded[s].record(copy_out)
    end.record(copy_out)
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / 1e3


def traffic_from_profiles(kernel_tag: str, workload: str):
    """DRAM bytes per launch of `kernel_tag` from the committed ncu summaries, only when they were
    captured on this same workload (another shape moves other bytes); else None."""
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None
    entries = json.loads(path.read_text()).get(kernel_tag, [])
    for entry in entries if isinstance(entries, list) else [entries]:
        if entry.get("workload") == workload:
            return entry.get("dram_bytes_per_launch")
    return None


def seeded_problem(batch: int, heads: int, seq: int, dim: int, lengths: list[int], upstream: bool):
    """The workload's inputs: Q, K, V (and dO) ~ N(0, 1) from seeds 101..104 drawn with the
    reference's generator (std::mt19937 + libstdc++ normal_distribution, restated in
    oracle/attention_oracle.c; the parity tests draw the same tensors), and the [batch, seq] mask
    with keys [0, length) visible. Returns (arrays, description), or (None, reason) when that
    generator's library is not available (the caller then draws from torch and reports no parity)."""
    import concurrent.futures

    import numpy as np

    try:
        from oracle import oracle

        oracle._load_oracle()
    except Exception as error:  # noqa: BLE001 - any failure to load the generator
        return None, f"seeded generator unavailable ({type(error).__name__})"
    count = batch * heads * seq * dim
    seeds = (101, 102, 103, 104) if upstream else (101, 102, 103)
    with concurrent.futures.ThreadPoolExecutor(len(seeds)) as pool:  # the generator releases the GIL
        drawn = list(pool.map(lambda seed: oracle.normal(count, seed).reshape(batch, heads, seq, dim), seeds))
    mask = np.zeros((batch, seq), np.uint8)
    for b, length in enumerate(lengths):
        mask[b, :length] = 1
    arrays = {"q": drawn[0], "k": drawn[1], "v": drawn[2], "mask": mask}
    if upstream:
        arrays["upstream"] = drawn[3]
    return arrays, ("synthetic N(0,1), seeds 101-104 (Q, K, V, dO) from std::mt19937 + libstdc++ normal_distribution, "
                    "the reference's generator")


def _normwise(actual, expected) -> float:
    """max|actual - expected| / max|expected| over finite entries; inf if the non-finite patterns differ."""
    import numpy as np

    a, e = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    finite = np.isfinite(e)
    if not np.array_equal(finite, np.isfinite(a)) or not np.array_equal(np.isnan(a), np.isnan(e)):
        return float("inf")
    if not finite.any():
        return 0.0
    scale = float(np.max(np.abs(e[finite])))
    diff = float(np.max(np.abs(a[finite] - e[finite])))
    return diff / scale if scale > 0 else diff


def parity_check(arrays: dict, results: dict, slices: list, radius: int, backward: bool) -> dict:
    """The CPU oracle (checker only) on the listed (batch, head) slices of the workload's own inputs,
    compared with the device's results for those slices (`results`: name -> [B, H, ...] arrays).
    Bars: O and lse normwise <= 1e-5, gradients <= 1e-4 (the parity tests' bars)."""
    import concurrent.futures

    import numpy as np
    from oracle import oracle

    def one(bh):
        b, h = bh
        cut = lambda x: np.ascontiguousarray(x[b:b + 1, h:h + 1])  # noqa: E731
        return oracle.attention(cut(arrays["q"]), cut(arrays["k"]), cut(arrays["v"]), arrays["mask"][b:b + 1],
                                cut(arrays["upstream"]) if backward else None, radius, forward_only=not backward)

    with concurrent.futures.ThreadPoolExecutor(max(1, min(len(slices), oracle.cpu_count()))) as pool:
        expected = list(pool.map(one, slices))
    names = [("O", "out", "output", None), ("lse_max", "lse", "lse", 0), ("lse_sum", "lse", "lse", 1)]
    if backward:
        names += [(n, n, n, None) for n in ("grad_q", "grad_k", "grad_v")]
    errors = {}
    for label, ours, theirs, column in names:
        worst = 0.0
        for (b, h), exp in zip(slices, expected):
            got = results[ours][b:b + 1, h:h + 1]
            want = exp[theirs]
            if column is not None:
                got, want = got[..., column], want[..., column]
            worst = max(worst, _normwise(got, want))
        errors[label] = worst
    ok = all(v <= (1e-4 if k.startswith("grad") else 1e-5) for k, v in errors.items())
    return {"ok": bool(ok), "slices": len(slices), **{f"max_rel_{k}": v for k, v in errors.items()},
            "bars": "normwise max|x-ref|/max|ref|: O, lse <= 1e-5; gradients <= 1e-4",
            "checker": "oracle/attention_oracle.c (ReferenceAttention restated, pinned bit-exact to the reference)"}


def c5_strong(args, device, world: int, rank: int, dist, api) -> dict:
    """BASELINE configs[4] (B64 H12 S4096 d32, forward + backward, full attention) strong-scaled:
    the global problem is split over the ranks by rocmkernels_b200.sharding (contiguous batch
    ranges), every rank making its calls through the library's entry points, no collective on the
    data path. Inputs are larger than L2 (1.6 GB), so no flush between steps. Rank 0 checks the
    (0, 0) slice, which it computes itself, against the oracle."""
    import torch

    from rocmkernels_b200.sharding import forward_workspace_bytes, run_backward, run_forward, shard_plan, workspace_bytes

    spec = WORKLOADS["c5_fwd_bwd_b64h12s4096d32"]
    B, H, S, D = spec["batch"], spec["heads"], spec["seq"], spec["dim"]
    arrays, data = seeded_problem(B, H, S, D, [S] * B, True)
    generator = torch.Generator(device=device)
    generator.manual_seed(101)
    t = {}
    for name in ("q", "k", "v", "upstream"):
        t[name] = (torch.from_numpy(arrays[name]).to(device) if arrays is not None
                   else torch.randn(B, H, S, D, device=device, generator=generator))
    t["mask"] = torch.ones(B, S, dtype=torch.uint8, device=device)
    t["out"] = torch.empty_like(t["q"])
    t["lse"] = torch.empty(B, H, S, 2, device=device)
    for name in ("grad_q", "grad_k", "grad_v"):
        t[name] = torch.empty_like(t["q"])
    t["delta"] = torch.empty(B, H, S, device=device)
    st = api.strides_of(t["q"])
    strides = {r: st for r in ("q", "k", "v", "out", "upstream")}
    plan = shard_plan(B, H, world, rank)
    geometry = dict(heads=H, queries=S, keys=S, width=D, radius=-1, strides=strides)
    stream = torch.cuda.current_stream(device)
    fwd_t = {r: t[r] for r in ("q", "k", "v", "mask", "out", "lse")}

    # The forward with a workspace: K and V split once per head by the operand pre-pass.
    forward_workspace = torch.empty(max(1, forward_workspace_bytes(api.attention_fp32_forward_flash_workspace_size, plan, S)),
                                    dtype=torch.uint8, device=device)

    def forward():
        status = run_forward(api.attention_fp32_forward_flash_workspace, fwd_t, plan, stream=stream, workspace=forward_workspace,
                             **geometry)
        if status != 0:
            raise api.HipError(status, "attention_fp32_forward_flash_workspace")

    two_pass, fused = "attention_fp32_backward", "attention_fp32_backward_fused"
    workspace = torch.empty(max(1, workspace_bytes(api.attention_fp32_backward_fused_workspace_size, plan, S)), dtype=torch.uint8,
                            device=device)

    def backward(entry):
        status = run_backward(getattr(api, entry), t, plan, stream=stream, workspace=workspace if entry == fused else None,
                              **geometry)
        if status != 0:
            raise api.HipError(status, entry)

    for _ in range(2):
        forward()
        backward(two_pass)
        backward(fused)
    steps = max(3, min(args.steps, 10))
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    for i in range(steps):
        marks[i][0].record(stream)
        forward()
        marks[i][1].record(stream)
        backward(two_pass)
        marks[i][2].record(stream)
        backward(fused)
        marks[i][3].record(stream)
    torch.cuda.synchronize(device)
    own = [sum(m[e].elapsed_time(m[e + 1]) for m in marks) / steps for e in range(3)]
    times = torch.tensor([own[0] + own[2], own[0] + own[1]] + own, device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, step_two_pass_ms, forward_ms, backward_ms, backward_fused_ms = times.tolist()
    slices = [c.batch * c.heads for c in plan]
    flops = 12.0 * B * H * S * S * D
    record = {"workload": "c5_fwd_bwd_b64h12s4096d32", "description": spec["description"], "scaling": "strong",
              "ranks": world, "steps": steps,
              "ms_per_step": step_ms, "tflops": flops / (step_ms * 1e-3) / 1e12,
              "step": "attention_fp32_forward_flash_workspace + attention_fp32_backward_fused (the single-pass backward)",
              "ms_per_step_two_pass": step_two_pass_ms, "tflops_two_pass": flops / (step_two_pass_ms * 1e-3) / 1e12,
              "forward_ms": forward_ms, "backward_two_pass_ms": backward_ms, "backward_fused_ms": backward_fused_ms,
              "rank0_slices": sum(slices), "rank0_active_pairs": sum(slices) * S * S,
              "partition": "rocmkernels_b200.sharding.shard_plan: contiguous batch ranges, no collective on the data path",
              "gpu_launches_per_rank": steps * len(plan) * (4 + (2 if api.flash_workspace_kernel_name(plan[0].batch, plan[0].heads, S, S)
                                                                      .endswith("-prepared") else 1)), "data": data,
              "time": "CUDA events per rank around each call, mean over steps, max over ranks; inputs > L2; both "
                      "backward forms run every step on the same forward output"}
    if rank == 0 and arrays is not None:
        results = {n: t[n][0:1, 0:1].cpu().numpy() for n in ("out", "lse", "grad_q", "grad_k", "grad_v")}
        record["parity"] = parity_check(arrays, results, [(0, 0)], -1, True)
        backward(two_pass)  # the (0, 0) slice through the two-pass backward as well
        torch.cuda.synchronize(device)
        results = {n: t[n][0:1, 0:1].cpu().numpy() for n in ("out", "lse", "grad_q", "grad_k", "grad_v")}
        record["parity_two_pass"] = parity_check(arrays, results, [(0, 0)], -1, True)
    if world > 1:
        dist.barrier()
    del t, fwd_t, workspace
    torch.cuda.empty_cache()
    return record


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    parser.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle leg")
    parser.add_argument("--no-c5", action="store_true", help="skip the C5 strong-scaling record of the default workload")
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
    from rocmkernels_b200.sharding import ShardCall, run_backward, run_forward, shard_plan, workspace_bytes

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        # NCCL may print a banner to stdout when its communicator starts; stdout carries only the
        # JSON line, so everything written during set-up (and the first collective) goes to stderr.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
            dist.barrier()
            torch.cuda.synchronize(device)
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

    spec = WORKLOADS[args.workload]
    if spec.get("kind") == "rotary":
        run_rotary(args, spec, device, world, rank, dist)
        return
    heads, seq, dim, radius, with_backward = spec["heads"], spec["seq"], spec["dim"], spec["radius"], spec["backward"]
    generic = spec.get("generic")  # None, or the generic forward's storage type
    rotary = spec.get("rotary", False)
    storage = torch.float16 if generic == "fp16" else torch.float32
    batch = spec["batch"]
    if with_backward:
        # Strong scaling: every rank holds the global problem and computes its shard of (batch,
        # head) slices through the library's calls (rocmkernels_b200.sharding).
        lengths = key_lengths(spec)
        plan = shard_plan(batch, heads, world, rank)
    else:
        # Weak scaling: every rank runs the whole per-GPU problem (the same seeded inputs).
        lengths = [seq] * batch
        plan = [ShardCall(0, batch, 0, heads)]
    arrays, data = seeded_problem(batch, heads, seq, dim, lengths, with_backward)
    generator = torch.Generator(device=device)
    generator.manual_seed(101)

    def device_input(name):
        if arrays is not None:
            return torch.from_numpy(arrays[name]).to(device).to(storage)
        return torch.randn(batch, heads, seq, dim, device=device, generator=generator).to(storage)

    q, k, v = device_input("q"), device_input("k"), device_input("v")
    mask = torch.zeros(batch, seq, dtype=torch.uint8, device=device)
    for i, length in enumerate(lengths):
        mask[i, :length] = 1
    out = torch.empty_like(q)
    lse = torch.empty(batch, heads, seq, 2, device=device)
    inputs, outputs = [q, k, v, mask], [out, lse]
    if rotary:
        angle = torch.rand(batch, seq, 16, device=device, generator=generator) * 6.0
        cos = torch.cat([torch.cos(angle)] * 2, dim=-1).contiguous()
        sin = torch.cat([torch.sin(angle)] * 2, dim=-1).contiguous()
        table_strides = api.Strides(seq * 32, 0, 32)
        rotated_q = torch.empty(batch, seq, heads, 32, device=device)
        rotated_k = torch.empty_like(rotated_q)
        inputs += [cos, sin]
    if with_backward:
        upstream = device_input("upstream").float()
        gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        delta = torch.empty(batch, heads, seq, device=device)
        inputs.append(upstream)
        outputs += [gq, gk, gv]
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    qs, ks, vs, os_ = (api.strides_of(t) for t in (q, k, v, out))
    forward_fn = (getattr(api, spec["entry"]) if spec.get("entry") else
                  api.attention_fp32_forward_flash if dim == 32 else api.attention64_fp32_forward)
    backward_fn = (getattr(api, spec["backward_entry"]) if spec.get("backward_entry") else
                   api.attention_fp32_backward if dim == 32 else api.attention64_fp32_backward)
    # This rank's work: the (batch, head) slices of its plan.
    rank_pairs = sum(active_pairs(seq, radius, lengths[b]) * (c.h1 - c.h0) for c in plan for b in range(c.b0, c.b1))
    rank_slices = sum(c.batch * c.heads for c in plan)
    flops_forward, flops_backward = 4.0 * rank_slices * seq * seq * dim, 8.0 * rank_slices * seq * seq * dim
    effective_forward, effective_backward = 4.0 * rank_pairs * dim, 8.0 * rank_pairs * dim
    # Whole-job totals over all ranks: under strong scaling the ranks hold different sequences
    # (key-padded lengths differ), so the job's active pairs are summed over the global batch;
    # under weak scaling every rank runs the same shape.
    if with_backward:
        job_pairs = sum(active_pairs(seq, radius, length) for length in lengths) * heads
        job_flops_per_step = (4.0 + 8.0) * batch * heads * seq * seq * dim
        job_effective_forward, job_effective_backward = 4.0 * job_pairs * dim, 8.0 * job_pairs * dim
    else:
        job_flops_per_step = world * flops_forward
        job_effective_forward, job_effective_backward = world * effective_forward, 0.0
    job_effective_per_step = job_effective_forward + job_effective_backward
    # The d = 32 split-FP32 flash forward (headline, rotary and FP32 generic d = 32) is two kernels:
    # the K/V operand pre-pass and the forward.
    forward_kernel = ("" if spec.get("entry") == "attention_fp32_forward" or generic == "fp16" or
                      (generic and dim != 32) else api.flash_kernel_name(batch, heads, seq, seq, dim))
    forward_launches = 2 if forward_kernel.endswith("-prepared") else 1
    launches_per_step = len(plan) * (forward_launches + (2 if with_backward else 0))

    # The step's device tensors by role (one set for the device-timed steps; the e2e leg uses two).
    tensors = dict(q=q, k=k, v=v, mask=mask, out=out, lse=lse)
    if rotary:
        tensors.update(cos=cos, sin=sin)
    if with_backward:
        tensors.update(upstream=upstream, grad_q=gq, grad_k=gk, grad_v=gv, delta=delta)
    strides = {"q": qs, "k": ks, "v": vs, "out": os_}
    if with_backward:
        strides["upstream"] = api.strides_of(upstream)

    fused_backward = with_backward and spec.get("backward_entry") == "attention_fp32_backward_fused"
    workspaces = {}  # the fused backward's workspace by size; every call using one is ordered on one stream

    def workspace_for(calls):
        if not fused_backward:
            return None
        size = workspace_bytes(api.attention_fp32_backward_fused_workspace_size, calls, seq)
        if size not in workspaces:
            workspaces[size] = torch.empty(max(size, 1), dtype=torch.uint8, device=device)
        return workspaces[size]

    def make_phases(t, st, calls, problem_batch):
        """The step's kernel calls on tensor set `t` (a problem of `problem_batch` sequences),
        making the calls of `calls`, launched on stream `st`."""
        geometry = dict(heads=heads, queries=seq, keys=seq, width=dim, radius=radius, strides=strides)
        workspace = workspace_for(calls)

        def forward():
            if rotary:
                status = api.attention_fp32_forward_flash_rotary(t["q"], t["k"], t["v"], t["cos"], t["sin"], t["mask"], t["out"],
                                                                 t["lse"], problem_batch, heads, seq, seq, radius, qs, ks, vs,
                                                                 table_strides, table_strides, os_, st)
                if status != 0:
                    raise api.HipError(status, "attention_fp32_forward_flash_rotary")
                return
            if generic:
                status = api.attention_generic_forward(t["q"], t["k"], t["v"], t["mask"], t["out"], t["lse"], problem_batch, heads,
                                                       seq, seq, dim, radius, qs, ks, vs, os_,
                                                       api.DType.Float16 if generic == "fp16" else api.DType.Float32, st)
            else:
                status = run_forward(forward_fn, {r: t[r] for r in ("q", "k", "v", "mask", "out", "lse")}, calls, stream=st,
                                     **geometry)
            if status != 0:
                raise api.HipError(status, "attention_generic_forward" if generic else forward_fn.__name__)

        def backward():
            status = run_backward(backward_fn, t, calls, stream=st, workspace=workspace, **geometry)
            if status != 0:
                raise api.HipError(status, backward_fn.__name__)

        return [forward, backward] if with_backward else [forward]

    phases = make_phases(tensors, stream, plan, batch)

    def unfused_rotary_forward():
        """rotary_fp32 into token-major buffers, then the flash forward on them (the unfused sequence)."""
        rs = api.Strides(seq * heads * 32, 32, heads * 32)
        status = api.rotary_fp32(q, k, cos, sin, rotated_q, rotated_k, batch, heads, seq, 0, qs, ks, table_strides, table_strides,
                                 stream)
        if status == 0:
            status = api.attention_fp32_forward_flash(rotated_q, rotated_k, v, mask, out, lse, batch, heads, seq, seq, radius, rs, rs,
                                                      vs, os_, stream)
        if status != 0:
            raise api.HipError(status, "rotary_fp32 + attention_fp32_forward_flash")

    # Host-buffer leg: pinned inputs copied in and outputs copied out every step, two device sets of
    # this rank's sequences [base, end) (its whole problem under weak scaling).
    base, end = min(c.b0 for c in plan), max(c.b1 for c in plan)
    local_plan = [ShardCall(c.b0 - base, c.b1 - base, c.h0, c.h1) for c in plan]
    local = {name: x[base:end] for name, x in tensors.items() if name not in ("cos", "sin")}
    if rotary:
        local.update(cos=cos, sin=sin)
    by_id = {id(x): name for name, x in tensors.items()}
    host_inputs = [local[by_id[id(x)]].cpu().pin_memory() for x in inputs]
    host_outputs = [torch.empty(local[by_id[id(x)]].shape, dtype=x.dtype).pin_memory() for x in outputs]
    h2d_bytes = sum(x.numel() * x.element_size() for x in host_inputs)
    d2h_bytes = sum(x.numel() * x.element_size() for x in host_outputs)
    second = {name: torch.empty_like(x) for name, x in local.items()}
    e2e_tensors = [local, second]
    e2e_sets = [([t[by_id[id(x)]] for x in inputs], [t[by_id[id(x)]] for x in outputs]) for t in e2e_tensors]

    def launch_set(index, st):
        for phase in make_phases(e2e_tensors[index], st, local_plan, end - base):
            phase()

    def timed(fns, steps):
        """Seconds summed over `steps`: in total and per callable of `fns` (events between them)."""
        marks = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fns) + 1)] for _ in range(steps)]
        for i in range(steps):
            flush.fill_(float(i))
            marks[i][0].record(stream)
            for j, fn in enumerate(fns):
                fn()
                marks[i][j + 1].record(stream)
        torch.cuda.synchronize(device)
        parts = [sum(m[j].elapsed_time(m[j + 1]) for m in marks) / 1e3 for j in range(len(fns))]
        return sum(parts), parts

    # Forward-only workloads: extra input sets so that the rotation over them exceeds L2 twice over
    # (each step's inputs were last touched a whole rotation earlier, so they come from HBM).
    rotation = [phases]
    if not with_backward:
        set_bytes = sum(x.numel() * x.element_size() for x in tensors.values())
        copies = max(2, -(-2 * L2_BYTES // set_bytes))
        for _ in range(copies - 1):
            copy = {name: x.clone() for name, x in tensors.items()}
            rotation.append(make_phases(copy, stream, plan, batch))
        rotation_bytes = set_bytes * copies

    def timed_rotating(steps):
        """Seconds for `steps` back-to-back steps over the rotating input sets (one event pair)."""
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(steps):
            for fn in rotation[i % len(rotation)]:
                fn()
        end.record(stream)
        torch.cuda.synchronize(device)
        return start.elapsed_time(end) / 1e3

    for i in range(args.warmup):
        flush.fill_(0.0)
        for phase in rotation[i % len(rotation)]:
            phase()
    torch.cuda.synchronize(device)

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    sampler = ClockSampler(visible.split(",")[local_rank].strip() if visible else str(local_rank))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    if with_backward:
        device_seconds, part_seconds = timed(phases, args.steps)
    else:
        device_seconds = timed_rotating(args.steps)
        part_seconds = [device_seconds]
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if rank == 0 else None

    # The results of the last timed step, for the parity check below (the outputs of the e2e leg
    # are other buffers).
    parity_results = None
    if rank == 0 and arrays is not None and not rotary and not generic:
        chosen = sorted({(b, h) for c in plan for b in range(c.b0, c.b1) for h in range(c.h0, c.h1)})
        if len(chosen) > 24:  # a bounded, declared subset: the first, middle and last slice of the rank
            chosen = [chosen[0], chosen[len(chosen) // 2], chosen[-1]]
        names = ["out", "lse"] + (["grad_q", "grad_k", "grad_v"] if with_backward else [])
        parity_slices = chosen
        parity_results = {n: tensors[n].cpu().numpy() for n in names}

    pipelined_e2e(device, e2e_sets, host_inputs, host_outputs, launch_set, 2)
    e2e_steps = max(1, min(args.steps, 50))
    e2e_seconds = pipelined_e2e(device, e2e_sets, host_inputs, host_outputs, launch_set, e2e_steps)

    # The per-step-flushed protocol of earlier lines (256 MiB flush, then events around the step), for continuity.
    flushed_seconds = timed(phases, args.steps)[0] if not with_backward else 0.0

    unfused_seconds = 0.0
    if rotary:
        for _ in range(args.warmup):
            unfused_rotary_forward()
        unfused_seconds, _ = timed([unfused_rotary_forward], args.steps)

    times = torch.tensor([device_seconds, e2e_seconds, unfused_seconds, flushed_seconds] + part_seconds, device=device,
                         dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    device_seconds, e2e_seconds, unfused_seconds, flushed_seconds, *part_seconds = times.tolist()

    value = job_flops_per_step * args.steps / device_seconds / 1e12
    e2e_value = job_flops_per_step * e2e_steps / e2e_seconds / 1e12
    peaks, peak_source = measured_peaks()
    sm_mhz = (clocks or {}).get("sm_mhz") or float(peaks.get("sm_max_mhz", 1965.0))
    fma_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
    if with_backward:
        # The dominant kernel pair is the backward (the tcgen05 split-FP16 query-major delta + dQ
        # pass and key-major dK/dV pass); effective FLOPs per launch pair, against the measured
        # dense bf16 rate (the kind::f16 MMAs' rate) and the FP32 CUDA-core rate for context.
        achieved = effective_backward / (part_seconds[1] / args.steps) / 1e12
        peak = float(peaks["bf16_tflops"])
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic_from_profiles(f"tcgen05-backward-d{dim}", args.workload),
                    "peak_source": f"{peak_source} bf16_tflops (burst); the TF32 dense rate is half of it",
                    "frac_of_tf32_dense": achieved / (peak / 2), "frac_of_fp32_fma": achieved / fma_peak,
                    "kernel": (f"tcgen05 split-FP16 fused single-pass backward d{dim} (column pre-pass, key-major dK/dV/dQ)"
                               if fused_backward else
                               f"tcgen05 split-FP16 backward d{dim} (query-major delta+dQ, key-major dK/dV)"),
                    "flops": "effective: 8*d per active (query, key) pair"}
    else:
        achieved = effective_forward / (part_seconds[0] / args.steps) / 1e12
        if generic:
            path = api.generic_kernel_name(batch, heads, seq, seq, dim,
                                           api.DType.Float16 if generic == "fp16" else api.DType.Float32)
        elif spec.get("entry") == "attention_fp32_forward":
            path = f"simt-fp32-forward-d{dim}"
        else:
            path = api.flash_kernel_name(batch, heads, seq, seq, dim) + ("+rotary" if rotary else "")
        if path.startswith("tcgen05"):
            peak = float(peaks["bf16_tflops"])
            roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                        "traffic": traffic_from_profiles(path, args.workload), "kernel": path}
            if forward_launches == 2:
                roofline["duration"] = "the whole step: K/V operand pre-pass + forward kernel (back to back)"
            if path.startswith("tcgen05-f16x2"):  # FP32 storage: compare with the TF32 dense rate as well
                roofline["peak_source"] = f"{peak_source} bf16_tflops (burst); the TF32 dense rate is half of it"
                roofline["frac_of_tf32_dense"] = achieved / (peak / 2)
            else:
                roofline["peak_source"] = f"{peak_source} bf16_tflops (burst), the FP16 dense rate"
        else:
            roofline = {"bound": "fp32-fma", "achieved": achieved, "peak": fma_peak, "unit": "TFLOP/s", "frac": achieved / fma_peak,
                        "traffic": traffic_from_profiles(path, args.workload),
                        "peak_source": "148 SMs x 128 FP32 lanes x 2 FLOP x median SM clock under load", "kernel": path}

    line = {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": device_seconds / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if with_backward else "weak",
        "vs_baseline": None if with_backward or generic or rotary else value / PUBLISHED_TFLOPS,
        "dtype": generic or "f32",
        "data": data if arrays is not None else f"synthetic N(0,1) from a seeded torch generator ({data})",
        "config": workload_config(args.workload, world),
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                "steps": e2e_steps},
        "roofline": roofline,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks,
    }
    if generic == "fp16" and arrays is not None:
        line["data"] += ", rounded to FP16 storage"
    if not with_backward:
        line["flushed"] = {"ms_per_step": flushed_seconds / args.steps * 1e3,
                           "value": job_flops_per_step * args.steps / flushed_seconds / 1e12, "unit": "TFLOP/s",
                           "protocol": "256 MiB written before every step, CUDA events around each step (summed)"}
        line["config"]["rotation"] = {"sets": len(rotation), "bytes": rotation_bytes}
    if with_backward:
        line["effective"] = {"value": job_effective_per_step * args.steps / device_seconds / 1e12, "unit": "TFLOP/s",
                             "flops": "12*d per active (query, key) pair"}
        line["parts"] = {"forward_ms": part_seconds[0] / args.steps * 1e3, "backward_ms": part_seconds[1] / args.steps * 1e3,
                         "forward_effective_tflops": job_effective_forward * args.steps / part_seconds[0] / 1e12,
                         "backward_effective_tflops": job_effective_backward * args.steps / part_seconds[1] / 1e12}
    if rotary:
        line["unfused"] = {"ms_per_step": unfused_seconds / args.steps * 1e3,
                           "sequence": "rotary_fp32 (token-major outputs) then attention_fp32_forward_flash",
                           "tflops": job_flops_per_step * args.steps / unfused_seconds / 1e12}
    if args.workload == DEFAULT_WORKLOAD and not args.no_c5:
        line["c5_strong"] = c5_strong(args, device, world, rank, dist, api)
    if parity_results is not None:
        line["parity"] = parity_check(arrays, parity_results, parity_slices, radius, with_backward)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(spec)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
