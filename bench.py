"""Benchmark: GEMM TFLOP/s of the fwd+dX+dW products of StaleyNET's width-768 decoder's training step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--global-batch S]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

Workload (BASELINE config 5 on the config 3 model, at every N): one optimizer step's worth of work over a global
batch of 256 sequences x 2048 tokens, split over the N ranks by whole sequences; each rank runs its 256/N sequences
as 32 x 2048 = 65,536-token micro-batches (8/N of them), each through the 12-block width-768 decoder's linear GEMMs
(QKV 768->2304, output 768->768, FFN 768->3072->768) and the 16 x 1024 codebook head, forward, every codebook's
cross-entropy, dX and dW, bf16 operands with f32 accumulation and fused bias / GELU / residual epilogues
(staleynet_b200/step.py). dW accumulates over the micro-batches; the f32 weight gradients are all-reduced with NCCL
once per step, per block, overlapped with the last micro-batch's backward. 38.35 TFLOP per micro-batch, 306.8 TFLOP
per step; the total work is fixed as N grows (strong scaling). --global-batch 0 runs one micro-batch per GPU
instead (config 3 per GPU, weak scaling).

One JSON line (rank 0): `value` = whole-job TFLOP/s with inputs resident in HBM; `e2e` = the same step through
the C ABI with every micro-batch's input activations copied from pinned host memory and the per-codebook loss sums
read back every step; `roofline` = the tcgen05 GEMM kernels' FLOP rate from CUDA events around each launch in the
timed region, against the measured bf16 peak; `gemms` = the same per GEMM of the step; `communication` (N > 1) =
the all-reduce time left exposed after the last GEMM; `dp_parity` (N > 1) = the all-reduced gradients against
rank 0 recomputing the global batch alone; `cpu_baseline` = the CPU restatement of the reference's f32 GEMM loop on
the host cores, timed on a sample of every GEMM's output rows and extrapolated by rows.
`--impl reference` times that CPU path alone (the reference's own implementation cannot be built here).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GEMM TFLOP/s (fwd+bwd) & % bf16 tensor peak at 1/2/4/8 B200 vs host-CPU ref"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
GENERATOR = "the reference's generator (SplitMix64 + Box-Muller, random.rs:27-70, seed = rank) drawn on the device"


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(shape) -> dict:
    """Per-launch DRAM traffic of the step's GEMM launches, summarised from an ncu capture of this workload
    (profiles/tc_gemm_cfg3_step_launches.json); empty when the workload differs or no capture is committed."""
    path = ROOT / "profiles" / "tc_gemm_cfg3_step_launches.json"
    from staleynet_b200.step import ModelShape

    if shape != ModelShape() or not path.exists():
        return {}
    return json.loads(path.read_text())


def load_profile_traffic(summary: str, kernel: str):
    """Per-launch DRAM bytes (read + write) of `kernel` from an ncu capture summarised in profiles/<summary>; None
    when no capture is committed."""
    path = ROOT / "profiles" / summary
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(kernel)
    return None if entry is None else entry.get("dram_bytes")


def profile_traffic_sum(summary: str, kernels) -> float | None:
    """Sum of the per-launch DRAM bytes of `kernels` in profiles/<summary> (one launch of each per step); None when
    any is missing."""
    parts = [load_profile_traffic(summary, k) for k in kernels]
    return None if any(x is None for x in parts) else float(sum(parts))


def load_kernel_traffic(kernel: str):
    """A fused-attention kernel's DRAM bytes per launch at BASELINE config 4."""
    return load_profile_traffic("fused_attention_cfg4_kernels.json", kernel)


def workload_config(shape, n_gpus: int, global_sequences: int = 256, micro_per_rank: int = 8,
                    model: str = "cfg3") -> dict:
    if model == "cfg1":
        workload = ("cfg1 6-block width-256 decoder: linear + 4x1024 codebook-head GEMMs, fwd+dX+dW with the codebook "
                    "cross-entropy between them, one 8x512 micro-batch per GPU")
    elif global_sequences:
        workload = (f"cfg5 data-parallel training step of the cfg3 model (12 blocks, width 768): global batch "
                    f"{global_sequences} x 2048 tokens split over {n_gpus} GPU(s), {micro_per_rank} micro-batch(es) "
                    f"of 32 x 2048 per GPU accumulating dW, linear + 16x1024 codebook-head GEMMs fwd+dX+dW with "
                    f"the codebook cross-entropy between them, f32 dW all-reduced once per step")
    else:
        workload = ("cfg3 12-block width-768 decoder: linear + 16x1024 codebook-head GEMMs, fwd+dX+dW with the "
                    "codebook cross-entropy between them, one 32x2048 micro-batch per GPU")
    return {
        "workload": workload,
        "model": (f"staleynet width-{shape.width} {shape.blocks}-block decoder, linear/head GEMMs"),
        "blocks": shape.blocks,
        "width": shape.width,
        "ffn": shape.ffn,
        "head": f"{shape.codebooks}x{shape.codebook_size}",
        "tokens_per_micro_batch": shape.tokens,
        "micro_batches_per_gpu": micro_per_rank,
        "global_batch": (8 * n_gpus if model == "cfg1" else
                         global_sequences if global_sequences else 32 * n_gpus),
        "seq_len": 512 if model == "cfg1" else SEQ_LEN,
        "parallelism": f"dp{n_gpus}",
        "operands": "bf16 in, f32 accumulate; dW f32 via reduce-add; activations bf16",
        "l2": "inputs larger than L2: one micro-batch moves > 20 GB through HBM (126 MB L2 flushed by the work "
              "itself)",
        "not_in_step": "attention score/softmax products, norms, bias-gradient column sums (not linear GEMMs)",
    }


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def start(self):
        """Starts sampling and returns once the first sample is written, so that the samples counted by stop() are
        the ones taken after this call (inside the timed region)."""
        self.skip = 0
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            self.file.flush()
            lines = [x for x in Path(self.file.name).read_text().splitlines() if x.strip()]
            if lines:
                self.skip = len(lines)
                break
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [line.split(",") for line in Path(self.file.name).read_text().splitlines() if line.strip()]
        os.unlink(self.file.name)
        rows = rows[self.skip:]   # samples taken while the timed region ran
        sm, smax, power, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1].split()[0]))
                smax = float(r[2].split()[0])
                power.append(float(r[3].split()[0]))
            except (ValueError, IndexError):
                continue
            for name, flag in zip(names, r[5:9]):
                if "Active" in flag and "Not" not in flag:
                    reasons.add(name)
        loaded = [v for v in sm if smax and v > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------------------------------------ CPU baseline
_OPERANDS: dict = {}


def _seeded_operand(stored_rows: int, stored_cols: int, slot: int = 0):
    """A dense row-major [stored_rows, stored_cols] f32 operand holding the parity tests' seeded LCG values
    (kernels_match_reference.rs:26-38), written straight into the buffer in address order. Kept for the process
    (keyed by shape and slot: slot 1 is a second operand of the same shape), so repeated CPU timings reuse it."""
    import numpy as np

    from oracle import oracle as o

    key = (stored_rows, stored_cols, slot)
    buf = _OPERANDS.get(key)
    if buf is None:
        buf = np.empty(stored_rows * stored_cols, np.float32)
        o.lib().snb_oracle_fill_lcg(1 + len(_OPERANDS), o._f(buf), buf.size)
        _OPERANDS[key] = buf
    return buf


def cpu_baseline(shape, budget_flops: float = 40e9, threads: int = 0) -> dict:
    """Times the CPU oracle (the reference's f32 GEMM loop, reference.rs:18-38) on a sample of every GEMM of the
    step and extrapolates by output elements (each output element costs the same `inner` multiply-adds).

    The sample of a GEMM is its first rows x cols output block with cols = min(N, 256), sized to `budget_flops`
    over the whole step. Operands are dense f32 tensors of the step's true shapes and strides, filled with seeded
    values. Each sample runs once untimed, then twice timed; the faster timed run counts."""
    import numpy as np

    from oracle import oracle as o
    from staleynet_b200.step import linear_shapes, step_flops

    s = shape
    T, w, V = s.tokens, s.width, s.head_width
    total = step_flops(s)
    frac = min(1.0, budget_flops / total)
    gemms = []  # (repeats per step, M, N, K, left transposed, right transposed)
    for _, i, out in linear_shapes(s):
        gemms.append((s.blocks, T, out, i, False, False))   # forward  Y = X W
        gemms.append((s.blocks, T, i, out, False, True))    # dX = dY W^T
        gemms.append((s.blocks, i, out, T, True, False))    # dW += X^T dY
    gemms += [(1, T, V, w, False, False), (1, T, w, V, False, True), (1, w, V, T, True, False)]
    seconds_full = 0.0
    sampled_flops = 0.0
    used_threads = 1
    t_start = time.perf_counter()
    for mult, M, N, K, lt, rt in gemms:
        cols = min(N, 256)
        rows = min(M, max(1, int(round(frac * M * N / cols))))
        # Stored shapes: a transposed left is [K, M], a transposed right [N, K].
        left_shape = (K, M) if lt else (M, K)
        right_shape = (N, K) if rt else (K, N)
        left = _seeded_operand(*left_shape)
        right = _seeded_operand(*right_shape, slot=1 if right_shape == left_shape else 0)
        out = np.zeros(rows * cols, np.float32)
        p = o.product(rows, cols, K, o.storage_strides(lt, M, K, 0), o.storage_strides(rt, K, N, 0), 0)
        o.matmul_rows(p, 1, left, right, out, 0, rows, threads)
        dt = float("inf")
        for _ in range(2):
            t0 = time.perf_counter()
            used_threads = o.matmul_rows(p, 1, left, right, out, 0, rows, threads)
            dt = min(dt, time.perf_counter() - t0)
        seconds_full += mult * dt * (M * N) / (rows * cols)
        sampled_flops += 2.0 * rows * cols * K
        del out
    wall = time.perf_counter() - t_start
    return {"value": total / seconds_full / 1e12, "unit": UNIT, "cores": used_threads, "kind": "port",
            "sample": f"first rows x min(N,256) output block of every GEMM of the step, {frac:.2e} of its "
                      f"outputs ({sampled_flops / 1e9:.1f} GFLOP per timed run, best of 2 after an untimed run, "
                      f"{wall:.1f} s wall), extrapolated by output elements; dense f32 operands of the step's true "
                      f"shapes and strides, seeded with the reference's parity-test LCG",
            "seconds_per_step_extrapolated": seconds_full}


def single_thread_baseline(shape, budget_flops: float) -> dict:
    """The reference-faithful form of the CPU baseline: the same loop on one thread, as reference::matmul runs."""
    r = cpu_baseline(shape, budget_flops=budget_flops, threads=1)
    return {"value": r["value"], "unit": r["unit"], "cores": r["cores"], "sample": r["sample"]}


# ------------------------------------------------------------------------------------------------ main paths
def run_reference(args, shape, rank: int, world: int) -> int:
    if rank != 0:
        return 0
    from oracle import oracle as o

    o.build()
    # Each step times a tenth of the GPU arm's CPU sample, so that --steps 20 --warmup 5 stays within minutes; the
    # operands are filled once and reused.
    budget = args.cpu_sample_flops / 10
    for _ in range(args.warmup):
        cpu_baseline(shape, budget_flops=budget)
    vals, secs = [], []
    for _ in range(args.steps):
        r = cpu_baseline(shape, budget_flops=budget)
        vals.append(r["value"])
        secs.append(r["seconds_per_step_extrapolated"])
    value = statistics.median(vals)
    # The sample times one micro-batch's GEMMs; a step is every micro-batch of one rank's share of the global batch.
    micro = max(1, args.global_batch // MICRO_SEQUENCES // max(1, args.gpus)) if args.global_batch else 1
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(secs) * 1e3 * micro,
        "higher_is_better": True, "scaling": "strong" if args.global_batch else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config(shape, args.gpus, args.global_batch, micro, args.model),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": r["cores"], "kind": "port", "sample": r["sample"],
                         "single_thread": single_thread_baseline(shape, args.cpu_sample_flops / 40)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU restatement of reference::matmul (crates/staleynet-cuda/src/reference.rs:18-38); the "
                "reference's Rust CPU path cannot be built here (no Rust toolchain)",
    }
    print(json.dumps(line), flush=True)
    return 0


SEQ_LEN = 2048
MICRO_SEQUENCES = 32   # sequences per micro-batch: config 3's 32 x 2048 tokens


def micro_batch_plan(global_sequences: int, world: int, rank: int) -> tuple[int, int, int]:
    """(first global micro-batch, micro-batches of this rank, micro-batches of the whole step).

    global_sequences > 0 (config 5): the global batch is split by whole sequences (shard_sequences) and each rank
    runs its sequences as 32 x 2048 micro-batches that accumulate into dW; the total work is fixed as N grows.
    global_sequences == 0: one micro-batch per rank (global batch 32 x N; per-GPU work fixed as N grows)."""
    from staleynet_b200.data_parallel import shard_sequences

    if global_sequences == 0:
        return rank, 1, world
    shard = shard_sequences(global_sequences, world, rank)
    if shard.first % MICRO_SEQUENCES or shard.count % MICRO_SEQUENCES or shard.count == 0:
        raise SystemExit(f"--global-batch {global_sequences} over {world} ranks gives rank {rank} sequences "
                         f"[{shard.first}, {shard.first + shard.count}), not whole {MICRO_SEQUENCES}-sequence "
                         f"micro-batches")
    return shard.first // MICRO_SEQUENCES, shard.count // MICRO_SEQUENCES, global_sequences // MICRO_SEQUENCES


def model_shape(name: str, tokens: int):
    """BASELINE config 3's model (12 blocks, width 768, 16 x 1024 head, 32 x 2048 tokens per micro-batch) or config
    1's (6 blocks, width 256, FFN 1024, 4 x 1024 head, 8 x 512 tokens)."""
    from staleynet_b200.step import ModelShape

    if name == "cfg1":
        return ModelShape(blocks=6, width=256, ffn=1024, codebooks=4, codebook_size=1024, tokens=8 * 512)
    return ModelShape(tokens=tokens)


def cublas_rate(device, precision: str, seconds: float = 3.0) -> dict:
    """cuBLAS (torch.matmul) on 8192^3 at the step's precision, as MEASURED_PEAKS.json measures bf16: best of 10
    launches (burst) and back to back for `seconds` (sustained). A comparison figure only; nothing of the step runs
    on cuBLAS."""
    import torch

    n = 8192
    dtype = torch.bfloat16 if precision == "bf16" else torch.float32
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = precision == "tf32"
    try:
        a = torch.randn(n, n, device=device, dtype=dtype)
        b = torch.randn(n, n, device=device, dtype=dtype)
        c = torch.empty(n, n, device=device, dtype=dtype)
        flops = 2.0 * n ** 3
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3)
        reps = max(1, int(seconds / best))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.matmul(a, b, out=c)
        e1.record()
        e1.synchronize()
        sustained = flops * reps / (e0.elapsed_time(e1) / 1e3) / 1e12
        return {"burst_tflops": flops / best / 1e12, "sustained_tflops": sustained,
                "how": f"torch.matmul {precision} {n}^3: best of 10 (burst), {reps} back to back (sustained)"}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def relative_frobenius(expected, actual) -> float:
    import torch

    e = expected.double()
    return float(torch.linalg.vector_norm(actual.double() - e) / torch.clamp(torch.linalg.vector_norm(e), min=1e-300))


def gemm_breakdown(step, ev_steps, peak_sus: float, peak_burst: float) -> dict:
    """Per GEMM of the step: launches, device ms per step, TFLOP/s from the CUDA events around each launch, and
    that rate as a percentage of the measured bf16 peaks."""
    table = {}
    n_steps = len(ev_steps)
    for ev_micro in ev_steps:
        for pairs in ev_micro:
            for (name, flops, _), (a, b) in zip(step.plan, pairs):
                row = table.setdefault(name, {"launches": 0, "ms": 0.0, "flops": 0.0})
                row["launches"] += 1
                row["ms"] += a.elapsed_time(b)
                row["flops"] += flops
    out = {}
    total_ms = sum(r["ms"] for r in table.values())
    for name, row in table.items():
        tflops = row["flops"] / (row["ms"] / 1e3) / 1e12
        out[name] = {"launches_per_step": row["launches"] // n_steps, "ms_per_step": row["ms"] / n_steps,
                     "tflops": tflops, "pct_sustained": 100.0 * tflops / peak_sus,
                     "pct_burst": 100.0 * tflops / peak_burst, "share": row["ms"] / total_ms}
    return out


def run_ours(args, shape, rank: int, world: int, local_rank: int) -> int:
    import torch
    import torch.distributed as dist

    from staleynet_b200.data_parallel import OverlappedAllReduce, global_grad_scale
    from staleynet_b200.step import TrainingStepGemms

    from staleynet_b200 import _ffi

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    precision = {"bf16": _ffi.PRECISION_BF16, "tf32": _ffi.PRECISION_TF32, "f32": _ffi.PRECISION_F32}[args.precision]
    first_micro, n_micro, global_micro = micro_batch_plan(args.global_batch, world, rank)
    # The loss-gradient scale counts the valid targets of the whole global batch (training.rs:214-221 counts the
    # local batch; every target drawn by below(1024) is valid).
    scale = global_grad_scale(n_micro * shape.tokens, shape.codebooks) if world > 1 else \
        1.0 / (n_micro * shape.tokens * shape.codebooks)
    step = TrainingStepGemms(shape, device, micro_batches=n_micro, first_micro_batch=first_micro, grad_scale=scale,
                             deterministic=args.deterministic, precision=precision)
    handle = stream.cuda_stream
    reducer = OverlappedAllReduce(compute_stream=stream) if world > 1 else None

    lib = step.lib

    def on_block(b):
        # The head's gradient is complete before block L-1's; both go out once block L-1's backward is queued. From
        # then on the rest of the backward's GEMMs may run on a reduced grid that leaves the collective its SMs.
        if b == shape.blocks - 1:
            reducer.submit(step.head_grad)
            if args.gemm_sm_budget:
                lib.snb_set_sm_budget(args.gemm_sm_budget)
        reducer.submit(step.block_grad_flat[b])

    # A captured micro-batch holds no collective: with --graph the all-reduces are issued after the backward.
    overlap = world > 1 and args.comm == "overlap" and not args.graph
    hook = on_block if overlap else None

    def finish(marks=None):
        """Ends a step: the compute stream waits for every all-reduce (with --comm after, they are issued here, once
        the whole backward is queued). With `marks` (two events) the exposed communication is bracketed: from the
        last GEMM's completion to the last all-reduce's."""
        if marks is not None:
            marks[0].record(stream)
        if reducer is not None:
            lib.snb_set_sm_budget(0)
            if not overlap:
                for _, t in step.grads.order():
                    reducer.submit(t)
            reducer.wait()
        if marks is not None:
            marks[1].record(stream)

    # Warm-up (also configures every kernel variant and builds the NCCL communicator).
    for _ in range(args.warmup):
        step.run_step(handle, on_block_done=hook)
        finish()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    # Timed region: device-resident inputs.
    n_launch = step.launches_per_step()
    timed = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    comm_marks = [(timed(), timed()) for _ in range(args.steps)]
    # The GEMM launch times of the roofline and of the per-GEMM breakdown come from one step run just before the
    # timed region with events around each launch. The timed steps carry no per-launch events: an event between two
    # GEMMs would make the second wait for the first to finish completely, where otherwise its CTAs start their
    # set-up during the first's tail (programmatic dependent launch).
    ev_pass = [[[(timed(), timed()) for _ in range(n_launch)] for _ in range(n_micro)]]
    step.run_step(handle, events=ev_pass[0])
    finish()
    torch.cuda.synchronize()
    graphs = [step.capture(m) for m in range(n_micro)] if args.graph else None
    if graphs is not None:
        torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = timed(), timed()
    start.record(stream)
    for k in range(args.steps):
        if graphs is None:
            step.run_step(handle, on_block_done=hook)
        else:
            step.zero_grads()
            for g in graphs:
                g.replay()
        finish(comm_marks[k])
    end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    ev_steps = ev_pass
    kernel_ms = sum(a.elapsed_time(b) for ev_micro in ev_pass for pairs in ev_micro for a, b in pairs) * args.steps
    exposed_ms = sum(a.elapsed_time(b) for a, b in comm_marks) / args.steps

    # End-to-end: every micro-batch's input activations come from pinned host memory and the step's per-codebook
    # loss sums are read back (the reference downloads its losses every step, training.rs:232). As a training loop
    # does, the next micro-batch's input is copied on a separate stream into the other of two buffers while the
    # current one runs (every copy starts inside the timed region; the first one is not overlapped).
    host_x = torch.empty(step.inputs.shape, dtype=step.inputs.dtype, pin_memory=True)
    host_x.copy_(step.inputs.cpu())
    host_loss = torch.empty(step.loss_sums.shape, dtype=torch.float32, pin_memory=True)
    h2d = host_x.numel() * host_x.element_size()
    d2h = host_loss.numel() * host_loss.element_size()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = timed(), timed()
    copy_stream = torch.cuda.Stream(device)
    bufs = [torch.empty_like(step.x_in), torch.empty_like(step.x_in)]
    # With --graph, one captured graph per (micro-batch, upload buffer), captured before the timed region.
    e2e_graphs = ({(m, b): step.capture(m, x=bufs[b]) for m in range(n_micro) for b in range(2)}
                  if args.graph else None)
    torch.cuda.synchronize()
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    released = [torch.cuda.Event(), torch.cuda.Event()]
    e_start.record(stream)
    copy_stream.wait_event(e_start)
    total_micro = args.steps * n_micro

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(released[b])   # micro-batch i-2, which read this buffer, has finished
            bufs[b].copy_(host_x[i % n_micro], non_blocking=True)
            ready[b].record(copy_stream)

    upload(0)
    for k in range(args.steps):
        step.zero_grads()
        for m in range(n_micro):
            i = k * n_micro + m
            if i + 1 < total_micro:
                upload(i + 1)
            stream.wait_event(ready[i % 2])
            if e2e_graphs is None:
                step.run(handle, on_block_done=hook if m == n_micro - 1 else None, micro_batch=m, x=bufs[i % 2])
            else:
                e2e_graphs[(m, i % 2)].replay()
            released[i % 2].record(stream)
        finish()
        host_loss.copy_(step.loss_sums, non_blocking=True)
    e_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_ms_total = e_start.elapsed_time(e_end)
    local_loss = float(host_loss.sum()) / (n_micro * shape.tokens * shape.codebooks)

    stats = torch.tensor([ms_total, e2e_ms_total, kernel_ms, exposed_ms], device=device, dtype=torch.float64)
    exposed_min = exposed_ms
    if world > 1:
        low = torch.tensor([exposed_ms], device=device, dtype=torch.float64)
        dist.all_reduce(low, op=dist.ReduceOp.MIN)
        exposed_min = float(low.item())
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms_total, kernel_ms, exposed_max = stats.tolist()

    # Data-parallel parity: the all-reduced gradients of one step against rank 0 recomputing the whole global batch
    # alone through the same kernels (every micro-batch rebuilt from the seeded streams, no collective).
    dp_parity = None
    if world > 1:
        step.run_step(handle, on_block_done=hook)
        finish()
        check_blocks = sorted({0, shape.blocks - 1})
        reduced = [step.head_grad.clone()] + [step.block_grad_flat[b].clone() for b in check_blocks]
        torch.cuda.synchronize()
        if rank == 0:
            step.zero_grads()
            for g in range(global_micro):
                step.load_micro_batch(g, step.inputs[0], step.targets[0])
                step.run(handle, micro_batch=0)
            torch.cuda.synchronize()
            alone = [step.head_grad] + [step.block_grad_flat[b] for b in check_blocks]
            errs = [relative_frobenius(x, r) for x, r in zip(alone, reduced)]
            names = ["head"] + [f"block{b}" for b in check_blocks]
            dp_parity = {"relative_frobenius": dict(zip(names, errs)), "max": max(errs), "tolerance": 1e-2,
                         "ok": max(errs) <= 1e-2,
                         "how": f"all-reduced dW of one step vs rank 0 alone over all {global_micro} micro-batches"}
        dist.barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(shape, budget_flops=args.cpu_sample_flops)
        cpu["single_thread"] = single_thread_baseline(shape, args.cpu_sample_flops / 40)

    attention = None
    if rank == 0 and world == 1 and args.precision == "bf16" and not args.no_attention_record:
        attention = attention_record(device, args.steps, args.warmup)

    cublas = cublas_rate(device, args.precision) if args.precision != "bf16" and rank == 0 else None
    if rank == 0:
        peaks, source = load_peaks()
        traffic = load_traffic(shape) if args.precision == "bf16" else {}
        peak_sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        peak_burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_source = (f"{source} bf16_tflops_sustained (kernel timed inside a long step); burst {peak_burst}")
        if cublas is not None:
            # TF32 and f32 have no driver-measured peak: the same cuBLAS measurement, taken in this run.
            peak_sus, peak_burst = cublas["sustained_tflops"], cublas["burst_tflops"]
            peak_source = f"cuBLAS {args.precision} measured in this run: {cublas['how']}; burst {peak_burst:.1f}"
        flops_rank = step.plan_flops * n_micro
        ms_step = ms_total / args.steps
        value = flops_rank * world * args.steps / (ms_total / 1e3) / 1e12
        e2e_value = flops_rank * world * args.steps / (e2e_ms_total / 1e3) / 1e12
        achieved = flops_rank * args.steps / (kernel_ms / 1e3) / 1e12
        launches = n_launch * n_micro
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if args.global_batch else "weak",
            "vs_baseline": None, "dtype": args.precision,
            "data": "synthetic: " + GENERATOR + f"; activations N(0,1), weights N(0,1/sqrt({shape.width})), "
                                                "targets below(1024)",
            "config": dict(workload_config(shape, world, args.global_batch, n_micro, args.model),
                           precision=args.precision, **({"deterministic": True} if args.deterministic else {}),
                           **({"cuda_graph": "each micro-batch replayed from a captured CUDA graph"}
                              if args.graph else {})),
            f"pct_{args.precision}_peak_sustained": 100.0 * (value / world) / peak_sus,
            f"pct_{args.precision}_peak_burst": 100.0 * (value / world) / peak_burst,
            "roofline": {
                "bound": "fp32-fma" if args.precision == "f32" else "tensor", "achieved": achieved, "peak": peak_sus,
                "unit": "TFLOP/s",
                "frac": achieved / peak_sus, "traffic": traffic.get("traffic_bytes_per_launch"),
                "traffic_source": traffic.get("source"),
                "algorithmic_bytes_per_launch": traffic.get("algorithmic_bytes_per_launch"),
                "achieved_hbm_gbs": (traffic["algorithmic_bytes_per_launch"] * launches * args.steps /
                                     (kernel_ms / 1e3) / 1e9) if "algorithmic_bytes_per_launch" in traffic else None,
                "hbm_peak_gbs": float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])),
                "kernel": ("snb::simt_gemm_kernel (exact f32 FMA)" if args.precision == "f32" else
                           "snb::tc_gemm_kernel / tc_gemm_pair_kernel") + " (all GEMM launches of a step on rank 0, timed by "
                                                                   "events in one step run before the timed region)",
                "peak_source": peak_source,
                "launches_per_step": launches,
                "flops_per_step": flops_rank,
            },
            "gemms": gemm_breakdown(step, ev_steps, peak_sus, peak_burst),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms_total / args.steps,
                    "path": "snb_gemm + snb_codebook_cross_entropy C ABI via ctypes; inputs from pinned host memory, "
                            "per-codebook loss sums read back every step", "loss": local_loss},
            "gpu_launches": (launches + n_micro) * args.steps,
            "clocks": clock_info,
        }
        if world > 1:
            line["communication"] = {
                "exposed_ms_per_step": exposed_max,
                "exposed_ms_per_step_least_rank": exposed_min,
                "what": "per step, from the last GEMM's completion to the last gradient all-reduce's (CUDA events "
                        "on the compute stream; max over ranks, and on the least-exposed rank: the difference is "
                        "the wait for a slower rank)",
                "all_reduce_bytes_per_step": 4 * (sum(t.numel() for t in step.block_grad_flat) +
                                                  step.head_grad.numel()),
                "collective": "NCCL all-reduce (sum, f32) per bucket: head, then blocks L-1..0, on a side stream",
                "mode": ("overlapped with the last micro-batch's backward" if args.comm == "overlap" else
                         "issued after the whole backward is queued") +
                        (f"; GEMM grid capped at {args.gemm_sm_budget} SMs meanwhile" if args.gemm_sm_budget and
                         args.comm == "overlap" else ""),
            }
            line["dp_parity"] = dp_parity
        if attention is not None:
            line["attention_cfg4"] = attention
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "single_thread")}
        print(json.dumps(line), flush=True)
    del step
    return 0


def attention_record(device, steps: int, warmup: int) -> dict:
    """BASELINE config 4's fused causal attention forward + backward, timed on the device after the step (its own
    warm-up, CUDA events and clock samples) so that the default step line carries the attention kernels too."""
    import torch

    from staleynet_b200.attention import AttentionShape, FusedAttention

    stream = torch.cuda.current_stream(device)
    shape = AttentionShape()
    att = FusedAttention(shape, device, seed=0)
    h = stream.cuda_stream
    for _ in range(max(3, warmup)):
        att.forward(h)
        att.backward(h)
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index or 0)
    clocks.start()
    # ~0.5 s of launches, so that the clock sampler (one sample per 100 ms) sees the timed region.
    n = max(600, steps)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n)]
    for e in ev:
        e[0].record(stream)
        att.forward(h)
        e[1].record(stream)
        att.backward(h)
        e[2].record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / n
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / n
    peaks, source = load_peaks()
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    bwd = att.backward_flops / (bwd_ms / 1e3) / 1e12
    record = {
        "workload": f"cfg4 causal attention (batch {shape.batch}, {shape.heads} heads of {shape.head_dim}, sequence "
                    f"{shape.time}) fwd+bwd through snb_causal_attention_forward/backward, bf16",
        "value": att.flops / ((fwd_ms + bwd_ms) / 1e3) / 1e12, "unit": UNIT, "steps": n,
        "forward_ms": fwd_ms, "backward_ms": bwd_ms,
        "backward_roofline": {"bound": "tensor", "achieved": bwd, "peak": peak, "unit": "TFLOP/s",
                              "frac": bwd / peak, "traffic": load_kernel_traffic("fb_backward_kernel"),
                              "peak_source": f"{source} bf16_tflops_sustained"},
        "clocks": clock_info,
    }
    del att
    torch.cuda.empty_cache()
    return record


def run_gemm(args, rank: int, world: int, local_rank: int) -> int:
    """Individual GEMMs of the training step, each timed alone: the step's buffers are built, one full micro-batch
    pass fills every activation and gradient, then each GEMM named in --names (block 0's instance, the head's for
    head.*) is launched --warmup times untimed and --steps times between CUDA events. For profiling one product of
    the step at a chosen token count (e.g. ncu on expand.fwd at 16,384 tokens)."""
    import torch

    from staleynet_b200 import _ffi
    from staleynet_b200.step import TrainingStepGemms

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    precision = {"bf16": _ffi.PRECISION_BF16, "tf32": _ffi.PRECISION_TF32, "f32": _ffi.PRECISION_F32}[args.precision]
    shape = model_shape(args.model, args.tokens)
    step = TrainingStepGemms(shape, device, precision=precision, deterministic=args.deterministic)
    handle = stream.cuda_stream
    step.run(handle)
    torch.cuda.synchronize()
    firsts = {}
    for name, flops, a in step.plan:
        firsts.setdefault(name, (flops, a))
    names = [n for n in args.names.split(",") if n] if args.names else list(firsts)
    unknown = [n for n in names if n not in firsts]
    if unknown:
        raise SystemExit(f"unknown GEMM name(s) {unknown}; the step's are {list(firsts)}")
    h = ctypes.c_void_p(handle)
    lib = _ffi.load()
    results = {}
    clocks = ClockSampler(local_rank)
    clocks.start()
    for name in names:
        flops, a = firsts[name]
        for _ in range(args.warmup):
            if lib.snb_gemm(h, ctypes.byref(a)) != _ffi.OK:
                raise SystemExit(f"{name}: {_ffi.last_error()}")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            lib.snb_gemm(h, ctypes.byref(a))
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        results[name] = {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12, "path": _ffi.last_path(),
                         "m_n_k": [a.product.rows, a.product.cols, a.product.inner]}
    clock_info = clocks.stop()
    if rank == 0:
        peaks, source = load_peaks()
        burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        for r in results.values():
            r["pct_bf16_burst"] = 100.0 * r["tflops"] / burst
        print(json.dumps({"workload": "gemm", "tokens": shape.tokens, "precision": args.precision,
                          "steps": args.steps, "warmup": args.warmup, "gemms": results, "clocks": clock_info,
                          "peak_source": f"{source} bf16_tflops (burst): isolated launches"}), flush=True)
    return 0


def attention_cpu_baseline(s, budget_flops: float = 10e9, threads: int = 0) -> dict:
    """The oracle's reference loop on a sample of rows of each of the six attention products (dense, as the
    reference's CPU matmul computes them), extrapolated by rows; softmax passes are not timed (elementwise)."""
    import numpy as np

    from oracle import oracle as o

    S, d, n = s.time, s.head_dim, s.count
    total_dense = 6 * 2.0 * S * S * d * n
    frac = min(1.0, budget_flops / total_dense)
    products = [(S, S, d, False, True), (S, d, S, False, False), (S, S, d, False, True), (S, d, S, True, False),
                (S, d, S, False, False), (S, d, S, True, False)]
    seconds = 0.0
    used = 1
    for M, N, K, lt, rt in products:
        rows = max(1, int(round(frac * M)))
        left = np.zeros(M * K, np.float32)
        right = np.zeros(K * N, np.float32)
        out = np.zeros(rows * N, np.float32)
        p = o.product(rows, N, K, o.storage_strides(lt, M, K, 0), o.storage_strides(rt, K, N, 0), 0)
        o.matmul_rows(p, 1, left, right, out, 0, rows, threads)
        t0 = time.perf_counter()
        used = o.matmul_rows(p, 1, left, right, out, 0, rows, threads)
        seconds += (time.perf_counter() - t0) * (M / rows) * n
    causal_flops = 6 * 2.0 * s.head_dim * sum(min(q + 1, S) for q in range(S)) * n
    return {"value": causal_flops / seconds / 1e12, "unit": UNIT, "cores": used, "kind": "port",
            "sample": f"{frac:.1e} of the rows of each of the six products of one head (dense f32 loop), "
                      f"extrapolated by rows and heads; softmax passes not included"}


def head_cpu_baseline(tokens: int, width: int, books: int, size: int, budget_flops: float = 10e9,
                      threads: int = 0) -> dict:
    """The oracle's reference loop on a sample of rows of the head GEMM plus reference::cross_entropy of every
    codebook on those rows, extrapolated by rows."""
    import numpy as np

    from oracle import oracle as o

    cols = books * size
    rows = max(1, min(tokens, int(budget_flops / (2.0 * width * cols))))
    x = np.random.default_rng(0).standard_normal(rows * width).astype(np.float32)
    w = np.random.default_rng(1).standard_normal(width * cols).astype(np.float32) / np.float32(width ** 0.5)
    logits = np.zeros(rows * cols, np.float32)
    grad = np.zeros(rows * cols, np.float32)
    losses = np.zeros(rows, np.float32)
    targets = np.random.default_rng(2).integers(0, size, rows * books).astype(np.uint32)
    prod = o.product(rows, cols, width, o.storage_strides(False, rows, width, 0), o.storage_strides(False, width, cols, 0), 0)
    o.matmul_rows(prod, 1, x, w, logits, 0, rows, threads)
    t0 = time.perf_counter()
    used = o.matmul_rows(prod, 1, x, w, logits, 0, rows, threads)
    for c in range(books):
        o.cross_entropy(logits, targets, cols, c * size, size, books, c, 1.0, losses, grad)
    seconds = (time.perf_counter() - t0) * tokens / rows
    return {"value": 2.0 * tokens * width * cols / seconds / 1e12, "unit": UNIT, "cores": used, "kind": "port",
            "sample": f"{rows} of {tokens} rows: head GEMM (all cores) + the 16 codebooks' cross-entropy (one core), "
                      f"extrapolated by rows"}


def run_head(args, rank: int, world: int, local_rank: int) -> int:
    """BASELINE config 3's output layer, forward + loss: logits = x W + b over 16 codebooks of 1024 classes for
    65,536 tokens, then every codebook's softmax cross-entropy and its gradient, and the loss on the host.

    --head-path fused (default): snb_head_cross_entropy — bf16 logits overwritten in place by their gradient, one
    pass, per-codebook loss sums on the device, one 64-byte copy to the host.
    --head-path reference-shaped: the reference's sequence (training.rs:201-235) on this library — the head GEMM
    writes f32 logits, then per codebook snb_cross_entropy (f32 gradient, per-row losses) and a download of the row
    losses summed on the host. `value` counts the head GEMM's FLOPs either way."""
    import torch

    from staleynet_b200.matmul import CrossEntropyHead, DeviceRandom, Gpu, MatmulSpec

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    tokens, width, books, size = args.tokens, 768, 16, 1024
    cols = books * size
    gpu = Gpu(local_rank)
    rng = DeviceRandom(gpu, rank)
    x = rng.normal_(torch.empty(tokens, width, device=device, dtype=torch.bfloat16))
    w = rng.normal_(torch.empty(width, cols, device=device, dtype=torch.bfloat16), 1.0 / width ** 0.5)
    bias = torch.zeros(cols, device=device)
    targets = rng.below_(torch.empty(tokens, books, device=device, dtype=torch.int32), size)
    scales = torch.full((books,), 1.0 / (tokens * books), device=device)
    spec = MatmulSpec.new(tokens, cols, width)
    fused = args.head_path == "fused"
    host_sums = torch.empty(books, dtype=torch.float32, pin_memory=True)
    host_rows = torch.empty(tokens, dtype=torch.float32, pin_memory=True)
    if fused:
        logits = torch.empty(tokens, cols, device=device, dtype=torch.bfloat16)
        loss_sums = torch.empty(books, device=device)
    else:
        logits = torch.empty(tokens, cols, device=device)
        grad = torch.empty(tokens, cols, device=device)
        row_losses = torch.empty(tokens, device=device)

    def step():
        if fused:
            gpu.head_cross_entropy(spec, x, w, logits, targets, books, scales, loss_sums, logits, bias=bias)
            host_sums.copy_(loss_sums, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return float(host_sums.sum()) / tokens / books
        gpu.gemm(spec, x, w, logits, bias=bias)
        total = 0.0
        for c in range(books):
            gpu.cross_entropy(logits, targets, CrossEntropyHead(c * size, size, books, c, 1.0 / (tokens * books)),
                              row_losses, grad)
            host_rows.copy_(row_losses, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            total += float(host_rows.sum()) / tokens
        return total / books

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The dominant kernels: the head GEMM alone (same output type), timed over the same number of launches.
    ge0, ge1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ge0.record(stream)
    for _ in range(args.steps):
        gpu.gemm(spec, x, w, logits, bias=bias)
    ge1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = ge0.elapsed_time(ge1) / args.steps
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    loss = 0.0
    for _ in range(args.steps):
        loss = step()
    end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    if rank != 0:
        return 0
    peaks, source = load_peaks()
    flops = 2.0 * tokens * width * cols
    ce_ms = max(ms - gemm_ms, 1e-6)
    logit_bytes = tokens * cols * (2 if fused else 4)
    ce_bytes = logit_bytes * 2 + tokens * books * 4   # logits read once, gradient written once, targets
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    line = {
        "metric": METRIC, "value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: " + GENERATOR + "; activations N(0,1), weights N(0,1/sqrt(768)), targets below(1024)",
        "config": {"workload": "cfg3 output layer forward + loss: 65,536 tokens x 768 -> 16 codebooks x 1024, "
                               "softmax cross-entropy with gradient, loss on the host",
                   "head_path": args.head_path, "tokens": tokens, "width": width, "codebooks": books,
                   "codebook_size": size, "l2": "inputs larger than L2 (logits 2.1 GB bf16 / 4.3 GB f32)"},
        "roofline": {"bound": "hbm", "kernel": "cross_entropy_kernel (step time minus the head GEMM's own time)",
                     "achieved": ce_bytes / (ce_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": ce_bytes / (ce_ms / 1e3) / 1e9 / hbm,
                     "traffic": load_profile_traffic("cross_entropy_cfg3_kernel.json", "cross_entropy_kernel")
                     if fused and tokens == 65536 else None,
                     "algorithmic_bytes_per_step": ce_bytes, "peak_source": f"{source} hbm_gbs",
                     "head_gemm_ms": gemm_ms, "loss_ms": ce_ms,
                     "head_gemm_tflops": flops / (gemm_ms / 1e3) / 1e12},
        "e2e": {"value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": books * 4 if fused else books * tokens * 4,
                "note": "the loss reaches the host inside every timed step; operands are resident"},
        "gpu_launches": (2 if fused else 1 + books) * args.steps, "clocks": clock_info, "loss": loss,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = head_cpu_baseline(tokens, width, books, size)
    print(json.dumps(line), flush=True)
    return 0


def model_parameter_shapes(s) -> list:
    """(name, elements, decayed) of every parameter of the BASELINE config 3 model (gpt.rs; weights decayed, gains,
    biases and embeddings exempt as parameter.rs marks them): token and position embeddings, per block two RMSNorm
    gains and four linears with biases, the final norm and the 16 x 1024 head."""
    out = [("token_embedding", s.codebooks * s.codebook_size * s.width, False),
           ("position_embedding", 2048 * s.width, False)]
    from staleynet_b200.step import linear_shapes

    for b in range(s.blocks):
        out.append((f"block{b}.attention_norm.gain", s.width, False))
        out.append((f"block{b}.ffn_norm.gain", s.width, False))
        for name, i, o in linear_shapes(s):
            out.append((f"block{b}.{name}.weight", i * o, True))
            out.append((f"block{b}.{name}.bias", o, False))
    out.append(("final_norm.gain", s.width, False))
    out.append(("head.weight", s.width * s.head_width, True))
    out.append(("head.bias", s.head_width, False))
    return out


def run_optimizer(args, rank: int, world: int, local_rank: int) -> int:
    """The optimizer step of BASELINE config 3's model (~111.5 M parameters): global gradient norm, clip, AdamW.

    --optimizer-path multi (default): snb_adamw_step_multi — two launches, the clip factor on the device.
    --optimizer-path reference-shaped: AdamW::step's sequence (model optimizer.rs:125-177) on this library — per
    tensor snb_sum_of_squares and a host read of it, then per tensor the gradient scaled and snb_adamw_step."""
    import torch

    from staleynet_b200.matmul import AdamWHyperparameters, DeviceRandom, Gpu
    from staleynet_b200.step import ModelShape

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    shapes = model_parameter_shapes(ModelShape())
    gpu = Gpu(local_rank)
    rng = DeviceRandom(gpu, rank)
    tensors = []
    for _, n, decayed in shapes:
        p = rng.normal_(torch.empty(n, device=device), 0.02)
        grad = rng.normal_(torch.empty(n, device=device), 1e-3)
        tensors.append((p, grad, torch.zeros(n, device=device), torch.zeros(n, device=device), 0.1 if decayed else 0.0))
    elements = sum(n for _, n, _ in shapes)
    multi = args.optimizer_path == "multi"
    square_sum = torch.zeros(1, device=device, dtype=torch.float64)
    host = torch.empty(1, dtype=torch.float64, pin_memory=True)
    state = {"step": 0}

    def step():
        state["step"] += 1
        if multi:
            gpu.adamw_step_multi(tensors, AdamWHyperparameters(3e-4, 0.9, 0.95, 1e-8, 0.0, state["step"]), 1.0,
                                 square_sum)
            return
        total = 0.0
        for _, grad, _, _, _ in tensors:
            gpu.sum_of_squares(grad, square_sum)
            host.copy_(square_sum, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            total += float(host)
        norm = total ** 0.5
        clip = 1.0 / norm if norm > 1.0 else 1.0
        for p, grad, m, v, wd in tensors:
            if clip != 1.0:
                grad.mul_(clip)   # the reference's gpu.scale pass (a torch op here: it is not this library's path)
            gpu.adamw_step(p, grad, m, v, AdamWHyperparameters(3e-4, 0.9, 0.95, 1e-8, wd, state["step"]))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    if rank != 0:
        return 0
    peaks, source = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    algorithmic = elements * 4 * (1 + 7)   # sum of squares reads the gradient; AdamW reads 4 and writes 3 arrays
    line = {
        "metric": "optimizer step (global norm + clip + AdamW) time", "value": ms, "unit": "ms",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic: " + GENERATOR + "; parameters N(0,0.02), gradients N(0,1e-3)",
        "config": {"workload": "cfg3 model optimizer step: 111.5 M f32 parameters in "
                               f"{len(shapes)} tensors, gradient-norm clip at 1.0, AdamW", "optimizer_path":
                   args.optimizer_path, "parameters": elements, "tensors": len(shapes),
                   "l2": "inputs larger than L2 (1.8 GB of parameters, gradients and moments)"},
        "roofline": {"bound": "hbm", "kernel": "multi_adamw_kernel + multi_sum_of_squares_kernel" if multi else
                     "sum_of_squares_kernel + adamw_kernel per tensor",
                     "achieved": algorithmic / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": algorithmic / (ms / 1e3) / 1e9 / hbm,
                     "traffic": profile_traffic_sum("norm_optim_cfg3_kernels.json",
                                                    ("multi_adamw_kernel", "multi_sum_of_squares_kernel"))
                     if multi else None, "traffic_unit": "DRAM bytes per step (ncu, profiles/norm_optim_cfg3_kernels.md)",
                     "algorithmic_bytes_per_step": algorithmic, "peak_source": f"{source} hbm_gbs"},
        "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0 if multi else 8 * len(shapes)},
        "gpu_launches": (2 if multi else 2 * len(shapes)) * args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_norm(args, rank: int, world: int, local_rank: int) -> int:
    """RMSNorm into the next GEMM at BASELINE config 3 (65,536 tokens, 768 -> 2304, the QKV product):
    --norm-path fused (default): snb_rms_norm_stats (1/rms only) + the GEMM on the raw rows with row_scale and the
    gain folded into the weights; --norm-path unfused: the normalised rows written as bf16, then the GEMM."""
    import torch

    from staleynet_b200.matmul import DeviceRandom, Gpu, MatmulSpec

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    tokens, width, cols, eps = args.tokens, 768, 2304, 1e-5
    gpu = Gpu(local_rank)
    rng = DeviceRandom(gpu, rank)
    x = rng.normal_(torch.empty(tokens, width, device=device, dtype=torch.bfloat16))
    gain = 1.0 + rng.normal_(torch.empty(width, device=device), 0.1)
    w = rng.normal_(torch.empty(width, cols, device=device, dtype=torch.bfloat16), 1.0 / width ** 0.5)
    bias = torch.zeros(cols, device=device)
    y = torch.empty(tokens, cols, device=device, dtype=torch.bfloat16)
    inv = torch.empty(tokens, device=device)
    spec = MatmulSpec.new(tokens, cols, width)
    fused = args.norm_path == "fused"
    wg = torch.empty_like(w)
    gpu.scale_rows(gain, w, wg)      # once per optimizer step, not per use
    xn = torch.empty_like(x)

    def step():
        if fused:
            gpu.rms_norm_stats(x, eps, inv)
            gpu.gemm(spec, x, wg, y, bias=bias, row_scale=inv)
        else:
            gpu.rms_norm_stats(x, eps, inv, gain=gain, output=xn)
            gpu.gemm(spec, xn, w, y, bias=bias)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    if rank != 0:
        return 0
    peaks, source = load_peaks()
    flops = 2.0 * tokens * width * cols
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    line = {
        "metric": METRIC, "value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: " + GENERATOR + "; rows N(0,1), gains 1 + N(0,0.1), weights N(0,1/sqrt(768))",
        "config": {"workload": "cfg3 RMSNorm + QKV product: 65,536 x 768 -> 2304", "norm_path": args.norm_path,
                   "tokens": tokens, "l2": "inputs larger than L2 (y: 302 MB bf16)"},
        "roofline": {"bound": "tensor", "kernel": "tc_gemm_kernel with row_scale (+ rms statistics)",
                     "achieved": flops / (ms / 1e3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": flops / (ms / 1e3) / 1e12 / peak,
                     "traffic": profile_traffic_sum("norm_optim_cfg3_kernels.json",
                                                    ("tc_gemm_kernel", "rms_norm_forward_kernel"))
                     if args.norm_path == "fused" and tokens == 65536 else None,
                     "traffic_unit": "DRAM bytes per step (ncu, profiles/norm_optim_cfg3_kernels.md)",
                     "peak_source": f"{source} bf16_tflops"},
        "e2e": {"value": flops / (ms / 1e3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 2 * args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_attention(args, rank: int, world: int, local_rank: int) -> int:
    """one causal attention forward + backward per step (batch 8, 12 heads of 64, sequence 3072).

    --attention-path fused (default): snb_causal_attention_forward + snb_causal_attention_backward, no [S, S] tensor.
    --attention-path materialised: the six batched products with the fp32 causal softmax and its backward between
    them, as the reference computes them. `value` counts the six products' causal FLOPs either way."""
    import torch

    from staleynet_b200.attention import AttentionProducts, AttentionShape, FusedAttention

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    shape = AttentionShape()
    fused = args.attention_path == "fused"
    att = FusedAttention(shape, device, seed=rank) if fused else AttentionProducts(shape, device, seed=rank)
    h = stream.cuda_stream
    for _ in range(args.warmup):
        att.forward(h)
        att.backward(h)
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The dominant kernel's launches are bracketed by their own events on the same stream.
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start.record(stream)
    for i in range(args.steps):
        if fused:
            att.forward(h)
            marks[i][0].record(stream)
            att.backward(h)
            marks[i][1].record(stream)
        else:
            att.forward(h)
            att.backward(h)
    end.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end)
    inputs = (att.q, att.k, att.v, att.d_out)
    host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in inputs]
    for hb, t in zip(host, inputs):
        hb.copy_(t.cpu())
    host_out = torch.empty(1, dtype=torch.float32, pin_memory=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for hb, t in zip(host, inputs):
            t.copy_(hb, non_blocking=True)
        att.forward(h)
        att.backward(h)
        host_out.copy_(att.dq.view(-1)[:1], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if rank != 0:
        return 0
    peaks, source = load_peaks()
    sec = ms / 1e3 / args.steps
    if fused:
        bwd_sec = sum(a.elapsed_time(b) for a, b in marks) / 1e3 / args.steps
        peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops"]))
        achieved = att.backward_flops / bwd_sec / 1e12
        traffic = load_kernel_traffic("fb_backward_kernel")
        roofline = {"bound": "tensor", "kernel": "fb_backward_kernel (+ its row-statistics kernel and dQ memset)",
                    "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic, "algorithmic_flops_per_launch": att.backward_flops,
                    "peak_source": f"{source} bf16_tflops_sustained", "ms_per_launch": bwd_sec * 1e3,
                    "forward_ms_per_launch": (ms / args.steps) - bwd_sec * 1e3}
        workload = ("cfg4 causal attention fwd+bwd through the fused entry points snb_causal_attention_forward/"
                    "backward (QK^T, online softmax, P.V; then P rebuilt from the log-sum-exp, dP, dV, dS, dQ, dK), "
                    "no [S, S] tensor")
        l2 = "inputs 96 x 3072 x 64 bf16 per tensor (38 MB each); every K/V tile is re-read from L2 by the query tiles"
    else:
        hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        achieved = att.bytes / sec / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": None, "algorithmic_bytes_per_step": att.bytes, "peak_source": f"{source} hbm_gbs"}
        workload = ("cfg4 batched causal attention products fwd+bwd (QK^T, P.V, dO.V^T, P^T.dO, dS.K, dS^T.Q) with "
                    "fp32 causal softmax and its backward between them")
        l2 = "inputs larger than L2 (scores 3.6 GB)"
    line = {
        "metric": METRIC, "value": att.flops / sec / 1e12, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic: " + GENERATOR + "; Q, K, V, dO N(0,1) in bf16",
        "config": {"workload": workload, "attention_path": args.attention_path,
                   "batch": shape.batch, "heads": shape.heads, "head_dim": shape.head_dim, "seq_len": shape.time,
                   "flops": "causal (visible query-key pairs) count of the six products", "l2": l2},
        "roofline": roofline,
        "e2e": {"value": att.flops / (e2e_ms / 1e3 / args.steps) / 1e12, "unit": UNIT,
                "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in host), "d2h_bytes_per_step": 4},
        "gpu_launches": att.launches() * args.steps, "clocks": clock_info,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = attention_cpu_baseline(shape)
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=32 * 2048, help="tokens per GPU (default: BASELINE config 3)")
    ap.add_argument("--cpu-sample-flops", type=float, default=40e9)
    ap.add_argument("--precision", choices=["bf16", "tf32", "f32"], default="bf16",
                    help="step workload: bf16 tensors on bf16 tensor cores (default); f32 tensors on TF32 tensor cores "
                         "(the reference's MatmulKernel::TensorCore); f32 tensors on the exact-f32 SIMT kernel "
                         "(MatmulKernel::Blocked)")
    ap.add_argument("--model", choices=["cfg3", "cfg1"], default="cfg3",
                    help="step workload's model: BASELINE config 3 (default; config 5 over GPUs) or config 1")
    ap.add_argument("--graph", action="store_true",
                    help="step workload: each micro-batch's launches captured once into a CUDA graph and replayed "
                         "(at N > 1 the all-reduces then follow the backward)")
    ap.add_argument("--comm", choices=["overlap", "after"], default="overlap",
                    help="N > 1: all-reduce each gradient bucket while the last micro-batch's backward runs "
                         "(overlap) or all of them once the backward is queued (after)")
    ap.add_argument("--gemm-sm-budget", type=int, default=0,
                    help="N > 1 with --comm overlap: SMs the GEMM grid may use while the all-reduces run (0: all)")
    ap.add_argument("--deterministic", action="store_true",
                    help="step workload: every GEMM with SNB_GEMM_DETERMINISTIC (fixed-order split-K sums)")
    ap.add_argument("--global-batch", type=int, default=256,
                    help="sequences of 2048 tokens per step over all GPUs (config 5: 256, run as 32-sequence "
                         "micro-batches); 0 = one 32-sequence micro-batch per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-attention-record", action="store_true",
                    help="step workload at N = 1: leave out the config-4 fused attention sub-record")
    ap.add_argument("--names", default="", help="gemm workload: comma-separated GEMMs of the step (default: all)")
    ap.add_argument("--workload", choices=["step", "attention", "head", "optimizer", "norm", "gemm"], default="step",
                    help="step: the cfg3 training-step GEMMs (default); attention: the cfg4 attention layer; "
                         "head: the cfg3 output layer's forward + cross-entropy; optimizer: the cfg3 AdamW step; "
                         "norm: RMSNorm into the QKV product; gemm: single products of the step (--names)")
    ap.add_argument("--attention-path", choices=["fused", "materialised"], default="fused",
                    help="attention workload: fused entry points (default) or the six materialised products")
    ap.add_argument("--head-path", choices=["fused", "reference-shaped"], default="fused",
                    help="head workload: snb_head_cross_entropy (default) or the reference's per-codebook sequence")
    ap.add_argument("--optimizer-path", choices=["multi", "reference-shaped"], default="multi")
    ap.add_argument("--norm-path", choices=["fused", "unfused"], default="fused")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

    shape = model_shape(args.model, args.tokens)
    if args.model == "cfg1":
        args.global_batch = 0   # config 1 is one 8 x 512 micro-batch per GPU
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, shape, rank, world)

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        # NCCL writes its version banner and warnings to the C stdout (fd 1) when NCCL_DEBUG is set. Rank 0's
        # stdout carries only the result line: Python keeps the original stdout, and fd 1 now points at stderr.
        sys.stdout.flush()
        sys.stdout = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "attention":
            return run_attention(args, rank, world, local_rank)
        if args.workload == "head":
            return run_head(args, rank, world, local_rank)
        if args.workload == "optimizer":
            return run_optimizer(args, rank, world, local_rank)
        if args.workload == "norm":
            return run_norm(args, rank, world, local_rank)
        if args.workload == "gemm":
            return run_gemm(args, rank, world, local_rank)
        return run_ours(args, shape, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
