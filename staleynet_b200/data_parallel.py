"""Data-parallel training step over the GEMM path: one process per GPU, token batch split by whole sequences, weight
gradients summed across ranks with one all-reduce per block, issued in the order backward produces them.

The reference trains on one GPU (crates/staleynet-cuda/src/device.rs:147-155; `open_gpu` opens device 0,
crates/staleynet-cli/src/commands/mod.rs:17-19); this is the multi-GPU extension its gradient accumulation
(`accumulate` GEMMs, crates/staleynet-model/src/layers/linear.rs:55-57) makes natural: dW = X^T dY is a sum over
tokens, so per-rank partial dW summed over ranks equals the single-process dW of the whole batch.

Parity rules kept from the reference's training step:
  * the loss gradient scale 1 / (valid targets x codebooks) (crates/staleynet-model/src/training.rs:214-221) must
    use the GLOBAL valid-target count, summed over ranks before the backward pass (`global_grad_scale`);
  * the global gradient norm (crates/staleynet-model/src/optimizer.rs:167-179) is taken after the all-reduce.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    """Sequences [first, first + count) of the global batch belong to this rank."""

    first: int
    count: int


def shard_sequences(global_sequences: int, world: int, rank: int) -> Shard:
    """Splits the global batch by whole sequences (attention stays rank-local); the first `global % world` ranks
    take one extra sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    base, extra = divmod(global_sequences, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return Shard(first, count)


def global_grad_scale(local_valid_targets: int, codebooks: int, group=None) -> float:
    """1 / (valid targets x codebooks) over the whole global batch (training.rs:214-221 computes it from the
    local batch; with data parallelism the count is summed over ranks first)."""
    import torch
    import torch.distributed as dist

    count = torch.tensor([float(local_valid_targets)], dtype=torch.float64)
    if dist.is_available() and dist.is_initialized():
        backend = dist.get_backend(group)
        if backend == "nccl":
            count = count.cuda()
        dist.all_reduce(count, op=dist.ReduceOp.SUM, group=group)
    total = float(count.item())
    if total <= 0:
        return 0.0
    return 1.0 / (total * codebooks)


class GradientBuckets:
    """Weight gradients of each block as views of one flat f32 buffer, so a block's gradients are all-reduced
    with one collective. Buckets are named and ordered as backward produces them: the head first, then blocks
    L-1 ... 0 (training.rs:247-274)."""

    def __init__(self, block_sizes: list[list[int]], head_size: int, device, dtype=None):
        import torch

        dtype = dtype or torch.float32
        self.flat = []
        self.views = []
        for sizes in block_sizes:
            flat = torch.zeros(sum(sizes), device=device, dtype=dtype)
            views, off = [], 0
            for n in sizes:
                views.append(flat[off:off + n])
                off += n
            self.flat.append(flat)
            self.views.append(views)
        self.head = torch.zeros(head_size, device=device, dtype=dtype)

    def order(self) -> list:
        """(label, tensor) in all-reduce order."""
        out = [("head", self.head)]
        for b in reversed(range(len(self.flat))):
            out.append((f"block{b}", self.flat[b]))
        return out

    def zero_(self) -> None:
        for f in self.flat:
            f.zero_()
        self.head.zero_()


class OverlappedAllReduce:
    """Issues each bucket's all-reduce on a side stream as soon as the compute stream has produced it, so the
    transfer over NVLink overlaps the remaining backward GEMMs; `wait()` makes the compute stream wait for all of
    them (the optimizer step reads the reduced gradients)."""

    def __init__(self, compute_stream=None, group=None):
        import torch

        self.group = group
        self.compute = compute_stream
        self.side = torch.cuda.Stream() if torch.cuda.is_available() and compute_stream is not None else None
        self.works = []

    def submit(self, tensor) -> None:
        import torch
        import torch.distributed as dist

        if self.side is None:
            self.works.append(dist.all_reduce(tensor, group=self.group, async_op=True))
            return
        ready = torch.cuda.Event()
        ready.record(self.compute)
        with torch.cuda.stream(self.side):
            self.side.wait_event(ready)
            self.works.append(dist.all_reduce(tensor, group=self.group, async_op=True))

    def wait(self, timeout_s: float | None = None) -> None:
        """Waits for every submitted all-reduce. With `timeout_s`, one that has not completed by then (a peer
        stopped taking part) raises CollectiveFailed instead of blocking: the caller then tears the process group
        down, since its communicator may still hold the collective."""
        import datetime

        works, self.works = self.works, []
        try:
            for w in works:
                if timeout_s is None:
                    w.wait()
                else:
                    w.wait(datetime.timedelta(seconds=timeout_s))
        except Exception as e:  # the backend raises its own error types for a timed-out or aborted collective
            raise CollectiveFailed(f"gradient all-reduce not complete within {timeout_s} s: {e}") from e


class CollectiveFailed(RuntimeError):
    """A gradient all-reduce did not complete within its deadline."""


class PeerLost(RuntimeError):
    """A peer rank did not reach the next step within the heartbeat timeout."""


class StepHeartbeat:
    """Host-side liveness check between steps. Before issuing any collective of step k a rank posts
    `ready/<rank>/<k>` to a key-value store and waits, bounded, for every peer's post; a rank that has left (between
    steps, with none of its kernels or collectives in flight) is detected here, on the host, before the survivors
    launch work that would wait on it."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = timeout_s

    def ready(self, step: int) -> None:
        import datetime

        self.store.set(f"snb/ready/{self.rank}/{step}", "1")
        keys = [f"snb/ready/{r}/{step}" for r in range(self.world) if r != self.rank]
        if not keys:
            return
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:  # the store raises its own timeout error type
            missing = [k for k in keys if not self.store.check([k])]
            raise PeerLost(f"step {step}: no heartbeat from {missing} within {self.timeout_s} s") from e
