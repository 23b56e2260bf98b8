"""Host logic of the data-parallel step (staleynet_b200/data_parallel.py) on CPU: sequence sharding, 2-rank gloo
all-reduce of per-block gradient buckets against the single-process gradients (the reference's f32 GEMM loop on
the whole batch), the global loss-gradient scale (crates/staleynet-model/src/training.rs:214-221), and a rank that
leaves between steps being reported by the host-side heartbeat before the survivors launch the next step."""
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

sys.path.insert(0, str(Path(__file__).resolve().parent))
import dp_workers  # noqa: E402

from staleynet_b200.data_parallel import shard_sequences  # noqa: E402


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("global_seq,world", [(256, 8), (256, 1), (7, 3), (2, 4)])
def test_sequences_are_split_whole_and_cover_the_batch(global_seq, world):
    shards = [shard_sequences(global_seq, world, r) for r in range(world)]
    assert sum(s.count for s in shards) == global_seq
    pos = 0
    for s in shards:
        assert s.first == pos
        pos += s.count
    assert max(s.count for s in shards) - min(s.count for s in shards) <= 1


def run_ranks(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        results.append(q.get(timeout=timeout))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def test_two_rank_gradients_equal_the_single_process_gradients():
    (status, err, scale, expected_scale), = run_ranks(dp_workers.gradient_parity)
    assert status == "ok", err
    assert err < 1e-5
    assert scale == pytest.approx(expected_scale, rel=1e-12)


def test_the_heartbeat_reports_a_rank_that_left_between_steps():
    (status, detail), = run_ranks(dp_workers.heartbeat_detects_a_departed_rank, timeout=60)
    assert status == "peer lost", detail
    assert "snb/ready/1/1" in detail


def test_a_collective_past_its_deadline_is_an_error_not_a_hang():
    (status, seconds, *detail), = run_ranks(dp_workers.collective_deadline_is_an_error, timeout=90)
    assert status == "collective failed", (status, detail)
    assert seconds < 30, seconds


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_micro_batches_tile_the_global_batch(world):
    # 256 sequences of 2048 tokens split over `world` ranks, each rank running 32-sequence
    # micro-batches; every micro-batch of the step belongs to exactly one rank, in order.
    import bench

    plans = [bench.micro_batch_plan(256, world, r) for r in range(world)]
    assert all(total == 8 for _, _, total in plans)
    seen = []
    for first, count, _ in plans:
        seen.extend(range(first, first + count))
    assert seen == list(range(8))
    assert bench.micro_batch_plan(0, world, world - 1) == (world - 1, 1, world)


def test_config5_rejects_a_split_into_partial_micro_batches():
    import bench

    with pytest.raises(SystemExit):
        bench.micro_batch_plan(256, 3, 0)
