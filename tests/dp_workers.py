"""Worker functions for the 2-rank gloo tests of staleynet_b200.data_parallel (run in spawned processes)."""
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def gradient_parity(rank, world, port, result_queue):
    """Each rank computes its sequences' partial dW += X^T dY (oracle GEMM, the reference's loop), the buckets are
    all-reduced, and rank 0 compares with the single-process dW of the whole batch."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle import oracle as o
    from staleynet_b200.data_parallel import GradientBuckets, OverlappedAllReduce, global_grad_scale, shard_sequences

    _init(rank, world, port)
    try:
        sequences, time, width, outputs, blocks = 6, 16, 12, 20, 3
        rng = o.Random(7)
        xs = [rng.normals(sequences * time * width) for _ in range(blocks)]
        dys = [rng.normals(sequences * time * outputs) for _ in range(blocks)]
        shard = shard_sequences(sequences, world, rank)
        tokens = shard.count * time
        lo = shard.first * time
        buckets = GradientBuckets([[width * outputs]] * blocks, width * outputs, "cpu")
        reducer = OverlappedAllReduce()
        for b in reversed(range(blocks)):
            x = np.ascontiguousarray(xs[b].reshape(-1, width)[lo:lo + tokens]).ravel()
            dy = np.ascontiguousarray(dys[b].reshape(-1, outputs)[lo:lo + tokens]).ravel()
            dw = np.zeros(width * outputs, np.float32)
            p = o.product(width, outputs, tokens, o.storage_strides(True, width, tokens, 0),
                          o.storage_strides(False, tokens, outputs, 0), 0, 1.0, True)
            o.matmul(p, 1, x, dy, dw)
            buckets.views[b][0].copy_(torch.from_numpy(dw))
            reducer.submit(buckets.flat[b])
        reducer.wait()
        # valid targets: rank-local counts differ; the scale must use their global sum
        scale = global_grad_scale(local_valid_targets=tokens - rank, codebooks=4)
        if rank == 0:
            errs = []
            for b in range(blocks):
                full = np.zeros(width * outputs, np.float32)
                T = sequences * time
                p = o.product(width, outputs, T, o.storage_strides(True, width, T, 0),
                              o.storage_strides(False, T, outputs, 0), 0, 1.0, True)
                o.matmul(p, 1, xs[b], dys[b], full)
                errs.append(o.relative_error(full, buckets.flat[b].numpy()))
            total_valid = sum(shard_sequences(sequences, world, r).count * time - r for r in range(world))
            result_queue.put(("ok", max(errs), scale, 1.0 / (total_valid * 4)))
    except Exception as e:  # noqa: BLE001
        result_queue.put(("error", repr(e), None, None))
        raise
    finally:
        dist.destroy_process_group()


def heartbeat_detects_a_departed_rank(rank, world, port, result_queue):
    """Step 0 completes on both ranks; rank 1 leaves; rank 0 learns of it from the store before launching step 1."""
    import datetime

    import torch.distributed as dist

    from staleynet_b200.data_parallel import PeerLost, StepHeartbeat

    store = dist.TCPStore("127.0.0.1", port, world, is_master=(rank == 0), timeout=datetime.timedelta(seconds=30))
    hb = StepHeartbeat(store, rank, world, timeout_s=2.0)
    hb.ready(0)
    if rank == 1:
        os._exit(0)
    try:
        hb.ready(1)
        result_queue.put(("no error", None))
    except PeerLost as e:
        result_queue.put(("peer lost", str(e)))
    result_queue.close()
    result_queue.join_thread()  # deliver the result before this process ends


def collective_deadline_is_an_error(rank, world, port, result_queue):
    """Step 0's all-reduce completes on both ranks; in step 1 rank 1 takes no part, and rank 0's bounded wait turns
    the missing peer into CollectiveFailed after its deadline instead of blocking."""
    import time

    import torch
    import torch.distributed as dist

    from staleynet_b200.data_parallel import CollectiveFailed, OverlappedAllReduce

    _init(rank, world, port)
    store = dist.distributed_c10d._get_default_store()
    try:
        reducer = OverlappedAllReduce()
        t = torch.full((1024,), float(rank + 1))
        reducer.submit(t)
        reducer.wait(timeout_s=20.0)
        assert float(t[0]) == 3.0
        if rank == 1:
            store.wait(["snb/test/done"], datetime.timedelta(seconds=60))   # stays alive, joins nothing
            return
        reducer.submit(torch.ones(1024))
        t0 = time.time()
        try:
            reducer.wait(timeout_s=2.0)
            result_queue.put(("no error", time.time() - t0))
        except CollectiveFailed as e:
            result_queue.put(("collective failed", time.time() - t0, str(e)[:80]))
        finally:
            store.set("snb/test/done", "1")
    except Exception as e:  # noqa: BLE001
        result_queue.put(("error", repr(e)))
        raise
