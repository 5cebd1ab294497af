"""Multi-rank host logic on CPU (gloo, world size 2): sequence sharding and the single final
token gather that `bench.py --gpus N` runs over NCCL, plus a rank that leaves before the
gather (the survivors fail with the process group's timeout instead of hanging).

No GPU is touched: each rank's "generated" block is a deterministic function of (global
sequence, step), so the gathered matrix can be checked exactly."""
import multiprocessing as mp
import socket
import time

import numpy as np
import pytest

from ane.shard import gather_tokens, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens_for(seqs, steps):
    return np.array([[1000 * s + k for s in seqs] for k in range(steps)], np.int32).reshape(steps, len(seqs))


def _worker(rank, world, port, n_total, steps, leave_early, q):
    import datetime
    import os

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
        own = shard_range(n_total, world, rank)
        local = _tokens_for(list(own), steps)
        if leave_early and rank == world - 1:
            q.put((rank, "left", None))
            q.close()
            q.join_thread()  # flush the message before the hard exit
            os._exit(0)  # leaves between steps: nothing of its own is in flight
        t0 = time.time()
        try:
            out = gather_tokens(local, n_total)
            q.put((rank, "ok", out.tolist()))
        except Exception as e:  # noqa: BLE001 - the error type depends on the backend
            q.put((rank, "error", f"{type(e).__name__} after {time.time() - t0:.1f}s"))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "setup-error", repr(e)))


def _run(world, n_total, steps, leave_early=False, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, steps, leave_early, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            r, status, payload = q.get(timeout=max(0.1, deadline - time.time()))
            results[r] = (status, payload)
        except Exception:  # noqa: BLE001 - queue.Empty
            break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
            p.join()
    return results


def test_shard_range_partitions_every_job():
    for world in range(1, 9):
        for n in range(0, 40):
            parts = [shard_range(n, world, r) for r in range(world)]
            flat = [i for p in parts for i in p]
            assert flat == list(range(n))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)
    # 2048 sequences over 8 GPUs -> 256 each
    assert [len(shard_range(2048, 8, r)) for r in range(8)] == [256] * 8
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


@pytest.mark.parametrize("n_total", [8, 5])
def test_gather_tokens_two_ranks(n_total):
    steps = 3
    res = _run(2, n_total, steps)
    want = _tokens_for(list(range(n_total)), steps)
    assert sorted(res) == [0, 1], res
    for r in (0, 1):
        status, payload = res[r]
        assert status == "ok", (r, status, payload)
        np.testing.assert_array_equal(np.array(payload, np.int32), want)


def test_rank_leaving_before_gather_fails_survivor_within_timeout():
    t0 = time.time()
    res = _run(2, 6, 2, leave_early=True)
    assert res.get(1, (None,))[0] == "left", res
    status, payload = res.get(0, (None, None))
    assert status == "error", res
    assert time.time() - t0 < 60


def test_library_shard_range_equals_python_partition():
    from ane.shard import library_shard_range
    for n_total in (0, 1, 7, 2048, 2049):
        for world in (1, 2, 3, 8):
            for r in range(world):
                assert library_shard_range(n_total, world, r) == shard_range(n_total, world, r)
