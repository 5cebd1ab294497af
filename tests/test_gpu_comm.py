"""The library's communicator and token gather (llm_comm_* / llm_gather_tokens, NCCL inside
libllm_cuda.so), through the C ABI.

One rank on one GPU always runs; two ranks (child processes, one GPU each) run when the box has
two GPUs, including a rank that never joins: the other rank's communicator set-up then fails
with an error within the timeout (no collective is in flight; NVLS off)."""
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

from ane import _abi
from ane.shard import Comm, shard_range

pytestmark = pytest.mark.gpu


def _tokens(n_total, world, rank, steps):
    own = shard_range(n_total, world, rank)
    return (np.arange(steps)[:, None] * 10000 + np.arange(own.start, own.stop)[None, :]).astype(np.int32)


def test_single_rank_gather_returns_the_block():
    c = Comm(Comm.unique_id(), 1, 0, 0, timeout_s=20)
    t = _tokens(37, 1, 0, 5)
    np.testing.assert_array_equal(c.gather_tokens(t, 37), t)
    with pytest.raises(_abi.LLMError, match="holds 36 sequences, its shard has 37"):
        c.gather_tokens(t[:, :36], 37)
    c.close()


def _rank_main(rank, world, n_total, steps, idfile, q, skip):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        if rank == 0:
            uid = Comm.unique_id()
            with open(idfile + ".tmp", "wb") as f:
                f.write(uid)
            os.replace(idfile + ".tmp", idfile)
        else:
            t0 = time.time()
            while not os.path.exists(idfile) and time.time() - t0 < 30:
                time.sleep(0.05)
            uid = open(idfile, "rb").read()
        if rank in skip:
            q.put((rank, "skipped"))
            return
        c = Comm(uid, world, rank, device=rank, timeout_s=5.0)
        out = c.gather_tokens(_tokens(n_total, world, rank, steps), n_total)
        c.close()
        q.put((rank, out))
    except _abi.LLMError as e:
        q.put((rank, f"error: {e}"))


def _run(world, n_total, steps, tmp_path, skip=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    idfile = str(tmp_path / "nccl.id")
    ps = [ctx.Process(target=_rank_main, args=(r, world, n_total, steps, idfile, q, skip)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    return res


two_gpus = pytest.mark.skipif(
    __import__("torch").cuda.device_count() < 2, reason="needs two GPUs")


@two_gpus
def test_two_rank_gather_in_global_order(tmp_path):
    res = _run(2, 11, 4, tmp_path)
    want = np.concatenate([_tokens(11, 2, r, 4) for r in range(2)], axis=1)
    for r in range(2):
        np.testing.assert_array_equal(res[r], want)


@two_gpus
def test_rank_that_never_joins_fails_the_other_within_the_timeout(tmp_path):
    t0 = time.time()
    res = _run(2, 8, 2, tmp_path, skip=(1,))
    assert res[1] == "skipped"
    assert isinstance(res[0], str) and "timed out" in res[0]
    assert time.time() - t0 < 90
