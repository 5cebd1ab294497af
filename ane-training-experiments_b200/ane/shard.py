"""Sequence sharding across ranks (one process per GPU) and the single output gather.

The reference decodes one sequence in one process (ane/stories/infer.go:136-202); it has no
multi-device code.  Here independent sequences are partitioned across ranks: rank r owns a
contiguous block of the job's sequences, weights are replicated, each rank's KV cache holds
only its own sequences, and no data crosses ranks while tokens are generated.  The one
collective is `gather_tokens`, run once at the end, which brings every rank's generated token
ids to every rank in global sequence order.

The functions work on any torch.distributed backend: NCCL over NVLink on the GPU box (tensors
on the rank's device) and gloo on CPU (the multi-rank tests).
"""
from __future__ import annotations

from typing import Optional

import numpy as np


def shard_range(n_total: int, world: int, rank: int) -> range:
    """Global sequence indices owned by `rank`: contiguous blocks, the first n_total % world
    ranks holding one sequence more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if n_total < 0:
        raise ValueError(f"sequence count {n_total} is negative")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_tokens(tokens: np.ndarray, n_total: int, group=None, device: Optional[str] = None) -> np.ndarray:
    """All-gather of generated token ids.

    tokens: this rank's [steps, n_local] int32 block (n_local = len(shard_range(...))).
    Returns [steps, n_total] on every rank, column j holding global sequence j.  Ranks with
    fewer sequences pad to the largest shard with -1; the padding is dropped after the gather.
    A rank that never joins makes the others fail with the process group's timeout instead of
    waiting forever."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    if tokens.ndim != 2:
        raise ValueError(f"tokens must be [steps, n_local], got shape {tokens.shape}")
    own = shard_range(n_total, world, rank)
    if tokens.shape[1] != len(own):
        raise ValueError(f"rank {rank} holds {tokens.shape[1]} sequences, its shard has {len(own)}")
    steps = tokens.shape[0]
    width = len(shard_range(n_total, world, 0))  # the largest shard
    buf = np.full((steps, width), -1, np.int32)
    buf[:, :tokens.shape[1]] = tokens
    t = torch.from_numpy(buf)
    if device is not None:
        t = t.to(device)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    out = np.empty((steps, n_total), np.int32)
    for r, part in enumerate(parts):
        rr = shard_range(n_total, world, r)
        out[:, rr.start:rr.stop] = part.cpu().numpy()[:, :len(rr)]
    return out


class Comm:
    """The library's communicator (llm_comm_create / llm_gather_tokens): NCCL inside
    libllm_cuda.so, every wait bounded by timeout_s on the host.  This is the path a Go host
    binds through cgo; gather_tokens above is the torch.distributed equivalent."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int = 0, timeout_s: float = 60.0):
        import ctypes as C
        from . import _abi
        self._abi = _abi
        self.nranks, self.rank = nranks, rank
        h = C.c_void_p()
        _abi.check(_abi.lib().llm_comm_create(uid, len(uid), nranks, rank, device, timeout_s, C.byref(h)))
        self.h = h

    @staticmethod
    def unique_id() -> bytes:
        import ctypes as C
        from . import _abi
        buf = C.create_string_buffer(_abi.LLM_COMM_ID_BYTES)
        _abi.check(_abi.lib().llm_comm_unique_id(buf, len(buf)))
        return buf.raw

    def gather_tokens(self, tokens: np.ndarray, n_total: int) -> np.ndarray:
        """This rank's [steps, n_local] block -> [steps, n_total] on every rank."""
        import ctypes as C
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.ndim != 2:
            raise ValueError(f"tokens must be [steps, n_local], got shape {t.shape}")
        out = np.empty((t.shape[0], n_total), np.int32)
        i32p = C.POINTER(C.c_int32)
        self._abi.check(self._abi.lib().llm_gather_tokens(self.h, t.ctypes.data_as(i32p), t.shape[0], t.shape[1],
                                                          n_total, out.ctypes.data_as(i32p)))
        return out

    def last_gather_ms(self) -> float:
        """Device time of the last gather (llm_comm_last_gather_ms)."""
        import ctypes as C
        v = C.c_double()
        self._abi.check(self._abi.lib().llm_comm_last_gather_ms(self.h, C.byref(v)))
        return v.value

    def close(self):
        if getattr(self, "h", None):
            self._abi.lib().llm_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


def library_shard_range(n_total: int, world: int, rank: int) -> range:
    """llm_shard_range through the C ABI (the same partition as shard_range)."""
    import ctypes as C
    from . import _abi
    s, n = C.c_int32(), C.c_int32()
    _abi.check(_abi.lib().llm_shard_range(n_total, world, rank, C.byref(s), C.byref(n)))
    return range(s.value, s.value + n.value)
