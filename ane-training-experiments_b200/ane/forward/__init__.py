"""Mirror of the reference's ane/forward package (ane/forward/conv.go:11-76): ConvEval runs a
linear kernel on row-major tokens [S, inDim] by transposing to channel-first [inDim, S],
evaluating, and transposing the [outDim, S] result back; the error texts are the reference's."""
from __future__ import annotations

import numpy as np

from ..model import EvalStats, Kernel


def ConvEvalWithStats(k: Kernel, x, s: int, inDim: int, outDim: int):
    x = np.asarray(x, np.float32).reshape(-1)
    if x.size != s * inDim:
        raise ValueError(f"ConvEval input len={x.size} want={s * inDim}")
    cf = ToChannelFirst(x, s, inDim)
    try:
        k.WriteInputF32(0, cf)
    except ValueError as e:
        raise ValueError(f"write input: {e}") from e
    try:
        est = k.EvalWithStats()
    except Exception as e:  # noqa: BLE001 - the reference wraps every eval failure
        raise ValueError(f"eval: {e}") from e
    outT = np.zeros(s * outDim, np.float32)
    try:
        k.ReadOutputF32(0, outT)
    except ValueError as e:
        raise ValueError(f"read output: {e}") from e
    return FromChannelFirst(outT, s, outDim), est


def ConvEval(k: Kernel, x, s: int, inDim: int, outDim: int) -> np.ndarray:
    out, _ = ConvEvalWithStats(k, x, s, inDim, outDim)
    return out


def ToChannelFirst(x, s: int, d: int) -> np.ndarray:
    x = np.asarray(x, np.float32).reshape(-1)
    if x.size != s * d:
        raise ValueError(f"ToChannelFirst input len={x.size} want={s * d}")
    return np.ascontiguousarray(x.reshape(s, d).T).reshape(-1)


def FromChannelFirst(x, s: int, d: int) -> np.ndarray:
    x = np.asarray(x, np.float32).reshape(-1)
    if x.size != s * d:
        raise ValueError(f"FromChannelFirst input len={x.size} want={s * d}")
    return np.ascontiguousarray(x.reshape(d, s).T).reshape(-1)


__all__ = ["ConvEval", "ConvEvalWithStats", "ToChannelFirst", "FromChannelFirst", "EvalStats"]
