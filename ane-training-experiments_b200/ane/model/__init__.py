"""Mirror of the reference's ane/model package for linear (1x1 convolution) kernels
(ane/model/model_darwin.go:27-53,138-414,542): Compile a kernel from its weights, write its
channel-first fp32 input, Eval / EvalWithStats, read its channel-first fp32 output, Close.

The reference compiles a MIL program for the ANE; here a kernel is a tcgen05 GEMM of the
library (llm_linear_*), with the weights converted on the device to the chosen arithmetic.
One input and one output tensor, as the linear kernels of the token loop use them."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np

from .. import _abi


@dataclass
class CompileOptions:
    """The weights replace model.CompileOptions.WeightBlob / MILText (model_darwin.go:27-37)."""

    Weights: Optional[np.ndarray] = None  # [OutDim, InDim] fp32, row-major
    SeqLen: int = 1                       # tokens per evaluation (the tensors' width)
    DType: str = "fp16"
    Device: int = 0


@dataclass
class EvalStats:
    HWExecutionNS: int = 0
    Metrics: Dict[str, float] = field(default_factory=dict)


class Kernel:
    def __init__(self, opts: CompileOptions):
        w = np.ascontiguousarray(opts.Weights, dtype=np.float32)
        if w.ndim != 2:
            raise ValueError("compile: Weights must be [out, in]")
        self.out_dim, self.in_dim = w.shape
        self.seq = int(opts.SeqLen)
        if self.seq <= 0:
            raise ValueError(f"compile: SeqLen {self.seq} must be positive")
        h = C.c_void_p()
        _abi.check(_abi.lib().llm_linear_create(opts.Device, _abi.DTYPES[opts.DType], _abi.ptr(w), self.out_dim,
                                                self.in_dim, C.byref(h)))
        self.h = h
        self._in = np.zeros(self.in_dim * self.seq, np.float32)
        self._out = np.zeros(self.out_dim * self.seq, np.float32)

    def closed(self) -> bool:
        return getattr(self, "h", None) is None

    def NumInputs(self) -> int:
        return 0 if self.closed() else 1

    def NumOutputs(self) -> int:
        return 0 if self.closed() else 1

    def InputBytes(self, i: int) -> int:
        return self.in_dim * self.seq * 4 if i == 0 and not self.closed() else 0

    def OutputBytes(self, i: int) -> int:
        return self.out_dim * self.seq * 4 if i == 0 and not self.closed() else 0

    def WriteInputF32(self, i: int, data) -> None:
        if self.closed():
            raise ValueError("write input f32: kernel is closed")
        if i != 0:
            raise ValueError(f"write input f32: index {i} out of range")
        d = np.asarray(data, np.float32).reshape(-1)
        if d.size != self._in.size:
            raise ValueError(f"write input f32: got {d.size} values, want {self._in.size}")
        self._in[:] = d

    def EvalWithStats(self) -> EvalStats:
        if self.closed():
            raise ValueError("eval: kernel is closed")
        ns = C.c_uint64()
        _abi.check(_abi.lib().llm_linear_eval_cf(self.h, _abi.ptr(self._in), self.seq, _abi.ptr(self._out),
                                                 C.byref(ns)))
        return EvalStats(HWExecutionNS=int(ns.value))

    def Eval(self) -> None:
        self.EvalWithStats()

    def ReadOutputF32(self, i: int, out) -> None:
        if self.closed():
            raise ValueError("read output f32: kernel is closed")
        if i != 0:
            raise ValueError(f"read output f32: index {i} out of range")
        if out.size != self._out.size:
            raise ValueError(f"read output f32: got {out.size} values, want {self._out.size}")
        out.reshape(-1)[:] = self._out

    def Close(self) -> None:
        if not self.closed():
            _abi.lib().llm_linear_destroy(self.h)
            self.h = None

    def __del__(self):
        self.Close()


def Compile(opts: CompileOptions) -> Kernel:
    """model.Compile (model_darwin.go:138-171)."""
    if opts.Weights is None:
        raise ValueError("compile: Weights is required")
    return Kernel(opts)
