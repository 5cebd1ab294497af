"""Host-side mirror of the reference's `ane/storiesane` inference surface over the CUDA C ABI.

Go reference (tmc/ane-training-experiments):
  ane/storiesane/engine.go:149-272  Open(Options) (seq default SeqDefault, seed default 42,
                                    .bin weights else a checkpoint)
  ane/storiesane/engine.go:363-376  EvalLogits: one full window -> channel-first logits [Vocab][seq]
  ane/storiesane/engine.go:804-842  evalLogitsCPUInto: the forward it computes (residual
                                    x + a*branch, a = 1/sqrt(2*layers); gate (h1*sig)*h3)
  ane/storiesane/decode.go:18-94    Decode: re-evaluates the BOS left-padded window of the last
                                    seq tokens for every generated token; fillDecodeWindow

The training half of the engine (Step, backward, Adam, ANE offload) is out of scope.  Every
evaluation runs on the B200 through llm_eval_window (no CPU fallback): the ANE branch and
its CPU fallback of evalLogitsInto are both replaced by the CUDA path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from .. import _abi
from .._abi import LLMError
from ..stories import (BOS, EOS, STORIES_110M, DecodeOptions, DecodeResult, Engine as _CudaEngine, ModelConfig,
                       ModelWeights, SeqDefault, Tokenizer)


@dataclass
class Options:
    """ane/storiesane/engine.go:23-45 (the inference fields).  Weights / Config / DType /
    Device are additions: in-memory weights instead of a file, and the CUDA arithmetic."""

    ModelPath: str = ""
    Seq: int = 0
    Seed: int = 0
    UseANE: bool = False  # accepted for source compatibility; evaluation always runs on CUDA
    Weights: Optional[ModelWeights] = None
    Config: ModelConfig = STORIES_110M
    DType: str = "fp16"
    Device: int = 0


@dataclass
class Diagnostics:
    """ane/storiesane/diagnostics.go:4-20: best-effort runtime state of an Engine."""

    UseANE: bool = False
    LayerForwardRequested: bool = False
    LayerForwardEnabled: bool = False
    CompiledLayers: int = 0
    LayerInitError: str = ""
    FinalHeadOffloadEnabled: bool = False
    HybridBackwardRequested: bool = False
    HybridBackwardEnabled: bool = False
    BackwardInitError: str = ""
    HasRMSForward: bool = False
    HasClassifierForward: bool = False
    HasSoftmax: bool = False
    HasClassifierBackward: bool = False
    HasRMSBackward: bool = False
    OffloadDiagnostics: str = ""


def fillDecodeWindow(dst: List[int], tokens: List[int]) -> None:
    """decode.go:83-94: BOS everywhere, then the last len(dst) tokens right-aligned."""
    for i in range(len(dst)):
        dst[i] = BOS
    if len(tokens) >= len(dst):
        tokens = tokens[len(tokens) - len(dst):]
    start = len(dst) - len(tokens)
    for i, t in enumerate(tokens):
        dst[start + i] = t


class Engine:
    """storiesane.Engine's evaluation API on one CUDA context (one sequence slot, a KV cache
    of one window)."""

    def __init__(self, cuda: _CudaEngine, seq: int, seed: int, use_ane: bool = False):
        self._e = cuda
        self.seq = seq
        self.seed = seed
        self.vocab = cuda.cfg.vocab
        self.use_ane = use_ane

    def Diagnostics(self) -> Diagnostics:
        """diagnostics.go:23-54.  On CUDA every layer's forward and the final head (RMSNorm,
        classifier, softmax / sampling) run on the device once the engine is open; there is no
        training path, so the backward fields stay false."""
        if self._e is None:
            return Diagnostics()
        cfg = self._e.cfg
        return Diagnostics(
            UseANE=self.use_ane, LayerForwardRequested=self.use_ane, LayerForwardEnabled=True,
            CompiledLayers=cfg.n_layers, FinalHeadOffloadEnabled=True, HasRMSForward=True,
            HasClassifierForward=True, HasSoftmax=True,
            OffloadDiagnostics=f"cuda device {self._e.device}: {cfg.name} {self._e.dtype}, "
                               f"{cfg.n_layers} layers, window {self.seq}")

    def EvalLogits(self, tokens) -> np.ndarray:
        """engine.go:363-376: tokens of length seq -> logits [Vocab * seq], channel-first
        (logits[v * seq + t])."""
        if self._e is None:
            raise LLMError(_abi.LLM_ERR_STATE, "storiesane eval logits: engine is closed")
        if len(tokens) != self.seq:
            raise LLMError(_abi.LLM_ERR_INVALID, f"storiesane eval logits: token len={len(tokens)} want={self.seq}")
        lg = np.empty(self.vocab * self.seq, np.float32)
        self._eval(tokens, lg)
        return lg

    def _eval(self, tokens, logits: Optional[np.ndarray]) -> int:
        t = _abi.i32(tokens)
        nxt = np.zeros(1, np.int32)
        _abi.check(_abi.lib().llm_eval_window(self._e.h, 0, _abi.ptr(t, C.c_int32), self.seq,
                                              _abi.LLM_ARITH_STORIESANE, _abi.ptr(nxt, C.c_int32),
                                              _abi.ptr(logits) if logits is not None else None))
        return int(nxt[0])

    def Decode(self, tok: Optional[Tokenizer], opts: DecodeOptions) -> DecodeResult:
        """decode.go:18-81: maxNew <= 0 -> 64, temperature < 0 -> 0, seed = opts.Seed or the
        engine's; a fresh generator per call (the device generator reseeded and its draws
        reset); the next token of each window is chosen on the device (argmax, or the sampler
        for temperature > 1e-6)."""
        if self._e is None:
            raise LLMError(_abi.LLM_ERR_STATE, "storiesane decode: engine is closed")
        max_new = opts.MaxNewTokens if opts.MaxNewTokens > 0 else 64
        temp = max(0.0, opts.Temperature)
        seed = opts.Seed if opts.Seed != 0 else self.seed
        prompt = list(opts.PromptTokens) or [BOS]
        if len(prompt) > self.seq:
            prompt = prompt[len(prompt) - self.seq:]
        for i, t in enumerate(prompt):
            if t < 0 or t >= self.vocab:
                raise LLMError(_abi.LLM_ERR_TOKEN_RANGE, f"storiesane decode: prompt token[{i}]={t} out of range")
        self._e.set_sampling(temp, seed, True)
        tokens = list(prompt)
        text = b""
        eos = False
        window = [0] * self.seq
        for _ in range(max_new):
            fillDecodeWindow(window, tokens)
            nxt = self._eval(window, None)
            tokens.append(nxt)
            if tok is not None:
                text += tok.DecodeBytes(nxt)
            if nxt == EOS:
                eos = True
                break
        self._e.set_sampling(0.0, seed, True)
        return DecodeResult(tokens, len(prompt), text.decode("utf-8", "surrogateescape"), eos)

    def Close(self) -> None:
        if self._e is not None:
            self._e.close()
            self._e = None


def Open(opts: Options) -> Engine:
    """engine.go:149-272 (inference part): the model comes from opts.Weights, else
    opts.ModelPath read as a llama2.c .bin and, if that fails, as a checkpoint (streamed to the
    device by llm_load_weights_file)."""
    if opts.Weights is None and not opts.ModelPath:
        raise LLMError(_abi.LLM_ERR_INVALID, "storiesane open: model path is empty")
    seq = opts.Seq if opts.Seq > 0 else SeqDefault
    seed = opts.Seed if opts.Seed != 0 else 42
    cfg = opts.Config if opts.Weights is None else opts.Weights.Config
    cfg = cfg.with_max_seq(max(cfg.max_seq, seq))
    eng = _CudaEngine(cfg, opts.DType, opts.Device)
    try:
        if opts.Weights is not None:
            eng.load(opts.Weights)
        else:
            try:
                eng.load_file(opts.ModelPath, "llama2c")
            except LLMError as bin_err:
                try:
                    eng.load_file(opts.ModelPath, "checkpoint")
                except LLMError:
                    raise LLMError(bin_err.code, f"storiesane open: load model: {bin_err}") from None
        eng.kv_alloc(1, seq)
    except Exception:
        eng.close()
        raise
    return Engine(eng, seq, seed, opts.UseANE)
