"""Host-side mirror of the reference's `ane/stories` package over the CUDA C ABI.

Go reference (tmc/ane-training-experiments):
  ane/stories/config.go:3-28     model constants, Llama2Config
  ane/stories/weights.go:13-122  LayerWeights / ModelWeights / NewModelWeights / LoadPretrained
  ane/stories/infer.go:15-202    DecodeOptions / DecodeResult / Decoder (NewDecoder, Decode,
                                 EvalNextLogits, ResetCache)
  ane/stories/tokenizer.go:16-69 Tokenizer / LoadTokenizer / Decode

Names, argument meaning and error texts follow the Go package; the Decoder runs on the
B200 through lib/libllm_cuda.so (no CPU fallback).  Additions beyond the Go API are the
runtime ModelConfig (Stories110M and Qwen3-0.6B presets), the dtype/device arguments of
NewDecoder, and the batched DecodeBatch.
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from .. import _abi
from .._abi import LLMError

# ane/stories/config.go:3-10
Dim = 768
Hidden = 2048
Heads = 12
SeqDefault = 256
NLayers = 12
Vocab = 32000

BOS = 1  # ane/stories/infer.go:10
EOS = 2  # ane/stories/infer.go:11


@dataclass(frozen=True)
class ModelConfig:
    """Runtime model description (the Go code hard-codes Stories110M in config.go)."""

    dim: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    max_seq: int = SeqDefault
    qk_norm: bool = False
    tied_embed: bool = True
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    name: str = "custom"

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def with_max_seq(self, max_seq: int) -> "ModelConfig":
        return ModelConfig(**{**self.__dict__, "max_seq": max_seq})

    def c_struct(self) -> _abi.llm_model_config:
        return _abi.llm_model_config(
            self.dim, self.hidden, self.n_layers, self.n_heads, self.n_kv_heads, self.head_dim, self.vocab,
            self.max_seq, int(self.qk_norm), int(self.tied_embed), float(self.norm_eps), float(self.rope_theta))

    def oracle_dict(self) -> dict:
        return dict(dim=self.dim, hidden=self.hidden, n_layers=self.n_layers, n_heads=self.n_heads,
                    n_kv_heads=self.n_kv_heads, head_dim=self.head_dim, vocab=self.vocab, max_seq=self.max_seq,
                    qk_norm=int(self.qk_norm), norm_eps=self.norm_eps, rope_theta=self.rope_theta)


# ane/stories/config.go:3-10, ane/stories/infer.go:102,307
STORIES_110M = ModelConfig(Dim, Hidden, NLayers, Heads, Heads, Dim // Heads, Vocab, SeqDefault,
                           qk_norm=False, tied_embed=True, norm_eps=1e-5, rope_theta=10000.0, name="stories110m")
# training/training_dynamic/models/qwen3_06b.h:6-16 plus the Qwen3 features of the spec
# (per-head QK RMSNorm, theta 1e6, eps 1e-6, tied 151936 vocab)
QWEN3_0_6B = ModelConfig(1024, 3072, 28, 16, 8, 128, 151936, 4096, qk_norm=True, tied_embed=True,
                         norm_eps=1e-6, rope_theta=1e6, name="qwen3-0.6b")

PRESETS = {"stories110m": STORIES_110M, "qwen3-0.6b": QWEN3_0_6B}


@dataclass
class LayerWeights:
    """ane/stories/weights.go:13-17 (fp32, row-major [out, in]) plus Qwen3 q/k norms."""

    Wq: np.ndarray
    Wk: np.ndarray
    Wv: np.ndarray
    Wo: np.ndarray
    W1: np.ndarray
    W2: np.ndarray
    W3: np.ndarray
    RMSAtt: np.ndarray
    RMSFFN: np.ndarray
    QNorm: Optional[np.ndarray] = None
    KNorm: Optional[np.ndarray] = None


@dataclass
class ModelWeights:
    """ane/stories/weights.go:19-24."""

    Layers: List[LayerWeights]
    RMSFinal: np.ndarray
    Embed: np.ndarray  # [vocab, dim]
    SharedCL: bool = True
    LMHead: Optional[np.ndarray] = None  # only when not SharedCL
    Config: ModelConfig = STORIES_110M

    def c_struct(self):
        """ctypes view (keeps the numpy arrays referenced by the returned tuple)."""
        layers = (_abi.llm_layer_weights_f32 * len(self.Layers))()
        keep = []
        for i, L in enumerate(self.Layers):
            for name, arr in (("wq", L.Wq), ("wk", L.Wk), ("wv", L.Wv), ("wo", L.Wo), ("w1", L.W1), ("w2", L.W2),
                              ("w3", L.W3), ("rms_att", L.RMSAtt), ("rms_ffn", L.RMSFFN), ("q_norm", L.QNorm),
                              ("k_norm", L.KNorm)):
                if arr is not None:
                    a = _abi.f32(arr)
                    keep.append(a)
                    setattr(layers[i], name, _abi.ptr(a))
        emb = _abi.f32(self.Embed)
        fin = _abi.f32(self.RMSFinal)
        keep += [emb, fin, layers]
        lm = None
        if not self.SharedCL:
            lm = _abi.f32(self.LMHead)
            keep.append(lm)
        w = _abi.llm_model_weights_f32(_abi.ptr(emb), _abi.ptr(fin), _abi.ptr(lm), layers)
        return w, keep


def NewModelWeights(vocab: int = Vocab, cfg: ModelConfig = STORIES_110M) -> ModelWeights:
    """ane/stories/weights.go:26-47: zeroed weights of the given config."""
    D, F, Q, KV, hd = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.head_dim
    z = lambda *s: np.zeros(s, dtype=np.float32)  # noqa: E731
    layers = [LayerWeights(z(Q, D), z(KV, D), z(KV, D), z(D, Q), z(F, D), z(D, F), z(F, D), z(D), z(D),
                           z(hd) if cfg.qk_norm else None, z(hd) if cfg.qk_norm else None) for _ in range(cfg.n_layers)]
    return ModelWeights(layers, z(D), z(vocab, D), True, None, cfg)


def SyntheticWeights(cfg: ModelConfig, seed: int = 1234, out_proj_scale: float = 1.0,
                     stddev: float = 0.02) -> ModelWeights:
    """Seeded N(0, stddev) weights from the library's counter-based generator (with the
    default 0.02 these are the values llm_load_weights_synthetic uploads); Wo and W2 also
    x out_proj_scale; norms = 1."""
    D, F, Q, KV, hd = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.head_dim
    g = lambda n, l, k, s=1.0: _abi.synth_normal(n, seed, _abi.synth_stream(l, k), stddev, s)  # noqa: E731
    layers = []
    for l in range(cfg.n_layers):
        layers.append(LayerWeights(
            g(Q * D, l, 0).reshape(Q, D), g(KV * D, l, 1).reshape(KV, D), g(KV * D, l, 2).reshape(KV, D),
            g(D * Q, l, 3, out_proj_scale).reshape(D, Q), g(F * D, l, 4).reshape(F, D),
            g(D * F, l, 5, out_proj_scale).reshape(D, F), g(F * D, l, 6).reshape(F, D),
            np.ones(D, np.float32), np.ones(D, np.float32),
            np.ones(hd, np.float32) if cfg.qk_norm else None, np.ones(hd, np.float32) if cfg.qk_norm else None))
    emb = g(cfg.vocab * D, 0, 7).reshape(cfg.vocab, D)
    lm = None if cfg.tied_embed else g(cfg.vocab * D, 0, 8).reshape(cfg.vocab, D)
    return ModelWeights(layers, np.ones(D, np.float32), emb, cfg.tied_embed, lm, cfg)


def LoadPretrained(path: str, cfg: Optional[ModelConfig] = None):
    """ane/stories/weights.go:49-122: llama2.c .bin reader (header of 7 int32, then embed,
    rms_att[L], wq[L], wk[L], wv[L], wo[L], rms_ffn[L], w1[L], w2[L], w3[L], rms_final;
    vocab < 0 means an unshared classifier follows... the Go loader only records SharedCL)."""
    with open(path, "rb") as f:
        hdr = f.read(28)
        if len(hdr) != 28:
            raise ValueError("read config: unexpected EOF")
        dim, hidden, n_layers, n_heads, n_kv, vocab, seq = struct.unpack("<7i", hdr)
        cfg = cfg or STORIES_110M
        if dim != cfg.dim or hidden != cfg.hidden or n_layers != cfg.n_layers:
            raise ValueError(f"config mismatch: got dim={dim} hidden={hidden} layers={n_layers}")
        shared = vocab > 0
        vocab = abs(vocab)
        mw = NewModelWeights(vocab, cfg)
        mw.SharedCL = shared

        def rd(arr, what):
            b = f.read(arr.nbytes)
            if len(b) != arr.nbytes:
                raise ValueError(f"read {what}: unexpected EOF")
            arr[...] = np.frombuffer(b, dtype="<f4").reshape(arr.shape)

        rd(mw.Embed, "embed")
        for name, attr in (("rms_att", "RMSAtt"), ("wq", "Wq"), ("wk", "Wk"), ("wv", "Wv"), ("wo", "Wo"),
                           ("rms_ffn", "RMSFFN"), ("w1", "W1"), ("w2", "W2"), ("w3", "W3")):
            for i, L in enumerate(mw.Layers):
                rd(getattr(L, attr), f"{name}[{i}]")
        rd(mw.RMSFinal, "rms_final")
    return mw, dict(Dim=dim, HiddenDim=hidden, NLayers=n_layers, NHeads=n_heads, NKVHeads=n_kv,
                    VocabSize=vocab if shared else -vocab, SeqLen=seq)


@dataclass
class TrainMeta:
    """ane/stories/ckpt.go:24-35."""

    Step: int = 0
    TotalSteps: int = 0
    LR: float = 0.0
    Loss: float = 0.0
    CumCompile: float = 0.0
    CumTrain: float = 0.0
    CumWall: float = 0.0
    CumSteps: int = 0
    CumBatches: int = 0
    AdamT: int = 0


CKPT_MAGIC = 0x424C5A54  # ane/stories/ckpt.go:12


def LoadCheckpoint(path: str, mw: "ModelWeights", opt=None) -> TrainMeta:
    """ane/stories/ckpt.go:237-447 for inference: fills mw's weights from a v2/v3 checkpoint
    and skips the optimizer moments (only opt=None is supported: training is out of scope).
    The header's layers/vocab/dim/hidden/heads must match mw.Config."""
    if opt is not None:
        raise ValueError("optimizer state is not loaded by the inference path")
    cfg = mw.Config
    with open(path, "rb") as f:
        def rd(n, what):
            b = f.read(n)
            if len(b) != n:
                raise ValueError(f"read {what}: " + ("EOF" if not b else "unexpected EOF"))
            return b
        magic, ver = struct.unpack("<ii", rd(8, "checkpoint header"))
        if magic != CKPT_MAGIC or ver not in (2, 3):
            raise ValueError(f"bad checkpoint header magic={magic & 0xffffffff:x} version={ver}")
        step, total, n_layers, vocab, dim, hidden, heads, _seq = struct.unpack("<8i", rd(32, "checkpoint header"))
        if (n_layers, vocab, dim, hidden, heads) != (cfg.n_layers, cfg.vocab, cfg.dim, cfg.hidden, cfg.n_heads):
            raise ValueError("checkpoint config mismatch")
        lr, loss = struct.unpack("<ff", rd(8, "checkpoint header"))
        cc, ct, cw = struct.unpack("<3d", rd(24, "checkpoint header"))
        cs, cb, at, _, _, _ = struct.unpack("<6i", rd(24, "checkpoint header"))

        def rdf(arr, what):
            arr[...] = np.frombuffer(rd(arr.nbytes, what), dtype="<f4").reshape(arr.shape)

        for i, L in enumerate(mw.Layers):
            for attr in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3", "RMSAtt", "RMSFFN"):
                rdf(getattr(L, attr), f"{attr.lower()}[{i}]")
        per_layer = sum(getattr(mw.Layers[0], a).size for a in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"))
        skip = len(mw.Layers) * (2 * per_layer + 4 * cfg.dim)
        rd(4 * skip, "layer optimizer state")
        rdf(mw.RMSFinal, "rms_final")
        rd(4 * 2 * cfg.dim, "rms_final optimizer state")
        rdf(mw.Embed, "embed")
        rd(4 * 2 * mw.Embed.size, "embed optimizer state")
    return TrainMeta(step, total, lr, loss, cc, ct, cw, cs, cb, at)


class Tokenizer:
    """ane/stories/tokenizer.go:11-69 (decode only).

    Pieces are kept as the file's raw bytes, as Go strings are.  DecodeBytes returns exactly
    the bytes Go's Decode returns; Decode returns them as a str through the surrogateescape
    error handler, so bytes that are not UTF-8 (single <0xHH> bytes) survive a round trip:
    ``Decode(i).encode("utf-8", "surrogateescape") == DecodeBytes(i)``."""

    def __init__(self, vocab: List[bytes]):
        self.vocab = [v if isinstance(v, bytes) else v.encode("utf-8") for v in vocab]

    def DecodeBytes(self, id: int) -> bytes:
        if id < 0 or id >= len(self.vocab):
            return b""
        s = self.vocab[id]
        if len(s) >= 5 and s[:3] == b"<0x" and s[-1:] == b">":
            b = _decode_hex_token_byte(s)
            if b is not None:
                return bytes([b])
        return s

    def Decode(self, id: int) -> str:
        return self.DecodeBytes(id).decode("utf-8", "surrogateescape")


def _decode_hex_token_byte(s: bytes) -> Optional[int]:
    """tokenizer.go:71-101: exactly "<0xHH>" with hex digits of either case."""
    if len(s) != 6:
        return None
    hexdigits = b"0123456789abcdefABCDEF"
    if s[3] not in hexdigits or s[4] not in hexdigits:
        return None
    return int(s[3:5], 16)


def LoadTokenizer(path: str, vocab_size: int = Vocab) -> Tokenizer:
    """ane/stories/tokenizer.go:16-55: int32 max token length, then per token a float32
    score, an int32 byte length (0 <= n <= 8 * max) and the bytes; Vocab entries."""
    with open(path, "rb") as f:
        b = f.read(4)
        if len(b) != 4:
            raise ValueError("read tokenizer header: " + ("EOF" if not b else "unexpected EOF"))
        (max_len,) = struct.unpack("<i", b)
        if max_len <= 0:
            raise ValueError(f"bad tokenizer header: max token len={max_len}")
        vocab = []
        for i in range(vocab_size):
            b = f.read(4)
            if len(b) == 0:
                raise ValueError(f"unexpected EOF at token {i}")
            if len(b) != 4:
                raise ValueError(f"read token[{i}] score: unexpected EOF")
            b = f.read(4)
            if len(b) != 4:
                raise ValueError(f"read token[{i}] length: " + ("EOF" if not b else "unexpected EOF"))
            (n,) = struct.unpack("<i", b)
            if n < 0 or n > max_len * 8:
                raise ValueError(f"bad token[{i}] length={n}")
            piece = f.read(n)
            if len(piece) != n:
                raise ValueError(f"read token[{i}] bytes: " + ("EOF" if not piece else "unexpected EOF"))
            vocab.append(piece)
    return Tokenizer(vocab)


@dataclass
class DecodeOptions:
    """ane/stories/infer.go:15-21."""

    MaxNewTokens: int = 0
    Temperature: float = 0.0
    Seed: int = 0
    PromptTokens: List[int] = field(default_factory=list)


@dataclass
class DecodeResult:
    """ane/stories/infer.go:23-28."""

    Tokens: List[int]
    PromptLength: int
    Text: str = ""
    StoppedOnEOS: bool = False


class Engine:
    """One CUDA context: weights on one device plus a paged KV cache of `max_batch`
    sequence slots of up to `max_pos` positions.  Thin wrapper of the C ABI."""

    def __init__(self, cfg: ModelConfig, dtype: str = "bf16", device: int = 0):
        self.cfg = cfg
        self.dtype = dtype
        self.device = device
        h = C.c_void_p()
        _abi.check(_abi.lib().llm_ctx_create(C.byref(cfg.c_struct()), _abi.DTYPES[dtype], device, C.byref(h)))
        self.h = h
        self.max_batch = 0
        self.max_pos = 0

    def load(self, w: ModelWeights) -> "Engine":
        cw, keep = w.c_struct()
        _abi.check(_abi.lib().llm_load_weights_f32(self.h, C.byref(cw)))
        del keep
        return self

    def set_sampling(self, temperature: float, seed: int, reset_draws: bool = True) -> None:
        """Temperature sampling for the following steps (<= 1e-6: greedy); see llm_set_sampling."""
        _abi.check(_abi.lib().llm_set_sampling(self.h, float(temperature), int(seed) & (2**64 - 1), int(reset_draws)))

    def load_file(self, path: str, fmt: str = "llama2c") -> "Engine":
        """Stream a llama2.c .bin ("llama2c") or a training checkpoint ("checkpoint") to the device."""
        code = {"llama2c": _abi.LLM_WEIGHTS_LLAMA2C, "checkpoint": _abi.LLM_WEIGHTS_CHECKPOINT}[fmt]
        _abi.check(_abi.lib().llm_load_weights_file(self.h, str(path).encode(), code))
        return self

    def load_synthetic(self, seed: int, out_proj_scale: float = 1.0) -> "Engine":
        _abi.check(_abi.lib().llm_load_weights_synthetic(self.h, seed, out_proj_scale))
        return self

    def kv_alloc(self, max_batch: int, max_pos: int) -> "Engine":
        _abi.check(_abi.lib().llm_kv_alloc(self.h, max_batch, max_pos, 16))
        self.max_batch, self.max_pos = max_batch, max_pos
        return self

    def release(self, seq: int) -> None:
        _abi.check(_abi.lib().llm_seq_release(self.h, seq))

    def prefill(self, seq_ids, prompts: List[List[int]], start_pos=None, want_logits=False):
        seq = _abi.i32(seq_ids)
        lens = _abi.i32([len(p) for p in prompts])
        flat = _abi.i32([t for p in prompts for t in p])
        sp = None if start_pos is None else _abi.i32(start_pos)
        nxt = np.zeros(len(prompts), np.int32)
        lg = np.zeros((len(prompts), self.cfg.vocab), np.float32) if want_logits else None
        _abi.check(_abi.lib().llm_prefill(self.h, _abi.ptr(seq, C.c_int32), _abi.ptr(flat, C.c_int32),
                                          _abi.ptr(lens, C.c_int32), _abi.ptr(sp, C.c_int32), len(prompts),
                                          _abi.ptr(nxt, C.c_int32), _abi.ptr(lg)))
        return (nxt, lg) if want_logits else nxt

    def decode_step(self, seq_ids, tokens, positions, want_logits=False):
        seq, tok, pos = _abi.i32(seq_ids), _abi.i32(tokens), _abi.i32(positions)
        n = len(seq)
        nxt = np.zeros(n, np.int32)
        lg = np.zeros((n, self.cfg.vocab), np.float32) if want_logits else None
        _abi.check(_abi.lib().llm_decode_step(self.h, _abi.ptr(seq, C.c_int32), _abi.ptr(tok, C.c_int32),
                                              _abi.ptr(pos, C.c_int32), n, _abi.ptr(nxt, C.c_int32), _abi.ptr(lg)))
        return (nxt, lg) if want_logits else nxt

    def generate(self, seq_ids, tokens, positions, steps: int) -> np.ndarray:
        seq, tok, pos = _abi.i32(seq_ids), _abi.i32(tokens), _abi.i32(positions)
        out = np.zeros((steps, len(seq)), np.int32)
        _abi.check(_abi.lib().llm_generate(self.h, _abi.ptr(seq, C.c_int32), _abi.ptr(tok, C.c_int32),
                                           _abi.ptr(pos, C.c_int32), len(seq), steps, _abi.ptr(out, C.c_int32)))
        return out

    def generate_begin(self, seq_ids, tokens, positions, max_steps: int) -> None:
        seq, tok, pos = _abi.i32(seq_ids), _abi.i32(tokens), _abi.i32(positions)
        _abi.check(_abi.lib().llm_generate_begin(self.h, _abi.ptr(seq, C.c_int32), _abi.ptr(tok, C.c_int32),
                                                 _abi.ptr(pos, C.c_int32), len(seq), max_steps))
        self._gen_n = len(seq)
        self._gen_max = max_steps

    def generate_steps(self, steps: int) -> None:
        _abi.check(_abi.lib().llm_generate_steps(self.h, steps))

    def generate_end(self) -> np.ndarray:
        out = np.zeros((self._gen_max, self._gen_n), np.int32)
        done = C.c_int32()
        _abi.check(_abi.lib().llm_generate_end(self.h, _abi.ptr(out, C.c_int32), C.byref(done)))
        return out[: done.value]

    def stream(self) -> int:
        s = C.c_void_p()
        _abi.check(_abi.lib().llm_ctx_stream(self.h, C.byref(s)))
        return s.value or 0

    def synchronize(self) -> None:
        _abi.check(_abi.lib().llm_synchronize(self.h))

    def step_parts(self, n: int) -> int:
        """Micro-batches a decode step of n sequences runs as (1 = single stream)."""
        k = C.c_int32()
        _abi.check(_abi.lib().llm_step_parts(self.h, n, C.byref(k)))
        return k.value

    def kernel_count(self, n: int) -> int:
        v = C.c_int32()
        _abi.check(_abi.lib().llm_step_kernel_count(self.h, n, C.byref(v)))
        return v.value

    def memory(self) -> dict:
        a, b, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _abi.check(_abi.lib().llm_memory_bytes(self.h, C.byref(a), C.byref(b), C.byref(c)))
        return dict(weights=a.value, kv_pool=b.value, other=c.value)

    def time_attention(self, iters: int):
        us, by = C.c_double(), C.c_double()
        _abi.check(_abi.lib().llm_time_attention(self.h, iters, C.byref(us), C.byref(by)))
        return us.value, by.value

    def set_option(self, option: int, value: int) -> None:
        _abi.check(_abi.lib().llm_set_option(self.h, option, int(value)))

    def profile_step(self, iters: int = 3):
        """Per-kernel table of one eager decode step of the current generate batch."""
        buf = C.create_string_buffer(16384)
        us = C.c_double()
        _abi.check(_abi.lib().llm_profile_step(self.h, iters, buf, len(buf), C.byref(us)))
        return buf.value.decode(), us.value

    def trace_begin(self) -> None:
        """Record the launch timeline of the following forward passes (see llm_trace_begin)."""
        _abi.check(_abi.lib().llm_trace_begin(self.h))

    def trace_end(self):
        buf = C.create_string_buffer(1 << 17)
        us = C.c_double()
        _abi.check(_abi.lib().llm_trace_end(self.h, buf, len(buf), C.byref(us)))
        return buf.value.decode(), us.value

    def trace_step(self):
        """Launch timeline (device globaltimer) of the next decode step of the generate batch."""
        buf = C.create_string_buffer(1 << 17)
        us = C.c_double()
        _abi.check(_abi.lib().llm_trace_step(self.h, buf, len(buf), C.byref(us)))
        return buf.value.decode(), us.value

    def read_kv(self, layer: int, seq: int, pos: int):
        k = np.zeros(self.cfg.kv_dim, np.float32)
        v = np.zeros(self.cfg.kv_dim, np.float32)
        _abi.check(_abi.lib().llm_debug_read_kv(self.h, layer, seq, pos, _abi.ptr(k), _abi.ptr(v)))
        return k, v

    def close(self) -> None:
        if getattr(self, "h", None):
            _abi.lib().llm_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Decoder:
    """ane/stories/infer.go:30-59: KV-cached decoder, here backed by the CUDA Engine."""

    def __init__(self, engine: Engine, maxSeq: int, seed: int):
        self.engine = engine
        self.maxSeq = maxSeq
        self.seed = seed
        # infer.go:131: the decoder's generator, seeded once; its draws persist across Decode
        # calls (per sequence slot on the device) until a Decode with a non-zero Seed reseeds
        engine.set_sampling(0.0, seed, True)

    def ResetCache(self) -> None:
        """infer.go:62-71."""
        for s in range(self.engine.max_batch):
            self.engine.release(s)

    def EvalNextLogits(self, token: int, pos: int) -> np.ndarray:
        """infer.go:73-77: logits after `token` at `pos` (sequence slot 0)."""
        if token < 0 or token >= self.engine.cfg.vocab:
            raise LLMError(_abi.LLM_ERR_TOKEN_RANGE, f"token out of range: {token}")
        if pos < 0 or pos >= self.maxSeq:
            raise LLMError(_abi.LLM_ERR_POS_RANGE, f"position out of range: {pos}")
        _, lg = self.engine.decode_step([0], [token], [pos], want_logits=True)
        return lg[0]

    def Decode(self, tok: Optional[Tokenizer], opts: DecodeOptions) -> DecodeResult:
        """infer.go:136-202 (greedy, or temperature sampling with the device generator)."""
        return self.DecodeBatch(tok, opts, [opts.PromptTokens])[0]

    def DecodeBatch(self, tok: Optional[Tokenizer], opts: DecodeOptions, prompts: List[List[int]]) -> List[DecodeResult]:
        """Decode of len(prompts) independent sequences in one batch (slots 0..n-1)."""
        n = len(prompts)
        if n > self.engine.max_batch:
            raise LLMError(_abi.LLM_ERR_INVALID, f"batch {n} exceeds the decoder's {self.engine.max_batch} slots")
        if opts.Temperature < 0:
            opts = DecodeOptions(opts.MaxNewTokens, 0.0, opts.Seed, opts.PromptTokens)
        if opts.Seed != 0:  # infer.go:150-152
            self.seed = opts.Seed
            self.engine.set_sampling(0.0, opts.Seed, True)
        lens = _abi.i32([len(p) for p in prompts])
        flat = _abi.i32([t for p in prompts for t in p] or [0])
        out = np.zeros((n, self.maxSeq), np.int32)
        ntok = np.zeros(n, np.int32)
        plen = np.zeros(n, np.int32)
        eos = np.zeros(n, np.int32)
        _abi.check(_abi.lib().llm_stories_decode_batch(
            self.engine.h, _abi.ptr(flat, C.c_int32), _abi.ptr(lens, C.c_int32), n, int(opts.MaxNewTokens),
            float(opts.Temperature), _abi.ptr(out, C.c_int32), _abi.ptr(ntok, C.c_int32), _abi.ptr(plen, C.c_int32),
            _abi.ptr(eos, C.c_int32)))
        res = []
        for i in range(n):
            toks = out[i, : ntok[i]].tolist()
            # infer.go:185-187: generatedText += tok.Decode(next), as bytes (Go strings)
            text = (b"".join(tok.DecodeBytes(t) for t in toks[plen[i]:]).decode("utf-8", "surrogateescape")
                    if tok is not None else "")
            res.append(DecodeResult(toks, int(plen[i]), text, bool(eos[i])))
        return res

    def Close(self) -> None:
        self.engine.close()


def NewDecoder(w: Optional[ModelWeights], maxSeq: int, seed: int, dtype: str = "fp16", device: int = 0,
               max_batch: int = 1) -> Decoder:
    """infer.go:80-133.  maxSeq <= 0 selects SeqDefault; it is not clamped to 256 (the
    CUDA path serves contexts up to the config's max_seq)."""
    if w is None:
        raise LLMError(_abi.LLM_ERR_INVALID, "nil model weights")
    cfg = w.Config
    if maxSeq <= 0:
        maxSeq = SeqDefault
    if len(w.Layers) != cfg.n_layers:
        raise LLMError(_abi.LLM_ERR_INVALID, f"layers={len(w.Layers)} want={cfg.n_layers}")
    if w.Embed.size % cfg.dim != 0:
        raise LLMError(_abi.LLM_ERR_INVALID, f"embed size={w.Embed.size} not divisible by dim={cfg.dim}")
    if maxSeq > cfg.max_seq:
        cfg = cfg.with_max_seq(maxSeq)
    eng = Engine(cfg, dtype, device)
    eng.load(w)
    eng.kv_alloc(max_batch, maxSeq)
    return Decoder(eng, maxSeq, seed)
