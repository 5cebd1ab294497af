"""ctypes wrapper of oracle/_build/liboracle.so -- TEST INFRASTRUCTURE.

The CPU restatement of the reference decoder (see oracle.h for the file:line map).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU legs use it, as the checker and as the
timed CPU baseline; the product path never imports it.  Parity of the end-to-end decoder
is unpinned by the reference (no golden vectors exist and the Go code cannot run here).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

F32, F16, BF16, W8A8_F16, W8A8_BF16 = 0, 1, 2, 3, 4
MODES = {"fp32": F32, "fp16": F16, "bf16": BF16, "w8a8_fp16": W8A8_F16, "w8a8_bf16": W8A8_BF16}
OK, EINVAL, ERANGE_TOKEN, ERANGE_POS = 0, -1, -2, -3


class oracle_config(C.Structure):
    _fields_ = [("dim", C.c_int32), ("hidden", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("vocab", C.c_int32), ("max_seq", C.c_int32),
                ("qk_norm", C.c_int32), ("mode", C.c_int32), ("norm_eps", C.c_double), ("rope_theta", C.c_double)]


_FP = C.POINTER(C.c_float)

# Model dimensions of the two reference models (ane/stories/config.go:3-10 with infer.go:102,307;
# training/training_dynamic/models/qwen3_06b.h:6-16 with per-head QK-norm, theta 1e6, eps 1e-6).
PRESETS = {
    "stories110m": dict(dim=768, hidden=2048, n_layers=12, n_heads=12, n_kv_heads=12, head_dim=64, vocab=32000,
                        max_seq=256, qk_norm=0, norm_eps=1e-5, rope_theta=10000.0, tied_embed=1),
    "qwen3-0.6b": dict(dim=1024, hidden=3072, n_layers=28, n_heads=16, n_kv_heads=8, head_dim=128, vocab=151936,
                       max_seq=4096, qk_norm=1, norm_eps=1e-6, rope_theta=1e6, tied_embed=1),
}


class oracle_layer_f32(C.Structure):
    _fields_ = [(n, _FP) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn", "q_norm", "k_norm")]


class oracle_weights_f32(C.Structure):
    _fields_ = [("embed", _FP), ("rms_final", _FP), ("lm_head", _FP), ("layers", C.POINTER(oracle_layer_f32))]


_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, seconds)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = C.CDLL(str(LIB_PATH))
    i32p = C.POINTER(C.c_int32)
    i8p = C.POINTER(C.c_int8)
    sig = {
        "oracle_model_new": (C.c_void_p, [C.POINTER(oracle_config), C.POINTER(oracle_weights_f32)]),
        "oracle_model_free": (None, [C.c_void_p]),
        "oracle_model_set_storiesane": (None, [C.c_void_p, C.c_int]),
        "oracle_model_set_gpu_order": (None, [C.c_void_p, C.c_int]),
        "oracle_model_set_decode_splitk": (None, [C.c_void_p, C.c_int]),
        "oracle_decode_splits": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int]),
        "oracle_gemm_mma_splitk": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_void_p]),
        "oracle_seq_set_prefill": (None, [C.c_void_p, C.c_int]),
        "oracle_seq_set_logits_from": (None, [C.c_void_p, C.c_int]),
        "oracle_exp2_det": (C.c_float, [C.c_float]),
        "oracle_mma16": (C.c_float, [C.c_float, _FP, _FP, C.c_int, C.c_int]),
        "oracle_gemm_mma": (None, [_FP, _FP, C.c_int, C.c_int, C.c_int, C.c_int, _FP]),
        "oracle_embed_lookup_cf": (None, [_FP, _FP, C.c_int, i32p, C.c_int, C.c_int]),
        "oracle_seq_new": (C.c_void_p, [C.c_void_p]),
        "oracle_seq_free": (None, [C.c_void_p]),
        "oracle_seq_reset": (None, [C.c_void_p]),
        "oracle_seq_fill_kv_synthetic": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_uint64]),
        "oracle_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, _FP]),
        "oracle_decode": (C.c_int, [C.c_void_p, C.c_void_p, i32p, C.c_int, C.c_int, i32p, i32p, i32p, i32p]),
        "oracle_teacher_forced": (C.c_int, [C.c_void_p, C.c_void_p, i32p, C.c_int, i32p, _FP]),
        "oracle_argmax": (C.c_int, [_FP, C.c_int]),
        "oracle_sample_from_logits": (C.c_int, [_FP, C.c_int, C.c_float, C.c_double]),
        "oracle_uniform": (C.c_double, [C.c_uint64, C.c_uint64, C.c_uint64]),
        "oracle_rmsnorm": (None, [_FP, _FP, _FP, C.c_int, C.c_double]),
        "oracle_rope_tables": (None, [C.c_int, C.c_int, C.c_double, _FP, _FP]),
        "oracle_softmax_prefix": (None, [_FP, _FP, C.c_int]),
        "oracle_silu": (C.c_float, [C.c_float]),
        "oracle_round_f16": (C.c_float, [C.c_float]),
        "oracle_round_bf16": (C.c_float, [C.c_float]),
        "oracle_quant_rows": (None, [_FP, C.c_int, C.c_int, i8p, _FP]),
        "oracle_norm_quant_rows_lane_order": (None, [_FP, _FP, C.c_int, C.c_int, C.c_double, i8p, _FP]),
        "oracle_norm_rows_lane_order": (None, [_FP, _FP, C.c_int, C.c_int, C.c_double, C.c_int, _FP]),
        "oracle_gemm_i8": (None, [i8p, i8p, C.c_int, C.c_int, C.c_int, i32p]),
        "oracle_dequant": (C.c_float, [C.c_int32, C.c_float, C.c_float]),
        "oracle_set_threads": (None, [C.c_int]),
        "oracle_synth_normal": (None, [_FP, C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, C.c_double]),
        "oracle_synth_stream": (C.c_uint64, [C.c_int, C.c_int]),
        "oracle_set_attn_reverse": (None, [C.c_int]),
        "oracle_set_matvec_reverse": (None, [C.c_int]),
        "oracle_get_threads": (C.c_int, []),
    }
    for n, (r, a) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = r, a
    _lib = L
    return L


def _p(a, t=C.c_float):
    return None if a is None else a.ctypes.data_as(C.POINTER(t))


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


class Model:
    """oracle_model over fp32 weights given as a dict or as ane.stories.ModelWeights."""

    def __init__(self, cfg: dict, weights, mode: str = "fp32", storiesane: bool = False, gpu_order: bool = False,
                 decode_splitk: bool = True):
        """gpu_order: restate the CUDA path's order of operations (bit-identical results in
        the emulation modes); default: the reference's arithmetic at the mode's precision."""
        self.cfg = dict(cfg)
        self.vocab = cfg["vocab"]
        self.max_seq = cfg["max_seq"]
        oc = oracle_config(cfg["dim"], cfg["hidden"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                           cfg["head_dim"], cfg["vocab"], cfg["max_seq"], int(cfg.get("qk_norm", 0)), MODES[mode],
                           float(cfg.get("norm_eps", 1e-5)), float(cfg.get("rope_theta", 10000.0)))
        self._keep = []
        L = len(weights.Layers)
        layers = (oracle_layer_f32 * L)()
        for i, lw in enumerate(weights.Layers):
            for name, arr in (("wq", lw.Wq), ("wk", lw.Wk), ("wv", lw.Wv), ("wo", lw.Wo), ("w1", lw.W1),
                              ("w2", lw.W2), ("w3", lw.W3), ("rms_att", lw.RMSAtt), ("rms_ffn", lw.RMSFFN),
                              ("q_norm", lw.QNorm), ("k_norm", lw.KNorm)):
                if arr is not None:
                    a = f32(arr)
                    self._keep.append(a)
                    setattr(layers[i], name, _p(a))
        emb, fin = f32(weights.Embed), f32(weights.RMSFinal)
        lm = None if weights.SharedCL else f32(weights.LMHead)
        self._keep += [emb, fin, lm, layers]
        w = oracle_weights_f32(_p(emb), _p(fin), _p(lm), layers)
        self.h = lib().oracle_model_new(C.byref(oc), C.byref(w))
        if not self.h:
            raise ValueError("oracle_model_new rejected the configuration")
        if storiesane:
            lib().oracle_model_set_storiesane(self.h, 1)
        self.gpu_order = bool(gpu_order) and mode != "fp32"
        if self.gpu_order:
            lib().oracle_model_set_gpu_order(self.h, 1)
            # decode rows' projections split K as the library's default (LLM_OPT_DECODE_SPLITK)
            lib().oracle_model_set_decode_splitk(self.h, 1 if decode_splitk else 0)

    def eval_window(self, tokens) -> np.ndarray:
        """ane/storiesane/engine.go:804-842: logits of every window position, channel-first
        [vocab, len(tokens)] (positions 0..len-1 from an empty cache; one prefill)."""
        _, lg = self.seq().teacher_forced(list(tokens), want_logits=True, n_prefill=len(tokens))
        return np.ascontiguousarray(lg.T)

    def seq(self) -> "Seq":
        return Seq(self)

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_model_free(self.h)
            self.h = None


class Seq:
    def __init__(self, m: Model):
        self.m = m
        self.h = lib().oracle_seq_new(m.h)

    def reset(self):
        lib().oracle_seq_reset(self.h)

    def fill_kv(self, n_pos: int, seed: int):
        lib().oracle_seq_fill_kv_synthetic(self.m.h, self.h, n_pos, seed)

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.m.vocab, np.float32)
        rc = lib().oracle_forward(self.m.h, self.h, token, pos, _p(out))
        if rc == ERANGE_TOKEN:
            raise ValueError(f"token out of range: {token}")
        if rc == ERANGE_POS:
            raise ValueError(f"position out of range: {pos}")
        if rc:
            raise ValueError(f"oracle_forward failed: {rc}")
        return out

    def decode(self, prompt, max_new: int):
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        out = np.zeros(self.m.max_seq + 1, np.int32)
        n, pl, eos = C.c_int32(), C.c_int32(), C.c_int32()
        rc = lib().oracle_decode(self.m.h, self.h, _p(p, C.c_int32), len(p), max_new, _p(out, C.c_int32),
                                 C.byref(n), C.byref(pl), C.byref(eos))
        if rc:
            raise ValueError(f"oracle_decode failed: {rc}")
        return out[: n.value].tolist(), pl.value, bool(eos.value)

    def teacher_forced(self, tokens, want_logits=False, n_prefill=0, logits_from=0):
        """n_prefill (GPU order): the first n_prefill positions were one prefill (the prompt);
        the rest decode steps.  Positions below logits_from skip the classifier (their logits
        and argmax are not meaningful)."""
        lib().oracle_seq_set_prefill(self.h, int(n_prefill))
        lib().oracle_seq_set_logits_from(self.h, int(logits_from))
        t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        am = np.zeros(len(t), np.int32)
        lg = np.zeros((len(t), self.m.vocab), np.float32) if want_logits else None
        rc = lib().oracle_teacher_forced(self.m.h, self.h, _p(t, C.c_int32), len(t), _p(am, C.c_int32), _p(lg))
        if rc:
            raise ValueError(f"oracle_teacher_forced failed: {rc}")
        return (am, lg) if want_logits else am

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_seq_free(self.h)
            self.h = None


# ---------------------------------------------------------------- building blocks
def rmsnorm(x, w, eps=1e-5):
    x, w = f32(x), f32(w)
    out = np.zeros_like(x)
    lib().oracle_rmsnorm(_p(out), _p(x), _p(w), len(x), eps)
    return out


def rope_tables(max_pos, hd, theta=10000.0):
    c = np.zeros((max_pos, hd // 2), np.float32)
    s = np.zeros_like(c)
    lib().oracle_rope_tables(max_pos, hd, theta, _p(c), _p(s))
    return c, s


def softmax_prefix(x):
    x = f32(x)
    out = np.zeros_like(x)
    lib().oracle_softmax_prefix(_p(out), _p(x), len(x))
    return out


def quant_rows(x):
    x = f32(x)
    q = np.zeros(x.shape, np.int8)
    s = np.zeros(x.shape[0], np.float32)
    lib().oracle_quant_rows(_p(x), x.shape[0], x.shape[1], _p(q, C.c_int8), _p(s))
    return q, s


def norm_quant_rows(x, w, eps):
    x, w = f32(x), f32(w)
    q = np.zeros(x.shape, np.int8)
    s = np.zeros(x.shape[0], np.float32)
    lib().oracle_norm_quant_rows_lane_order(_p(x), _p(w), x.shape[0], x.shape[1], eps, _p(q, C.c_int8), _p(s))
    return q, s


def gemm_i8(A, B):
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    Cm = np.zeros((A.shape[0], B.shape[0]), np.int32)
    lib().oracle_gemm_i8(_p(A, C.c_int8), _p(B, C.c_int8), A.shape[0], B.shape[0], A.shape[1], _p(Cm, C.c_int32))
    return Cm


def exp2_det(x: float) -> float:
    return lib().oracle_exp2_det(x)


def mma16(c: float, a, b, act: int) -> float:
    """One tensor-core MMA step (see oracle.h oracle_mma16); act 1 fp16, 2 bf16."""
    a, b = f32(a), f32(b)
    return lib().oracle_mma16(c, _p(a), _p(b), a.size, act)


def gemm_mma(A, B, act: int):
    """C = A . B^T as the 16-bit GEMM kernels form it (MMA chain over k, no split-K)."""
    A, B = f32(A), f32(B)
    Cm = np.zeros((A.shape[0], B.shape[0]), np.float32)
    lib().oracle_gemm_mma(_p(A), _p(B), A.shape[0], B.shape[0], A.shape[1], act, _p(Cm))
    return Cm


def gemm_mma_splitk(A, B, act: int, splits: int):
    """oracle_gemm_mma_splitk: the MMA chains of gemm_mma over `splits` contiguous ranges of
    64-element K slices, summed in range order."""
    A = f32(A)
    B = f32(B)
    M, K = A.shape
    N = B.shape[0]
    out = np.zeros((M, N), np.float32)
    lib().oracle_gemm_mma_splitk(_p(A), _p(B), M, N, K, act, splits, _p(out))
    return out


def decode_splits(in8: bool, n: int, k: int, bnmax: int) -> int:
    """Split-K of a decode step's projection (oracle_decode_splits)."""
    return int(lib().oracle_decode_splits(1 if in8 else 0, n, k, bnmax))


def embed_lookup_cf(embed, tokens, dim: int, seq: int):
    """ane/stories/cpu.go:41-72 EmbedLookup: [dim * seq] channel-first."""
    e = f32(embed)
    t = np.ascontiguousarray(np.asarray(tokens, np.int32))
    out = np.full(dim * seq, np.nan, np.float32)
    lib().oracle_embed_lookup_cf(_p(out), _p(e), e.size // dim, _p(t, C.c_int32), dim, seq)
    return out


def round_f16(x: float) -> float:
    return lib().oracle_round_f16(x)


def round_bf16(x: float) -> float:
    return lib().oracle_round_bf16(x)


SAMPLE_STREAM_BASE = 0x5A4D000000000000


def uniform(seed: int, slot: int, counter: int) -> float:
    """The CUDA path's sampling uniform for sequence slot `slot`, draw number `counter`."""
    return lib().oracle_uniform(seed, SAMPLE_STREAM_BASE + slot, counter)


def sample_from_logits(logits, temperature: float, u: float) -> int:
    """ane/stories/infer.go:347-371 with the uniform given."""
    a = f32(logits)
    return lib().oracle_sample_from_logits(_p(a), a.size, temperature, u)


class _Layer:
    def __init__(self, **kw):
        self.__dict__.update(kw)


class SynthWeights:
    """The synthetic model's fp32 weights from oracle_synth_normal (the layout O.Model reads)."""

    def __init__(self, cfg: dict, seed: int = 1234, out_proj_scale: float = 1.0, stddev: float = 0.02):
        D, F, L = cfg["dim"], cfg["hidden"], cfg["n_layers"]
        hd = cfg["head_dim"]
        Q, KV = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd

        def g(n, l, k, s=1.0):
            out = np.empty(n, np.float32)
            lib().oracle_synth_normal(_p(out), n, seed, lib().oracle_synth_stream(l, k), stddev, s)
            return out

        qk = bool(cfg.get("qk_norm", 0))
        self.Layers = [_Layer(Wq=g(Q * D, l, 0).reshape(Q, D), Wk=g(KV * D, l, 1).reshape(KV, D),
                              Wv=g(KV * D, l, 2).reshape(KV, D), Wo=g(D * Q, l, 3, out_proj_scale).reshape(D, Q),
                              W1=g(F * D, l, 4).reshape(F, D), W2=g(D * F, l, 5, out_proj_scale).reshape(D, F),
                              W3=g(F * D, l, 6).reshape(F, D), RMSAtt=np.ones(D, np.float32),
                              RMSFFN=np.ones(D, np.float32), QNorm=np.ones(hd, np.float32) if qk else None,
                              KNorm=np.ones(hd, np.float32) if qk else None) for l in range(L)]
        self.RMSFinal = np.ones(D, np.float32)
        self.Embed = g(cfg["vocab"] * D, 0, 7).reshape(cfg["vocab"], D)
        self.SharedCL = bool(cfg.get("tied_embed", 1))
        self.LMHead = None if self.SharedCL else g(cfg["vocab"] * D, 0, 8).reshape(cfg["vocab"], D)


def set_attn_reverse(on: bool):
    lib().oracle_set_attn_reverse(int(on))


def set_matvec_reverse(on: bool):
    lib().oracle_set_matvec_reverse(int(on))


def set_threads(n: int):
    lib().oracle_set_threads(n)


def get_threads() -> int:
    return lib().oracle_get_threads()
