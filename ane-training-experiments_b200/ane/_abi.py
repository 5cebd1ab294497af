"""ctypes binding of include/llm_cuda.h (the token loop's C ABI).

This module only marshals arguments; every computation happens in lib/libllm_cuda.so.
Loading fails loudly when the library has not been built: there is no Python or CPU
fallback for the token loop.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG_ROOT = Path(__file__).resolve().parent.parent          # ane-training-experiments_b200/
LIB_PATH = PKG_ROOT / "lib" / "libllm_cuda.so"

LLM_OK = 0
LLM_ERR_INVALID = -1
LLM_ERR_TOKEN_RANGE = -2
LLM_ERR_POS_RANGE = -3
LLM_ERR_CUDA = -4
LLM_ERR_OOM = -5
LLM_ERR_STATE = -6
LLM_ERR_UNSUPPORTED = -7
LLM_ERR_DEVICE = -8

LLM_DTYPE_F16 = 1
LLM_DTYPE_BF16 = 2
LLM_DTYPE_W8A8_F16 = 3
LLM_DTYPE_W8A8_BF16 = 4

LLM_WEIGHTS_LLAMA2C = 1
LLM_WEIGHTS_CHECKPOINT = 2

LLM_ARITH_STORIES = 0
LLM_ARITH_STORIESANE = 1

DTYPES = {
    "fp16": LLM_DTYPE_F16,
    "bf16": LLM_DTYPE_BF16,
    "w8a8_fp16": LLM_DTYPE_W8A8_F16,
    "w8a8_bf16": LLM_DTYPE_W8A8_BF16,
}

# every symbol include/llm_cuda.h declares
EXPORTS = [
    "llm_last_error", "llm_ctx_create", "llm_ctx_destroy", "llm_load_weights_f32", "llm_load_weights_file",
    "llm_load_weights_synthetic", "llm_synth_normal", "llm_synth_stream", "llm_kv_alloc",
    "llm_seq_release", "llm_prefill", "llm_decode_step", "llm_generate_begin",
    "llm_generate_steps", "llm_generate_end", "llm_generate", "llm_stories_decode",
    "llm_stories_decode_batch", "llm_ctx_stream", "llm_synchronize", "llm_step_kernel_count", "llm_step_parts",
    "llm_memory_bytes", "llm_time_attention", "llm_profile_step", "llm_trace_step", "llm_trace_begin", "llm_trace_end", "llm_debug_norm_quant", "llm_debug_gemm_i8",
    "llm_debug_gemm_f16", "llm_debug_read_kv", "llm_gemm_i8_splitk_noalloc", "llm_set_option", "llm_set_sampling", "llm_sample_uniform", "llm_debug_sample", "llm_debug_wait_timeout",
    "llm_eval_window", "llm_debug_exp2", "llm_shard_range", "llm_comm_unique_id", "llm_comm_create",
    "llm_comm_destroy", "llm_gather_tokens", "llm_comm_last_gather_ms", "llm_linear_create", "llm_linear_eval_cf", "llm_linear_destroy",
]

LLM_COMM_ID_BYTES = 128
LLM_OPT_CUDA_GRAPHS = 1
LLM_OPT_TCGEN05_GEMM = 2
LLM_OPT_PDL = 3
LLM_OPT_OVERLAP = 4
LLM_OPT_OVERLAP_RING_KB = 5
LLM_OPT_ATTN_SPLITS = 6
LLM_OPT_ATTN_CHAIN = 7
LLM_OPT_MICRO_BATCHES = 8
LLM_OPT_OVERLAP_GRAPHS = 9
LLM_OPT_CHAIN_PDL = 10
LLM_OPT_PREFILL_TILES = 11
LLM_OPT_PREFILL_RING_KB = 13
LLM_OPT_PREFILL_BN = 14
LLM_OPT_PREFILL_TC = 15
LLM_OPT_PREFILL_PERSIST = 16
LLM_OPT_DECODE_SPLITK = 17


class LLMError(RuntimeError):
    """A non-zero status from the C ABI; .code is the LLM_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class llm_model_config(C.Structure):
    _fields_ = [
        ("dim", C.c_int32), ("hidden", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("vocab", C.c_int32), ("max_seq", C.c_int32),
        ("qk_norm", C.c_int32), ("tied_embed", C.c_int32), ("norm_eps", C.c_double), ("rope_theta", C.c_double),
    ]


_FP = C.POINTER(C.c_float)


class llm_layer_weights_f32(C.Structure):
    _fields_ = [(n, _FP) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn", "q_norm", "k_norm")]


class llm_model_weights_f32(C.Structure):
    _fields_ = [("embed", _FP), ("rms_final", _FP), ("lm_head", _FP), ("layers", C.POINTER(llm_layer_weights_f32))]


_lib = None


def lib() -> C.CDLL:
    """Load lib/libllm_cuda.so (raises if it is missing; build with `make -C ane-training-experiments_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() or make -C {PKG_ROOT}")
    L = C.CDLL(str(LIB_PATH))
    i32p = C.POINTER(C.c_int32)
    sig = {
        "llm_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
        "llm_ctx_create": (C.c_int, [C.POINTER(llm_model_config), C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
        "llm_ctx_destroy": (C.c_int, [C.c_void_p]),
        "llm_load_weights_f32": (C.c_int, [C.c_void_p, C.POINTER(llm_model_weights_f32)]),
        "llm_load_weights_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float]),
        "llm_synth_normal": (None, [_FP, C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, C.c_double]),
        "llm_synth_stream": (C.c_uint64, [C.c_int, C.c_int]),
        "llm_kv_alloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int]),
        "llm_seq_release": (C.c_int, [C.c_void_p, C.c_int]),
        "llm_prefill": (C.c_int, [C.c_void_p, i32p, i32p, i32p, i32p, C.c_int, i32p, _FP]),
        "llm_decode_step": (C.c_int, [C.c_void_p, i32p, i32p, i32p, C.c_int, i32p, _FP]),
        "llm_generate_begin": (C.c_int, [C.c_void_p, i32p, i32p, i32p, C.c_int, C.c_int]),
        "llm_generate_steps": (C.c_int, [C.c_void_p, C.c_int]),
        "llm_generate_end": (C.c_int, [C.c_void_p, i32p, i32p]),
        "llm_generate": (C.c_int, [C.c_void_p, i32p, i32p, i32p, C.c_int, C.c_int, i32p]),
        "llm_stories_decode": (C.c_int, [C.c_void_p, C.c_int, i32p, C.c_int, C.c_int, C.c_float, i32p, i32p, i32p, i32p]),
        "llm_stories_decode_batch": (C.c_int, [C.c_void_p, i32p, i32p, C.c_int, C.c_int, C.c_float, i32p, i32p, i32p, i32p]),
        "llm_ctx_stream": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
        "llm_synchronize": (C.c_int, [C.c_void_p]),
        "llm_step_kernel_count": (C.c_int, [C.c_void_p, C.c_int, i32p]),
        "llm_step_parts": (C.c_int, [C.c_void_p, C.c_int, i32p]),
        "llm_memory_bytes": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
        "llm_time_attention": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "llm_load_weights_file": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
        "llm_set_sampling": (C.c_int, [C.c_void_p, C.c_float, C.c_uint64, C.c_int]),
        "llm_sample_uniform": (C.c_double, [C.c_uint64, C.c_int32, C.c_uint64]),
        "llm_debug_sample": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_void_p]),
        "llm_eval_window": (C.c_int, [C.c_void_p, C.c_int, i32p, C.c_int, C.c_int, i32p, _FP]),
        "llm_trace_begin": (C.c_int, [C.c_void_p]),
        "llm_trace_end": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_double)]),
        "llm_profile_step": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_double)]),
        "llm_trace_step": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_double)]),
        "llm_debug_norm_quant": (C.c_int, [C.c_int, _FP, _FP, C.c_int, C.c_int, C.c_double, C.POINTER(C.c_int8), _FP]),
        "llm_debug_gemm_i8": (C.c_int, [C.c_int, C.POINTER(C.c_int8), C.POINTER(C.c_int8), C.c_int, C.c_int, C.c_int, C.c_int, i32p]),
        "llm_debug_gemm_f16": (C.c_int, [C.c_int, C.c_int, _FP, _FP, C.c_int, C.c_int, C.c_int, C.c_int, _FP]),
        "llm_debug_read_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, _FP, _FP]),
        "llm_debug_exp2": (C.c_int, [C.c_int, _FP, C.c_int, _FP]),
        "llm_shard_range": (C.c_int, [C.c_int, C.c_int, C.c_int, i32p, i32p]),
        "llm_comm_unique_id": (C.c_int, [C.c_char_p, C.c_size_t]),
        "llm_comm_create": (C.c_int, [C.c_char_p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_double,
                                      C.POINTER(C.c_void_p)]),
        "llm_comm_destroy": (C.c_int, [C.c_void_p]),
        "llm_gather_tokens": (C.c_int, [C.c_void_p, i32p, C.c_int, C.c_int, C.c_int, i32p]),
        "llm_comm_last_gather_ms": (C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
        "llm_linear_create": (C.c_int, [C.c_int, C.c_int, _FP, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
        "llm_linear_eval_cf": (C.c_int, [C.c_void_p, _FP, C.c_int, _FP, C.POINTER(C.c_uint64)]),
        "llm_linear_destroy": (C.c_int, [C.c_void_p]),
        "llm_set_option": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
        "llm_gemm_i8_splitk_noalloc": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_void_p, C.c_void_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib().llm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != LLM_OK:
        raise LLMError(rc, last_error())


def ptr(a: np.ndarray | None, ctype=C.c_float):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the C ABI must be C-contiguous"
    return a.ctypes.data_as(C.POINTER(ctype))


def i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def synth_normal(n: int, seed: int, stream: int, stddev: float = 0.02, scale: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().llm_synth_normal(ptr(out), n, seed, stream, stddev, scale)
    return out


def synth_stream(layer: int, kind: int) -> int:
    return int(lib().llm_synth_stream(layer, kind))
