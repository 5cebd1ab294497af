"""CPU tests of the C ABI library: it loads, exports every symbol include/llm_cuda.h declares,
the seeded weight generator is deterministic with the documented statistics, and the
host-side error paths work without a GPU (no compute call is made here)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from ane import _abi
from ane.stories import STORIES_110M, QWEN3_0_6B, SyntheticWeights, ModelConfig

HEADER = Path(__file__).resolve().parent.parent / "include" / "llm_cuda.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _abi.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    missing = [s for s in decl if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(decl) == sorted(_abi.EXPORTS)


def test_synthetic_generator_deterministic_and_normal():
    a = _abi.synth_normal(1 << 20, 1234, _abi.synth_stream(0, 0))
    b = _abi.synth_normal(1 << 20, 1234, _abi.synth_stream(0, 0))
    c = _abi.synth_normal(1 << 20, 1235, _abi.synth_stream(0, 0))
    d = _abi.synth_normal(1 << 20, 1234, _abi.synth_stream(0, 1))
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c) and not np.array_equal(a, d)
    assert abs(float(a.mean())) < 1e-4
    assert abs(float(a.std()) - 0.02) < 1e-4
    # element i depends only on (seed, stream, i): a prefix is a prefix
    np.testing.assert_array_equal(_abi.synth_normal(1001, 1234, _abi.synth_stream(0, 0)), a[:1001])
    # scale folds into one rounding: (float)(0.02 * s * z)
    s = _abi.synth_normal(4096, 1234, _abi.synth_stream(0, 0), 0.02, 0.5)
    np.testing.assert_allclose(s, a[:4096] * 0.5, rtol=1e-6)


def test_synth_streams_distinct():
    ids = {_abi.synth_stream(l, k) for l in range(28) for k in range(7)} | {_abi.synth_stream(0, 7), _abi.synth_stream(0, 8)}
    assert len(ids) == 28 * 7 + 2


def test_synthetic_weights_shapes():
    cfg = ModelConfig(dim=128, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, vocab=300,
                      max_seq=64, qk_norm=True, tied_embed=True, norm_eps=1e-6, rope_theta=1e6)
    w = SyntheticWeights(cfg, 7, out_proj_scale=0.5)
    L = w.Layers[0]
    assert L.Wq.shape == (256, 128) and L.Wk.shape == (128, 128) and L.Wo.shape == (128, 256)
    assert L.W1.shape == (256, 128) and L.W2.shape == (128, 256) and L.QNorm.shape == (64,)
    assert w.Embed.shape == (300, 128)
    assert abs(float(L.Wo.std()) - 0.01) < 2e-3


def test_presets_match_reference_dims():
    # ane/stories/config.go:3-10
    assert (STORIES_110M.dim, STORIES_110M.hidden, STORIES_110M.n_heads, STORIES_110M.n_layers, STORIES_110M.vocab) == (768, 2048, 12, 12, 32000)
    # training/training_dynamic/models/qwen3_06b.h:6-16
    q = QWEN3_0_6B
    assert (q.dim, q.hidden, q.n_heads, q.n_kv_heads, q.head_dim, q.q_dim, q.kv_dim, q.n_layers, q.vocab) == (
        1024, 3072, 16, 8, 128, 2048, 1024, 28, 151936)


def test_last_error_and_invalid_arguments_without_gpu():
    L = _abi.lib()
    out = C.c_void_p()
    rc = L.llm_ctx_create(None, 1, 0, C.byref(out))
    assert rc == _abi.LLM_ERR_INVALID
    assert "nil config" in _abi.last_error()
    cfg = STORIES_110M.c_struct()
    rc = L.llm_ctx_create(C.byref(cfg), 99, 0, C.byref(out))
    assert rc == _abi.LLM_ERR_INVALID and "unknown dtype" in _abi.last_error()
    bad = ModelConfig(dim=768, hidden=2048, n_layers=1, n_heads=12, n_kv_heads=12, head_dim=32, vocab=10).c_struct()
    rc = L.llm_ctx_create(C.byref(bad), 1, 0, C.byref(out))
    assert rc == _abi.LLM_ERR_UNSUPPORTED and "head_dim" in _abi.last_error()
    assert L.llm_ctx_destroy(None) == _abi.LLM_ERR_INVALID


def test_no_cpu_fallback_without_device(gpu_available):
    if gpu_available:
        pytest.skip("a GPU is present")
    L = _abi.lib()
    out = C.c_void_p()
    cfg = STORIES_110M.c_struct()
    rc = L.llm_ctx_create(C.byref(cfg), 1, 0, C.byref(out))
    assert rc == _abi.LLM_ERR_CUDA
    assert "no CPU fallback" in _abi.last_error()
