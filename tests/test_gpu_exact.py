"""Bit-exact parity of the CUDA token loop with the oracle in GPU order.

The oracle's GPU-order mode restates the CUDA path's arithmetic step for step: the measured
rounding of the tensor-core MMA (exact products, terms truncated to a 26-bit window below the
largest alignment exponent, the sum rounded toward zero), the deterministic exp2 of the softmax
and SwiGLU gate, the row kernel's lane-ordered float64 RMS sums, and the fixed reduction orders
of the prefill and decode attention kernels.  These tests check each piece on the device and
then whole decodes, where logits and tokens must be identical bit for bit.  The decode
attention's reduction order does not depend on the split count, so a sequence's results do not
depend on the batch it runs in (reference rows are independent: ane/stories/infer.go:204-299)."""
import numpy as np
import pytest

import oracle as O
from ane import _abi
from ane.stories import ModelConfig, SyntheticWeights
from parity import gpu_order, gpu_run, oracle_check
from test_gpu_decode import TINY_GQA, TINY_MHA, engine, weights

pytestmark = pytest.mark.gpu


def _act_values(rng, shape, act, kind):
    if kind == "normal":
        x = rng.standard_normal(shape)
    else:  # exponents spread over 2^-12 .. 2^4, random signs
        x = rng.choice([-1.0, 1.0], shape) * rng.uniform(1, 2, shape) * np.exp2(rng.integers(-12, 5, shape))
    x = x.astype(np.float32)
    r = O.round_f16 if act == 1 else O.round_bf16
    return np.vectorize(r, otypes=[np.float32])(x)


@pytest.mark.parametrize("act", [1, 2], ids=["fp16", "bf16"])
@pytest.mark.parametrize("path", [-1, 1], ids=["tcgen05", "mma.sync"])
@pytest.mark.parametrize("kind", ["normal", "wide"])
def test_gemm_kernels_follow_the_tensor_core_model(act, path, kind):
    """The 16-bit GEMM kernels (tcgen05 and mma.sync, no split-K) against O.gemm_mma: every
    output bit-identical."""
    rng = np.random.default_rng(10 * act + (path > 0) + (kind == "wide") * 100)
    M, N, K = 128, 128, 256
    A = _act_values(rng, (M, K), act, kind)
    B = _act_values(rng, (N, K), act, kind)
    C = np.zeros((M, N), np.float32)
    _abi.check(_abi.lib().llm_debug_gemm_f16(0, act, _abi.ptr(A), _abi.ptr(B), M, N, K, path, _abi.ptr(C)))
    want = O.gemm_mma(A, B, act)
    bad = np.count_nonzero(C.view(np.uint32) != want.view(np.uint32))
    assert bad == 0, f"{bad} of {C.size} outputs differ from the model"


@pytest.mark.parametrize("act,M,N,K,S", [(1, 64, 768, 2048, 8), (2, 128, 1024, 3072, 8), (2, 37, 256, 1024, 4),
                                         (1, 128, 2304, 768, 4), (2, 5, 512, 384, 2), (1, 100, 96, 512, 4)])
def test_split_k_gemm_follows_the_model(act, M, N, K, S):
    """Decode projections split K over clusters of S CTAs (contiguous ranges of 64-element
    slices, one MMA chain each, the partial tiles summed in rank order through distributed
    shared memory): every output bit-identical to O.gemm_mma_splitk."""
    rng = np.random.default_rng(M + N + K + S + act)
    A = _act_values(rng, (M, K), act, "normal")
    B = _act_values(rng, (N, K), act, "wide")
    C = np.zeros((M, N), np.float32)
    _abi.check(_abi.lib().llm_debug_gemm_f16(0, act, _abi.ptr(A), _abi.ptr(B), M, N, K, -(1000 + S), _abi.ptr(C)))
    want = O.gemm_mma_splitk(A, B, act, S)
    bad = np.count_nonzero(C.view(np.uint32) != want.view(np.uint32))
    assert bad == 0, f"{bad} of {C.size} outputs differ from the model"
    if S > 1:  # the split changes the rounding (the model tells which)
        assert np.count_nonzero(want.view(np.uint32) != O.gemm_mma(A, B, act).view(np.uint32)) > 0


@pytest.mark.parametrize("M,N,K,S", [(64, 768, 2048, 8), (256, 1024, 3072, 8), (7, 384, 768, 2), (130, 512, 1024, 4)])
def test_split_k_int8_gemm_exact(M, N, K, S):
    """int8 split-K partials are int32 sums: the result is the exact product."""
    import ctypes as C_
    rng = np.random.default_rng(M * 3 + S)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    out = np.zeros((M, N), np.int32)
    _abi.check(_abi.lib().llm_debug_gemm_i8(0, _abi.ptr(A, C_.c_int8), _abi.ptr(B, C_.c_int8), M, N, K, -(1000 + S),
                                            _abi.ptr(out, C_.c_int32)))
    np.testing.assert_array_equal(out, A.astype(np.int64) @ B.astype(np.int64).T)


def test_device_exp2_equals_oracle():
    rng = np.random.default_rng(3)
    x = np.concatenate([np.linspace(-130, 130, 20001), rng.uniform(-30, 1, 20000), [-np.inf, np.inf, 0.0, -126.0,
                                                                                   127.49, 127.5]]).astype(np.float32)
    out = np.zeros_like(x)
    _abi.check(_abi.lib().llm_debug_exp2(0, _abi.ptr(x), x.size, _abi.ptr(out)))
    want = np.array([O.exp2_det(float(v)) for v in x], np.float32)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))
    ok = (x > -120) & (x < 120)
    rel = np.abs(out[ok].astype(np.float64) - np.exp2(x[ok].astype(np.float64))) / np.exp2(x[ok].astype(np.float64))
    assert rel.max() < 2.5e-7  # within ~2 ulp of 2^x


def _exact(cfg, dtype, w, prompts, steps, max_pos, splits=0):
    eng = engine(cfg, dtype, w, max_batch=len(prompts), max_pos=max_pos)
    if splits:
        eng.set_option(_abi.LLM_OPT_ATTN_SPLITS, splits)
    toks, logits = gpu_run(eng, prompts, steps)
    eng.close()
    return toks, logits


@pytest.mark.parametrize("cfg", [TINY_MHA, TINY_GQA], ids=lambda c: c.name)
@pytest.mark.parametrize("dtype", ["fp16", "bf16", "w8a8_fp16", "w8a8_bf16"])
def test_tiny_decode_bit_exact(cfg, dtype):
    """Prompts across prefill tiles (64 positions), decode continuing into a second 32-page
    segment (512 positions): logits and tokens equal the GPU-order oracle's bit for bit."""
    cfg = cfg.with_max_seq(640)
    w = weights(cfg)
    rng = np.random.default_rng(7)
    lens = [1, 17, 64, 65, 130, 500]
    prompts = [rng.integers(3, cfg.vocab, L).tolist() for L in lens]
    toks, logits = _exact(cfg, dtype, w, prompts, steps=20, max_pos=544)
    m = gpu_order(cfg, w, dtype)
    worst, agree, n = oracle_check(m, prompts, toks, logits)
    print(f"{cfg.name} {dtype}: max|dlogit| vs GPU-order oracle = {worst:.3e}, top1 {agree:.4f} over {n}")
    assert worst == 0.0 and agree == 1.0


@pytest.mark.parametrize("dtype", ["bf16", "w8a8_bf16"])
def test_split_count_does_not_change_results(dtype):
    """The same sequences decoded with 1, 2 and 3 CTAs per (sequence, kv head): identical."""
    cfg = TINY_GQA.with_max_seq(1700)
    w = weights(cfg)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(3, cfg.vocab, L).tolist() for L in (1100, 1530, 5)]  # up to 4 segments
    runs = [_exact(cfg, dtype, w, prompts, steps=12, max_pos=1600, splits=s) for s in (1, 2, 3)]
    for toks, logits in runs[1:]:
        assert toks == runs[0][0]
        for a, b in zip(logits, runs[0][1]):
            assert np.array_equal(a, b)
