"""GPU kernel checks through the C ABI debug hooks against the CPU oracle.

Bit-exact: the per-token RMSNorm + int8 quantiser (bridge/ane_bridge.m:374-398 applied per
row, float64 sum of squares in the documented lane order) and the int8 GEMM's int32
accumulators.  Tolerance: the fp16/bf16 GEMM against an fp32 product of the same rounded
inputs (1e-4 of sum |a||b|: only the summation order differs)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from ane import _abi

pytestmark = pytest.mark.gpu


def dev_norm_quant(x, w, eps):
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    _abi.check(_abi.lib().llm_debug_norm_quant(0, _abi.ptr(x), _abi.ptr(w), rows, cols, eps,
                                               _abi.ptr(q, C.c_int8), _abi.ptr(s)))
    return q, s


@pytest.mark.parametrize("cols", [128, 768, 1024, 2048, 3072])
@pytest.mark.parametrize("rows", [37, 1100])  # 1100: the warp-per-row kernel of prefill-sized RMSNorms
def test_norm_quant_bit_exact(cols, rows):
    rng = np.random.default_rng(cols)
    x = (rng.standard_normal((rows, cols)) * rng.uniform(1e-3, 30, (rows, 1))).astype(np.float32)
    x[3] = 0.0  # all-zero row: scale falls back to 1
    w = (1 + 0.3 * rng.standard_normal(cols)).astype(np.float32)
    for eps in (1e-5, 1e-6):
        q, s = dev_norm_quant(x, w, eps)
        qo, so = O.norm_quant_rows(x, w, eps)
        np.testing.assert_array_equal(s, so)
        np.testing.assert_array_equal(q, qo)


def test_quant_only_bit_exact():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 2048)) * 5).astype(np.float32)
    x[0, :] = 0.49999997  # f32 `v + 0.5` rounding case of the bridge rule
    x[0, 0] = 127.0
    q, s = dev_norm_quant(x, None, 1e-5)
    qo, so = O.quant_rows(x)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(q, qo)


def test_quantiser_rounding_boundaries_bit_exact():
    """Values within a few ulps of every k + 0.5 quotient for a non-power-of-two scale: the
    device quantiser's reciprocal fast path must fall back to the IEEE quotient there."""
    rows = []
    for mx in (100.0, 3.7, 0.0123, 5000.0):
        sc = np.float32(mx) / np.float32(127.0)
        vals = []
        for k in range(-128, 127):
            c = np.float32((k + 0.5) * sc)
            for d in range(-3, 4):
                vals.append(np.float32(c) if d == 0 else np.nextafter(c, np.float32(np.inf if d > 0 else -np.inf), dtype=np.float32))
                for _ in range(abs(d) - 1):
                    vals[-1] = np.nextafter(vals[-1], np.float32(np.inf if d > 0 else -np.inf), dtype=np.float32)
        vals = np.array(vals, np.float32)
        vals = np.clip(vals, -mx, mx)
        n = (len(vals) + 1 + 127) // 128 * 128
        row = np.zeros(n, np.float32)
        row[0] = mx
        row[1:1 + len(vals)] = vals
        rows.append(row)
    width = max(len(r) for r in rows)
    x = np.stack([np.pad(r, (0, width - len(r))) for r in rows]).astype(np.float32)
    q, s = dev_norm_quant(x, None, 1e-5)
    qo, so = O.quant_rows(x)
    np.testing.assert_array_equal(s, so)
    np.testing.assert_array_equal(q, qo)


def dev_gemm_i8(A, B, splits):
    """splits < 0: the tcgen05 kernel (-1 the model's channel tile, -bn tile width bn);
    otherwise the warp-level kernel with that split."""
    M, K = A.shape
    N = B.shape[0]
    Cm = np.zeros((M, N), np.int32)
    _abi.check(_abi.lib().llm_debug_gemm_i8(0, _abi.ptr(A, C.c_int8), _abi.ptr(B, C.c_int8), M, N, K, splits,
                                            _abi.ptr(Cm, C.c_int32)))
    return Cm


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (7, 384, 768), (64, 1000, 1024), (256, 1024, 3072),
                                   (130, 4096, 1024), (300, 256, 2048)])
@pytest.mark.parametrize("splits", [-1, -16, -32, -64, -128, -256, 0, 1, 3],
                         ids=["tcgen05", "tcgen05-n16", "tcgen05-n32", "tcgen05-n64", "tcgen05-n128", "tcgen05-n256",
                              "mma-auto", "mma-1", "mma-3"])
def test_gemm_i8_bit_exact(M, N, K, splits):
    rng = np.random.default_rng(M * 7 + N + K + splits)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    A[0, :] = -128  # extreme accumulators
    B[0, :] = -128
    np.testing.assert_array_equal(dev_gemm_i8(A, B, splits), O.gemm_i8(A, B))


def round_to(x, dtype):
    import torch
    t = torch.from_numpy(x).to(torch.float16 if dtype == _abi.LLM_DTYPE_F16 else torch.bfloat16)
    return t.float().numpy()


@pytest.mark.parametrize("dtype", [_abi.LLM_DTYPE_F16, _abi.LLM_DTYPE_BF16])
@pytest.mark.parametrize("M,N,K,splits", [(1, 128, 64, 0), (64, 2304, 768, 0), (129, 1000, 1024, 2), (256, 1024, 3072, 0),
                                          (1, 128, 64, -1), (64, 2304, 768, -1), (129, 1000, 1024, -1),
                                          (256, 1024, 3072, -1), (600, 384, 256, -1), (256, 1024, 2048, -16),
                                          (129, 1000, 1024, -32), (300, 2048, 512, -256)])
def test_gemm_16bit_matches_fp32_reference(dtype, M, N, K, splits):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    _abi.check(_abi.lib().llm_debug_gemm_f16(0, dtype, _abi.ptr(A), _abi.ptr(B), M, N, K, splits, _abi.ptr(Cm)))
    ref = round_to(A, dtype).astype(np.float64) @ round_to(B, dtype).astype(np.float64).T
    scale = np.abs(round_to(A, dtype)).astype(np.float64) @ np.abs(round_to(B, dtype)).astype(np.float64).T
    assert np.all(np.abs(Cm - ref) <= 1e-4 * scale + 1e-6)

