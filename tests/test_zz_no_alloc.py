"""The allocation-free split-K int8 GEMM (llm_gemm_i8_splitk_noalloc) against the oracle's exact
int8 GEMM (an independent CPU product) and the allocating entry point (llm_debug_gemm_i8).

It serves callers that cannot allocate device memory while they run: a server whose KV page
pool already holds the GPU's memory, a decode loop that must not take cudaFree's device-wide
synchronisation mid-step, or an FFI host that owns the memory policy.  They pass their own
device buffers; the split-K partials and counters live in a fixed array inside the library.
Collected last so a failure here cannot hide earlier results; it also passes on its own."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from ane import _abi

pytestmark = pytest.mark.gpu


def allocating_reference(A, B, splits):
    M, K = A.shape
    N = B.shape[0]
    out = np.zeros((M, N), np.int32)
    _abi.check(_abi.lib().llm_debug_gemm_i8(0, _abi.ptr(A, C.c_int8), _abi.ptr(B, C.c_int8), M, N, K, splits,
                                            _abi.ptr(out, C.c_int32)))
    return out


@pytest.mark.parametrize("M,N,K,splits", [(64, 1024, 2048, 4), (256, 512, 3072, 8), (7, 384, 768, 3), (130, 256, 256, 1)])
def test_noalloc_split_k_gemm_matches_allocating_entry_point(M, N, K, splits):
    import torch
    rng = np.random.default_rng(M + N + K + splits)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    want = O.gemm_i8(A, B)
    np.testing.assert_array_equal(want, A.astype(np.int64) @ B.astype(np.int64).T)
    np.testing.assert_array_equal(allocating_reference(A, B, splits), want)
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.empty((M, N), dtype=torch.int32, device="cuda")
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        dC.fill_(-7)
        _abi.check(_abi.lib().llm_gemm_i8_splitk_noalloc(0, dA.data_ptr(), dB.data_ptr(), M, N, K, splits,
                                                         dC.data_ptr(), None))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dC.cpu().numpy(), want)


def test_noalloc_rejects_shapes_beyond_the_scratch_array():
    import torch
    dA = torch.zeros((256, 1024), dtype=torch.int8, device="cuda")
    dB = torch.zeros((4096, 1024), dtype=torch.int8, device="cuda")
    dC = torch.zeros((256, 4096), dtype=torch.int32, device="cuda")
    rc = _abi.lib().llm_gemm_i8_splitk_noalloc(0, dA.data_ptr(), dB.data_ptr(), 256, 4096, 1024, 8, dC.data_ptr(), None)
    assert rc == _abi.LLM_ERR_INVALID
    assert "scratch" in _abi.last_error()


def test_noalloc_rejects_misaligned_buffers():
    import torch
    dA = torch.zeros(64 * 256 + 16, dtype=torch.int8, device="cuda")
    dB = torch.zeros((128, 256), dtype=torch.int8, device="cuda")
    dC = torch.zeros((64, 128), dtype=torch.int32, device="cuda")
    rc = _abi.lib().llm_gemm_i8_splitk_noalloc(0, dA.data_ptr() + 8, dB.data_ptr(), 64, 128, 256, 1, dC.data_ptr(), None)
    assert rc == _abi.LLM_ERR_INVALID and "misaligned" in _abi.last_error()
    rc = _abi.lib().llm_gemm_i8_splitk_noalloc(0, dA.data_ptr(), dB.data_ptr(), 64, 128, 256, 1, dC.data_ptr() + 2, None)
    assert rc == _abi.LLM_ERR_INVALID and "misaligned" in _abi.last_error()
