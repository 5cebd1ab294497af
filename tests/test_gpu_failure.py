"""Failure detection on the GPU without a fault: a kernel whose wait nothing completes gives up
after a bounded number of polls, records the timeout in its error word, and the host turns it
into LLM_ERR_DEVICE ("bounded wait expired"); the device stays usable afterwards.  Every
mbarrier wait of the token loop's kernels takes this path on expiry."""
import ctypes as C

import numpy as np
import pytest

from ane import _abi
from ane.stories import Engine
from test_gpu_decode import TINY_MHA, weights

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_into_an_error_status():
    rc = _abi.lib().llm_debug_wait_timeout(0, 1000)
    assert rc == _abi.LLM_ERR_DEVICE
    assert "bounded wait expired" in _abi.last_error()
    # the context is still usable: an int8 GEMM on the same device is exact
    rng = np.random.default_rng(0)
    A = rng.integers(-128, 128, (16, 128), dtype=np.int8)
    B = rng.integers(-128, 128, (32, 128), dtype=np.int8)
    out = np.zeros((16, 32), np.int32)
    _abi.check(_abi.lib().llm_debug_gemm_i8(0, _abi.ptr(A, C.c_int8), _abi.ptr(B, C.c_int8), 16, 32, 128, 1,
                                            _abi.ptr(out, C.c_int32)))
    np.testing.assert_array_equal(out, A.astype(np.int64) @ B.astype(np.int64).T)


def test_engine_still_decodes_after_an_expired_wait():
    assert _abi.lib().llm_debug_wait_timeout(0, 10) == _abi.LLM_ERR_DEVICE
    eng = Engine(TINY_MHA, "fp16").load(weights(TINY_MHA))
    eng.kv_alloc(2, 32)
    nxt = eng.prefill([0], [[5, 6, 7]])
    assert 0 <= int(nxt[0]) < TINY_MHA.vocab
    eng.close()
