"""Linear (1x1 convolution) kernels through the C ABI (llm_linear_*) and the reference-shaped
Python API (ane.model.Compile / Kernel, ane.forward.ConvEval: ane/model/model_darwin.go:138-414,
ane/forward/conv.go:11-48): bit-identical to the oracle's restatement of the GEMM arithmetic."""
import numpy as np
import pytest

import oracle as O
from ane.forward import ConvEval, ConvEvalWithStats
from ane.model import Compile, CompileOptions

pytestmark = pytest.mark.gpu


def _round(a, act):
    r = O.round_f16 if act == 1 else O.round_bf16
    return np.vectorize(r, otypes=[np.float32])(a.astype(np.float32))


@pytest.mark.parametrize("dtype", ["fp16", "bf16", "w8a8_fp16", "w8a8_bf16"])
@pytest.mark.parametrize("out_dim,in_dim,s", [(384, 768, 37), (2048, 768, 130), (768, 2048, 5)])
def test_conv_eval_matches_oracle(dtype, out_dim, in_dim, s):
    rng = np.random.default_rng(out_dim + in_dim + s)
    W = (rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float32)
    x = rng.standard_normal(s * in_dim).astype(np.float32)  # row-major tokens [s, in_dim]
    k = Compile(CompileOptions(Weights=W, SeqLen=s, DType=dtype))
    y, st = ConvEvalWithStats(k, x, s, in_dim, out_dim)
    k.Close()
    assert st.HWExecutionNS > 0
    xt = x.reshape(s, in_dim)
    if dtype.startswith("w8a8"):
        qx, sx = O.quant_rows(xt)
        qw, sw = O.quant_rows(W)
        acc = O.gemm_i8(qx, qw).astype(np.float32)
        want = (acc * sx[:, None]).astype(np.float32) * sw[None, :]
    else:
        act = 1 if dtype == "fp16" else 2
        want = O.gemm_mma(_round(xt, act), _round(W, act), act)
    np.testing.assert_array_equal(y.reshape(s, out_dim), want.astype(np.float32))


def test_kernel_io_errors():
    W = np.zeros((16, 128), np.float32)
    k = Compile(CompileOptions(Weights=W, SeqLen=4, DType="bf16"))
    assert k.InputBytes(0) == 128 * 4 * 4 and k.OutputBytes(0) == 16 * 4 * 4 and k.NumInputs() == 1
    with pytest.raises(ValueError, match="write input f32: got 3 values, want 512"):
        k.WriteInputF32(0, np.zeros(3, np.float32))
    with pytest.raises(ValueError, match="read output f32: index 1 out of range"):
        k.ReadOutputF32(1, np.zeros(64, np.float32))
    np.testing.assert_array_equal(ConvEval(k, np.ones(4 * 128, np.float32), 4, 128, 16), np.zeros(64, np.float32))
    k.Close()
    with pytest.raises(ValueError, match="write input f32: kernel is closed"):
        k.WriteInputF32(0, np.zeros(512, np.float32))
