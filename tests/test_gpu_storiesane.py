"""storiesane on CUDA: EvalLogits of a full window (channel-first [Vocab][seq]) against the
oracle's storiesane arithmetic (ane/storiesane/engine.go:804-842) at the precision the engine
runs -- bit-identical to the oracle in GPU order, within the noise floor of the reference's
order -- and the windowed Decode (decode.go:18-94) against the oracle's window argmax."""
import numpy as np
import pytest

import oracle as O
from ane import _abi
from ane.stories import STORIES_110M, DecodeOptions, SyntheticWeights
from ane.storiesane import Open, Options, fillDecodeWindow
from parity import REF_ORDER_TOL, gpu_order
from test_gpu_decode import TINY_MHA, weights
from test_formats import TINY, write_llama2c

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["fp16", "bf16", "w8a8_fp16"])
def test_eval_logits_matches_oracle(dtype):
    cfg = TINY_MHA
    w = weights(cfg)
    seq = 48
    eng = Open(Options(Weights=w, Seq=seq, DType=dtype))
    rng = np.random.default_rng(6)
    window = [1] * 10 + rng.integers(3, cfg.vocab, seq - 10).tolist()
    got = eng.EvalLogits(window).reshape(cfg.vocab, seq)
    np.testing.assert_array_equal(got, gpu_order(cfg, w, dtype, storiesane=True).eval_window(window))
    want = O.Model(cfg.oracle_dict(), w, dtype, storiesane=True).eval_window(window)
    worst = float(np.abs(got - want).max())
    print(f"storiesane {dtype}: vs reference-order oracle max|dlogit|={worst:.3e}")
    assert worst <= REF_ORDER_TOL[dtype]
    agree = np.mean(got.argmax(0) == want.argmax(0))
    assert agree >= 0.95
    with pytest.raises(_abi.LLMError, match=f"storiesane eval logits: token len=3 want={seq}"):
        eng.EvalLogits([1, 2, 3])
    eng.Close()


def test_eval_logits_stories110m_fp16_vs_reference_fp32():
    cfg = STORIES_110M
    w = SyntheticWeights(cfg, 1234, 1.0)  # storiesane scales the residual branch itself
    seq = 64
    eng = Open(Options(Weights=w, Seq=seq, DType="fp16"))
    rng = np.random.default_rng(1)
    window = [1] + rng.integers(3, cfg.vocab, seq - 1).tolist()
    got = eng.EvalLogits(window).reshape(cfg.vocab, seq)
    eng.Close()
    ref = O.Model(cfg.oracle_dict(), w, "fp32", storiesane=True).eval_window(window)
    worst = float(np.abs(got - ref).max())
    print(f"Stories110M storiesane fp16 vs fp32 reference arithmetic: {worst:.3e}")
    assert worst <= 2e-2


def test_windowed_decode_follows_oracle_argmax_and_reseeds():
    cfg = TINY_MHA
    w = weights(cfg)
    seq = 24
    eng = Open(Options(Weights=w, Seq=seq, DType="fp16"))
    m = gpu_order(cfg, w, "fp16", storiesane=True)
    res = eng.Decode(None, DecodeOptions(MaxNewTokens=40, PromptTokens=[5, 9, 300]))
    assert res.PromptLength == 3
    gen = res.Tokens[3:]
    assert len(gen) == 40 or res.StoppedOnEOS
    ok = 0
    win = [0] * seq
    for j, t in enumerate(gen):
        fillDecodeWindow(win, res.Tokens[:3 + j])  # the window grows past seq and slides
        ok += int(m.eval_window(win)[:, -1].argmax() == t)
    assert ok == len(gen)
    a = eng.Decode(None, DecodeOptions(MaxNewTokens=15, Temperature=1.1, Seed=3, PromptTokens=[5]))
    b = eng.Decode(None, DecodeOptions(MaxNewTokens=15, Temperature=1.1, Seed=3, PromptTokens=[5]))
    c = eng.Decode(None, DecodeOptions(MaxNewTokens=15, Temperature=1.1, Seed=4, PromptTokens=[5]))
    assert a.Tokens == b.Tokens and a.Tokens != c.Tokens
    with pytest.raises(_abi.LLMError, match=r"storiesane decode: prompt token\[0\]=1000 out of range"):
        eng.Decode(None, DecodeOptions(MaxNewTokens=2, PromptTokens=[1000]))
    eng.Close()


def test_open_from_llama2c_file(tmp_path):
    path = tmp_path / "model.bin"
    write_llama2c(path, TINY, np.random.default_rng(2), scale=0.05)
    eng = Open(Options(ModelPath=str(path), Seq=16, Config=TINY, DType="fp16"))
    lg = eng.EvalLogits([1] * 16)
    assert lg.shape == (TINY.vocab * 16,) and np.isfinite(lg).all()
    eng.Close()
    with pytest.raises(_abi.LLMError, match="storiesane open: load model"):
        Open(Options(ModelPath=str(tmp_path / "missing.bin"), Seq=16, Config=TINY))


def test_out_of_range_window_token_is_a_zero_embedding_column():
    """EmbedLookup (ane/stories/cpu.go:41-72): a window token outside [0, vocab) contributes a
    zero embedding column instead of an error; bit-identical to the GPU-order oracle."""
    cfg = TINY_MHA
    w = weights(cfg)
    seq = 16
    eng = Open(Options(Weights=w, Seq=seq, DType="bf16"))
    window = [1, 5, 40000, 7] + [9] * (seq - 4)
    got = eng.EvalLogits(window).reshape(cfg.vocab, seq)
    eng.Close()
    np.testing.assert_array_equal(got, gpu_order(cfg, w, "bf16", storiesane=True).eval_window(window))


def test_diagnostics_report_the_device_forward():
    cfg = TINY_MHA
    eng = Open(Options(Weights=weights(cfg), Seq=8, DType="fp16", UseANE=True))
    d = eng.Diagnostics()
    assert d.UseANE and d.LayerForwardRequested and d.LayerForwardEnabled
    assert d.CompiledLayers == cfg.n_layers and d.HasClassifierForward and not d.HybridBackwardEnabled
    eng.Close()
    assert eng.Diagnostics().CompiledLayers == 0
