"""Host-side rules of the storiesane mirror (CPU): the decode window (ane/storiesane/
engine_test.go:313-322 TestFillDecodeWindow and its tail/long cases), Open's argument errors,
and the oracle's storiesane arithmetic (residual x + a*branch, a = 1/sqrt(2*layers))."""
import numpy as np
import pytest

import oracle as O
from ane import _abi
from ane.stories import ModelConfig, SyntheticWeights
from ane.storiesane import Open, Options, fillDecodeWindow

TINY = ModelConfig(dim=128, hidden=256, n_layers=2, n_heads=2, n_kv_heads=2, head_dim=64, vocab=500,
                   max_seq=64, qk_norm=False, tied_embed=True, norm_eps=1e-5, rope_theta=10000.0, name="tiny")


def test_fill_decode_window_reference_case():
    got = [0] * 5
    fillDecodeWindow(got, [7, 8])
    assert got == [1, 1, 1, 7, 8]


def test_fill_decode_window_keeps_the_tail():
    got = [0] * 3
    fillDecodeWindow(got, [4, 5, 6, 7, 8])
    assert got == [6, 7, 8]
    got = [9] * 2
    fillDecodeWindow(got, [])
    assert got == [1, 1]


def test_open_requires_a_model():
    with pytest.raises(_abi.LLMError, match="storiesane open: model path is empty"):
        Open(Options())


def test_oracle_storiesane_residual_equals_prescaled_output_projections():
    """x + a*(Wo.att) is algebraically x + (a*Wo).att: the storiesane forward on unscaled
    weights tracks stories.Decoder on weights whose Wo and W2 carry the scale."""
    a = np.float32(1.0 / np.sqrt(2.0 * TINY.n_layers))
    w = SyntheticWeights(TINY, 5, 1.0, stddev=0.05)
    ws = SyntheticWeights(TINY, 5, 1.0, stddev=0.05)
    for L in ws.Layers:
        L.Wo *= a
        L.W2 *= a
    toks = [1, 1, 17, 300, 42, 7]
    sa = O.Model(TINY.oracle_dict(), w, "fp32", storiesane=True).eval_window(toks)
    st = O.Model(TINY.oracle_dict(), ws, "fp32").eval_window(toks)
    assert sa.shape == (TINY.vocab, len(toks))
    assert np.abs(sa - st).max() < 1e-4
    plain = O.Model(TINY.oracle_dict(), w, "fp32").eval_window(toks)
    assert np.abs(sa - plain).max() > 1e-3  # the switch changes the arithmetic
