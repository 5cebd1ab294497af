"""Host-side mirrors of reference unit tests near the token loop (no GPU):
ane/forward/conv_test.go:5-20 TestChannelFirstRoundTrip and ane/stories/cpu_test.go:56-74
TestEmbedLookupOutOfRangeTokenZeroesColumn (against the oracle's EmbedLookup restatement), plus
the ConvEval argument checks with the reference's error texts."""
import numpy as np
import pytest

import oracle as O
from ane.forward import ConvEval, FromChannelFirst, ToChannelFirst


def test_channel_first_round_trip():
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    cf = ToChannelFirst(x, 2, 3)
    np.testing.assert_array_equal(cf, [1, 4, 2, 5, 3, 6])
    np.testing.assert_array_equal(FromChannelFirst(cf, 2, 3), x)
    with pytest.raises(ValueError, match="ToChannelFirst input len=5 want=6"):
        ToChannelFirst(x[:5], 2, 3)
    with pytest.raises(ValueError, match="FromChannelFirst input len=5 want=6"):
        FromChannelFirst(x[:5], 2, 3)


def test_embed_lookup_out_of_range_token_zeroes_column():
    dim, seq = 3, 2
    embed = np.array([1, 2, 3, 4, 5, 6], np.float32)  # vocab 2
    out = O.embed_lookup_cf(embed, [1, 5], dim, seq)   # token 5 is out of range
    for d in range(dim):
        assert out[d * seq + 0] == embed[dim + d]
        assert out[d * seq + 1] == 0


def test_conv_eval_rejects_bad_input_length():
    with pytest.raises(ValueError, match="ConvEval input len=5 want=6"):
        ConvEval(None, np.zeros(5, np.float32), 2, 3, 4)
