"""Temperature sampling on the device (ane/stories/infer.go:347-371).

The sampler given the same logits and uniform must pick the oracle's index; the token loop
must draw, per sequence slot, the documented uniforms in order (prefill draw 0, then one per
step), through host-driven steps and the device-resident generate loop; the Decoder mirror
reseeds on a non-zero DecodeOptions.Seed as Decode does (infer.go:150-152)."""
import numpy as np
import pytest

import oracle as O
from ane import _abi
from ane.stories import DecodeOptions, Engine, NewDecoder, SyntheticWeights
from test_gpu_decode import TINY_GQA, TINY_MHA, weights

pytestmark = pytest.mark.gpu


def device_sample(logits, temperature, u):
    logits = np.ascontiguousarray(logits, np.float32)
    u = np.ascontiguousarray(u, np.float64)
    out = np.zeros(logits.shape[0], np.int32)
    _abi.check(_abi.lib().llm_debug_sample(0, logits.ctypes.data, logits.shape[0], logits.shape[1], temperature,
                                           u.ctypes.data, out.ctypes.data))
    return out


@pytest.mark.parametrize("vocab", [7, 1000, 32000, 151936])
@pytest.mark.parametrize("temperature", [0.05, 0.7, 1.0, 2.5])
def test_device_sampler_matches_oracle(vocab, temperature):
    rng = np.random.default_rng(vocab + int(temperature * 100))
    rows = 24
    logits = (rng.standard_normal((rows, vocab)) * rng.uniform(0.5, 6.0, (rows, 1))).astype(np.float32)
    u = rng.random(rows)
    u[0], u[1] = 0.0, np.nextafter(1.0, 0.0)
    got = device_sample(logits, temperature, u)
    want = [O.sample_from_logits(logits[i], temperature, u[i]) for i in range(rows)]
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("cfg,dtype", [(TINY_MHA, "fp16"), (TINY_GQA, "w8a8_bf16")], ids=["mha-fp16", "gqa-w8a8"])
def test_token_loop_draws_documented_uniforms(cfg, dtype):
    w = weights(cfg)
    T, seed = 0.9, 4242
    eng = Engine(cfg, dtype).load(w)
    eng.kv_alloc(4, 96)
    eng.set_sampling(T, seed, True)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(3, cfg.vocab, L).tolist() for L in (3, 17, 30)]
    slots = [0, 1, 2]
    nxt, lg = eng.prefill(slots, prompts, want_logits=True)
    toks = [[int(t)] for t in nxt]
    logits = [[lg[i]] for i in range(3)]
    cur, pos = nxt.copy(), np.array([len(p) for p in prompts], np.int32)
    for _ in range(12):
        nxt, lg = eng.decode_step(slots, cur, pos, want_logits=True)
        for i in range(3):
            toks[i].append(int(nxt[i]))
            logits[i].append(lg[i])
        cur, pos = nxt, pos + 1
    greedy = 0
    for i, s in enumerate(slots):
        for k, (t, row) in enumerate(zip(toks[i], logits[i])):
            assert t == O.sample_from_logits(row, T, O.uniform(seed, s, k)), (i, k)
            greedy += int(t == int(np.argmax(row)))
    assert greedy < 3 * 13  # at T = 0.9 some draws leave the argmax
    # the device-resident loop draws the same sequence after a reseed
    eng.set_sampling(T, seed, True)
    for s in slots:
        eng.release(s)
    first = eng.prefill(slots, prompts)
    assert [int(x) for x in first] == [t[0] for t in toks]
    gen = eng.generate(slots, first, [len(p) for p in prompts], 12)
    np.testing.assert_array_equal(gen.T, np.array([t[1:] for t in toks]))
    eng.close()


def test_decoder_sampling_reseed_and_greedy_default():
    cfg = TINY_MHA.with_max_seq(64)
    w = SyntheticWeights(cfg, 91, 1.0, stddev=0.05)
    w.Config = cfg
    dec = NewDecoder(w, 60, 7, dtype="fp16")
    a = dec.Decode(None, DecodeOptions(MaxNewTokens=30, Temperature=1.2, Seed=99, PromptTokens=[5, 6]))
    b = dec.Decode(None, DecodeOptions(MaxNewTokens=30, Temperature=1.2, Seed=99, PromptTokens=[5, 6]))
    assert a.Tokens == b.Tokens  # a non-zero Seed reseeds (infer.go:150-152)
    c = dec.Decode(None, DecodeOptions(MaxNewTokens=30, Temperature=1.2, PromptTokens=[5, 6]))
    assert c.Tokens != a.Tokens  # Seed 0 continues the decoder's generator
    g1 = dec.Decode(None, DecodeOptions(MaxNewTokens=20, PromptTokens=[5, 6]))
    g2 = dec.Decode(None, DecodeOptions(MaxNewTokens=20, Temperature=-1.0, PromptTokens=[5, 6]))
    assert g1.Tokens == g2.Tokens  # temperature <= 0 is greedy
    m = O.Model(cfg.oracle_dict(), w, "fp16", gpu_order=True)
    am = m.seq().teacher_forced(g1.Tokens, n_prefill=g1.PromptLength)
    gen = g1.Tokens[g1.PromptLength:]
    assert [int(am[g1.PromptLength - 1 + j]) for j in range(len(gen))] == gen
    dec.Close()
