"""CPU tests of the oracle (the checker): known answers from the reference's arithmetic and
an independent pure-Python restatement of ane/stories/infer.go that must agree bit for bit
with the C restatement.

Reference pins used (tmc/ane-training-experiments):
  infer.go:373-383 argmax first-maximum rule; infer.go:301-311 rmsNormVec; infer.go:97-107
  RoPE tables; infer.go:328-345 softmaxPrefix; infer.go:324-326 silu;
  bridge/ane_bridge.m:374-398 quantiser; infer.go:136-202 Decode control flow.
"""
import math

import numpy as np
import pytest

import oracle as O
from ane.stories import LayerWeights, ModelWeights, ModelConfig

f32 = np.float32


# ---------------------------------------------------------------- pure-Python restatement
def py_rms(x, w, eps):
    s = 0.0
    for v in x:
        s += float(v) * float(v)
    rr = f32(1.0 / math.sqrt(s / len(x) + eps))
    return np.array([f32(f32(x[i] * rr) * w[i]) for i in range(len(x))], dtype=np.float32)


def py_matvec(mat, vec):
    out = np.zeros(mat.shape[0], np.float32)
    for r in range(mat.shape[0]):
        s = f32(0)
        for c in range(mat.shape[1]):
            s = f32(s + f32(mat[r, c] * vec[c]))
        out[r] = s
    return out


def py_silu(x):
    return f32(x / f32(f32(1) + f32(math.exp(-float(x)))))


def py_softmax(src):
    mx = src[0]
    for v in src[1:]:
        if v > mx:
            mx = v
    s = 0.0
    e = []
    for v in src:
        ev = f32(math.exp(float(f32(v - mx))))
        e.append(ev)
        s += float(ev)
    inv = f32(1.0 / s)
    return [f32(v * inv) for v in e]


def py_forward(cfg, w, kc, vc, cos, sin, token, pos):
    D, hd, H, KVH = cfg.dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    grp = H // KVH
    x = w.Embed[token].astype(np.float32).copy()
    for l, L in enumerate(w.Layers):
        xn = py_rms(x, L.RMSAtt, cfg.norm_eps)
        q, k, v = py_matvec(L.Wq, xn), py_matvec(L.Wk, xn), py_matvec(L.Wv, xn)
        if cfg.qk_norm:
            for h in range(H):
                q[h * hd:(h + 1) * hd] = py_rms(q[h * hd:(h + 1) * hd], L.QNorm, cfg.norm_eps)
            for h in range(KVH):
                k[h * hd:(h + 1) * hd] = py_rms(k[h * hd:(h + 1) * hd], L.KNorm, cfg.norm_eps)
        for vec, nh in ((q, H), (k, KVH)):
            for h in range(nh):
                for i in range(hd // 2):
                    c, s = cos[pos, i], sin[pos, i]
                    a0, a1 = vec[h * hd + 2 * i], vec[h * hd + 2 * i + 1]
                    vec[h * hd + 2 * i] = f32(f32(a0 * c) - f32(a1 * s))
                    vec[h * hd + 2 * i + 1] = f32(f32(a0 * s) + f32(a1 * c))
        kc[l][pos] = k
        vc[l][pos] = v
        inv = f32(1.0 / math.sqrt(hd))
        att = np.zeros(H * hd, np.float32)
        for h in range(H):
            kh = h // grp
            sc = []
            for t in range(pos + 1):
                d = f32(0)
                for i in range(hd):
                    d = f32(d + f32(q[h * hd + i] * kc[l][t][kh * hd + i]))
                sc.append(f32(d * inv))
            pr = py_softmax(sc)
            for i in range(hd):
                s = f32(0)
                for t in range(pos + 1):
                    s = f32(s + f32(pr[t] * vc[l][t][kh * hd + i]))
                att[h * hd + i] = s
        x2 = py_matvec(L.Wo, att)
        x2 = (x2 + x).astype(np.float32)
        xn = py_rms(x2, L.RMSFFN, cfg.norm_eps)
        h1, h3 = py_matvec(L.W1, xn), py_matvec(L.W3, xn)
        g = np.array([f32(py_silu(h1[i]) * h3[i]) for i in range(len(h1))], np.float32)
        x = (x2 + py_matvec(L.W2, g)).astype(np.float32)
    xn = py_rms(x, w.RMSFinal, cfg.norm_eps)
    return py_matvec(w.Embed, xn)


def tiny_cfg(qk_norm):
    return ModelConfig(dim=16, hidden=24, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=4, vocab=40, max_seq=12,
                       qk_norm=qk_norm, tied_embed=True, norm_eps=1e-6 if qk_norm else 1e-5,
                       rope_theta=1e6 if qk_norm else 10000.0, name="tiny")


def tiny_weights(cfg, seed):
    rng = np.random.default_rng(seed)
    D, F, Q, KV, hd = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.head_dim
    n = lambda *s: (rng.standard_normal(s) * 0.3).astype(np.float32)  # noqa: E731
    layers = [LayerWeights(n(Q, D), n(KV, D), n(KV, D), n(D, Q), n(F, D), n(D, F), n(F, D),
                           (1 + 0.1 * rng.standard_normal(D)).astype(np.float32),
                           (1 + 0.1 * rng.standard_normal(D)).astype(np.float32),
                           (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if cfg.qk_norm else None,
                           (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if cfg.qk_norm else None)
              for _ in range(cfg.n_layers)]
    return ModelWeights(layers, (1 + 0.1 * rng.standard_normal(D)).astype(np.float32), n(cfg.vocab, D), True, None, cfg)


@pytest.mark.parametrize("qk_norm", [False, True])
def test_c_oracle_matches_python_restatement_bitwise(qk_norm):
    cfg = tiny_cfg(qk_norm)
    w = tiny_weights(cfg, 7)
    m = O.Model(cfg.oracle_dict(), w, "fp32")
    s = m.seq()
    cos, sin = O.rope_tables(cfg.max_seq, cfg.head_dim, cfg.rope_theta)
    kc = [[None] * cfg.max_seq for _ in range(cfg.n_layers)]
    vc = [[None] * cfg.max_seq for _ in range(cfg.n_layers)]
    for pos, tok in enumerate([1, 17, 3, 39, 0, 22]):
        got = s.forward(tok, pos)
        want = py_forward(cfg, w, kc, vc, cos, sin, tok, pos)
        np.testing.assert_array_equal(got, want)


# ---------------------------------------------------------------- known answers
def test_argmax_first_maximum_wins():
    v = O.f32([0.5, 3.0, -1.0, 3.0, 2.0])
    assert O.lib().oracle_argmax(v.ctypes.data_as(O._FP), len(v)) == 1


def test_rmsnorm_known_answer():
    x, w = O.f32([1, 2, 3, 4]), O.f32([1, 0.5, 2, 1])
    rr = f32(1.0 / math.sqrt(30.0 / 4 + 1e-5))
    want = np.array([f32(f32(x[i] * rr) * w[i]) for i in range(4)], np.float32)
    np.testing.assert_array_equal(O.rmsnorm(x, w, 1e-5), want)


def test_rope_tables_known_answer():
    c, s = O.rope_tables(3, 4, 10000.0)
    assert c[0].tolist() == [1.0, 1.0] and s[0].tolist() == [0.0, 0.0]
    assert c[1, 0] == f32(math.cos(1.0)) and s[1, 0] == f32(math.sin(1.0))
    assert c[2, 1] == f32(math.cos(2.0 / 100.0)) and s[2, 1] == f32(math.sin(2.0 / 100.0))


def test_softmax_prefix_uniform_and_known():
    np.testing.assert_array_equal(O.softmax_prefix([2.0, 2.0, 2.0, 2.0]), O.f32([0.25] * 4))
    x = [0.0, 1.0, -2.0]
    np.testing.assert_array_equal(O.softmax_prefix(x), O.f32(py_softmax(O.f32(x))))


def test_silu_known_answer():
    for x in (-3.0, -0.5, 0.0, 0.75, 4.0):
        assert O.lib().oracle_silu(x) == py_silu(f32(x))


def test_quantiser_bridge_rule():
    # all-zero row: scale 0 -> 1 (bridge/ane_bridge.m:384)
    q, s = O.quant_rows(np.zeros((1, 8), np.float32))
    assert s[0] == 1.0 and not q.any()
    # maxabs/127 scale, half-away rounding of x/scale, f32 `v + 0.5` then truncation
    x = O.f32([[127.0, -63.5, 0.5, -0.5, 1.49, -126.6, 0.0, 64.5]])
    q, s = O.quant_rows(x)
    assert s[0] == f32(127.0) / f32(127.0)
    assert q[0].tolist() == [127, -64, 1, -1, 1, -127, 0, 65]
    # the f32 addition can round up: v = 0.49999997 -> v + 0.5 == 1.0 in f32 -> 1
    row = O.f32([[127.0, 0.49999997]])
    q, s = O.quant_rows(row)
    assert q[0, 1] == 1


def test_quantiser_random_rows_match_numpy_restatement():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((17, 96)) * rng.uniform(0.01, 10, (17, 1))).astype(np.float32)
    q, s = O.quant_rows(x)
    mx = np.abs(x).max(axis=1).astype(np.float32)
    sc = (mx / f32(127)).astype(np.float32)
    sc[sc == 0] = 1
    v = (x / sc[:, None]).astype(np.float32)
    v = np.clip(v, -128, 127).astype(np.float32)
    r = (v + np.where(v >= 0, f32(0.5), f32(-0.5))).astype(np.float32)
    np.testing.assert_array_equal(s, sc)
    np.testing.assert_array_equal(q, np.trunc(r).astype(np.int8))


def test_norm_quant_lane_order_matches_numpy():
    rng = np.random.default_rng(5)
    for cols in (128, 256, 768, 1024, 3072):
        x = rng.standard_normal((3, cols)).astype(np.float32)
        w = (1 + 0.2 * rng.standard_normal(cols)).astype(np.float32)
        q, s = O.norm_quant_rows(x, w, 1e-5)
        G = 2 if cols >= 512 else 1
        T = cols // (4 * G)
        for r in range(3):
            total = None
            for wp in range((T + 31) // 32):
                parts = np.zeros(32)
                for l in range(32):
                    t = 32 * wp + l
                    acc = 0.0
                    if t < T:
                        for j in range(G):
                            for c in range(4):
                                e = 4 * t + 4 * T * j + c
                                acc = acc + float(x[r, e]) * float(x[r, e])
                    parts[l] = acc
                for k in (16, 8, 4, 2, 1):
                    parts = np.array([parts[i] + parts[i ^ k] for i in range(32)])
                total = parts[0] if total is None else total + parts[0]
            rr = f32(1.0 / math.sqrt(total / cols + 1e-5))
            y = ((x[r] * rr).astype(np.float32) * w).astype(np.float32)
            qq, ss = O.quant_rows(y[None, :])
            np.testing.assert_array_equal(q[r], qq[0])
            assert s[r] == ss[0]


def test_gemm_i8_exact():
    rng = np.random.default_rng(11)
    A = rng.integers(-128, 128, (9, 256), dtype=np.int8)
    B = rng.integers(-128, 128, (13, 256), dtype=np.int8)
    np.testing.assert_array_equal(O.gemm_i8(A, B), (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32))


def test_rounding_helpers():
    assert O.round_bf16(1.0 + 2 ** -8) == 1.0          # tie -> even
    assert O.round_bf16(1.0 + 3 * 2 ** -9) == 1.0 + 2 ** -7
    assert O.round_f16(1.0 + 2 ** -11) == 1.0          # tie -> even
    assert O.round_f16(65520.0) == float("inf")


# ---------------------------------------------------------------- Decode control flow (infer.go:136-202)
def test_decode_rules_bos_default_and_max_seq_stop():
    cfg = tiny_cfg(False)
    w = tiny_weights(cfg, 9)
    m = O.Model(cfg.oracle_dict(), w, "fp32")
    s = m.seq()
    toks, plen, eos = s.decode([], 100)
    assert toks[0] == 1 and plen == 1                   # empty prompt -> [BOS]
    if not eos:
        assert len(toks) == cfg.max_seq                  # stops at maxSeq
    # prompt longer than maxSeq keeps its last maxSeq tokens; no room -> no generation
    long = list(range(3, 3 + cfg.max_seq + 4))
    long = [t % cfg.vocab for t in long]
    toks, plen, eos = s.decode(long, 5)
    assert plen == cfg.max_seq and toks == long[-cfg.max_seq:]


def test_decode_matches_teacher_forced_argmax():
    cfg = tiny_cfg(True)
    w = tiny_weights(cfg, 4)
    m = O.Model(cfg.oracle_dict(), w, "bf16")
    s = m.seq()
    toks, plen, eos = s.decode([5, 6, 7], 6)
    am = s.teacher_forced(toks)
    # every generated token is the argmax after its predecessor (EOS stops the loop)
    for i in range(plen, len(toks)):
        assert toks[i] == am[i - 1]
    if eos:
        assert toks[-1] == 2


def test_forward_range_errors():
    cfg = tiny_cfg(False)
    m = O.Model(cfg.oracle_dict(), tiny_weights(cfg, 1), "fp32")
    s = m.seq()
    with pytest.raises(ValueError, match="token out of range: 40"):
        s.forward(40, 0)
    with pytest.raises(ValueError, match="position out of range: 12"):
        s.forward(1, 12)


@pytest.mark.parametrize("mode", ["fp16", "bf16", "w8a8_fp16", "w8a8_bf16"])
def test_emulation_modes_stay_close_to_fp32(mode):
    cfg = tiny_cfg(True)
    w = tiny_weights(cfg, 21)
    ref = O.Model(cfg.oracle_dict(), w, "fp32").seq()
    emu = O.Model(cfg.oracle_dict(), w, mode).seq()
    toks = [1, 9, 4, 33, 2, 17, 8]
    _, lr = ref.teacher_forced(toks, want_logits=True)
    _, le = emu.teacher_forced(toks, want_logits=True)
    tol = {"fp16": 0.05, "bf16": 0.3, "w8a8_fp16": 0.5, "w8a8_bf16": 0.6}[mode]
    assert np.abs(lr - le).max() < tol


# ---------------------------------------------------------------- sensitivity of the precision modes
@pytest.mark.parametrize("mode,lo,hi", [("w8a8_fp16", 0.03, 0.1), ("bf16", 0.0, 0.02)])
def test_w8a8_order_sensitivity(mode, lo, hi):
    """How far the oracle moves when only the attention PV summation order is reversed, on
    Stories110M with the benchmark's synthetic weights.  W8A8 moves by more than 3e-2 (so
    the spec's 5e-2 logit tolerance is not reachable by a non-bit-identical implementation;
    the GPU tests use 1e-1), bf16 stays inside the spec's 2e-2."""
    from ane.stories import STORIES_110M, SyntheticWeights
    cfg = STORIES_110M.with_max_seq(64)
    w = SyntheticWeights(cfg, 1234, 24 ** -0.5)
    toks = np.random.default_rng(5).integers(3, cfg.vocab, 40).tolist()
    m = O.Model(cfg.oracle_dict(), w, mode)
    _, a = m.seq().teacher_forced(toks, want_logits=True)
    O.set_attn_reverse(True)
    try:
        _, b = m.seq().teacher_forced(toks, want_logits=True)
    finally:
        O.set_attn_reverse(False)
    d = float(np.abs(a - b).max())
    agree = float(np.mean(a.argmax(1) == b.argmax(1)))
    print(f"{mode}: oracle vs oracle with reversed PV order: max |dlogit| = {d:.4f}, top-1 agreement {agree:.3f}")
    assert lo <= d < hi
    if mode.startswith("w8a8"):
        assert agree >= 0.9


def test_bf16_qwen3_order_sensitivity():
    """The oracle against itself on Qwen3-0.6B bf16 (the benchmark's synthetic weights) when
    its f32 attention-PV and matVec sums are taken in reverse order: the logits move by
    0.019-0.024, i.e. the spec's 2e-2 bf16 tolerance is the checker's own noise floor on this
    model; the GPU parity tests use 3e-2 for bf16."""
    from ane.stories import QWEN3_0_6B, SyntheticWeights
    cfg = QWEN3_0_6B.with_max_seq(64)
    w = SyntheticWeights(cfg, 7, 1.0)
    rng = np.random.default_rng(8)
    toks = rng.integers(3, cfg.vocab, 48).tolist()
    m = O.Model(cfg.oracle_dict(), w, "bf16")
    _, a = m.seq().teacher_forced(toks, want_logits=True)
    O.set_attn_reverse(True)
    O.set_matvec_reverse(True)
    try:
        _, b = m.seq().teacher_forced(toks, want_logits=True)
    finally:
        O.set_attn_reverse(False)
        O.set_matvec_reverse(False)
    d = float(np.abs(a - b).max())
    print(f"qwen3 bf16: oracle vs oracle with reversed sums: max |dlogit| = {d:.4f}")
    assert 0.012 <= d < 0.03


def _splitmix64(x):
    m = (1 << 64) - 1
    x = (x + 0x9E3779B97F4A7C15) & m
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
    return x ^ (x >> 31)


def _uniform_py(seed, stream, counter):
    m = (1 << 64) - 1
    key = _splitmix64(seed ^ _splitmix64((stream * 0xD1B54A32D192ED03 + 0x8CB92BA72F3D8DD7) & m))
    return (_splitmix64((key + counter) & m) >> 11) * (1.0 / 9007199254740992.0)


def _sample_py(logits, temperature, u):
    """ane/stories/infer.go:347-371 restated in plain Python (float64 sums, f32 1/T)."""
    import math
    lg = [float(np.float32(v)) for v in logits]
    if temperature <= 1e-6:
        return int(np.argmax(np.asarray(logits, np.float32)))
    mx = lg[0]
    for v in lg[1:]:
        if v > mx:
            mx = v
    inv_t = float(np.float32(1.0) / np.float32(temperature))
    total = 0.0
    for v in lg:
        total += math.exp((v - mx) * inv_t)
    target = u * total
    acc = 0.0
    for i, v in enumerate(lg):
        acc += math.exp((v - mx) * inv_t)
        if acc >= target:
            return i
    return len(lg) - 1


def test_sampling_uniform_matches_restatement_and_library():
    from ane import _abi
    for seed, slot, ctr in [(0, 0, 0), (1234, 5, 17), (2**63 + 11, 255, 2**40), (7, 4095, 3)]:
        want = _uniform_py(seed, O.SAMPLE_STREAM_BASE + slot, ctr)
        assert O.uniform(seed, slot, ctr) == want
        assert _abi.lib().llm_sample_uniform(seed, slot, ctr) == want
        assert 0.0 <= want < 1.0


def test_sample_from_logits_known_answers_and_restatement():
    # two tokens with weights 1/3 and 1 at T=1 (total 4/3): u <= 1/4 -> 0, else 1
    lg = np.array([0.0, np.log(3.0)], np.float32)
    assert O.sample_from_logits(lg, 1.0, 0.2) == 0
    assert O.sample_from_logits(lg, 1.0, 0.3) == 1
    assert O.sample_from_logits(lg, 1e-7, 0.0) == 1          # greedy branch
    assert O.sample_from_logits(np.zeros(5, np.float32), 0.5, 0.0) == 0
    assert O.sample_from_logits(np.zeros(5, np.float32), 0.5, 0.999999) == 4
    rng = np.random.default_rng(3)
    for _ in range(50):
        n = int(rng.integers(1, 300))
        lg = (rng.standard_normal(n) * rng.uniform(0.1, 8)).astype(np.float32)
        t = float(rng.choice([0.0, 0.3, 0.8, 1.0, 1.7]))
        u = float(rng.random())
        assert O.sample_from_logits(lg, t, u) == _sample_py(lg, t, u)


def test_oracle_weight_generator_equals_the_library():
    """The CPU legs of bench.py build the synthetic model with the oracle's restatement of the
    generator (so they load no product code): bit-identical to llm_synth_normal."""
    from ane.stories import QWEN3_0_6B, ModelConfig, SyntheticWeights
    cfg = ModelConfig(dim=64, hidden=96, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, vocab=333, max_seq=32,
                      qk_norm=True, tied_embed=False, name="gen")
    a = SyntheticWeights(cfg, 99, 0.25, stddev=0.05)
    b = O.SynthWeights(dict(cfg.oracle_dict(), tied_embed=0), 99, 0.25, stddev=0.05)
    pairs = [(a.Embed, b.Embed), (a.LMHead, b.LMHead)]
    for la, lb in zip(a.Layers, b.Layers):
        pairs += [(getattr(la, k), getattr(lb, k)) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")]
    for x, y in pairs:
        assert x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))
    q = O.PRESETS["qwen3-0.6b"]
    assert (q["dim"], q["hidden"], q["n_layers"], q["n_heads"], q["n_kv_heads"], q["head_dim"], q["vocab"]) == (
        QWEN3_0_6B.dim, QWEN3_0_6B.hidden, QWEN3_0_6B.n_layers, QWEN3_0_6B.n_heads, QWEN3_0_6B.n_kv_heads,
        QWEN3_0_6B.head_dim, QWEN3_0_6B.vocab)


def test_exp2_det_known_values_and_accuracy():
    assert O.exp2_det(0.0) == 1.0 and O.exp2_det(1.0) == 2.0 and O.exp2_det(-1.0) == 0.5
    assert O.exp2_det(-126.0) == 2.0 ** -126 and O.exp2_det(-127.0) == 0.0 and O.exp2_det(float("-inf")) == 0.0
    assert O.exp2_det(-300.0) == 0.0 and 0.0 < O.exp2_det(-126.4) < 2.0 ** -126   # a rounded subnormal
    assert O.exp2_det(127.5) == O.exp2_det(1e30) and abs(O.exp2_det(127.5) / 2.0 ** 127.49999 - 1) < 1e-5
    xs = np.random.default_rng(4).uniform(-100, 100, 20000).astype(np.float32)
    got = np.array([O.exp2_det(float(x)) for x in xs], np.float64)
    ref = np.exp2(xs.astype(np.float64))
    assert (np.abs(got - ref) / ref).max() < 2.5e-7


def test_mma_model_known_cases():
    """The tensor-core step's rules on hand-made cases: exact products, a 26-bit window below
    the largest alignment exponent with truncation toward zero, the sum rounded toward zero."""
    one = np.zeros(16, np.float32)
    a = one.copy(); b = one.copy()
    a[0], b[0] = 1.0, 1.0
    a[1], b[1] = 3 * 2.0 ** -13, 2.0 ** -12       # 0.75 ulp of 1.0
    assert O.mma16(0.0, a, b, 2) == 1.0            # rounded toward zero (nearest would give 1 + 2^-23)
    a[1], b[1] = -(2.0 ** -13), 2.0 ** -12         # 1 - 2^-25: exact sum just below 1
    assert O.mma16(0.0, a, b, 2) == np.float32(1 - 2.0 ** -24)
    a[1], b[1] = -(2.0 ** -20), 2.0 ** -10         # -2^-30: below the window of the product 1*1 -> dropped
    assert O.mma16(0.0, a, b, 2) == 1.0
    # the accumulator's alignment exponent is e(c) + 1
    assert O.mma16(1.0, np.zeros(16, np.float32), np.zeros(16, np.float32), 2) == 1.0
    c = np.float32(1.0 + 2.0 ** -23)
    a = one.copy(); b = one.copy(); a[0], b[0] = 2.0 ** -24, 1.0
    assert O.mma16(float(c), a, b, 2) == c         # adds less than an ulp: truncated
