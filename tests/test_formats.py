"""File formats on the token loop's host side, checked on CPU against writers that follow the
reference's byte layouts: the llama2.c tokenizer.bin (ane/stories/tokenizer.go:16-101) and its
Decode rules, the llama2.c weight file (ane/stories/weights.go:49-122)."""
import struct

import numpy as np
import pytest

from ane.stories import LoadPretrained, LoadTokenizer, ModelConfig, Tokenizer

TINY = ModelConfig(dim=128, hidden=256, n_layers=2, n_heads=2, n_kv_heads=2, head_dim=64, vocab=300,
                   max_seq=64, qk_norm=False, tied_embed=True, norm_eps=1e-5, rope_theta=10000.0, name="tiny")


def write_tokenizer(path, pieces, max_len=None):
    max_len = max_len or max(1, max(len(p) for p in pieces))
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max_len))
        for i, p in enumerate(pieces):
            f.write(struct.pack("<f", -float(i)))
            f.write(struct.pack("<i", len(p)))
            f.write(p)


def synthetic_pieces(n):
    pieces = [b"<unk>", b"<s>", b"</s>"]
    pieces += [b"<0x%02X>" % i for i in range(256)]
    words = [b" once", b" upon", b" a", b" time", "été".encode(), b"<0x1G>", b"<0x41x>", b"<0x4a>"]
    while len(pieces) < n:
        pieces.append(words[len(pieces) % len(words)] + b"%d" % len(pieces))
    pieces[259:259 + len(words)] = words
    return pieces[:n]


def test_tokenizer_roundtrip_and_decode_rules(tmp_path):
    pieces = synthetic_pieces(300)
    path = tmp_path / "tokenizer.bin"
    write_tokenizer(path, pieces)
    tok = LoadTokenizer(str(path), vocab_size=300)
    assert tok.vocab == pieces
    # <0xHH> pieces decode to the single byte (upper and lower case hex), anything else verbatim
    assert tok.DecodeBytes(3 + 0x41) == b"A"
    assert tok.DecodeBytes(3 + 0xC3) == b"\xc3"
    assert tok.DecodeBytes(259 + 7) == b"J"          # "<0x4a>"
    assert tok.DecodeBytes(259 + 5) == b"<0x1G>"     # not a hex digit
    assert tok.DecodeBytes(259 + 6) == b"<0x41x>"    # wrong length
    assert tok.DecodeBytes(259 + 4) == "été".encode()
    # out of range ids decode to ""
    assert tok.DecodeBytes(-1) == b"" and tok.DecodeBytes(300) == b""
    # a raw byte survives the str view
    assert tok.Decode(3 + 0xC3).encode("utf-8", "surrogateescape") == b"\xc3"
    # two single-byte pieces concatenate into one UTF-8 character, as Go's string concatenation
    text = b"".join(tok.DecodeBytes(i) for i in (3 + 0xC3, 3 + 0xA9)).decode("utf-8", "surrogateescape")
    assert text == "é"


@pytest.mark.parametrize("cut,msg", [
    (0, "read tokenizer header: EOF"),
    (2, "read tokenizer header: unexpected EOF"),
    (4, "unexpected EOF at token 0"),
    (6, r"read token\[0\] score: unexpected EOF"),
    (10, r"read token\[0\] length: unexpected EOF"),
    (12, r"read token\[0\] bytes: EOF"),
    (14, r"read token\[0\] bytes: unexpected EOF"),
])
def test_tokenizer_truncation_errors(tmp_path, cut, msg):
    path = tmp_path / "tok.bin"
    write_tokenizer(path, [b"<unk>", b"<s>"])
    data = path.read_bytes()[:cut]
    path.write_bytes(data)
    with pytest.raises(ValueError, match=msg):
        LoadTokenizer(str(path), vocab_size=2)


def test_tokenizer_bad_header_and_length(tmp_path):
    path = tmp_path / "tok.bin"
    path.write_bytes(struct.pack("<i", 0))
    with pytest.raises(ValueError, match="bad tokenizer header: max token len=0"):
        LoadTokenizer(str(path), vocab_size=1)
    path.write_bytes(struct.pack("<i", 1) + struct.pack("<f", 0.0) + struct.pack("<i", 9))
    with pytest.raises(ValueError, match=r"bad token\[0\] length=9"):
        LoadTokenizer(str(path), vocab_size=1)


def test_tokenizer_decode_without_file():
    tok = Tokenizer([b"a", b"<0xff>"])
    assert tok.DecodeBytes(1) == b"\xff"


def write_llama2c(path, cfg, rng, shared=True, scale=1.0):
    """weights.go:49-122 order: header (7 int32), embed, rms_att[L], wq[L], wk[L], wv[L],
    wo[L], rms_ffn[L], w1[L], w2[L], w3[L], rms_final; negative vocab = unshared classifier."""
    D, F, L, V = cfg.dim, cfg.hidden, cfg.n_layers, cfg.vocab
    qd, kvd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    t = {"embed": rng.standard_normal((V, D), np.float32) * np.float32(scale)}
    for name, shape in (("rms_att", (D,)), ("wq", (qd, D)), ("wk", (kvd, D)), ("wv", (kvd, D)), ("wo", (D, qd)),
                        ("rms_ffn", (D,)), ("w1", (F, D)), ("w2", (D, F)), ("w3", (F, D))):
        sc = np.float32(1.0 if name.startswith("rms") else scale)
        t[name] = [rng.standard_normal(shape, np.float32) * sc for _ in range(L)]
    t["rms_final"] = rng.standard_normal(D, np.float32)
    with open(path, "wb") as f:
        f.write(struct.pack("<7i", D, F, L, cfg.n_heads, cfg.n_kv_heads, V if shared else -V, cfg.max_seq))
        f.write(t["embed"].astype("<f4").tobytes())
        for name in ("rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3"):
            for a in t[name]:
                f.write(a.astype("<f4").tobytes())
        f.write(t["rms_final"].astype("<f4").tobytes())
    return t


@pytest.mark.parametrize("shared", [True, False])
def test_llama2c_loader_reads_reference_layout(tmp_path, shared):
    rng = np.random.default_rng(3)
    path = tmp_path / "model.bin"
    t = write_llama2c(path, TINY, rng, shared)
    mw, hdr = LoadPretrained(str(path), TINY)
    assert hdr["Dim"] == TINY.dim and hdr["VocabSize"] == (TINY.vocab if shared else -TINY.vocab)
    assert mw.SharedCL == shared
    np.testing.assert_array_equal(mw.Embed, t["embed"])
    for i, L in enumerate(mw.Layers):
        for name, attr in (("rms_att", "RMSAtt"), ("wq", "Wq"), ("wk", "Wk"), ("wv", "Wv"), ("wo", "Wo"),
                           ("rms_ffn", "RMSFFN"), ("w1", "W1"), ("w2", "W2"), ("w3", "W3")):
            np.testing.assert_array_equal(getattr(L, attr).reshape(t[name][i].shape), t[name][i])
    np.testing.assert_array_equal(mw.RMSFinal, t["rms_final"])


def test_llama2c_loader_errors(tmp_path):
    rng = np.random.default_rng(4)
    path = tmp_path / "model.bin"
    write_llama2c(path, TINY, rng)
    data = path.read_bytes()
    (tmp_path / "short.bin").write_bytes(data[:20])
    with pytest.raises(ValueError, match="read config"):
        LoadPretrained(str(tmp_path / "short.bin"), TINY)
    (tmp_path / "trunc.bin").write_bytes(data[:28 + 4 * TINY.vocab * TINY.dim + 100])
    with pytest.raises(ValueError, match=r"read rms_att\[0\]"):
        LoadPretrained(str(tmp_path / "trunc.bin"), TINY)
    bad = bytearray(data)
    bad[0:4] = struct.pack("<i", 64)
    (tmp_path / "bad.bin").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="config mismatch: got dim=64 hidden=256 layers=2"):
        LoadPretrained(str(tmp_path / "bad.bin"), TINY)


def write_checkpoint(path, cfg, rng, version=3, meta=(7, 100, 3e-4, 2.5, 1.0, 2.0, 3.0, 11, 12, 13), scale=1.0):
    """ckpt.go:68-235 layout: 96-byte header, per layer wq wk wv wo w1 w2 w3 rms_att rms_ffn,
    per layer Adam moments (random for v3, zeros for v2), rms_final + moments, embed + moments."""
    D, F, L, V = cfg.dim, cfg.hidden, cfg.n_layers, cfg.vocab
    qd, kvd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    shapes = (("wq", (qd, D)), ("wk", (kvd, D)), ("wv", (kvd, D)), ("wo", (D, qd)), ("w1", (F, D)), ("w2", (D, F)),
              ("w3", (F, D)), ("rms_att", (D,)), ("rms_ffn", (D,)))
    t = {name: [rng.standard_normal(sh, np.float32) * np.float32(1.0 if name.startswith("rms") else scale)
                for _ in range(L)] for name, sh in shapes}
    t["rms_final"] = rng.standard_normal(D, np.float32)
    t["embed"] = rng.standard_normal((V, D), np.float32) * np.float32(scale)
    step, total, lr, loss, cc, ct, cw, cs, cb, at = meta
    with open(path, "wb") as f:
        f.write(struct.pack("<10i", 0x424C5A54, version, step, total, L, V, D, F, cfg.n_heads, cfg.max_seq))
        f.write(struct.pack("<ff3d6i", lr, loss, cc, ct, cw, cs, cb, at, 0, 0, 0))
        for i in range(L):
            for name, _ in shapes:
                f.write(t[name][i].astype("<f4").tobytes())
        per_layer = sum(int(np.prod(sh)) for _, sh in shapes)
        for i in range(L):
            mom = rng.standard_normal(2 * per_layer).astype("<f4") if version == 3 else np.zeros(2 * per_layer, "<f4")
            f.write(mom.tobytes())
        f.write(t["rms_final"].astype("<f4").tobytes())
        f.write(np.zeros(2 * D, "<f4").tobytes())
        f.write(t["embed"].astype("<f4").tobytes())
        f.write(rng.standard_normal(2 * V * D).astype("<f4").tobytes())
    return t


@pytest.mark.parametrize("version", [2, 3])
def test_checkpoint_loader_reads_reference_layout(tmp_path, version):
    from ane.stories import LoadCheckpoint, NewModelWeights
    rng = np.random.default_rng(10 + version)
    path = tmp_path / "ckpt.bin"
    t = write_checkpoint(path, TINY, rng, version)
    mw = NewModelWeights(TINY.vocab, TINY)
    meta = LoadCheckpoint(str(path), mw)
    assert (meta.Step, meta.TotalSteps, meta.CumSteps, meta.CumBatches, meta.AdamT) == (7, 100, 11, 12, 13)
    assert abs(meta.LR - 3e-4) < 1e-9 and meta.CumWall == 3.0
    for i, L in enumerate(mw.Layers):
        for name, attr in (("wq", "Wq"), ("wk", "Wk"), ("wv", "Wv"), ("wo", "Wo"), ("w1", "W1"), ("w2", "W2"),
                           ("w3", "W3"), ("rms_att", "RMSAtt"), ("rms_ffn", "RMSFFN")):
            np.testing.assert_array_equal(getattr(L, attr), t[name][i])
    np.testing.assert_array_equal(mw.RMSFinal, t["rms_final"])
    np.testing.assert_array_equal(mw.Embed, t["embed"])


def test_checkpoint_loader_errors(tmp_path):
    from ane.stories import LoadCheckpoint, NewModelWeights
    rng = np.random.default_rng(5)
    path = tmp_path / "ckpt.bin"
    write_checkpoint(path, TINY, rng, 3)
    data = bytearray(path.read_bytes())
    bad = bytearray(data)
    bad[4:8] = struct.pack("<i", 4)
    (tmp_path / "v4.bin").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="bad checkpoint header magic=424c5a54 version=4"):
        LoadCheckpoint(str(tmp_path / "v4.bin"), NewModelWeights(TINY.vocab, TINY))
    bad = bytearray(data)
    bad[24:28] = struct.pack("<i", 64)  # dim
    (tmp_path / "dim.bin").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="checkpoint config mismatch"):
        LoadCheckpoint(str(tmp_path / "dim.bin"), NewModelWeights(TINY.vocab, TINY))
    (tmp_path / "trunc.bin").write_bytes(bytes(data[:-10]))
    with pytest.raises(ValueError, match="embed optimizer state"):
        LoadCheckpoint(str(tmp_path / "trunc.bin"), NewModelWeights(TINY.vocab, TINY))
