"""Weight files streamed to the device by llm_load_weights_file (llama2.c .bin of
ane/stories/weights.go:49-122, checkpoint v2/v3 of ane/stories/ckpt.go:237-447) must give
bit-identical logits to the same weights loaded from host arrays by the Python readers, and
report the reference's errors for malformed files."""
import struct

import numpy as np
import pytest

from ane import _abi
from ane.stories import Engine, LoadCheckpoint, LoadPretrained, NewModelWeights
from parity import gpu_run
from test_formats import TINY, write_checkpoint, write_llama2c

pytestmark = pytest.mark.gpu


def run(eng, prompts):
    eng.kv_alloc(len(prompts), 64)
    return gpu_run(eng, prompts, 6)


@pytest.mark.parametrize("fmt,version", [("llama2c", 0), ("checkpoint", 2), ("checkpoint", 3)])
@pytest.mark.parametrize("dtype", ["fp16", "w8a8_fp16"])
def test_file_loader_equals_host_loader(tmp_path, fmt, version, dtype):
    rng = np.random.default_rng(21)
    path = tmp_path / "w.bin"
    if fmt == "llama2c":
        write_llama2c(path, TINY, rng, scale=0.05)
        mw, _ = LoadPretrained(str(path), TINY)
    else:
        write_checkpoint(path, TINY, rng, version, scale=0.05)
        mw = NewModelWeights(TINY.vocab, TINY)
        LoadCheckpoint(str(path), mw)
    prompts = [[5, 9, 200], [17] * 20]
    host = Engine(TINY, dtype).load(mw)
    t_host, l_host = run(host, prompts)
    host.close()
    dev = Engine(TINY, dtype).load_file(str(path), fmt)
    t_dev, l_dev = run(dev, prompts)
    dev.close()
    assert t_host == t_dev
    assert all(np.isfinite(a).all() for a in l_host)
    for a, b in zip(l_host, l_dev):
        np.testing.assert_array_equal(a, b)


def test_file_loader_errors(tmp_path):
    rng = np.random.default_rng(22)
    path = tmp_path / "w.bin"
    write_llama2c(path, TINY, rng)
    data = path.read_bytes()
    bad = bytearray(data)
    bad[4:8] = struct.pack("<i", 512)
    (tmp_path / "bad.bin").write_bytes(bytes(bad))
    eng = Engine(TINY, "fp16")
    with pytest.raises(_abi.LLMError, match="config mismatch: got dim=128 hidden=512 layers=2"):
        eng.load_file(str(tmp_path / "bad.bin"))
    (tmp_path / "trunc.bin").write_bytes(data[: len(data) - 4 * TINY.dim - 8])
    with pytest.raises(_abi.LLMError, match=r"read w3\[1\]|read rms_final"):
        eng.load_file(str(tmp_path / "trunc.bin"))
    with pytest.raises(_abi.LLMError, match="bad checkpoint header magic"):
        eng.load_file(str(path), "checkpoint")
    eng.close()
