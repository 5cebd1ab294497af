"""The stories-generate mirror end to end on the GPU: the reference's three output lines, and
the greedy tokens of the stories.Decoder path (cmd/stories-generate-go/main.go:60-97)."""
import io
import re

import pytest

from ane.cmd.stories_generate import main
from ane.stories import STORIES_110M, DecodeOptions, NewDecoder, SyntheticWeights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ane", [False, True])
def test_cli_lines_and_tokens(ane):
    buf = io.StringIO()
    args = ["-synthetic-seed", "1234", "-prompt-ids", "1,345,12", "-max-new", "12", "-temperature", "0", "-seq", "64"]
    assert main(args + (["-ane"] if ane else []), out=buf) == 0
    lines = buf.getvalue().strip().split("\n")
    assert len(lines) == 3
    m = re.fullmatch(r"source=synthetic prompt_tokens=3 generated_tokens=(\d+) elapsed=\S+ tok/s=\d+\.\d\d eos=(true|false)",
                     lines[0])
    assert m, lines[0]
    toks = [int(t) for t in lines[1][len("tokens="):].split(",")]
    assert toks[:3] == [1, 345, 12] and len(toks) == 3 + int(m.group(1))
    assert lines[2] == "text=(tokenizer not provided)"
    if not ane:
        w = SyntheticWeights(STORIES_110M, 1234, 24 ** -0.5)
        dec = NewDecoder(w, 64, 7, dtype="fp16")
        assert dec.Decode(None, DecodeOptions(MaxNewTokens=12, PromptTokens=[1, 345, 12])).Tokens == toks
        dec.Close()


def test_cli_errors():
    assert main(["-prompt-ids", "1,x"]) == 1
    assert main(["-model", "/nonexistent/model.bin", "-temperature", "0"]) == 1
