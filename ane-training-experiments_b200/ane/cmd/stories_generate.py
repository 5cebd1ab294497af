"""Mirror of cmd/stories-generate-go (cmd/stories-generate-go/main.go:16-161) on the CUDA token
loop: the same flags, the same three output lines

    source=<src> prompt_tokens=<n> generated_tokens=<n> elapsed=<Go duration> tok/s=<f> eos=<bool>
    tokens=<comma-separated ids>
    text=<decoded text> | text=(tokenizer not provided)

and the same error texts.  Additive flags: -engine cuda (the only engine), -dtype
fp16|bf16|w8a8, -model-family stories|qwen3, -synthetic-seed (seeded N(0, 0.02) weights in place
of a file; the reference's RandomInit stream cannot be reproduced), -batch (decode that many
copies of the prompt as independent sequences; one block of lines per sequence), -device.

    python -m ane.cmd.stories_generate -synthetic-seed 1234 -prompt-ids 1 -max-new 64 -temperature 0
"""
from __future__ import annotations

import argparse
import sys
import time
from typing import List, Optional

from .. import _abi
from ..stories import (PRESETS, DecodeOptions, LoadCheckpoint, LoadPretrained, LoadTokenizer, NewDecoder,
                       NewModelWeights, SeqDefault, SyntheticWeights)


def parse_token_list(s: str) -> List[int]:
    """main.go:120-141: empty -> [1]; comma-separated ints, blanks skipped."""
    s = s.strip()
    if s == "":
        return [1]
    out = []
    for i, p in enumerate(s.split(",")):
        p = p.strip()
        if p == "":
            continue
        try:
            out.append(int(p, 10))
        except ValueError:
            raise ValueError(f'token[{i}]="{p}": strconv.Atoi: parsing "{p}": invalid syntax') from None
    return out or [1]


def go_duration(seconds: float) -> str:
    """time.Duration.Round(time.Millisecond).String() for non-negative durations."""
    ms = int(round(seconds * 1000))
    if ms == 0:
        return "0s"
    if ms < 1000:
        return f"{ms}ms"
    h, rem = divmod(ms, 3600_000)
    m, rem = divmod(rem, 60_000)
    s, frac = divmod(rem, 1000)
    sec = f"{s}" + (f".{frac:03d}".rstrip("0") if frac else "") + "s"
    if h:
        return f"{h}h{m}m{sec}"
    if m:
        return f"{m}m{sec}"
    return sec


def _flags(argv: Optional[List[str]]):
    ap = argparse.ArgumentParser(prog="stories-generate", prefix_chars="-", allow_abbrev=False)
    ap.add_argument("-model", default="", help="path to stories110M.bin")
    ap.add_argument("-ckpt", default="", help="optional checkpoint path (overrides -model)")
    ap.add_argument("-tokenizer", default="", help="optional tokenizer.bin path for decoded text")
    ap.add_argument("-prompt-ids", dest="prompt_ids", default="1", help="comma-separated prompt token IDs")
    ap.add_argument("-max-new", dest="max_new", type=int, default=64, help="maximum new tokens to generate")
    ap.add_argument("-temperature", type=float, default=0.8, help="sampling temperature (0 for greedy)")
    ap.add_argument("-seed", type=int, default=time.time_ns(), help="sampling seed")
    ap.add_argument("-seq", type=int, default=SeqDefault, help="max sequence length")
    ap.add_argument("-ane", action="store_true", help="use storiesane full-sequence engine")
    ap.add_argument("-engine", default="cuda", choices=["cuda"])
    ap.add_argument("-dtype", default="fp16", choices=["fp16", "bf16", "w8a8"])
    ap.add_argument("-model-family", dest="family", default="stories", choices=["stories", "qwen3"])
    ap.add_argument("-synthetic-seed", dest="synthetic_seed", type=int, default=0)
    ap.add_argument("-batch", type=int, default=1)
    ap.add_argument("-device", type=int, default=0)
    return ap.parse_args(argv)


def main(argv: Optional[List[str]] = None, out=None) -> int:
    out = out or sys.stdout
    a = _flags(argv)
    try:
        prompt = parse_token_list(a.prompt_ids)
    except ValueError as e:
        print(f"parse prompt tokens: {e}", file=sys.stderr)
        return 1
    tok = None
    if a.tokenizer:
        try:
            tok = LoadTokenizer(a.tokenizer)
        except (OSError, ValueError) as e:
            print(f"load tokenizer: {e}", file=sys.stderr)
            return 1
    cfg = PRESETS["stories110m" if a.family == "stories" else "qwen3-0.6b"]
    dtype = {"fp16": "fp16", "bf16": "bf16", "w8a8": "w8a8_fp16" if a.family == "stories" else "w8a8_bf16"}[a.dtype]
    opts = DecodeOptions(MaxNewTokens=a.max_new, Temperature=float(a.temperature), Seed=a.seed, PromptTokens=prompt)
    start = time.perf_counter()
    try:
        if a.synthetic_seed:
            w = SyntheticWeights(cfg, a.synthetic_seed, 24 ** -0.5 if a.family == "stories" else 1.0)
            src = "synthetic"
        elif a.ckpt:
            w = NewModelWeights()
            LoadCheckpoint(a.ckpt, w, None)
            src = "checkpoint"
        else:
            w, _ = LoadPretrained(a.model)
            src = "pretrained"
        if a.ane:
            from ..storiesane import Open, Options
            eng = Open(Options(Weights=w, Seq=a.seq, Seed=a.seed, UseANE=True, DType=dtype, Device=a.device))
            results = [eng.Decode(tok, opts) for _ in range(a.batch)]
            eng.Close()
        else:
            dec = NewDecoder(w, a.seq, a.seed, dtype=dtype, device=a.device, max_batch=a.batch)
            results = dec.DecodeBatch(tok, opts, [prompt] * a.batch)
            dec.Close()
    except (_abi.LLMError, OSError, ValueError) as e:
        print(f"decode: {e}", file=sys.stderr)
        return 1
    elapsed = time.perf_counter() - start
    for res in results:
        new = len(res.Tokens) - res.PromptLength
        tps = new / elapsed if elapsed > 0 else 0.0
        print(f"source={src} prompt_tokens={res.PromptLength} generated_tokens={new} elapsed={go_duration(elapsed)} "
              f"tok/s={tps:.2f} eos={'true' if res.StoppedOnEOS else 'false'}", file=out)
        print("tokens=" + ",".join(str(t) for t in res.Tokens), file=out)
        print(f"text={res.Text}" if tok is not None else "text=(tokenizer not provided)", file=out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
