"""Parity at the benchmark configurations' shapes, through the C ABI.

Each test prefills a full batch at the configuration's prompt length, runs >= 16 greedy decode
steps with logits, and checks a few of its rows teacher-forced against the oracle:
  - in GPU order at the north_star's bounds (logits max-abs 2e-2 fp16 / bf16, 5e-2 W8A8,
    top-1 >= 99%) -- the rows are in fact bit-identical;
  - in the reference's order of operations at the same precision, where the printed numbers are
    the spec-order distances and the bounds are the checker's noise floor (parity.REF_ORDER_*).
The config 5 test runs the regime the benchmark times: Qwen3-0.6B W8A8, contexts past 1024, a
batch of 128 rows decoded as 4 overlapped micro-batches with one attention CTA per (sequence,
kv head).  Reference rows are independent (ane/stories/infer.go:136-245), so checking a few rows
of the batch checks the batch."""
import numpy as np
import pytest

import oracle as O
from ane import _abi
from ane.stories import QWEN3_0_6B, STORIES_110M, Engine, SyntheticWeights
from parity import LOGIT_TOL, REF_ORDER_TOL, REF_ORDER_TOP1, TOP1_MIN, gpu_order, oracle_check

pytestmark = pytest.mark.gpu


def run_batch(eng, prompts, steps, check):
    """Prefill every prompt, `steps` decode steps of the whole batch; tokens of every row and
    logits of the rows in `check` ([steps + 1, vocab] each)."""
    n = len(prompts)
    seqs = list(range(n))
    nxt, lg = eng.prefill(seqs, prompts, want_logits=True)
    toks = [[int(t)] for t in nxt]
    logits = {i: [lg[i]] for i in check}
    cur = nxt.copy()
    pos = np.array([len(p) for p in prompts], np.int32)
    for _ in range(steps):
        nxt, lg = eng.decode_step(seqs, cur, pos, want_logits=True)
        for i in range(n):
            toks[i].append(int(nxt[i]))
        for i in check:
            logits[i].append(lg[i])
        cur, pos = nxt, pos + 1
    return toks, {i: np.stack(v) for i, v in logits.items()}


def check_rows(cfg, w, dtype, prompts, toks, logits, rows, label):
    ps = [prompts[i] for i in rows]
    ts = [toks[i] for i in rows]
    ls = [logits[i] for i in rows]
    worst, agree, total = oracle_check(gpu_order(cfg, w, dtype), ps, ts, ls)
    print(f"{label}: vs GPU-order oracle max|dlogit|={worst:.3e} top1={agree:.4f} over {total}")
    assert worst <= LOGIT_TOL[dtype] and agree >= TOP1_MIN[dtype], (worst, agree)
    assert worst == 0.0 and agree == 1.0
    worst, agree, _ = oracle_check(O.Model(cfg.oracle_dict(), w, dtype), ps, ts, ls)
    print(f"{label}: vs reference-order oracle (same precision) max|dlogit|={worst:.3e} top1={agree:.4f}")
    assert worst <= REF_ORDER_TOL[dtype] and agree >= REF_ORDER_TOP1[dtype], (worst, agree)
    if dtype == "fp16":
        worst32, agree32, _ = oracle_check(O.Model(cfg.oracle_dict(), w, "fp32"), ps, ts, ls)
        print(f"{label}: vs the reference's fp32 arithmetic max|dlogit|={worst32:.3e} top1={agree32:.4f}")
        assert worst32 <= 2e-2


@pytest.mark.parametrize("name,cfg,dtype,out_scale,batch,P,steps,rows", [
    ("config2", STORIES_110M, "fp16", 1 / np.sqrt(24), 64, 128, 16, [0, 21, 42, 63]),
    ("config3", STORIES_110M, "w8a8_fp16", 1 / np.sqrt(24), 256, 64, 16, [0, 85, 170, 255]),
    ("config4", QWEN3_0_6B, "bf16", 1.0, 128, 512, 16, [0, 127]),
], ids=["config2-stories-fp16-b64-p128", "config3-stories-w8a8-b256-p64", "config4-qwen3-bf16-b128-p512"])
def test_config_prompt_lengths(name, cfg, dtype, out_scale, batch, P, steps, rows):
    cfg = cfg.with_max_seq(P + steps + 16)
    w = SyntheticWeights(cfg, 1234, out_scale)
    eng = Engine(cfg, dtype)
    eng.load(w)
    eng.kv_alloc(batch, P + steps + 1)
    rng = np.random.default_rng(1235)
    prompts = [rng.integers(3, cfg.vocab, P).tolist() for _ in range(batch)]
    toks, logits = run_batch(eng, prompts, steps, rows)
    eng.close()
    check_rows(cfg, w, dtype, prompts, toks, logits, rows, f"{name} {cfg.name} {dtype}")


def test_config5_regime_long_context_overlapped_batch():
    cfg = QWEN3_0_6B.with_max_seq(1200)
    w = SyntheticWeights(cfg, 1234, 1.0)
    batch, steps = 128, 16
    eng = Engine(cfg, "w8a8_bf16")
    eng.load(w)
    eng.kv_alloc(batch, 1200)
    eng.set_option(_abi.LLM_OPT_OVERLAP, 2)        # the overlapped micro-batch schedule
    eng.set_option(_abi.LLM_OPT_MICRO_BATCHES, 4)
    assert eng.step_parts(batch) == 4
    rng = np.random.default_rng(1236)
    lens = rng.integers(1024, 1100, batch)
    prompts = [rng.integers(3, cfg.vocab, int(L)).tolist() for L in lens]
    rows = [0, 77]
    toks, logits = run_batch(eng, prompts, steps, rows)
    eng.close()
    assert min(len(prompts[i]) for i in rows) >= 1024
    check_rows(cfg, w, "w8a8_bf16", prompts, toks, logits, rows, "config5 regime qwen3 w8a8 b128 ctx>=1024")
