"""Long context (config C4): a 2048-token prompt through the chunked prefill
(chunks of 32 tokens while more than 32 remain, then of 8; one graph replay
each, no host wait in between), then MTP speculation at that context, where
the attention reads 2048+ cached positions in 64 chunks per head.  A 32-token
chunk runs its attention as 4 groups of 8 queries and its IQ4_XS GEMVs in one
sweep on the wide tcgen05 GEMM once qb_enable_wide made its tiles (else in
8-row chunks).

  - WIDE4 (4 layers at full width) against the compiled reference engine run
    live: prefill logits relative L2 <= 1e-4, then tokens and accept lengths
    bit-exact under the forced schedule, logits after the stream <= 1e-4;
  - FULL (the 64-layer benchmark model) against tests/golden/full_long.npz
    (tests/golden/make_golden_long.py): prefill logits <= 1e-4 on every 61st
    entry with the same top-1, then 64 speculative tokens bit-exact.
"""
import os

import numpy as np
import pytest

from conftest import ROOT, oracle, qb

pytestmark = pytest.mark.gpu

RTOL = 1e-4
N_PROMPT = 2048


def rel(a, b):
    return float(np.linalg.norm(np.float64(a) - np.float64(b)) / max(np.linalg.norm(np.float64(b)), 1e-30))


def forced_schedule(n=4096):
    return np.random.default_rng(0).integers(0, 4, n).astype(np.uint32)


@pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")
def test_long_prompt_wide4_matches_reference(wide_gguf):
    prompt = np.random.default_rng(21).integers(0, qb.WIDE4["vocab"], N_PROMPT).astype(np.uint32)
    forced = forced_schedule()
    n_ctx = N_PROMPT + 128
    g, r = qb.Model(wide_gguf, n_ctx), oracle.RefModel(wide_gguf, n_ctx, 0)
    g.prefill(prompt, 1)
    r.prefill(prompt, 1)
    assert rel(g.logits(), r.logits()) < RTOL
    gt, gj = g.spec_generate(48, 3, forced=forced)
    rt, rj = r.spec_generate(48, 3, forced=forced)
    np.testing.assert_array_equal(gt, rt)
    np.testing.assert_array_equal(gj, rj)
    assert rel(g.logits(), r.logits()) < RTOL
    assert g.pos == r.pos
    # the KV cache of an attention layer at the far end of the context
    il = next(i for i in range(qb.WIDE4["n_layer"]) if (i + 1) % 4 == 0)
    n = (g.pos - 4) * 1024   # positions [0, pos - 4): the prompt and accepted tokens, not rewritten since
    assert rel(g.read_state(il, 2, n), r.state(il, 2, n)) < RTOL
    assert rel(g.read_state(il, 3, n), r.state(il, 3, n)) < RTOL
    g.close()
    r.close()


@pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("wide", [False, True])
def test_prefill_chunking_matches_reference(tiny_gguf, wide):
    """Prompt lengths around the 32- and 8-token chunk boundaries, with and without
    the wide tcgen05 GEMM: prefill logits, MTP hidden state and the speculative
    stream after it equal the reference's."""
    for n in (31, 32, 33, 40, 41, 64, 65, 100, 129):
        prompt = np.random.default_rng(n).integers(0, 2048, n).astype(np.uint32)
        g = qb.Model(tiny_gguf, 256)
        if wide:
            g.enable_wide()
        g.prefill(prompt, 1)
        r = oracle.RefModel(tiny_gguf, 256, 0)
        r.prefill(prompt, 1)
        assert rel(g.logits(), r.logits()) < RTOL, n
        assert rel(g.mtp_h(), r.mtp_h()) < RTOL, n
        gt, gj = g.spec_generate(24, 3, forced=forced_schedule())
        rt, rj = r.spec_generate(24, 3, forced=forced_schedule())
        np.testing.assert_array_equal(gt, rt, err_msg=f"n = {n}")
        np.testing.assert_array_equal(gj, rj, err_msg=f"n = {n}")
        g.close()
        r.close()


def test_long_prompt_full_matches_golden(full_gguf):
    gold = np.load(os.path.join(ROOT, "tests", "golden", "full_long.npz"))
    n = int(gold["prompt_len"])
    prompt = np.random.default_rng(int(gold["prompt_seed"])).integers(0, qb.FULL["vocab"], n).astype(np.uint32)
    m = qb.Model(full_gguf, n + 256)
    m.enable_wide()   # the benchmark's C4 path: 32-token chunks on the wide tcgen05 GEMM
    m.prefill(prompt, 1)
    lg = m.logits()
    assert rel(lg[:: int(gold["sub_stride"])], gold["prefill_sub"]) < RTOL
    assert int(np.argmax(lg)) == int(gold["prefill_top"][0])
    toks, js = m.spec_generate(int(gold["n_predict"]), 3, forced=gold["forced"])
    first_diff = next((i for i in range(min(len(toks), len(gold["tokens"])))
                       if toks[i] != gold["tokens"][i]), None)
    assert first_diff is None, f"first differing token at {first_diff}"
    np.testing.assert_array_equal(toks, gold["tokens"])
    np.testing.assert_array_equal(js, gold["accept"])
    m.close()
