"""Parity on the 64-layer benchmark model itself (the FULL synthetic model that
bench.py times: hidden 5120, FFN 17408, vocab 248320, 48 DeltaNet + 16
attention layers + the MTP block; 15.3 GB of weights).

Checked against tests/golden/full_spec.npz, the compiled reference engine's
output for exactly bench.py's workload (tests/golden/make_golden_full.py):
  - prefill logits of the 128-token prompt: relative L2 <= 1e-4 on every 61st
    entry, same top-1 id;
  - MTP speculation, k = 3, under the forced accept schedule: tokens and
    accept lengths bit-exact (36 cycles, 96 tokens);
  - greedy decode after a non-speculative prefill: 16 tokens bit-exact (the
    reference's smallest top-1 / top-2 gap on these steps is 0.0104);
  - natural acceptance: speculation without forcing emits the greedy stream.
"""
import os

import numpy as np
import pytest

from conftest import ROOT, qb

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm(np.float64(a) - np.float64(b)) / max(np.linalg.norm(np.float64(b)), 1e-30))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(ROOT, "tests", "golden", "full_spec.npz"))


@pytest.fixture(scope="module")
def model(full_gguf):
    m = qb.Model(full_gguf, 512)
    yield m
    m.close()


def test_full_prefill_logits(model, gold):
    model.reset()
    model.prefill(gold["prompt"], 1)
    lg = model.logits()
    assert rel(lg[:: int(gold["sub_stride"])], gold["prefill_sub"]) < RTOL
    assert int(np.argmax(lg)) == int(gold["prefill_top"][0])


def test_full_spec_stream_bit_exact(model, gold):
    model.reset()
    model.prefill(gold["prompt"], 1)
    toks, js = model.spec_generate(int(gold["n_predict"]), 3, forced=gold["forced"])
    first_diff = next((i for i in range(min(len(toks), len(gold["tokens"])))
                       if toks[i] != gold["tokens"][i]), None)
    assert first_diff is None, f"first differing token at {first_diff}"
    np.testing.assert_array_equal(toks, gold["tokens"])
    np.testing.assert_array_equal(js, gold["accept"])


def test_full_greedy_bit_exact(model, gold):
    model.reset()
    model.prefill(gold["prompt"], 0)
    got = model.greedy_generate(len(gold["greedy"]))
    bad = [(i, int(got[i]), int(gold["greedy"][i]), float(gold["greedy_gap"][i]))
           for i in range(len(got)) if got[i] != gold["greedy"][i]]
    assert not bad, f"(step, ours, reference, reference top-1/top-2 gap): {bad}"


def test_full_natural_spec_equals_greedy(model, gold):
    model.reset()
    model.prefill(gold["prompt"], 1)
    toks, _ = model.spec_generate(len(gold["greedy"]), 3)
    np.testing.assert_array_equal(toks, gold["greedy"])
