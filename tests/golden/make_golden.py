"""Regenerates tests/golden/*.npz from the reference engine (oracle/_ref).

    python tests/golden/make_golden.py

The inputs are the seeded synthetic models of qwen_b200.py (TINY, seed 1 /
TINY mixed-format, seed 2); the outputs are what the compiled reference
produces for them: prefill logits, the MTP-speculative token stream under
a seeded forced accept schedule, the accept lengths, and plain greedy
tokens.  Run only where the reference sources exist.
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from conftest import oracle, qb  # noqa: E402


def forced_schedule(n, seed):
    return np.random.default_rng(seed).integers(0, 4, n).astype(np.uint32)


def make(name, shape, seed, profile, n_predict=64):
    with tempfile.TemporaryDirectory() as d:
        path = qb.write_synth_gguf(os.path.join(d, "m.gguf"), shape, seed=seed, profile=profile)
        prompt = (np.arange(12, dtype=np.uint64) * 2654435761 % shape["vocab"]).astype(np.uint32)
        forced = forced_schedule(64, seed)
        m = oracle.RefModel(path, 256, 0)
        m.prefill(prompt, 1)
        prefill_logits64 = m.logits()[:64].astype(np.float32)
        tokens, accept = m.spec_generate(n_predict, 3, forced=forced)
        m.close()
        g = oracle.RefModel(path, 256, 0)
        g.prefill(prompt, 0)
        greedy = g.greedy_generate(32)
        g.close()
    np.savez(os.path.join(HERE, f"{name}.npz"), prompt=prompt, forced=forced, n_predict=n_predict,
             prefill_logits64=prefill_logits64, tokens=tokens, accept=accept, greedy=greedy)
    print(name, tokens[:16], accept[:16], greedy[:8])


if __name__ == "__main__":
    make("tiny_spec", qb.TINY, 1, 0)
    make("tiny_mixed_spec", qb.TINY, 2, 1)
