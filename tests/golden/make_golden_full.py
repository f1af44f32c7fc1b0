"""Writes tests/golden/full_spec.npz: the compiled reference engine (oracle/_ref)
on the 64-layer benchmark model, so the GPU engine's output on that model can be
checked on a box where the reference sources do not exist.

    python tests/golden/make_golden_full.py [--out DIR]

Inputs are exactly bench.py's workload: the FULL synthetic model (seed 0), the
128-token prompt `rng(1000).integers(0, vocab, 128)` and the forced accept
schedule `rng(0).integers(0, 4, n)`.  Outputs:

  prefill_sub / prefill_top   the prefill logits (every 61st entry, and the
                              top 8 ids and values)
  tokens / accept             MTP speculative stream (k = 3) under the forced
                              schedule, src/main.c:158-225
  greedy / greedy_gap         plain greedy decode after a non-speculative
                              prefill (src/main.c:232-248) and, per step, the
                              reference's top-1 minus top-2 logit gap, so that a
                              flipped token can be told apart from a near tie

Needs about 16 GB of free disk for the GGUF and a few minutes on 8 cores.
"""
import argparse
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from conftest import oracle, qb  # noqa: E402

PROMPT_LEN = 128
N_PREDICT = 96
N_GREEDY = 16
SUB = 61


def prompt_tokens():
    return np.random.default_rng(1000).integers(0, qb.FULL["vocab"], PROMPT_LEN).astype(np.uint32)


def forced_schedule(n=4096):
    return np.random.default_rng(0).integers(0, 4, n).astype(np.uint32)


def top2_gap(x):
    i = int(np.argmax(x))
    y = x.copy()
    y[i] = -np.inf
    return float(x[i] - y.max())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--gguf", default="", help="reuse an existing FULL seed-0 GGUF")
    args = ap.parse_args()
    with tempfile.TemporaryDirectory(dir="/tmp") as d:
        path = args.gguf or qb.write_synth_gguf(os.path.join(d, "full.gguf"), qb.FULL, seed=0)
        prompt, forced = prompt_tokens(), forced_schedule()
        t0 = time.time()
        m = oracle.RefModel(path, 512, 0)
        m.prefill(prompt, 1)
        lg = m.logits()
        order = np.argsort(-lg, kind="stable")[:8]
        print(f"prefill {time.time() - t0:.1f}s top {order[:4]}", flush=True)
        tokens, accept = m.spec_generate(N_PREDICT, 3, forced=forced)
        print(f"spec {time.time() - t0:.1f}s {tokens[:12]} {accept[:12]}", flush=True)
        m.close()

        g = oracle.RefModel(path, 512, 0)
        g.prefill(prompt, 0)
        greedy, gaps = [], []
        for _ in range(N_GREEDY):
            lgt = g.logits()
            greedy.append(int(np.argmax(lgt)))
            gaps.append(top2_gap(lgt))
            if len(greedy) < N_GREEDY:
                g.forward(greedy[-1], g.pos)
        g.close()
        print(f"greedy {time.time() - t0:.1f}s {greedy} min gap {min(gaps):.3g}", flush=True)
    np.savez(os.path.join(args.out, "full_spec.npz"), prompt=prompt, forced=forced[:256],
             n_predict=N_PREDICT, prefill_sub=lg[::SUB].astype(np.float32), sub_stride=SUB,
             prefill_top=order.astype(np.uint32), prefill_top_val=lg[order].astype(np.float32),
             tokens=tokens, accept=accept, greedy=np.array(greedy, np.uint32),
             greedy_gap=np.array(gaps, np.float32))


if __name__ == "__main__":
    main()
