"""Writes tests/golden/full_long.npz: the compiled reference engine (oracle/_ref)
on the 64-layer benchmark model with a long prompt (config C4: a 2048-token
prompt, then MTP speculative decode at that context), so that the GPU engine's
long-context output can be checked on a box where the reference sources do not
exist.

    python tests/golden/make_golden_long.py [--gguf FULL_SEED0.gguf] [--out DIR]

Inputs are bench.py's C4 workload: the FULL synthetic model (seed 0), the prompt
`rng(2000).integers(0, vocab, 2048)` and the forced accept schedule
`rng(0).integers(0, 4, n)`.  Outputs:

  prefill_sub / prefill_top   the logits after the 2048-token prefill (every
                              61st entry, and the top 8 ids and values)
  tokens / accept             MTP speculative stream (k = 3) under the forced
                              schedule from position 2048, src/main.c:158-225

Needs about 16 GB of free disk for the GGUF and about ten minutes on 8 cores.
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

PROMPT_LEN = 2048
N_PREDICT = 64
SUB = 61


def prompt_tokens():
    return np.random.default_rng(2000).integers(0, qb.FULL["vocab"], PROMPT_LEN).astype(np.uint32)


def forced_schedule(n=4096):
    return np.random.default_rng(0).integers(0, 4, n).astype(np.uint32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--gguf", default="", help="reuse an existing FULL seed-0 GGUF")
    args = ap.parse_args()
    with tempfile.TemporaryDirectory(dir="/tmp") as d:
        path = args.gguf or qb.write_synth_gguf(os.path.join(d, "full.gguf"), qb.FULL, seed=0)
        prompt, forced = prompt_tokens(), forced_schedule()
        t0 = time.time()
        m = oracle.RefModel(path, PROMPT_LEN + 256, 0)
        m.prefill(prompt, 1)
        lg = m.logits()
        order = np.argsort(-lg, kind="stable")[:8]
        print(f"prefill {time.time() - t0:.1f}s top {order[:4]}", flush=True)
        tokens, accept = m.spec_generate(N_PREDICT, 3, forced=forced)
        print(f"spec {time.time() - t0:.1f}s {tokens[:12]} {accept[:12]}", flush=True)
        m.close()
    np.savez(os.path.join(args.out, "full_long.npz"), prompt_seed=2000, prompt_len=PROMPT_LEN,
             forced=forced[:256], n_predict=N_PREDICT, prefill_sub=lg[::SUB].astype(np.float32), sub_stride=SUB,
             prefill_top=order.astype(np.uint32), prefill_top_val=lg[order].astype(np.float32),
             tokens=tokens, accept=accept)


if __name__ == "__main__":
    main()
