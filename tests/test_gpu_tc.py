"""The tcgen05 IQ4_XS GEMV (QB_TC=1): the same parity bar as the default path.

The switch is read once per process, so each check runs in a child process:
the 17408x5120 micro GEMV at n = 1, 2, 4 against the reference gemv_batch,
and the speculative token stream of the TINY model (IQ4_XS projections)
against the golden reference stream.
"""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import os, sys
import numpy as np
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from conftest import qb, oracle
import tempfile

def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))

K, rows = 5120, 17408
raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=0, d_sigma=0.02)
t = qb.tensor(raw, qb.GGML_IQ4_XS, K, rows)
for n in (1, 2, 4):
    x = qb.synth_normal(n * K, seed=100 + n).reshape(n, K)
    got = qb.gemv_batch(t, x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for i in range(n):
        r = rel(got[i], ref[i])
        assert r < 1e-5, (n, i, r)

g = np.load(os.path.join({root!r}, "tests", "golden", "tiny_spec.npz"))
with tempfile.TemporaryDirectory() as d:
    path = qb.write_synth_gguf(os.path.join(d, "m.gguf"), qb.TINY, seed=1)
    m = qb.Model(path, 256)
    m.prefill(g["prompt"], 1)
    toks, js = m.spec_generate(int(g["n_predict"]), 3, forced=g["forced"])
    assert np.array_equal(toks, g["tokens"]), (toks[:16], g["tokens"][:16])
    assert np.array_equal(js, g["accept"]), (js, g["accept"])
    m.close()
print("tc ok")
"""


def test_tcgen05_iq4_path_parity():
    env = dict(os.environ, QB_TC="1")
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "tc ok" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
