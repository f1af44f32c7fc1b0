"""Fused GEMV epilogues against the unfused kernel sequence.

With QB_FUSE=1 a residual GEMV (FFN down, attention / DeltaNet output
projection) prepares the next RMSNorm'd GEMV input per 256-row block as its
tile pairs finish, and the gate / up GEMV applies SwiGLU and prepares the
down projection's input.  QB_FUSE=0 (the default) runs the separate RMSNorm,
SwiGLU and activation-prep kernels instead.
Both must reproduce the golden reference token streams, and their logits
must agree to fp32 rounding.  The switch is read at model load, so each run
is a child process.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import os, sys
import numpy as np
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from conftest import qb
out = {{}}
for name, seed, profile in (("tiny_spec", 1, 0), ("tiny_mixed_spec", 2, 1)):
    g = np.load(os.path.join({root!r}, "tests", "golden", name + ".npz"))
    path = qb.write_synth_gguf(os.path.join({tmp!r}, name + ".gguf"), qb.TINY, seed=seed, profile=profile)
    m = qb.Model(path, 256)
    m.prefill(g["prompt"], 1)
    out[name + "_prefill"] = m.logits().copy()
    toks, js = m.spec_generate(int(g["n_predict"]), 3, forced=g["forced"])
    assert np.array_equal(toks, g["tokens"]), (name, toks[:16], g["tokens"][:16])
    assert np.array_equal(js, g["accept"]), (name, js, g["accept"])
    out[name + "_end"] = m.logits().copy()
    m.close()
np.savez({dst!r}, **out)
print("fuse ok")
"""


def run_child(tmp_path, fuse):
    dst = str(tmp_path / f"logits_fuse{fuse}.npz")
    env = dict(os.environ, QB_FUSE=str(fuse))
    env.pop("QB_TC", None)
    code = CHILD.format(root=ROOT, tmp=str(tmp_path), dst=dst)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "fuse ok" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
    return np.load(dst)


def test_fused_and_unfused_agree(tmp_path):
    fused, plain = run_child(tmp_path, 1), run_child(tmp_path, 0)
    for k in fused.files:
        a, b = np.float64(fused[k]), np.float64(plain[k])
        rel = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert rel < 1e-5, (k, rel)
