"""Synthetic GGUF writer: deterministic, thread-count independent, and
parsed identically by the reference (tests/test_oracle.py) and the engine."""
import hashlib
import os

import numpy as np

from conftest import qb


def _sha(p):
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def test_deterministic_across_thread_counts(tmp_path):
    a = qb.write_synth_gguf(str(tmp_path / "a.gguf"), qb.TINY, seed=7, n_threads=1)
    b = qb.write_synth_gguf(str(tmp_path / "b.gguf"), qb.TINY, seed=7, n_threads=8)
    c = qb.write_synth_gguf(str(tmp_path / "c.gguf"), qb.TINY, seed=8, n_threads=8)
    assert _sha(a) == _sha(b)
    assert _sha(a) != _sha(c)


def test_file_size_matches_layout(tmp_path):
    p = qb.write_synth_gguf(str(tmp_path / "t.gguf"), qb.TINY, seed=1)
    data = qb.synth_lib().qb_synth_file_size(qb.synth_cfg(qb.TINY))
    assert 0 < data < os.path.getsize(p) < data + 65536


def test_full_model_size():
    """The benchmark model is the 64-layer hybrid: ~15.3 GB of GGUF data."""
    n = qb.synth_lib().qb_synth_file_size(qb.synth_cfg(qb.FULL))
    assert 15.0e9 < n < 15.6e9


def test_fp16_conversion_round_to_nearest_even():
    f = qb.synth_lib().qb_f32_to_f16
    f.argtypes = [np.ctypeslib.ctypes.c_float]
    f.restype = np.ctypeslib.ctypes.c_uint16
    for v in [0.0, 1.0, -2.5, 65504.0, 1e-5, 6.1e-5, 3.0e-8, 0.1, 1234.567]:
        assert f(v) == np.float16(v).view(np.uint16), v
    rng = np.random.default_rng(0)
    for v in rng.standard_normal(2000).astype(np.float32) * np.float32(1e-4):
        assert f(float(v)) == np.float16(v).view(np.uint16)
