"""Pins the oracle: the compiled reference (oracle/_ref) against its own
known-answer suite and the numpy restatement (oracle/ref.py) against the
compiled reference, on synthetic blocks of every hot-path format."""
import os
import subprocess

import numpy as np
import pytest

from conftest import oracle, qb, ROOT

pytestmark = pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")

FORMATS = [qb.GGML_IQ4_XS, qb.GGML_Q6_K, qb.GGML_Q8_0, qb.GGML_Q4_K, qb.GGML_Q5_K]


def test_reference_test_ops_passes():
    """The reference's own op KAT/sweep suite (src/test_ops.c) on the checker build."""
    exe = os.path.join(ROOT, "oracle", "_ref", "test_ops")
    if not os.path.exists(exe):
        pytest.skip("test_ops not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:]
    assert "Failures: 0" in r.stdout


def test_reference_build_has_four_verify_slots():
    assert oracle.ref().ref_spec_max_b() == 4


@pytest.mark.parametrize("gtype", FORMATS)
def test_port_dequant_bit_exact(gtype):
    K, rows = 1024, 9
    raw = qb.synth_matrix(gtype, rows, K, seed=11 + gtype, d_sigma=0.02)
    port = oracle.port_dequant(raw, gtype, K)
    rb = qb.row_bytes(gtype, K)
    for r in range(rows):
        ref = oracle.ref_dequant_row(raw[r * rb:(r + 1) * rb], gtype, K)
        np.testing.assert_array_equal(port[r], ref)


@pytest.mark.parametrize("gtype", FORMATS)
@pytest.mark.parametrize("n", [1, 3, 8])
def test_port_gemv_matches_reference(gtype, n):
    K, rows = 2048, 64
    raw = qb.synth_matrix(gtype, rows, K, seed=5, d_sigma=0.01)
    x = qb.synth_normal(n * K, seed=7).reshape(n, K)
    ref = oracle.ref_gemv_batch(raw, gtype, K, rows, x)
    port = oracle.port_gemv(raw, gtype, K, x)
    err = np.linalg.norm(ref - port) / np.linalg.norm(port)
    assert err < 1e-6, err


def test_reference_batch_equals_single_token():
    """src/kernels.c:323-327 invariant (reference test_batch.c:44-57)."""
    K, rows = 1024, 48
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=9, d_sigma=0.02)
    x = qb.synth_normal(8 * K, seed=3).reshape(8, K)
    batch = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for t in range(8):
        single = oracle.ref_gemv(raw, qb.GGML_IQ4_XS, K, rows, x[t])
        np.testing.assert_array_equal(batch[t], single)


@pytest.mark.parametrize("name", ["rmsnorm", "l2norm", "silu", "sigmoid", "softplus", "softmax"])
@pytest.mark.parametrize("n", [1, 7, 8, 128, 1000, 5120])
def test_port_ops_match_reference(name, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)
    ref = oracle.ref_op(name, x, w if name == "rmsnorm" else None, 1e-6)
    port = {"rmsnorm": lambda: oracle.port_rmsnorm(x, w, 1e-6), "l2norm": lambda: oracle.port_l2norm(x, 1e-6),
            "silu": lambda: oracle.port_silu(x), "sigmoid": lambda: oracle.port_sigmoid(x),
            "softplus": lambda: oracle.port_softplus(x), "softmax": lambda: oracle.port_softmax(x)}[name]()
    np.testing.assert_allclose(ref, port, rtol=1e-4, atol=1e-6)


def test_reference_accepts_synthetic_gguf(tiny_gguf):
    m = oracle.RefModel(tiny_gguf, 128, 4)
    assert m.V == qb.TINY["vocab"] and m.E == qb.TINY["n_embd"] and m.n_layer == qb.TINY["n_layer"]
    assert [m.is_recurrent(i) for i in range(4)] == [True, True, True, False]
    m.forward(5, 0)
    lg = m.logits()
    assert np.isfinite(lg).all() and 0.2 < lg.std() < 5.0
    m.close()


def test_reference_spec_equals_sequential_greedy(tiny_gguf):
    """Lossless speculation (src/main.c:158-225, reference debug_spec2.c): the
    natural-acceptance stream equals plain greedy decoding."""
    prompt = np.arange(12, dtype=np.uint32) * 37 % qb.TINY["vocab"]
    a = oracle.RefModel(tiny_gguf, 256, 4)
    a.prefill(prompt, 1)
    toks_spec, _ = a.spec_generate(40, 3)
    b = oracle.RefModel(tiny_gguf, 256, 4)
    b.prefill(prompt, 0)
    toks_greedy = b.greedy_generate(40)
    np.testing.assert_array_equal(toks_spec, toks_greedy)
    a.close()
    b.close()


def test_reference_rollback_equals_replay(tiny_gguf):
    """batch -> rollback -> batch == sequential (reference debug_rollback.c:25-57)."""
    prompt = np.array([3, 1, 4, 1, 5], np.uint32)
    x = oracle.RefModel(tiny_gguf, 128, 4)
    y = oracle.RefModel(tiny_gguf, 128, 4)
    for i, t in enumerate(prompt):
        x.forward(int(t), i)
        y.forward(int(t), i)
    x.forward_batch([9, 2, 6], 5, 1)
    x.rollback_to(1)
    x.pos = 8
    y.forward(9, 5)
    y.forward(2, 6)
    x.forward_batch([5, 3, 5], 7, 1)
    for i, t in enumerate([5, 3]):
        y.forward(t, 7 + i)
        np.testing.assert_allclose(x.logits_b(3)[i], y.logits(), rtol=0, atol=1e-5)
    x.close()
    y.close()


def test_golden_fixtures_reproduce(tiny_gguf):
    """The committed goldens (tests/golden/make_golden.py) still come out of
    the reference on a freshly generated synthetic model."""
    path = os.path.join(ROOT, "tests", "golden", "tiny_spec.npz")
    g = np.load(path)
    m = oracle.RefModel(tiny_gguf, 256, 4)
    m.prefill(g["prompt"], 1)
    np.testing.assert_array_equal(np.float32(m.logits()[:64]), g["prefill_logits64"])
    toks, js = m.spec_generate(int(g["n_predict"]), 3, forced=g["forced"])
    np.testing.assert_array_equal(toks, g["tokens"])
    np.testing.assert_array_equal(js, g["accept"])
    m.close()


def _argmax_edge_rows(n=4099):
    """Rows where an ordering by float bits would differ from the reference's
    `>` scan: signed zeros, NaN after the maximum, NaN at entry 0, all NaN."""
    rows = []
    x = np.full(n, -1.0, np.float32); x[5] = -0.0; x[9] = 0.0; rows.append(x)          # -0 first: 5 wins
    x = np.full(n, -1.0, np.float32); x[5] = 0.0; x[9] = -0.0; rows.append(x)
    x = np.random.default_rng(3).standard_normal(n).astype(np.float32); x[17] = np.nan; rows.append(x)
    x = np.random.default_rng(4).standard_normal(n).astype(np.float32); x[0] = np.nan; rows.append(x)
    x = np.full(n, np.nan, np.float32); rows.append(x)
    x = np.full(n, np.nan, np.float32); x[n - 1] = -np.inf; rows.append(x)
    x = np.full(n, -np.inf, np.float32); rows.append(x)
    return rows


@pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")
def test_port_argmax_matches_reference_edge_cases():
    L = oracle.ref()
    for x in _argmax_edge_rows():
        want = L.ref_argmax(x.ctypes.data_as(oracle.C.POINTER(oracle.C.c_float)), x.size)
        assert oracle.port_argmax(x) == want
