"""GPU gemv_batch / gemv_rows_batch (include/qwen_b200.h -> include/kernels.h
API) against the compiled reference on the same seeded blocks.

Tolerance: the kernels multiply exact weight codes on the tensor cores with
activations split into fp16 hi+lo (~22 bits), accumulating in fp32, so
results carry fp32-level error; the bar is relative L2 <= 1e-5 per row set
(north_star allows 1e-2)."""
import numpy as np
import pytest

from conftest import oracle, qb

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")]

FORMATS = [qb.GGML_IQ4_XS, qb.GGML_Q6_K, qb.GGML_Q8_0, qb.GGML_Q4_K, qb.GGML_Q5_K]
RTOL = 1e-5


def rel(a, b):
    return float(np.linalg.norm(np.float64(a) - np.float64(b)) / max(np.linalg.norm(np.float64(b)), 1e-30))


@pytest.mark.parametrize("gtype", FORMATS)
@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8])
def test_gemv_batch_formats(gtype, n):
    K, rows = 2048, 333        # rows not a multiple of the 16-row tile
    raw = qb.synth_matrix(gtype, rows, K, seed=100 + gtype, d_sigma=0.01)
    x = qb.synth_normal(n * K, seed=n).reshape(n, K)
    t = qb.tensor(raw, gtype, K, rows)
    got = qb.gemv_batch(t, x)
    ref = oracle.ref_gemv_batch(raw, gtype, K, rows, x)
    for i in range(n):
        assert rel(got[i], ref[i]) < RTOL, (i, rel(got[i], ref[i]))


@pytest.mark.parametrize("gtype", [qb.GGML_IQ4_XS, qb.GGML_Q6_K])
def test_gemv_rows_subrange(gtype):
    K, rows = 1024, 200
    raw = qb.synth_matrix(gtype, rows, K, seed=3, d_sigma=0.01)
    x = qb.synth_normal(3 * K, seed=9).reshape(3, K)
    t = qb.tensor(raw, gtype, K, rows)
    got = qb.gemv_rows_batch(t, x, 37, 151)
    ref = oracle.ref_gemv_batch(raw, gtype, K, rows, x)
    assert np.all(got[:, :37] == 0) and np.all(got[:, 151:] == 0)
    assert rel(got[:, 37:151], ref[:, 37:151]) < RTOL


def test_gemv_wide_dynamic_range():
    """Activations spanning 1e-6 .. 1e4 exercise the per-256-block power-of-two scale."""
    K, rows = 4096, 64
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=1, d_sigma=0.01)
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((4, K)) * 10.0 ** rng.uniform(-6, 4, (4, K))).astype(np.float32)
    got = qb.gemv_batch(qb.tensor(raw, qb.GGML_IQ4_XS, K, rows), x)
    ref = oracle.port_gemv(raw, qb.GGML_IQ4_XS, K, x)
    assert rel(got, ref) < RTOL


def test_gemv_f32():
    K, rows = 300, 17
    W = qb.synth_normal(rows * K, seed=4)
    x = qb.synth_normal(2 * K, seed=5).reshape(2, K)
    raw = W.view(np.uint8)
    got = qb.gemv_batch(qb.tensor(raw, qb.GGML_F32, K, rows), x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_F32, K, rows, x)
    assert rel(got, ref) < 1e-6


def test_gemv_batch_equals_single_token():
    """Same invariant as the reference's test_batch.c:44-57, on the GPU path:
    every row of a batch equals the single-token result bit for bit."""
    K, rows = 2048, 96
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=21, d_sigma=0.01)
    t = qb.tensor(raw, qb.GGML_IQ4_XS, K, rows)
    x = qb.synth_normal(4 * K, seed=22).reshape(4, K)
    batch = qb.gemv_batch(t, x)
    for i in range(4):
        single = qb.gemv_batch(t, x[i:i + 1])
        np.testing.assert_array_equal(batch[i], single[0])


@pytest.mark.parametrize("n", [1, 2, 4])
def test_micro_config_c1(n):
    """W 17408x5120 IQ4_XS, d = |N|*0.02, x ~ N(0,1)."""
    K, rows = 5120, 17408
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=0, d_sigma=0.02)
    x = qb.synth_normal(n * K, seed=100 + n).reshape(n, K)
    got = qb.gemv_batch(qb.tensor(raw, qb.GGML_IQ4_XS, K, rows), x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for i in range(n):
        assert rel(got[i], ref[i]) < RTOL


def test_weight_cache_follows_new_contents_at_same_address():
    """The host API caches device copies by weight pointer (the reference hands
    out stable mmap pointers); new bytes at the same address must be picked up."""
    K, rows = 1024, 512
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=5, d_sigma=0.02)
    x = qb.synth_normal(2 * K, seed=6).reshape(2, K)
    t = qb.tensor(raw, qb.GGML_IQ4_XS, K, rows)
    first = qb.gemv_batch(t, x)
    raw[:] = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=7, d_sigma=0.02)   # same buffer, new weights
    second = qb.gemv_batch(t, x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for i in range(2):
        assert rel(second[i], ref[i]) < RTOL
    assert rel(first[0], second[0]) > 0.1


def test_sample_greedy_first_max_wins():
    x = np.zeros(248320, np.float32)
    x[[7, 100, 200000]] = 3.0
    assert qb.sample_greedy(x) == 7
    x[5] = -1.0
    x[248319] = 3.5
    assert qb.sample_greedy(x) == 248319
    rng = np.random.default_rng(1)
    y = rng.standard_normal(248320).astype(np.float32)
    assert qb.sample_greedy(y) == oracle.port_argmax(y)


def test_sample_greedy_nan_and_signed_zero():
    """The device argmax returns what the reference's `>` scan returns
    (src/model.c:746-756), NaN entries and -0 / +0 ties included."""
    from test_oracle import _argmax_edge_rows
    for x in _argmax_edge_rows(248320):
        assert qb.sample_greedy(x) == oracle.port_argmax(x)


@pytest.mark.parametrize("name", ["silu", "sigmoid", "softplus", "softmax", "rmsnorm", "l2norm"])
@pytest.mark.parametrize("n", [8, 13, 5120])
def test_ops_against_reference(name, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)
    got = qb.op(name, x, w if name == "rmsnorm" else None)
    ref = oracle.ref_op(name, x, w if name == "rmsnorm" else None)
    if name in ("silu", "sigmoid") and n % 8 == 0:
        np.testing.assert_array_equal(got, ref)   # polynomial exp restated exactly
    else:
        np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("n", [1, 3, 8, 11])
def test_gemv_multi_batch_one_dispatch(n):
    """gemv_multi_batch (include/kernels.h:32-34): every matrix reads the same x,
    the formats differ, n above QB_MAX_TOK runs in chunks.  Each output is
    bit-identical to a separate gemv_batch call (the reference's invariant,
    src/kernels.c:650-655) and matches the compiled reference."""
    K = 1024
    spec = [(qb.GGML_IQ4_XS, 300), (qb.GGML_Q6_K, 520), (qb.GGML_Q8_0, 64), (qb.GGML_IQ4_XS, 48)]
    raws = [qb.synth_matrix(g, r, K, seed=40 + i, d_sigma=0.01) for i, (g, r) in enumerate(spec)]
    ts = [qb.tensor(raw, g, K, r) for raw, (g, r) in zip(raws, spec)]
    x = qb.synth_normal(n * K, seed=77 + n).reshape(n, K)
    outs = qb.gemv_multi_batch(ts, x)
    for raw, (g, r), t, o in zip(raws, spec, ts, outs):
        np.testing.assert_array_equal(o, qb.gemv_batch(t, x))
        ref = oracle.ref_gemv_batch(raw, g, K, r, x)
        assert rel(o, ref) < RTOL


def test_gemv_multi_single_vector_and_limits():
    K = 512
    raws = [qb.synth_matrix(qb.GGML_IQ4_XS, 64 + 32 * i, K, seed=i, d_sigma=0.01) for i in range(3)]
    ts = [qb.tensor(raw, qb.GGML_IQ4_XS, K, 64 + 32 * i) for i, raw in enumerate(raws)]
    x = qb.synth_normal(K, seed=5)
    for o, t in zip(qb.gemv_multi(ts, x), ts):
        np.testing.assert_array_equal(o, qb.gemv_batch(t, x[None])[0])
    with pytest.raises(RuntimeError, match="at most 8"):
        qb.gemv_multi(ts * 3, x)


@pytest.mark.parametrize("n", [9, 12, 16, 17, 32, 33, 64])
def test_gemv_batch_iq4_wide_tcgen05(n):
    """More than 8 vectors: IQ4_XS runs up to 32 per weight sweep on the tcgen05
    kernel (qb_qmv_tcw: sub-block scales folded into two int8 weight planes, one
    accumulator per plane and digit).  The reference's gemv_batch runs them 8 at a time,
    each chunk bit-identical to a single-vector sweep (src/test_batch.c:44-57),
    so the bar is the same as for the mma.sync path."""
    K, rows = 2048, 333        # rows not a multiple of the 128-row tile
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=200 + n, d_sigma=0.01)
    x = qb.synth_normal(n * K, seed=300 + n).reshape(n, K)
    t = qb.tensor(raw, qb.GGML_IQ4_XS, K, rows)
    got = qb.gemv_batch(t, x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for i in range(n):
        assert rel(got[i], ref[i]) < RTOL, (i, rel(got[i], ref[i]))


@pytest.mark.parametrize("n", [16, 32])
def test_gemv_batch_iq4_wide_micro_shape(n):
    """The C1 micro matrix (17408 x 5120) at the prefill / multi-stream widths."""
    K, rows = 5120, 17408
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=0, d_sigma=0.02)
    x = qb.synth_normal(n * K, seed=n).reshape(n, K)
    got = qb.gemv_batch(qb.tensor(raw, qb.GGML_IQ4_XS, K, rows), x)
    ref = oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x)
    for i in range(n):
        assert rel(got[i], ref[i]) < RTOL, (i, rel(got[i], ref[i]))


def test_gemv_iq4_wide_rows_do_not_depend_on_width():
    """The 32-token and the 16-token instantiation of qb_qmv_tcw give every
    vector the same bits (the per-(tile, block) integer sums are exact and the
    tile split over CTAs depends on the matrix only), at any width 9..32."""
    K, rows = 2048, 333
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=41, d_sigma=0.01)
    t = qb.tensor(raw, qb.GGML_IQ4_XS, K, rows)
    x = qb.synth_normal(32 * K, seed=42).reshape(32, K)
    full = qb.gemv_batch(t, x)                  # one 32-token sweep
    for n in (9, 16, 17, 24):
        np.testing.assert_array_equal(qb.gemv_batch(t, x[:n]), full[:n], err_msg=f"n = {n}")


def test_gemv_multi_batch_iq4_wide():
    """gemv_multi_batch with 20 vectors over IQ4_XS matrices: the 32-token
    kernel, each matrix bit-identical to its own gemv_batch."""
    K, n = 1024, 20
    specs = [(300, 1), (520, 2), (64, 3)]
    raws = [qb.synth_matrix(qb.GGML_IQ4_XS, r, K, seed=s, d_sigma=0.01) for r, s in specs]
    ts = [qb.tensor(raw, qb.GGML_IQ4_XS, K, r) for raw, (r, _) in zip(raws, specs)]
    x = qb.synth_normal(n * K, seed=9).reshape(n, K)
    outs = qb.gemv_multi_batch(ts, x)
    for raw, (r, _), t, o in zip(raws, specs, ts, outs):
        np.testing.assert_array_equal(o, qb.gemv_batch(t, x))
        assert rel(o, oracle.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, r, x)) < RTOL
