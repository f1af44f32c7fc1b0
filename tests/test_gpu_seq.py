"""Multi-sequence speculative decode (qb_seq_init / qb_seq_prefill /
qb_seq_generate): S sequences on one set of weights advance together, the
verify of all of them in one weight sweep per GEMV chunk of 8 rows.

Bar: every sequence emits exactly the tokens and accept lengths that it emits
alone (qb_spec_generate on a fresh model) and that the compiled reference
engine emits for it (src/main.c:158-225), for widths up to the 32-row limit
(8 sequences x 4 verify tokens), over mixed quantisation formats, with forced
and with natural acceptance, and across two generate calls.
"""
import numpy as np
import pytest

from conftest import oracle, qb

pytestmark = pytest.mark.gpu


def forced_schedule(n=4096, seed=0):
    return np.random.default_rng(seed).integers(0, 4, n).astype(np.uint32)


def prompts(n_seq, vocab, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, int(rng.integers(5, 40))).astype(np.uint32) for _ in range(n_seq)]


def alone(path, n_ctx, p, n_cycles, forced, k=3, calls=1):
    m = qb.Model(path, n_ctx)
    m.prefill(p, 1)
    toks, js = [], []
    for _ in range(calls):
        t, j = m.spec_generate(10 ** 6, k, forced=forced, max_cycles=n_cycles)
        toks.append(t)
        js.append(j)
    m.close()
    return np.concatenate(toks), np.concatenate(js)


@pytest.mark.parametrize("n_seq,k", [(3, 3), (8, 3), (5, 2), (1, 3)])
def test_sequences_match_single_runs(tiny_mixed_gguf, n_seq, k):
    ps = prompts(n_seq, 2048, seed=n_seq * 10 + k)
    forced = forced_schedule(seed=k)
    n_cycles = 12
    m = qb.Model(tiny_mixed_gguf, 256)
    m.seq_init(n_seq)
    for s, p in enumerate(ps):
        m.seq_prefill(s, p)
    toks, js = m.seq_generate(n_cycles, k, forced=forced)
    m.close()
    for s, p in enumerate(ps):
        t1, j1 = alone(tiny_mixed_gguf, 256, p, n_cycles, forced, k)
        np.testing.assert_array_equal(js[s], j1, err_msg=f"sequence {s}")
        np.testing.assert_array_equal(toks[s], t1, err_msg=f"sequence {s}")


@pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")
def test_sequences_match_reference(tiny_gguf):
    n_seq, n_cycles = 4, 10
    ps = prompts(n_seq, 2048, seed=77)
    forced = forced_schedule(seed=5)
    m = qb.Model(tiny_gguf, 256)
    m.seq_init(n_seq)
    for s, p in enumerate(ps):
        m.seq_prefill(s, p)
    toks, js = m.seq_generate(n_cycles, 3, forced=forced)
    m.close()
    for s, p in enumerate(ps):
        r = oracle.RefModel(tiny_gguf, 256, 0)
        r.prefill(p, 1)
        rt, rj = r.spec_generate(10 ** 6, 3, forced=forced, max_cycles=n_cycles)
        r.close()
        np.testing.assert_array_equal(js[s], rj, err_msg=f"sequence {s}")
        np.testing.assert_array_equal(toks[s], rt, err_msg=f"sequence {s}")


def test_natural_acceptance_and_two_calls(tiny_gguf):
    """No forced schedule (acceptance by the drafts' own argmax), and the state
    carried from one generate call into the next."""
    n_seq, n_cycles = 6, 8
    ps = prompts(n_seq, 2048, seed=3)
    m = qb.Model(tiny_gguf, 256)
    m.seq_init(n_seq)
    for s, p in enumerate(ps):
        m.seq_prefill(s, p)
    t1, j1 = m.seq_generate(n_cycles, 3)
    t2, j2 = m.seq_generate(n_cycles, 3)
    m.close()
    for s, p in enumerate(ps):
        want_t, want_j = alone(tiny_gguf, 256, p, n_cycles, None, 3, calls=2)
        np.testing.assert_array_equal(np.concatenate([j1[s], j2[s]]), want_j, err_msg=f"sequence {s}")
        np.testing.assert_array_equal(np.concatenate([t1[s], t2[s]]), want_t, err_msg=f"sequence {s}")


def test_full_width_eight_sequences(wide_gguf):
    """Full-width kernels (hidden 5120, FFN 17408, vocab 248320) at the 32-row
    limit: 8 sequences x 4 verify tokens, 4 GEMV chunks per weight sweep."""
    n_seq, n_cycles = 8, 6
    ps = prompts(n_seq, qb.WIDE4["vocab"], seed=8)
    forced = forced_schedule(seed=8)
    m = qb.Model(wide_gguf, 128)
    m.seq_init(n_seq)
    for s, p in enumerate(ps):
        m.seq_prefill(s, p)
    toks, js = m.seq_generate(n_cycles, 3, forced=forced)
    m.close()
    for s, p in enumerate(ps):
        t1, j1 = alone(wide_gguf, 128, p, n_cycles, forced, 3)
        np.testing.assert_array_equal(js[s], j1, err_msg=f"sequence {s}")
        np.testing.assert_array_equal(toks[s], t1, err_msg=f"sequence {s}")


def test_seq_limits(tiny_gguf):
    m = qb.Model(tiny_gguf, 64)
    with pytest.raises(RuntimeError):
        m.seq_init(9)                        # at most 8 sequences
    m.seq_init(8)
    with pytest.raises(RuntimeError):
        m.seq_generate(2, 3)                 # no prefill yet
    for s in range(8):
        m.seq_prefill(s, np.arange(4, dtype=np.uint32))
    toks, js = m.seq_generate(100, 3)        # stops before any sequence passes n_ctx = 64
    assert all(len(j) < 100 for j in js)
    m.close()
