"""Device sampling (sampler_init / sampler_sample, qb_sample_generate) against
the compiled reference sampler (src/sampler.c) on seeded streams.

Bar: the same tokens, the same generator state after every draw, and the
same penalised logits (the reference edits them in place), bit for bit."""
import numpy as np
import pytest

from conftest import oracle, qb

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")]

# (temp, top_p, top_k, repeat_penalty, seed): the CLI defaults, wide top-k, a
# tight nucleus, the top_k == 0 default (40), heavy penalties, and both greedy
# branches of src/sampler.c:78-88
PARAMS = [(0.7, 0.9, 40, 1.1, 42), (1.0, 1.0, 256, 1.0, 7), (1.3, 0.5, 100, 1.3, 0), (0.8, 0.95, 0, 1.05, 99),
          (0.0, 0.9, 40, 1.1, 5), (0.9, 0.9, 1, 1.2, 6), (0.6, 0.99, 300, 2.0, 123456789)]


@pytest.mark.parametrize("params", PARAMS)
@pytest.mark.parametrize("V", [2048, 248320])
def test_sampler_stream_matches_reference(params, V):
    rng = np.random.default_rng(hash(params) % 2**32 + V)
    ours, ref = qb.Sampler(*params), oracle.RefSampler(*params)
    history = list(rng.integers(0, V, 70).astype(np.uint32))   # longer than the 64-token window
    history += history[-5:]                                       # repeats: penalised once per occurrence
    for step in range(40):
        logits = (rng.standard_normal(V) * 3.0).astype(np.float32)
        a, b = logits.copy(), logits.copy()
        ta = ours.sample(a, np.array(history, np.uint32))
        tb = ref.sample(b, np.array(history, np.uint32))
        assert ta == tb, (step, ta, tb)
        assert ours.rng_state == ref.rng_state, step
        np.testing.assert_array_equal(a, b)
        history.append(ta)
    ours.close()
    ref.close()


def test_sampler_empty_history_and_small_vocab():
    ours, ref = qb.Sampler(0.9, 0.9, 40, 1.1, 3), oracle.RefSampler(0.9, 0.9, 40, 1.1, 3)
    rng = np.random.default_rng(11)
    for V in (7, 40, 300):   # top_k clamps to the vocabulary
        for _ in range(10):
            x = rng.standard_normal(V).astype(np.float32)
            assert ours.sample(x.copy(), []) == ref.sample(x.copy(), [])
            assert ours.rng_state == ref.rng_state


@pytest.fixture(params=["tiny", "tiny_mixed"])
def gguf(request, tiny_gguf, tiny_mixed_gguf):
    return {"tiny": tiny_gguf, "tiny_mixed": tiny_mixed_gguf}[request.param]


@pytest.mark.parametrize("params", [(0.7, 0.9, 40, 1.1, 42), (1.2, 0.8, 200, 1.3, 17)])
def test_sample_generate_matches_reference_loop(gguf, params):
    """qb_sample_generate (forward + draw on the device per token) against the
    reference's src/main.c:232-248 loop with its own sampler."""
    prompt = np.random.default_rng(3).integers(0, 2048, 12).astype(np.uint32)
    g, r = qb.Model(gguf, 256), oracle.RefModel(gguf, 256, 4)
    g.prefill(prompt, 0)
    r.prefill(prompt, 0)
    sg, sr = qb.Sampler(*params), oracle.RefSampler(*params)
    got = g.sample_generate(sg, 60, prompt)
    want = r.sample_generate(sr, 60, prompt)
    np.testing.assert_array_equal(got, want)
    assert sg.rng_state == sr.rng_state
    assert g.pos == r.pos
    g.close(); r.close(); sg.close(); sr.close()
