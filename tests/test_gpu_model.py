"""GPU model path (model_forward*, rollback, MTP, device spec loop) against
the compiled reference engine on the same seeded synthetic GGUF.

Bars (north_star): tokens and accept lengths bit-exact; logits and hidden
states within 1e-2 relative L2 -- here held to 1e-4."""
import numpy as np
import pytest

from conftest import oracle, qb

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.available(), reason="oracle/_ref not built")]

RTOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm(np.float64(a) - np.float64(b)) / max(np.linalg.norm(np.float64(b)), 1e-30))


def prompt_for(V, n, seed=0):
    return np.random.default_rng(seed).integers(0, V, n).astype(np.uint32)


@pytest.fixture(params=["tiny", "tiny_mixed"])
def gguf(request, tiny_gguf, tiny_mixed_gguf):
    return {"tiny": tiny_gguf, "tiny_mixed": tiny_mixed_gguf}[request.param]


def test_forward_sequence(gguf):
    g, r = qb.Model(gguf, 64), oracle.RefModel(gguf, 64, 4)
    for pos, tok in enumerate(prompt_for(r.V, 10)):
        g.forward(int(tok), pos)
        r.forward(int(tok), pos)
        assert rel(g.logits(), r.logits()) < RTOL
        assert rel(g.x(), r.x()) < RTOL
        assert int(np.argmax(g.logits())) == r.logits().argmax()
    g.close(); r.close()


def test_forward_batch_and_rollback(gguf):
    g, r = qb.Model(gguf, 64), oracle.RefModel(gguf, 64, 4)
    p = prompt_for(r.V, 8, 1)
    g.forward_batch(p, 0, 0)
    r.forward_batch(p, 0, 0)
    assert rel(g.logits_b(8), r.logits_b(8)) < RTOL
    assert rel(g.h_save(8), r.h_save(8)) < RTOL
    for j, cand in [(1, [11, 22, 33, 44]), (0, [5, 6, 7, 8]), (2, [9, 10, 11, 12]), (3, [1, 2, 3, 4])]:
        P = r.pos - 1
        g.forward_batch(cand, P + 1, 1)
        r.forward_batch(cand, P + 1, 1)
        assert rel(g.logits_b(4), r.logits_b(4)) < RTOL
        if j < 3:
            g.rollback_to(j)
            r.rollback_to(j)
        g.pos = r.pos = P + j + 2
        for il in range(r.n_layer):
            if r.is_recurrent(il):
                n_ssm = qb.TINY["ssm_v_heads"] * 128 * 128
                assert rel(g.read_state(il, 1, n_ssm), r.state(il, 1, n_ssm)) < RTOL
                n_conv = (2 * qb.TINY["ssm_groups"] * 128 + qb.TINY["ssm_v_heads"] * 128) * 4
                assert rel(g.read_state(il, 0, n_conv), r.state(il, 0, n_conv)) < RTOL
    g.close(); r.close()


def test_mtp_forward(gguf):
    g, r = qb.Model(gguf, 64), oracle.RefModel(gguf, 64, 4)
    p = prompt_for(r.V, 6, 2)
    g.prefill(p, 1)
    r.prefill(p, 1)
    assert rel(g.mtp_h(), r.mtp_h()) < RTOL
    for s in range(3):
        tok = 17 + s
        g.mtp_forward(tok, 6 + s, 1)
        r.mtp_forward(tok, 6 + s, 1)
        assert rel(g.logits(), r.logits()) < RTOL
        assert rel(g.mtp_h(), r.mtp_h()) < RTOL
    g.close(); r.close()


@pytest.mark.parametrize("name", ["tiny_spec", "tiny_mixed_spec"])
def test_spec_generate_matches_golden(name, tiny_gguf, tiny_mixed_gguf):
    import os
    from conftest import ROOT
    gold = np.load(os.path.join(ROOT, "tests", "golden", f"{name}.npz"))
    path = tiny_gguf if name == "tiny_spec" else tiny_mixed_gguf
    g = qb.Model(path, 256)
    g.prefill(gold["prompt"], 1)
    assert rel(g.logits()[:64], gold["prefill_logits64"]) < RTOL
    toks, js = g.spec_generate(int(gold["n_predict"]), 3, forced=gold["forced"])
    np.testing.assert_array_equal(toks, gold["tokens"])
    np.testing.assert_array_equal(js, gold["accept"])
    g.close()


def test_spec_generate_matches_reference_live(gguf):
    p = prompt_for(2048, 20, 5)
    forced = np.random.default_rng(5).integers(0, 4, 50).astype(np.uint32)
    g, r = qb.Model(gguf, 256), oracle.RefModel(gguf, 256, 4)
    g.prefill(p, 1)
    r.prefill(p, 1)
    gt, gj = g.spec_generate(90, 3, forced=forced)
    rt, rj = r.spec_generate(90, 3, forced=forced)
    np.testing.assert_array_equal(gt, rt)
    np.testing.assert_array_equal(gj, rj)
    assert g.pos == r.pos
    assert rel(g.logits(), r.logits()) < RTOL
    g.close(); r.close()


def test_natural_spec_equals_greedy(gguf):
    """Lossless speculation on the device: natural acceptance == greedy."""
    p = prompt_for(2048, 16, 6)
    a, b = qb.Model(gguf, 256), qb.Model(gguf, 256)
    a.prefill(p, 1)
    b.prefill(p, 0)
    sa, _ = a.spec_generate(48, 3)
    sb = b.greedy_generate(48)
    np.testing.assert_array_equal(sa, sb)
    r = oracle.RefModel(gguf, 256, 4)
    r.prefill(p, 0)
    np.testing.assert_array_equal(sb, r.greedy_generate(48))
    a.close(); b.close(); r.close()


def test_wide_model_spec(wide_gguf):
    """Full layer widths (5120 / 17408 / 248320, 24q/4kv, 16k/48v heads), 4 layers."""
    p = prompt_for(qb.WIDE4["vocab"], 12, 7)
    forced = np.array([3, 0, 2, 1, 3, 3, 0, 1], np.uint32)
    g, r = qb.Model(wide_gguf, 128), oracle.RefModel(wide_gguf, 128, 0)
    g.prefill(p, 1)
    r.prefill(p, 1)
    assert rel(g.logits(), r.logits()) < RTOL
    gt, gj = g.spec_generate(24, 3, forced=forced)
    rt, rj = r.spec_generate(24, 3, forced=forced)
    np.testing.assert_array_equal(gt, rt)
    np.testing.assert_array_equal(gj, rj)
    assert rel(g.logits(), r.logits()) < RTOL
    g.close(); r.close()


def test_single_layers_against_reference(gguf):
    """attention_layer / gdn_layer (include/model.h:121-122) one token at a time on
    m->x, layer by layer, against the reference's own layer functions: the hidden
    state after every layer and the recurrent state after the DeltaNet layers."""
    g, r = qb.Model(gguf, 64), oracle.RefModel(gguf, 64, 4)
    rng = np.random.default_rng(8)
    for pos in range(3):
        x = rng.standard_normal(g.E).astype(np.float32)
        g.set_x(x)
        r.set_x(x)
        for il in range(r.n_layer):
            g.layer(il, pos)
            r.layer(il, pos)
            assert rel(g.x(), r.x()) < RTOL, (pos, il, rel(g.x(), r.x()))
            if r.is_recurrent(il):
                n_ssm = qb.TINY["ssm_v_heads"] * 128 * 128
                assert rel(g.read_state(il, 1, n_ssm), r.state(il, 1, n_ssm)) < RTOL
    g.close(); r.close()
