"""Pin the C restatement (oracle/g4_oracle.c) to the reference.

Against the committed golden fixtures (generated from the reference build by
tests/golden/make_golden.py) always, and against the live reference build
(oracle/_ref/libg4ref.so) when it is present.  CPU only.
"""
import numpy as np
import pytest

from _tol import assert_close, dense_term_scale, kquant_term_scale

Q4, Q5, Q6, BF16, F16, F32 = 12, 13, 14, 30, 1, 0


def test_q8K_bit_exact(orc, golden):
    for x, y in zip(golden["q8_x"], golden["q8_out"]):
        assert (orc.quantize_q8K(x) == y).all()


@pytest.mark.parametrize("name,t", [("q4", Q4), ("q5", Q5)])
def test_kquant_block_sums_exact(orc, golden, name, t):
    ss, sm = orc.block_sums(golden[name + "_w"], t, 512, 16, golden[name + "_q8"])
    assert (ss == golden[name + "_ss"]).all()
    assert (sm == golden[name + "_sm"]).all()


@pytest.mark.parametrize("name,t", [("q4", Q4), ("q5", Q5)])
def test_kquant_dot(orc, golden, name, t):
    w, x, q8 = golden[name + "_w"], golden[name + "_x"], golden[name + "_q8"]
    o = orc.mm(x, w, 512, 16, t)
    # the restatement follows the generic build's order exactly
    assert (o == golden[name + "_dot_generic"]).all()
    scale = kquant_term_scale(w, t, 512, q8, golden[name + "_ss"], golden[name + "_sm"])
    assert_close(o, golden[name + "_dot"], scale, what=name + " vs AVX2")
    assert_close(o, golden[name + "_mm"], scale, what=name + " mm")


def test_dequant_exact(orc, golden):
    for name, t in (("q4", Q4), ("q5", Q5), ("q6", Q6)):
        assert (orc.dequant(golden[name + "_w"][0].copy(), t, 2) == golden[name + "_deq0"]).all(), name


def test_q6K_mm_exact(orc, golden):
    assert (orc.mm(golden["q6_x"], golden["q6_w"], 512, 8, Q6) == golden["q6_mm"]).all()


def test_dense_mm(orc, golden):
    x = golden["dense_x"]
    for name, t in (("bf16", BF16), ("f16", F16)):
        assert (orc.mm(x, golden[name + "_w"], 384, 8, t) == golden[name + "_mm"]).all(), name
    w = golden["f32_w"]
    assert_close(orc.mm(x, w, 384, 8, F32), golden["f32_mm"], dense_term_scale(w, x), what="f32 vs OpenBLAS")


def test_rope_exact(orc, golden):
    v, ff = golden["rope_in"], golden["rope_ff"]
    for i, p in enumerate(golden["rope_pos"]):
        assert (orc.rope(v, 8, 64, 64, int(p), 1e4) == golden["rope_swa"][i]).all()
        assert (orc.rope(v, 8, 64, 64, int(p), 1e6, 1.0, ff) == golden["rope_full"][i]).all()
        assert (orc.rope(v, 8, 64, 32, int(p), 1e4) == golden["rope_partial"][i]).all()


def test_gelu_exact(orc, golden):
    got = np.array([orc.gelu(float(a)) for a in golden["gelu_in"]], np.float32)
    assert (got == golden["gelu_out"]).all()


def test_argmax_first_index(orc):
    v = np.array([1.0, 3.0, -2.0, 3.0, 3.0], np.float32)
    assert orc.argmax_first(v) == 1


def test_attention_matches_softmax_definition(orc, golden):
    # the restated attention uses the reference softmax order; check one head by hand
    rng = np.random.default_rng(5)
    hd, nwin, stride = 64, 37, 1024
    q = rng.standard_normal(2 * hd).astype(np.float32)
    k = rng.standard_normal(nwin * stride).astype(np.float32)
    v = rng.standard_normal(nwin * stride).astype(np.float32)
    out = orc.attention(q, k, v, nwin, stride, 2, 1, hd)
    K = k.reshape(nwin, stride)[:, :hd].astype(np.float64)
    V = v.reshape(nwin, stride)[:, :hd].astype(np.float64)
    for h in range(2):
        s = K @ q[h * hd:(h + 1) * hd]
        p = np.exp(s - s.max())
        p /= p.sum()
        np.testing.assert_allclose(out[h * hd:(h + 1) * hd], p @ V, rtol=2e-5, atol=2e-6)


def agree_prefix(a, b):
    n = min(len(a), len(b))
    d = np.flatnonzero(np.asarray(a[:n]) != np.asarray(b[:n]))
    return int(d[0]) if d.size else n


def test_tiny_fp32_path_model(g4, orc, golden):
    """TINY_F has no Q8_K activation rounding: the restated forward must match
    the reference to float summation order and its greedy stream exactly."""
    m = g4.synth.make_model(g4.synth.TINY_F, seed=3)
    om = orc.model(m.desc(), 64)
    prompt = golden["tiny_prompt"]
    for pos in range(8):
        om.forward(int(prompt[pos]), pos, 0 if pos < 7 else 1)
    assert_close(om.logits(), golden["tinyf_logits_p7"], rel=5e-5, what="tinyf logits")
    assert_close(om.hidden(), golden["tinyf_hidden_p7"], rel=5e-5, what="tinyf hidden")
    k, v = om.kv(0, 1, 128)
    assert_close(k, golden["tinyf_k_l0_p1"], rel=1e-5, what="K layer 0 pos 1")
    assert_close(v, golden["tinyf_v_l0_p1"], rel=1e-5, what="V layer 0 pos 1")
    k, v = om.kv(5, 5, 256)
    assert_close(k, golden["tinyf_k_l5_p5"], rel=1e-5, what="K layer 5 pos 5")
    assert_close(v, golden["tinyf_v_l5_p5"], rel=1e-5, what="V layer 5 pos 5")
    om.close()
    assert (orc.model(m.desc(), 64).generate_greedy(prompt, 32) == golden["tinyf_greedy"]).all()


def test_tiny_q4km_model(g4, orc, golden):
    """The Q4_K_M mix re-rounds activations to Q8_K before every integer
    GEMV, so last-ulp differences flip some int8 values and grow to ~1e-2 in
    the logits; the reference's own AVX2 and generic-dot builds differ that
    much, and their greedy streams part after a few tokens.  Checked: the
    logits stay within that spread (token-exact streams are checked on the
    fp32-path model above)."""
    m = g4.synth.make_model(g4.synth.TINY, seed=3)
    om = orc.model(m.desc(), 64)
    prompt = golden["tiny_prompt"]
    for pos in range(8):
        om.forward(int(prompt[pos]), pos, 0 if pos < 7 else 1)
    assert_close(om.logits(), golden["tiny_logits_p7"], rel=0.1, what="tiny logits")
    om.close()


def test_live_reference_kernels(orc, ref):
    rng = np.random.default_rng(11)
    import g4b200
    for trial in range(3):
        x = rng.standard_normal(2560).astype(np.float32) * np.float32(10 ** rng.uniform(-2, 2))
        assert (orc.quantize_q8K(x) == ref.quantize_q8K(x)).all()
    for t in (Q4, Q5):
        w = g4b200.synth.rand_blocks(rng, t, 32, 2560, 1e-3, 2e-2)
        x = rng.standard_normal(2560).astype(np.float32)
        q8 = ref.quantize_q8K(x)
        gen = np.array([ref.vec_dot(t, 2560, w[r], q8, generic=True) for r in range(32)], np.float32)
        assert (orc.mm(x, w, 2560, 32, t) == gen).all()
    w6 = g4b200.synth.rand_blocks(rng, Q6, 16, 2560, 1e-3, 2e-2)
    x6 = rng.standard_normal(2560).astype(np.float32)
    assert (orc.mm(x6, w6, 2560, 16, Q6) == ref.mm(x6, w6, 2560, 16, Q6)).all()
