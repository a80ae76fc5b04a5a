"""Batch invariance of the decode engine: a sequence decoded in a batch of B
(B >= the tensor-core threshold: Q4_K/Q5_K/Q6_K projections and the LM head
on tcgen05 GEMMs, dense matrices on the multi-sequence GEMV) gives exactly the
result of decoding it alone (streaming GEMVs).

The reference decodes one sequence at a time (forward, gemma4-4b/cpu-blas/
main.c:1838-2029), so a batch of independent sequences must reproduce each
sequence's own stream.  Every path computes each super-block's contribution
exactly (integer block sums of Q4_K/Q5_K; exact fixed-point Q6_K block dots)
and sums a row's blocks in one canonical order, the attention splits its
window at fixed row counts, and the norms use one summation order, so the
comparison is bit for bit: hidden states, K/V rows and greedy tokens, on the
fp32-path model and on the Q4_K_M mix alike.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tinyf(g4):
    return g4.synth.make_model(g4.synth.TINY_F, seed=3)


@pytest.fixture(scope="module")
def tiny(g4):
    return g4.synth.make_model(g4.synth.TINY, seed=3)


@pytest.fixture(scope="module")
def tinyq5(g4):
    return g4.synth.make_model(g4.synth.TINY_Q5, seed=8)


def batched_stream(g4, model, prompts, steps, max_seq=48):
    B = prompts.shape[0]
    eb = g4.Engine(model, 0, max_seq=max_seq, max_batch=B)
    toks = prompts[:, 0].copy()
    npre = prompts.shape[1]
    outs, hid = [], None
    for pos in range(npre - 1 + steps):
        lm = 0 if pos < npre - 1 else 1
        nxt = eb.decode_batch(toks, pos, lm)
        if pos == npre - 1:
            hid = np.stack([eb.hidden(b) for b in range(B)])
        toks = prompts[:, pos + 1].copy() if pos < npre - 1 else nxt
        if lm:
            outs.append(nxt.copy())
    eb.close()
    return np.stack(outs, 1), hid


def single(g4, model, prompt, steps, max_seq=48):
    es = g4.Engine(model, 0, max_seq=max_seq, max_batch=1)
    got = es.generate_greedy(prompt, steps)
    es.close()
    e2 = g4.Engine(model, 0, max_seq=max_seq, max_batch=1)
    for pos in range(len(prompt)):
        e2.forward(int(prompt[pos]), pos, 0 if pos < len(prompt) - 1 else 1)
    h = e2.hidden(0)
    e2.close()
    return got, h


@pytest.mark.parametrize("which,B", [("tiny", 2), ("tiny", 8), ("tinyf", 9), ("tinyf", 16), ("tiny", 15), ("tiny", 24),
                                     ("tinyq5", 17)])
def test_batched_streams_identical_to_single(g4, gpu, request, which, B):
    model = request.getfixturevalue(which)
    rng = np.random.default_rng(100 + B)
    prompts = rng.integers(0, 4096, (B, 4)).astype(np.int32)
    outs, hid = batched_stream(g4, model, prompts, 10)
    for b in range(B):
        got, h = single(g4, model, prompts[b], 10)
        assert (hid[b] == h).all(), (b, float(np.abs(hid[b] - h).max()))
        assert (got == outs[b]).all(), (b, got, outs[b])


def _first_step(g4, model, toks, max_seq=16):
    """Batched step at position 0: next tokens, layer-0 K/V rows and hidden states per sequence."""
    B = len(toks)
    eb = g4.Engine(model, 0, max_seq=max_seq, max_batch=B)
    nxt = eb.decode_batch(np.asarray(toks, np.int32), 0, 1)
    kvd = model.shape.n_kv_heads * model.shape.head_dim_swa  # layer 0 is a sliding-window layer
    kv = [eb.kv(0, 0, kvd, b) for b in range(B)]
    hid = [eb.hidden(b) for b in range(B)]
    eb.close()
    return nxt, kv, hid


@pytest.mark.parametrize("B", [64, 65])
def test_tc_batched_64_sequences_bitwise(g4, gpu, tiny, B):
    """A full group of 64 (the residual/norm launches write the GEMM operands
    themselves) and 64 + 1 (a second group; separate operand launches), on
    the Q4_K_M mix: every sequence bit-identical to decoding it alone."""
    toks = np.random.default_rng(11).integers(0, 4096, B)
    nxt, kv, hid = _first_step(g4, tiny, toks)
    es = g4.Engine(tiny, 0, max_seq=16, max_batch=1)
    kvd = tiny.shape.n_kv_heads * tiny.shape.head_dim_swa
    try:
        for b in range(B):
            n1 = es.forward(int(toks[b]), 0, 1)
            k1, v1 = es.kv(0, 0, kvd)
            h1 = es.hidden(0)
            assert (kv[b][0] == k1).all() and (kv[b][1] == v1).all(), b
            assert (hid[b] == h1).all(), (b, float(np.abs(hid[b] - h1).max()))
            assert nxt[b] == n1, (b, nxt[b], n1)
    finally:
        es.close()


def test_e4b_batch_invariance_at_long_context(g4, gpu):
    """The benchmarked shape (E4B, Q4_K_M) at context 516: 40 sequences
    (eight different caches, every sequence its own token) decoded in one
    batched step equal each sequence decoded alone from the same cache:
    hidden state, K/V rows of every KV layer and the greedy token, bit for
    bit.  At 40 sequences a sliding-window layer has more 64-row splits than
    two CTAs per SM, so its CTAs take several consecutive splits each, while
    the single-sequence decode gives every split its own CTA."""
    S = g4.synth
    shape = S.E4B
    m = S.make_model(shape, seed=3)
    B, ctx, ncache = 40, 516, 8
    rng = np.random.default_rng(17)
    caches = []
    for b in range(ncache):
        per = []
        for l in range(24):
            hd = shape.head_dim_swa if S.is_swa(shape, l) else shape.head_dim_full
            n = shape.n_kv_heads * hd
            per.append(((rng.standard_normal((ctx, n)) * 0.25).astype(np.float32),
                        rng.standard_normal((ctx, n)).astype(np.float32)))
        caches.append(per)
    toks = rng.integers(0, shape.vocab_size, B).astype(np.int32)
    eb = g4.Engine(m, 0, max_seq=ctx + 4, max_batch=B)
    try:
        for b in range(B):
            for l in range(24):
                eb.set_kv(l, 0, caches[b % ncache][l][0], caches[b % ncache][l][1], b=b)
        nxt = eb.decode_batch(toks, ctx, 1)
        hid = [eb.hidden(b) for b in range(B)]
        kvs = [[eb.kv(l, ctx, shape.n_kv_heads * (shape.head_dim_swa if S.is_swa(shape, l) else shape.head_dim_full), b)
                for l in (0, 5, 22, 23)] for b in range(B)]
    finally:
        eb.close()
    es = g4.Engine(m, 0, max_seq=ctx + 4, max_batch=1)
    try:
        for b in range(B):
            for l in range(24):
                es.set_kv(l, 0, caches[b % ncache][l][0], caches[b % ncache][l][1])
            n1 = es.forward(int(toks[b]), ctx, 1)
            assert (es.hidden(0) == hid[b]).all(), (b, float(np.abs(es.hidden(0) - hid[b]).max()))
            for i, l in enumerate((0, 5, 22, 23)):
                k1, v1 = es.kv(l, ctx, kvs[b][i][0].size)
                assert (k1 == kvs[b][i][0]).all() and (v1 == kvs[b][i][1]).all(), (b, l)
            assert n1 == nxt[b], (b, n1, nxt[b])
    finally:
        es.close()


@pytest.mark.parametrize("which", ["tiny", "tinyq5"])
def test_batch1_gemv_kernels_identical_in_engine(g4, gpu, request, which):
    """Batch-1 decode (fused residual/norm prologues, Q+K and gate/up launches) on the row-owner GEMV
    and on the tiled GEMV: identical hidden states and greedy tokens."""
    model = request.getfixturevalue(which)
    prompt = np.random.default_rng(5).integers(0, model.shape.vocab_size, 6).astype(np.int32)
    out = []
    prev = g4.set_gemv_rows(True)
    try:
        for on in (True, False):
            g4.set_gemv_rows(on)
            out.append(single(g4, model, prompt, 6))
    finally:
        g4.set_gemv_rows(prev)
    (ga, ha), (gb, hb) = out
    assert list(ga) == list(gb)
    assert (ha.view(np.uint32) == hb.view(np.uint32)).all()
