"""Batched prefill (g4_prefill): the prompt loop of generate (lm_mode 0
forwards, gemma4-4b/cpu-blas/main.c:2366-2402) for many positions and
sequences at once, on the tensor-core GEMMs.  Every row runs with the decode
step's own arithmetic (batch-invariant GEMMs; the K/V rows of a call stored
first, then each row's attention over its causal window with the decode
kernel), so the result must equal decoding the prompt one position at a time
bit for bit: K/V cache rows, hidden states and the next tokens.  Prompts run
past the 16-row sliding window (ring wrap) into the shared-KV layers.
"""
import numpy as np
import pytest

from _tol import assert_close

pytestmark = pytest.mark.gpu


def _sequential(g4, model, prompts, max_seq):
    B, T = prompts.shape
    es = g4.Engine(model, 0, max_seq=max_seq, max_batch=B)
    for pos in range(T):
        nxt = es.decode_batch(prompts[:, pos], pos, 1 if pos == T - 1 else 0)
    return es, nxt


def _kv_all(g4, eng, model, B, T):
    S = g4.synth
    out = {}
    for l in (0, 5, 22, 23):
        hd = model.shape.head_dim_swa if S.is_swa(model.shape, l) else model.shape.head_dim_full
        lo = max(0, T - model.shape.sliding_window) if S.is_swa(model.shape, l) else 0
        for b in range(B):
            for p in range(lo, T):
                out[(l, b, p)] = eng.kv(l, p, model.shape.n_kv_heads * hd, b)
    return out


@pytest.mark.parametrize("which,rows", [("TINY_F", 24), ("TINY", 48), ("TINY_Q5", 20)])
def test_prefill_bitwise_equals_sequential(g4, gpu, which, rows):
    model = g4.synth.make_model(getattr(g4.synth, which), seed=3)
    B, T, max_seq = 3, 40, 48
    prompts = np.random.default_rng(rows).integers(0, 4096, (B, T)).astype(np.int32)
    ep = g4.Engine(model, 0, max_seq=max_seq, max_batch=B, prefill_rows=rows)
    es, nxt_s = _sequential(g4, model, prompts, max_seq)
    try:
        ep.prefill_prompts(prompts, T - 1)
        nxt_p = ep.decode_batch(prompts[:, T - 1], T - 1, 1)
        assert (nxt_p == nxt_s).all(), (nxt_p, nxt_s)
        for b in range(B):
            assert (ep.hidden(b) == es.hidden(b)).all(), b
        kp, ks = _kv_all(g4, ep, model, B, T), _kv_all(g4, es, model, B, T)
        for key in ks:
            assert (kp[key][0] == ks[key][0]).all() and (kp[key][1] == ks[key][1]).all(), key
        # and decoding continues identically from the prefilled cache
        a, b_ = nxt_p.copy(), nxt_s.copy()
        for pos in range(T, T + 4):
            a = ep.decode_batch(a, pos, 1)
            b_ = es.decode_batch(b_, pos, 1)
            assert (a == b_).all(), (pos, a, b_)
    finally:
        ep.close()
        es.close()


def test_prefill_matches_reference(g4, gpu, ref):
    """The fp32-path model: prefill then the last prompt token, against the
    reference's position-by-position forward (logits within 5e-5, K/V rows
    within 1e-5 / 2e-5 as in the decode tests)."""
    m = g4.synth.make_model(g4.synth.TINY_F, seed=5)
    T = 30
    toks = np.random.default_rng(5).integers(0, 4096, T).astype(np.int32)
    eng = g4.Engine(m, 0, max_seq=40, prefill_rows=12)
    rm = ref.model(m.desc(), 40)
    try:
        eng.prefill_prompts(toks[None, :], T - 1)
        am, lg = eng.forward(int(toks[-1]), T - 1, 1, want_logits=True)
        for pos in range(T):
            rm.forward(int(toks[pos]), pos, 1 if pos == T - 1 else 0)
        assert_close(lg, rm.logits(), rel=5e-5, what="logits after prefill")
        for l, hd in ((0, 64), (5, 128), (22, 64), (23, 128)):
            k, v = eng.kv(l, T - 3, 2 * hd)
            rk, rv = rm.kv(l, T - 3, 2 * hd)
            assert_close(k, rk, rel=2e-5, what="K L%d" % l)
            assert_close(v, rv, rel=2e-5, what="V L%d" % l)
    finally:
        eng.close()
        rm.close()


def test_prefill_rejects_bad_rows(g4, gpu):
    m = g4.synth.make_model(g4.synth.TINY_F, seed=1)
    eng = g4.Engine(m, 0, max_seq=32, max_batch=2, prefill_rows=8)
    try:
        with pytest.raises(g4.G4Error):  # more rows than prefill_rows
            eng.prefill(np.zeros(9, np.int32), np.arange(9), np.ones(9))
        with pytest.raises(g4.G4Error):  # the same (sequence, position) twice
            eng.prefill([0, 0], [3, 3], [1, 2])
        with pytest.raises(g4.G4Error):  # sequence out of range
            eng.prefill([2], [0], [1])
    finally:
        eng.close()
