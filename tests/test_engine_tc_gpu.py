"""The batched decode step on the tensor cores (B >= 9: Q4_K/Q5_K/Q6_K GEMMs
through tcgen05, the LM head with the softcap+argmax epilogue) against
decoding each sequence alone on the streaming-GEMV path.

The reference decodes one sequence at a time (forward, gemma4-4b/cpu-blas/
main.c:1838-2029); a batch of independent sequences must reproduce each
sequence's greedy stream.  On the fp32-path model (TINY_F: Q6_K and dense
projections, no Q8_K activation rounding) the batched float sums differ from
the single-sequence ones only in order, so the streams are token-identical.
On the Q4_K_M mix, a last-ulp difference can flip a Q8_K rounding of the
next activation (the reference's own AVX2 and generic builds differ the same
way), so there the hidden states are compared within that spread and the
first greedy token must match.
"""
import numpy as np
import pytest

from _tol import normwise

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tinyf(g4):
    return g4.synth.make_model(g4.synth.TINY_F, seed=3)


@pytest.fixture(scope="module")
def tiny(g4):
    return g4.synth.make_model(g4.synth.TINY, seed=3)


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


@pytest.mark.parametrize("B", [16, 24])
def test_tc_batched_fp32_path_streams_identical(g4, gpu, tinyf, B):
    rng = np.random.default_rng(100 + B)
    prompts = rng.integers(0, 4096, (B, 4)).astype(np.int32)
    outs, hid = batched_stream(g4, tinyf, prompts, 10)
    for b in range(B):
        got, h = single(g4, tinyf, prompts[b], 10)
        # float summation order only: the same 5e-5 bound the fp32-path model meets against the reference
        assert normwise(hid[b], h) < 5e-5, (b, normwise(hid[b], h))
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


def _single_first_step(g4, model, tok, max_seq=16):
    es = g4.Engine(model, 0, max_seq=max_seq, max_batch=1)
    nxt = es.forward(int(tok), 0, 1)
    kv = es.kv(0, 0, model.shape.n_kv_heads * model.shape.head_dim_swa)
    h = es.hidden(0)
    es.close()
    return nxt, kv, h


def test_tc_batched_q4km_mix(g4, gpu, tiny):
    """Q4_K_M mix.  Layer 0's K (Q4_K) and V (Q6_K) rows at position 0 come
    from GEMMs of an input that is identical in both paths, so they must agree
    to float summation order.  Downstream, one flipped Q8_K rounding of a later
    activation changes the output by up to a few 1e-2 (the same spread the
    single-sequence engine shows against the oracle on this model), so the
    hidden states are checked at that bound and most greedy tokens must agree."""
    B = 20
    toks = np.random.default_rng(7).integers(0, 4096, B)
    nxt, kv, hid = _first_step(g4, tiny, toks)
    same = 0
    for b in range(B):
        n1, (k1, v1), h1 = _single_first_step(g4, tiny, toks[b])
        assert normwise(kv[b][0], k1) < 1e-5 and normwise(kv[b][1], v1) < 1e-5, (b, normwise(kv[b][0], k1))
        assert normwise(hid[b], h1) < 0.3, (b, normwise(hid[b], h1))
        same += int(nxt[b] == n1)
    assert same >= int(0.8 * B), (same, B)


@pytest.mark.parametrize("B", [64, 65])
def test_tc_batched_64_sequences(g4, gpu, tiny, B):
    """A full group of 64 (NP = 64 kernels; the residual/norm launches write the
    GEMM operands themselves) and 64 + 1 (a second group; separate operand
    launches)."""
    toks = np.random.default_rng(11).integers(0, 4096, B)
    nxt, kv, hid = _first_step(g4, tiny, toks)
    for b in sorted({0, 31, 63, B - 1}):
        n1, (k1, v1), h1 = _single_first_step(g4, tiny, toks[b])
        assert normwise(kv[b][0], k1) < 1e-5 and normwise(kv[b][1], v1) < 1e-5, b
        assert normwise(hid[b], h1) < 0.3, (b, normwise(hid[b], h1))
