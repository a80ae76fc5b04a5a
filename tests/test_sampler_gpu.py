"""The sampler (sample_token, apply_repetition_penalty, rng_f32 of
gemma4-4b/cpu-blas/main.c:2035-2126) on the GPU: the repetition penalty and
the top-k candidates on the device, the temperature / top-p tail replayed on
the host with the reference's expressions.  Given the same logits and rng
state the token and the next rng state must equal the reference's exactly;
whole sampled streams of the fp32-path model must equal the reference's
generate, and batched sampling must equal sampling each sequence alone.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _logits_cases(rng):
    n = 4096
    base = rng.standard_normal(n).astype(np.float32) * 3.0
    ties = base.copy()
    ties[rng.integers(0, n, 300)] = np.float32(7.25)      # many equal values around the top-40 boundary
    capped = np.clip(base * 20.0, -30.0, 30.0).astype(np.float32)  # softcap saturation: ties at 30.0
    zeros = np.where(rng.random(n) < 0.5, np.float32(0.0), np.float32(-0.0)).astype(np.float32)
    zeros[rng.integers(0, n, 20)] = rng.standard_normal(20).astype(np.float32) * 1e-3
    big = rng.standard_normal(262144).astype(np.float32) * 4.0
    return [base, ties, capped, zeros, big]


@pytest.mark.parametrize("temp,topp,topk", [(0.0, 0.9, 40), (0.6, 0.9, 40), (1.0, 0.0, 40), (0.8, 0.5, 64),
                                            (1.3, 0.95, 1), (0.7, 1.0, 17)])
def test_sample_token_matches_reference(gpu, ref, temp, topp, topk):
    g4 = gpu
    rng = np.random.default_rng(int(100 * temp) + topk)
    for lg in _logits_cases(rng):
        for seed in (1, 42, 0x9E3779B97F4A7C15):
            tok, st = g4.sample_token(lg, temp, topp, topk, seed)
            rtok, rst = ref.sample(lg, temp, topp, topk, seed)
            assert (tok, st) == (rtok, rst), (temp, topp, topk, seed, tok, rtok)


def test_generate_sampled_stream_matches_reference(g4, gpu, ref):
    m = g4.synth.make_model(g4.synth.TINY_F, seed=3)
    eng = g4.Engine(m, 0, max_seq=64)
    rm = ref.model(m.desc(), 64)
    prompt = np.random.default_rng(5).integers(0, 4096, 8).astype(np.int32)
    try:
        for kw in (dict(temp=0.8, topp=0.9, repeat_penalty=1.1, penalty_last_n=16, seed=42),
                   dict(temp=1.2, topp=0.0, repeat_penalty=1.0, penalty_last_n=64, seed=7),
                   dict(temp=0.0, topp=0.9, repeat_penalty=1.3, penalty_last_n=8, seed=1)):
            got = eng.generate(prompt, 24, kw["temp"], kw["topp"], 40, kw["repeat_penalty"], kw["penalty_last_n"],
                               kw["seed"])
            want = rm.generate_sample(prompt, 24, kw["temp"], kw["topp"], kw["repeat_penalty"], kw["penalty_last_n"],
                                      kw["seed"])
            assert (got == want).all(), (kw, got, want)
    finally:
        eng.close()
        rm.close()


@pytest.mark.parametrize("which,B", [("TINY_F", 4), ("TINY", 16)])
def test_batched_sampling_equals_single(g4, gpu, which, B):
    """decode_batch_sample over B sequences (the tensor-core step at B = 16)
    draws, for every sequence, the token of that sequence decoded alone with
    the same rng state and penalty history."""
    m = g4.synth.make_model(getattr(g4.synth, which), seed=3)
    rng = np.random.default_rng(B)
    toks = rng.integers(0, 4096, B).astype(np.int32)
    steps = 6
    eb = g4.Engine(m, 0, max_seq=32, max_batch=B)
    states = np.arange(1, B + 1, dtype=np.uint64) * np.uint64(0x9E3779B9)
    hist = np.zeros((B, steps), np.int32)
    outs = []
    cur = toks.copy()
    try:
        for pos in range(steps):
            nrec = np.full(B, pos, np.int32)
            cur = eb.decode_batch_sample(cur, pos, 0.9, 0.8, 40, states, repeat_penalty=1.2, recent=hist, n_recent=nrec)
            hist[:, pos] = cur
            outs.append(cur.copy())
    finally:
        eb.close()
    outs = np.stack(outs, 1)
    es = g4.Engine(m, 0, max_seq=32, max_batch=1)
    try:
        for b in range(B):
            st = np.array([np.uint64(b + 1) * np.uint64(0x9E3779B9)], np.uint64)
            h1 = np.zeros((1, steps), np.int32)
            cur1 = np.array([toks[b]], np.int32)
            for pos in range(steps):
                cur1 = es.decode_batch_sample(cur1, pos, 0.9, 0.8, 40, st, repeat_penalty=1.2, recent=h1,
                                              n_recent=np.array([pos], np.int32))
                h1[0, pos] = cur1[0]
            assert (h1[0] == outs[b]).all(), (b, h1[0], outs[b])
    finally:
        es.close()
