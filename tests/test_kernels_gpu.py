"""GPU parity of the per-call C ABI (libg4b200.so) against the oracle.

Integer results bit-exact; float results within the term-scaled tolerance of
tests/_tol.py (1e-5).  Sizes go up to the single-GEMV benchmark shape (Q4_K 10240 x 2560).
"""
import numpy as np
import pytest

from _tol import assert_close, dense_term_scale, kquant_term_scale

pytestmark = pytest.mark.gpu
Q4, Q5, Q6, BF16, F16, F32 = 12, 13, 14, 30, 1, 0


def test_quantize_q8K_golden(gpu, golden):
    for x, y in zip(golden["q8_x"], golden["q8_out"]):
        assert (gpu.quantize_row_q8_K(x) == y).all()


@pytest.mark.parametrize("scale", [1e-30, 1e-3, 1.0, 3e4])
def test_quantize_q8K_random(gpu, orc, scale):
    rng = np.random.default_rng(int(scale * 7) % 1000 + 1)
    x = (rng.standard_normal(2560 * 8) * scale).astype(np.float32)
    x[256:512] = 0.0
    big = np.abs(x[768:1024]).max() * 2
    x[1000], x[1001] = big, -big  # tie of |x| inside a block: the first index wins
    assert (gpu.quantize_row_q8_K(x) == orc.quantize_q8K(x)).all()


@pytest.mark.parametrize("name,t", [("q4", Q4), ("q5", Q5)])
def test_block_sums_golden(gpu, golden, name, t):
    ss, sm = gpu.block_sums(golden[name + "_w"], 512, 16, t, golden[name + "_q8"])
    assert (ss == golden[name + "_ss"]).all() and (sm == golden[name + "_sm"]).all()


@pytest.mark.parametrize("t", [Q4, Q5])
def test_block_sums_random(gpu, orc, g4, t):
    rng = np.random.default_rng(t)
    w = g4.synth.rand_blocks(rng, t, 48, 2560, 1e-3, 2e-2)
    q8 = orc.quantize_q8K(rng.standard_normal(2560).astype(np.float32))
    ss, sm = gpu.block_sums(w, 2560, 48, t, q8)
    ess, esm = orc.block_sums(w, t, 2560, 48, q8)
    assert (ss == ess).all() and (sm == esm).all()


@pytest.mark.parametrize("name,t", [("q4", Q4), ("q5", Q5)])
def test_kquant_gemv_golden(gpu, golden, name, t):
    w, x, q8 = golden[name + "_w"], golden[name + "_x"], golden[name + "_q8"]
    scale = kquant_term_scale(w, t, 512, q8, golden[name + "_ss"], golden[name + "_sm"])
    q8buf = gpu.q8_buffer(512)
    o = gpu.mm(x, w, 512, 16, t, q8buf, 0)
    assert (q8buf == q8).all(), "mm must leave the quantized activation in q8 (main.c:1686)"
    assert_close(o, golden[name + "_dot"], scale, what=name + " vs reference AVX2")
    o2 = gpu.mm_quant_dot_rows(w, 512, 16, t, q8)
    assert (o2 == o).all()
    r = np.array([gpu.vec_dot(t, 512, w[i], q8) for i in range(16)], np.float32)
    assert_close(r, golden[name + "_dot"], scale, what=name + " vec_dot")


@pytest.mark.parametrize("t,rows,n", [(Q4, 10240, 2560), (Q4, 2560, 2048), (Q4, 512, 2560), (Q5, 2048, 2560),
                                      (Q4, 2560, 10240), (Q5, 7, 4096)])
def test_kquant_gemv_sizes(gpu, orc, g4, t, rows, n):
    rng = np.random.default_rng(rows + n + t)
    w = g4.synth.rand_blocks(rng, t, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal(n).astype(np.float32)
    q8 = orc.quantize_q8K(x)
    o = gpu.mm(x, w, n, rows, t)
    e = orc.mm(x, w, n, rows, t)
    ss, sm = gpu.block_sums(w, n, rows, t, q8)
    assert_close(o, e, kquant_term_scale(w, t, n, q8, ss, sm), what="Q%dK %dx%d" % (t - 8, rows, n))


@pytest.mark.parametrize("rows,n", [(8, 512), (512, 2560), (2560, 10240), (4096, 2560), (13, 256)])
def test_q6K_gemv(gpu, orc, g4, rows, n):
    rng = np.random.default_rng(rows * 3 + n)
    w = g4.synth.rand_blocks(rng, Q6, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal(n).astype(np.float32)
    o = gpu.mm(x, w, n, rows, Q6)
    e = orc.mm(x, w, n, rows, Q6)
    deq = np.stack([orc.dequant(w[r].copy(), Q6, n // 256) for r in range(rows)])
    assert_close(o, e, dense_term_scale(deq, x), what="Q6K %dx%d" % (rows, n))
    o2 = gpu.mm_quant_rows(x, w, n, rows, Q6)
    assert (o2 == o).all()


def test_q6K_golden(gpu, golden, orc):
    w, x = golden["q6_w"], golden["q6_x"]
    deq = np.stack([orc.dequant(w[r].copy(), Q6, 2) for r in range(8)])
    assert_close(gpu.mm(x, w, 512, 8, Q6), golden["q6_mm"], dense_term_scale(deq, x), what="Q6K golden")


@pytest.mark.parametrize("t", [Q4, Q5])
def test_mm_quant_rows_fp32_path(gpu, orc, g4, t):
    """mm_quant_rows on Q4_K/Q5_K rows: fp32 dequant-dot (the --f32-matmul path)."""
    rng = np.random.default_rng(9 + t)
    w = g4.synth.rand_blocks(rng, t, 33, 1024, 1e-3, 2e-2)
    x = rng.standard_normal(1024).astype(np.float32)
    o = gpu.mm_quant_rows(x, w, 1024, 33, t)
    rb = w.shape[1]
    e = np.array([orc._rowdot(x.ctypes.data, w.ctypes.data + r * rb, 1024, t) for r in range(33)], np.float32)
    deq = np.stack([orc.dequant(w[r].copy(), t, 4) for r in range(33)])
    assert_close(o, e, dense_term_scale(deq, x), what="fp32 dequant-dot")


@pytest.mark.parametrize("t,name", [(BF16, "bf16"), (F16, "f16"), (F32, "f32")])
def test_dense_gemv(gpu, orc, golden, g4, t, name):
    x, w = golden["dense_x"], golden[name + "_w"]
    wf = w.astype(np.float32) if t == F32 else (w.view(np.float16).astype(np.float32) if t == F16 else
                                                 (w.astype(np.uint32) << 16).view(np.float32))
    assert_close(gpu.mm(x, w, 384, 8, t), golden[name + "_mm"], dense_term_scale(wf, x), what=name)
    rng = np.random.default_rng(t + 77)
    for n in (100, 10752, 2560):   # n % 8 != 0 takes the scalar path
        w2 = g4.synth._qmat(rng, t, 37, n, 0.05)
        x2 = rng.standard_normal(n).astype(np.float32)
        wf2 = w2.astype(np.float32) if t == F32 else (w2.view(np.float16).astype(np.float32) if t == F16 else
                                                       (w2.astype(np.uint32) << 16).view(np.float32))
        assert_close(gpu.mm(x2, w2, n, 37, t), orc.mm(x2, w2, n, 37, t), dense_term_scale(wf2, x2), what=name)


def test_argmax_row(gpu, orc, golden, g4):
    assert gpu.mm_argmax_row(golden["q4_x"], golden["q4_w"], 512, 16, Q4) == int(golden["q4_argmax"])
    assert gpu.mm_argmax_row(golden["q6_x"], golden["q6_w"], 512, 8, Q6) == int(golden["q6_argmax"])
    rng = np.random.default_rng(4)
    w = g4.synth.rand_blocks(rng, Q6, 3000, 512, 1e-3, 2e-2)
    x = rng.standard_normal(512).astype(np.float32)
    e = orc.mm(x, w, 512, 3000, Q6)
    s = np.sort(e)
    assert s[-1] - s[-2] > 1e-3 * abs(s[-1])
    assert gpu.mm_argmax_row(x, w, 512, 3000, Q6) == int(np.argmax(e))
    # duplicated best row: the lowest index wins
    w[2999] = w[int(np.argmax(e))]
    w2 = np.ascontiguousarray(w)
    gpu.registry_clear()
    assert gpu.mm_argmax_row(x, w2, 512, 3000, Q6) == int(np.argmax(e))


def test_rope_bit_exact(gpu, golden):
    v, ff = golden["rope_in"], golden["rope_ff"]
    for i, p in enumerate(golden["rope_pos"]):
        assert (gpu.apply_rope_neox(v, 8, 64, 64, int(p), 1e4) == golden["rope_swa"][i]).all()
        assert (gpu.apply_rope_neox(v, 8, 64, 64, int(p), 1e6, 1.0, ff) == golden["rope_full"][i]).all()
        assert (gpu.apply_rope_neox(v, 8, 64, 32, int(p), 1e4) == golden["rope_partial"][i]).all()


@pytest.mark.parametrize("hd,nwin", [(64, 1), (64, 37), (128, 16), (256, 512), (256, 8192), (512, 700)])
def test_attention(gpu, orc, hd, nwin):
    rng = np.random.default_rng(hd + nwin)
    nh, nkv, stride = 8, 2, 2 * hd + 64
    q = (rng.standard_normal(nh * hd) * 0.2).astype(np.float32)
    k = rng.standard_normal(nwin * stride).astype(np.float32)
    v = rng.standard_normal(nwin * stride).astype(np.float32)
    o = gpu.attn_decode(q, k, v, nwin, stride, nh, nkv, hd)
    e = orc.attention(q, k, v, nwin, stride, nh, nkv, hd)
    assert_close(o, e, rel=1e-5, what="attention hd %d nwin %d" % (hd, nwin))


def test_logits_tied(gpu, orc, g4):
    rng = np.random.default_rng(12)
    emb = g4.synth.rand_blocks(rng, Q6, 4096, 512, 5e-5, 1.5e-4)
    x = rng.standard_normal(512).astype(np.float32)
    lg, am = gpu.logits_tied(x, emb, Q6, 512, 4096, 30.0)
    e = orc.logits_tied(x, emb, Q6, 512, 4096, 30.0)
    assert_close(lg, e, rel=1e-5, what="softcapped logits")
    assert am == orc.argmax_first(e)
    _, am2 = gpu.logits_tied(x, emb, Q6, 512, 4096, 30.0, want_logits=False)
    assert am2 == am


@pytest.mark.parametrize("t,rows,n", [(Q4, 10240, 2560), (Q4, 2560, 2048), (Q4, 7, 768), (Q5, 2048, 2560),
                                      (Q4, 2560, 10240), (Q5, 13, 1280)])
def test_batch1_gemv_kernels_bitwise(gpu, g4, t, rows, n):
    """The row-owner batch-1 GEMV and the tiled streaming GEMV fold every row's exact block terms in
    the same canonical order: identical bits (ragged tiles, odd block counts, long rows)."""
    rng = np.random.default_rng(rows * 5 + n + t)
    w = g4.synth.rand_blocks(rng, t, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal(n).astype(np.float32)
    prev = g4.set_gemv_rows(True)
    try:
        a = gpu.mm(x, w, n, rows, t)
        g4.set_gemv_rows(False)
        b = gpu.mm(x, w, n, rows, t)
    finally:
        g4.set_gemv_rows(prev)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
