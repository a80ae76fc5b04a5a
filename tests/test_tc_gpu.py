"""Batched K-quant GEMMs on the tensor cores (tcgen05, k_gemm_tc.cu,
k_gemm_q6tc.cu) through the C ABI (g4d_mm with batch >= the tensor-core
threshold), against the oracle per sequence and, bit for bit, against the
streaming GEMV on the same inputs.

The reference computes one activation at a time (mm_quant_dot_rows,
gemma4-4b/cpu-blas/main.c:1558-1566); a batch of B activations must give, for
every sequence, the same result as B separate calls within the K-quant
tolerance (integer block sums exact, float sum order free).
"""
import numpy as np
import pytest

from _tol import assert_close, kquant_term_scale

pytestmark = pytest.mark.gpu

Q4, Q5 = 12, 13


def _run(g4, torch, w, x, t, n, rows, tc_min):
    B = x.shape[0]
    dev = torch.device("cuda:0")
    wd = g4.weight_upload(w, t, n, rows)
    try:
        xd = torch.from_numpy(x).to(dev)
        q8 = torch.zeros(B * (n // 256) * 292, dtype=torch.uint8, device=dev)
        o = torch.full((B, rows), float("nan"), dtype=torch.float32, device=dev)
        prev = g4.set_tc_min_batch(tc_min)
        try:
            g4.mm_device(o.data_ptr(), xd.data_ptr(), wd, n, rows, t, q8.data_ptr(), 0, B,
                         torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
        finally:
            g4.set_tc_min_batch(prev)
        return o.cpu().numpy(), q8.cpu().numpy().reshape(B, -1)
    finally:
        g4.free(wd)


@pytest.fixture
def torch_cuda(gpu):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("torch sees no CUDA device")
    return torch


@pytest.mark.parametrize("t,rows,n,B", [
    (Q4, 300, 2560, 16),     # one ragged row tile, NP = 16
    (Q4, 2048, 2560, 20),    # NP = 32 with padding sequences
    (Q4, 2560, 2048, 64),    # O-projection shape, NP = 64
    (Q4, 10240, 2560, 64),   # gate/up shape
    (Q4, 2560, 10240, 33),   # long K: many K-slices per tile
    (Q5, 1000, 4096, 40),
    (Q4, 512, 2560, 70),     # two groups (64 + 6)
])
def test_tc_gemm_vs_oracle(gpu, torch_cuda, orc, g4, t, rows, n, B):
    rng = np.random.default_rng(1000 * t + rows + n + B)
    w = g4.synth.rand_blocks(rng, t, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal((B, n)).astype(np.float32)
    x[1] *= 50.0  # per-sequence scales differ
    o, q8 = _run(g4, torch_cuda, w, x, t, n, rows, tc_min=1)
    assert np.isfinite(o).all()
    for s in range(B):
        q8s = orc.quantize_q8K(x[s])
        assert (q8[s] == q8s.reshape(-1)).all(), "Q8_K bytes of sequence %d" % s
        e = orc.mm(x[s], w, n, rows, t)
        ss, sm = g4.block_sums(w, n, rows, t, q8s)  # exact; pinned against the oracle elsewhere
        assert_close(o[s], e, kquant_term_scale(w, t, n, q8s, ss, sm), what="TC Q%dK seq %d" % (t - 8, s))


@pytest.mark.parametrize("t,rows,n,B", [
    (Q4, 640, 2560, 24), (Q5, 640, 2560, 24),
    (Q4, 10240, 2560, 64),   # gate/up shape: stream-K segments inside row tiles
    (Q4, 2560, 10240, 33),   # long rows
    (Q5, 1000, 4096, 40),    # uniform K slices
])
def test_tc_gemm_vs_gemv_bitwise(gpu, torch_cuda, g4, t, rows, n, B):
    """Same inputs through the tensor-core GEMM and the streaming GEMV: both
    sum each row's exact per-block terms in the same canonical order, so the
    results are identical bit for bit (a sequence's output does not depend on
    the batch it is computed in)."""
    rng = np.random.default_rng(77 + t + rows + B)
    w = g4.synth.rand_blocks(rng, t, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal((B, n)).astype(np.float32)
    x[2] *= 1e3
    o_tc, _ = _run(g4, torch_cuda, w, x, t, n, rows, tc_min=1)
    o_sv, _ = _run(g4, torch_cuda, w, x, t, n, rows, tc_min=1 << 30)
    bad = np.flatnonzero((o_tc != o_sv).any(axis=1))
    assert bad.size == 0, "sequences %s differ (max |diff| %.3g)" % (bad[:8], np.abs(o_tc - o_sv).max())


def test_tc_gemm_repeat_deterministic(gpu, torch_cuda, g4):
    """K-slice partials are summed in a fixed order: repeated calls agree bitwise."""
    rows, n, B = 2560, 10240, 64
    rng = np.random.default_rng(5)
    w = g4.synth.rand_blocks(rng, Q4, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal((B, n)).astype(np.float32)
    a, _ = _run(g4, torch_cuda, w, x, Q4, n, rows, tc_min=1)
    b, _ = _run(g4, torch_cuda, w, x, Q4, n, rows, tc_min=1)
    assert (a == b).all()


Q6 = 14


def _run6(g4, torch, w, x, n, rows, tc_min):
    B = x.shape[0]
    dev = torch.device("cuda:0")
    wd = g4.weight_upload(w, Q6, n, rows)
    try:
        xd = torch.from_numpy(x).to(dev)
        o = torch.full((B, rows), float("nan"), dtype=torch.float32, device=dev)
        prev = g4.set_tc_min_batch(tc_min)
        try:
            g4.mm_device(o.data_ptr(), xd.data_ptr(), wd, n, rows, Q6, 0, 0, B, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
        finally:
            g4.set_tc_min_batch(prev)
        return o.cpu().numpy()
    finally:
        g4.free(wd)


@pytest.mark.parametrize("rows,n,B", [
    (300, 2560, 16),     # ragged row tile
    (512, 2560, 20),     # V shape, padding sequences
    (2560, 10240, 64),   # FFN down shape
    (4096, 2560, 64),
    (2560, 2048, 33),
    (200, 1024, 70),     # two groups
])
def test_tc_q6K_vs_oracle(gpu, torch_cuda, orc, g4, rows, n, B):
    """Q6_K fp32 dequant-dot (mm_quant_rows, main.c:1539-1556) for B activations at once."""
    from _tol import dense_term_scale
    rng = np.random.default_rng(7 * rows + n + B)
    w = g4.synth.rand_blocks(rng, Q6, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal((B, n)).astype(np.float32)
    x[1] *= 3e4    # per-sequence magnitudes far apart
    x[2] *= 1e-4
    x[3, : n // 2] = 0.0   # all-zero super-blocks
    x[4, 5] = 1e3          # one outlier in a block
    o = _run6(g4, torch_cuda, w, x, n, rows, tc_min=1)
    assert np.isfinite(o).all()
    deq = np.stack([orc.dequant(w[r].copy(), Q6, n // 256) for r in range(rows)])
    for s in range(B):
        e = orc.mm(x[s], w, n, rows, Q6)
        assert_close(o[s], e, dense_term_scale(deq, x[s]), what="TC Q6K seq %d" % s)


@pytest.mark.parametrize("rows,n,B", [(640, 2560, 24), (2560, 10240, 64), (512, 2560, 16), (300, 2048, 40)])
def test_tc_q6K_vs_gemv_bitwise(gpu, torch_cuda, g4, rows, n, B):
    """Q6_K on the tensor cores and on the streaming GEMV: the block dots are
    exact integers in both, summed in the same canonical order, so the
    results are identical bit for bit."""
    rng = np.random.default_rng(99 + rows + B)
    w = g4.synth.rand_blocks(rng, Q6, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal((B, n)).astype(np.float32)
    x[1] *= 3e4
    x[3, : n // 2] = 0.0
    o_tc = _run6(g4, torch_cuda, w, x, n, rows, tc_min=1)
    o_sv = _run6(g4, torch_cuda, w, x, n, rows, tc_min=1 << 30)
    bad = np.flatnonzero((o_tc != o_sv).any(axis=1))
    assert bad.size == 0, "sequences %s differ (max |diff| %.3g)" % (bad[:8], np.abs(o_tc - o_sv).max())


BF16 = 30


@pytest.mark.parametrize("rows,n,B", [
    (256, 2560, 64),     # per-layer-embedding gate shape
    (2560, 256, 64),     # per-layer-embedding projection shape
    (1000, 2560, 20),    # ragged tile, padding sequences
    (130, 512, 70),      # two groups
])
def test_tc_bf16_vs_oracle(gpu, torch_cuda, orc, g4, rows, n, B):
    """BF16 rows (mm_bf16, main.c:1520-1537): fp32 dot of x with bf16 weights, for B activations at once."""
    from _tol import dense_term_scale
    rng = np.random.default_rng(31 * rows + n + B)
    wf = rng.standard_normal((rows, n)).astype(np.float32) * 0.05
    w = ((wf.view(np.uint32) + 0x8000) >> 16).astype(np.uint16)  # round to bf16
    deq = (w.astype(np.uint32) << 16).view(np.float32)
    x = rng.standard_normal((B, n)).astype(np.float32)
    x[1] *= 1e4
    x[2] *= 1e-5
    dev = torch_cuda.device("cuda:0")
    wd = g4.weight_upload(w, BF16, n, rows)
    try:
        xd = torch_cuda.from_numpy(x).to(dev)
        o = torch_cuda.full((B, rows), float("nan"), dtype=torch_cuda.float32, device=dev)
        prev = g4.set_tc_min_batch(1)
        try:
            g4.mm_device(o.data_ptr(), xd.data_ptr(), wd, n, rows, BF16, 0, 0, B, torch_cuda.cuda.current_stream().cuda_stream)
            torch_cuda.cuda.synchronize()
        finally:
            g4.set_tc_min_batch(prev)
        o = o.cpu().numpy()
    finally:
        g4.free(wd)
    assert np.isfinite(o).all()
    for s in range(B):
        e = orc.mm(x[s], w, n, rows, BF16)
        assert_close(o[s], e, dense_term_scale(deq, x[s]), what="TC BF16 seq %d" % s)
