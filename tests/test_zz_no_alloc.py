"""g4d_attn_decode_noalloc: decode attention for callers that cannot allocate.

Some callers of this library cannot let it call cudaMalloc: a server that owns
all device memory through its own pools, or code running inside another
process's memory budget.  This entry point takes only device pointers for its
inputs and outputs and keeps its scratch in a fixed array inside the library.
The tests call it several times in a row through the C ABI and check each
result against g4_attn_decode, the existing entry point, and against the CPU
oracle's attention (the restatement of gemma4-4b/cpu-blas/main.c:1924-1950),
with the tolerance the other attention tests use.  The cases cover the
streaming kernel (head dim 64/128/256), the head-dim-512 kernel, and a case
near the static limit.  This file is collected last so a failure here leaves
the rest of the suite already run; it passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

from _tol import assert_close

pytestmark = pytest.mark.gpu


def _inputs(seed, nwin, hd, nh, stride):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal(nh * hd) * 0.2).astype(np.float32)
    k = rng.standard_normal(nwin * stride).astype(np.float32)
    v = rng.standard_normal(nwin * stride).astype(np.float32)
    return q, k, v


def _noalloc(g4, q, k, v, nwin, stride, nh, nkv, hd):
    import torch
    L = g4.lib()
    # the K/V rows in the device layout [n_kv][nwin][hd]
    kh = np.ascontiguousarray(k.reshape(nwin, stride)[:, :nkv * hd].reshape(nwin, nkv, hd).transpose(1, 0, 2))
    vh = np.ascontiguousarray(v.reshape(nwin, stride)[:, :nkv * hd].reshape(nwin, nkv, hd).transpose(1, 0, 2))
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, kh, vh))
    out = torch.full((nh * hd,), float("nan"), device="cuda")
    rc = L.g4d_attn_decode_noalloc(C.c_void_p(out.data_ptr()), C.c_void_p(qd.data_ptr()),
                                   C.c_void_p(kd.data_ptr()), C.c_void_p(vd.data_ptr()), nwin, nh, nkv, hd, None)
    assert rc == 0, g4.last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


# (head_dim, positions, kv row stride, seed, query heads, kv heads)
CASES = [
    (256, 700, 2 * 256 + 64, 1, 8, 2),
    (128, 4096, 2 * 128, 2, 8, 2),
    (512, 96, 2 * 512, 3, 8, 2),        # the head-dim-512 kernel
    (256, 8192, 2 * 256, 4, 8, 2),      # about 2.1 MiB of the 4 MiB static scratch
    (64, 33, 4 * 64, 5, 4, 4),          # one query head per kv head, a ragged last chunk
]


def test_attn_decode_noalloc_matches_existing_entry_point_and_oracle(gpu, orc):
    g4 = gpu
    for hd, nwin, stride, seed, nh, nkv in CASES:  # several calls in a row share the static scratch
        q, k, v = _inputs(seed, nwin, hd, nh, stride)
        got = _noalloc(g4, q, k, v, nwin, stride, nh, nkv, hd)
        expect = g4.attn_decode(q, k, v, nwin, stride, nh, nkv, hd)
        assert_close(got, expect, rel=1e-5, what="noalloc vs g4_attn_decode hd %d nwin %d" % (hd, nwin))
        ref = orc.attention(q, k, v, nwin, stride, nh, nkv, hd)
        assert_close(got, ref, rel=1e-5, what="noalloc vs oracle hd %d nwin %d" % (hd, nwin))
    # the first case again after the others: leftovers in the shared array must not leak in
    hd, nwin, stride, seed, nh, nkv = CASES[0]
    q, k, v = _inputs(seed, nwin, hd, nh, stride)
    again = _noalloc(g4, q, k, v, nwin, stride, nh, nkv, hd)
    assert_close(again, orc.attention(q, k, v, nwin, stride, nh, nkv, hd), rel=1e-5, what="repeat call")


def test_attn_decode_noalloc_rejects_oversize(gpu):
    g4 = gpu
    L = g4.lib()
    # 8 heads x 512 dims x 8192 positions needs more than the 4 MiB static scratch
    rc = L.g4d_attn_decode_noalloc(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 8192, 8, 2, 512,
                                   None)
    assert rc == g4.G4_ERR_ARG
    assert "static limit" in g4.last_error()[1]
