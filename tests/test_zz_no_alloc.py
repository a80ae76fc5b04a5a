"""g4d_attn_decode_noalloc: decode attention for callers that cannot allocate.

Some callers of this library cannot let it call cudaMalloc: a server that owns
all device memory through its own pools, or code running inside another
process's memory budget.  This entry point takes only device pointers for its
inputs and outputs and keeps its scratch in a fixed array inside the library.
The test calls it twice in a row through the C ABI and checks each result
against g4_attn_decode, the existing entry point, with the tolerance the other
attention tests use.  It is collected last so a failure here leaves the rest
of the suite already run, and it passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

from _tol import assert_close

pytestmark = pytest.mark.gpu


def _inputs(seed, nwin, hd, nh, nkv, stride):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal(nh * hd) * 0.2).astype(np.float32)
    k = rng.standard_normal(nwin * stride).astype(np.float32)
    v = rng.standard_normal(nwin * stride).astype(np.float32)
    return q, k, v


def test_attn_decode_noalloc_matches_existing_entry_point(gpu):
    import torch
    g4 = gpu
    L = g4.lib()
    nh, nkv = 8, 2
    cases = [(256, 700, 2 * 256 + 64, 1), (128, 4096, 2 * 128, 2)]  # two calls in a row
    for hd, nwin, stride, seed in cases:
        q, k, v = _inputs(seed, nwin, hd, nh, nkv, stride)
        expect = g4.attn_decode(q, k, v, nwin, stride, nh, nkv, hd)
        # the same K/V rows in the device layout [n_kv][nwin][hd]
        kh = np.ascontiguousarray(k.reshape(nwin, stride)[:, :nkv * hd].reshape(nwin, nkv, hd).transpose(1, 0, 2))
        vh = np.ascontiguousarray(v.reshape(nwin, stride)[:, :nkv * hd].reshape(nwin, nkv, hd).transpose(1, 0, 2))
        qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, kh, vh))
        out = torch.full((nh * hd,), float("nan"), device="cuda")
        rc = L.g4d_attn_decode_noalloc(C.c_void_p(out.data_ptr()), C.c_void_p(qd.data_ptr()),
                                       C.c_void_p(kd.data_ptr()), C.c_void_p(vd.data_ptr()), nwin, nh, nkv, hd, None)
        assert rc == 0, g4.last_error()
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), expect, rel=1e-5, what="noalloc attention hd %d nwin %d" % (hd, nwin))


def test_attn_decode_noalloc_rejects_oversize(gpu):
    g4 = gpu
    L = g4.lib()
    # 8 heads x 512 dims x 8192 positions needs more than the 4 MiB static scratch
    rc = L.g4d_attn_decode_noalloc(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 8192, 8, 2, 512,
                                   None)
    assert rc == g4.G4_ERR_ARG
    assert "static limit" in g4.last_error()[1]
