"""Parity tolerances (shared by the CPU and GPU tests).

Integer results (Q8_K bytes, per-block integer sums, argmax indices, greedy
token ids) must be bit-exact.  Float results cannot be: the reference's own
AVX2 and generic builds disagree elementwise by up to ~1e-3 relative where
d*sumi_s - dmin*sumi_m cancels.  So float outputs are checked two ways:
  * norm-wise:   ||a - b|| / ||b|| <= 1e-5 per output vector;
  * elementwise: |a_i - b_i| <= 1e-5 * scale_i + 1e-30, where scale_i is the
    magnitude of the terms summed into output i (sum |w x| for fp32 dots,
    sum |d_x d_w sumi_s| + |d_x dmin_w sumi_m| for K-quant integer dots).
"""
import numpy as np

REL = 1e-5


def normwise(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def assert_close(a, b, scale=None, rel=REL, what=""):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    nw = normwise(a, b)
    assert nw <= rel, "%s: norm-wise relative error %.3g > %.1g" % (what, nw, rel)
    if scale is not None:
        bad = np.abs(a - b) > rel * np.asarray(scale, np.float64) + 1e-30
        assert not bad.any(), "%s: %d elements outside the term-scaled bound (first %s)" % (
            what, int(bad.sum()), np.flatnonzero(bad)[:5])


def q8_fields(q8):
    b = np.asarray(q8, np.uint8).reshape(-1, 292)
    d = b[:, 0:4].copy().view(np.float32).reshape(-1)
    qs = b[:, 4:260].copy().view(np.int8)
    return d, qs


def f16(u16):
    return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)


def kquant_term_scale(w, t, n, q8, ss, sm):
    """sum over blocks of |d_x d_w sumi_s| + |d_x dmin_w sumi_m| per row."""
    bb = {12: 144, 13: 176}[t]
    nb = n // 256
    dx, _ = q8_fields(q8)
    wb = np.asarray(w, np.uint8).reshape(w.shape[0], nb, bb)
    dw = f16(wb[:, :, 0:2].copy().view(np.uint16)[..., 0])
    dm = f16(wb[:, :, 2:4].copy().view(np.uint16)[..., 0])
    return (np.abs(dx[None, :] * dw * ss) + np.abs(dx[None, :] * dm * sm)).sum(axis=1)


def dense_term_scale(wdeq, x):
    """sum |w_ij x_j| per row for fp32 dots."""
    return np.abs(np.asarray(wdeq, np.float64) * np.asarray(x, np.float64)[None, :]).sum(axis=1)
