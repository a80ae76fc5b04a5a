"""ctypes bindings of the two CPU oracles.  TEST INFRASTRUCTURE ONLY.

* `Oracle`   -> oracle/liboracle.so, the C restatement (g4_oracle.c).
* `Reference`-> oracle/_ref/libg4ref.so, gemma4-4b/cpu-blas/main.c compiled
  unchanged (ref_harness.c); absent when the reference tree was never built.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arms use this module, always as the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libg4ref.so")

Q8_BYTES = 292
vp, fp, ip = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int)


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def q8_buffer(n: int) -> np.ndarray:
    return np.zeros(((n + 255) // 256) * Q8_BYTES, dtype=np.uint8)


def q8_fields(q8: np.ndarray):
    """Split raw Q8_K bytes into (d float32[nb], qs int8[nb,256], bsums int16[nb,16])."""
    b = q8.reshape(-1, Q8_BYTES)
    d = b[:, 0:4].copy().view(np.float32).reshape(-1)
    qs = b[:, 4:260].copy().view(np.int8)
    bs = b[:, 260:292].copy().view(np.int16)
    return d, qs, bs


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.lib = C.CDLL(path)
        self.prefix = prefix

    def fn(self, name, restype, *argtypes):
        f = getattr(self.lib, self.prefix + name)
        f.restype = restype
        f.argtypes = list(argtypes)
        return f


class Oracle(_Lib):
    """The C restatement."""

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path, "or_")
        self._q8 = self.fn("quantize_row_q8_K", None, vp, vp, C.c_int)
        self._bsums = self.fn("qk_block_sums", None, vp, C.c_int, vp, ip, ip)
        self._vdot = self.fn("vec_dot_qk", C.c_float, C.c_int, vp, C.c_int, vp)
        self._deq = self.fn("dequant_block", None, vp, C.c_int, vp)
        self._mm = self.fn("mm", C.c_int, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, C.c_int)
        self._rowdot = self.fn("row_dot_f32", C.c_float, vp, vp, C.c_int, C.c_int)
        self._rope = self.fn("rope_neox", None, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, vp)
        self._attn = self.fn("attention", None, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int)
        self._logits = self.fn("logits_tied", None, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, vp)
        self._argmax = self.fn("argmax_first", C.c_int, vp, C.c_int)
        self._rms = self.fn("rmsnorm", None, vp, vp, vp, C.c_int, C.c_float)
        self._gelu = self.fn("gelu", C.c_float, C.c_float)
        self._mcreate = self.fn("model_create", vp, vp, C.c_int)
        self._mfree = self.fn("model_free", None, vp)
        self._fwd = self.fn("forward", C.c_int, vp, C.c_int, C.c_int, C.c_int)
        self._mlog = self.fn("model_logits", fp, vp)
        self._mx = self.fn("model_x", fp, vp)
        self._mkc = self.fn("model_kc", fp, vp, C.c_int, C.c_int)
        self._mvc = self.fn("model_vc", fp, vp, C.c_int, C.c_int)
        self._gen = self.fn("generate_greedy", C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, vp)

    def quantize_q8K(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = q8_buffer(x.size)
        self._q8(_p(x), _p(y), x.size)
        return y

    def block_sums(self, w: np.ndarray, t: int, n: int, d: int, q8: np.ndarray):
        nb = n // 256
        bb = {12: 144, 13: 176}[t]
        wv = w.reshape(d, nb * bb)
        ss = np.zeros((d, nb), np.int32)
        sm = np.zeros((d, nb), np.int32)
        a = C.c_int()
        b = C.c_int()
        base = w.ctypes.data
        qb = q8.ctypes.data
        for r in range(d):
            for k in range(nb):
                self._bsums(C.c_void_p(base + r * nb * bb + k * bb), t, C.c_void_p(qb + k * Q8_BYTES),
                            C.byref(a), C.byref(b))
                ss[r, k], sm[r, k] = a.value, b.value
        del wv
        return ss, sm

    def dequant(self, blocks: np.ndarray, t: int, nblocks: int) -> np.ndarray:
        bb = {12: 144, 13: 176, 14: 210}[t]
        out = np.zeros(nblocks * 256, np.float32)
        for b in range(nblocks):
            self._deq(C.c_void_p(blocks.ctypes.data + b * bb), t, C.c_void_p(out.ctypes.data + b * 1024))
        return out

    def mm(self, x, w, n, d, t, q8=None, q8_ready=0):
        o = np.zeros(d, np.float32)
        q8 = q8_buffer(max(n, 256)) if q8 is None else q8
        rc = self._mm(_p(o), _p(np.ascontiguousarray(x, np.float32)), _p(w), n, d, t, _p(q8), q8_ready)
        if rc != 0:
            raise ValueError("oracle mm rejected type %d / n %d" % (t, n))
        return o

    def rope(self, vec, n_heads, hd, n_rot, pos, base, fscale=1.0, ff=None):
        v = np.array(vec, dtype=np.float32, copy=True)
        self._rope(_p(v), n_heads, hd, n_rot, pos, base, fscale, _p(ff))
        return v

    def attention(self, q, k, v, nwin, kv_stride, n_heads, n_kv, hd):
        out = np.zeros(n_heads * hd, np.float32)
        self._attn(_p(out), _p(q), _p(k), _p(v), nwin, kv_stride, n_heads, n_kv, hd)
        return out

    def logits_tied(self, x, embd, t, dim, vocab, cap):
        lg = np.zeros(vocab, np.float32)
        self._logits(_p(lg), _p(np.ascontiguousarray(x, np.float32)), _p(embd), t, dim, vocab, cap,
                     _p(q8_buffer(dim)))
        return lg

    def argmax_first(self, v):
        v = np.ascontiguousarray(v, np.float32)
        return self._argmax(_p(v), v.size)

    def rmsnorm(self, x, w, eps):
        o = np.zeros_like(x, dtype=np.float32)
        self._rms(_p(o), _p(x), _p(w), x.size, eps)
        return o

    def gelu(self, x: float) -> float:
        return self._gelu(x)

    # --- whole model ---
    def model(self, desc, max_seq):
        return _Model(self, self._mcreate(C.byref(desc), max_seq), desc, "or")


class Reference(_Lib):
    """gemma4-4b/cpu-blas/main.c compiled unchanged."""

    def __init__(self, path: str = REF_SO, threads: int | None = None):
        super().__init__(path, "ref_")
        self.fn("set_threads", None, C.c_int)(threads or 0)
        self.max_threads = self.fn("max_threads", C.c_int)()
        self._q8 = self.fn("quantize_row_q8_K", None, vp, vp, C.c_int)
        self._q8s = self.fn("quantize_row_q8_K_scalar", None, vp, vp, C.c_int)
        self._vd4 = self.fn("vec_dot_q4_K_q8_K", None, C.c_int, vp, vp, vp)
        self._vd5 = self.fn("vec_dot_q5_K_q8_K", None, C.c_int, vp, vp, vp)
        self._vd4g = self.fn("vec_dot_q4_K_q8_K_generic", None, C.c_int, vp, vp, vp)
        self._vd5g = self.fn("vec_dot_q5_K_q8_K_generic", None, C.c_int, vp, vp, vp)
        self._deq = self.fn("dequant", None, vp, C.c_int, vp, C.c_int)
        self._mm = self.fn("mm", None, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, C.c_int)
        self._argmax_row = self.fn("mm_argmax_row", C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, vp)
        self._rope = self.fn("apply_rope_neox", None, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, vp)
        self._rms = self.fn("rmsnorm", None, vp, vp, vp, C.c_int, C.c_float)
        self._softmax = self.fn("softmax", None, vp, C.c_int)
        self._gelu = self.fn("gelu", C.c_float, C.c_float)
        self._sample = self.fn("sample_token", C.c_int, vp, C.c_int, C.c_float, C.c_float, C.c_int, vp)
        self._mcreate = self.fn("model_create", vp, vp, C.c_int)
        self._mfree = self.fn("model_free", None, vp)
        self._fwd = self.fn("forward", None, vp, C.c_int, C.c_int, C.c_int)
        self._mlog = self.fn("model_logits", fp, vp)
        self._marg = self.fn("model_argmax", C.c_int, vp)
        self._mx = self.fn("model_x", fp, vp)
        self._mkc = self.fn("model_kc", fp, vp, C.c_int, C.c_int)
        self._mvc = self.fn("model_vc", fp, vp, C.c_int, C.c_int)
        self._gen = self.fn("generate_greedy", C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, vp)
        self._fillkv = self.fn("model_fill_kv", None, vp, C.c_int, C.c_uint64)
        self._gens = self.fn("generate_sample", C.c_int, vp, vp, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float,
                             C.c_int, C.c_uint64, C.c_int, vp)
        self._pen = self.fn("apply_repetition_penalty", None, vp, vp, C.c_int, C.c_float, C.c_int)
        try:
            with open(os.path.join(os.path.dirname(path), "BLAS")) as f:
                self.blas = f.read().strip()
        except OSError:
            self.blas = "unknown"

    def quantize_q8K(self, x, scalar=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = q8_buffer(x.size)
        (self._q8s if scalar else self._q8)(_p(x), _p(y), x.size)
        return y

    def vec_dot(self, t, n, row, q8, generic=False):
        out = C.c_float()
        f = {(12, False): self._vd4, (13, False): self._vd5, (12, True): self._vd4g, (13, True): self._vd5g}[(t, generic)]
        f(n, _p(row), _p(q8), C.byref(out))
        return out.value

    def dequant(self, blocks, t, nblocks):
        out = np.zeros(nblocks * 256, np.float32)
        self._deq(_p(blocks), t, _p(out), nblocks)
        return out

    def mm(self, x, w, n, d, t, q8=None, q8_ready=0):
        o = np.zeros(d, np.float32)
        q8 = q8_buffer(max(n, 256)) if q8 is None else q8
        self._mm(_p(o), _p(np.ascontiguousarray(x, np.float32)), _p(w), n, d, t, _p(q8), q8_ready)
        return o

    def mm_argmax_row(self, x, w, n, d, t):
        return self._argmax_row(_p(np.ascontiguousarray(x, np.float32)), _p(w), n, d, t, _p(q8_buffer(n)))

    def rope(self, vec, n_heads, hd, n_rot, pos, base, fscale=1.0, ff=None):
        v = np.array(vec, dtype=np.float32, copy=True)
        self._rope(_p(v), n_heads, hd, n_rot, pos, base, fscale, _p(ff))
        return v

    def rmsnorm(self, x, w, eps):
        o = np.zeros_like(x, dtype=np.float32)
        self._rms(_p(o), _p(x), _p(w), x.size, eps)
        return o

    def softmax(self, x):
        v = np.array(x, dtype=np.float32, copy=True)
        self._softmax(_p(v), v.size)
        return v

    def gelu(self, x):
        return self._gelu(x)

    def sample(self, logits, temp, topp, topk, rng_state):
        """sample_token on a copy of the logits; returns (token, new rng state)."""
        v = np.array(logits, dtype=np.float32, copy=True)
        rng = C.c_uint64(rng_state)
        t = self._sample(_p(v), v.size, temp, topp, topk, C.byref(rng))
        return t, rng.value

    def repetition_penalty(self, logits, tokens, penalty, last_n):
        v = np.array(logits, dtype=np.float32, copy=True)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        self._pen(_p(v), _p(t), t.size, penalty, last_n)
        return v

    def sample_greedy(self, logits):
        v = np.ascontiguousarray(logits, np.float32)
        rng = C.c_uint64(1)
        return self._sample(_p(v), v.size, 0.0, 0.9, 40, C.byref(rng))

    def model(self, desc, max_seq):
        return _Model(self, self._mcreate(C.byref(desc), max_seq), desc, "ref")


class _Model:
    def __init__(self, lib, handle, desc, kind):
        self.lib, self.h, self.desc, self.kind = lib, handle, desc, kind
        self.vocab = desc.vocab_size
        self.dim = desc.dim

    def forward(self, token, pos, lm_mode=1):
        r = self.lib._fwd(self.h, token, pos, lm_mode)
        if self.kind == "ref":
            return self.lib._marg(self.h) if lm_mode == 2 else None
        return r

    def logits(self):
        return np.ctypeslib.as_array(self.lib._mlog(self.h), shape=(self.vocab,)).copy()

    def hidden(self):
        return np.ctypeslib.as_array(self.lib._mx(self.h), shape=(self.dim,)).copy()

    def kv(self, layer, pos, n):
        k = np.ctypeslib.as_array(self.lib._mkc(self.h, layer, pos), shape=(n,)).copy()
        v = np.ctypeslib.as_array(self.lib._mvc(self.h, layer, pos), shape=(n,)).copy()
        return k, v

    def fill_kv(self, npos, seed=1):
        self.lib._fillkv(self.h, npos, seed)

    def generate_sample(self, prompt, max_new, temp, topp=0.9, repeat_penalty=1.0, penalty_last_n=64, seed=1, eos=-1):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = self.lib._gens(self.h, _p(p), p.size, max_new, temp, topp, repeat_penalty, penalty_last_n, seed, eos, _p(out))
        return out[:n]

    def generate_greedy(self, prompt, max_new, eos=-1):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = self.lib._gen(self.h, _p(p), p.size, max_new, eos, _p(out))
        return out[:n]

    def close(self):
        if self.h:
            self.lib._mfree(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def have_reference() -> bool:
    return os.path.exists(REF_SO)
