"""gemma4.c_b200 — Python view of libg4b200.so, the B200 (sm_100a) decode engine
for the Gemma 4 E4B Q4_K_M hot path of thamada/Gemma4.c.

The product is the C ABI in include/g4b200.h (the reference's C host calls it
directly).  This module binds the same entry points with ctypes, under the
reference's own names (quantize_row_q8_K, mm, mm_quant_rows, mm_argmax_row,
apply_rope_neox, logits_tied, forward, generate), for the tests and bench.py.
There is no CPU fallback: every call runs the CUDA kernels, and a missing or
unbuilt library raises.

The directory name is not a Python identifier; load it with
    importlib.util.spec_from_file_location("g4b200", ".../gemma4.c_b200/__init__.py",
                                           submodule_search_locations=[".../gemma4.c_b200"])
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import synth  # noqa: F401  (re-exported)
from .synth import BF16, F16, F32, Q4_K, Q5_K, Q6_K, Desc, row_bytes  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libg4b200.so")
Q8_BYTES = 292

G4_OK, G4_ERR_ARG, G4_ERR_TYPE, G4_ERR_CUDA, G4_ERR_OOM, G4_ERR_NO_DEVICE, G4_ERR_STATE, G4_ERR_TIMEOUT = range(8)


class G4Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__("g4 error %d: %s" % (code, msg))
        self.code = code


vp, ip, fp = C.c_void_p, C.c_int, C.c_float

# (name, restype, argtypes): every entry point of include/g4b200.h
SIGNATURES = [
    ("g4_last_error", ip, []),
    ("g4_last_error_string", C.c_char_p, []),
    ("g4_clear_error", None, []),
    ("g4_set_device", ip, [ip]),
    ("g4_registry_clear", ip, []),
    ("g4_registry_stats", ip, [vp, vp]),
    ("g4_kernel_launch_count", C.c_uint64, []),
    ("g4_quantize_row_q8_K", None, [vp, vp, ip]),
    ("g4_quantize_row_q8_K_ex", ip, [vp, vp, ip]),
    ("g4_vec_dot_q4_K_q8_K", None, [ip, vp, vp, vp]),
    ("g4_vec_dot_q5_K_q8_K", None, [ip, vp, vp, vp]),
    ("g4_vec_dot_q4_K_q8_K_ex", ip, [ip, vp, vp, vp]),
    ("g4_vec_dot_q5_K_q8_K_ex", ip, [ip, vp, vp, vp]),
    ("g4_quant_dot_block_sums", ip, [vp, ip, ip, ip, vp, vp, vp]),
    ("g4_mm", None, [vp, vp, vp, ip, ip, ip, vp, ip]),
    ("g4_mm_ex", ip, [vp, vp, vp, ip, ip, ip, vp, ip]),
    ("g4_mm_quant_dot_rows", None, [vp, vp, ip, ip, ip, vp]),
    ("g4_mm_quant_dot_rows_ex", ip, [vp, vp, ip, ip, ip, vp]),
    ("g4_mm_quant_rows", None, [vp, vp, vp, ip, ip, ip]),
    ("g4_mm_quant_rows_ex", ip, [vp, vp, vp, ip, ip, ip]),
    ("g4_mm_argmax_row", ip, [vp, vp, ip, ip, ip, vp]),
    ("g4_apply_rope_neox", None, [vp, ip, ip, ip, ip, fp, fp, vp]),
    ("g4_apply_rope_neox_ex", ip, [vp, ip, ip, ip, ip, fp, fp, vp]),
    ("g4_logits_tied", ip, [vp, vp, vp, vp, ip, ip, ip, fp]),
    ("g4_attn_decode", ip, [vp, vp, vp, vp, ip, ip, ip, ip, ip]),
    ("g4_sample_token", ip, [vp, ip, fp, fp, ip, vp]),
    ("g4d_weight_upload", ip, [vp, ip, ip, ip, vp]),
    ("g4d_free", ip, [vp]),
    ("g4d_quantize_row_q8_K", ip, [vp, vp, ip, ip, vp]),
    ("g4d_mm", ip, [vp, vp, vp, ip, ip, ip, vp, ip, ip, vp]),
    ("g4d_attn_decode_noalloc", ip, [vp, vp, vp, vp, ip, ip, ip, ip, vp]),
    ("g4_model_desc_bytes", C.c_size_t, []),
    ("g4_engine_create", vp, [vp, ip, ip, ip]),
    ("g4_engine_create_ex", vp, [vp, ip, ip, ip, ip]),
    ("g4_prefill", ip, [vp, ip, vp, vp, vp]),
    ("g4_engine_destroy", ip, [vp]),
    ("g4_engine_device_bytes", C.c_size_t, [vp]),
    ("g4_forward", ip, [vp, ip, ip, ip, vp]),
    ("g4_generate_greedy", ip, [vp, vp, ip, ip, ip, vp]),
    ("g4_decode_batch", ip, [vp, ip, vp, ip, ip, vp]),
    ("g4_generate", ip, [vp, vp, ip, ip, fp, fp, ip, fp, ip, C.c_uint64, ip, vp]),
    ("g4_decode_batch_sample", ip, [vp, ip, vp, ip, fp, fp, ip, fp, vp, ip, vp, vp, vp]),
    ("g4_decode_batch_device", ip, [vp, ip, vp, ip, ip, vp]),
    ("g4_engine_sync", ip, [vp]),
    ("g4_engine_stream", vp, [vp]),
    ("g4_engine_get_hidden", ip, [vp, ip, vp]),
    ("g4_engine_get_kv", ip, [vp, ip, ip, ip, vp, vp]),
    ("g4_engine_set_kv", ip, [vp, ip, ip, ip, ip, vp, vp]),
    ("g4_engine_last_step_kernels", ip, [vp]),
    ("g4_engine_fill_kv", ip, [vp, ip, C.c_uint64]),
    ("g4_engine_time_attention", ip, [vp, vp, ip, ip, ip, vp]),
    ("g4_set_tc_min_batch", ip, [ip]),
    ("g4_set_gemv_rows", ip, [ip]),
    ("g4_nccl_unique_id", ip, [vp]),
    ("g4_engine_lm_split", ip, [vp, vp, ip, ip]),
    ("g4_lm_split_rows", ip, [ip, ip, ip, vp, vp]),
    ("g4_lm_split_merge", ip, [vp, ip, ip, ip, ip, vp]),
    ("g4_argmax_keys", ip, [vp, ip, ip, vp]),
    ("g4_engine_set_tc_min_batch", ip, [vp, ip]),
    ("g4_engine_set_attn_split", ip, [vp, ip, ip]),
]

_lib = None


def lib() -> C.CDLL:
    """The loaded libg4b200.so (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libg4b200.so is not built; run `python gemma4.c_b200/build.py` "
                               "(or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _check(rc: int):
    if rc != 0:
        L = lib()
        raise G4Error(rc, (L.g4_last_error_string() or b"").decode())


def last_error():
    L = lib()
    return L.g4_last_error(), (L.g4_last_error_string() or b"").decode()


def q8_buffer(n: int) -> np.ndarray:
    return np.zeros(((n + 255) // 256) * Q8_BYTES, dtype=np.uint8)


# ------------------------------------------------------------------ per-call API
def quantize_row_q8_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = q8_buffer(x.size)
    _check(lib().g4_quantize_row_q8_K_ex(_p(x), _p(y), x.size))
    return y


def vec_dot(t: int, n: int, row: np.ndarray, q8: np.ndarray) -> float:
    out = C.c_float()
    f = lib().g4_vec_dot_q4_K_q8_K_ex if t == Q4_K else lib().g4_vec_dot_q5_K_q8_K_ex
    _check(f(n, _p(row), _p(q8), C.byref(out)))
    return out.value


def block_sums(w: np.ndarray, n: int, d: int, t: int, q8: np.ndarray):
    nb = n // 256
    ss = np.zeros((d, nb), np.int32)
    sm = np.zeros((d, nb), np.int32)
    _check(lib().g4_quant_dot_block_sums(_p(w), n, d, t, _p(q8), _p(ss), _p(sm)))
    return ss, sm


def mm(x, w, n, d, t, q8=None, q8_ready=0):
    o = np.zeros(d, np.float32)
    if q8 is None:
        q8 = q8_buffer(max(n, 256))
    xa = None if x is None else np.ascontiguousarray(x, np.float32)
    _check(lib().g4_mm_ex(_p(o), _p(xa), _p(w), n, d, t, _p(q8), q8_ready))
    return o


def mm_quant_dot_rows(w, n, d, t, q8):
    o = np.zeros(d, np.float32)
    _check(lib().g4_mm_quant_dot_rows_ex(_p(o), _p(w), n, d, t, _p(q8)))
    return o


def mm_quant_rows(x, w, n, d, t):
    o = np.zeros(d, np.float32)
    _check(lib().g4_mm_quant_rows_ex(_p(o), _p(np.ascontiguousarray(x, np.float32)), _p(w), n, d, t))
    return o


def mm_argmax_row(x, w, n, d, t, q8=None):
    q8 = q8_buffer(n) if q8 is None else q8
    r = lib().g4_mm_argmax_row(_p(np.ascontiguousarray(x, np.float32)), _p(w), n, d, t, _p(q8))
    if r < 0:
        _check(lib().g4_last_error() or G4_ERR_CUDA)
    return r


def apply_rope_neox(vec, n_heads, hd, n_rot, pos, base, fscale=1.0, ff=None):
    v = np.array(vec, dtype=np.float32, copy=True)
    _check(lib().g4_apply_rope_neox_ex(_p(v), n_heads, hd, n_rot, pos, base, fscale, _p(ff)))
    return v


def logits_tied(x, embd, t, dim, vocab, cap, want_logits=True):
    lg = np.zeros(vocab, np.float32) if want_logits else None
    am = C.c_int(-1)
    _check(lib().g4_logits_tied(_p(lg), C.byref(am), _p(np.ascontiguousarray(x, np.float32)), _p(embd), t, dim,
                                vocab, cap))
    return lg, am.value


def attn_decode(q, k, v, nwin, kv_stride, n_heads, n_kv, hd):
    out = np.zeros(n_heads * hd, np.float32)
    _check(lib().g4_attn_decode(_p(out), _p(q), _p(k), _p(v), nwin, kv_stride, n_heads, n_kv, hd))
    return out


def sample_token(logits, temp: float, topp: float, topk: int, rng_state: int):
    """sample_token (main.c:2044-2112) on host logits; returns (token, new rng state)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    st = C.c_uint64(rng_state)
    r = lib().g4_sample_token(_p(lg), lg.size, temp, topp, topk, C.byref(st))
    if r < 0:
        _check(lib().g4_last_error() or G4_ERR_ARG)
    return r, st.value


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().g4_nccl_unique_id(buf))
    return buf.raw


def lm_split_rows(vocab: int, world: int, rank: int):
    r0, r1 = C.c_int(), C.c_int()
    chunk = lib().g4_lm_split_rows(vocab, world, rank, C.byref(r0), C.byref(r1))
    if chunk < 0:
        _check(G4_ERR_ARG)
    return chunk, r0.value, r1.value


def lm_split_merge(keys_all: np.ndarray, world: int, rank: int, B: int, chunk: int) -> np.ndarray:
    ka = np.ascontiguousarray(keys_all, dtype=np.uint64)
    out = np.zeros(B, np.uint64)
    _check(lib().g4_lm_split_merge(_p(ka), world, rank, B, chunk, _p(out)))
    return out


def argmax_key(logits, row0: int = 0) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    k = C.c_uint64()
    _check(lib().g4_argmax_keys(_p(lg), lg.size, row0, C.byref(k)))
    return k.value


def weight_upload(host: np.ndarray, t: int, n: int, rows: int) -> int:
    """Device copy of a weight tensor (device layout); returns the pointer."""
    d = C.c_void_p()
    _check(lib().g4d_weight_upload(_p(host), t, n, rows, C.byref(d)))
    return d.value


def free(dev: int):
    _check(lib().g4d_free(dev))


def mm_device(o, x, w, n, d, t, q8, q8_ready, batch, stream):
    """g4d_mm on raw device pointers (ints)."""
    _check(lib().g4d_mm(o, x, w, n, d, t, q8, q8_ready, batch, stream))


def set_tc_min_batch(b: int) -> int:
    """Batch size from which g4d_mm runs Q4_K/Q5_K on the tensor cores; returns the previous value."""
    r = lib().g4_set_tc_min_batch(b)
    if r < 0:
        _check(G4_ERR_ARG)
    return r


def set_gemv_rows(on: bool) -> int:
    """Batch-1 Q4_K/Q5_K GEMVs on the row-owner kernel (True) or the tiled kernel; returns the previous."""
    return int(lib().g4_set_gemv_rows(1 if on else 0))


def registry_clear():
    _check(lib().g4_registry_clear())


def kernel_launch_count() -> int:
    return int(lib().g4_kernel_launch_count())


# ------------------------------------------------------------------ engine
class Engine:
    """Device-resident decode engine for one model on one GPU."""

    def __init__(self, model: "synth.SynthModel", device: int = 0, max_seq: int = 1024, max_batch: int = 1,
                 prefill_rows: int = 0):
        self.model = model          # keeps the host tensors alive while uploading
        self.desc = model.desc()
        self.vocab = self.desc.vocab_size
        self.dim = self.desc.dim
        self.max_batch = max_batch
        self.prefill_rows = prefill_rows
        h = lib().g4_engine_create_ex(C.byref(self.desc), device, max_seq, max_batch, prefill_rows)
        if not h:
            _check(lib().g4_last_error() or G4_ERR_CUDA)
        self.h = h

    def forward(self, token: int, pos: int, lm_mode: int = 1, want_logits: bool = False):
        lg = np.zeros(self.vocab, np.float32) if want_logits else None
        r = lib().g4_forward(self.h, token, pos, lm_mode, _p(lg))
        if r < 0:
            _check(lib().g4_last_error() or G4_ERR_CUDA)
        return (r, lg) if want_logits else r

    def generate_greedy(self, prompt, max_new: int, eos: int = -1) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = lib().g4_generate_greedy(self.h, _p(p), p.size, max_new, eos, _p(out))
        if n < 0:
            _check(lib().g4_last_error() or G4_ERR_CUDA)
        return out[:n]

    def generate(self, prompt, max_new: int, temp: float, topp: float = 0.9, topk: int = 40,
                 repeat_penalty: float = 1.0, penalty_last_n: int = 64, seed: int = 1, eos: int = -1) -> np.ndarray:
        """generate with the reference's sampler (temp > 0: top-k / top-p / repetition penalty)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = lib().g4_generate(self.h, _p(p), p.size, max_new, temp, topp, topk, repeat_penalty, penalty_last_n, seed,
                              eos, _p(out))
        if n < 0:
            _check(lib().g4_last_error() or G4_ERR_CUDA)
        return out[:n]

    def decode_batch_sample(self, tokens, pos: int, temp: float, topp: float, topk: int, rng,
                            repeat_penalty: float = 1.0, recent=None, n_recent=None):
        """One batched step with the sampler; rng is a uint64 array of per-sequence states (advanced in place)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(t.size, np.int32)
        assert rng.dtype == np.uint64 and rng.size == t.size
        rec = None if recent is None else np.ascontiguousarray(recent, dtype=np.int32)
        nr = None if n_recent is None else np.ascontiguousarray(n_recent, dtype=np.int32)
        _check(lib().g4_decode_batch_sample(self.h, t.size, _p(t), pos, temp, topp, topk, repeat_penalty, _p(rec),
                                            0 if rec is None else rec.shape[1], _p(nr), _p(rng), _p(nxt)))
        return nxt

    def prefill(self, seq, pos, tokens):
        """Batched prefill rows (sequence, position, token); see g4_prefill."""
        sq = np.ascontiguousarray(seq, dtype=np.int32)
        ps = np.ascontiguousarray(pos, dtype=np.int32)
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        assert sq.size == ps.size == tk.size
        _check(lib().g4_prefill(self.h, sq.size, _p(sq), _p(ps), _p(tk)))

    def prefill_prompts(self, prompts, upto: int):
        """Prefill positions [0, upto) of every sequence's prompt (prompts: [B][>= upto]) in calls of at
        most prefill_rows rows, interleaving the sequences position-major."""
        prompts = np.asarray(prompts, dtype=np.int32)
        B = prompts.shape[0]
        per = max(1, self.prefill_rows // B)  # positions per call
        for p0 in range(0, upto, per):
            p1 = min(upto, p0 + per)
            ps = np.repeat(np.arange(p0, p1, dtype=np.int32), B)
            sq = np.tile(np.arange(B, dtype=np.int32), p1 - p0)
            self.prefill(sq, ps, prompts[sq, ps])

    def decode_batch(self, tokens, pos: int, lm_mode: int = 1) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(t.size, np.int32)
        _check(lib().g4_decode_batch(self.h, t.size, _p(t), pos, lm_mode, _p(nxt)))
        return nxt

    def decode_batch_device(self, B: int, tokens_dev_ptr, pos: int, lm_mode: int, next_dev_ptr):
        _check(lib().g4_decode_batch_device(self.h, B, tokens_dev_ptr, pos, lm_mode, next_dev_ptr))

    def sync(self):
        _check(lib().g4_engine_sync(self.h))

    def stream(self) -> int:
        return lib().g4_engine_stream(self.h) or 0

    def hidden(self, b: int = 0) -> np.ndarray:
        x = np.zeros(self.dim, np.float32)
        _check(lib().g4_engine_get_hidden(self.h, b, _p(x)))
        return x

    def kv(self, layer: int, pos: int, n: int, b: int = 0):
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        _check(lib().g4_engine_get_kv(self.h, b, layer, pos, _p(k), _p(v)))
        return k, v

    def set_kv(self, layer: int, pos0: int, k, v, b: int = 0):
        """Write K/V rows [npos][n_kv*hd] of positions pos0.. of sequence b (test tap)."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        assert k.shape == v.shape and k.ndim == 2
        _check(lib().g4_engine_set_kv(self.h, b, layer, pos0, k.shape[0], _p(k), _p(v)))

    def fill_kv(self, npos: int, seed: int = 1):
        _check(lib().g4_engine_fill_kv(self.h, npos, seed))

    def time_attention(self, layers, batch: int, reps: int) -> float:
        """Milliseconds for `reps` rounds of the attention of `layers` (CUDA events, engine stream)."""
        ls = np.ascontiguousarray(layers, dtype=np.int32)
        ms = np.zeros(1, np.float32)
        _check(lib().g4_engine_time_attention(self.h, _p(ls), len(ls), batch, reps, _p(ms)))
        return float(ms[0])

    def lm_split(self, nccl_id: bytes, rank: int, world: int):
        """Row-split the LM head over `world` ranks (one engine per GPU); nccl_id from nccl_unique_id()."""
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        _check(lib().g4_engine_lm_split(self.h, buf, rank, world))

    def set_tc_min_batch(self, b: int) -> int:
        r = lib().g4_engine_set_tc_min_batch(self.h, b)
        if r < 0:
            _check(G4_ERR_ARG)
        return r

    def set_attn_split(self, sliding: int, global_: int):
        """Attention rows per CTA for sliding / global layers (multiples of 32; 0: default)."""
        _check(lib().g4_engine_set_attn_split(self.h, sliding, global_))

    def last_step_kernels(self) -> int:
        return int(lib().g4_engine_last_step_kernels(self.h))

    def device_bytes(self) -> int:
        return int(lib().g4_engine_device_bytes(self.h))

    def close(self):
        if getattr(self, "h", None):
            lib().g4_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
