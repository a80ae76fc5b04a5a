"""Seeded synthetic inputs for the Gemma 4 E4B Q4_K_M hot path.

There is no network and no real GGUF here, so every benchmark and parity test
runs on seeded synthetic tensors with the shapes and value distributions of
the reference's configurations:

* random K-quant super-blocks in the exact GGUF byte layouts of
  gemma4-4b/cpu-blas/main.c:95-115 (Q4_K 144 B, Q5_K 176 B, Q6_K 210 B per
  256 weights), with fp16 d/dmin and uniformly random 4/5/6-bit quants and
  6-bit (Q4/Q5) or int8 (Q6) sub-block scales;
* a random-init model shaped like Gemma 4 E4B (42 layers, d_model 2560, FFN
  10240, 8:2 GQA, head_dim 256, PLE 256, vocab 262144, window 512, tied
  Q6_K head) at "small-scale" init: d is chosen so dequantized weights have an
  RMS near 1/sqrt(n_in) and logits stay well below the softcap of 30, so
  greedy decoding is not dominated by ties at the cap.

Host tensors are numpy arrays; `SynthModel.desc()` returns a ctypes
g4_model_desc pointing into them (the arrays must outlive every user).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

F32, F16, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 12, 13, 14, 30
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
QK_K = 256


def row_bytes(t: int, n: int) -> int:
    if t == F32:
        return 4 * n
    if t in (F16, BF16):
        return 2 * n
    return (n // QK_K) * BLOCK_BYTES[t]


def _uniform_f16(rng, shape, lo, hi):
    return rng.uniform(lo, hi, size=shape).astype(np.float16).view(np.uint8).reshape(*shape, 2)


def random_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniformly random bytes (uint8[n], writable) from the generator's raw
    64-bit output (an order of magnitude faster than Generator.bytes)."""
    words = rng.bit_generator.random_raw((n + 7) // 8)
    return words.view(np.uint8)[:n]


def rand_blocks(rng: np.random.Generator, t: int, rows: int, n: int, d_lo: float, d_hi: float,
                dmin_lo: float | None = None, dmin_hi: float | None = None) -> np.ndarray:
    """Random `rows` x `n` tensor of type t (Q4_K/Q5_K/Q6_K) as uint8[rows, row_bytes].

    Quant bits and scale bytes are uniform random bytes (every 6-bit scale and
    min of the 12-byte K4 scale field is then uniform in [0, 63]; Q6_K scales
    uniform in [-128, 127]); d (and dmin) are fp16 uniform in [lo, hi]."""
    assert n % QK_K == 0
    nb = n // QK_K
    bb = BLOCK_BYTES[t]
    raw = random_bytes(rng, rows * nb * bb).reshape(rows, nb, bb)
    if t in (Q4_K, Q5_K):
        raw[..., 0:2] = _uniform_f16(rng, (rows, nb), d_lo, d_hi)
        lo = d_lo if dmin_lo is None else dmin_lo
        hi = d_hi if dmin_hi is None else dmin_hi
        raw[..., 2:4] = _uniform_f16(rng, (rows, nb), lo, hi)
    else:
        raw[..., 208:210] = _uniform_f16(rng, (rows, nb), d_lo, d_hi)
    return raw.reshape(rows, nb * bb)


def rand_bf16(rng, rows, n, std):
    w = (rng.standard_normal((rows, n), dtype=np.float32) * np.float32(std))
    return (w.view(np.uint32) >> 16).astype(np.uint16)  # truncation to bf16


def rand_f16(rng, rows, n, std):
    return (rng.standard_normal((rows, n), dtype=np.float32) * np.float32(std)).astype(np.float16).view(np.uint16)


def config0_weights(seed: int = 0, rows: int = 10240, n: int = 2560, t: int = Q4_K):
    """Config 0: Q4_K 10240 x 2560, d/dmin ~ U(1e-3, 2e-2), x ~ N(0,1) fp32[n]."""
    rng = np.random.default_rng(seed)
    w = rand_blocks(rng, t, rows, n, 1e-3, 2e-2)
    x = rng.standard_normal(n, dtype=np.float32)
    return w, x


# ---------------------------------------------------------------------------
# Synthetic model
# ---------------------------------------------------------------------------

@dataclass
class ModelShape:
    n_layers: int = 42
    dim: int = 2560
    hidden_dim: int = 10240
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim_swa: int = 256
    head_dim_full: int = 256
    n_rot_swa: int = 256
    n_rot_full: int = 256
    ple_dim: int = 256
    vocab_size: int = 262144
    sliding_window: int = 512
    swa_pattern: int = 6
    rope_theta: float = 1e6
    rope_theta_swa: float = 1e4
    norm_eps: float = 1e-6
    logit_softcapping: float = 30.0
    # tensor types: the Q4_K_M mix (Q/K/O/gate/up Q4_K, V/down Q6_K, BF16 per-layer-embedding matrices)
    wq_t: int = Q4_K
    wk_t: int = Q4_K
    wv_t: int = Q6_K
    wo_t: int = Q4_K
    gate_t: int = Q4_K
    up_t: int = Q4_K
    down_t: int = Q6_K
    inp_gate_t: int = BF16
    proj_t: int = BF16
    embd_t: int = Q6_K
    ple_tok_t: int = Q6_K
    ple_proj_t: int = BF16
    with_rope_freqs: bool = True
    with_out_scale: bool = True


E4B = ModelShape()
# The real E4B global layers use head_dim 512 with p-RoPE (true-E4B variant).
E4B_TRUE = ModelShape(head_dim_full=512, n_rot_full=512)
# Small shapes for fast parity tests: 30 layers so layers 24..29 read the
# shared KV of layers 22 (SWA) and 23 (global), as main.c:739-746 hard-codes.
TINY = ModelShape(n_layers=30, dim=512, hidden_dim=1024, head_dim_swa=64, head_dim_full=128,
                  n_rot_swa=64, n_rot_full=128, ple_dim=128, vocab_size=4096, sliding_window=16)
# Every projection on an fp32 path (Q6_K dequant-dot, dense): no Q8_K
# activation rounding, so a forward is reproducible to float summation order
# and greedy streams can be compared token for token over long horizons.
TINY_F = ModelShape(n_layers=30, dim=512, hidden_dim=1024, head_dim_swa=64, head_dim_full=128,
                    n_rot_swa=64, n_rot_full=128, ple_dim=128, vocab_size=4096, sliding_window=16,
                    wq_t=Q6_K, wk_t=Q6_K, wv_t=Q6_K, wo_t=Q6_K, gate_t=Q6_K, up_t=Q6_K, down_t=Q6_K,
                    inp_gate_t=F16, proj_t=F32, ple_proj_t=BF16)
TINY_Q5 = ModelShape(n_layers=30, dim=512, hidden_dim=1024, head_dim_swa=64, head_dim_full=128,
                     n_rot_swa=64, n_rot_full=128, ple_dim=128, vocab_size=4096, sliding_window=16,
                     wq_t=Q5_K, wo_t=Q5_K, up_t=Q5_K, down_t=Q4_K, wv_t=Q6_K, embd_t=Q6_K,
                     inp_gate_t=F16, proj_t=F32, ple_proj_t=BF16)


def is_swa(shape: ModelShape, l: int) -> bool:
    """Fallback layer pattern of main.c:716-721 (global when l % 6 == 5)."""
    if shape.swa_pattern <= 0:
        return False
    return (l % shape.swa_pattern) < (shape.swa_pattern - 1)


class Desc(C.Structure):
    """ctypes mirror of g4_model_desc (include/g4b200.h)."""
    _fields_ = [
        ("dim", C.c_int), ("hidden_dim", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int), ("vocab_size", C.c_int), ("ple_dim", C.c_int), ("sliding_window", C.c_int),
        ("head_dim_swa", C.c_int), ("head_dim_full", C.c_int), ("n_rot_swa", C.c_int), ("n_rot_full", C.c_int),
        ("rope_theta", C.c_float), ("rope_theta_swa", C.c_float), ("norm_eps", C.c_float),
        ("logit_softcapping", C.c_float),
        ("swa_layers", C.POINTER(C.c_int)), ("swa_pattern", C.c_int),
        ("embd", C.c_void_p), ("embd_t", C.c_int),
        ("ple_tok", C.c_void_p), ("ple_tok_t", C.c_int),
        ("ple_proj", C.c_void_p), ("ple_proj_t", C.c_int),
        ("ple_proj_norm", C.c_void_p), ("rope_freqs", C.c_void_p), ("norm_out", C.c_void_p),
        ("attn_norm", C.POINTER(C.c_void_p)), ("post_attn_norm", C.POINTER(C.c_void_p)),
        ("ffn_norm", C.POINTER(C.c_void_p)), ("post_ffw_norm", C.POINTER(C.c_void_p)),
        ("q_norm", C.POINTER(C.c_void_p)), ("k_norm", C.POINTER(C.c_void_p)),
        ("post_norm", C.POINTER(C.c_void_p)), ("out_scale", C.POINTER(C.c_void_p)),
        ("wq", C.POINTER(C.c_void_p)), ("wq_t", C.POINTER(C.c_int)),
        ("wk", C.POINTER(C.c_void_p)), ("wk_t", C.POINTER(C.c_int)),
        ("wv", C.POINTER(C.c_void_p)), ("wv_t", C.POINTER(C.c_int)),
        ("wo", C.POINTER(C.c_void_p)), ("wo_t", C.POINTER(C.c_int)),
        ("gate", C.POINTER(C.c_void_p)), ("gate_t", C.POINTER(C.c_int)),
        ("up", C.POINTER(C.c_void_p)), ("up_t", C.POINTER(C.c_int)),
        ("down", C.POINTER(C.c_void_p)), ("down_t", C.POINTER(C.c_int)),
        ("inp_gate", C.POINTER(C.c_void_p)), ("inp_gate_t", C.POINTER(C.c_int)),
        ("proj", C.POINTER(C.c_void_p)), ("proj_t", C.POINTER(C.c_int)),
    ]


def _ptr(a):
    return None if a is None else a.ctypes.data


@dataclass
class SynthModel:
    shape: ModelShape
    seed: int
    t: dict = field(default_factory=dict)          # global tensors
    layers: list = field(default_factory=list)     # per-layer dict of tensors
    _keep: list = field(default_factory=list)

    def weight_bytes(self) -> int:
        total = sum(a.nbytes for a in self.t.values() if a is not None)
        for lt in self.layers:
            total += sum(a.nbytes for a in lt.values() if a is not None)
        return total

    def streamed_bytes(self, batch: int) -> int:
        """Weight bytes one decode step reads for `batch` sequences: every
        tensor once, except the per-layer token table, of which only the
        `batch` token rows are gathered (emb_lookup, main.c:1696-1723)."""
        ple = self.t["ple_tok"]
        return self.weight_bytes() - ple.nbytes + batch * (ple.nbytes // ple.shape[0])

    def desc(self) -> Desc:
        s = self.shape
        L = s.n_layers
        d = Desc()
        d.dim, d.hidden_dim, d.n_layers = s.dim, s.hidden_dim, L
        d.n_heads, d.n_kv_heads, d.vocab_size = s.n_heads, s.n_kv_heads, s.vocab_size
        d.ple_dim, d.sliding_window = s.ple_dim, s.sliding_window
        d.head_dim_swa, d.head_dim_full, d.n_rot_swa, d.n_rot_full = (
            s.head_dim_swa, s.head_dim_full, s.n_rot_swa, s.n_rot_full)
        d.rope_theta, d.rope_theta_swa = s.rope_theta, s.rope_theta_swa
        d.norm_eps, d.logit_softcapping = s.norm_eps, s.logit_softcapping
        d.swa_layers = None
        d.swa_pattern = s.swa_pattern
        d.embd, d.embd_t = _ptr(self.t["embd"]), s.embd_t
        d.ple_tok, d.ple_tok_t = _ptr(self.t["ple_tok"]), s.ple_tok_t
        d.ple_proj, d.ple_proj_t = _ptr(self.t["ple_proj"]), s.ple_proj_t
        d.ple_proj_norm = _ptr(self.t["ple_proj_norm"])
        d.rope_freqs = _ptr(self.t.get("rope_freqs"))
        d.norm_out = _ptr(self.t["norm_out"])

        def parr(key):
            arr = (C.c_void_p * L)(*[_ptr(lt.get(key)) for lt in self.layers])
            self._keep.append(arr)
            return C.cast(arr, C.POINTER(C.c_void_p))

        def tarr(key):
            arr = (C.c_int * L)(*([getattr(s, key + "_t")] * L))
            self._keep.append(arr)
            return C.cast(arr, C.POINTER(C.c_int))

        for k in ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffw_norm", "q_norm", "k_norm",
                  "post_norm", "out_scale"):
            setattr(d, k, parr(k))
        for k in ("wq", "wk", "wv", "wo", "gate", "up", "down", "inp_gate", "proj"):
            setattr(d, k, parr(k))
            setattr(d, k + "_t", tarr(k))
        return d


def _qmat(rng, t, rows, n, rms):
    """Random K-quant / dense matrix whose dequantized RMS is about `rms`."""
    if t == Q4_K or t == Q5_K:
        # w = d*sc*q - dmin*m, sc, m ~ U[0,63], q ~ U[0,15] (Q5: U[0,31]);
        # dmin = 7.5 d (15.5 d) centres w; then RMS(w) ~ 255 d (~520 d).
        qmid, k = (7.5, 255.0) if t == Q4_K else (15.5, 520.0)
        d = rms / k
        return rand_blocks(rng, t, rows, n, 0.5 * d, 1.5 * d, qmid * 0.9 * d, qmid * 1.1 * d)
    if t == Q6_K:
        d = rms / 1367.0   # RMS of sc * (q - 32) with sc ~ U[-128,127], q ~ U[0,63]
        return rand_blocks(rng, t, rows, n, 0.5 * d, 1.5 * d)
    if t == BF16:
        return rand_bf16(rng, rows, n, rms)
    if t == F16:
        return rand_f16(rng, rows, n, rms)
    if t == F32:
        return rng.standard_normal((rows, n), dtype=np.float32) * np.float32(rms)
    raise ValueError(t)


def _norm_w(rng, n):
    return rng.uniform(0.8, 1.2, size=n).astype(np.float32)


def make_model(shape: ModelShape = E4B, seed: int = 3, logit_std: float = 3.0, post_scale: float = 1.0,
               qk_scale: float | None = None) -> SynthModel:
    """Random-init model of `shape` (seeded), small-scale init (see module doc).

    Two choices keep the random network's dynamics tame, as a trained one
    is: the q/k norm weights are scaled by hd**-0.25 (attention scores of
    unit variance instead of O(hd), which would make the softmax an argmax
    over positions), and the three post-sublayer norm weights by
    `post_scale` (1 by default).  With unscaled q/k norms the reference
    disagrees with itself (AVX2 vs generic dot builds) on greedy tokens
    within a few positions."""
    s = shape
    rng = np.random.default_rng(seed)
    m = SynthModel(shape=s, seed=seed)
    L = s.n_layers
    m.t["embd"] = _qmat(rng, s.embd_t, s.vocab_size, s.dim, logit_std / np.sqrt(s.dim))
    m.t["ple_tok"] = _qmat(rng, s.ple_tok_t, s.vocab_size, s.ple_dim * L, 1.0 / np.sqrt(s.ple_dim))
    m.t["ple_proj"] = _qmat(rng, s.ple_proj_t, s.ple_dim * L, s.dim, 1.0 / np.sqrt(s.dim))
    m.t["ple_proj_norm"] = _norm_w(rng, s.ple_dim)
    m.t["norm_out"] = _norm_w(rng, s.dim)
    if s.with_rope_freqs:
        ff = np.ones(s.n_rot_full // 2, dtype=np.float32)
        ff[s.n_rot_full // 8:] = 1e30   # p-RoPE: only the first quarter of the pairs rotates
        m.t["rope_freqs"] = ff
    for l in range(L):
        swa = is_swa(s, l)
        hd = s.head_dim_swa if swa else s.head_dim_full
        qd, kvd = s.n_heads * hd, s.n_kv_heads * hd
        lt = {}
        qk = (hd ** -0.25) if qk_scale is None else qk_scale
        lt["attn_norm"] = _norm_w(rng, s.dim)
        lt["post_attn_norm"] = _norm_w(rng, s.dim) * np.float32(post_scale)
        lt["ffn_norm"] = _norm_w(rng, s.dim)
        lt["post_ffw_norm"] = _norm_w(rng, s.dim) * np.float32(post_scale)
        lt["post_norm"] = _norm_w(rng, s.dim) * np.float32(post_scale)
        lt["q_norm"] = _norm_w(rng, hd) * np.float32(qk)
        lt["k_norm"] = _norm_w(rng, hd) * np.float32(qk)
        lt["out_scale"] = (rng.uniform(0.6, 1.0, size=1).astype(np.float32) if s.with_out_scale else None)
        lt["wq"] = _qmat(rng, s.wq_t, qd, s.dim, 1.0 / np.sqrt(s.dim))
        if l < 24:   # layers >= 24 reuse the KV of layers 22/23 (main.c:739-746)
            lt["wk"] = _qmat(rng, s.wk_t, kvd, s.dim, 1.0 / np.sqrt(s.dim))
            lt["wv"] = _qmat(rng, s.wv_t, kvd, s.dim, 1.0 / np.sqrt(s.dim))
        else:
            lt["wk"] = lt["wv"] = None
        lt["wo"] = _qmat(rng, s.wo_t, s.dim, qd, 1.0 / np.sqrt(qd))
        lt["gate"] = _qmat(rng, s.gate_t, s.hidden_dim, s.dim, 1.0 / np.sqrt(s.dim))
        lt["up"] = _qmat(rng, s.up_t, s.hidden_dim, s.dim, 1.0 / np.sqrt(s.dim))
        lt["down"] = _qmat(rng, s.down_t, s.dim, s.hidden_dim, 1.0 / np.sqrt(s.hidden_dim))
        lt["inp_gate"] = _qmat(rng, s.inp_gate_t, s.ple_dim, s.dim, 1.0 / np.sqrt(s.dim))
        lt["proj"] = _qmat(rng, s.proj_t, s.dim, s.ple_dim, 1.0 / np.sqrt(s.ple_dim))
        m.layers.append(lt)
    return m
