"""Generate tests/golden/golden.npz from the reference engine itself.

    python tests/golden/make_golden.py

Runs gemma4-4b/cpu-blas/main.c compiled unchanged (oracle/_ref/libg4ref.so,
built by `make -C oracle`) on small seeded inputs and stores inputs and
outputs.  The reference has no golden vectors of its own for synthetic
inputs (its only goldens need the real E4B GGUF), so these fixtures pin the
C restatement in oracle/ and the CUDA kernels to the reference's behaviour.
Integer-valued outputs (Q8_K bytes, per-block integer sums, argmax indices,
greedy token ids) are exact; float outputs are the reference's AVX2/OpenBLAS
results.
"""
import importlib.util
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
PKG = os.path.join(ROOT, "gemma4.c_b200")
spec = importlib.util.spec_from_file_location("g4b200", os.path.join(PKG, "__init__.py"),
                                              submodule_search_locations=[PKG])
g4b200 = importlib.util.module_from_spec(spec)
sys.modules["g4b200"] = g4b200
spec.loader.exec_module(g4b200)
synth = g4b200.synth

import oracle  # noqa: E402

Q4, Q5, Q6, BF16, F16, F32 = 12, 13, 14, 30, 1, 0


def block_sums_via_reference(ref, w, t, n, d, q8):
    """Per-block integer sums from the reference's own generic dot: with the
    block's d = 1, dmin = 0 and the activation's d = 1 the result is exactly
    float(sumi_s); with d = 0, dmin = 1 it is -float(sumi_m)."""
    bb = {Q4: 144, Q5: 176}[t]
    nb = n // 256
    ss = np.zeros((d, nb), np.int64)
    sm = np.zeros((d, nb), np.int64)
    one, zero = np.float16(1.0).view(np.uint16), np.uint16(0)
    for k in range(nb):
        yb = q8.reshape(nb, 292)[k].copy()
        yb[0:4] = np.frombuffer(np.float32(1.0).tobytes(), np.uint8)
        for r in range(d):
            blk = w[r, k * bb:(k + 1) * bb].copy()
            blk[0:2] = np.frombuffer(one.tobytes(), np.uint8)
            blk[2:4] = np.frombuffer(zero.tobytes(), np.uint8)
            v = ref.vec_dot(t, 256, blk, yb, generic=True)
            assert abs(v) < 2 ** 24 and v == int(v)
            ss[r, k] = int(v)
            blk[0:2] = np.frombuffer(zero.tobytes(), np.uint8)
            blk[2:4] = np.frombuffer(one.tobytes(), np.uint8)
            v = ref.vec_dot(t, 256, blk, yb, generic=True)
            assert v == int(v)
            sm[r, k] = -int(v)
    return ss.astype(np.int32), sm.astype(np.int32)


def main():
    ref = oracle.Reference(threads=1)
    g = {}
    rng = np.random.default_rng(2024)
    # --- Q8_K quantization: scales, an all-zero block, ties of |x|, signed max
    xs = []
    for s in (1e-3, 1.0, 37.0, 1e4):
        xs.append(rng.standard_normal(512).astype(np.float32) * np.float32(s))
    z = rng.standard_normal(512).astype(np.float32)
    z[:256] = 0.0
    xs.append(z)
    t = rng.standard_normal(512).astype(np.float32)
    t[5], t[77] = -9.0, 9.0          # tie: the first index (negative) must win
    t[300], t[400] = 7.0, -7.0
    xs.append(t)
    g["q8_x"] = np.stack(xs)
    g["q8_out"] = np.stack([ref.quantize_q8K(x) for x in xs])
    for x, y in zip(xs, g["q8_out"]):
        assert (ref.quantize_q8K(x, scalar=True) == y).all()
    # --- Q4_K / Q5_K integer dots
    for t, name in ((Q4, "q4"), (Q5, "q5")):
        w = synth.rand_blocks(rng, t, 16, 512, 1e-3, 2e-2)
        x = rng.standard_normal(512).astype(np.float32)
        q8 = ref.quantize_q8K(x)
        g[name + "_w"], g[name + "_x"], g[name + "_q8"] = w, x, q8
        g[name + "_dot"] = np.array([ref.vec_dot(t, 512, w[r], q8) for r in range(16)], np.float32)
        g[name + "_dot_generic"] = np.array([ref.vec_dot(t, 512, w[r], q8, generic=True) for r in range(16)], np.float32)
        g[name + "_mm"] = ref.mm(x, w, 512, 16, t)
        g[name + "_ss"], g[name + "_sm"] = block_sums_via_reference(ref, w, t, 512, 16, q8)
        g[name + "_argmax"] = np.array(ref.mm_argmax_row(x, w, 512, 16, t), np.int32)
    # --- Q6_K fp32 dequant dot
    w6 = synth.rand_blocks(rng, Q6, 8, 512, 1e-3, 2e-2)
    x6 = rng.standard_normal(512).astype(np.float32)
    g["q6_w"], g["q6_x"] = w6, x6
    g["q6_mm"] = ref.mm(x6, w6, 512, 8, Q6)
    g["q6_deq0"] = ref.dequant(w6[0].copy(), Q6, 2)
    g["q6_argmax"] = np.array(ref.mm_argmax_row(x6, w6, 512, 8, Q6), np.int32)
    g["q4_deq0"] = ref.dequant(g["q4_w"][0].copy(), Q4, 2)
    g["q5_deq0"] = ref.dequant(g["q5_w"][0].copy(), Q5, 2)
    # --- dense GEMVs
    xd = rng.standard_normal(384).astype(np.float32)
    g["dense_x"] = xd
    for t, name in ((BF16, "bf16"), (F16, "f16"), (F32, "f32")):
        wd = synth._qmat(rng, t, 8, 384, 0.05)
        g[name + "_w"] = wd
        g[name + "_mm"] = ref.mm(xd, wd, 384, 8, t)
    # --- Neox RoPE at pos >= 1 (a pos-0 test is a false positive)
    v = rng.standard_normal(8 * 64).astype(np.float32)
    ff = np.ones(32, np.float32)
    ff[8:] = 1e30
    g["rope_in"], g["rope_ff"] = v, ff
    g["rope_pos"] = np.array([1, 7, 300, 8191], np.int32)
    g["rope_swa"] = np.stack([ref.rope(v, 8, 64, 64, int(p), 1e4) for p in g["rope_pos"]])
    g["rope_full"] = np.stack([ref.rope(v, 8, 64, 64, int(p), 1e6, 1.0, ff) for p in g["rope_pos"]])
    g["rope_partial"] = np.stack([ref.rope(v, 8, 64, 32, int(p), 1e4) for p in g["rope_pos"]])
    # --- softmax / gelu
    sx = (rng.standard_normal(100) * 5).astype(np.float32)
    g["softmax_in"], g["softmax_out"] = sx, ref.softmax(sx)
    gx = np.linspace(-6, 6, 97).astype(np.float32)
    g["gelu_in"], g["gelu_out"] = gx, np.array([ref.gelu(float(a)) for a in gx], np.float32)
    # --- whole tiny models (regenerated from their seeds by synth.make_model)
    refg = oracle.Reference(path=oracle.REF_SO.replace("libg4ref.so", "libg4ref_generic.so"), threads=1)
    prompt = rng.integers(0, synth.TINY.vocab_size, size=12).astype(np.int32)
    g["tiny_prompt"] = prompt
    for tag, shape in (("tinyf", synth.TINY_F), ("tiny", synth.TINY)):
        m = synth.make_model(shape, seed=3)
        desc = m.desc()
        rm = ref.model(desc, 64)
        for pos in range(8):
            rm.forward(int(prompt[pos]), pos, 0 if pos < 7 else 1)
        g[tag + "_logits_p7"] = rm.logits()
        g[tag + "_hidden_p7"] = rm.hidden()
        k1, v1 = rm.kv(0, 1, shape.n_kv_heads * shape.head_dim_swa)
        k5, v5 = rm.kv(5, 5, shape.n_kv_heads * shape.head_dim_full)
        g[tag + "_k_l0_p1"], g[tag + "_v_l0_p1"], g[tag + "_k_l5_p5"], g[tag + "_v_l5_p5"] = k1, v1, k5, v5
        rm.close()
        g[tag + "_greedy"] = ref.model(desc, 64).generate_greedy(prompt, 32)
        g[tag + "_greedy_generic"] = refg.model(desc, 64).generate_greedy(prompt, 32)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(out, **g)
    print("wrote", out, os.path.getsize(out), "bytes;", "BLAS:", ref.blas)


if __name__ == "__main__":
    main()
