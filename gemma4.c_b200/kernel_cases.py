"""Small single-kernel cases of the decode hot path, for profiler captures.

    python gemma4.c_b200/kernel_cases.py q4|q6|gemv|attn [--reps N]

Each case launches one kernel family a few times on cuda:0 through the C ABI,
on inputs larger than L2 but a few GB on the device at most, then exits 0:
  q4    Q4_K 10240 x 2560 (FFN gate/up shape) at batch 64 -> gemm_q4tc_kernel
  q6    Q6_K 2560 x 10240 (FFN down shape) at batch 64    -> gemm_q6tc_kernel
  gemv  Q4_K 10240 x 2560 at batch 1                      -> gemv_tma_kernel
  attn  six-layer E4B-shaped model, 64 sequences at context 2048, three
        decode steps -> attn_stream_kernel (five sliding-window layers, then
        one global layer per step)
The matrices of q4/q6/gemv are rotated over copies that together exceed the
126 MB L2, so every launch streams its weights from HBM.
"""
from __future__ import annotations

import argparse
import dataclasses
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load():
    if "g4b200" in sys.modules:
        return sys.modules["g4b200"]
    spec = importlib.util.spec_from_file_location("g4b200", os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["g4b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def matrix_case(g4, which: str, reps: int) -> None:
    import torch
    S = g4.synth
    t, rows, n, B = {"q4": (S.Q4_K, 10240, 2560, 64), "q6": (S.Q6_K, 2560, 10240, 64),
                     "gemv": (S.Q4_K, 10240, 2560, 1)}[which]
    copies = max(2, int(np.ceil(300e6 / (S.row_bytes(t, n) * rows))))
    rng = np.random.default_rng(1)
    ws = [g4.weight_upload(S.rand_blocks(rng, t, rows, n, 1e-3, 2e-2), t, n, rows) for _ in range(copies)]
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(B, n, device=dev)
    q8 = torch.zeros(B * (n // 256) * 292, dtype=torch.uint8, device=dev)
    o = torch.zeros(B, rows, device=dev)
    for i in range(reps):
        g4.mm_device(o.data_ptr(), x.data_ptr(), ws[i % copies], n, rows, t, q8.data_ptr(), 0, B, st)
    torch.cuda.synchronize()
    for w in ws:
        g4.free(w)
    assert torch.isfinite(o).all().item()


def attn_case(g4, steps: int) -> None:
    shape = dataclasses.replace(g4.synth.E4B, n_layers=6)
    m = g4.synth.make_model(shape, seed=3)
    B, ctx = 64, 2048
    eng = g4.Engine(m, 0, max_seq=ctx + steps + 8, max_batch=B)
    try:
        eng.fill_kv(ctx - 1, seed=5)
        toks = np.arange(B, dtype=np.int32) % shape.vocab_size
        for i in range(steps):
            toks = eng.decode_batch(toks, ctx - 1 + i, 1)
        eng.sync()
    finally:
        eng.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["q4", "q6", "gemv", "attn"])
    ap.add_argument("--reps", type=int, default=4)
    a = ap.parse_args()
    g4 = _load()
    if g4.lib().g4_set_device(0) != 0:
        raise SystemExit("g4_set_device(0) failed: %s" % g4.last_error())
    if a.case == "attn":
        attn_case(g4, max(a.reps, 3))
    else:
        matrix_case(g4, a.case, a.reps)
    print("ok", a.case)


if __name__ == "__main__":
    main()
