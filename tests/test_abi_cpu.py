"""The C-ABI library loads, exports every symbol include/g4b200.h declares, and
rejects bad arguments with the documented status codes before any device
work (CPU only; no compute calls)."""
import ctypes as C
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", f)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names |= set(re.findall(r"\b(g4_\w+)\s*\(", txt))
    return names


def test_library_exports_all_declared_symbols(g4):
    lib = g4.lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in sorted(syms) if not hasattr(lib, s)]
    assert not missing, missing
    bound = {n for n, _, _ in g4.SIGNATURES}
    assert syms <= bound, syms - bound


def test_desc_layout_matches_header(g4):
    assert g4.lib().g4_model_desc_bytes() == C.sizeof(g4.Desc)


def test_argument_errors_without_device(g4):
    L = g4.lib()
    x = np.zeros(100, np.float32)
    y = np.zeros(2 * 292, np.uint8)
    assert L.g4_quantize_row_q8_K_ex(x.ctypes.data, y.ctypes.data, 100) == g4.G4_ERR_ARG
    assert "256" in g4.last_error()[1]
    o = np.zeros(4, np.float32)
    w = np.zeros(4 * 144, np.uint8)
    assert L.g4_mm_ex(o.ctypes.data, x.ctypes.data, w.ctypes.data, 256, 4, 99, None, 0) == g4.G4_ERR_TYPE
    assert L.g4_mm_ex(o.ctypes.data, x.ctypes.data, w.ctypes.data, 100, 4, g4.Q4_K, y.ctypes.data, 0) == g4.G4_ERR_ARG
    assert L.g4_mm_quant_rows_ex(o.ctypes.data, x.ctypes.data, w.ctypes.data, 256, 4, g4.BF16) == g4.G4_ERR_TYPE
    assert L.g4_mm_argmax_row(x.ctypes.data, w.ctypes.data, 256, 4, g4.F16, y.ctypes.data) == -1
    assert L.g4_last_error() == g4.G4_ERR_TYPE
    assert L.g4_attn_decode(o.ctypes.data, x.ctypes.data, x.ctypes.data, x.ctypes.data, 2, 8, 8, 3, 64) == g4.G4_ERR_ARG
    assert L.g4_apply_rope_neox_ex(x.ctypes.data, 1, 64, 66, 1, 1e4, 1.0, None) == g4.G4_ERR_ARG
    assert not L.g4_engine_create(None, 0, 64, 1)
    assert L.g4_last_error() == g4.G4_ERR_ARG
    assert L.g4_forward(None, 0, 0, 1, None) == -1
    L.g4_clear_error()
    assert L.g4_last_error() == 0
