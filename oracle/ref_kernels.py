"""ctypes access to the reference's own AIE2 row kernels built for the host CPU
(oracle/Makefile -> oracle/_ref/*.so). TEST INFRASTRUCTURE ONLY.

The row designs of src/rowops.py:60-218 call the kernel once per row with the
row's (window) width; run_rows() does the same.
"""
import ctypes
from pathlib import Path

import numpy as np

from rowops_ref import bf16_bits, bits_to_f32, RNE

_DIR = Path(__file__).resolve().parent / "_ref"
_LIBS = {}

# op name -> (library, symbol, input dtype)
KERNELS = {
    "g4": ("gelu_row4.so", "gelu_row4_bf16", "bf16"),
    "g4r": ("gelu_row4_rne.so", "gelu_row4_bf16", "bf16"),
    "g4f": ("gelu_row4f.so", "gelu_row4f_bf16", "f32"),
    "s1": ("softmax_row.so", "softmax_row_bf16", "bf16"),
    "s2": ("softmax_row2.so", "softmax_row2_bf16", "bf16"),
    "s3": ("softmax_row3.so", "softmax_row3_bf16", "bf16"),
    "s4": ("softmax_row4.so", "softmax_row4_bf16", "bf16"),
    "s4r": ("softmax_row4_rne.so", "softmax_row4r_bf16", "bf16"),
    "ln": ("layer_norm_gb.so", "layer_norm_bf16", "bf16"),
}


def available():
    return all((_DIR / lib).exists() for lib, _, _ in KERNELS.values())


def _fn(op):
    lib, sym, _ = KERNELS[op]
    if lib not in _LIBS:
        _LIBS[lib] = ctypes.CDLL(str(_DIR / lib))
    f = getattr(_LIBS[lib], sym)
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
    f.restype = None
    return f


def run_rows(op, x, valid=0):
    """Run kernel `op` over every row of x (fp32 array; bf16-representable for
    bf16-input ops), on the first `valid` columns when valid > 0. Returns the
    (rows, w) result as fp32."""
    f = _fn(op)
    x = np.ascontiguousarray(x, np.float32)
    rows = x.shape[0]
    w = x.shape[1] if valid <= 0 else valid
    if KERNELS[op][2] == "bf16":
        src = np.ascontiguousarray(bf16_bits(x[:, :w], RNE))
    else:
        src = np.ascontiguousarray(x[:, :w])
    dst = np.zeros((rows, w), np.uint16)
    for r in range(rows):
        f(src[r].ctypes.data, dst[r].ctypes.data, w)
    return bits_to_f32(dst)
