"""The C-ABI library loads without a GPU, exports every entry point
include/wxb200.h declares, and its host-side tables equal the oracle's (the
preconditions of the bit-exact row-op parity). No kernel is launched here.
"""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import rowops_ref as O

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "wxb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("wx_gemm_bf16", "wx_attention", "wx_gelu_poly4", "wx_softmax_rows",
              "wx_layernorm_rows", "wx_encoder_forward", "wx_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(wxlib):
    missing = [n for n in declared_functions() if not hasattr(wxlib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from wxb200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_channel(wxlib):
    assert wxlib.wx_version() >= 100
    buf = ctypes.create_string_buffer(64)
    assert wxlib.wx_last_error(buf, 64) >= 0


@pytest.mark.parametrize("mode", [O.TRUNC, O.RNE])
def test_exp_table_matches_oracle(wxlib, mode):
    n = 0xC300 - 0x8000
    t16 = np.zeros(n, np.uint16)
    t32 = np.zeros(n, np.float32)
    got = wxlib.wx_softmax_exp_table(mode, t16.ctypes.data_as(ctypes.c_void_p),
                                     t32.ctypes.data_as(ctypes.c_void_p), n)
    assert got == n
    assert np.array_equal(t16, O.softmax_exp_table(mode))
    assert np.array_equal(t32.view(np.uint32), O.softmax_exp_table_f32().view(np.uint32))


@pytest.mark.parametrize("mode", [O.TRUNC, O.RNE])
def test_gelu_table_matches_oracle(wxlib, mode):
    t = np.zeros(24, np.float32)
    assert wxlib.wx_gelu4_table(mode, t.ctypes.data_as(ctypes.c_void_p), 24) == 24
    exp = np.concatenate([O.rbf(O.GELU4_BREAK, mode), O.rbf(O.GELU4_SHIFT, mode),
                          O.rbf(O.GELU4_SCALE, mode), O.rbf(O.GELU4_COEF, mode).ravel()])
    assert np.array_equal(t, exp)


def test_selftest_limits_checked_without_a_gpu(wxlib):
    """The wait-timeout diagnostic validates its limit before touching a device."""
    import ctypes
    fn = wxlib.wx_selftest_wait_timeout
    fn.restype, fn.argtypes = ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p]
    assert fn(0, None) == -1
    assert fn(3_000_000_000, None) == -1


def test_invalid_arguments_rejected_before_any_launch(wxlib):
    from wxb200 import _lib as L
    nul = ctypes.c_void_p(0)
    # negative shapes / bad enums / bad strides are refused on the host
    assert wxlib.wx_gelu_poly4(nul, 0, nul, -1, 8, 8, 8, 1, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_softmax_rows(nul, nul, 4, 16, 32, 16, 16, 1.0, 4, 1, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_softmax_rows(nul, nul, 4, 16, 0, 16, 16, 1.0, 2, 1, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_gemm_bf16(nul, nul, nul, nul, nul, 0, 8, 8, 8, 8, 8, 8, 0, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_attention(nul, nul, nul, nul, 1, 1, 16, 32, 64, 64, 64, 64, 0.125,
                              nul) == L.WX_ERR_UNSUPPORTED
    assert "head dim" in L.last_error()
    h = ctypes.c_void_p()
    assert wxlib.wx_encoder_create(ctypes.byref(h), 80, 384, 5, 4, 1536, 1500, 1, 0) == \
        L.WX_ERR_UNSUPPORTED
    # zero-sized row ops are a no-op success
    assert wxlib.wx_gelu_poly4(nul, 0, nul, 0, 8, 8, 8, 1, nul) == L.WX_OK
    # int8 path: quantising no rows is a no-op; an empty row has no scale (the
    # reference's np.abs(A).max(axis=1) raises on it); int8 GEMM rows must be
    # 16-byte aligned; the encoder handle and mode are checked
    assert wxlib.wx_quantize_rows(nul, L.WX_DTYPE_F32, 0, 8, 8, nul, 0, nul, 16, nul, nul) == L.WX_OK
    assert wxlib.wx_quantize_rows(nul, L.WX_DTYPE_F32, 4, 0, 8, nul, 0, nul, 16, nul,
                                  nul) == L.WX_ERR_INVALID
    assert wxlib.wx_quantize_rows(nul, 7, 4, 8, 8, nul, 0, nul, 16, nul, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_absmax_rows(nul, L.WX_DTYPE_BF16, 0, 8, 8, nul, 1, nul) == L.WX_OK
    assert wxlib.wx_absmax_rows(nul, L.WX_DTYPE_BF16, 4, 8, 4, nul, 1, nul) == L.WX_ERR_INVALID
    assert wxlib.wx_layernorm_quant_rows(nul, nul, nul, nul, nul, 4, 6, 8, 8, 1e-5,
                                         nul) == L.WX_ERR_INVALID
    assert wxlib.wx_gemm_i8(nul, nul, nul, nul, nul, nul, nul, 0, 8, 16, 16, 16, 8, 0, 0, nul,
                            nul) == L.WX_ERR_INVALID
    a = ctypes.c_void_p(256)   # not dereferenced: the stride check comes first
    assert wxlib.wx_gemm_i8(a, a, a, a, nul, nul, a, 32, 32, 24, 24, 24, 32, 0, 0, nul,
                            nul) == L.WX_ERR_INVALID
    assert "16-byte" in L.last_error()
    assert wxlib.wx_gemm_i8(a, a, a, a, nul, nul, a, 32, 32, 32, 32, 32, 32, 0, 9, nul,
                            nul) == L.WX_ERR_INVALID
    assert wxlib.wx_encoder_set_quant(nul, L.WX_QUANT_INT8_PERCHAN) == L.WX_ERR_INVALID
    # the pipelined host entry points check the handle before any CUDA call
    assert wxlib.wx_encoder_submit_host(nul, nul, nul, 1, 400, 1) == L.WX_ERR_INVALID
    assert wxlib.wx_encoder_wait_host(nul) == L.WX_ERR_INVALID
