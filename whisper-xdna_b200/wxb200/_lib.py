"""ctypes binding of libwxb200.so (include/wxb200.h).

The library is the only compute path: if it is missing, or a CUDA device is
missing when a kernel is called, the call raises; nothing falls back to the CPU.
"""
import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwxb200.so"

# status codes and enums of include/wxb200.h
WX_OK = 0
WX_ERR_INVALID = -1
WX_ERR_CUDA = -2
WX_ERR_UNSUPPORTED = -3
WX_ERR_DEVICE = -4
WX_ERR_NOMEM = -5
WX_DEVERR_TIMEOUT = 1
WX_DTYPE_BF16 = 0
WX_DTYPE_F32 = 1
WX_ROUND_TRUNC = 0
WX_ROUND_RNE = 1
WX_LN_AIE = 0
WX_LN_FP32 = 1
WX_EPI_F32 = 0
WX_EPI_BF16 = 1
WX_EPI_F32_RESID = 2
WX_EPI_BF16_GELU = 3
WX_EPI_BF16_GELU_ERF = 4
WX_GELU_POLY4 = 0
WX_GELU_ERF = 1
WX_QUANT_NONE = 0
WX_QUANT_INT8_PERCHAN = 1
WX_QUANT_INT8_PERTENSOR = 2

_c = ctypes
_p, _i, _i64, _f = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float

# name -> (restype, argtypes), in the order of include/wxb200.h
SIGNATURES = {
    "wx_version": (_i, []),
    "wx_last_error": (_i, [_c.c_char_p, _i64]),
    "wx_device_error": (_i, [_c.POINTER(_i), _i]),
    "wx_gelu_poly4": (_i, [_p, _i, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "wx_softmax_rows": (_i, [_p, _p, _i64, _i64, _i64, _i64, _i64, _f, _i, _i, _p]),
    "wx_layernorm_rows": (_i, [_p, _i, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _f, _i, _i, _p]),
    "wx_softmax_exp_table": (_i, [_i, _p, _p, _i64]),
    "wx_gelu4_table": (_i, [_i, _p, _i64]),
    "wx_gemm_bf16": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i, _p]),
    "wx_absmax_rows": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p]),
    "wx_layernorm_quant_rows": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _p]),
    "wx_quantize_rows": (_i, [_p, _i, _i64, _i64, _i64, _p, _i64, _p, _i64, _p, _p]),
    "wx_gemm_i8": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i,
                        _p, _p]),
    "wx_gemm_f32": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "wx_attention": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f, _p]),
    "wx_mlp_bf16_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _p]),
    "wx_encoder_create": (_i, [_c.POINTER(_p), _i, _i, _i, _i, _i, _i, _i, _i]),
    "wx_encoder_destroy": (_i, [_p]),
    "wx_encoder_set_frontend": (_i, [_p, _p, _p, _p, _p, _p]),
    "wx_encoder_set_layer": (_i, [_p, _i] + [_p] * 15),
    "wx_encoder_set_ln_post": (_i, [_p, _p, _p]),
    "wx_encoder_set_quant": (_i, [_p, _i]),
    "wx_encoder_forward": (_i, [_p, _p, _p, _i64, _i64, _i, _p]),
    "wx_encoder_forward_host": (_i, [_p, _p, _p, _i64, _i64, _i, _p]),
    "wx_encoder_submit_host": (_i, [_p, _p, _p, _i64, _i64, _i]),
    "wx_encoder_wait_host": (_i, [_p]),
    "wx_encoder_device_bytes": (_i64, [_p]),
    "wx_log_mel": (_i, [_p, _i64, _i64, _i64, _i, _p, _p]),
    "wx_selftest_wait_timeout": (_i, [_c.c_uint64, _p]),
}

_lib = None


def lib():
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() or "
                "`python -m wxb200._build` (nvcc, sm_100a). There is no CPU fallback.")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def last_error():
    buf = ctypes.create_string_buffer(2048)
    lib().wx_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


class WxError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"libwxb200 status {status}: {msg}")
        self.status = status


def check(status):
    """Raise for a non-zero status: ValueError for bad arguments (as the
    reference's row designs do for bad widths, src/rowops.py:78-79), WxError
    (a RuntimeError, like the reference's failed runs, src/rawxrt.py:319-324)
    otherwise."""
    if status == WX_OK:
        return status
    msg = last_error()
    if status == WX_ERR_INVALID:
        raise ValueError(msg)
    raise WxError(status, msg)


def device_error(clear=True):
    """Synchronize and return the device error word (WX_DEVERR_* bits)."""
    flags = ctypes.c_int(0)
    check(lib().wx_device_error(ctypes.byref(flags), 1 if clear else 0))
    return flags.value
