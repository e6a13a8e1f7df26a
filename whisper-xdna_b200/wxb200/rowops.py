"""The reference's row-op surface (src/rowops.py:221-330) on the B200.

Each design function has the reference's signature, `design(a_in, c_out, *,
rows, cols[, valid][, out_cols])`, and writes its result into c_out. a_in and
c_out are CUDA tensors (bf16; fp32 input for gelu_row4f) holding rows x cols
(2-D or flat), or numpy arrays (ml_dtypes.bfloat16 / float32), in which case
the result is copied back into c_out. The NPU designs needed every window
width to be a multiple of 16 and raised ValueError otherwise
(src/rowops.py:78-79); these functions keep that contract so callers see the
same errors, while the C ABI underneath (wx_softmax_rows, wx_gelu_poly4,
wx_layernorm_rows) takes any width.

Two entry points go beyond the reference's surface, as its north star asks:
layer_norm_gb (LayerNorm WITH gamma/beta) and softmax_rows (a scale argument
and a choice of rounding).
"""
import numpy as np
import torch

from . import _lib as L
from . import ops


def _check_width(sym, w):
    if w % 16:
        raise ValueError(f"{sym}: row width {w} is not a multiple of 16")


def _to_dev(a, rows, cols, dtype):
    if isinstance(a, torch.Tensor):
        if not a.is_cuda:
            raise ValueError("a_in must be a CUDA tensor or a numpy array")
        t = a.reshape(rows, -1) if a.dim() != 2 else a
        if t.dtype != dtype:
            raise ValueError(f"a_in dtype {t.dtype}, expected {dtype}")
        return t
    arr = np.asarray(a)
    if arr.dtype.name == "bfloat16":
        t = torch.from_numpy(np.ascontiguousarray(arr).view(np.uint16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
        if dtype == torch.bfloat16:
            t = t.to(torch.bfloat16)
    return t.reshape(rows, -1).to("cuda")


def _out_view(c_out, rows, cols, out_cols=0):
    """(device view to write, finisher). A CUDA c_out is written in place; a
    numpy c_out receives a copy after the kernel."""
    oc = out_cols if out_cols > 0 else cols
    if isinstance(c_out, torch.Tensor):
        if not c_out.is_cuda or c_out.dtype != torch.bfloat16:
            raise ValueError("c_out must be a bf16 CUDA tensor or a numpy array")
        t = c_out if (c_out.dim() == 2 and c_out.stride(1) == 1) else c_out.view(rows, oc)
        return t[:, :cols], (lambda: None)
    dev = torch.zeros(rows, oc, dtype=torch.bfloat16, device="cuda")
    host = np.asarray(c_out)

    def finish():
        torch.cuda.current_stream().synchronize()
        res = dev.cpu().view(torch.uint16).numpy()
        flat = host.reshape(rows, oc)
        if host.dtype.name == "bfloat16":
            flat.view(np.uint16)[:, :cols] = res[:, :cols]
        else:
            flat[:, :cols] = (res[:, :cols].astype(np.uint32) << 16).view(np.float32)
    return dev[:, :cols], finish


def _softmax(sym, variant, rounding, a_in, c_out, rows, cols, valid=0, scale=1.0):
    w = valid if valid > 0 else cols
    _check_width(sym, w)
    x = _to_dev(a_in, rows, cols, torch.bfloat16)
    out, fin = _out_view(c_out, rows, cols)
    ops.softmax_rows(x, out=out, valid=valid, scale=scale, variant=variant, rounding=rounding)
    fin()


def _gelu(sym, rounding, a_in, c_out, rows, cols, f32_in=False, out_cols=0):
    _check_width(sym, cols)
    x = _to_dev(a_in, rows, cols, torch.float32 if f32_in else torch.bfloat16)
    out, fin = _out_view(c_out, rows, cols, out_cols)
    ops.gelu_poly4(x, out=out, rounding=rounding)
    fin()


# ---------------------------------------------------------------- LayerNorm
def layer_norm(a_in, c_out, *, rows, cols):
    """kernels/layer_norm_gb.cc: (x - mean) / sqrt(var + 1e-5), no affine,
    bf16 in/out, the part's default (truncating) rounding (src/rowops.py:221)."""
    _check_width("layer_norm_bf16", cols)
    x = _to_dev(a_in, rows, cols, torch.bfloat16)
    out, fin = _out_view(c_out, rows, cols)
    ops.layer_norm_rows(x, out=out, mode=L.WX_LN_AIE, rounding=L.WX_ROUND_TRUNC)
    fin()


def layer_norm_gb(a_in, c_out, *, rows, cols, gamma=None, beta=None, eps=1e-5,
                  rounding=L.WX_ROUND_RNE):
    """LayerNorm with learned gamma/beta in the device kernel's arithmetic
    (the affine the reference had to fold into the next GEMM, layer_norm_gb.cc:38-47)."""
    _check_width("layer_norm_gb", cols)
    x = _to_dev(a_in, rows, cols, torch.bfloat16)
    out, fin = _out_view(c_out, rows, cols)
    g = None if gamma is None else torch.as_tensor(np.asarray(gamma, np.float32)).cuda()
    b = None if beta is None else torch.as_tensor(np.asarray(beta, np.float32)).cuda()
    ops.layer_norm_rows(x, gamma=g, beta=b, out=out, eps=eps, mode=L.WX_LN_AIE,
                        rounding=rounding)
    fin()


# ---------------------------------------------------------------- softmax
def softmax_row(a_in, c_out, *, rows, cols):
    """v1: bf16 reciprocal (kernels/softmax_row.cc)."""
    _softmax("softmax_row_bf16", 1, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols)


def softmax_row2(a_in, c_out, *, rows, cols):
    """v2 (kernels/softmax_row2.cc) -- the same arithmetic as v4."""
    _softmax("softmax_row2_bf16", 4, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols)


def softmax_row3(a_in, c_out, *, rows, cols):
    """v3: exponential and reciprocal split hi/lo (kernels/softmax_row3.cc)."""
    _softmax("softmax_row3_bf16", 3, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols)


def softmax_row3_win(a_in, c_out, *, rows, cols, valid):
    _softmax("softmax_row3_bf16", 3, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols, valid)


def softmax_row4(a_in, c_out, *, rows, cols):
    """v4: one exp evaluation, split reciprocal (kernels/softmax_row4_body.inc)."""
    _softmax("softmax_row4_bf16", 4, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols)


def softmax_row4_win(a_in, c_out, *, rows, cols, valid):
    _softmax("softmax_row4_bf16", 4, L.WX_ROUND_TRUNC, a_in, c_out, rows, cols, valid)


def softmax_row4r_win(a_in, c_out, *, rows, cols, valid):
    """v4 with round-to-nearest-even (kernels/softmax_row4_rne.cc)."""
    _softmax("softmax_row4r_bf16", 4, L.WX_ROUND_RNE, a_in, c_out, rows, cols, valid)


def softmax_rows(a_in, c_out, *, rows, cols, valid=0, scale=1.0, variant=4,
                 rounding=L.WX_ROUND_RNE):
    """Windowed row softmax with an input scale (the attention scores' 1/sqrt(hd))."""
    _softmax("softmax_rows", variant, rounding, a_in, c_out, rows, cols, valid, scale)


# ---------------------------------------------------------------- GELU
def gelu_row4(a_in, c_out, *, rows, cols):
    """g4: piecewise poly4 erf-GELU, truncating (kernels/gelu_row4.cc)."""
    _gelu("gelu_row4_bf16", L.WX_ROUND_TRUNC, a_in, c_out, rows, cols)


def gelu_row4_rne(a_in, c_out, *, rows, cols):
    """g4r: the same with round-to-nearest-even (kernels/gelu_row4_rne.cc)."""
    _gelu("gelu_row4_bf16", L.WX_ROUND_RNE, a_in, c_out, rows, cols)


def gelu_row4f(a_in, c_out, *, rows, cols, out_cols=0):
    """g4f: fp32 input (a GEMM accumulator), bf16 written as a column band of
    an out_cols-wide buffer (kernels/gelu_row4f.cc)."""
    _gelu("gelu_row4f_bf16", L.WX_ROUND_RNE, a_in, c_out, rows, cols, f32_in=True,
          out_cols=out_cols)


def _superseded(name, why):
    def f(*a, **kw):
        raise NotImplementedError(f"{name}: {why}")
    f.__name__ = name
    return f


gelu_row = _superseded("gelu_row", "the stock tanh-GELU kernel (gl) is superseded by g4; "
                       "use gelu_row4_rne")
gelu_row2 = _superseded("gelu_row2", "the logistic-form GELU (g2) is superseded by g4; "
                        "use gelu_row4_rne")
gelu_row3 = _superseded("gelu_row3", "the 5-piece monomial GELU (g3) is superseded by g4; "
                        "use gelu_row4_rne")
