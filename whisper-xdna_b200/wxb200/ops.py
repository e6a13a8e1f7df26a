"""Device-tensor wrappers of the C ABI: torch CUDA tensors in and out, work
enqueued on torch's current stream.

Every function takes 2-D tensors whose last dimension is contiguous (row
stride = tensor.stride(0)), so column bands and column slices of wider
buffers are accepted as they are -- the banded outputs of src/rowops.py:80-88
and the per-head slices of a fused QKV buffer.
"""
import ctypes

import torch

from . import _lib as L


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _mat(t, name, dtypes):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with a contiguous last dimension")
    if t.dtype not in dtypes:
        raise ValueError(f"{name} dtype {t.dtype} not in {dtypes}")
    return t


def _vec(t, n, name):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32:
        raise ValueError(f"{name} must be a float32 CUDA tensor")
    t = t.contiguous()
    if t.numel() != n:
        raise ValueError(f"{name} has {t.numel()} elements, expected {n}")
    return t


def gelu_poly4(x, out=None, rounding=L.WX_ROUND_RNE):
    """GELU-poly4 of a bf16 (g4 / g4r) or fp32 (g4f) matrix into bf16 `out`."""
    _mat(x, "x", (torch.bfloat16, torch.float32))
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.bfloat16, device=x.device)
    _mat(out, "out", (torch.bfloat16,))
    if tuple(out.shape) != (rows, cols):
        raise ValueError("out shape mismatch")
    dt = L.WX_DTYPE_F32 if x.dtype == torch.float32 else L.WX_DTYPE_BF16
    L.check(L.lib().wx_gelu_poly4(_ptr(x), dt, _ptr(out), rows, cols, x.stride(0),
                                  out.stride(0), rounding, _stream()))
    return out


def softmax_rows(x, out=None, valid=0, scale=1.0, variant=4, rounding=L.WX_ROUND_TRUNC):
    """Row softmax over the first `valid` columns (all if 0) of bf16 rows."""
    _mat(x, "x", (torch.bfloat16,))
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.bfloat16, device=x.device)
    _mat(out, "out", (torch.bfloat16,))
    if out.shape[0] != rows or out.shape[1] < (valid if valid > 0 else cols):
        raise ValueError("out shape mismatch")
    L.check(L.lib().wx_softmax_rows(_ptr(x), _ptr(out), rows, cols, valid, x.stride(0),
                                    out.stride(0), float(scale), variant, rounding, _stream()))
    return out


def layer_norm_rows(x, gamma=None, beta=None, out=None, eps=1e-5, mode=L.WX_LN_AIE,
                    rounding=L.WX_ROUND_TRUNC, out_dtype=None):
    """LayerNorm of each row (mode WX_LN_AIE: the reference's device kernel,
    bf16; WX_LN_FP32: fp32 two-pass, bf16 or fp32 in and out)."""
    _mat(x, "x", (torch.bfloat16, torch.float32))
    rows, cols = x.shape
    if out is None:
        od = out_dtype or (torch.bfloat16 if mode == L.WX_LN_AIE else x.dtype)
        out = torch.empty(rows, cols, dtype=od, device=x.device)
    _mat(out, "out", (torch.bfloat16, torch.float32))
    g, b = _vec(gamma, cols, "gamma"), _vec(beta, cols, "beta")
    idt = L.WX_DTYPE_F32 if x.dtype == torch.float32 else L.WX_DTYPE_BF16
    odt = L.WX_DTYPE_F32 if out.dtype == torch.float32 else L.WX_DTYPE_BF16
    L.check(L.lib().wx_layernorm_rows(_ptr(x), idt, _ptr(g), _ptr(b), _ptr(out), odt, rows,
                                      cols, x.stride(0), out.stride(0), float(eps), mode,
                                      rounding, _stream()))
    return out


def gemm(A, W, bias=None, residual=None, out=None, epilogue=None):
    """epilogue(A @ W^T) on the tensor cores: A (M, K) bf16, W (N, K) bf16.

    Default epilogue: fp32 output (+ residual when given)."""
    _mat(A, "A", (torch.bfloat16,))
    _mat(W, "W", (torch.bfloat16,))
    M, K = A.shape
    N, K2 = W.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    if epilogue is None:
        epilogue = L.WX_EPI_F32_RESID if residual is not None else L.WX_EPI_F32
    f32_out = epilogue in (L.WX_EPI_F32, L.WX_EPI_F32_RESID)
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if f32_out else torch.bfloat16,
                          device=A.device)
    _mat(out, "out", (torch.float32,) if f32_out else (torch.bfloat16,))
    b = _vec(bias, N, "bias")
    r = None
    if residual is not None:
        r = _mat(residual, "residual", (torch.float32,))
    L.check(L.lib().wx_gemm_bf16(_ptr(A), _ptr(W), _ptr(b), _ptr(r), _ptr(out), M, N, K,
                                 A.stride(0), W.stride(0), out.stride(0),
                                 r.stride(0) if r is not None else 0, epilogue, _stream()))
    return out


def gemm_f32(A, W, bias=None, out=None):
    """A @ W^T (+ bias) in fp32 on the FMA pipe: A (M, K), W (N, K) float32
    CUDA tensors with unit column stride; each output sums k in ascending order."""
    _mat(A, "A", (torch.float32,))
    _mat(W, "W", (torch.float32,))
    M, K = A.shape
    N, K2 = W.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=A.device)
    _mat(out, "out", (torch.float32,))
    b = _vec(bias, N, "bias")
    L.check(L.lib().wx_gemm_f32(_ptr(A), _ptr(W), _ptr(b), _ptr(out), M, N, K, A.stride(0),
                                W.stride(0), out.stride(0), _stream()))
    return out


def _outvec(t, n, name):
    """A float32 CUDA vector written in place: must be contiguous already."""
    _vec(t, n, name)
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _dtype_code(t, name):
    if t.dtype == torch.bfloat16:
        return L.WX_DTYPE_BF16
    if t.dtype == torch.float32:
        return L.WX_DTYPE_F32
    raise TypeError(f"{name}: bf16 or fp32 expected, got {t.dtype}")


def absmax_rows(x, out=None, per_row=True):
    """max |x| per row (per_row) or over the whole matrix, folded into `out`
    (fp32, zeroed when created here)."""
    _mat(x, "x", (torch.bfloat16, torch.float32))
    rows, cols = x.shape
    if out is None:
        out = torch.zeros(rows if per_row else 1, dtype=torch.float32, device=x.device)
    _outvec(out, rows if per_row else 1, "out")
    L.check(L.lib().wx_absmax_rows(_ptr(x), _dtype_code(x, "x"), rows, cols, x.stride(0),
                                   _ptr(out), 1 if per_row else 0, _stream()))
    return out


def quantize_rows(x, rowmax=None, q=None, scale=None):
    """Per-row int8 quantisation: scale = max|row| / 127 (1 for a zero row),
    q = rint(x / scale). rowmax: precomputed maxima, one per row or a single
    value for every row. Returns (q int8 (rows, cols), scale fp32 (rows,))."""
    _mat(x, "x", (torch.bfloat16, torch.float32))
    rows, cols = x.shape
    if q is None:
        q = torch.empty(rows, (cols + 15) // 16 * 16, dtype=torch.int8, device=x.device)[:, :cols]
    _mat(q, "q", (torch.int8,))
    if scale is None:
        scale = torch.empty(rows, dtype=torch.float32, device=x.device)
    _outvec(scale, rows, "scale")
    stride = 0
    if rowmax is not None:
        if rowmax.numel() not in (1, rows):
            raise ValueError("rowmax: one value per row or one in all")
        stride = 1 if rowmax.numel() == rows and rows > 1 else 0
        rowmax = _vec(rowmax, rowmax.numel(), "rowmax")
    L.check(L.lib().wx_quantize_rows(_ptr(x), _dtype_code(x, "x"), rows, cols, x.stride(0),
                                     _ptr(rowmax), stride, _ptr(q), q.stride(0), _ptr(scale),
                                     _stream()))
    return q, scale


def layer_norm_quant_rows(x, gamma=None, beta=None, eps=1e-5, q=None, scale=None):
    """fp32 LayerNorm of each row of x quantised per row to int8, in one pass:
    the same (q, scale) as quantize_rows(layer_norm_rows(x, ..., fp32 out))."""
    _mat(x, "x", (torch.float32,))
    rows, cols = x.shape
    if q is None:
        q = torch.empty(rows, (cols + 15) // 16 * 16, dtype=torch.int8, device=x.device)[:, :cols]
    _mat(q, "q", (torch.int8,))
    if scale is None:
        scale = torch.empty(rows, dtype=torch.float32, device=x.device)
    _outvec(scale, rows, "scale")
    g = _vec(gamma, cols, "gamma")
    b = _vec(beta, cols, "beta")
    L.check(L.lib().wx_layernorm_quant_rows(_ptr(x), _ptr(g), _ptr(b), _ptr(q), _ptr(scale), rows,
                                            cols, x.stride(0), q.stride(0), eps, _stream()))
    return q, scale


def gemm_i8(Aq, Wq, sa, sw, bias=None, residual=None, out=None, epilogue=None, rowmax=None):
    """epilogue((float(Aq @ Wq^T) * sa[:, None]) * sw[None, :]) on the int8
    tensor cores: Aq (M, K) and Wq (N, K) int8 with rows 16-byte aligned, sa
    (M,) and sw (N,) fp32. rowmax (M,) fp32 collects max |out| per row for the
    bf16 epilogues."""
    _mat(Aq, "Aq", (torch.int8,))
    _mat(Wq, "Wq", (torch.int8,))
    M, K = Aq.shape
    N, K2 = Wq.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    if epilogue is None:
        epilogue = L.WX_EPI_F32_RESID if residual is not None else L.WX_EPI_F32
    f32_out = epilogue in (L.WX_EPI_F32, L.WX_EPI_F32_RESID)
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if f32_out else torch.bfloat16,
                          device=Aq.device)
    _mat(out, "out", (torch.float32,) if f32_out else (torch.bfloat16,))
    sa = _vec(sa, M, "sa")
    sw = _vec(sw, N, "sw")
    b = _vec(bias, N, "bias")
    if rowmax is not None:
        _outvec(rowmax, M, "rowmax")
    r = None
    if residual is not None:
        r = _mat(residual, "residual", (torch.float32,))
    L.check(L.lib().wx_gemm_i8(_ptr(Aq), _ptr(Wq), _ptr(sa), _ptr(sw), _ptr(b), _ptr(r),
                               _ptr(out), M, N, K, Aq.stride(0), Wq.stride(0), out.stride(0),
                               r.stride(0) if r is not None else 0, epilogue, _ptr(rowmax),
                               _stream()))
    return out


def attention(q, k, v, n_batch, n_head, scale, out=None):
    """softmax(scale * q k^T) v per (batch, head); q, k, v: (n_batch*T, n_head*64)
    bf16 (column slices of one QKV buffer are fine)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _mat(t, n, (torch.bfloat16,))
    rows, width = q.shape
    if rows % n_batch:
        raise ValueError("rows not divisible by n_batch")
    T = rows // n_batch
    hd = width // n_head
    if out is None:
        out = torch.empty(rows, width, dtype=torch.bfloat16, device=q.device)
    _mat(out, "out", (torch.bfloat16,))
    L.check(L.lib().wx_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), n_batch, n_head, T, hd,
                                 q.stride(0), k.stride(0), v.stride(0), out.stride(0),
                                 float(scale), _stream()))
    return out


def log_mel(audio, n_mels=80, out=None):
    """whisper's log-mel features of 16 kHz audio on the GPU: audio a CUDA
    float32 tensor (batch, n_samples) or (n_samples,), each clip zero-padded or
    trimmed to 30 s -> (batch, n_mels, 3000) float32 (or (n_mels, 3000))."""
    squeeze = audio.dim() == 1
    a = audio.unsqueeze(0) if squeeze else audio
    if not a.is_cuda or a.dtype != torch.float32 or a.dim() != 2 or a.stride(1) != 1:
        raise ValueError("audio must be a CUDA float32 tensor with contiguous rows")
    B, n = a.shape
    if out is None:
        out = torch.empty(B, n_mels, 3000, dtype=torch.float32, device=a.device)
    if out.shape != (B, n_mels, 3000) or not out.is_contiguous() or out.dtype != torch.float32:
        raise ValueError("out must be a contiguous float32 (batch, n_mels, 3000) tensor")
    L.check(L.lib().wx_log_mel(_ptr(a), B, n, a.stride(0) if B > 1 else n, int(n_mels),
                               _ptr(out), _stream()))
    return out[0] if squeeze else out
