"""The reference's int8 matmul on the int8 tensor cores.

q_matmul_factory(mode) mirrors bench/probe_int8_decode.py:48-74: it returns a
callable with the reference's `mm` signature, q_matmul(A, B, bias=None, **kw)
-> fp32 (M, N) numpy, that the reference encoder (or this package's) can take
as its matmul, e.g. E.encoder(W, mel, q_matmul_factory("perchan"),
E.np_matmul, n_layer, n_head, fold_bias=False) as the probe calls it
(:140-142). Modes:
  "perchan"   per-token activation scales, per-column weight scales
  "pertensor" per-token activation scales, one weight scale per matrix
  "fp32"      the unquantised control, A @ B in fp32 (wx_gemm_f32, FMA pipe)
The quantisation (wx_quantize_rows), the int8 product with s32 accumulation
and the (r * sa) * sw scaling (wx_gemm_i8) reproduce the reference's float32
arithmetic step for step, so the result equals the probe's numpy output bit
for bit.
"""
import numpy as np
import torch

from . import ops

MODES = ("perchan", "pertensor", "fp32")


def quantize_weight(Wt, mode):
    """The torch-layout weight Wt (N, K), CUDA fp32 -> (int8 (N, K), scales (N,))
    with one scale per row (output channel) or one for all rows."""
    if mode == "perchan":
        return ops.quantize_rows(Wt)
    if mode == "pertensor":
        return ops.quantize_rows(Wt, rowmax=ops.absmax_rows(Wt, per_row=False))
    raise ValueError(f"mode must be 'perchan' or 'pertensor', got {mode!r}")


def q_matmul_factory(mode):
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")

    def q_matmul(A, B, bias=None, **kw):
        if not torch.cuda.is_available():
            raise RuntimeError("q_matmul needs a CUDA device; there is no CPU fallback")
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        dev = torch.device("cuda", torch.cuda.current_device())
        dA = torch.from_numpy(A).to(dev)
        b = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, np.float32)).to(dev)
        dW = torch.from_numpy(np.ascontiguousarray(B.T)).to(dev)   # (N, K)
        if mode == "fp32":
            return ops.gemm_f32(dA, dW, bias=b).cpu().numpy()
        qa, sa = ops.quantize_rows(dA)
        qw, sw = quantize_weight(dW, mode)
        out = ops.gemm_i8(qa, qw, sa, sw, bias=b)
        return out.cpu().numpy()

    return q_matmul
