"""The reference's fused-attention entry (src/attn_fused.py:140-145) on the B200.

attn_head(q_in, kv_in, o_out, *, ctx, hd, bq, bk, nvalid=0) computes one head,
O = softmax(Q K^T / sqrt(hd)) V, with Q and K unscaled as the reference passes
them (kernels/attn_mmul.cc:22-24, src/rawxrt.py:771). The NPU version wanted
its operands pre-tiled into mmul block layouts; here they are plain row-major:
  q_in  (ctx, hd) bf16,  kv_in (2, ctx, hd) or (2*ctx, hd) bf16 (K rows, then
  V rows), o_out (ctx, hd) bf16 -- CUDA tensors, written in place.
bq and bk were the NPU's tile sizes and are accepted and ignored (the kernel's
tiles are 128 x 128). nvalid > 0 masks keys at and past nvalid exactly, and
only the first nvalid query rows are computed; the rest of o_out is zeroed.
attn_heads() does all heads of a (ctx, nh*hd) activation in one launch.
"""
import math

import torch

from . import ops


def attn_head(q_in, kv_in, o_out, *, ctx, hd, bq=48, bk=32, nvalid=0):
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in (q_in, kv_in, o_out)):
        raise ValueError("attn_head: q_in, kv_in and o_out must be CUDA tensors")
    n = nvalid if nvalid > 0 else ctx
    if n > ctx:
        raise ValueError(f"nvalid {nvalid} > ctx {ctx}")
    q = q_in.reshape(ctx, hd)
    kv = kv_in.reshape(2 * ctx, hd)
    o = o_out.reshape(ctx, hd)
    res = ops.attention(q[:n], kv[:n], kv[ctx:ctx + n], 1, 1, 1.0 / math.sqrt(hd),
                        out=o[:n] if o.is_contiguous() else None)
    if not o.is_contiguous():
        o[:n].copy_(res)
    if n < ctx:
        o[n:].zero_()
    return o_out


def attn_heads(qkv, n_head, scale=None, out=None, n_batch=1):
    """All heads of a fused (n_batch*ctx, 3*d) bf16 QKV activation at once."""
    d = qkv.shape[1] // 3
    hd = d // n_head
    s = 1.0 / math.sqrt(hd) if scale is None else scale
    return ops.attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], n_batch, n_head, s,
                         out=out)
