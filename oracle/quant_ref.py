"""TEST INFRASTRUCTURE ONLY (CPU oracle): the reference's int8 projection/MLP
mode, restated in numpy. Imported by tests/ and bench.py's CPU legs only.

The reference measures int8 GEMMs with a numpy simulation that its encoder
calls as the matmul: q_matmul_factory(mode) in bench/probe_int8_decode.py:48-74,
run as E.encoder(W, mel, q_matmul_factory(mode), E.np_matmul, ...,
fold_bias=False) (:140-142) after E.prepare_mlp_chunks(W, n_layer, d, 0)
(:99). This file restates
  - q_matmul(A, B, bias, mode): per-token activation scales, per-channel
    ("perchan") or whole-matrix ("pertensor") weight scales, round half to even,
    exact integer products, (r * sa) * sw, + bias (:54-74);
  - quantize_rows(x): the per-row quantisation both operands go through;
  - encoder_int8_np: the reference's numpy encoder (src/npu_whisper_encoder.py
    :436-541) with that matmul for the 290 projection / MLP / conv GEMMs,
    fold_bias=False, host attention in fp32, fc1 split into the column chunks of
    prepare_mlp_chunks (:383-406) when it is wider than 4096.

Pinned in tests/test_quant_oracle.py against fixtures made by running the
reference's own q_matmul_factory and encoder (tests/golden/make_quant_golden.py).
"""
import numpy as np

from encoder_ref import (gelu_np, geometry_of, im2col, layer_norm_np, mm as mm_f32,
                         softmax_np)

MAX_GEMM_N = 4096   # src/npu_whisper_encoder.py:361


def quantize_rows(x):
    """(q int8, scale float32 per row): scale = max|row| / 127 (1 for a zero
    row), q = rint(x / scale) -- the activation side of q_matmul (:61-62, :67)."""
    x = np.ascontiguousarray(x, np.float32)
    sa = np.abs(x).max(axis=1, keepdims=True) / np.float32(127.0)
    sa[sa == 0] = 1.0
    q = np.rint(x / sa).astype(np.int8)
    return q, sa[:, 0].astype(np.float32)


def weight_scales(B, mode):
    """(1, N) float32 weight scales of B (K, N): per column, or one for all."""
    B = np.ascontiguousarray(B, np.float32)
    if mode == "pertensor":
        sw = np.full((1, B.shape[1]), np.abs(B).max() / np.float32(127.0), np.float32)
    else:
        sw = np.abs(B).max(axis=0, keepdims=True) / np.float32(127.0)
    sw[sw == 0] = 1.0
    return sw


def q_matmul(A, B, bias=None, mode="perchan"):
    """int8 A @ B with fp32 out (:54-74). mode "fp32" is the unquantised
    control."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    if mode == "fp32":
        r = A @ B
        return r if bias is None else r + bias
    qa, sa = quantize_rows(A)
    sw = weight_scales(B, mode)
    qb = np.rint(B / sw).astype(np.int8)
    r = (qa.astype(np.float64) @ qb.astype(np.float64)).astype(np.float32)
    r = r * sa[:, None] * sw
    return r if bias is None else r + bias


def mlp_chunk_width(N, d):
    """Column chunk of fc1 in prepare_mlp_chunks(W, n_layer, d, 0) (:388-398):
    N itself up to MAX_GEMM_N, else d when d divides N, else N split evenly."""
    if N <= MAX_GEMM_N:
        return N
    if N % d == 0:
        return d
    return N // ((N + MAX_GEMM_N - 1) // MAX_GEMM_N)


def encoder_int8_np(W, mel, n_layer=None, n_head=None, mode="perchan"):
    """The reference encoder as the int8 probe runs it (fold_bias=False)."""
    if n_layer is None or n_head is None:
        nl, nh = geometry_of(W)
        n_layer = nl if n_layer is None else n_layer
        n_head = nh if n_head is None else n_head
    mm = lambda A, B: q_matmul(A, B, mode=mode)
    c1w = W["w.conv1.weight"]
    O, C, KS = c1w.shape
    x = mm(im2col(mel, KS, 1, 1), np.ascontiguousarray(c1w.reshape(O, C * KS).T)) \
        + W["w.conv1.bias"]
    x = gelu_np(x)
    c2w = W["w.conv2.weight"]
    O2, C2, KS2 = c2w.shape
    x = mm(im2col(np.ascontiguousarray(x.T), KS2, 2, 1),
           np.ascontiguousarray(c2w.reshape(O2, C2 * KS2).T)) + W["w.conv2.bias"]
    x = gelu_np(x)
    x = x + W["w.positional_embedding"][:x.shape[0]]
    ctx, d = x.shape
    hd = d // n_head
    scale = hd ** -0.25
    for L in range(n_layer):
        p = f"w.blocks.{L}."
        h = layer_norm_np(x, W[p + "attn_ln.weight"], W[p + "attn_ln.bias"])
        q = mm(h, W[p + "attn.query.weight"].T) + W[p + "attn.query.bias"]
        k = mm(h, W[p + "attn.key.weight"].T)
        v = mm(h, W[p + "attn.value.weight"].T) + W[p + "attn.value.bias"]
        o = np.empty_like(q)
        for hh in range(n_head):
            sl = slice(hh * hd, (hh + 1) * hd)
            s = mm_f32(np.ascontiguousarray(q[:, sl] * scale),
                       np.ascontiguousarray(k[:, sl].T) * scale)
            o[:, sl] = mm_f32(softmax_np(s), np.ascontiguousarray(v[:, sl]))
        x = x + mm(o, W[p + "attn.out.weight"].T) + W[p + "attn.out.bias"]
        h = layer_norm_np(x, W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"])
        W1, b1 = W[p + "mlp.0.weight"].T, W[p + "mlp.0.bias"]
        w = mlp_chunk_width(W1.shape[1], d)
        f = np.concatenate([mm(h, np.ascontiguousarray(W1[:, j:j + w])) + b1[j:j + w]
                            for j in range(0, W1.shape[1], w)], axis=1)
        f = gelu_np(f)
        x = x + mm(f, W[p + "mlp.2.weight"].T) + W[p + "mlp.2.bias"]
    return layer_norm_np(x, W["w.ln_post.weight"], W["w.ln_post.bias"])
