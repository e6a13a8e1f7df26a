"""The RawRT surface (src/rawxrt.py) on the B200 and the rowops design
functions (src/rowops.py), driven the way the reference's callers drive them.
"""
import math

import ml_dtypes
import numpy as np
import pytest
import torch

import encoder_ref as R
import rowops_ref as O
from wxb200 import rowops
from wxb200.runtime import B200RT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt(cuda):
    return B200RT()


def test_matmul_with_folded_bias(rt):
    rng = np.random.default_rng(0)
    A = rng.standard_normal((1500, 384)).astype(np.float32)
    B = (0.05 * rng.standard_normal((384, 1152))).astype(np.float32)
    b = rng.standard_normal(1152).astype(np.float32)
    rt.register_weights([B, b])
    got = rt.matmul(A, B, akey="x", bias=b)
    ref = O.rbf(A, O.RNE) @ O.rbf(B, O.RNE) + b
    assert np.abs(got - ref).max() < 1e-4 * np.abs(ref).max()
    # the named activation is reused, the registered weight is cached
    h = rt.mm_start(A, B, akey="x", bias=b)
    assert np.array_equal(rt.mm_finish(h), got)


def test_attn_chain_matches_reference_math(rt):
    """attn_chain(q, k, v, nh, scale): softmax((q*s)(k*s)^T) v per head."""
    rng = np.random.default_rng(1)
    ctx, nh, hd = 1500, 6, 64
    q, k, v = (rng.standard_normal((ctx, nh * hd)).astype(np.float32) for _ in range(3))
    s = hd ** -0.25
    got = rt.attn_chain(q, k, v, nh, s)
    ref = np.empty_like(q)
    for h in range(nh):
        sl = slice(h * hd, (h + 1) * hd)
        ref[:, sl] = O.softmax_fp32((q[:, sl] * s) @ (k[:, sl] * s).T) @ v[:, sl]
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-2


def test_mlp_chunks_and_gelu(rt):
    rng = np.random.default_rng(2)
    d, ffn, M = 384, 1536, 700
    h = rng.standard_normal((M, d)).astype(np.float32)
    W1 = (0.05 * rng.standard_normal((d, ffn))).astype(np.float32)
    b1 = (0.1 * rng.standard_normal(ffn)).astype(np.float32)
    W2 = (0.05 * rng.standard_normal((ffn, d))).astype(np.float32)
    parts = [(np.ascontiguousarray(W1[:, j:j + 512]), b1[j:j + 512]) for j in range(0, ffn, 512)]
    got = rt.mlp(h, parts, W2)
    hb, w1b, w2b = O.rbf(h, O.RNE), O.rbf(W1, O.RNE), O.rbf(W2, O.RNE)
    f = O.gelu_row4f(hb @ w1b + b1)
    ref = f @ w2b
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-3


def test_gelu_any_shape(rt):
    rng = np.random.default_rng(3)
    x = (3 * rng.standard_normal((3000, 384))).astype(np.float32)
    got = rt.gelu(x)
    assert got.shape == x.shape
    assert np.array_equal(got, O.gelu_row4_rne(O.rbf(x, O.RNE)))


def test_softmax_stack(rt):
    rng = np.random.default_rng(4)
    mats = [rng.normal(0, 6, (1500, 1500)).astype(np.float32) for _ in range(3)]
    got = rt.softmax_stack(mats)
    for g, m in zip(got, mats):
        assert g.shape == (1500, 1500)
        xb = O.rbf(m, O.RNE)
        pad = np.concatenate([xb, np.full((1500, 4), -29952.0, np.float32)], axis=1)
        ref = O.softmax_row(pad, mode=O.TRUNC, variant=3)[:, :1500]
        assert np.array_equal(g, ref)


def test_rowop_codes(rt):
    rng = np.random.default_rng(5)
    x = O.rbf(rng.normal(0, 3, (64, 1024)).astype(np.float32), O.RNE).astype(ml_dtypes.bfloat16)
    xf = x.astype(np.float32)
    assert np.array_equal(rt.rowop("g4r", x, 64, 1024).astype(np.float32), O.gelu_row4_rne(xf))
    assert np.array_equal(rt.rowop("s4w", x, 64, 1024, valid=1008)[:, :1008].astype(np.float32),
                          O.softmax_row(xf, mode=O.TRUNC, variant=4, valid=1008))
    assert np.array_equal(rt.rowop("ln", x, 64, 1024).astype(np.float32),
                          O.layer_norm_aie(xf, O.TRUNC))
    with pytest.raises(ValueError):
        rt.rowop("s4w", x, 64, 1024, valid=1000)


def test_rowops_designs_in_place(cuda):
    """design(a_t, c_t, rows=..., cols=...) writes into c_t (tests/test_rowops.py:19-23)."""
    rng = np.random.default_rng(6)
    rows, cols = 1536, 384
    x = O.rbf(rng.normal(0, 1, (rows, cols)).astype(np.float32), O.RNE)
    a_t = torch.from_numpy(O.bf16_bits(x, O.RNE).view(np.int16)).view(torch.bfloat16).cuda()
    c_t = torch.zeros(rows, cols, dtype=torch.bfloat16, device="cuda")
    rowops.layer_norm(a_t, c_t, rows=rows, cols=cols)
    got = (c_t.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(got, O.layer_norm_aie(x, O.TRUNC))
    c_np = np.zeros((rows, cols), ml_dtypes.bfloat16)
    rowops.softmax_row4r_win(x.astype(ml_dtypes.bfloat16), c_np, rows=rows, cols=cols, valid=368)
    assert np.array_equal(c_np[:, :368].astype(np.float32),
                          O.softmax_row(x, mode=O.RNE, variant=4, valid=368))
    with pytest.raises(ValueError, match="multiple of 16"):
        rowops.softmax_row4_win(a_t, c_t, rows=rows, cols=cols, valid=370)
    with pytest.raises(NotImplementedError):
        rowops.gelu_row(a_t, c_t, rows=rows, cols=cols)


def test_gelu_row4f_band(cuda):
    rng = np.random.default_rng(7)
    rows, w = 512, 256
    xs = [(3 * rng.standard_normal((rows, w))).astype(np.float32) for _ in range(2)]
    big = torch.zeros(rows, 2 * w, dtype=torch.bfloat16, device="cuda")
    for j, x in enumerate(xs):
        rowops.gelu_row4f(torch.from_numpy(x).cuda(), big[:, j * w:], rows=rows, cols=w,
                          out_cols=2 * w)
    got = (big.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    for j, x in enumerate(xs):
        assert np.array_equal(got[:, j * w:(j + 1) * w], O.gelu_row4f(x))


def test_fault_injection_surfaces_as_exception(rt, monkeypatch):
    """The reference's test 4 (tests/test_encoder_golden.py:137-160) injected a
    failing device chain and expected a host fallback. There is no host path
    here: an injected failure must surface as an exception, not a silent
    result."""
    from wxb200 import ops

    def boom(*a, **kw):
        raise RuntimeError("injected: kernel launch failed")

    monkeypatch.setattr(ops, "attention", boom)
    q = np.zeros((64, 384), np.float32)
    with pytest.raises(RuntimeError, match="injected"):
        rt.attn_chain(q, q, q, 6, 0.35)
    assert rt.fallbacks == []


def test_encoder_engine_rebuilt_when_an_array_is_replaced(rt):
    """The engine cache follows the arrays of W: replacing one (here ln_post's
    bias, +1 on every output) builds a new engine; an unchanged W reuses it."""
    W = R.make_weights("tiny", seed=5, n_layer=1, n_ctx=64)
    mel = R.make_mel(80, 128, seed=5)
    from wxb200.encoder import encoder
    a = encoder(W, mel, rt.matmul, n_layer=1, n_head=6)
    eng = rt.encoder_engine(W, 1, 6)
    assert rt.encoder_engine(W, 1, 6) is eng
    W["w.ln_post.bias"] = np.asarray(W["w.ln_post.bias"], np.float32) + 1.0
    b = encoder(W, mel, rt.matmul, n_layer=1, n_head=6)
    assert rt.encoder_engine(W, 1, 6) is not eng
    assert np.allclose(b, a + 1.0, atol=1e-5)
