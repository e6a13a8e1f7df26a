"""tcgen05 GEMM against a plain torch fp32 reference of the same op.

Operands are bf16 (exact in fp32), so the reference is the fp32 product of
the same values; the device accumulates in fp32 in a different order, so the
bar is a relative error of 1e-5 of the output scale for fp32 epilogues and one
bf16 rounding (2^-8 relative) for bf16 ones. The GELU epilogue is compared
bit-exactly to the oracle applied to the device's own fp32 accumulator
(WX_EPI_F32 of the same GEMM).
"""
import numpy as np
import pytest
import torch

import rowops_ref as O
from wxb200 import _lib as L
from wxb200 import ops

pytestmark = pytest.mark.gpu


def rand_bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).cuda()


def ref_mm(A, W, bias=None, resid=None):
    r = A.float() @ W.float().T
    if bias is not None:
        r = r + bias
    if resid is not None:
        r = r + resid
    return r


SHAPES = [
    (1500, 1152, 384),     # tiny QKV
    (1500, 384, 1536),     # tiny fc2
    (3000, 384, 240),      # tiny conv1 (K = 3 * 80, not a multiple of 64)
    (1500, 3840, 1280),    # large-v3 QKV
    (1500, 5120, 1280),    # large-v3 fc1
    (1500, 1280, 5120),    # large-v3 fc2
    (4500, 1280, 1280),    # three clips, out-proj
    (1, 128, 64), (129, 136, 72), (200, 40, 8), (257, 520, 1000),  # ragged tails
]


# Shapes large enough for the 2-SM kernel (CTA pairs, 256 x 256 tiles: at
# least 74 pair tiles), with M, N and K off every tile boundary.
PAIR_SHAPES = [(5000, 1000, 1000), (4100, 1288, 1336), (19000, 256, 64), (1500, 5120, 1280)]


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
@pytest.mark.parametrize("epi", ["f32", "bf16", "resid", "gelu"])
def test_gemm_pair_kernel_epilogues(cuda, M, N, K, epi):
    A, W = rand_bf16((M, K), M + 3), rand_bf16((N, K), N + 5, 0.05)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(K)).cuda() * 0.1
    if epi == "f32":
        got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_F32)
        ref = ref_mm(A, W, bias)
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-5
    elif epi == "bf16":
        got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_BF16).float()
        ref = ref_mm(A, W, bias)
        assert ((got - ref).abs() <= ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max()).all()
    elif epi == "resid":
        x = torch.randn(M, N, generator=torch.Generator().manual_seed(M)).cuda()
        ref = ref_mm(A, W, bias, x)
        ops.gemm(A, W, bias=bias, residual=x, out=x, epilogue=L.WX_EPI_F32_RESID)
        assert (x - ref).abs().max().item() / ref.abs().max().item() < 1e-5
    else:
        acc = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_F32)
        got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_BF16_GELU)
        g = (got.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16)
        assert np.array_equal(g.view(np.float32), O.gelu_row4f(acc.cpu().numpy()))
    assert L.device_error() == 0


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_f32_bias(cuda, M, N, K):
    A, W = rand_bf16((M, K), M + K), rand_bf16((N, K), N + 1, 0.05)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(N)).cuda() * 0.1
    got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_F32)
    ref = ref_mm(A, W, bias)
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


@pytest.mark.parametrize("M,N,K", SHAPES[:6])
def test_gemm_bf16_out(cuda, M, N, K):
    A, W = rand_bf16((M, K), 3), rand_bf16((N, K), 4, 0.05)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(5)).cuda() * 0.1
    got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_BF16).float()
    ref = ref_mm(A, W, bias)
    assert ((got - ref).abs() <= ref.abs() * 2 ** -8 + 1e-3 * ref.abs().max()).all()


@pytest.mark.parametrize("M,N,K", [(1500, 1280, 1280), (1500, 384, 1536), (300, 520, 200)])
def test_gemm_residual_in_place(cuda, M, N, K):
    A, W = rand_bf16((M, K), 6), rand_bf16((N, K), 7, 0.05)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(8)).cuda() * 0.1
    x = torch.randn(M, N, generator=torch.Generator().manual_seed(9)).cuda()
    ref = ref_mm(A, W, bias, x)
    ops.gemm(A, W, bias=bias, residual=x, out=x, epilogue=L.WX_EPI_F32_RESID)
    err = (x - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


@pytest.mark.parametrize("M,N,K", [(19200, 1280, 5120), (19017, 1280, 4096)])
def test_gemm_residual_in_place_equals_separate_output(cuda, M, N, K):
    """Long-K residual GEMMs on CTA pairs (fc2's shape) add the residual in
    place by a TMA reduce-add in L2 when C is the residual; the bits equal those
    of the path that loads the residual into the epilogue (a separate output)."""
    A, W = rand_bf16((M, K), 11), rand_bf16((N, K), 12, 0.02)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(13)).cuda() * 0.1
    x = torch.randn(M, N, generator=torch.Generator().manual_seed(14)).cuda()
    y = torch.empty_like(x)
    ops.gemm(A, W, bias=bias, residual=x, out=y, epilogue=L.WX_EPI_F32_RESID)
    ops.gemm(A, W, bias=bias, residual=x, out=x, epilogue=L.WX_EPI_F32_RESID)
    assert torch.equal(x, y)
    assert L.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(1500, 5120, 1280), (1500, 1536, 384), (77, 264, 72)])
def test_gemm_gelu_epilogue_matches_g4f(cuda, M, N, K):
    """fc1 -> g4f fused: bit-exact to the oracle's g4f of the fp32 accumulator."""
    A, W = rand_bf16((M, K), 10), rand_bf16((N, K), 11, 0.1)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(12)).cuda()
    acc = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_F32)
    got = ops.gemm(A, W, bias=bias, epilogue=L.WX_EPI_BF16_GELU)
    g = (got.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(g, O.gelu_row4f(acc.cpu().numpy()))


def test_gemm_gelu_erf_epilogue(cuda):
    A, W = rand_bf16((1500, 1280), 13), rand_bf16((5120, 1280), 14, 0.05)
    got = ops.gemm(A, W, epilogue=L.WX_EPI_BF16_GELU_ERF).float()
    ref = torch.nn.functional.gelu(ref_mm(A, W))
    assert ((got - ref).abs() <= ref.abs() * 2 ** -8 + 1e-4).all()


def test_gemm_strided_operands(cuda):
    """A as a column slice of a wider buffer, C written into a band."""
    big = rand_bf16((700, 3 * 128), 15)
    W = rand_bf16((96, 128), 16)
    out = torch.zeros(700, 256, device="cuda")
    ops.gemm(big[:, 128:256], W, out=out[:, 64:160], epilogue=L.WX_EPI_F32)
    ref = ref_mm(big[:, 128:256], W)
    assert (out[:, 64:160] - ref).abs().max().item() < 1e-4 * ref.abs().max().item()
    assert out[:, :64].abs().max().item() == 0 and out[:, 160:].abs().max().item() == 0


def test_no_device_error_recorded(cuda):
    assert L.device_error() == 0
