"""The allocation-free MLP entry point, wx_mlp_bf16_noalloc, through the C ABI.

It exists for callers that cannot call cudaMalloc -- processes whose device
memory belongs to another allocator, callers that must not allocate after
start-up -- and keeps the fc1 activation in the library's fixed device array
instead of memory the caller provides. Its result must equal the same
computation through the existing entry point (wx_gemm_bf16 for fc1 + GELU
into a caller buffer, then for fc2) on two calls in a row with different
inputs, so the shared array cannot hand one call's activation to the next.
A call after the first one leaves the device's free memory unchanged, and no
bounded wait of its kernels reports a timeout (wx_device_error covers this
path's own error word). This file is named to be collected last and passes
alone in a fresh process as well as after the other tests.
"""
import ctypes

import pytest
import torch

from wxb200 import _lib as L
from wxb200 import ops

pytestmark = pytest.mark.gpu

SCRATCH_ELEMS = 8 * 1024 * 1024  # the documented limit on M * ffn


def p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def inputs(M, d, ffn, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(M, d, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(ffn, d, generator=g) * 0.05).to(torch.bfloat16).cuda()
    w2 = (torch.randn(d, ffn, generator=g) * 0.05).to(torch.bfloat16).cuda()
    b1 = (torch.randn(ffn, generator=g) * 0.1).cuda()
    b2 = (torch.randn(d, generator=g) * 0.1).cuda()
    return h, w1, b1, w2, b2


def with_existing_entry_point(h, w1, b1, w2, b2, gelu_epi):
    f = ops.gemm(h, w1, bias=b1, epilogue=gelu_epi)           # caller-owned activation
    return ops.gemm(f, w2, bias=b2, epilogue=L.WX_EPI_F32)


def noalloc(h, w1, b1, w2, b2, gelu_mode):
    M, d = h.shape
    ffn = w1.shape[0]
    out = torch.empty(M, d, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L.check(L.lib().wx_mlp_bf16_noalloc(p(h), p(w1), p(b1), p(w2), p(b2), p(out), M, d, ffn,
                                        h.stride(0), out.stride(0), gelu_mode, st))
    return out


@pytest.mark.parametrize("M,d,ffn,gelu_mode,gelu_epi", [
    (1500, 1280, 5120, L.WX_GELU_POLY4, L.WX_EPI_BF16_GELU),    # one large-v3 clip
    (3000, 384, 1536, L.WX_GELU_POLY4, L.WX_EPI_BF16_GELU),     # two whisper-tiny clips
    (257, 384, 1536, L.WX_GELU_ERF, L.WX_EPI_BF16_GELU_ERF),    # ragged rows
])
def test_noalloc_matches_existing_entry_point_twice(M, d, ffn, gelu_mode, gelu_epi):
    assert torch.cuda.is_available()
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        args = inputs(M, d, ffn, seed + M)
        ref = with_existing_entry_point(*args, gelu_epi)
        got = noalloc(*args, gelu_mode)
        torch.cuda.synchronize()
        err = (got - ref).abs().max().item() / ref.abs().max().item()
        assert err < 1e-5, (call, err)           # the GEMM tests' fp32 bar
        assert torch.equal(got, ref), call       # same kernels: identical in practice
    assert L.device_error() == 0


def test_noalloc_warm_call_leaves_free_memory_unchanged():
    M, d, ffn = 1500, 1280, 5120
    h, w1, b1, w2, b2 = inputs(M, d, ffn, 7)
    out = torch.empty(M, d, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        L.check(L.lib().wx_mlp_bf16_noalloc(p(h), p(w1), p(b1), p(w2), p(b2), p(out), M, d,
                                            ffn, d, d, L.WX_GELU_POLY4, st))
        torch.cuda.synchronize()

    call()                                        # first call on the device: set-up
    free0, _ = torch.cuda.mem_get_info()
    call()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert L.device_error() == 0


def test_noalloc_rejects_sizes_beyond_the_scratch():
    assert torch.cuda.is_available()
    d, ffn = 1280, 5120
    M = SCRATCH_ELEMS // ffn + 1
    h = torch.empty(M, d, dtype=torch.bfloat16, device="cuda")
    w1 = torch.empty(ffn, d, dtype=torch.bfloat16, device="cuda")
    w2 = torch.empty(d, ffn, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(M, d, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lib().wx_mlp_bf16_noalloc(p(h), p(w1), None, p(w2), None, p(out), M, d, ffn, d, d,
                                     L.WX_GELU_POLY4, st)
    assert rc == L.WX_ERR_INVALID
    assert "exceeds the fixed scratch" in L.last_error()
