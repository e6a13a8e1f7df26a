"""Time one kernel of the hot path at the encoder's shapes, through the C ABI.

    PYTHONPATH=whisper-xdna_b200 python -m wxb200.kernel_bench --kernel attention --batch 4

Kernels: encoder (a whole forward), attention, fc1 (GEMM + GELU), fc2 (GEMM + residual), qkv, outproj,
their int8 twins fc1_i8, fc2_i8, qkv_i8, outproj_i8 (the int8 mode's GEMMs),
quantize_bf16 (fc2's input rows, maxima given) and quantize_f32 (an LN output),
layernorm (fp32 -> bf16, the encoder's), and the standalone row ops at the
BASELINE row-op sizes: gelu (g4r 1500x5120), gelu_f32 (g4f 1500x5120), softmax
(s4r 20x1500x1500, scale 1/8), layernorm_gb (1500x1280 with gamma/beta), and
log_mel (batch clips of 30 s audio -> 128 x 3000 features; FLOP = the direct
DFT's 4 per sample, bin and frame).
Each launch is timed with CUDA events on the launching stream after warm-up;
with --flush the L2 (126 MB) is overwritten between launches, which the row
ops need since their inputs fit in L2. Prints one JSON line.
"""
import argparse
import json

import torch

from . import _lib as L
from . import ops

D, H, FFN, T = 1280, 20, 5120, 1500


def setup(kernel, batch, dev="cuda", ctx=T, layers=32):
    """Return (fn, flop_per_launch, bytes_per_launch) for one kernel; ctx is
    the frame count of the attention kernel's clips (the encoder's T).
    kernel "encoder": one whole large-v3 forward of `batch` clips (ctx 1500,
    `layers` layers, random weights), the captured launch sequence."""
    g = torch.Generator(device=dev).manual_seed(0)
    if kernel == "encoder":
        from .encoder import Encoder, synthetic_weights
        enc = Encoder(synthetic_weights(n_layer=layers), n_layer=layers, max_batch=batch)
        mel = torch.rand(batch, 128, 2 * T, device=dev, generator=g) * 2 - 0.8
        out = torch.empty(batch, T, D, device=dev)
        flop = batch * (layers * (8 * T * D * D + 4 * T * D * FFN + 4 * T * T * D)
                        + 2 * (2 * T) * (3 * 128) * D + 2 * T * (3 * D) * D)
        return (lambda: enc.forward(mel, out=out)), float(flop), batch * (128 * 2 * T + T * D) * 4
    M = batch * T
    rn = lambda *s, sc=1.0: (torch.randn(*s, device=dev, generator=g) * sc)
    if kernel == "attention":
        Ma = batch * ctx
        qkv = rn(Ma, 3 * D).to(torch.bfloat16)
        o = torch.empty(Ma, D, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], batch, H, 0.125,
                                   out=o)
        return fn, 4.0 * batch * ctx * ctx * D, 4.0 * Ma * D * 2
    if kernel in ("fc1", "fc2", "qkv", "outproj"):
        K, N = {"fc1": (D, FFN), "fc2": (FFN, D), "qkv": (D, 3 * D), "outproj": (D, D)}[kernel]
        A = rn(M, K).to(torch.bfloat16)
        W = rn(N, K, sc=0.02).to(torch.bfloat16)
        b = torch.zeros(N, device=dev)
        if kernel in ("fc2", "outproj"):
            x = rn(M, N)
            fn = lambda: ops.gemm(A, W, bias=b, residual=x, out=x, epilogue=L.WX_EPI_F32_RESID)
            byt = M * K * 2 + N * K * 2 + 2 * M * N * 4
        else:
            C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            epi = L.WX_EPI_BF16_GELU if kernel == "fc1" else L.WX_EPI_BF16
            fn = lambda: ops.gemm(A, W, bias=b, out=C, epilogue=epi)
            byt = M * K * 2 + N * K * 2 + M * N * 2
        return fn, 2.0 * M * N * K, byt
    if kernel in ("fc1_i8", "fc2_i8", "qkv_i8", "outproj_i8"):
        # the int8 mode's GEMMs (int8 operands, s32 accumulation, dequantising epilogue)
        base = kernel[:-3]
        K, N = {"fc1": (D, FFN), "fc2": (FFN, D), "qkv": (D, 3 * D), "outproj": (D, D)}[base]
        Aq = torch.randint(-127, 128, (M, K), device=dev, dtype=torch.int8, generator=g)
        Wq = torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8, generator=g)
        sa = torch.rand(M, device=dev, generator=g) * 1e-2
        sw = torch.rand(N, device=dev, generator=g) * 1e-3
        b = torch.zeros(N, device=dev)
        if base in ("fc2", "outproj"):
            x = rn(M, N)
            fn = lambda: ops.gemm_i8(Aq, Wq, sa, sw, bias=b, residual=x, out=x,
                                     epilogue=L.WX_EPI_F32_RESID)
            byt = M * K + N * K + 2 * M * N * 4
        else:
            C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            epi = L.WX_EPI_BF16_GELU if base == "fc1" else L.WX_EPI_BF16
            rm = torch.zeros(M, device=dev) if base == "fc1" else None
            fn = lambda: ops.gemm_i8(Aq, Wq, sa, sw, bias=b, out=C, epilogue=epi, rowmax=rm)
            byt = M * K + N * K + M * N * 2
        return fn, 2.0 * M * N * K, byt
    if kernel in ("quantize_bf16", "quantize_f32"):
        # per-token quantisation of the fc2 input (bf16, M x ffn, maxima given)
        # or of an LN output (fp32, M x d)
        if kernel == "quantize_bf16":
            x = rn(M, FFN).to(torch.bfloat16)
            rm = x.float().abs().amax(dim=1)
        else:
            x, rm = rn(M, D), None
        q = torch.empty(x.shape, device=dev, dtype=torch.int8)
        sc = torch.empty(M, device=dev)
        fn = lambda: ops.quantize_rows(x, rowmax=rm, q=q, scale=sc)
        return fn, 0.0, x.numel() * (x.element_size() + 1) + M * 4
    if kernel == "layernorm":
        x = rn(M, D)
        h = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        gm, bt = torch.ones(D, device=dev), torch.zeros(D, device=dev)
        fn = lambda: ops.layer_norm_rows(x, gm, bt, out=h, mode=L.WX_LN_FP32)
        return fn, 0.0, M * D * (4 + 2) + 2 * D * 4
    # standalone row ops, BASELINE sizes (batch ignored)
    if kernel.startswith("copy:"):
        # the floor for moving the same bytes: torch's device copy (y <- x) of
        # the named row op's input and output tensors, for scale
        name = kernel[5:]
        shapes = {"gelu": (1500, 5120), "gelu_1536": (1500, 1536), "gelu_f32": (1500, 5120),
                  "softmax": (20 * 1500, 1500), "layernorm_gb": (1500, 1280),
                  "layernorm_gb_384": (1500, 384)}
        if name not in shapes:
            raise ValueError(f"copy: of {name!r}")
        shape = shapes[name]
        x = rn(*shape)
        if name != "gelu_f32":
            x = x.to(torch.bfloat16)
        y = torch.empty(*shape, device=dev, dtype=torch.bfloat16)
        return (lambda: y.copy_(x)), 0.0, x.numel() * x.element_size() + y.numel() * 2
    if kernel == "gelu_1536":   # the sweep's smaller GELU (whisper-tiny's FFN width)
        x = (rn(1500, 1536) * 3).to(torch.bfloat16)
        y = torch.empty_like(x)
        return (lambda: ops.gelu_poly4(x, out=y, rounding=L.WX_ROUND_RNE)), 0.0, x.numel() * 4
    if kernel == "layernorm_gb_384":   # the sweep's smaller LayerNorm (whisper-tiny's width)
        x = (rn(1500, 384) * 3).to(torch.bfloat16)
        y = torch.empty_like(x)
        gm, bt = rn(384, sc=0.1) + 1, rn(384, sc=0.1)
        fn = lambda: ops.layer_norm_rows(x, gm, bt, out=y, mode=L.WX_LN_AIE,
                                         rounding=L.WX_ROUND_RNE)
        return fn, 0.0, x.numel() * 4 + 2 * 384 * 4
    if kernel == "gelu":
        x = (rn(1500, 5120) * 3).to(torch.bfloat16)
        y = torch.empty_like(x)
        return (lambda: ops.gelu_poly4(x, out=y, rounding=L.WX_ROUND_RNE)), 0.0, x.numel() * 4
    if kernel == "gelu_f32":
        x = rn(1500, 5120) * 3
        y = torch.empty(1500, 5120, device=dev, dtype=torch.bfloat16)
        return (lambda: ops.gelu_poly4(x, out=y, rounding=L.WX_ROUND_RNE)), 0.0, x.numel() * 6
    if kernel == "softmax":
        x = (rn(20 * 1500, 1500) * 3).to(torch.bfloat16)
        y = torch.empty_like(x)
        fn = lambda: ops.softmax_rows(x, out=y, scale=0.125, variant=4, rounding=L.WX_ROUND_RNE)
        return fn, 0.0, x.numel() * 4
    if kernel == "layernorm_gb":
        x = (rn(1500, 1280) * 3).to(torch.bfloat16)
        y = torch.empty_like(x)
        gm, bt = rn(1280, sc=0.1) + 1, rn(1280, sc=0.1)
        fn = lambda: ops.layer_norm_rows(x, gm, bt, out=y, mode=L.WX_LN_AIE,
                                         rounding=L.WX_ROUND_RNE)
        return fn, 0.0, x.numel() * 4 + 2 * 1280 * 4
    if kernel == "log_mel":
        # batch clips of 30 s audio -> (batch, 128, 3000) features
        a = rn(batch, 480000, sc=0.1)
        y = torch.empty(batch, 128, 3000, device=dev)
        fn = lambda: ops.log_mel(a, n_mels=128, out=y)
        return fn, batch * 3000 * 201 * 400 * 4.0, batch * (480000 + 128 * 3000) * 4
    raise ValueError(f"unknown kernel {kernel!r}")


def time_kernel(kernel, batch=4, iters=10, warmup=3, flush=False, ctx=T, graph=False,
                flush_mode="write", layers=32):
    """graph=True captures the `iters` launches in one CUDA graph and times its
    replay, so kernels shorter than the host's per-call cost (small batches)
    are timed as they run inside the encoder's graph, not at the rate the
    host can issue them."""
    """flush_mode: how L2 is emptied between launches with flush=True: "write"
    fills a 1 GiB buffer (L2 is left full of dirty lines, whose write-back the
    timed kernel then pays for as it evicts them), "read" sums it (L2 is left
    full of clean lines)."""
    fn, flop, byt = setup(kernel, batch, ctx=ctx, layers=layers)
    if graph:
        if flush:
            raise ValueError("graph timing does not flush L2 between launches")
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            for _ in range(warmup):
                fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream()
        e0.record(cur)
        g.replay()
        e1.record(cur)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / iters
        res = {"kernel": kernel, "batch": batch, "s": t, "flop": flop, "bytes": byt,
               "flush_l2": False, "graph": True}
        if kernel == "attention":
            res["ctx"] = ctx
        if flop:
            res["tflops"] = flop / t / 1e12
        res["gbs"] = byt / t / 1e9
        return res
    # 1 GiB: its fill (~160 us) outlasts the host-side cost of one launch
    junk = torch.ones(1024 * 1024 * 1024 // 4, device="cuda") if flush else None
    junk_sum = torch.empty((), device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    if flush:
        # Everything is enqueued before one synchronize: while the GPU writes
        # the flush buffer the host has already queued the timed launch, so
        # the event pair brackets the kernel, not the host's launch overhead.
        evs = []
        for _ in range(iters):
            if flush_mode == "read":
                torch.sum(junk, dim=0, out=junk_sum)
            else:
                junk.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        total = sum(a.elapsed_time(b) for a, b in evs) / 1e3
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(iters):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        total = e0.elapsed_time(e1) / 1e3
    t = total / iters
    res = {"kernel": kernel, "batch": batch, "s": t, "flop": flop, "bytes": byt,
           "flush_l2": bool(flush)}
    if flush:
        res["flush_mode"] = flush_mode
    if kernel == "attention":
        res["ctx"] = ctx
    if flop:
        res["tflops"] = flop / t / 1e12
    res["gbs"] = byt / t / 1e9
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="attention")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--flush", action="store_true")
    ap.add_argument("--flush-mode", choices=["write", "read"], default="write")
    ap.add_argument("--layers", type=int, default=32, help="encoder only: layers")
    ap.add_argument("--graph", action="store_true",
                    help="time the launches captured in one CUDA graph")
    ap.add_argument("--ctx", type=int, default=T,
                    help="attention only: frames per clip (T <= 1344 runs the persistent kernel)")
    a = ap.parse_args()
    res = time_kernel(a.kernel, a.batch, a.iters, a.warmup, a.flush, ctx=a.ctx, graph=a.graph,
                      flush_mode=a.flush_mode, layers=a.layers)
    res["device_error"] = L.device_error()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
