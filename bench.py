#!/usr/bin/env python3
"""Benchmark of the Whisper-encoder hot path on B200: large-v3 encoder forward,
ctx 1500, clips sharded across GPUs (one encoder replica per GPU, no
collective on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]

A step is one encoder forward over the rank's B clips (default 64, the
BASELINE batch-64 config; weak scaling: each GPU encodes B clips per step).
Prints ONE JSON line on rank 0. Synthetic data: random N(0, 0.02) weights of
the large-v3 architecture, log-mel ~ U[-0.8, 1.2] seeded per clip (no
checkpoint or audio can be fetched here).

--impl reference times the reference's own CPU implementation of the path --
its numpy encoder (src/npu_whisper_encoder.py:encoder with np_matmul),
restated in oracle/encoder_ref.py because the reference's Python cannot travel
to the GPU box -- on all the host cores, one whole 32-layer clip per step.

Beside the weak-scaling value the line carries `fixed_global_batch`: the same
loop with one global batch (--global-batch, default 64) split into contiguous
per-GPU slices (strong scaling), and `per_rank`: every rank's own step time,
SM clock and power, so the rank that limits the max-over-ranks time is named.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "whisper-xdna_b200"))

METRIC = "large-v3 encoder clips/s @ctx1500"
UNIT = "clips/s"
N_MELS, D, N_HEAD, N_LAYER, FFN, CTX = 128, 1280, 20, 32, 5120, 1500
# DRAM bytes (read + write) of one attention launch per clip, measured by ncu
# on one launch at the benchmarked 64 clips (profiles/attention_ncu_b64.md:
# 737.57 MB read = Q, K, V once; 226.14 MB written of the 245.8 MB of O)
ATTN_DRAM_BYTES_PER_CLIP = (737.565e6 + 226.136e6) / 64
# nominal fp32 FMA rate (148 SMs x 128 lanes x 2 FLOP x 1.965 GHz) for the
# log-mel kernel's DFT, which runs on the FMA pipe (no measured fp32 peak)
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# ctx 512: 32 layers at T = 512 + the conv frontend over 1024 frames
FLOP_PER_CLIP_512 = (32 * (8 * 512 * 1280 * 1280 + 4 * 512 * 1280 * 5120 + 4 * 512 * 512 * 1280)
                     + 2 * 1024 * 384 * 1280 + 2 * 512 * 3840 * 1280)
FLOP_PER_CLIP = (N_LAYER * (8 * CTX * D * D + 4 * CTX * D * FFN + 4 * CTX * CTX * D)
                 + 2 * (2 * CTX) * (3 * N_MELS) * D + 2 * CTX * (3 * D) * D)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=64, help="clips per GPU per step")
    ap.add_argument("--global-batch", type=int, default=64,
                    help="fixed-batch leg: this many clips per step split across the GPUs")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quant", choices=["none", "int8-perchan", "int8-pertensor"],
                    default="none",
                    help="int8 projection/MLP mode (the reference's int8 probe); not the "
                         "headline configuration, which is bf16")
    return ap.parse_args()


def arm_config(batch, world, quant="none"):
    """The workload both arms report (the reference arm times a bounded sample
    of it)."""
    cfg = {"workload": f"large-v3 encoder forward, ctx 1500, {batch} clips per GPU per step "
                       "(BASELINE batch-64 config, clip-sharded)",
           "model": "whisper large-v3 encoder (32 layers, d 1280, 20x64 heads, ffn 5120)",
           "global_batch": batch * world, "seq_len": CTX,
           "parallelism": f"dp{world} (independent replicas, no collective)",
           "gelu": "poly4 RNE (the reference's device GELU)",
           "l2": "inputs larger than L2 (no flush)", "cuda_graph": True}
    if quant != "none":
        cfg["quant"] = (f"{quant}: int8 conv/QKV/out-proj/fc1/fc2 GEMMs with per-token "
                        "activation scales (bench/probe_int8_decode.py:48-74), bf16 attention")
    return cfg


# ------------------------------------------------------------------ CPU side

def cpu_clips(W, min_seconds=10.0, max_clips=3, first_seed=0):
    """Time the oracle port of the reference's numpy encoder on whole large-v3
    clips (frontend, 32 layers, ln_post; ctx 1500) until at least
    min_seconds have passed or max_clips are done.
    Returns (clips_per_s, seconds_spent, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import encoder_ref as R
    t0 = time.perf_counter()
    n = 0
    while n < max_clips:
        mel = R.make_mel(N_MELS, 2 * CTX, seed=first_seed + n)
        R.encoder_np(W, mel, n_layer=N_LAYER, n_head=N_HEAD)
        n += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    spent = time.perf_counter() - t0
    desc = (f"{n} whole clip{'s' if n > 1 else ''} of large-v3 ctx 1500 (frontend, 32 layers, "
            f"ln_post), {spent / n:.1f} s per clip")
    return n / spent, spent, desc


def cpu_cores():
    try:
        import numpy as np  # noqa: F401
        from threadpoolctl import threadpool_info
        n = max((i.get("num_threads", 0) for i in threadpool_info()), default=0)
        if n:
            return n
    except Exception:
        pass
    return os.cpu_count() or 1


def run_reference(args, rank):
    if rank != 0:
        return
    # All host threads. torchrun gives each worker OMP_NUM_THREADS=1, and the
    # BLAS libraries read their thread count when they load, so the variables
    # are set before numpy or torch is first imported (nothing above imports
    # either); the limits are applied again once they are loaded.
    n = os.cpu_count() or 1
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    import torch
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    sys.path.insert(0, str(ROOT / "oracle"))
    import encoder_ref as R
    W = make_weights_fast(seed=1)
    for i in range(args.warmup):   # one layer per warm-up step
        R.encoder_np(W, R.make_mel(N_MELS, 2 * CTX, seed=100 + i), n_layer=1, n_head=N_HEAD)
    vals, desc = [], ""
    for i in range(args.steps):    # one whole clip per step
        v, _, desc = cpu_clips(W, min_seconds=0.0, max_clips=1, first_seed=i)
        vals.append(v)
    value = statistics.median(vals)
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": arm_config(args.batch, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                         "sample": desc + "; the oracle port of the reference's numpy encoder, "
                                          "all host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ GPU side

class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, mx, pw, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            try:
                pw.append(float(f[3]))
            except ValueError:
                pass
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(pw) if pw else None}


def make_weights_fast(seed):
    """Random N(0, 0.02) large-v3 weights (torch CPU generator, bf16-exact),
    LayerNorm 1 / 0, sinusoidal positions, in the reference's W-dict layout."""
    from wxb200.encoder import synthetic_weights
    return synthetic_weights(N_MELS, D, FFN, N_LAYER, CTX, seed=seed)


def kernel_rooflines(batch, peaks):
    """Time the encoder's kernels one at a time (CUDA events on the launching
    stream) at this rank's shapes, whose inputs are larger than L2, and the
    standalone row ops at the BASELINE row-op sizes with L2 flushed between
    launches (their inputs fit in L2)."""
    from wxb200.kernel_bench import time_kernel
    res = {}
    for k in ("attention", "fc1", "fc2", "qkv", "outproj", "layernorm"):
        r = time_kernel(k, batch=batch, iters=5 if k == "attention" else 10)
        if r["flop"]:
            r["frac_of_measured_bf16"] = r["tflops"] / peaks["bf16_tflops"]
        else:
            r["frac_of_measured_hbm"] = r["gbs"] / peaks["hbm_gbs"]
        res[k] = r
    rows = {}
    for k in ("gelu", "gelu_1536", "gelu_f32", "softmax", "layernorm_gb", "layernorm_gb_384"):
        r = time_kernel(k, iters=20, flush=True)
        r["frac_of_measured_hbm"] = r["gbs"] / peaks["hbm_gbs"]
        rows[k] = r
    # the device log-mel frontend (row f2): this rank's clips of 30 s audio
    r = time_kernel("log_mel", batch=batch, iters=5)
    r["clips_per_s"] = batch / r["s"]
    r["frac_of_nominal_fp32"] = r["tflops"] / FP32_NOMINAL_TFLOPS
    res["log_mel"] = r
    return res, rows


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "src": "fallback"}


def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    from wxb200.encoder import Encoder

    B = args.batch
    W = make_weights_fast(seed=1)
    quant = None if args.quant == "none" else args.quant
    enc = Encoder(W, max_batch=B, gelu="poly4", quant=quant)
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline and quant is None
    if not want_cpu:
        del W
    # per-clip seeded mel, pinned host copy for the end-to-end leg
    g = torch.Generator().manual_seed(1000 + rank)
    mel_host = torch.empty(B, N_MELS, 2 * CTX, pin_memory=True)
    mel_host.copy_(torch.rand(B, N_MELS, 2 * CTX, generator=g) * 2.0 - 0.8)
    out_host = torch.empty(B, CTX, D, pin_memory=True)
    mel = mel_host.cuda()
    out = torch.empty(B, CTX, D, device="cuda")
    st = torch.cuda.current_stream()

    from wxb200 import dist as wdist
    barrier = wdist.barrier
    max_over_ranks = wdist.max_over_ranks

    # ---- device-resident timing
    for _ in range(args.warmup):
        enc.forward(mel, out=out)
    torch.cuda.synchronize()
    barrier()
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    e0.record(st)
    for _ in range(args.steps):
        enc.forward(mel, out=out)
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    t_rank = e0.elapsed_time(e1) / 1e3
    t_dev = max_over_ranks(t_rank)
    finite = bool(torch.isfinite(out).all().item())
    # which rank limits the job: each rank's own step time, clock and power
    per_rank = wdist.gather_to_all({
        "rank": rank, "ms_per_step": t_rank / args.steps * 1e3, "sm_mhz": clk.get("sm_mhz"),
        "power_w_max": clk.get("power_w_max"), "reasons": clk.get("reasons")})

    # ---- fixed global batch (BASELINE batch-64 config with the clips sharded
    # across the GPUs): each rank encodes its contiguous slice of the same
    # global batch (wxb200.dist.shard), so per-GPU work shrinks as N grows
    gb = args.global_batch
    lo, hi = wdist.shard(gb, world, rank)
    nloc = hi - lo
    t_fixed_rank = 0.0
    if nloc > 0:
        mel_s, out_s = mel[:nloc], out[:nloc]
        for _ in range(args.warmup):
            enc.forward(mel_s, out=out_s)
        torch.cuda.synchronize()
    barrier()
    if nloc > 0:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(st)
        for _ in range(args.steps):
            enc.forward(mel_s, out=out_s)
        f1.record(st)
        torch.cuda.synchronize()
        t_fixed_rank = f0.elapsed_time(f1) / 1e3
    barrier()
    t_fixed = max_over_ranks(t_fixed_rank)
    fixed_per_rank = wdist.gather_to_all({"rank": rank, "clips": nloc,
                                          "ms_per_step": t_fixed_rank / args.steps * 1e3})

    # the ctx-512 variant of the same configuration: each clip's mel cut to its
    # first 1024 frames (bench/run_raw_encoder.py:63-65), the same clips
    mel512 = mel[:, :, :1024].contiguous()
    out512 = torch.empty(B, 512, D, device="cuda")
    for _ in range(args.warmup):
        enc.forward(mel512, out=out512)
    torch.cuda.synchronize()
    barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(st)
    for _ in range(args.steps):
        enc.forward(mel512, out=out512)
    c1.record(st)
    torch.cuda.synchronize()
    barrier()
    t_512 = max_over_ranks(c0.elapsed_time(c1) / 1e3)
    del mel512, out512

    # ---- end to end through the public API, host buffers in and out. Every
    # step copies its mel in from pinned host memory and its features out to
    # pinned host memory. Pipelined (submit_host / wait_host): two input/output
    # pairs alternate, and one step's copies overlap the next step's compute.
    mel_np, out_np = mel_host.numpy(), out_host.numpy()
    mel_host2 = torch.empty(B, N_MELS, 2 * CTX, pin_memory=True)
    mel_host2.copy_(torch.rand(B, N_MELS, 2 * CTX, generator=g) * 2.0 - 0.8)
    out_host2 = torch.empty(B, CTX, D, pin_memory=True)
    mels, outs = (mel_np, mel_host2.numpy()), (out_np, out_host2.numpy())
    for i in range(args.warmup):
        enc.submit_host(mels[i % 2], outs[i % 2])
    enc.wait_host()
    barrier()
    w0 = time.perf_counter()
    for i in range(args.steps):
        enc.submit_host(mels[i % 2], outs[i % 2])
    enc.wait_host()
    t_e2e = max_over_ranks(time.perf_counter() - w0)
    barrier()
    # the same with the synchronous call (each step returns with its features)
    for _ in range(args.warmup):
        enc.forward_host(mel_np, out=out_np)
    barrier()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        enc.forward_host(mel_np, out=out_np)
    t_e2e_sync = max_over_ranks(time.perf_counter() - w0)
    barrier()
    del mel_host2, out_host2, mels, outs

    # one clip at a time, as the reference's server encodes a window (its
    # published 3344 ms per large-v3 pass is this batch-1 latency)
    lat = None
    if rank == 0:
        # 30 untimed forwards first: right after the 64-clip loop the SM clock
        # is still at the power cap's level, and a server encoding one window
        # after another runs at its steady state
        one_d, one_o = mel[:1], out[:1]
        for _ in range(30):
            enc.forward(one_d, out=one_o)
        torch.cuda.synchronize()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(st)
        for _ in range(100):
            enc.forward(one_d, out=one_o)
        l1.record(st)
        torch.cuda.synchronize()
        one_h, one_oh = mel_np[:1], out_np[:1]
        for _ in range(5):
            enc.forward_host(one_h, out=one_oh)
        w1 = time.perf_counter()
        for _ in range(20):
            enc.forward_host(one_h, out=one_oh)
        lat = {"device_ms": l0.elapsed_time(l1) / 100,
               "e2e_ms": (time.perf_counter() - w1) / 20 * 1e3,
               "note": "one clip per forward, ctx 1500, after 30 untimed forwards; device: "
                       "100 forwards back to back; e2e: 20 synchronous host calls; the "
                       "reference publishes 3344 ms for this on its NPU"}

    total_clips = B * world * args.steps
    value = total_clips / t_dev
    e2e = total_clips / t_e2e
    peaks = load_peaks()
    if lat is not None:
        # the whole one-clip forward against the dense bf16 peak
        lat["tflops"] = FLOP_PER_CLIP / (lat["device_ms"] * 1e-3) / 1e12
        lat["frac_of_bf16_peak"] = lat["tflops"] / peaks["bf16_tflops"]
    roof, cpu = None, None
    kernels, row_ops = {}, {}
    if rank == 0:
        kernels, row_ops = kernel_rooflines(B, peaks)
        # the dominant kernel of the launch list (profiles/launches_encoder_b64.md)
        k = kernels["attention"]
        roof = {"bound": "tensor", "kernel": "attention_kernel (fused QK^T-softmax-PV, 20 heads)",
                "achieved": k["tflops"], "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": k["tflops"] / peaks["bf16_tflops"], "peak_source": peaks["src"],
                "flop_per_launch": 4.0 * B * CTX * CTX * D,
                "traffic": ATTN_DRAM_BYTES_PER_CLIP * B,
                "traffic_note": "dram read+write per launch, from one ncu capture at 64 clips "
                                "(profiles/attention_ncu_b64.md), per clip x B",
                "whole_step": {"achieved": FLOP_PER_CLIP * B / (t_dev / args.steps) / 1e12,
                               "frac": FLOP_PER_CLIP * B / (t_dev / args.steps) / 1e12
                               / peaks["bf16_tflops"]}}
        if want_cpu:
            v, spent, desc = cpu_clips(W, min_seconds=10.0, max_clips=3)
            del W
            cpu = {"value": v, "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                   "sample": desc + f"; {spent:.1f} s of CPU time, the oracle port of the "
                                    "reference's numpy encoder, all BLAS threads"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_dev / args.steps * 1e3,
            "ms_per_clip_per_gpu": t_dev / args.steps * 1e3 / B,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if quant is None else "int8 GEMMs (s32 accumulation), bf16 attention",
            "data": "synthetic (random N(0,0.02) large-v3 weights, U[-0.8,1.2] log-mel per clip)",
            "config": arm_config(B, world, args.quant),
            "e2e": {"value": e2e, "unit": UNIT,
                    "h2d_bytes_per_step": int(mel_host.numel() * 4),
                    "d2h_bytes_per_step": int(out_host.numel() * 4),
                    "api": "Encoder.submit_host / wait_host (wx_encoder_submit_host): "
                           "pinned host buffers, two steps in flight",
                    "sync_value": total_clips / t_e2e_sync,
                    "sync_api": "Encoder.forward_host (wx_encoder_forward_host), one "
                                "step at a time"},
            # per step: im2col, [quantise,] GEMM for each conv; per layer LN, QKV,
            # attention, out-proj, LN, fc1, fc2 (+ the quantisation of O and of
            # fc1's output in int8 mode, where LN and quantisation are one kernel);
            # ln_post; and set_io_kernel, which points the graph at this
            # step's buffers before each replay
            "gpu_launches": ((2 + 2 + 7 * N_LAYER + 1 + 1) if quant is None
                             else (3 + 3 + 9 * N_LAYER + 1 + 1)) * args.steps,
            "roofline": roof, "kernels": kernels, "row_ops": row_ops, "clocks": clk,
            "batch1_latency": lat,
            "per_rank": per_rank,
            "fixed_global_batch": {
                "value": gb * args.steps / t_fixed, "unit": UNIT, "global_batch": gb,
                "ms_per_step": t_fixed / args.steps * 1e3, "scaling": "strong",
                "per_rank": fixed_per_rank,
                "note": "the same timed loop with one global batch split into contiguous "
                        "per-GPU slices (wxb200.dist.shard); max over ranks"},
            "ctx512": {"value": B * world * args.steps / t_512, "unit": UNIT,
                       "ms_per_clip_per_gpu": t_512 / args.steps * 1e3 / B,
                       "flop_per_clip": FLOP_PER_CLIP_512,
                       "note": "the same clips with mel cut to 1024 frames (audio_ctx 512)"},
            "cpu_baseline": cpu, "output_finite": finite,
            "flop_per_clip": FLOP_PER_CLIP,
        }
        print(json.dumps(line), flush=True)
    enc.close()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
