"""Host-side pieces of bench.py's contract, on CPU: the workload description,
the options, the synthetic weights' layout and the algorithmic FLOP count the
throughput figures are based on."""
import sys

import numpy as np
import pytest

import bench
import encoder_ref as R


def test_flop_per_clip_matches_the_work_table():
    # large-v3, ctx 1500: 32 x 70.50 GFLOP layers + 17.69 GFLOP conv = 2.2738 TFLOP
    assert bench.FLOP_PER_CLIP == pytest.approx(2.2738e12, rel=1e-4)
    # ctx 512 (mel cut to 1024 frames): 0.6932 TFLOP
    assert bench.FLOP_PER_CLIP_512 == pytest.approx(0.6932e12, rel=1e-4)


def test_arm_config_names_the_workload():
    c = bench.arm_config(64, 8)
    assert c["global_batch"] == 512 and c["seq_len"] == 1500
    assert "large-v3" in c["model"] and "dp8" in c["parallelism"]
    assert "quant" not in c
    q = bench.arm_config(64, 1, "int8-perchan")
    assert "int8-perchan" in q["quant"]


def test_options(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py", "--quant", "int8-pertensor", "--steps", "4"])
    a = bench.parse()
    assert a.quant == "int8-pertensor" and a.steps == 4 and a.gpus == 1 and a.impl == "b200"
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.quant == "none" and a.warmup >= 3


def test_synthetic_weights_have_the_reference_layout():
    W = bench.make_weights_fast(seed=1)
    ref = R.make_weights("large-v3", seed=1, n_layer=1)
    for k, v in ref.items():
        if k.startswith("w.blocks.") and not k.startswith("w.blocks.0."):
            continue
        assert k in W and W[k].shape == v.shape and W[k].dtype == np.float32, k
    assert sum(k.startswith("w.blocks.31.") for k in W) > 0
    w = W["w.blocks.0.mlp.0.weight"]
    assert abs(float(w.std()) - 0.02) < 1e-3                          # N(0, 0.02)
    assert np.array_equal(w, w.astype(np.float32).view(np.uint32).__and__(0xFFFF0000).view(np.float32))


def test_kernel_bench_attention_work_follows_ctx():
    """kernel_bench's attention FLOP and byte counts at any frame count (its
    --ctx option; the persistent kernel runs T <= 1344): 4 B T^2 d FLOP, and
    Q, K, V read and O written once, 2 bytes each."""
    from wxb200 import kernel_bench as KB
    for ctx in (1500, 512):
        _, flop, byt = KB.setup("attention", 2, dev="cpu", ctx=ctx)
        assert flop == 4.0 * 2 * ctx * ctx * 1280
        assert byt == 4.0 * 2 * ctx * 1280 * 2
