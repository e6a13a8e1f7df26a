"""Pin the CPU oracle (oracle/) before trusting it (no GPU).

1. The numpy encoder restatement reproduces outputs of the reference's own
   numpy path (tests/golden/encoder_np_*.npz, made by tests/golden/make_golden.py
   from src/npu_whisper_encoder.py:encoder with np_matmul).
2. The torch fp32 restatement agrees with it to fp32 round-off.
3. The row-op restatements are bit-exact to the reference's own AIE kernel
   sources compiled for the CPU (oracle/Makefile -> oracle/_ref/), on every
   bf16 input for GELU and on seeded rows for softmax and LayerNorm.
4. The reference's own known-answer checks (tests/test_rowops.py:35-76):
   softmax rel L2 < 0.02 and finite at 10240x512 and 9216x1536 with N(0,6)
   logits, the +200 overflow case, LayerNorm rel L2 < 0.02.
"""
from pathlib import Path

import numpy as np
import pytest

import encoder_ref as R
import rowops_ref as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden_case(name):
    z = np.load(GOLDEN / f"encoder_np_{name}.npz")
    geom = str(z["geometry"])
    nl, ctx = int(z["n_layer"]), int(z["ctx"])
    n_mels, d, nh, _, _ = R.GEOMETRY[geom]
    W = R.make_weights(geom, seed=int(z["weight_seed"]), n_layer=nl,
                       ln_random=bool(z["ln_random"]))
    mel = R.make_mel(n_mels, 2 * ctx, seed=int(z["mel_seed"]))
    return W, mel, nl, nh, z["out"]


CASES = ["tiny_l4_ctx128", "tiny_l2_ctx32_lnrand", "large_l1_ctx64"]


@pytest.mark.parametrize("name", CASES)
def test_numpy_restatement_matches_reference_outputs(name):
    W, mel, nl, nh, ref = golden_case(name)
    out = R.encoder_np(W, mel, nl, nh)
    assert out.shape == ref.shape
    assert np.abs(out - ref).max() < 1e-4
    assert R.cosine(out, ref) > 1 - 1e-9


@pytest.mark.parametrize("name", CASES)
def test_torch_restatement_matches_reference_outputs(name):
    W, mel, nl, nh, ref = golden_case(name)
    out = R.encoder_torch(W, mel, nl, nh)
    assert R.rel_l2(out, ref) < 1e-5


def test_sinusoids_known_values():
    p = R.sinusoids(1500, 384)
    assert p.shape == (1500, 384)
    assert np.allclose(p[0, :192], 0.0) and np.allclose(p[0, 192:], 1.0)
    assert abs(p[1, 0] - np.sin(1.0)) < 1e-6


# ------------------------------------------------------------------ row ops

def all_bf16():
    return O.bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)).reshape(256, 256)


def test_gelu_poly4_tracks_erf_gelu():
    """The fitted bump approximates the exact erf-GELU (the function the
    coefficients of kernels/gelu_poly4_coeffs.h were fitted to)."""
    x = O.rbf(np.linspace(-8, 8, 4097).astype(np.float32), O.RNE)
    err = np.abs(O.gelu_row4_rne(x) - O.gelu_erf_exact(x))
    assert err.max() < 0.02
    assert err.mean() < 2e-3
    big = O.rbf(np.array([5.0, 100.0, 3e38, -5.0, -100.0, -3e38], np.float32), O.RNE)
    assert np.array_equal(O.gelu_row4_rne(big), np.array([5, 100, big[2], 0, 0, 0], np.float32))


def test_bf16_rounding_helpers():
    import ml_dtypes
    rng = np.random.default_rng(0)
    x = rng.normal(0, 10, 100000).astype(np.float32)
    ref = x.astype(ml_dtypes.bfloat16).astype(np.float32)
    assert np.array_equal(O.rbf(x, O.RNE), ref)
    t = O.rbf(x, O.TRUNC)
    assert np.all(np.abs(t) <= np.abs(x))


def test_lane_sum_order():
    a = np.arange(40, dtype=np.float32)[None, :]
    assert O.lane_sum16(a)[0] == a.sum()


ref_kernels = pytest.importorskip("ref_kernels")
needs_ref = pytest.mark.skipif(not ref_kernels.available(),
                               reason="oracle/_ref not built (make -C oracle)")


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


@needs_ref
@pytest.mark.parametrize("op,fn", [("g4", O.gelu_row4), ("g4r", O.gelu_row4_rne)])
def test_gelu_oracle_bit_exact_to_reference_source_every_bf16(op, fn):
    x = all_bf16()
    finite = np.isfinite(x)
    a, b = ref_kernels.run_rows(op, x), fn(x)
    assert same_bits(np.where(finite, a, 0), np.where(finite, b, 0))


@needs_ref
def test_gelu_f32_oracle_bit_exact_to_reference_source():
    rng = np.random.default_rng(1)
    x = (rng.normal(-2, 3, (64, 1024)) * rng.choice([1, 1e-3, 1e3], (64, 1024))).astype(np.float32)
    assert same_bits(ref_kernels.run_rows("g4f", x), O.gelu_row4f(x))


@needs_ref
@pytest.mark.parametrize("op,variant,mode", [("s1", 1, O.TRUNC), ("s2", 4, O.TRUNC),
                                             ("s3", 3, O.TRUNC), ("s4", 4, O.TRUNC),
                                             ("s4r", 4, O.RNE)])
@pytest.mark.parametrize("valid", [0, 1504])
def test_softmax_oracle_bit_exact_to_reference_source(op, variant, mode, valid):
    """softmax_row2.cc (s2) is checked against the v4 restatement: the two
    kernels compute the same arithmetic, which is why rowops.softmax_row2
    runs the v4 device kernel."""
    rng = np.random.default_rng(2)
    x = O.rbf(rng.normal(0, 6, (96, 1536)).astype(np.float32), O.RNE)
    a = ref_kernels.run_rows(op, x, valid=valid)
    b = O.softmax_row(x, mode=mode, variant=variant, valid=valid)
    assert same_bits(a, b)


@needs_ref
@pytest.mark.parametrize("cols", [384, 1280])
def test_layernorm_oracle_bit_exact_to_reference_source(cols):
    rng = np.random.default_rng(3)
    x = O.rbf(rng.normal(0.5, 2.0, (64, cols)).astype(np.float32), O.RNE)
    assert same_bits(ref_kernels.run_rows("ln", x), O.layer_norm_aie(x, O.TRUNC))


@pytest.mark.parametrize("rows,cols", [(10240, 512), (9216, 1536)])
def test_softmax_reference_known_answer(rows, cols):
    """tests/test_rowops.py:35-53 of the reference, on the oracle (v1 softmax,
    the kernel that test ran)."""
    rng = np.random.default_rng(0)
    x = O.rbf(rng.normal(0, 6.0, (rows, cols)).astype(np.float32), O.RNE)
    out = O.softmax_row(x, mode=O.TRUNC, variant=1)
    ref = O.softmax_fp32(x)
    assert np.isfinite(out).all()
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 0.02


def test_softmax_overflow_known_answer():
    rng = np.random.default_rng(0)
    x = O.rbf((rng.normal(0, 6.0, (512, 512)) + 200.0).astype(np.float32), O.RNE)
    for variant in (1, 3, 4):
        out = O.softmax_row(x, mode=O.TRUNC, variant=variant)
        ref = O.softmax_fp32(x)
        assert np.isfinite(out).all()
        assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 0.02


@pytest.mark.parametrize("rows,cols", [(512, 1280), (1536, 384)])
def test_layernorm_reference_known_answer(rows, cols):
    rng = np.random.default_rng(0)
    x = O.rbf(rng.normal(0, 1.0, (rows, cols)).astype(np.float32), O.RNE)
    out = O.layer_norm_aie(x, O.TRUNC)
    ref = (x - x.mean(1, keepdims=True)) / np.sqrt(x.var(1, keepdims=True) + 1e-5)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 0.02
