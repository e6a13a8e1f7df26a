"""The int8 oracle (oracle/quant_ref.py) pinned to the reference's own int8
code: fixtures made by executing bench/probe_int8_decode.py:48-74
(q_matmul_factory) and the reference encoder as the probe calls it
(tests/golden/make_quant_golden.py). CPU only."""
from pathlib import Path

import numpy as np
import pytest

import encoder_ref as R
import quant_ref as Q

GOLD = Path(__file__).resolve().parent / "golden"


def gemm_inputs(M, K, N, seed):
    # the generator's recipe (tests/golden/make_quant_golden.py:gemm_inputs)
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((M, K)) * rng.uniform(0.2, 3.0, (M, 1))).astype(np.float32)
    B = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    A[M // 3] = 0.0
    B[:, N // 2] = 0.0
    return A, B, bias


def enc_case(name):
    z = np.load(GOLD / f"quant_enc_{name}.npz")
    geom = str(z["geometry"])
    nl, ctx = int(z["n_layer"]), int(z["ctx"])
    n_mels, d, nh, _, _ = R.GEOMETRY[geom]
    W = R.make_weights(geom, seed=int(z["weight_seed"]), n_layer=nl)
    mel = R.make_mel(n_mels, 2 * ctx, seed=int(z["mel_seed"]))
    return W, mel, nl, nh, str(z["mode"]), z["out"]


@pytest.mark.parametrize("mode", ["perchan", "pertensor", "fp32"])
def test_q_matmul_equals_reference(mode):
    z = np.load(GOLD / "quant_gemm.npz")
    for i, (M, K, N) in enumerate(z["shapes"]):
        A, B, bias = gemm_inputs(int(M), int(K), int(N), seed=100 + i)
        ref = z[f"s{i}_{mode}"]
        out = Q.q_matmul(A, B, bias, mode=mode)
        assert out.dtype == np.float32 and np.array_equal(out, ref), (i, mode)


@pytest.mark.parametrize("name", ["tiny_l2_ctx64_perchan", "tiny_l2_ctx64_pertensor",
                                  "large_l1_ctx32_perchan", "large_l1_ctx32_pertensor"])
def test_int8_encoder_equals_reference(name):
    W, mel, nl, nh, mode, ref = enc_case(name)
    out = Q.encoder_int8_np(W, mel, nl, nh, mode=mode)
    assert out.shape == ref.shape
    assert R.cosine(out, ref) > 1 - 1e-9, R.cosine(out, ref)
    assert np.allclose(out, ref, rtol=1e-5, atol=1e-5)


def test_quantize_rows_edges():
    x = np.array([[0, 0, 0, 0],                  # zero row: scale 1, q 0
                  [1.27, -0.635, 0.005, 0.015],  # 0.635 / 0.01 = 63.5 -> 64 (half to even)
                  [-3, 1, 2, 3]], np.float32)
    q, s = Q.quantize_rows(x)
    assert s.dtype == np.float32 and s[0] == 1.0
    assert np.array_equal(q[0], [0, 0, 0, 0])
    assert q[1, 0] == 127 and q[2, 0] == -127 and q[2, 3] == 127
    assert np.array_equal(q[1], np.rint(x[1] / s[1]).astype(np.int8))
    assert np.abs(q.astype(np.int32)).max() == 127


def test_weight_scales_and_chunks():
    B = np.array([[1.0, 0.0, -2.54], [0.5, 0.0, 1.0]], np.float32)
    assert np.array_equal(Q.weight_scales(B, "perchan"),
                          np.array([[1.0 / np.float32(127), 1.0, 2.54 / np.float32(127)]],
                                   np.float32))
    assert np.all(Q.weight_scales(B, "pertensor") == np.float32(2.54) / np.float32(127))
    assert Q.mlp_chunk_width(5120, 1280) == 1280    # large-v3: 4 chunks
    assert Q.mlp_chunk_width(1536, 384) == 1536     # tiny: one
    assert Q.mlp_chunk_width(6000, 1280) == 3000


def test_fp32_control_is_plain_matmul():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((5, 7)).astype(np.float32)
    B = rng.standard_normal((7, 3)).astype(np.float32)
    assert np.array_equal(Q.q_matmul(A, B, mode="fp32"), A @ B)
