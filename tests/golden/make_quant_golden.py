#!/usr/bin/env python3
"""Generate the int8 fixtures by running the REFERENCE'S OWN int8 code.

Run in a container that has the reference checkout (not needed, and not
present, where the tests run):

    python tests/golden/make_quant_golden.py /path/to/whisper-xdna

The reference's int8 matmul lives in bench/probe_int8_decode.py, a script
that imports openai-whisper (absent here) at the top and then needs recordings.
This script therefore parses that file and executes only its
q_matmul_factory definition (:48-74), unchanged, with numpy and the STAT
counter it uses; it imports src/npu_whisper_encoder.py unchanged and calls the
encoder the way the probe does (:140-142), after E.prepare_mlp_chunks (:99).

Stored: the seeds of the inputs and the reference's outputs.
  quant_gemm.npz     q_matmul(A, B, bias) in modes perchan / pertensor / fp32
                     on seeded A, B (with a zero row in A and a zero column in B)
  quant_enc_*.npz    the encoder's output with q_matmul_factory(mode) as mm
"""
import ast
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))

import encoder_ref as R  # noqa: E402

GEMM_SHAPES = [(64, 256, 96), (37, 200, 136)]   # (M, K, N)
# name: (geometry, n_layer, ctx, weight seed, mel seed, mode)
ENC_CASES = {
    "tiny_l2_ctx64_perchan": ("tiny", 2, 64, 1, 0, "perchan"),
    "tiny_l2_ctx64_pertensor": ("tiny", 2, 64, 1, 0, "pertensor"),
    "large_l1_ctx32_perchan": ("large-v3", 1, 32, 2, 1, "perchan"),
    "large_l1_ctx32_pertensor": ("large-v3", 1, 32, 2, 1, "pertensor"),
}


def gemm_inputs(M, K, N, seed):
    """Seeded operands of the GEMM fixtures (tests regenerate them)."""
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((M, K)) * rng.uniform(0.2, 3.0, (M, 1))).astype(np.float32)
    B = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    A[M // 3] = 0.0      # a zero activation row: scale 1
    B[:, N // 2] = 0.0   # a zero weight column: scale 1
    return A, B, bias


def load_q_matmul_factory(ref_root):
    path = Path(ref_root) / "bench" / "probe_int8_decode.py"
    tree = ast.parse(path.read_text())
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "q_matmul_factory"]
    assert len(fn) == 1, "q_matmul_factory not found"
    ns = {"np": np, "STAT": {"n": 0}}
    exec(compile(ast.Module(body=fn, type_ignores=[]), str(path), "exec"), ns)
    return ns["q_matmul_factory"]


def main(ref_root):
    factory = load_q_matmul_factory(ref_root)
    out = {}
    for i, (M, K, N) in enumerate(GEMM_SHAPES):
        A, B, bias = gemm_inputs(M, K, N, seed=100 + i)
        for mode in ("perchan", "pertensor", "fp32"):
            out[f"s{i}_{mode}"] = factory(mode)(A, B, bias=bias)
    np.savez_compressed(HERE / "quant_gemm.npz", shapes=np.array(GEMM_SHAPES), **out)
    print("quant_gemm", sorted(out))

    sys.path.insert(0, str(Path(ref_root) / "src"))
    import npu_whisper_encoder as E   # the reference, unchanged

    for name, (geom, nl, ctx, wseed, mseed, mode) in ENC_CASES.items():
        n_mels, d, nh, _, _ = R.GEOMETRY[geom]
        W = R.add_transposed(R.make_weights(geom, seed=wseed, n_layer=nl))
        E.prepare_mlp_chunks(W, nl, d, 0)
        mel = R.make_mel(n_mels, 2 * ctx, seed=mseed)
        y = E.encoder(W, mel, factory(mode), E.np_matmul, n_layer=nl, n_head=nh,
                      fold_bias=False)
        np.savez_compressed(HERE / f"quant_enc_{name}.npz", out=y.astype(np.float32),
                            geometry=np.array(geom), n_layer=nl, ctx=ctx,
                            weight_seed=wseed, mel_seed=mseed, mode=np.array(mode))
        print(name, y.shape, float(np.abs(y).mean()))


if __name__ == "__main__":
    # the reference checkout: first argument, else $WX_REFERENCE_DIR, else a
    # checkout named "reference" beside this repository
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "WX_REFERENCE_DIR", str(REPO.parent / "reference")))
