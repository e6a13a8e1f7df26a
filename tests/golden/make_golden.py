#!/usr/bin/env python3
"""Generate the golden encoder fixtures by running the REFERENCE ITSELF.

Run in a container that has the reference checkout (it is not needed, and not
present, where the tests run):

    python tests/golden/make_golden.py /path/to/whisper-xdna

It imports the reference's src/npu_whisper_encoder.py unchanged and calls its
CPU path, encoder(W, mel, np_matmul, np_matmul, n_layer, n_head) (the
`--backend numpy` path of src/npu_whisper_encoder.py:575-592), on seeded
synthetic weights and mel from oracle/encoder_ref.py. Only the inputs' seeds and
the reference's outputs are stored: the tests regenerate the inputs from the
seeds, so the fixtures stay small.
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))

import encoder_ref as R  # noqa: E402

# name: (geometry, n_layer, ctx, weight seed, mel seed, ln_random)
CASES = {
    "tiny_l4_ctx128": ("tiny", 4, 128, 1, 0, False),
    "tiny_l2_ctx32_lnrand": ("tiny", 2, 32, 7, 3, True),
    "large_l1_ctx64": ("large-v3", 1, 64, 1, 0, False),
}


def main(ref_root):
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import npu_whisper_encoder as E   # the reference, unchanged

    for name, (geom, nl, ctx, wseed, mseed, lnr) in CASES.items():
        n_mels, d, nh, _, _ = R.GEOMETRY[geom]
        W = R.add_transposed(R.make_weights(geom, seed=wseed, n_layer=nl,
                                            ln_random=lnr))
        mel = R.make_mel(n_mels, 2 * ctx, seed=mseed)
        out = E.encoder(W, mel, E.np_matmul, E.np_matmul, n_layer=nl,
                        n_head=nh)
        np.savez_compressed(HERE / f"encoder_np_{name}.npz",
                            out=out.astype(np.float32),
                            geometry=np.array(geom), n_layer=nl, ctx=ctx,
                            weight_seed=wseed, mel_seed=mseed,
                            ln_random=lnr)
        print(name, out.shape, float(np.abs(out).mean()))


if __name__ == "__main__":
    # the reference checkout: first argument, else $WX_REFERENCE_DIR, else a
    # checkout named "reference" beside this repository
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "WX_REFERENCE_DIR", str(REPO.parent / "reference")))
