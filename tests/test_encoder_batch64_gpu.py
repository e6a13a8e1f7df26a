"""large-v3 at the benchmarked configuration: 64 clips per forward, ctx 1500
and ctx 512 (mel cut to 1024 frames), the shapes bench.py times.

At 64 clips every GEMM runs M = 96,000 rows through the 2-SM tile scheduler
and attention runs 64 x 20 (clip, head) items; at one clip the GEMMs take the
one-SM kernel. Each clip's features must not depend on the batch it is
encoded in, so every clip of a 64-clip forward is checked bit for bit against
its own one-clip forward, through the device entry point and through the
pipelined host entry point (submit_host / wait_host). Clips 0 and 63 are also
checked against the torch fp32 CPU encoder.

The int8 mode is checked the same way at 64 clips (its CTA-pair int8 GEMMs
against the one-SM kernels of a one-clip forward).

The reference's own gate does the same at its production configuration:
cosine against torch, then equality to a golden output
(tests/test_encoder_golden.py:99-116 of the reference).

Cosine bars sit near the values measured on a B200 (printed as MEASURED
lines), with about twice the measured distance from 1 as margin.
"""
import numpy as np
import pytest
import torch

import encoder_ref as R
from wxb200 import _lib as L
from wxb200.encoder import Encoder

pytestmark = pytest.mark.gpu

B = 64
# measured on a B200 with 2 layers: 1 - cos = 4.1e-6 at ctx 1500 and at ctx
# 512, clips 0 and 63 (printed below)
COS_2L = 0.999991
# measured on a B200 at 32 layers, clip 0: 1 - cos = 9.9e-6
COS_32L = 0.99998


def clip_mels(frames, first_seed=1000):
    """Clip i of the batch is seeded with first_seed + i, as bench.py seeds per clip."""
    return np.stack([R.make_mel(128, frames, seed=first_seed + i) for i in range(B)])


@pytest.fixture(scope="module")
def enc2(cuda):
    W = R.make_weights("large-v3", seed=1, n_layer=2)
    enc = Encoder(W, n_layer=2, n_head=20, max_batch=B)
    yield W, enc
    enc.close()


def check_batch_equals_single(enc, mel_dev, out):
    for i in range(B):
        one = enc.forward(mel_dev[i:i + 1])
        torch.cuda.synchronize()
        assert torch.equal(one[0], out[i]), f"clip {i} differs from its one-clip forward"


@pytest.mark.parametrize("frames", [3000, 1024])
def test_batch64_every_clip_equals_its_single_clip_forward(enc2, frames):
    W, enc = enc2
    mels = clip_mels(frames)
    mel_dev = torch.from_numpy(mels).cuda()
    out = enc.forward(mel_dev)
    torch.cuda.synchronize()
    assert out.shape == (B, frames // 2, 1280)
    assert bool(torch.isfinite(out).all())
    check_batch_equals_single(enc, mel_dev, out)
    for i in (0, B - 1):
        ref = R.encoder_torch(W, mels[i], 2, 20)
        cos = R.cosine(out[i].cpu().numpy(), ref)
        print(f"MEASURED large-v3 2 layers frames {frames} clip {i}: cos {cos:.8f}, "
              f"rel L2 {R.rel_l2(out[i].cpu().numpy(), ref):.3e}")
        assert cos >= COS_2L, (i, cos)
    assert L.device_error() == 0


@pytest.mark.parametrize("frames", [3000, 1024])
def test_batch64_pipelined_host_entry_matches_device_forward(enc2, frames):
    """submit_host / wait_host with two pinned input/output pairs in flight,
    as bench.py's e2e leg runs them: each batch equals the device forward."""
    W, enc = enc2
    mels = [clip_mels(frames, first_seed=s) for s in (2000, 3000, 4000)]
    pinned = [torch.from_numpy(m).pin_memory() for m in mels]
    outs = [torch.full((B, frames // 2, 1280), float("nan")).pin_memory() for _ in range(3)]
    for k in range(3):                  # the third waits for the first's staging slot
        enc.submit_host(pinned[k].numpy(), outs[k].numpy())
    enc.wait_host()
    for k in range(3):
        ref = enc.forward(torch.from_numpy(mels[k]).cuda())
        torch.cuda.synchronize()
        assert np.array_equal(outs[k].numpy(), ref.cpu().numpy()), k
    assert L.device_error() == 0


@pytest.mark.slow
def test_large_v3_32_layers_batch64(cuda):
    """BASELINE configs 4 and 5 at full depth: 32 layers, 64 clips, ctx 1500.
    Every clip equals its one-clip forward bit for bit; clip 0 (the mel of the
    one-clip cosine case) against the torch fp32 encoder (CPU, about a minute)."""
    W = R.make_weights("large-v3", seed=1)
    mels = clip_mels(3000)
    mels[0] = R.make_mel(128, 3000, seed=0)
    enc = Encoder(W, max_batch=B, gelu="poly4")
    try:
        mel_dev = torch.from_numpy(mels).cuda()
        out = enc.forward(mel_dev)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(out).all())
        check_batch_equals_single(enc, mel_dev, out)
        got0 = out[0].cpu().numpy()
    finally:
        enc.close()
    ref = R.encoder_torch(W, mels[0], 32, 20)
    cos = R.cosine(got0, ref)
    print(f"MEASURED large-v3 32 layers clip 0: cos {cos:.8f}, rel L2 {R.rel_l2(got0, ref):.3e}")
    assert cos >= COS_32L, cos
    assert L.device_error() == 0


def test_int8_batch64_every_clip_equals_its_single_clip_forward(cuda):
    """The int8 mode at the same shape (bench.py --quant int8-perchan): CTA-pair
    int8 GEMMs with the 16-warp GELU epilogue, the fc1 row maxima folded by
    atomics and the residual added in place, against the one-SM kernels of a
    one-clip forward; every clip bit for bit."""
    W = R.make_weights("large-v3", seed=1, n_layer=2)
    enc = Encoder(W, n_layer=2, n_head=20, max_batch=B, quant="int8-perchan")
    try:
        mel_dev = torch.from_numpy(clip_mels(3000, first_seed=3000)).cuda()
        out = enc.forward(mel_dev)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(out).all())
        check_batch_equals_single(enc, mel_dev, out)
        assert L.device_error() == 0
    finally:
        enc.close()
