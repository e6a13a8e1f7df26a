"""MultiGPUEncoder: one host batch split by clip index over several encoder
replicas, each on its own host thread. On a one-GPU machine the replicas
share device 0 (the splitting, threading and output placement are the same);
with two or more GPUs the second test spreads over all of them.
"""
import numpy as np
import pytest
import torch

import encoder_ref as R
from wxb200 import _lib as L
from wxb200.encoder import Encoder
from wxb200.multi import MultiGPUEncoder

pytestmark = pytest.mark.gpu


def _case(batch, frames=400, seed=300):
    W = R.make_weights("tiny", seed=9, n_layer=2)
    mels = np.stack([R.make_mel(80, frames, seed=seed + i) for i in range(batch)])
    return W, mels


@pytest.mark.parametrize("batch", [7, 3, 1])
def test_replicas_on_one_device_match_one_encoder(cuda, batch):
    W, mels = _case(batch)
    ref = Encoder(W, n_layer=2, max_batch=batch)
    try:
        want = ref.forward_host(mels)
    finally:
        ref.close()
    multi = MultiGPUEncoder(W, devices=[0, 0, 0], max_batch=8, n_layer=2)
    try:
        assert multi.slices(batch)[0][0] == 0 and multi.slices(batch)[-1][1] == batch
        got = multi.forward_host(mels)
        assert np.array_equal(got, want)
        pm, po = multi.host_buffers(batch, mels.shape[2])
        pm[...] = mels
        assert multi.forward_host(pm, out=po) is po
        assert np.array_equal(po, want)
        with pytest.raises(ValueError):
            multi.forward_host(np.concatenate([mels] * 9))        # over max_batch
    finally:
        multi.close()
    assert L.device_error() == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two or more GPUs")
def test_batch_spread_over_all_gpus(cuda):
    n = torch.cuda.device_count()
    W, mels = _case(2 * n + 1)
    multi = MultiGPUEncoder(W, max_batch=2 * n + 1, n_layer=2)
    try:
        got = multi.forward_host(mels)
    finally:
        multi.close()
    ref = Encoder(W, n_layer=2, max_batch=3)
    try:
        for i in range(mels.shape[0]):
            assert np.array_equal(got[i], ref.forward_host(mels[i])), i
    finally:
        ref.close()
