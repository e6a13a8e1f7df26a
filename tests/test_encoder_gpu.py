"""The whole encoder on the GPU against the CPU oracle.

Tolerances (north star): cosine >= 0.9999 against the torch fp32 encoder at
whisper-tiny depth, >= 0.99 at 32-layer large-v3 depth (that case, at the
benchmarked batch of 64 clips, is in test_encoder_batch64_gpu.py, with a bar
near the measured value). The golden fixtures
are outputs of the reference's own numpy path (tests/golden/make_golden.py),
so the first test compares against the reference itself.
"""
import numpy as np
import pytest
import torch

import encoder_ref as R
from wxb200 import _lib as L
from wxb200.encoder import Encoder, encoder
from wxb200.runtime import B200RT

from test_oracle import golden_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["tiny_l4_ctx128", "tiny_l2_ctx32_lnrand", "large_l1_ctx64"])
@pytest.mark.parametrize("gelu", ["poly4", "erf"])
def test_encoder_matches_reference_golden(cuda, name, gelu):
    W, mel, nl, nh, ref = golden_case(name)
    enc = Encoder(W, n_layer=nl, n_head=nh, gelu=gelu)
    out = enc.forward_host(mel)
    assert out.shape == ref.shape
    assert R.cosine(out, ref) >= 0.9999, R.cosine(out, ref)


@pytest.mark.parametrize("gelu", ["poly4", "erf"])
def test_tiny_full_context_cosine(cuda, gelu):
    """whisper-tiny, 4 layers, ctx 1500."""
    W = R.make_weights("tiny", seed=1)
    mel = R.make_mel(80, 3000, seed=0)
    ref = R.encoder_torch(W, mel, 4, 6)
    out = Encoder(W, gelu=gelu).forward_host(mel)
    assert R.cosine(out, ref) >= 0.9999


def test_batch_equals_single_clips_and_graph_replay(cuda):
    """Clips in a batch are independent: batched output == per-clip output,
    and graph replay == eager launches, bit for bit."""
    W = R.make_weights("tiny", seed=2)
    mels = np.stack([R.make_mel(80, 3000, seed=s) for s in range(3)])
    enc = Encoder(W, max_batch=3)
    batched = enc.forward_host(mels, use_graph=True)
    again = enc.forward_host(mels, use_graph=True)
    eager = enc.forward_host(mels, use_graph=False)
    assert np.array_equal(batched, again) and np.array_equal(batched, eager)
    for i in range(3):
        assert np.array_equal(enc.forward_host(mels[i]), batched[i])


def test_reduced_audio_ctx(cuda):
    """audio_ctx 512: mel cut to 1024 frames (bench/run_raw_encoder.py:63-65)."""
    W = R.make_weights("tiny", seed=3)
    mel = R.make_mel(80, 1024, seed=4)
    out = Encoder(W).forward_host(mel)
    ref = R.encoder_torch(W, mel, 4, 6)
    assert out.shape == (512, 384)
    assert R.cosine(out, ref) >= 0.9999


def test_graph_replays_follow_the_buffers(cuda):
    """One captured graph per (batch, frames) serves any input and output
    buffers: interleaved forwards with different buffers each read their own
    mel and write their own output, equal to eager launches."""
    W = R.make_weights("tiny", seed=6, n_layer=2)
    enc = Encoder(W, n_layer=2, n_head=6, max_batch=2)
    try:
        mels = [torch.from_numpy(np.stack([R.make_mel(80, 300, seed=50 + 2 * i + j)
                                           for j in range(2)])).cuda() for i in range(3)]
        outs = [torch.full((2, 150, 384), float("nan"), device="cuda") for _ in range(4)]
        enc.forward(mels[0], out=outs[0])
        enc.forward(mels[1], out=outs[1])
        enc.forward(mels[2], out=outs[2])
        enc.forward(mels[0], out=outs[3])
        torch.cuda.synchronize()
        for i, m in ((0, 0), (1, 1), (2, 2), (3, 0)):
            ref = enc.forward(mels[m], use_graph=False)
            torch.cuda.synchronize()
            assert torch.equal(outs[i], ref), i
        assert not torch.equal(outs[0], outs[1])
    finally:
        enc.close()


def test_device_forward_matches_host_forward(cuda):
    W = R.make_weights("tiny", seed=5)
    mel = R.make_mel(80, 3000, seed=6)
    enc = Encoder(W)
    host = enc.forward_host(mel)
    dev = enc.forward(torch.from_numpy(mel).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


@pytest.mark.parametrize("batch", [31, 32, 33])
def test_pipelined_host_forward_matches_device_forward(cuda, batch):
    """forward_host runs batches of 32 or more in two halves with the copies
    overlapping compute (31 -> one chunk, 32 -> 16+16, 33 -> 17+16); every clip
    equals the one-launch device forward of the whole batch."""
    W = R.make_weights("tiny", seed=5, n_layer=2)
    mels = np.stack([R.make_mel(80, 400, seed=40 + i) for i in range(batch)])
    enc = Encoder(W, n_layer=2, max_batch=batch)
    try:
        pinned = torch.from_numpy(mels).pin_memory()
        out = torch.empty(batch, 200, 384).pin_memory()
        host = enc.forward_host(pinned.numpy(), out=out.numpy())
        dev = enc.forward(torch.from_numpy(mels).cuda())
        torch.cuda.synchronize()
        ref = dev.cpu().numpy()
        for i in range(batch):
            assert np.allclose(host[i], ref[i], rtol=1e-5, atol=1e-5), i
            assert R.cosine(host[i], ref[i]) >= 0.999999
        again = enc.forward_host(pinned.numpy(), out=out.numpy())   # graphs replayed
        assert np.array_equal(again, host)
    finally:
        enc.close()
    assert L.device_error() == 0


def test_forwards_on_different_streams_are_ordered(cuda):
    """The workspace is shared: a submitted host batch, a graph forward on one
    stream and an eager forward on another, issued without synchronising,
    each equal the same forward run alone."""
    W = R.make_weights("tiny", seed=8, n_layer=2)
    enc = Encoder(W, n_layer=2, max_batch=2)
    try:
        mels = [np.stack([R.make_mel(80, 400, seed=90 + 2 * i + j) for j in range(2)])
                for i in range(3)]
        alone = []
        for m in mels:
            alone.append(enc.forward(torch.from_numpy(m).cuda(), use_graph=False).cpu().numpy())
        dev = [torch.from_numpy(m).cuda() for m in mels[1:]]
        torch.cuda.synchronize()
        pinned = torch.from_numpy(mels[0]).pin_memory()
        out0 = torch.full((2, 200, 384), float("nan")).pin_memory()
        enc.submit_host(pinned.numpy(), out0.numpy())
        side = torch.cuda.Stream()
        g = enc.forward(dev[0])                                  # graph, current stream
        with torch.cuda.stream(side):
            e = enc.forward(dev[1], use_graph=False)             # eager, another stream
        enc.wait_host()
        torch.cuda.synchronize()
        assert np.array_equal(out0.numpy(), alone[0])
        assert np.array_equal(g.cpu().numpy(), alone[1])
        assert np.array_equal(e.cpu().numpy(), alone[2])
    finally:
        enc.close()
    assert L.device_error() == 0


def test_submitted_batches_match_device_forward(cuda):
    """submit_host / wait_host: a stream of batches of different sizes and
    frame counts, two in flight, pinned and pageable buffers, with a
    synchronous forward_host in between; each batch's features equal the
    device forward of that batch."""
    W = R.make_weights("tiny", seed=5, n_layer=2)
    enc = Encoder(W, n_layer=2, max_batch=4)
    try:
        cases = [(4, 400), (3, 400), (4, 300), (1, 400), (4, 400), (2, 200)]
        mels = [np.stack([R.make_mel(80, F, seed=70 + 10 * k + i) for i in range(B)])
                for k, (B, F) in enumerate(cases)]
        pinned = [torch.from_numpy(m).pin_memory() for m in mels]
        outs = [torch.full((B, F // 2, 384), float("nan")).pin_memory() for B, F in cases]
        pageable_out = np.full((3, 200, 384), np.nan, dtype=np.float32)
        enc.submit_host(pinned[0].numpy(), outs[0].numpy())
        enc.submit_host(mels[1], pageable_out)                 # pageable: the copies block
        enc.submit_host(pinned[2].numpy(), outs[2].numpy())    # waits for batch 0's slot
        sync = enc.forward_host(mels[3])                       # drains the queue first
        enc.submit_host(pinned[4].numpy(), outs[4].numpy())
        enc.submit_host(pinned[5].numpy(), outs[5].numpy())
        enc.wait_host()
        enc.wait_host()                                        # nothing in flight: returns
        got = [outs[0].numpy(), pageable_out, outs[2].numpy(), sync, outs[4].numpy(),
               outs[5].numpy()]
        for k, m in enumerate(mels):
            ref = enc.forward(torch.from_numpy(m).cuda())
            torch.cuda.synchronize()
            assert np.array_equal(got[k], ref.cpu().numpy()), k
        with pytest.raises(ValueError):
            enc.submit_host(mels[0], np.empty((4, 199, 384), dtype=np.float32))
        with pytest.raises(ValueError):
            enc.submit_host(np.stack([R.make_mel(80, 400, seed=1)] * 5),
                            np.empty((5, 200, 384), dtype=np.float32))   # over max_batch
    finally:
        enc.close()
    assert L.device_error() == 0


def test_dropin_encoder_signature(cuda):
    """encoder(W, mel, RT.matmul, RT.matmul, ..., attn_fn=RT.attn_chain,
    mlp_fn=RT.mlp, fold_bias=True) -- the server's call (serve/npu_stt_server.py:340-342)."""
    W = R.add_transposed(R.make_weights("tiny", seed=1, n_layer=2))
    mel = R.make_mel(80, 256, seed=0)
    rt = B200RT()
    prof = {}
    out = encoder(W, mel, rt.matmul, rt.matmul, prof=prof, npu_softmax=False, n_layer=2,
                  n_head=6, attn_fn=rt.attn_chain, mlp_fn=rt.mlp, fold_bias=True)
    ref = R.encoder_np(W, mel, 2, 6)
    assert out.shape == ref.shape and "total" in prof
    assert R.cosine(out, ref) >= 0.9999
    with pytest.raises(TypeError):
        encoder(W, mel, R.mm, R.mm, n_layer=2, n_head=6)


def test_no_device_error_recorded(cuda):
    assert L.device_error() == 0
