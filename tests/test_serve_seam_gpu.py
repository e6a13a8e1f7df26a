"""The reference server's backend calls, replayed with this package in place
of the reference's src/ on sys.path: the weight preparation of load_backend
(serve/npu_stt_server.py:185-207), the encode of each 30 s window in _window
(:331-342) at contexts of the server's ladder (:68-70), the geometry release
of ensure_geometry between contexts (:299-328) and the re-arming of
recover_if_degraded (:367-393). The audio front end and the decoder come from
openai-whisper, which is not on the encoder path (and not installed here); a
seeded mel stands in for each window.
"""
import numpy as np
import pytest

import encoder_ref as R
import npu_whisper_encoder as E
import rawxrt
from wxb200 import _lib as L
from wxb200.encoder import Encoder

pytestmark = pytest.mark.gpu


def _load_backend(n_layer=2):
    """load_backend (:185-207) with a synthetic checkpoint of the same keys."""
    W = R.make_weights("tiny", seed=1, n_layer=n_layer)
    for k in [k for k in list(W) if k.endswith(".weight") and W[k].ndim == 2
              and not k.endswith("_ln.weight")]:
        W[k[:-len("weight")] + "weight_T"] = np.ascontiguousarray(W[k].T)
    n_layer = 1 + max(int(k.split(".")[2]) for k in W if k.startswith("w.blocks."))
    d_model = W["w.ln_post.weight"].shape[0]
    n_head = d_model // 64
    extra = E.prepare_mlp_chunks(W, n_layer, d_model, 0)
    rt = rawxrt.RawRT()
    rt.register_weights([v for v in W.values() if isinstance(v, np.ndarray)] + extra)
    E.gelu = rt.gelu
    return rt, W, n_layer, n_head


def _window(rt, W, mel_full, ctx, n_layer, n_head):
    """_window's encoder call (:335-342)."""
    mel_np = np.ascontiguousarray(mel_full.astype(np.float32)[:, :2 * ctx])
    return E.encoder(W, mel_np, rt.matmul, rt.matmul, prof={}, npu_softmax=False,
                     n_layer=n_layer, n_head=n_head, attn_fn=rt.attn_chain, mlp_fn=rt.mlp,
                     fold_bias=True)


def _release(rt):
    """The geometry release of ensure_geometry (:315-322) and recover_if_degraded
    (:381-386); `while RT._live: RT._evict_lru()` must terminate."""
    rt._chains.clear()
    rt._scratch.clear()
    rt._scratch_owner.clear()
    n = 0
    while rt._live:
        rt._evict_lru()
        n += 1
        assert n < 1000
    rt._views.clear()


def test_ladder_contexts_with_geometry_switches(cuda):
    rt, W, nl, nh = _load_backend()
    mel = R.make_mel(80, 3000, seed=4)
    outs = {}
    for ctx in (512, 1500, 768, 512):          # switches, then back to the first context
        _release(rt)
        out = _window(rt, W, mel, ctx, nl, nh)
        assert out.shape == (ctx, 384) and out.dtype == np.float32
        ref = R.encoder_np(W, mel[:, :2 * ctx], nl, nh)
        assert R.cosine(out, ref) >= 0.9999
        outs.setdefault(ctx, []).append(out)
    assert np.array_equal(outs[512][0], outs[512][1])   # the same answer after the switches
    assert rt.chain_ok and rt.fused_ok and rt.mlp_ok and rt.softmax_ok and not rt.fallbacks
    assert L.device_error() == 0


def test_recover_if_degraded_rearms(cuda):
    rt, W, nl, nh = _load_backend()
    rt.chain_ok = False
    rt.fallbacks.append("attn_chain: injected")      # what a failed pass would leave
    if not (rt.chain_ok and rt.mlp_ok and rt.softmax_ok):   # recover_if_degraded, RECOVER on
        _release(rt)
        rt.chain_ok = rt.fused_ok = rt.mlp_ok = rt.softmax_ok = True
    mel = R.make_mel(80, 3000, seed=5)
    out = _window(rt, W, mel, 1024, nl, nh)
    assert R.cosine(out, R.encoder_np(W, mel[:, :2048], nl, nh)) >= 0.9999


def test_long_recording_windows_in_one_batch(cuda):
    """transcribe's 30 s windows (:400-425) encoded one by one equal the same
    windows encoded as one batch (Encoder.forward_host)."""
    rt, W, nl, nh = _load_backend()
    mels = np.stack([R.make_mel(80, 3000, seed=10 + i) for i in range(3)])
    single = [_window(rt, W, m, 1500, nl, nh) for m in mels]
    enc = Encoder(W, n_layer=nl, n_head=nh, max_batch=3)
    try:
        batch = enc.forward_host(mels)
    finally:
        enc.close()
    for i in range(3):
        assert R.cosine(batch[i], single[i]) >= 0.99999
    assert L.device_error() == 0
