"""The log-mel frontend kernel (wx_log_mel) against the CPU oracle
(oracle/mel_ref.py, pinned to transformers' WhisperFeatureExtractor), and the
audio -> features -> encoder chain on the device. Tolerance: 2e-4 absolute on
the normalised features (values in [-1.5, ~2]; fp32 DFT against float64)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import encoder_ref as R
import mel_ref as M
from wxb200 import _lib as L
from wxb200 import audio as A
from wxb200 import ops
from wxb200.encoder import Encoder

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("mel_*.npz")), ids=lambda p: p.stem)
def test_log_mel_matches_oracle_and_fixture(cuda, path):
    z = np.load(path)
    n_mels = int(z["n_mels"])
    audio = M.synthetic_audio(float(z["seconds"]), int(z["seed"]), str(z["kind"]))
    got = ops.log_mel(torch.from_numpy(audio).cuda(), n_mels=n_mels).cpu().numpy()
    ref = M.log_mel_spectrogram(audio, n_mels)
    assert got.shape == (n_mels, 3000)
    assert np.abs(got - ref).max() < 2e-4
    assert np.abs(got[:, ::8] - z["frames_every8"]).max() < 3e-4


def test_batch_of_ragged_clips_with_row_stride(cuda):
    """Clips of different lengths in one launch: each row holds n_samples
    valid samples at a row stride larger than that; past the recording the
    window is zero (pad_or_trim), and a row longer than 30 s is trimmed."""
    lens = [16000, 123457, 480000, 500000]
    rows = np.zeros((4, 520000), np.float32)
    clips = []
    for i, n in enumerate(lens):
        x = M.synthetic_audio(n / 16000, 30 + i)[:n]
        clips.append(x)
        rows[i, :n] = x
    dev = torch.from_numpy(rows).cuda()
    for i, n in enumerate(lens):      # one clip at a time: only n_samples of the row count
        out = torch.empty(1, 128, 3000, device="cuda")
        L.check(L.lib().wx_log_mel(dev[i].data_ptr(), 1, n, n, 128, out.data_ptr(), None))
        ref = M.log_mel_spectrogram(clips[i], 128)
        assert np.abs(out[0].cpu().numpy() - ref).max() < 2e-4
    batch = ops.log_mel(dev, n_mels=128).cpu().numpy()    # all 520000 samples, trimmed
    for i in range(4):
        ref = M.log_mel_spectrogram(rows[i], 128)
        assert np.abs(batch[i] - ref).max() < 2e-4
    assert L.device_error() == 0


def test_silence_and_whisper_shaped_api(cuda):
    out = A.log_mel_spectrogram(np.zeros(8000, np.float32), n_mels=80)
    assert out.device.type == "cpu" and out.shape == (80, 3000)
    assert torch.all(out == -1.5)
    x = torch.from_numpy(M.synthetic_audio(2.0, 5)).cuda()
    got = A.log_mel_spectrogram(A.pad_or_trim(x), n_mels=80)
    assert got.is_cuda
    assert np.abs(got.cpu().numpy() - M.log_mel_spectrogram(x.cpu().numpy(), 80)).max() < 2e-4


def test_audio_to_encoder_on_device(cuda):
    """audio -> wx_log_mel -> encoder without leaving the GPU equals the
    encoder run on the oracle's features."""
    W = R.make_weights("tiny", seed=7, n_layer=2)
    clips = np.stack([M.pad_or_trim(M.synthetic_audio(s, 40 + i)) for i, s in enumerate((3, 9))])
    enc = Encoder(W, n_layer=2, max_batch=2)
    try:
        feats = ops.log_mel(torch.from_numpy(clips).cuda(), n_mels=80)
        got = enc.forward(feats).cpu().numpy()
        ref_mel = np.stack([M.log_mel_spectrogram(c, 80) for c in clips])
        ref = enc.forward_host(ref_mel)
    finally:
        enc.close()
    for i in range(2):
        assert R.cosine(got[i], ref[i]) >= 0.99999


def test_bad_arguments(cuda):
    out = torch.empty(1, 80, 3000, device="cuda")
    a = torch.zeros(100, device="cuda")
    with pytest.raises(ValueError):
        L.check(L.lib().wx_log_mel(a.data_ptr(), 1, 100, 50, 80, out.data_ptr(), None))
    with pytest.raises(L.WxError):
        L.check(L.lib().wx_log_mel(a.data_ptr(), 1, 100, 100, 64, out.data_ptr(), None))


def test_encode_recording_equals_windows_one_by_one(cuda):
    """A 67 s recording: three 30 s windows (the last 7 s, zero-padded) as one
    batch through log-mel and the encoder equal the windows done one by one,
    as the reference's transcribe loop does them (serve/npu_stt_server.py:
    421-431 and _window :331-342), at a reduced audio_ctx of 512."""
    import encoder_ref as R
    from wxb200 import audio as A
    from wxb200.encoder import Encoder
    rec = np.concatenate([M.synthetic_audio(30, 1), M.synthetic_audio(30, 2, "noise"),
                          M.synthetic_audio(7, 3)]).astype(np.float32)
    W = R.make_weights("tiny", seed=3, n_layer=2)
    enc = Encoder(W, n_layer=2, n_head=6, max_batch=2)     # two forwards: 2 + 1 windows
    try:
        feats, cut = A.encode_recording(enc, rec, ctx=512)
        assert cut == 0.0 and tuple(feats.shape) == (3, 512, 384)
        for i, off in enumerate(A.split_windows(rec.size)[0]):
            mel = A.log_mel_spectrogram(A.pad_or_trim(rec[off:off + A.N_SAMPLES]), 80,
                                        device="cuda")
            one = enc.forward(mel[:, :1024].contiguous())
            assert torch.equal(one, feats[i]), i
        feats2, cut2 = A.encode_recording(enc, rec, ctx=512, max_windows=2)
        assert cut2 == pytest.approx(7.0) and torch.equal(feats2, feats[:2])
    finally:
        enc.close()
