"""Pin the log-mel oracle (oracle/mel_ref.py) on CPU: against fixtures made
with transformers' WhisperFeatureExtractor (tests/golden/make_mel_golden.py),
against torch.stft for the STFT, and against torchaudio's Slaney mel
filterbank (the filters openai-whisper ships are librosa's Slaney filters)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import mel_ref as M

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(GOLDEN.glob("mel_*.npz"))


def test_fixtures_present():
    assert len(FIXTURES) >= 6


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: p.stem)
def test_oracle_matches_whisper_feature_extractor(path):
    z = np.load(path)
    audio = M.synthetic_audio(float(z["seconds"]), int(z["seed"]), str(z["kind"]))
    got = M.log_mel_spectrogram(audio, int(z["n_mels"]))
    assert np.isclose(got.max(), float(z["max"]), atol=1e-5)
    assert np.abs(got[:, ::8] - z["frames_every8"]).max() < 2e-4


@pytest.mark.parametrize("n_mels", [80, 128])
def test_filterbank_matches_torchaudio_slaney(n_mels):
    ta = pytest.importorskip("torchaudio")
    fb = ta.functional.melscale_fbanks(M.N_BINS, 0.0, 8000.0, n_mels, M.SAMPLE_RATE,
                                       norm="slaney", mel_scale="slaney").numpy().T
    ours = M.mel_filters(n_mels)
    assert ours.shape == fb.shape
    # torchaudio builds the filters in float32: agreement to float32 round-off
    assert np.abs(ours - fb).max() < 1e-5 * np.abs(fb).max()


def test_stft_power_matches_torch_stft():
    audio = M.pad_or_trim(M.synthetic_audio(4.0, 3))
    x = torch.from_numpy(audio.astype(np.float64))
    st = torch.stft(x, M.N_FFT, M.HOP, window=torch.hann_window(M.N_FFT, dtype=torch.float64),
                    return_complex=True)
    ref = (st[..., :-1].abs() ** 2).numpy()
    ours = M.stft_power(audio)
    assert ours.shape == ref.shape == (M.N_BINS, M.N_FRAMES)
    assert np.abs(ours - ref).max() <= 1e-9 * ref.max()


def test_silence_is_constant():
    out = M.log_mel_spectrogram(np.zeros(100, np.float32), 80)
    assert np.all(out == np.float32(-1.5))
