"""Test infrastructure (CPU oracle): whisper's log-mel frontend, restated.

The reference computes the encoder input with openai-whisper's
`log_mel_spectrogram` (serve/npu_stt_server.py:334-336, tools/dump_ref.py:55-56):
openai-whisper is a dependency the reference does not vendor (version
unpinned in its Dockerfile:75-77) and it is not installed here, so this file
restates its published algorithm:

  audio, 16 kHz, padded or trimmed to 30 s (480000 samples; pad_or_trim)
  STFT: n_fft 400, hop 160, periodic Hann window, centred frames (the signal
        reflect-padded by 200 on both sides), 1 + 480000/160 = 3001 frames of
        which the last is dropped -> 3000 frames, bins 0..200
  power |X|^2 -> mel filterbank (Slaney mel scale, Slaney area normalisation,
        0 .. 8 kHz) -> log10(max(., 1e-10)) -> max(., max - 8) -> (. + 4) / 4

Pinned in tests/test_mel_oracle.py against fixtures made with the Hugging
Face transformers WhisperFeatureExtractor (an independent implementation of
the same frontend; the generating script is tests/golden/make_mel_golden.py)
and against torch.stft and torchaudio's Slaney filterbank. Only tests/,
__graft_entry__.smoke() and bench.py's CPU legs use this module.
"""
import numpy as np

SAMPLE_RATE = 16000
N_FFT = 400
HOP = 160
N_SAMPLES = 30 * SAMPLE_RATE
N_FRAMES = N_SAMPLES // HOP          # 3000
N_BINS = N_FFT // 2 + 1              # 201


def pad_or_trim(audio, length=N_SAMPLES):
    """whisper.pad_or_trim on the last axis: zero-pad or cut to `length`."""
    audio = np.asarray(audio, dtype=np.float32)
    n = audio.shape[-1]
    if n > length:
        return audio[..., :length]
    if n < length:
        pad = [(0, 0)] * (audio.ndim - 1) + [(0, length - n)]
        return np.pad(audio, pad)
    return audio


def hann_periodic(n=N_FFT):
    """torch.hann_window(n) (periodic): 0.5 - 0.5 cos(2 pi k / n)."""
    k = np.arange(n, dtype=np.float64)
    return 0.5 - 0.5 * np.cos(2.0 * np.pi * k / n)


def _hz_to_mel_slaney(f):
    f = np.asarray(f, dtype=np.float64)
    f_sp = 200.0 / 3.0
    mels = f / f_sp
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, 1e-12) / min_log_hz) / logstep,
                    mels)


def _mel_to_hz_slaney(m):
    m = np.asarray(m, dtype=np.float64)
    f_sp = 200.0 / 3.0
    freqs = f_sp * m
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), freqs)


def mel_filters(n_mels, sr=SAMPLE_RATE, n_fft=N_FFT, fmin=0.0, fmax=None):
    """Slaney-style mel filterbank (n_mels, n_fft // 2 + 1), float64: triangles
    between consecutive mel-spaced band edges, each scaled by 2 / (bandwidth
    in Hz) (Slaney area normalisation)."""
    fmax = sr / 2.0 if fmax is None else fmax
    fft_freqs = np.linspace(0.0, sr / 2.0, n_fft // 2 + 1)
    mel_pts = np.linspace(_hz_to_mel_slaney(fmin), _hz_to_mel_slaney(fmax), n_mels + 2)
    hz_pts = _mel_to_hz_slaney(mel_pts)
    fdiff = np.diff(hz_pts)
    ramps = hz_pts[:, None] - fft_freqs[None, :]
    lower = -ramps[:-2] / fdiff[:-1, None]
    upper = ramps[2:] / fdiff[1:, None]
    weights = np.maximum(0.0, np.minimum(lower, upper))
    enorm = 2.0 / (hz_pts[2:n_mels + 2] - hz_pts[:n_mels])
    return weights * enorm[:, None]


def stft_power(audio):
    """|STFT|^2 of 30 s of audio: (N_BINS, N_FRAMES) float64 (the centred,
    reflect-padded frames of torch.stft, last frame dropped)."""
    audio = np.asarray(audio, dtype=np.float64)
    padded = np.pad(audio, (N_FFT // 2, N_FFT // 2), mode="reflect")
    n_frames = 1 + (padded.size - N_FFT) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(n_frames)[:, None]
    frames = padded[idx] * hann_periodic()[None, :]
    spec = np.fft.rfft(frames, axis=1)
    return (np.abs(spec) ** 2).T[:, :-1]


def log_mel_spectrogram(audio, n_mels=80):
    """whisper's log_mel_spectrogram of one clip of N_SAMPLES samples ->
    (n_mels, N_FRAMES) float32."""
    audio = pad_or_trim(audio)
    mel = mel_filters(n_mels) @ stft_power(audio)
    log_spec = np.log10(np.maximum(mel, 1e-10))
    log_spec = np.maximum(log_spec, log_spec.max() - 8.0)
    return ((log_spec + 4.0) / 4.0).astype(np.float32)


def synthetic_audio(seconds, seed, kind="speechlike"):
    """Seeded 16 kHz test signals: 'speechlike' (harmonic tones with a
    syllable envelope plus noise), 'noise', 'silence', 'click' (isolated
    impulses)."""
    rng = np.random.default_rng(seed)
    n = int(seconds * SAMPLE_RATE)
    t = np.arange(n) / SAMPLE_RATE
    if kind == "silence":
        return np.zeros(n, np.float32)
    if kind == "noise":
        return (0.1 * rng.standard_normal(n)).astype(np.float32)
    if kind == "click":
        x = np.zeros(n, np.float32)
        x[rng.integers(0, n, 20)] = rng.uniform(-0.9, 0.9, 20)
        return x
    f0 = 110.0 + 60.0 * rng.random()
    env = 0.5 * (1 - np.cos(2 * np.pi * 3.0 * t)) * (t < seconds)
    x = sum((0.3 / k) * np.sin(2 * np.pi * k * f0 * t + rng.uniform(0, 2 * np.pi))
            for k in range(1, 12))
    x = env * x + 0.01 * rng.standard_normal(n)
    return x.astype(np.float32)
