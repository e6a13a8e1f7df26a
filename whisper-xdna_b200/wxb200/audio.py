"""whisper's audio front end, for the reference server's _window
(serve/npu_stt_server.py:334-336: pad_or_trim, then log_mel_spectrogram), on
the GPU. openai-whisper is what the reference calls; it is not a dependency
here. The features stay on the device for Encoder.forward.
"""
import numpy as np
import torch

from . import ops

SAMPLE_RATE = 16000
N_SAMPLES = 30 * SAMPLE_RATE
N_FRAMES = 3000


def pad_or_trim(array, length=N_SAMPLES):
    """Zero-pad or cut the last axis to `length` (numpy or torch)."""
    if torch.is_tensor(array):
        n = array.shape[-1]
        if n > length:
            return array[..., :length]
        if n < length:
            return torch.nn.functional.pad(array, (0, length - n))
        return array
    array = np.asarray(array)
    n = array.shape[-1]
    if n > length:
        return array[..., :length]
    if n < length:
        return np.pad(array, [(0, 0)] * (array.ndim - 1) + [(0, length - n)])
    return array


def log_mel_spectrogram(audio, n_mels=80, device=None):
    """Log-mel features of 16 kHz mono audio ((n_samples,) or (batch,
    n_samples); numpy or torch), computed on the GPU. Returns a float32
    tensor (n_mels, 3000) (or (batch, n_mels, 3000)) on `device`, by default
    the audio's device if it is a CUDA tensor, else the CPU -- as whisper
    returns it on the input's device."""
    if torch.is_tensor(audio):
        src_dev = audio.device
        a = audio.detach().to(torch.float32)
    else:
        src_dev = torch.device("cpu")
        a = torch.from_numpy(np.ascontiguousarray(audio, dtype=np.float32))
    dev = torch.device("cuda") if not a.is_cuda else a.device
    a = a.to(dev).contiguous()
    out = ops.log_mel(a, n_mels=n_mels)
    target = device if device is not None else (src_dev if src_dev.type == "cuda" else "cpu")
    return out.to(target)


def split_windows(n_samples, max_windows=0):
    """Window offsets of a recording as the reference's transcribe loop takes
    them (serve/npu_stt_server.py:421-431): a fixed 30 s stride from sample 0
    (one window even for empty audio), a tail shorter than half a second
    after the first window dropped as not speech, at most `max_windows`
    windows (0: no limit). Returns (offsets, seconds dropped by the limit)."""
    offs, truncated = [], 0.0
    for off in range(0, max(int(n_samples), 1), N_SAMPLES):
        if off and n_samples - off < SAMPLE_RATE // 2:
            break
        if max_windows and len(offs) >= max_windows:
            truncated = (n_samples - off) / SAMPLE_RATE
            break
        offs.append(off)
    return offs, truncated


def encode_recording(encoder, audio, ctx=None, max_windows=0):
    """A whole recording through `encoder` (wxb200.encoder.Encoder) with its
    30 s windows as the batch dimension: the windows of split_windows, each
    zero-padded to 30 s as pad_or_trim does, get their log-mel features on the
    GPU in one launch and go through the encoder together (in groups of the
    encoder's max_batch). ctx: frames per window (the reference's audio_ctx,
    mel cut to 2*ctx; default the encoder's n_ctx). Returns (features
    (n_windows, ctx, d) float32 CUDA tensor, seconds dropped by max_windows)."""
    ctx = encoder.n_ctx if ctx is None else int(ctx)
    if torch.is_tensor(audio):
        a = audio.detach().to(device=encoder.device, dtype=torch.float32).reshape(-1)
    else:
        a = torch.from_numpy(np.ascontiguousarray(audio, dtype=np.float32).reshape(-1)).to(
            encoder.device)
    n = a.numel()
    offs, truncated = split_windows(n, max_windows)
    win = torch.zeros(len(offs), N_SAMPLES, dtype=torch.float32, device=encoder.device)
    for i, off in enumerate(offs):
        size = min(N_SAMPLES, n - off)
        if size > 0:
            win[i, :size] = a[off:off + size]
    mel = ops.log_mel(win, n_mels=encoder.n_mels)[:, :, :2 * ctx].contiguous()
    feats = torch.empty(len(offs), ctx, encoder.d, dtype=torch.float32, device=encoder.device)
    for s in range(0, len(offs), encoder.max_batch):
        e = min(len(offs), s + encoder.max_batch)
        encoder.forward(mel[s:e], out=feats[s:e])
    return feats, truncated
