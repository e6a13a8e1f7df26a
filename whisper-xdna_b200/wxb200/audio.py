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
