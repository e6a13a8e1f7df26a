"""Generate the log-mel fixtures that pin oracle/mel_ref.py.

Run here (the container with Hugging Face transformers installed):

    python tests/golden/make_mel_golden.py

transformers' WhisperFeatureExtractor (version recorded in each fixture) is an
independent implementation of openai-whisper's log_mel_spectrogram, the
function the reference calls (serve/npu_stt_server.py:334-336); openai-whisper
itself is not installed. Each fixture stores the case parameters (the audio is
regenerated from its seed by oracle/mel_ref.synthetic_audio), every 8th frame
of the extractor's output and the output's maximum.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "oracle"))
import mel_ref as M  # noqa: E402

CASES = [
    ("speechlike", 5.0, 11, 80),
    ("speechlike", 12.0, 12, 128),
    ("noise", 30.0, 13, 128),
    ("click", 30.0, 14, 80),
    ("silence", 3.0, 15, 80),
    ("speechlike", 31.0, 16, 80),       # longer than a window: trimmed to 30 s
]


def main():
    import transformers
    from transformers import WhisperFeatureExtractor
    for kind, seconds, seed, n_mels in CASES:
        audio = M.synthetic_audio(seconds, seed, kind)
        fe = WhisperFeatureExtractor(feature_size=n_mels)
        feats = fe(audio, sampling_rate=M.SAMPLE_RATE, return_tensors="np")["input_features"][0]
        assert feats.shape == (n_mels, M.N_FRAMES), feats.shape
        name = f"mel_{kind}_{int(seconds)}s_{n_mels}.npz"
        np.savez_compressed(HERE / name, kind=kind, seconds=seconds, seed=seed, n_mels=n_mels,
                            frames_every8=feats[:, ::8].astype(np.float32),
                            max=np.float32(feats.max()),
                            generator=f"transformers {transformers.__version__} "
                                      "WhisperFeatureExtractor")
        print(name, feats.shape, float(feats.max()))


if __name__ == "__main__":
    main()
