"""The 30 s window split of long recordings (wxb200.audio.split_windows)
against the reference's transcribe loop (serve/npu_stt_server.py:421-431),
restated here as the oracle: a fixed 30 s stride, a tail under half a second
dropped after the first window, at most NPU_STT_MAX_WINDOWS windows. CPU."""
import pytest

from wxb200.audio import N_SAMPLES, SAMPLE_RATE, split_windows


def reference_windows(n_samples, max_windows=0):
    offs, truncated = [], 0.0
    for off in range(0, max(n_samples, 1), N_SAMPLES):
        chunk = min(N_SAMPLES, n_samples - off) if n_samples > off else 0
        if off and chunk < SAMPLE_RATE // 2:
            break
        if max_windows and len(offs) >= max_windows:
            truncated = (n_samples - off) / SAMPLE_RATE
            break
        offs.append(off)
    return offs, truncated


@pytest.mark.parametrize("seconds", [0, 0.2, 29.9, 30, 30.3, 30.5, 45, 60.49, 60.5, 67, 300])
@pytest.mark.parametrize("max_windows", [0, 1, 2])
def test_split_matches_the_reference_loop(seconds, max_windows):
    n = int(round(seconds * SAMPLE_RATE))
    assert split_windows(n, max_windows) == reference_windows(n, max_windows)


def test_split_examples():
    assert split_windows(0) == ([0], 0.0)                        # silence: one window
    assert split_windows(67 * SAMPLE_RATE) == ([0, N_SAMPLES, 2 * N_SAMPLES], 0.0)
    assert split_windows(int(60.3 * SAMPLE_RATE)) == ([0, N_SAMPLES], 0.0)   # 0.3 s tail dropped
    offs, cut = split_windows(100 * SAMPLE_RATE, max_windows=2)
    assert offs == [0, N_SAMPLES] and cut == 40.0
