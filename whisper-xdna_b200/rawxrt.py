"""Drop-in for the reference's src/rawxrt.py: RawRT is the CUDA runtime
wxb200.runtime.B200RT (device buffers, streams, tcgen05 kernels, CUDA graphs)."""
from wxb200.runtime import B200RT, ROWOPS, default_runtime  # noqa: F401

RawRT = B200RT
MAX_CTX = None          # no hardware-context ceiling on the GPU
PROF = {}               # the reference's timing accumulator; kept for readers
