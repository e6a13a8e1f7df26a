"""Drop-in for the reference's src/npu_whisper_encoder.py on the B200.

encoder() keeps the reference's signature and return value (src/npu_whisper_encoder.py
:436-541) and runs the whole forward on the GPU (wxb200.encoder). The host
utilities the reference's callers use around it -- prepare_mlp_chunks,
zero_bias, new_block, clear_tensor_cache -- are provided; the reference's numpy
compute path (np_matmul, layer_norm, gelu, softmax, im2col) is not: this
module never computes on the CPU.
"""
import numpy as np

from wxb200.encoder import Encoder, encoder, geometry  # noqa: F401

MAX_GEMM_N = 4096
CPU_PROF = {}
FC1_TAP = None
_ZERO_BIAS = {}


def zero_bias(d):
    """A stable all-zero bias row (the key projection has none)."""
    b = _ZERO_BIAS.get(d)
    if b is None:
        b = _ZERO_BIAS[d] = np.zeros(d, dtype=np.float32)
    return b


def new_block():
    """Nothing to invalidate: activations never leave the device."""


def clear_tensor_cache():
    """Nothing to clear: device buffers belong to the runtime's engines."""


def prepare_mlp_chunks(W, n_layer, d, chunk=0):
    """Split each fc1 weight into column chunks under w.blocks.L.mlp.0.parts,
    as the reference's NPU GEMM needed (src/npu_whisper_encoder.py:364-406);
    returns the new arrays. The B200 kernels need no chunking -- the full
    weight stays in W and is what the encoder engine uploads -- but
    RawRT.mlp callers pass the parts."""
    made = []
    for L in range(n_layer):
        p = f"w.blocks.{L}."
        key = p + "mlp.0.weight_T"
        W1 = W[key] if key in W else np.ascontiguousarray(np.asarray(W[p + "mlp.0.weight"]).T)
        b1 = W[p + "mlp.0.bias"]
        N = W1.shape[1]
        if chunk:
            width = chunk
        elif N <= MAX_GEMM_N:
            continue
        elif N % d == 0:
            width = d
        else:
            width = N // ((N + MAX_GEMM_N - 1) // MAX_GEMM_N)
        if N <= width:
            continue
        parts = []
        for j in range(0, N, width):
            wc = np.ascontiguousarray(W1[:, j:j + width])
            bc = np.ascontiguousarray(b1[j:j + width])
            parts.append((wc, bc))
            made += [wc, bc]
        W[p + "mlp.0.parts"] = parts
    return made
