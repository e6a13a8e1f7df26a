"""wxb200: the Whisper-encoder hot path of drakosha/whisper-xdna, on NVIDIA
B200 (sm_100a).

The compute lives in libwxb200.so (csrc/, C ABI in include/wxb200.h): tcgen05
GEMMs with fused epilogues, a fused tcgen05 attention kernel and the
bandwidth-bound row ops (polynomial GELU, row softmax, LayerNorm). This
package is the host side: ctypes bindings (_lib), device-tensor wrappers
(ops), the reference's RawRT surface (runtime.B200RT), its row-op designs
(rowops), its fused-attention entry (attn) and its encoder entry point
(encoder.encoder / encoder.Encoder).
"""
from . import _lib  # noqa: F401

__all__ = ["ops", "runtime", "rowops", "attn", "encoder"]
