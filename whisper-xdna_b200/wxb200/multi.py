"""One host batch of clips encoded across the GPUs of this machine: one
Encoder replica per device, the batch split into contiguous per-device slices
by clip index (wxb200.dist.shard), no exchange between the devices.

The reference encodes one window at a time on one NPU (a Semaphore(1) around
every pass, serve/npu_stt_server.py:131,338-342); clips are independent, so
a batch of windows spreads over N GPUs with nothing to combine but the
output rows, which each device writes straight into its slice of `out`.

This is the in-process form of the clip sharding that bench.py runs as one
process per GPU under torchrun. Each device is driven from its own host
thread: the engine's host entry point blocks on its own copies, and ctypes
releases the GIL for the call, so the devices run at the same time. With
pinned host buffers (`host_buffers`) the copies run at full PCIe speed.
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from .dist import shard
from .encoder import Encoder


class MultiGPUEncoder:
    """Encoder replicas on `devices` (default: every visible GPU).

    max_batch is the largest host batch one call takes; each device's replica
    is sized for its share, ceil(max_batch / n_devices) clips. The other
    arguments are Encoder's."""

    def __init__(self, W, devices=None, max_batch=64, n_layer=None, n_head=None, gelu="poly4",
                 quant=None):
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 encoder needs CUDA devices; there is no CPU fallback")
        self.devices = (list(range(torch.cuda.device_count())) if devices is None
                        else [int(d) for d in devices])
        if not self.devices:
            raise ValueError("no devices")
        self.max_batch = int(max_batch)
        per_dev = -(-self.max_batch // len(self.devices))
        self.encoders = [Encoder(W, n_layer=n_layer, n_head=n_head, max_batch=per_dev,
                                 gelu=gelu, device=d, quant=quant) for d in self.devices]
        e0 = self.encoders[0]
        self.n_mels, self.d, self.n_ctx = e0.n_mels, e0.d, e0.n_ctx
        self._pool = ThreadPoolExecutor(max_workers=len(self.devices),
                                        thread_name_prefix="wx-encoder")

    def slices(self, batch):
        """The [start, stop) clip range each device takes of a batch."""
        return [shard(batch, len(self.devices), r) for r in range(len(self.devices))]

    def host_buffers(self, batch, n_frames):
        """Pinned (mel, out) numpy arrays for a batch: (batch, n_mels, n_frames)
        and (batch, n_frames // 2, d) float32."""
        mel = torch.empty(batch, self.n_mels, n_frames, pin_memory=True)
        out = torch.empty(batch, n_frames // 2, self.d, pin_memory=True)
        return mel.numpy(), out.numpy()

    def forward_host(self, mel, out=None):
        """mel: host float32 (batch, n_mels, n_frames) -> features (batch,
        n_frames // 2, d) float32, written into `out` if given. Clip i of the
        output is clip i of the input, whatever device encoded it; each clip's
        features equal a one-device forward of that clip bit for bit."""
        mel = np.ascontiguousarray(np.asarray(mel, dtype=np.float32))
        if mel.ndim != 3 or mel.shape[1] != self.n_mels:
            raise ValueError(f"mel must be (batch, {self.n_mels}, n_frames)")
        B, _, F = mel.shape
        if B > self.max_batch:
            raise ValueError(f"batch {B} > max_batch {self.max_batch}")
        if out is None:
            out = np.empty((B, F // 2, self.d), dtype=np.float32)
        if (not isinstance(out, np.ndarray) or out.dtype != np.float32
                or out.shape != (B, F // 2, self.d) or not out.flags.c_contiguous):
            raise ValueError(f"out must be a C-contiguous float32 array of shape "
                             f"{(B, F // 2, self.d)}")

        def run(i):
            lo, hi = self.slices(B)[i]
            if hi > lo:
                enc = self.encoders[i]
                with torch.cuda.device(enc.device):
                    enc.forward_host(mel[lo:hi], out=out[lo:hi])

        for f in [self._pool.submit(run, i) for i in range(len(self.devices))]:
            f.result()
        return out

    def close(self):
        for e in self.encoders:
            e.close()
        self._pool.shutdown(wait=True)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
