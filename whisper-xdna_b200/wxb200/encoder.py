"""The Whisper encoder on the B200: an engine that owns the device weights and
workspace (wx_encoder_*), and `encoder()`, the drop-in for the reference's
entry point src/npu_whisper_encoder.py:436-541.
"""
import ctypes
import time

import numpy as np
import torch

from . import _lib as L


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _linear(W, key):
    """(out, in) weight from the reference's W dict, which may hold the torch
    layout under `...weight` and/or the transposed copy under `...weight_T`
    (src/npu_whisper_encoder.py:563-566)."""
    if key + "weight" in W:
        return _f32(W[key + "weight"])
    return _f32(np.asarray(W[key + "weight_T"]).T)


def geometry(W, n_layer=None, n_head=None):
    """(n_mels, d_model, n_head, n_layer, ffn, n_ctx) read off the weights, like
    src/npu_whisper_encoder.py:571-572 does."""
    c1 = np.asarray(W["w.conv1.weight"])
    d, n_mels = c1.shape[0], c1.shape[1]
    have = 1 + max(int(k.split(".")[2]) for k in W if k.startswith("w.blocks."))
    nl = have if n_layer is None else n_layer
    if nl > have:
        raise ValueError(f"n_layer={nl} but the weights hold {have} layers")
    nh = d // 64 if n_head is None else n_head
    ffn = np.asarray(W["w.blocks.0.mlp.0.bias"]).shape[0]
    n_ctx = np.asarray(W["w.positional_embedding"]).shape[0]
    return n_mels, d, nh, nl, ffn, n_ctx


def synthetic_weights(n_mels=128, d=1280, ffn=5120, n_layer=32, n_ctx=1500, seed=1):
    """Random N(0, 0.02) weights of a Whisper encoder in the reference's W-dict
    layout (bf16-exact fp32 arrays, torch CPU generator), LayerNorm gamma 1 and
    beta 0, sinusoidal positions: the synthetic stand-in for a checkpoint that
    the benchmarks use (defaults: large-v3 geometry)."""
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    inc = np.log(10000) / (d // 2 - 1)
    t = np.arange(n_ctx)[:, None] * np.exp(-inc * np.arange(d // 2))[None, :]
    pos = np.concatenate([np.sin(t), np.cos(t)], axis=1).astype(np.float32)
    W = {"w.conv1.weight": rn(d, n_mels, 3), "w.conv1.bias": rn(d),
         "w.conv2.weight": rn(d, d, 3), "w.conv2.bias": rn(d),
         "w.positional_embedding": pos,
         "w.ln_post.weight": np.ones(d, np.float32), "w.ln_post.bias": np.zeros(d, np.float32)}
    for l in range(n_layer):
        p = f"w.blocks.{l}."
        for ln in ("attn_ln", "mlp_ln"):
            W[p + ln + ".weight"] = np.ones(d, np.float32)
            W[p + ln + ".bias"] = np.zeros(d, np.float32)
        for n, sh in (("attn.query.weight", (d, d)), ("attn.query.bias", (d,)),
                      ("attn.key.weight", (d, d)), ("attn.value.weight", (d, d)),
                      ("attn.value.bias", (d,)), ("attn.out.weight", (d, d)),
                      ("attn.out.bias", (d,)), ("mlp.0.weight", (ffn, d)), ("mlp.0.bias", (ffn,)),
                      ("mlp.2.weight", (d, ffn)), ("mlp.2.bias", (d,))):
            W[p + n] = rn(*sh)
    return W


class Encoder:
    """A Whisper encoder resident on one GPU.

    gelu: "poly4" -- the reference's device GELU (g4f / g4r: the RNE piecewise
    polynomial of kernels/gelu_poly4_eval.inc), "erf" -- exact erf-GELU (the
    reference's numpy path).
    quant: None (bf16 GEMMs), "int8-perchan" or "int8-pertensor" -- the
    reference's int8 projection/MLP mode (bench/probe_int8_decode.py:48-74):
    int8 operands on the int8 tensor cores, per-token activation scales,
    per-channel or per-matrix weight scales. The probe runs it with the erf
    GELU, so pass gelu="erf" to follow it.
    """

    QUANT_MODES = {None: L.WX_QUANT_NONE, "int8-perchan": L.WX_QUANT_INT8_PERCHAN,
                   "int8-pertensor": L.WX_QUANT_INT8_PERTENSOR}

    def __init__(self, W, n_layer=None, n_head=None, max_batch=1, gelu="poly4", device=None,
                 quant=None):
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 encoder needs a CUDA device; there is no CPU fallback")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        (self.n_mels, self.d, self.n_head, self.n_layer, self.ffn,
         self.n_ctx) = geometry(W, n_layer, n_head)
        self.max_batch = int(max_batch)
        self.gelu = gelu
        mode = {"poly4": L.WX_GELU_POLY4, "erf": L.WX_GELU_ERF}[gelu]
        if quant not in self.QUANT_MODES:
            raise ValueError(f"quant must be one of {list(self.QUANT_MODES)}")
        self.quant = quant
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.check(L.lib().wx_encoder_create(ctypes.byref(h), self.n_mels, self.d,
                                              self.n_head, self.n_layer, self.ffn,
                                              self.n_ctx, self.max_batch, mode))
        self._h = h
        if quant is not None:
            with torch.cuda.device(self.device):
                L.check(L.lib().wx_encoder_set_quant(h, self.QUANT_MODES[quant]))
        self._load(W)

    def _load(self, W):
        lib = L.lib()
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        keep = []

        def arr(a):
            a = _f32(a)
            keep.append(a)
            return p(a)

        with torch.cuda.device(self.device):
            L.check(lib.wx_encoder_set_frontend(
                self._h, arr(W["w.conv1.weight"]), arr(W["w.conv1.bias"]),
                arr(W["w.conv2.weight"]), arr(W["w.conv2.bias"]),
                arr(np.asarray(W["w.positional_embedding"])[:self.n_ctx])))
            for l in range(self.n_layer):
                b = f"w.blocks.{l}."
                L.check(lib.wx_encoder_set_layer(
                    self._h, l, arr(W[b + "attn_ln.weight"]), arr(W[b + "attn_ln.bias"]),
                    arr(_linear(W, b + "attn.query.")), arr(W[b + "attn.query.bias"]),
                    arr(_linear(W, b + "attn.key.")),
                    arr(_linear(W, b + "attn.value.")), arr(W[b + "attn.value.bias"]),
                    arr(_linear(W, b + "attn.out.")), arr(W[b + "attn.out.bias"]),
                    arr(W[b + "mlp_ln.weight"]), arr(W[b + "mlp_ln.bias"]),
                    arr(_linear(W, b + "mlp.0.")), arr(W[b + "mlp.0.bias"]),
                    arr(_linear(W, b + "mlp.2.")), arr(W[b + "mlp.2.bias"])))
                keep.clear()
            L.check(lib.wx_encoder_set_ln_post(self._h, arr(W["w.ln_post.weight"]),
                                               arr(W["w.ln_post.bias"])))

    @property
    def device_bytes(self):
        return int(L.lib().wx_encoder_device_bytes(self._h))

    def forward(self, mel, out=None, use_graph=True):
        """mel: CUDA fp32 (batch, n_mels, n_frames) (or (n_mels, n_frames)) on this
        encoder's device -> (batch, n_frames // 2, d) fp32 CUDA tensor, on torch's
        current stream of that device."""
        squeeze = mel.dim() == 2
        if squeeze:
            mel = mel.unsqueeze(0)
        if not mel.is_cuda or mel.dtype != torch.float32:
            raise ValueError("mel must be a float32 CUDA tensor")
        if mel.device != self.device:
            raise ValueError(f"mel is on {mel.device}, the encoder on {self.device}")
        mel = mel.contiguous()
        B, C, F = mel.shape
        if C != self.n_mels:
            raise ValueError(f"mel has {C} bins, the weights expect {self.n_mels}")
        if out is None:
            out = torch.empty(B, F // 2, self.d, dtype=torch.float32, device=mel.device)
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        L.check(L.lib().wx_encoder_forward(self._h, ctypes.c_void_p(mel.data_ptr()),
                                           ctypes.c_void_p(out.data_ptr()), B, F,
                                           1 if use_graph else 0, st))
        return out[0] if squeeze else out

    def forward_host(self, mel, out=None, use_graph=True):
        """The same from HOST memory: numpy fp32 (batch, n_mels, n_frames) or
        (n_mels, n_frames) in, numpy (batch, T, d) / (T, d) out. Copies in,
        runs and copies out through wx_encoder_forward_host (synchronous)."""
        mel = np.asarray(mel, dtype=np.float32)
        squeeze = mel.ndim == 2
        if squeeze:
            mel = mel[None]
        mel = np.ascontiguousarray(mel)
        B, C, F = mel.shape
        if C != self.n_mels:
            raise ValueError(f"mel has {C} bins, the weights expect {self.n_mels}")
        if out is None:
            out = np.empty((B, F // 2, self.d), dtype=np.float32)
        elif squeeze and out.shape == (F // 2, self.d):
            out = out[None]
        if (not isinstance(out, np.ndarray) or out.dtype != np.float32
                or out.shape != (B, F // 2, self.d) or not out.flags.c_contiguous):
            raise ValueError(f"out must be a C-contiguous float32 array of shape "
                             f"{(B, F // 2, self.d)}")
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        L.check(L.lib().wx_encoder_forward_host(self._h, mel.ctypes.data_as(ctypes.c_void_p),
                                                out.ctypes.data_as(ctypes.c_void_p), B, F,
                                                1 if use_graph else 0, st))
        return out[0] if squeeze else out

    def submit_host(self, mel, out):
        """Pipelined forward_host for a stream of batches: enqueue the copy-in,
        forward and copy-out of one batch and return at once, so one batch's
        copies overlap its neighbours' compute (wx_encoder_submit_host). `mel`
        (batch, n_mels, n_frames) and `out` (batch, n_frames/2, d) are C-contiguous
        fp32 numpy arrays, pinned for the overlap (e.g. views of pinned torch
        tensors); both must stay untouched until wait_host(). Two batches are in
        flight at most: a call waits for the batch submitted two calls earlier."""
        if not (isinstance(mel, np.ndarray) and isinstance(out, np.ndarray)):
            raise TypeError("submit_host takes numpy arrays (the copies read and write them later)")
        if (mel.dtype != np.float32 or out.dtype != np.float32 or mel.ndim != 3 or out.ndim != 3
                or not mel.flags.c_contiguous or not out.flags.c_contiguous):
            raise ValueError("submit_host: mel and out must be C-contiguous 3-D fp32 arrays")
        B, C, F = mel.shape
        if C != self.n_mels:
            raise ValueError(f"mel has {C} bins, the weights expect {self.n_mels}")
        if out.shape != (B, F // 2, self.d):
            raise ValueError(f"out must be {(B, F // 2, self.d)}, got {out.shape}")
        L.check(L.lib().wx_encoder_submit_host(self._h, mel.ctypes.data_as(ctypes.c_void_p),
                                               out.ctypes.data_as(ctypes.c_void_p), B, F, 1))
        self._inflight = (getattr(self, "_inflight", []) + [(mel, out)])[-2:]

    def wait_host(self):
        """Block until every submitted batch's features are in its `out`."""
        L.check(L.lib().wx_encoder_wait_host(self._h))
        self._inflight = []

    def close(self):
        if getattr(self, "_h", None):
            L.lib().wx_encoder_destroy(self._h)
            self._h = None
            self._inflight = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def encoder(W, mel, mm=None, attn_mm=None, n_layer=4, n_head=6, prof=None,
            fused_gelu=False, npu_softmax=False, attn_fn=None, mlp_fn=None,
            fold_bias=True):
    """Drop-in for src/npu_whisper_encoder.py:436-541: W (reference weight
    dict), mel (n_mels, 2*ctx) fp32 -> (ctx, d) fp32 numpy.

    The whole forward runs on the B200 as one captured launch sequence, so the
    per-operation callables of the reference (mm, attn_mm, attn_fn, mlp_fn) only
    select the runtime: they must be methods of a B200RT (whose engine cache is
    used) or None (the default runtime). fused_gelu, npu_softmax and fold_bias
    are accepted for compatibility; the device path always fuses bias, GELU and
    softmax. Any other callable is an error -- this module never computes on the
    CPU.
    """
    from .runtime import B200RT, default_runtime
    rt = None
    for fn in (mm, attn_mm, attn_fn, mlp_fn):
        if fn is None:
            continue
        owner = getattr(fn, "__self__", None)
        if not isinstance(owner, B200RT):
            raise TypeError(
                f"encoder(): {getattr(fn, '__name__', fn)!r} is not a B200RT method; the B200 "
                "encoder runs every stage on the GPU and takes no host callables")
        rt = owner if rt is None else rt
    rt = rt or default_runtime()
    t0 = time.perf_counter()
    out = rt.encoder_engine(W, n_layer, n_head).forward_host(mel)
    if prof is not None:
        prof["total"] = time.perf_counter() - t0
    return out
