"""B200RT: the reference's RawRT surface (src/rawxrt.py) on CUDA.

RawRT manages XRT buffer objects, hw_contexts and run-lists for the NPU; here
the same methods drive CUDA device buffers, the tcgen05 kernels of
libwxb200.so and, for the whole encoder, a captured CUDA graph:

  matmul / mm_start / mm_finish   src/rawxrt.py:926-996
  attn_chain / attn_fused         src/rawxrt.py:761-891
  mlp                             src/rawxrt.py:436-544
  gelu                            src/rawxrt.py:546-565
  softmax_stack                   src/rawxrt.py:569-585
  rowop                           src/rawxrt.py:384-400
  register_weights                src/rawxrt.py:307-316

Host arrays (numpy fp32 or bf16) are accepted where the reference takes them
and results come back as fp32 numpy arrays, as the reference returns them;
CUDA tensors are accepted too and stay on the device. Errors raise (ValueError
for bad shapes, RuntimeError for device failures); the reference's degradation
ladder (chain -> host path) is not reproduced because there is no host path:
the `*_ok` flags and `fallbacks` list exist for callers that read them and
stay True / empty.
"""
import os
import time

import numpy as np
import torch

from . import _lib as L
from . import ops
from .encoder import Encoder

# op codes of src/compile_rowop.py:12-31 -> (kind, arguments)
ROWOPS = {
    "g4": ("gelu", L.WX_ROUND_TRUNC),
    "g4r": ("gelu", L.WX_ROUND_RNE),
    "g4f": ("gelu_f32", L.WX_ROUND_RNE),
    "sm": ("softmax", 1, L.WX_ROUND_TRUNC),
    "s2": ("softmax", 4, L.WX_ROUND_TRUNC),
    "s3": ("softmax", 3, L.WX_ROUND_TRUNC),
    "s3w": ("softmax", 3, L.WX_ROUND_TRUNC),
    "s4": ("softmax", 4, L.WX_ROUND_TRUNC),
    "s4w": ("softmax", 4, L.WX_ROUND_TRUNC),
    "s4rw": ("softmax", 4, L.WX_ROUND_RNE),
    "ln": ("layernorm", L.WX_ROUND_TRUNC),
}


def _bf16_host(x):
    """numpy (fp32 or ml_dtypes bf16) -> torch bf16 CPU tensor (RNE, as
    ml_dtypes and the reference's astype(bfloat16) round)."""
    a = np.asarray(x)
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.uint16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


class _Handle:
    __slots__ = ("out", "event", "M", "N", "t_submit")


class B200RT:
    # Kept for callers that read them; the GPU has no overlay or context limit.
    GELU_ROWS, GELU_COLS = 7680, 1024
    GELU_OP = os.environ.get("GELU_OP", "g4r")
    GELU_F32_OP = os.environ.get("GELU_F32_OP", "g4f")
    SM_OP = os.environ.get("SM_OP", "s3")

    def __init__(self, max_ctx=None, device=None):
        if not torch.cuda.is_available():
            raise RuntimeError("B200RT needs a CUDA device; there is no CPU fallback")
        L.lib()
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        self.max_ctx = max_ctx
        self.calls = 0
        self.ctx_creates = 0
        self.evictions = 0
        self.chain_ok = self.fused_ok = self.mlp_ok = self.softmax_ok = True
        self.fallbacks = []
        self._known = {}      # id(array) -> key, for registered (immutable) arrays
        self._keep = []       # the registered arrays, so their ids stay unique
        self._wdev = {}       # (key, tag) -> device tensor
        self._akey = None     # (akey, tensor): the last named activation
        self._engines = {}    # (id(W), n_layer, n_head, gelu) -> (array ids, arrays, Encoder)
        # the reference's state containers, read/cleared by the STT server
        # (serve/npu_stt_server.py:315-325, 379-387)
        self._chains, self._scratch, self._scratch_owner = {}, {}, {}
        self._live, self._views = {}, {}
        self.gelu_mode = os.environ.get("WX_GELU", "poly4")

    # ---------------------------------------------------------------- buffers
    def register_weights(self, arrays):
        """Name arrays that never change so their device copy is made once
        (src/rawxrt.py:307-316). References are held, so ids stay unique."""
        for a in arrays:
            if id(a) not in self._known:
                self._known[id(a)] = f"w{len(self._known)}"
                self._keep.append(a)

    def _evict_lru(self):
        """Drop every cached device buffer (the server calls this to release a
        geometry, serve/npu_stt_server.py:318-320)."""
        self._wdev.clear()
        self._akey = None
        self._live.clear()

    def _dev(self, x, dtype):
        if isinstance(x, torch.Tensor):
            return x.to(device=self.device, dtype=dtype)
        if dtype == torch.bfloat16:
            return _bf16_host(x).to(self.device, non_blocking=False)
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(self.device)

    def _weight_nk(self, B, bkey=None):
        """B (K, N) as passed by the reference (weight_T) -> device bf16 (N, K),
        cached when B is registered or named."""
        key = bkey if bkey is not None else self._known.get(id(B))
        if key is not None and (key, "nk") in self._wdev:
            return self._wdev[(key, "nk")]
        t = self._dev(B, torch.bfloat16).t().contiguous()
        if key is not None:
            self._wdev[(key, "nk")] = t
        return t

    def _bias(self, b):
        if b is None:
            return None
        key = self._known.get(id(b))
        if key is not None and (key, "f32") in self._wdev:
            return self._wdev[(key, "f32")]
        t = self._dev(b, torch.float32).reshape(-1).contiguous()
        if key is not None:
            self._wdev[(key, "f32")] = t
        return t

    def _activation(self, A, akey=None):
        if akey is not None and self._akey is not None and self._akey[0] == akey:
            return self._akey[1]
        t = self._dev(A, torch.bfloat16).contiguous()
        if t.shape[1] % 8:
            t = torch.nn.functional.pad(t, (0, 8 - t.shape[1] % 8))
        if akey is not None:
            self._akey = (akey, t)
        return t

    # ---------------------------------------------------------------- GEMM
    def mm_start(self, A, B, akey=None, bkey=None, bias=None, cbo=None):
        """Submit A @ B (+ bias) and return a handle; mm_finish collects it.
        A (M, K), B (K, N): bf16 operands, fp32 accumulation (src/rawxrt.py:926)."""
        M, K = A.shape
        K2, N = B.shape
        if K != K2:
            raise ValueError(f"shape mismatch {A.shape} @ {B.shape}")
        a = self._activation(A, akey)
        w = self._weight_nk(B, bkey)
        if w.shape[1] != a.shape[1]:
            w = torch.nn.functional.pad(w, (0, a.shape[1] - w.shape[1]))
            w = w.contiguous()
        out = cbo if cbo is not None else torch.empty(M, N, dtype=torch.float32,
                                                      device=self.device)
        ops.gemm(a, w, bias=self._bias(bias), out=out, epilogue=L.WX_EPI_F32)
        h = _Handle()
        h.out, h.M, h.N = out, M, N
        h.event = torch.cuda.Event()
        h.event.record()
        h.t_submit = time.perf_counter()
        self.calls += 1
        return h

    def mm_finish(self, h):
        h.event.synchronize()
        return h.out.cpu().numpy()

    def matmul(self, A, B, akey=None, bkey=None, bias=None):
        """A (M,K) @ B (K,N) -> (M,N) fp32, bf16 in, fp32 accumulate (src/rawxrt.py:993)."""
        return self.mm_finish(self.mm_start(A, B, akey=akey, bkey=bkey, bias=bias))

    # ---------------------------------------------------------------- attention
    def attn_chain(self, q, k, v, nh, scale):
        """o = concat_h softmax((q_h*scale)(k_h*scale)^T) v_h for (ctx, d) inputs
        (src/rawxrt.py:813): one fused tcgen05 kernel over all heads."""
        ctx, d = q.shape
        qd = self._dev(q, torch.bfloat16).contiguous()
        kd = self._dev(k, torch.bfloat16).contiguous()
        vd = self._dev(v, torch.bfloat16).contiguous()
        o = ops.attention(qd, kd, vd, 1, nh, float(scale) * float(scale))
        self.calls += 1
        if isinstance(q, torch.Tensor):
            return o.float()
        return o.float().cpu().numpy()

    def attn_fused(self, q, k, v, nh, scale):
        """The reference's fused-attention overlay (src/rawxrt.py:761): the same
        kernel as attn_chain here."""
        return self.attn_chain(q, k, v, nh, scale)

    # ---------------------------------------------------------------- MLP
    def mlp(self, h, parts, B, akey=None, bkey=None):
        """fc2(GELU(fc1(h))) without fc2's bias (src/rawxrt.py:436): every fc1
        column chunk (W1_j, b1_j) runs with bias + GELU fused in its epilogue and
        writes its band of fc2's bf16 input; fc2 runs from that buffer."""
        a = self._activation(h, akey)
        M = a.shape[0]
        widths = [np.asarray(wc).shape[1] for wc, _ in parts]
        F = sum(widths)
        f = torch.empty(M, F, dtype=torch.bfloat16, device=self.device)
        epi = L.WX_EPI_BF16_GELU if self.gelu_mode == "poly4" else L.WX_EPI_BF16_GELU_ERF
        c0 = 0
        for (wc, bc), w in zip(parts, widths):
            ops.gemm(a, self._weight_nk(wc), bias=self._bias(bc), out=f[:, c0:c0 + w],
                     epilogue=epi)
            c0 += w
        out = ops.gemm(f, self._weight_nk(B, bkey), epilogue=L.WX_EPI_F32)
        self.calls += 1 + len(parts)
        return out.cpu().numpy()

    # ---------------------------------------------------------------- row ops
    def gelu(self, x):
        """GELU of any-shaped fp32 array through GELU_OP (default g4r: the input
        rounded to bf16, RNE poly4), fp32 out (src/rawxrt.py:546-565)."""
        a = np.asarray(x, dtype=np.float32)
        flat = a.reshape(1, -1)
        if self.GELU_OP == "g4f":
            t = self._dev(flat, torch.float32)
            r = ops.gelu_poly4(t, rounding=L.WX_ROUND_RNE)
        else:
            kind = ROWOPS[self.GELU_OP]
            t = self._dev(flat, torch.bfloat16)
            r = ops.gelu_poly4(t, rounding=kind[1])
        self.calls += 1
        return r.float().cpu().numpy().reshape(a.shape)

    def softmax_stack(self, mats):
        """Row softmax of every head's (L0, L1) score matrix in one launch,
        stacked into (nh*L0, ceil16(L1)) and padded with -30000
        (src/rawxrt.py:569-585); SM_OP selects the variant (default s3)."""
        nh = len(mats)
        L0, L1 = np.asarray(mats[0]).shape
        cols = (L1 + 15) // 16 * 16
        big = torch.full((nh * L0, cols), -30000.0, dtype=torch.bfloat16, device=self.device)
        for i, m in enumerate(mats):
            big[i * L0:(i + 1) * L0, :L1] = self._dev(m, torch.bfloat16)
        kind = ROWOPS[self.SM_OP]
        r = ops.softmax_rows(big, variant=kind[1], rounding=kind[2])
        f = r.float().cpu().numpy()
        self.calls += 1
        return [f[i * L0:(i + 1) * L0, :L1] for i in range(nh)]

    def rowop(self, op, buf_bf16, rows, cols, valid=0, out_cols=0):
        """Run row op `op` (a src/compile_rowop.py code) over a (rows, cols)
        buffer; returns bf16 (ml_dtypes) numpy (src/rawxrt.py:384-400)."""
        import ml_dtypes
        if op not in ROWOPS:
            raise ValueError(f"unknown row op {op!r}; this build implements {sorted(ROWOPS)}")
        kind = ROWOPS[op]
        w = valid if valid > 0 else cols
        if w % 16:
            raise ValueError(f"{op}: row width {w} is not a multiple of 16")
        src = np.asarray(buf_bf16).reshape(rows, cols)
        if kind[0] == "gelu_f32":
            t = self._dev(src, torch.float32)
        else:
            t = self._dev(src, torch.bfloat16)
        if kind[0] in ("gelu", "gelu_f32"):
            oc = out_cols if out_cols > 0 else cols
            out = torch.zeros(rows, oc, dtype=torch.bfloat16, device=self.device)
            ops.gelu_poly4(t, out=out[:, :cols], rounding=kind[1])
        elif kind[0] == "softmax":
            out = torch.zeros(rows, cols, dtype=torch.bfloat16, device=self.device)
            ops.softmax_rows(t, out=out, valid=valid, variant=kind[1], rounding=kind[2])
        else:
            out = ops.layer_norm_rows(t, mode=L.WX_LN_AIE, rounding=kind[1])
        self.calls += 1
        return out.cpu().view(torch.uint16).numpy().view(ml_dtypes.bfloat16)

    # ---------------------------------------------------------------- encoder
    def encoder_engine(self, W, n_layer=None, n_head=None, max_batch=1, gelu=None):
        """The device-resident encoder for weight dict W, built once per W and
        rebuilt when an array of W has been replaced by another object. Arrays
        are taken as immutable, as register_weights takes them (src/rawxrt.py:
        307-316): one changed in place keeps its engine."""
        gelu = gelu or self.gelu_mode
        key = (id(W), n_layer, n_head, gelu)
        arrays = [(k, v) for k, v in sorted(W.items()) if k.startswith("w.")]
        ids = tuple((k, id(v)) for k, v in arrays)
        hit = self._engines.get(key)
        eng = hit[2] if hit is not None and hit[0] == ids else None
        if eng is None or eng.max_batch < max_batch:
            # a replaced engine is freed by Encoder.__del__ once no caller holds it
            eng = Encoder(W, n_layer=n_layer, n_head=n_head, max_batch=max_batch, gelu=gelu,
                          device=self.device.index)
            # the arrays are held so that their ids cannot be reused by new ones
            self._engines[key] = (ids, [v for _, v in arrays], eng)
            self._keep.append(W)
        return eng


_DEFAULT = None


def default_runtime():
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = B200RT()
    return _DEFAULT
