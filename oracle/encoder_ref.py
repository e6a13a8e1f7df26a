"""CPU oracle for the Whisper encoder forward (test infrastructure).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, never by the product path.

Two restatements of one function:

  * encoder_np     -- the reference's own CPU path, `encoder(W, mel, np_matmul,
                      np_matmul, ...)` of src/npu_whisper_encoder.py:436-541 with
                      the host attention (:491-511), fp32 softmax (:416-419),
                      exact-erf GELU via A&S 7.1.26 (:284-300), host LayerNorm
                      (:278-281) and im2col (:422-431). Pinned against outputs of
                      the reference itself (tests/golden/encoder_np_*.npz, made by
                      tests/golden/make_golden.py).
  * encoder_torch  -- a torch fp32 CPU restatement written from the Whisper
                      encoder architecture (conv1 k3 s1 p1 + GELU, conv2 k3 s2 p1
                      + GELU, + positions, pre-LN blocks, attention with q and k
                      each scaled by hd**-0.25, GELU MLP, ln_post). This is the
                      "torch fp32 CPU encoder" the tolerances are quoted against.

Weights follow the reference's dict layout: "w.<torch state_dict key>" fp32
arrays, Linear weights (out, in), pre-transposed copies under "...weight_T"
(src/npu_whisper_encoder.py:563-566).

Synthetic inputs (no checkpoint or audio can be fetched here): weights and
biases ~ N(0, 0.02) rounded to bf16, LayerNorm gamma = 1 and beta = 0,
sinusoidal positions, log-mel ~ U[-0.8, 1.2]; the recipe of
bench/run_raw_block.py:71-92 and the build's BASELINE configs.
"""
import math

import numpy as np

from rowops_ref import rbf, RNE

GEOMETRY = {
    # name: (n_mels, d_model, n_head, n_layer, ffn)
    "tiny": (80, 384, 6, 4, 1536),
    "base": (80, 512, 8, 6, 2048),
    "small": (80, 768, 12, 12, 3072),
    "medium": (80, 1024, 16, 24, 4096),
    "large-v3": (128, 1280, 20, 32, 5120),
}


# ------------------------------------------------------------------ inputs

def sinusoids(length, channels, max_timescale=10000):
    """Whisper's sinusoidal positional embedding (sin half, then cos half)."""
    assert channels % 2 == 0
    log_inc = np.log(max_timescale) / (channels // 2 - 1)
    inv = np.exp(-log_inc * np.arange(channels // 2))
    t = np.arange(length)[:, None] * inv[None, :]
    return np.concatenate([np.sin(t), np.cos(t)], axis=1).astype(np.float32)


def _normal(seed, tag, shape, std=0.02):
    rng = np.random.default_rng([seed] + list(tag))
    return rbf(rng.normal(0.0, std, size=shape).astype(np.float32), RNE)


def make_weights(geom="tiny", seed=1, n_layer=None, n_ctx=1500,
                 ln_random=False):
    """Synthetic encoder weights in the reference's W-dict layout.

    Every tensor has its own stream (seed, layer, slot), so the first L layers
    do not depend on how many layers are generated. ln_random=True draws LN
    gamma ~ 1 + N(0, 0.1) and beta ~ N(0, 0.1) instead of 1 / 0.
    """
    n_mels, d, nh, nl, ffn = GEOMETRY[geom] if isinstance(geom, str) else geom
    nl = nl if n_layer is None else n_layer
    W = {}
    W["w.conv1.weight"] = _normal(seed, (1000, 0), (d, n_mels, 3))
    W["w.conv1.bias"] = _normal(seed, (1000, 1), (d,))
    W["w.conv2.weight"] = _normal(seed, (1000, 2), (d, d, 3))
    W["w.conv2.bias"] = _normal(seed, (1000, 3), (d,))
    W["w.positional_embedding"] = sinusoids(n_ctx, d)

    def ln(tag):
        if ln_random:
            g = rbf(1.0 + _normal(seed, tag + (0,), (d,), 0.1), RNE)
            b = _normal(seed, tag + (1,), (d,), 0.1)
        else:
            g, b = np.ones(d, np.float32), np.zeros(d, np.float32)
        return g, b

    for L in range(nl):
        p = f"w.blocks.{L}."
        W[p + "attn_ln.weight"], W[p + "attn_ln.bias"] = ln((L, 0))
        W[p + "attn.query.weight"] = _normal(seed, (L, 1), (d, d))
        W[p + "attn.query.bias"] = _normal(seed, (L, 2), (d,))
        W[p + "attn.key.weight"] = _normal(seed, (L, 3), (d, d))
        W[p + "attn.value.weight"] = _normal(seed, (L, 4), (d, d))
        W[p + "attn.value.bias"] = _normal(seed, (L, 5), (d,))
        W[p + "attn.out.weight"] = _normal(seed, (L, 6), (d, d))
        W[p + "attn.out.bias"] = _normal(seed, (L, 7), (d,))
        W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"] = ln((L, 8))
        W[p + "mlp.0.weight"] = _normal(seed, (L, 9), (ffn, d))
        W[p + "mlp.0.bias"] = _normal(seed, (L, 10), (ffn,))
        W[p + "mlp.2.weight"] = _normal(seed, (L, 11), (d, ffn))
        W[p + "mlp.2.bias"] = _normal(seed, (L, 12), (d,))
    W["w.ln_post.weight"], W["w.ln_post.bias"] = ln((2000, 0))
    return W


def add_transposed(W):
    """Pre-transpose every Linear weight once (src/npu_whisper_encoder.py:563-566)."""
    for k in [k for k in W if k.endswith(".weight") and W[k].ndim == 2
              and not k.endswith("_ln.weight")]:
        W[k[:-len("weight")] + "weight_T"] = np.ascontiguousarray(W[k].T)
    return W


def make_mel(n_mels=80, frames=3000, seed=0):
    rng = np.random.default_rng(seed)
    return rng.uniform(-0.8, 1.2, size=(n_mels, frames)).astype(np.float32)


def geometry_of(W):
    """Read (n_layer, n_head) off the weights (src/npu_whisper_encoder.py:571-572)."""
    n_layer = 1 + max(int(k.split(".")[2]) for k in W if k.startswith("w.blocks."))
    n_head = W["w.ln_post.weight"].shape[0] // 64
    return n_layer, n_head


# ------------------------------------------------------------------ numpy path

def _erf(x):
    """Abramowitz-Stegun 7.1.26, as src/npu_whisper_encoder.py:290-300 uses."""
    a1, a2, a3, a4, a5, p = (0.254829592, -0.284496736, 1.421413741,
                             -1.453152027, 1.061405429, 0.3275911)
    sign = np.sign(x)
    ax = np.abs(x)
    t = 1.0 / (1.0 + p * ax)
    y = 1.0 - (((((a5 * t + a4) * t) + a3) * t + a2) * t + a1) * t * np.exp(-ax * ax)
    return sign * y


def gelu_np(x):
    """src/npu_whisper_encoder.py:284-287. The divisor is a Python float
    (math.sqrt there), so float32 input stays float32 as in the reference."""
    return 0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))


def layer_norm_np(x, w, b, eps=1e-5):
    mu = x.mean(axis=-1, keepdims=True)
    v = x.var(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(v + eps) * w + b


def softmax_np(x):
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def im2col(x, kernel, stride, pad):
    """x (C, T) -> (T_out, C*kernel), column c*kernel + j = x[c, t*stride + j - pad]
    (src/npu_whisper_encoder.py:422-431)."""
    C, T = x.shape
    xp = np.zeros((C, T + 2 * pad), dtype=x.dtype)
    xp[:, pad:pad + T] = x
    T_out = (T + 2 * pad - kernel) // stride + 1
    cols = np.empty((T_out, C * kernel), dtype=x.dtype)
    for j in range(kernel):
        cols[:, j::kernel] = xp[:, j:j + (T_out - 1) * stride + 1:stride].T
    return cols


def mm(A, B):
    return A.astype(np.float32) @ B.astype(np.float32)


def encoder_np(W, mel, n_layer=None, n_head=None):
    """The reference's numpy encoder (src/npu_whisper_encoder.py:436-541 with
    mm = attn_mm = np_matmul, fold_bias=True, host attention)."""
    if n_layer is None or n_head is None:
        nl, nh = geometry_of(W)
        n_layer = nl if n_layer is None else n_layer
        n_head = nh if n_head is None else n_head
    c1w = W["w.conv1.weight"]
    O, C, KS = c1w.shape
    x = mm(im2col(mel, KS, 1, 1), c1w.reshape(O, C * KS).T) + W["w.conv1.bias"]
    x = gelu_np(x)
    c2w = W["w.conv2.weight"]
    O2, C2, KS2 = c2w.shape
    x = mm(im2col(np.ascontiguousarray(x.T), KS2, 2, 1),
           c2w.reshape(O2, C2 * KS2).T) + W["w.conv2.bias"]
    x = gelu_np(x)
    x = x + W["w.positional_embedding"][:x.shape[0]]
    ctx, d = x.shape
    hd = d // n_head
    scale = hd ** -0.25
    for L in range(n_layer):
        p = f"w.blocks.{L}."
        h = layer_norm_np(x, W[p + "attn_ln.weight"], W[p + "attn_ln.bias"])
        q = mm(h, W[p + "attn.query.weight"].T) + W[p + "attn.query.bias"]
        k = mm(h, W[p + "attn.key.weight"].T)
        v = mm(h, W[p + "attn.value.weight"].T) + W[p + "attn.value.bias"]
        o = np.empty_like(q)
        for hh in range(n_head):
            sl = slice(hh * hd, (hh + 1) * hd)
            s = mm(np.ascontiguousarray(q[:, sl] * scale),
                   np.ascontiguousarray(k[:, sl].T) * scale)
            o[:, sl] = mm(softmax_np(s), np.ascontiguousarray(v[:, sl]))
        x = x + (mm(o, W[p + "attn.out.weight"].T) + W[p + "attn.out.bias"])
        h = layer_norm_np(x, W[p + "mlp_ln.weight"], W[p + "mlp_ln.bias"])
        f = gelu_np(mm(h, W[p + "mlp.0.weight"].T) + W[p + "mlp.0.bias"])
        x = x + mm(f, W[p + "mlp.2.weight"].T) + W[p + "mlp.2.bias"]
    return layer_norm_np(x, W["w.ln_post.weight"], W["w.ln_post.bias"])


# ------------------------------------------------------------------ torch path

def encoder_torch(W, mel, n_layer=None, n_head=None, threads=None):
    """Torch fp32 CPU Whisper encoder restated from the architecture."""
    import torch
    import torch.nn.functional as F
    if threads:
        torch.set_num_threads(threads)
    if n_layer is None or n_head is None:
        nl, nh = geometry_of(W)
        n_layer = nl if n_layer is None else n_layer
        n_head = nh if n_head is None else n_head
    t = lambda k: torch.from_numpy(np.ascontiguousarray(W[k], np.float32))
    with torch.no_grad():
        x = torch.from_numpy(np.ascontiguousarray(mel, np.float32))[None]
        x = F.gelu(F.conv1d(x, t("w.conv1.weight"), t("w.conv1.bias"), padding=1))
        x = F.gelu(F.conv1d(x, t("w.conv2.weight"), t("w.conv2.bias"),
                            stride=2, padding=1))
        x = x.permute(0, 2, 1)[0]
        T, d = x.shape
        x = x + t("w.positional_embedding")[:T]
        hd = d // n_head
        s = hd ** -0.25
        for L in range(n_layer):
            p = f"w.blocks.{L}."
            h = F.layer_norm(x, (d,), t(p + "attn_ln.weight"), t(p + "attn_ln.bias"))
            q = F.linear(h, t(p + "attn.query.weight"), t(p + "attn.query.bias"))
            k = F.linear(h, t(p + "attn.key.weight"))
            v = F.linear(h, t(p + "attn.value.weight"), t(p + "attn.value.bias"))
            q = q.view(T, n_head, hd).permute(1, 0, 2) * s
            k = k.view(T, n_head, hd).permute(1, 2, 0) * s
            v = v.view(T, n_head, hd).permute(1, 0, 2)
            a = torch.softmax(q @ k, dim=-1) @ v
            o = a.permute(1, 0, 2).reshape(T, d)
            x = x + F.linear(o, t(p + "attn.out.weight"), t(p + "attn.out.bias"))
            h = F.layer_norm(x, (d,), t(p + "mlp_ln.weight"), t(p + "mlp_ln.bias"))
            f = F.gelu(F.linear(h, t(p + "mlp.0.weight"), t(p + "mlp.0.bias")))
            x = x + F.linear(f, t(p + "mlp.2.weight"), t(p + "mlp.2.bias"))
        x = F.layer_norm(x, (d,), t("w.ln_post.weight"), t("w.ln_post.bias"))
    return x.numpy()


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))
