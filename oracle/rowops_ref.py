"""CPU oracle for the row ops of the Whisper-encoder hot path (test infrastructure).

This module is TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py may import it, and only as the checker. The product
path (whisper-xdna_b200/) never imports it and has no CPU fallback.

It restates, in numpy, the arithmetic of the reference's AIE2 row kernels with
every bf16 rounding point explicit:

  * GELU poly4        kernels/gelu_poly4_eval.inc:27-65, coefficients
                      kernels/gelu_poly4_coeffs.h:4-13; entry points
                      gelu_row4.cc:44-61 (g4, truncating), gelu_row4_rne.cc:44-66
                      (g4r, RNE) and gelu_row4f.cc:58-84 (g4f, fp32 in, RNE).
  * row softmax v4    kernels/softmax_row4_body.inc:17-60, RNE twin
                      softmax_row4_rne.cc:41-49, window src/rowops.py:60-73;
                      v1 softmax_row.cc:25-59 and v3 softmax_row3.cc:34-86.
  * LayerNorm         kernels/layer_norm_gb.cc:22-85 (device form) and
                      src/npu_whisper_encoder.py:278-281 (host form, gamma/beta).

Rounding model (the AIE2 vector unit): every bf16 vector result is an fp32
value converted to bf16 with the kernel's rounding mode -- truncation toward
zero by default (the reference's comments at gelu_row4_rne.cc:45-48 and
softmax_row4_rne.cc:43-46), round-to-nearest-even after
aie::set_rounding(conv_even). bf16 x bf16 products are exact in fp32. Scalar
casts follow the same mode. fp32 adds round to nearest even.

Summation order: the AIE kernels accumulate 16 fp32 lanes, lane l taking
elements l, l+16, l+32, ... in order, then reduce the 16 lanes. The lane order
is the reference's; the 16->1 reduction (aie::reduce_add) is external and its
tree is not published, so the oracle fixes a halving tree
((l, l+8) -> (l, l+4) -> (l, l+2) -> (l, l+1)) and the CUDA kernels use the
same one. getExpBf16 (an external lookup table in MLIR-AIE) is restated as the
exact exponential rounded to fp32, then to bf16; aie::inv as the IEEE fp32
reciprocal. Those two are the only places where this oracle and the real NPU
may differ by 1 bf16 ulp.
"""
import numpy as np

TRUNC = 0   # AIE2 default: truncate toward zero
RNE = 1     # aie::set_rounding(aie::rounding_mode::conv_even)

# kernels/gelu_poly4_coeffs.h:6-13 -- the constant table the kernels consume.
GELU4_BREAK = np.array([1.0, 2.0, 4.0], np.float32)
GELU4_SHIFT = np.array([0.5, 1.5, 3.0], np.float32)
GELU4_SCALE = np.array([2.0, 2.0, 1.0], np.float32)
GELU4_COEF = np.array([
    [-0.0020446777, -0.013000488, 0.077148438, -0.06640625, -0.15429688],
    [0.0021514893, -0.0071716309, -0.0040283203, 0.063964844, -0.10009766],
    [-0.0029296875, 0.010681152, -0.015869141, 0.012023926, -0.0040283203],
], np.float32)


# ------------------------------------------------------------------ bf16 helpers

def bf16_bits(x, mode):
    """fp32 -> bf16 bit pattern (uint16) with the given rounding mode."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    if mode == TRUNC:
        out = (u >> 16).astype(np.uint16)
    else:
        bias = ((u >> 16) & 1) + np.uint32(0x7FFF)
        out = ((u.astype(np.uint64) + bias) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, ((u >> 16) | 0x0040).astype(np.uint16), out)
    return out


def bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rbf(x, mode):
    """Round fp32 values to bf16-representable fp32 values."""
    return bits_to_f32(bf16_bits(np.asarray(x, np.float32), mode))


def f32(x):
    return np.asarray(x, np.float32)


# ------------------------------------------------------------------ GELU poly4

def gelu_poly4(x, mode=RNE):
    """gelu_poly4_eval (kernels/gelu_poly4_eval.inc:27-65) on bf16 inputs.

    x: float32 array holding bf16-representable values. Returns float32 array of
    bf16-representable values.
    """
    x = f32(x)
    # every table entry is cast (bfloat16)float at its point of use (:43-45,
    # :52, :55, :60), which rounds with the kernel's mode
    coef, shift, scale, brk = (rbf(GELU4_COEF, mode), rbf(GELU4_SHIFT, mode),
                               rbf(GELU4_SCALE, mode), rbf(GELU4_BREAK, mode))
    zero = np.float32(0.0)
    with np.errstate(all="ignore"):
        s = np.maximum(x, zero - x)                    # :33  s = max(x, 0 - x)
        q = np.zeros_like(x)                           # :39
        for p in range(2, -1, -1):                     # :40  outer piece first
            t = rbf(s - shift[p], mode)                # :43  bf16 sub
            u = rbf(t * scale[p], mode)                # :42-46 bf16 mul -> bf16
            acc = np.full_like(x, coef[p, 0])          # :51  c0 * 1
            for k in range(1, 5):                      # :53-58 Horner, fp32 MAC
                ah = rbf(acc, mode)
                acc = f32(coef[p, k] + ah * u)         # product exact, one add
            inside = s < brk[p]                        # :59-60
            q = np.where(inside, rbf(acc, mode), q)    # :61  tightest piece wins
        return rbf(np.maximum(x, zero) + q, mode)      # :64  relu(x) + q


def gelu_row4(x_bf16):
    """g4: bf16 in/out, truncating (gelu_row4.cc:44-61)."""
    return gelu_poly4(x_bf16, TRUNC)


def gelu_row4_rne(x_bf16):
    """g4r: bf16 in/out, RNE (gelu_row4_rne.cc:44-66)."""
    return gelu_poly4(x_bf16, RNE)


def gelu_row4f(x_f32):
    """g4f: fp32 in, rounded to bf16 RNE first, bf16 out (gelu_row4f.cc:58-84)."""
    return gelu_poly4(rbf(x_f32, RNE), RNE)


def gelu_erf_exact(x):
    """The function the polynomial approximates: exact erf-GELU (float64)."""
    from math import erf, sqrt
    v = np.vectorize(lambda t: 0.5 * t * (1.0 + erf(t / sqrt(2.0))))
    return v(np.asarray(x, np.float64))


# ------------------------------------------------------------------ lane sums

def lane_sum16(a):
    """Sum each row the AIE way: 16 fp32 lanes, lane l accumulating elements
    l, l+16, ... in order, then the fixed halving tree. a: (rows, w) fp32."""
    a = f32(a)
    rows, w = a.shape
    wp = (w + 15) // 16 * 16
    if wp != w:
        a = np.concatenate([a, np.zeros((rows, wp - w), np.float32)], axis=1)
    a = a.reshape(rows, wp // 16, 16)
    acc = np.zeros((rows, 16), np.float32)
    for i in range(wp // 16):
        acc = f32(acc + a[:, i, :])
    acc = f32(acc[:, :8] + acc[:, 8:])
    acc = f32(acc[:, :4] + acc[:, 4:])
    acc = f32(acc[:, :2] + acc[:, 2:])
    return f32(acc[:, 0] + acc[:, 1])


# ------------------------------------------------------------------ softmax

SOFTMAX_MAX_INIT = np.float32(-29952.0)   # (bfloat16)-30000.0f, body.inc:23


def _exp_f32(xp):
    """getExpBf16's value before its bf16 conversion: exp rounded to fp32."""
    return np.exp(np.asarray(xp, np.float64)).astype(np.float32)


def softmax_row(x, mode=TRUNC, variant=4, scale=1.0, valid=0):
    """Row softmax over the first `valid` columns (all if 0) of bf16 rows.

    variant 4: kernels/softmax_row4_body.inc:17-60 (v4, the chain's s4w);
    variant 1: kernels/softmax_row.cc:25-59 (bf16 reciprocal);
    variant 3: kernels/softmax_row3.cc:34-86 (exp and reciprocal split hi/lo).
    scale != 1 multiplies the bf16 input by `scale` first, rounding to bf16 (the
    build's addition: the reference kernel has no scale argument).
    Returns the window's probabilities as bf16-representable fp32 (rows, w).
    """
    x = f32(x)
    w = x.shape[1] if valid <= 0 else valid
    x = x[:, :w]
    if scale != 1.0:
        x = rbf(x * np.float32(scale), mode)
    rmax = np.maximum(x.max(axis=1), SOFTMAX_MAX_INIT)[:, None]    # pass 1
    xs = rbf(x - rmax, mode)                                       # aie::sub
    ea = _exp_f32(xs)
    e = rbf(ea, mode)                                              # pass 2
    s = lane_sum16(e)
    inv = f32(np.float32(1.0) / s)                                 # aie::inv
    if variant == 1:
        ib = rbf(inv, mode)[:, None]
        return rbf(e * ib, mode)
    ihi = rbf(inv, mode)
    ilo = rbf(f32(inv - ihi), mode)
    ihi, ilo = ihi[:, None], ilo[:, None]
    if variant == 4:
        return rbf(f32(e * ihi) + f32(e * ilo), mode)              # pass 3
    if variant == 3:
        ehi = rbf(ea, mode)
        elo = rbf(f32(ea - ehi), mode)
        p = f32(ehi * ihi)
        p = f32(p + f32(ehi * ilo))
        p = f32(p + f32(elo * ihi))
        return rbf(p, mode)
    raise ValueError(f"unknown softmax variant {variant}")


def softmax_exp_table(mode):
    """e = R(exp(x')) for every bf16 x' in [-128, 0] (bit patterns 0x8000 up to
    0xC300, exclusive), as uint16 bf16 bits; the kernels index it by x' bits."""
    bits = np.arange(0x8000, 0xC300, dtype=np.uint32).astype(np.uint16)
    return bf16_bits(_exp_f32(bits_to_f32(bits)), mode)


def softmax_exp_table_f32():
    bits = np.arange(0x8000, 0xC300, dtype=np.uint32).astype(np.uint16)
    return _exp_f32(bits_to_f32(bits))


def softmax_fp32(x):
    """Plain fp32 softmax (src/npu_whisper_encoder.py:416-419)."""
    x = np.asarray(x, np.float32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


# ------------------------------------------------------------------ LayerNorm

def rsqrt_nr(x):
    """kernels/layer_norm_gb.cc:22-34: bit-trick seed + 3 Newton steps, every
    fp32 operation rounded on its own (no fused multiply-add)."""
    x = f32(x)
    i = np.uint32(0x5F3759DF) - (x.view(np.uint32) >> np.uint32(1))
    y = i.astype(np.uint32).view(np.float32)
    half = np.float32(0.5)
    th = np.float32(1.5)
    for _ in range(3):
        t = f32(f32(f32(half * x) * y) * y)
        y = f32(y * f32(th - t))
    return y


def layer_norm_aie(x, mode=TRUNC, gamma=None, beta=None, eps=1e-5):
    """The device LayerNorm of kernels/layer_norm_gb.cc:48-86 on bf16 rows.

    sum and sum of squares in 16 fp32 lanes (:56-67), var = E[x^2] - mean^2
    (:69-71), inv_std = rsqrt_nr(var + eps) (:72), mean and inv_std rounded to
    bf16 (:74-77), out = R(R(x - mean) * inv) (:80-85). The reference kernel has
    no affine; when gamma/beta are given (the build's extension) the result is
    R(out * gamma + beta) with gamma, beta in fp32 and two separate roundings.
    """
    x = f32(x)
    rows, cols = x.shape
    s1 = lane_sum16(x)
    s2 = lane_sum16(f32(x * x))
    inv_n = f32(np.float32(1.0) / np.float32(cols))
    mean = f32(s1 * inv_n)
    var = f32(f32(s2 * inv_n) - f32(mean * mean))
    inv = rsqrt_nr(f32(var + np.float32(eps)))
    mb = rbf(mean, mode)[:, None]
    ib = rbf(inv, mode)[:, None]
    o = rbf(rbf(x - mb, mode) * ib, mode)
    if gamma is not None or beta is not None:
        g = f32(np.ones(cols) if gamma is None else gamma)[None, :]
        b = f32(np.zeros(cols) if beta is None else beta)[None, :]
        o = rbf(f32(f32(o * g) + b), mode)
    return o


def layer_norm_host(x, w, b, eps=1e-5):
    """src/npu_whisper_encoder.py:278-281 verbatim in fp32."""
    x = np.asarray(x, np.float32)
    mu = x.mean(axis=-1, keepdims=True)
    v = x.var(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(v + eps) * w + b
