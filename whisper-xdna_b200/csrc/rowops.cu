// Row ops of the Whisper-encoder hot path as bandwidth-bound sm_100a kernels:
// polynomial GELU (g4 / g4r / g4f), row softmax (v1 / v3 / v4, windowed, with
// an optional input scale) and LayerNorm (the reference's device arithmetic,
// and the fp32 host form the encoder uses).
//
// The bf16 rounding points, the 16-lane summation order and the constant
// tables follow the reference's AIE2 kernels exactly, so the RNE variants are
// bit-exact to the CPU restatement:
//   GELU     kernels/gelu_poly4_eval.inc:27-65, kernels/gelu_poly4_coeffs.h:6-13
//   softmax  kernels/softmax_row4_body.inc:17-60, softmax_row.cc:25-59,
//            softmax_row3.cc:34-86, windowing src/rowops.py:60-73
//   LN       kernels/layer_norm_gb.cc:22-85
// Memory access: 16-byte vector loads and stores, rows staged in shared memory
// so HBM is read and written once.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "ln_row.cuh"

namespace wx {

// ---------------------------------------------------------------- host tables
// The reference's GELU table (kernels/gelu_poly4_coeffs.h:6-13), consumed as
// constants: breaks, shifts, scales and the degree-4 coefficients of each of
// the three pieces, highest degree first.
static const float kGeluBreak[3] = {1.000000f, 2.000000f, 4.000000f};
static const float kGeluShift[3] = {0.500000f, 1.500000f, 3.000000f};
static const float kGeluScale[3] = {2.000000f, 2.000000f, 1.000000f};
static const float kGeluCoef[3][5] = {
    {-0.0020446777f, -0.013000488f, 0.077148438f, -0.06640625f, -0.15429688f},
    {0.0021514893f, -0.0071716309f, -0.0040283203f, 0.063964844f, -0.10009766f},
    {-0.0029296875f, 0.010681152f, -0.015869141f, 0.012023926f, -0.0040283203f},
};

static inline uint32_t h_f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float h_u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
uint16_t host_bf16_bits(float f, int mode) {
  uint32_t u = h_f2u(f);
  if (std::isnan(f)) return (uint16_t)((u >> 16) | 0x40);
  if (mode == RND_TRUNC) return (uint16_t)(u >> 16);
  uint32_t bias = ((u >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)((uint64_t(u) + bias) >> 16);
}
float host_rbf(float f, int mode) { return h_u2f(uint32_t(host_bf16_bits(f, mode)) << 16); }

Gelu4Table gelu4_table(int mode) {
  Gelu4Table t;
  for (int p = 0; p < 3; p++) {
    t.brk[p] = host_rbf(kGeluBreak[p], mode);
    t.shift[p] = host_rbf(kGeluShift[p], mode);
    t.scale[p] = host_rbf(kGeluScale[p], mode);
    for (int k = 0; k < 5; k++) t.c[p][k] = host_rbf(kGeluCoef[p][k], mode);
  }
  return t;
}

// exp of every bf16 x' in [-128, -0]: bit patterns [0x8000, 0xC300). Below -128
// the exponential is 0 in fp32 and bf16; x' = +0 gives 1.
constexpr int kExpTabBase = 0x8000;
constexpr int kExpTabN = 0xC300 - 0x8000;

static void host_exp_tables(uint16_t* t16_trunc, uint16_t* t16_rne, float* t32) {
  for (int i = 0; i < kExpTabN; i++) {
    float x = h_u2f(uint32_t(kExpTabBase + i) << 16);
    float e = (float)std::exp((double)x);
    t32[i] = e;
    t16_trunc[i] = host_bf16_bits(e, RND_TRUNC);
    t16_rne[i] = host_bf16_bits(e, RND_RNE);
  }
}

struct ExpTablesDev {
  uint16_t* t16[2] = {nullptr, nullptr};
  float* t32 = nullptr;
};

static std::mutex g_tab_mu;
static ExpTablesDev g_tabs[64];

static int exp_tables(ExpTablesDev** out) {
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64) return fail(WX_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_tab_mu);
  ExpTablesDev& t = g_tabs[dev];
  if (!t.t32) {
    std::vector<uint16_t> a(kExpTabN), b(kExpTabN);
    std::vector<float> c(kExpTabN);
    host_exp_tables(a.data(), b.data(), c.data());
    WX_CUDA_TRY(cudaMalloc(&t.t16[0], kExpTabN * 2));
    WX_CUDA_TRY(cudaMalloc(&t.t16[1], kExpTabN * 2));
    WX_CUDA_TRY(cudaMalloc(&t.t32, kExpTabN * 4));
    WX_CUDA_TRY(cudaMemcpy(t.t16[0], a.data(), kExpTabN * 2, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(t.t16[1], b.data(), kExpTabN * 2, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(t.t32, c.data(), kExpTabN * 4, cudaMemcpyHostToDevice));
  }
  *out = &t;
  return WX_OK;
}

// ---------------------------------------------------------------- GELU
// Rows are strided over blockIdx.y, VEC-element column groups over
// blockIdx.x and the threads, so no thread divides an index.
template <int R, bool F32IN, int VEC>
__global__ void __launch_bounds__(128) gelu_poly4_kernel(const void* __restrict__ in,
                                                         uint16_t* __restrict__ out,
                                                         int64_t rows, int64_t cols,
                                                         int64_t ld_in, int64_t ld_out) {
  const int64_t per_row = cols / VEC;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i * VEC;
    float x[VEC];
    if (F32IN) {
      const float* src = reinterpret_cast<const float*>(in) + r * ld_in + c;
      if (VEC == 8) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
        x[0] = src[0];
      }
#pragma unroll
      for (int j = 0; j < VEC; j++) x[j] = rbf<R>(x[j]);  // gelu_row4f.cc:78-80
    } else {
      const uint16_t* src = reinterpret_cast<const uint16_t*>(in) + r * ld_in + c;
      if (VEC == 8) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          x[2 * j] = __uint_as_float(w[j] << 16);
          x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      } else {
        x[0] = bits_f32(src[0]);
      }
    }
    uint16_t* dst = out + r * ld_out + c;
    if (VEC == 8 && R == RND_RNE) {   // packed bf16x2 form
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; j++)
        w[j] = gelu_poly4_bf16x2_rne(pack_bf16x2_rne(x[2 * j], x[2 * j + 1]));
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if (VEC == 8) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) gelu_poly4_x2<R>(x[j], x[j + 1]);
      uint4 o;
      o.x = pack_bf16x2<R>(x[0], x[1]);
      o.y = pack_bf16x2<R>(x[2], x[3]);
      o.z = pack_bf16x2<R>(x[4], x[5]);
      o.w = pack_bf16x2<R>(x[6], x[7]);
      *reinterpret_cast<uint4*>(dst) = o;
    } else {
      dst[0] = (uint16_t)bf16_bits<R>(gelu_poly4<R>(x[0]));
    }
  }
}

// ---------------------------------------------------------------- row helpers
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// The 16 lane partial sums of lanes 0..15 reduced by the halving tree
// (l, l+8) -> (l, l+4) -> (l, l+2) -> (l, l+1); every lane of the half gets it.
__device__ __forceinline__ float lane16_tree(float acc) {
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8, 16));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4, 16));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2, 16));
  acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1, 16));
  return acc;
}

// Stage one bf16 row window (w elements) in shared memory, optionally scaled
// (x' = R(x * scale)), and return the row max seeded with `init`.
template <int R>
__device__ __forceinline__ float stage_row(const uint16_t* __restrict__ src, uint16_t* buf, int w,
                                           bool vec, bool do_scale, float scale, float init,
                                           bool want_max) {
  const int lane = lane_id();
  float m = init;
  int done = 0;
  if (vec) {
    const int nv = w / 8;
    for (int v = lane; v < nv; v += 32) {
      uint4 q = __ldg(reinterpret_cast<const uint4*>(src) + v);
      if (do_scale || want_max) {
        uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          float lo = __uint_as_float(wd[j] << 16), hi = __uint_as_float(wd[j] & 0xFFFF0000u);
          if (do_scale) {
            lo = rbf<R>(lo * scale);
            hi = rbf<R>(hi * scale);
            wd[j] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
          }
          if (want_max) m = fmaxf(m, fmaxf(lo, hi));
        }
        q = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
      reinterpret_cast<uint4*>(buf)[v] = q;
    }
    done = nv * 8;
  }
  for (int c = done + lane; c < w; c += 32) {
    float x = bits_f32(src[c]);
    if (do_scale) x = rbf<R>(x * scale);
    buf[c] = (uint16_t)(__float_as_uint(x) >> 16);
    if (want_max) m = fmaxf(m, x);
  }
  return want_max ? warp_max(m) : m;
}

// e = R(exp(R(x - max))) via the table; ea = the fp32 exponential (v3 only).
template <int R, bool NEED32>
__device__ __forceinline__ float exp_lookup(float x, float m, const uint16_t* t16, const float* t32,
                                            float* ea) {
  const float d = rbf<R>(__fsub_rn(x, m));
  const uint32_t b = __float_as_uint(d) >> 16;
  float e, a;
  if (b == 0u) {
    e = 1.0f;
    a = 1.0f;
  } else if (b >= (uint32_t)kExpTabBase && b < (uint32_t)(kExpTabBase + kExpTabN)) {
    e = bits_f32(t16[b - kExpTabBase]);
    a = NEED32 ? t32[b - kExpTabBase] : e;
  } else {
    e = 0.0f;
    a = 0.0f;
  }
  if (NEED32) *ea = a;
  return e;
}

// ---------------------------------------------------------------- softmax
// e = R(exp(R(x - max))) as the table holds it (the correctly rounded fp32
// exponential, then bf16 in mode R), computed on the SFU: exp2(d * log2 e)
// carries a relative error below 2^-17 (argument rounding 2^-18 for |d| <= 87,
// the log2 e constant 2^-18, ex2.approx 2^-22), i.e. under 64 fp32 ulps, so
// wherever the approximate value lies more than 1024 ulps from a bf16
// rounding boundary it rounds to the same bf16 as the exact one. Near a
// boundary, below -87 (subnormal results) or at d = 0 the table decides.
template <int R>
__device__ __forceinline__ uint32_t exp_bits_checked(float x, float m, const uint16_t* t16) {
  constexpr uint32_t kMargin = 1024;
  const float d = rbf<R>(__fsub_rn(x, m));
  const uint32_t b = __float_as_uint(d) >> 16;
  if (d > -87.0f && b != 0u && b != 0x8000u) {
    const float e = fast_exp2(__fmul_rn(d, 1.44269504f));
    const uint32_t lo = __float_as_uint(e) & 0xFFFFu;
    const bool near = (R == RND_RNE) ? (lo + kMargin - 0x8000u <= 2 * kMargin)
                                     : (lo <= kMargin || lo >= 0x10000u - kMargin);
    if (!near) return bf16_bits<R>(e);
  }
  if (b == 0u || b == 0x8000u) return 0x3F80u;  // exp(0) = 1
  if (b >= (uint32_t)kExpTabBase && b < (uint32_t)(kExpTabBase + kExpTabN))
    return t16[b - kExpTabBase];
  return 0u;
}

template <int R, int VAR>
__global__ void __launch_bounds__(256) softmax_rows_kernel(
    const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int64_t rows, int w,
    int64_t ld_in, int64_t ld_out, float scale, const uint16_t* __restrict__ t16_g,
    const float* __restrict__ t32_g, int wpad, int vec_in, int vec_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr bool N32 = (VAR == 3);
  uint16_t* t16 = reinterpret_cast<uint16_t*>(smem);
  float* t32 = reinterpret_cast<float*>(smem + ((kExpTabN * 2 + 15) / 16) * 16);
  uint8_t* rows_base = smem + ((kExpTabN * 2 + 15) / 16) * 16 + (N32 ? kExpTabN * 4 : 0);
  for (int i = threadIdx.x; i < kExpTabN; i += blockDim.x) {
    t16[i] = t16_g[i];
    if (N32) t32[i] = t32_g[i];
  }
  __syncthreads();
  const int warps = blockDim.x / 32, warp = warp_id(), lane = lane_id();
  uint16_t* buf = reinterpret_cast<uint16_t*>(rows_base) + (size_t)warp * wpad;
  const bool do_scale = scale != 1.0f;
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows;
       row += (int64_t)gridDim.x * warps) {
    // pass 1: stage the window, row max seeded with (bfloat16)-30000 (body.inc:22-28)
    const float m = stage_row<R>(in + row * ld_in, buf, w, vec_in, do_scale, scale, -29952.0f, true);
    __syncwarp();
    if (VAR != 3) {
      // the exponentials, once, in place of the staged inputs (all 32 lanes)
      const int nv = (w % 8 == 0) ? w / 8 : 0;
      for (int v = lane; v < nv; v += 32) {
        uint4 q = reinterpret_cast<const uint4*>(buf)[v];
        uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; j++)
          wd[j] = exp_bits_checked<R>(__uint_as_float(wd[j] << 16), m, t16) |
                  (exp_bits_checked<R>(__uint_as_float(wd[j] & 0xFFFF0000u), m, t16) << 16);
        reinterpret_cast<uint4*>(buf)[v] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
      for (int c = nv * 8 + lane; c < w; c += 32)
        buf[c] = (uint16_t)exp_bits_checked<R>(bits_f32(buf[c]), m, t16);
      __syncwarp();
    }
    // pass 2: 16 fp32 lanes, lane l summing e over columns l, l+16, ... (body.inc:31-40)
    float acc = 0.0f;
    if (lane < 16) {
      for (int c = lane; c < w; c += 16) {
        float e;
        if (VAR != 3) {
          e = bits_f32(buf[c]);
        } else {
          float ea;
          e = exp_lookup<R, false>(bits_f32(buf[c]), m, t16, t32, &ea);
        }
        acc = __fadd_rn(acc, e);
      }
    }
    const float sum = __shfl_sync(0xffffffffu, lane16_tree(acc), 0);
    const float inv = __fdiv_rn(1.0f, sum);                 // aie::inv
    const float ihi = rbf<R>(inv);                          // body.inc:45-46
    const float ilo = rbf<R>(__fsub_rn(inv, ihi));
    // pass 3: p = R(e*hi + e*lo) (body.inc:51-60), or the v1 / v3 forms
    auto prob = [&](float x) -> float {
      float ea = 0.0f, e;
      if (VAR != 3) e = x;  // buf already holds e
      else e = exp_lookup<R, N32>(x, m, t16, t32, &ea);
      if (VAR == 1) return rbf<R>(__fmul_rn(e, ihi));       // softmax_row.cc:50-57
      if (VAR == 3) {                                       // softmax_row3.cc:76-84
        const float ehi = rbf<R>(ea);
        const float elo = rbf<R>(__fsub_rn(ea, ehi));
        float p = __fmul_rn(ehi, ihi);
        p = __fadd_rn(p, __fmul_rn(ehi, ilo));
        p = __fadd_rn(p, __fmul_rn(elo, ihi));
        return rbf<R>(p);
      }
      return rbf<R>(__fadd_rn(__fmul_rn(e, ihi), __fmul_rn(e, ilo)));
    };
    uint16_t* dst = out + row * ld_out;
    int done = 0;
    if (vec_out) {
      const int nv = w / 8;
      for (int v = lane; v < nv; v += 32) {
        const uint4 q = reinterpret_cast<const uint4*>(buf)[v];
        const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          o[j] = pack_bf16x2<R>(prob(__uint_as_float(wd[j] << 16)),
                                prob(__uint_as_float(wd[j] & 0xFFFF0000u)));
        reinterpret_cast<uint4*>(dst)[v] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      done = nv * 8;
    }
    for (int c = done + lane; c < w; c += 32) dst[c] = (uint16_t)bf16_bits<R>(prob(bits_f32(buf[c])));
    __syncwarp();
  }
}

// The v1 / v4 forms for windows of up to 256 * NV - 7 columns: each warp holds
// its row in registers as NV 16-byte chunks per lane (chunk v = lane + 32k),
// read from the row start rounded down to 16 bytes, so any bf16 row layout
// (e.g. 1500 columns, rows alternately 0 and 8 bytes off a 16-byte boundary)
// reads and writes HBM once with 16-byte accesses; elements outside the
// window in the edge chunks are masked to -inf and never written. The
// exponentials go to shared memory in that chunk layout for the 16-lane
// summation and are read back from there for the output. Values stay packed
// as bf16 pairs: the max is a bf16x2 max (exact), x' - max in RNE mode a
// bf16x2 subtraction, whose correctly rounded result equals the fp32
// difference rounded to bf16 (fp32 carries more than 2 * 8 + 2 significand
// bits, so the double rounding is innocuous). The exponential is the bf16
// table in shared memory, indexed without branches: x' <= max, so d <= 0 and
// its magnitude bits are the table index; d <= -128, and NaN, clamp to a
// trailing zero entry.
constexpr int kSmRegThreads = 512;
constexpr int kExpTabBytes = ((kExpTabN + 1) * 2 + 15) / 16 * 16;

__device__ __forceinline__ int chunk_head(const void* p) {
  return (int)((reinterpret_cast<uintptr_t>(p) & 15) >> 1);
}

template <int R, int VAR, int NV>
__global__ void __launch_bounds__(kSmRegThreads, 2) softmax_rows_reg_kernel(
    const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int64_t rows, int w,
    int64_t ld_in, int64_t ld_out, float scale, const uint16_t* __restrict__ t16_g) {
  extern __shared__ __align__(16) uint8_t smem[];
  for (int i = threadIdx.x; i < kExpTabN / 8; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = __ldg(reinterpret_cast<const uint4*>(t16_g) + i);
  if (threadIdx.x == 0) reinterpret_cast<uint16_t*>(smem)[kExpTabN] = 0;
  __syncthreads();
  const uint8_t* tab = smem;
  const int warps = blockDim.x >> 5, warp = warp_id(), lane = lane_id();
  uint4* buf = reinterpret_cast<uint4*>(smem + kExpTabBytes) + (size_t)warp * (NV * 32);
  const uint16_t* buf16 = reinterpret_cast<const uint16_t*>(buf);
  const bool do_scale = scale != 1.0f;
  // In RNE mode with a bf16 scale (1/8 for attention scores), R(x * scale) is
  // one bf16x2 multiply: the fp32 product of two bf16 values is exact, and the
  // bf16x2 instruction rounds that exact product once, to nearest even.
  const bool scale_bf16x2 = R == RND_RNE && do_scale && rbf<RND_RNE>(scale) == scale;
  const __nv_bfloat162 scale2 = __float2bfloat162_rn(scale);
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows;
       row += (int64_t)gridDim.x * warps) {
    const uint16_t* src_row = in + row * ld_in;
    const int h = chunk_head(src_row);  // elements before column 0 in chunk 0
    const int nch = (w + h + 7) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(src_row - h);
    uint32_t x[NV * 4];
#pragma unroll
    for (int k = 0; k < NV; k++) {
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      if (lane + 32 * k < nch) q = __ldg(src + lane + 32 * k);
      x[4 * k] = q.x; x[4 * k + 1] = q.y; x[4 * k + 2] = q.z; x[4 * k + 3] = q.w;
    }
    // x' = R(x * scale); elements outside [0, w) become -inf
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int c0 = 8 * (lane + 32 * k) - h;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint32_t& v = x[4 * k + j];
        if (scale_bf16x2) {
          const __nv_bfloat162 t = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&v), scale2);
          v = *reinterpret_cast<const uint32_t*>(&t);
        } else if (do_scale) {
          v = pack_bf16x2<R>(__fmul_rn(__uint_as_float(v << 16), scale),
                             __fmul_rn(__uint_as_float(v & 0xFFFF0000u), scale));
        }
        if (c0 < 0 || c0 + 8 > w) {
          const int c = c0 + 2 * j;
          if (c < 0 || c >= w) v = (v & 0xFFFF0000u) | 0xFF80u;
          if (c + 1 < 0 || c + 1 >= w) v = (v & 0xFFFFu) | 0xFF800000u;
        }
      }
    }
    // row max seeded with (bfloat16)-30000 (softmax_row4_body.inc:22-28)
    __nv_bfloat162 mx = *reinterpret_cast<const __nv_bfloat162*>(&x[0]);
#pragma unroll
    for (int i = 1; i < NV * 4; i++)
      mx = __hmax2(mx, *reinterpret_cast<const __nv_bfloat162*>(&x[i]));
    const float m = fmaxf(warp_max(fmaxf(__low2float(mx), __high2float(mx))), -29952.0f);
    const __nv_bfloat162 m2 = __float2bfloat162_rn(m);
    // e = R(exp(R(x' - m))), in place of x'
#pragma unroll
    for (int i = 0; i < NV * 4; i++) {
      uint32_t d;
      if (R == RND_RNE) {
        const __nv_bfloat162 t = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&x[i]), m2);
        d = *reinterpret_cast<const uint32_t*>(&t);
      } else {
        d = pack_bf16x2<R>(__fsub_rn(__uint_as_float(x[i] << 16), m),
                           __fsub_rn(__uint_as_float(x[i] & 0xFFFF0000u), m));
      }
      const uint32_t off = (d << 1) & 0xFFFEFFFEu;  // magnitude * 2 in each half
      const uint32_t olo = min(off & 0xFFFFu, (uint32_t)(2 * kExpTabN));
      const uint32_t ohi = min(off >> 16, (uint32_t)(2 * kExpTabN));
      x[i] = (uint32_t)*reinterpret_cast<const uint16_t*>(tab + olo) |
             ((uint32_t)*reinterpret_cast<const uint16_t*>(tab + ohi) << 16);
    }
#pragma unroll
    for (int k = 0; k < NV; k++)
      buf[lane + 32 * k] = make_uint4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
    __syncwarp();
    // 16 fp32 lanes, lane l summing e over columns l, l+16, ... (softmax_row4_body.inc:31-40)
    float acc = 0.0f;
    if (lane < 16) {
#pragma unroll 16
      for (int c = lane; c < w; c += 16) acc = __fadd_rn(acc, bits_f32(buf16[c + h]));
    }
    const float sum = __shfl_sync(0xffffffffu, lane16_tree(acc), 0);
    const float inv = __fdiv_rn(1.0f, sum);                 // aie::inv
    const float ihi = rbf<R>(inv);                          // softmax_row4_body.inc:45-46
    const float ilo = rbf<R>(__fsub_rn(inv, ihi));
    // p = R(e*hi + e*lo) (softmax_row4_body.inc:51-60); v1 is R(e*hi)
    // (softmax_row.cc:50-57). The products are kept as separate roundings: they
    // are exact except in the subnormal range, where an fma could differ.
    uint16_t* dst_row = out + row * ld_out;
    const int ho = chunk_head(dst_row);
    const int ncho = (w + ho + 7) >> 3;
    uint4* dst = reinterpret_cast<uint4*>(dst_row - ho);
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int u = lane + 32 * k;
      if (u < ncho) {
        const int c0 = 8 * u - ho;
        uint32_t e[4];
        if (ho == h) {
          const uint4 q = buf[u];
          e[0] = q.x; e[1] = q.y; e[2] = q.z; e[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int c = c0 + 2 * j;
            const uint32_t lo = (c >= 0 && c < w) ? buf16[c + h] : 0u;
            const uint32_t hi = (c + 1 >= 0 && c + 1 < w) ? buf16[c + 1 + h] : 0u;
            e[j] = lo | (hi << 16);
          }
        }
        // packed fp32 pairs: each product and sum rounded on its own, as above
        uint32_t o[4];
        const float2 ihi2 = make_float2(ihi, ihi), ilo2 = make_float2(ilo, ilo);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 ev = make_float2(__uint_as_float(e[j] << 16),
                                        __uint_as_float(e[j] & 0xFFFF0000u));
          float2 p;
          if (VAR == 1) p = __fmul2_rn(ev, ihi2);
          else p = __fadd2_rn(__fmul2_rn(ev, ihi2), __fmul2_rn(ev, ilo2));
          o[j] = pack_bf16x2<R>(p.x, p.y);
        }
        if (c0 >= 0 && c0 + 8 <= w) {
          dst[u] = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int c = c0 + j;
            if (c >= 0 && c < w) dst_row[c] = (uint16_t)(o[j >> 1] >> (16 * (j & 1)));
          }
        }
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- LayerNorm
// kernels/layer_norm_gb.cc:22-34, every fp32 operation rounded on its own.
__device__ __forceinline__ float rsqrt_nr(float x) {
  float y = __uint_as_float(0x5f3759dfu - (__float_as_uint(x) >> 1));
#pragma unroll
  for (int i = 0; i < 3; i++) {
    const float t = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, x), y), y);
    y = __fmul_rn(y, __fsub_rn(1.5f, t));
  }
  return y;
}

template <int R>
__global__ void __launch_bounds__(256) layernorm_aie_kernel(
    const uint16_t* __restrict__ in, const float* __restrict__ gamma,
    const float* __restrict__ beta, uint16_t* __restrict__ out, int64_t rows, int w,
    int64_t ld_in, int64_t ld_out, float eps, int wpad, int vec_in, int vec_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warps = blockDim.x / 32, warp = warp_id(), lane = lane_id();
  uint16_t* buf = reinterpret_cast<uint16_t*>(smem) + (size_t)warp * wpad;
  const bool affine = gamma != nullptr || beta != nullptr;
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows;
       row += (int64_t)gridDim.x * warps) {
    stage_row<R>(in + row * ld_in, buf, w, vec_in, false, 1.0f, 0.0f, false);
    __syncwarp();
    // pass 1 (:61-67): sum and sum of squares in 16 fp32 lanes
    float s1 = 0.0f, s2 = 0.0f;
    if (lane < 16) {
      for (int c = lane; c < w; c += 16) {
        const float x = bits_f32(buf[c]);
        s1 = __fadd_rn(s1, x);
        s2 = __fadd_rn(s2, __fmul_rn(x, x));
      }
    }
    s1 = __shfl_sync(0xffffffffu, lane16_tree(s1), 0);
    s2 = __shfl_sync(0xffffffffu, lane16_tree(s2), 0);
    const float inv_n = __fdiv_rn(1.0f, (float)w);                       // :69
    const float mean = __fmul_rn(s1, inv_n);                             // :70
    const float var = __fsub_rn(__fmul_rn(s2, inv_n), __fmul_rn(mean, mean));  // :71
    const float inv = rsqrt_nr(__fadd_rn(var, eps));                     // :72
    const float mb = rbf<R>(mean), ib = rbf<R>(inv);                     // :74-77
    auto norm = [&](float x, int c) -> float {                           // :80-85
      float o = rbf<R>(__fmul_rn(rbf<R>(__fsub_rn(x, mb)), ib));
      if (affine) {
        const float g = gamma ? gamma[c] : 1.0f, b = beta ? beta[c] : 0.0f;
        o = rbf<R>(__fadd_rn(__fmul_rn(o, g), b));
      }
      return o;
    };
    uint16_t* dst = out + row * ld_out;
    int done = 0;
    if (vec_out) {
      const int nv = w / 8;
      for (int v = lane; v < nv; v += 32) {
        const uint4 q = reinterpret_cast<const uint4*>(buf)[v];
        const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
          o[j] = pack_bf16x2<R>(norm(__uint_as_float(wd[j] << 16), v * 8 + 2 * j),
                                norm(__uint_as_float(wd[j] & 0xFFFF0000u), v * 8 + 2 * j + 1));
        reinterpret_cast<uint4*>(dst)[v] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      done = nv * 8;
    }
    for (int c = done + lane; c < w; c += 32) dst[c] = (uint16_t)bf16_bits<R>(norm(bits_f32(buf[c]), c));
    __syncwarp();
  }
}

// The same arithmetic for rows of up to 256 * NV - 7 columns, one warp per
// row, arranged for latency (a 1500-row call has about ten rows per SM, so a
// row's own critical path is the kernel's time):
//  - the row is read as 16-byte chunks from its start rounded down to 16
//    bytes (the softmax_rows_reg_kernel layout) into registers, with all of
//    its loads in flight together and issued before gamma / beta are staged;
//  - the reference's 16 lane sums (lane l adds columns l, l+16, ... in order,
//    layer_norm_gb.cc:61-67) run from registers: each lane scatters its
//    elements into a lane-transposed copy in shared memory, t[l][k] =
//    x[l + 16k], whose row stride (8m + 4 elements) makes the 8-byte reads of
//    the 16 summing lanes hit 32 distinct banks; columns past the row are
//    zeros, which leave the sums' bits unchanged (a sum that starts at +0
//    never becomes -0);
//  - in RNE mode R(x - mean) and R(d * inv) are bf16x2 subtractions and
//    products of bf16 operands: fp32 carries more than 2 * 8 + 2 significand
//    bits, so the reference's fp32 operation followed by the bf16 rounding
//    equals the single correctly rounded bf16x2 result; gamma / beta are
//    applied in fp32, each product and sum rounded on its own.
template <int R, int NV>
__global__ void __launch_bounds__(256) layernorm_aie_reg_kernel(
    const uint16_t* __restrict__ in, const float* __restrict__ gamma,
    const float* __restrict__ beta, uint16_t* __restrict__ out, int64_t rows, int w,
    int64_t ld_in, int64_t ld_out, float eps, int tstride) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warps = blockDim.x / 32, warp = warp_id(), lane = lane_id();
  const bool affine = gamma != nullptr || beta != nullptr;
  const int wp = (w + 3) & ~3;                                 // gamma / beta stride
  float* g_s = reinterpret_cast<float*>(smem);                 // [wp] gamma, then [wp] beta
  float* b_s = g_s + wp;
  uint16_t* tbuf = reinterpret_cast<uint16_t*>(g_s + 2 * wp) + (size_t)warp * 16 * tstride;
  const int kcols = (w + 15) >> 4;                             // columns of t per lane row
  const int kread = (kcols + 3) & ~3;                          // read in groups of four
  const float inv_n = __fdiv_rn(1.0f, (float)w);                       // :69
  int64_t row = (int64_t)blockIdx.x * warps + warp;
  uint32_t x[NV * 4];
  int h = 0;
  auto load_row = [&](int64_t r) {
    const uint16_t* src_row = in + r * ld_in;
    h = chunk_head(src_row);
    const int nch = (w + h + 7) >> 3;
    const uint4* src = reinterpret_cast<const uint4*>(src_row - h);
#pragma unroll
    for (int k = 0; k < NV; k++) {
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      if (lane + 32 * k < nch) q = __ldg(src + lane + 32 * k);
      x[4 * k] = q.x; x[4 * k + 1] = q.y; x[4 * k + 2] = q.z; x[4 * k + 3] = q.w;
    }
  };
  if (row < rows) load_row(row);
  if (affine) {
    for (int c = threadIdx.x; c < wp; c += blockDim.x) {
      g_s[c] = c < w ? (gamma ? gamma[c] : 1.0f) : 0.0f;
      b_s[c] = c < w ? (beta ? beta[c] : 0.0f) : 0.0f;
    }
  }
  __syncthreads();
  for (; row < rows; row += (int64_t)gridDim.x * warps) {
    if (row != (int64_t)blockIdx.x * warps + warp) load_row(row);
    // t: zero the last read group of every lane row, then scatter the row
    for (int i = lane; i < 16 * (kread - (kcols - 1 > 0 ? kcols - 1 : 0)); i += 32) {
      const int l = i & 15, k = (kcols > 0 ? kcols - 1 : 0) + (i >> 4);
      tbuf[l * tstride + k] = 0;
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int c0 = 8 * (lane + 32 * k) - h;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int c = c0 + j;
        if (c >= 0 && c < w)
          tbuf[(c & 15) * tstride + (c >> 4)] = (uint16_t)(x[4 * k + (j >> 1)] >> (16 * (j & 1)));
      }
    }
    __syncwarp();
    // pass 1 (:61-67): sum and sum of squares in 16 fp32 lanes, in column order
    float s1 = 0.0f, s2 = 0.0f;
    if (lane < 16) {
      const uint2* tl = reinterpret_cast<const uint2*>(tbuf + lane * tstride);
#pragma unroll 4
      for (int q = 0; q < kread / 4; q++) {
        const uint2 v = tl[q];
        const float e0 = __uint_as_float(v.x << 16), e1 = __uint_as_float(v.x & 0xFFFF0000u);
        const float e2 = __uint_as_float(v.y << 16), e3 = __uint_as_float(v.y & 0xFFFF0000u);
        s1 = __fadd_rn(s1, e0);
        s2 = __fadd_rn(s2, __fmul_rn(e0, e0));
        s1 = __fadd_rn(s1, e1);
        s2 = __fadd_rn(s2, __fmul_rn(e1, e1));
        s1 = __fadd_rn(s1, e2);
        s2 = __fadd_rn(s2, __fmul_rn(e2, e2));
        s1 = __fadd_rn(s1, e3);
        s2 = __fadd_rn(s2, __fmul_rn(e3, e3));
      }
    }
    s1 = __shfl_sync(0xffffffffu, lane16_tree(s1), 0);
    s2 = __shfl_sync(0xffffffffu, lane16_tree(s2), 0);
    const float mean = __fmul_rn(s1, inv_n);                             // :70
    const float var = __fsub_rn(__fmul_rn(s2, inv_n), __fmul_rn(mean, mean));  // :71
    const float inv = rsqrt_nr(__fadd_rn(var, eps));                     // :72
    const float mb = rbf<R>(mean), ib = rbf<R>(inv);                     // :74-77
    const __nv_bfloat162 mb2 = __float2bfloat162_rn(mb), ib2 = __float2bfloat162_rn(ib);
    // o = R(R(x - mean) * inv) of two bf16 values packed in a word (:80-85),
    // then R(o * gamma + beta) for columns c, c + 1
    auto norm2 = [&](uint32_t xw, int c, bool pair_in_row) -> uint32_t {
      float o0, o1;
      if (R == RND_RNE) {
        const __nv_bfloat162 d = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&xw), mb2);
        const __nv_bfloat162 o = __hmul2(d, ib2);
        const uint32_t ow = *reinterpret_cast<const uint32_t*>(&o);
        if (!affine) return ow;
        o0 = __uint_as_float(ow << 16);
        o1 = __uint_as_float(ow & 0xFFFF0000u);
      } else {
        o0 = rbf<R>(__fmul_rn(rbf<R>(__fsub_rn(__uint_as_float(xw << 16), mb)), ib));
        o1 = rbf<R>(__fmul_rn(rbf<R>(__fsub_rn(__uint_as_float(xw & 0xFFFF0000u), mb)), ib));
        if (!affine) return pack_bf16x2<R>(o0, o1);
      }
      float2 g, b;
      if (pair_in_row) {
        g = *reinterpret_cast<const float2*>(g_s + c);
        b = *reinterpret_cast<const float2*>(b_s + c);
      } else {
        g = make_float2(c >= 0 && c < w ? g_s[c] : 0.0f, c + 1 >= 0 && c + 1 < w ? g_s[c + 1] : 0.0f);
        b = make_float2(c >= 0 && c < w ? b_s[c] : 0.0f, c + 1 >= 0 && c + 1 < w ? b_s[c + 1] : 0.0f);
      }
      // scalar products and sums: gamma is a full fp32 value, so the product
      // is inexact and must stay a separate rounding (never an fma)
      return pack_bf16x2<R>(__fadd_rn(__fmul_rn(o0, g.x), b.x), __fadd_rn(__fmul_rn(o1, g.y), b.y));
    };
    uint16_t* dst_row = out + row * ld_out;
    const int ho = chunk_head(dst_row);
    const int ncho = (w + ho + 7) >> 3;
    uint4* dst = reinterpret_cast<uint4*>(dst_row - ho);
#pragma unroll
    for (int k = 0; k < NV; k++) {
      const int u = lane + 32 * k;
      if (u < ncho) {
        const int c0 = 8 * u - ho;
        uint32_t xs[4];
        if (ho == h) {
          xs[0] = x[4 * k]; xs[1] = x[4 * k + 1]; xs[2] = x[4 * k + 2]; xs[3] = x[4 * k + 3];
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int c = c0 + 2 * j;
            const uint32_t lo = (c >= 0 && c < w) ? tbuf[(c & 15) * tstride + (c >> 4)] : 0u;
            const uint32_t hi =
                (c + 1 >= 0 && c + 1 < w) ? tbuf[((c + 1) & 15) * tstride + ((c + 1) >> 4)] : 0u;
            xs[j] = lo | (hi << 16);
          }
        }
        const bool full = c0 >= 0 && c0 + 8 <= w;
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; j++) o[j] = norm2(xs[j], c0 + 2 * j, full && (c0 % 2 == 0));
        if (full) {
          dst[u] = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int c = c0 + j;
            if (c >= 0 && c < w) dst_row[c] = (uint16_t)(o[j >> 1] >> (16 * (j & 1)));
          }
        }
      }
    }
    __syncwarp();
  }
}

// fp32 two-pass LayerNorm, one warp per row; the row is kept in registers as
// NV float4 per lane (NV * 128 >= width; NV = 0: any width, re-read from L2).
// out_ind: when not NULL, the output pointer is read from device memory there
// (so that a captured graph can write to a different buffer on each replay).
template <bool IN_BF16, bool OUT_BF16, int NV>
__global__ void __launch_bounds__(256) layernorm_fp32_kernel(
    const void* __restrict__ in, const float* __restrict__ gamma,
    const float* __restrict__ beta, void* __restrict__ out, int64_t rows, int w, int64_t ld_in,
    int64_t ld_out, float eps, void* const* __restrict__ out_ind) {
  pdl_launch_dependents();
  pdl_wait();   // the rows come from the previous kernel
  if (out_ind) out = *out_ind;
  constexpr int NR = NV > 0 ? NV : 1;
  const int warps = blockDim.x / 32, warp = warp_id(), lane = lane_id();
  auto load4 = [&](int64_t row, int c) -> float4 {
    if (IN_BF16) {
      const uint2 q = __ldg(reinterpret_cast<const uint2*>(
          reinterpret_cast<const uint16_t*>(in) + row * ld_in + c));
      return make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                         __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
    }
    return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in) +
                                                 row * ld_in + c));
  };
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows;
       row += (int64_t)gridDim.x * warps) {
    float4 v[NR];
    float mean, rstd;
    if (NV > 0) {
#pragma unroll
      for (int i = 0; i < NR; i++) {
        const int c = (i * 32 + lane) * 4;
        v[i] = c < w ? load4(row, c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      ln_row_stats<NR>(v, w, lane, eps, mean, rstd);
    } else {
      // wider than the register buckets: the same sums over the row re-read from L2
      float s = 0.0f;
      for (int c = lane * 4; c < w; c += 128) {
        const float4 t = load4(row, c);
        s += (t.x + t.y) + (t.z + t.w);
      }
      mean = warp_sum(s) / (float)w;
      float q = 0.0f;
      for (int c = lane * 4; c < w; c += 128) {
        const float4 t = load4(row, c);
        const float a = t.x - mean, b = t.y - mean, d = t.z - mean, e = t.w - mean;
        q += (a * a + b * b) + (d * d + e * e);
      }
      rstd = 1.0f / sqrtf(warp_sum(q) / (float)w + eps);
    }
    auto emit = [&](int c, float4 t) {
      const float4 y = ln_affine4(t, mean, rstd, gamma, beta, c);
      if (OUT_BF16) {
        uint2 o;
        o.x = pack_bf16x2_rne(y.x, y.y);
        o.y = pack_bf16x2_rne(y.z, y.w);
        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + row * ld_out + c) = o;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * ld_out + c) = y;
      }
    };
    if (NV > 0) {
#pragma unroll
      for (int i = 0; i < NR; i++) {
        const int c = (i * 32 + lane) * 4;
        if (c < w) emit(c, v[i]);
      }
    } else {
      for (int c = lane * 4; c < w; c += 128) emit(c, load4(row, c));
    }
  }
}

// The encoder's fp32 LayerNorm fused with the int8 mode's per-token
// quantisation of its output (the activation side of q_matmul,
// bench/probe_int8_decode.py:61-67): the normalised row stays in registers,
// its max |y| gives scale = max / 127 (1 for a zero row) and q = rint(y /
// scale). Mean, variance and y follow layernorm_fp32_kernel step for step, so
// q equals quantising that kernel's fp32 output.
template <int NV>
__global__ void __launch_bounds__(256) layernorm_quant_kernel(
    const float* __restrict__ in, const float* __restrict__ gamma, const float* __restrict__ beta,
    int8_t* __restrict__ q, int64_t ld_q, float* __restrict__ scale, int64_t rows, int w,
    int64_t ld_in, float eps) {
  pdl_launch_dependents();
  pdl_wait();   // the rows come from the previous kernel
  const int warps = blockDim.x / 32, warp = warp_id(), lane = lane_id();
  for (int64_t row = (int64_t)blockIdx.x * warps + warp; row < rows;
       row += (int64_t)gridDim.x * warps) {
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int c = (i * 32 + lane) * 4;
      v[i] = c < w ? __ldg(reinterpret_cast<const float4*>(in + row * ld_in + c))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean, rstd;
    ln_row_stats<NV>(v, w, lane, eps, mean, rstd);
    uint32_t mx = 0;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int c = (i * 32 + lane) * 4;
      if (c < w) {
        v[i] = ln_affine4(v[i], mean, rstd, gamma, beta, c);
        mx = max(mx, max(max(__float_as_uint(v[i].x) & 0x7FFFFFFFu,
                             __float_as_uint(v[i].y) & 0x7FFFFFFFu),
                         max(__float_as_uint(v[i].z) & 0x7FFFFFFFu,
                             __float_as_uint(v[i].w) & 0x7FFFFFFFu)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sa = __fdiv_rn(__uint_as_float(mx), 127.0f);
    if (sa == 0.0f) sa = 1.0f;
    const float rcp = __frcp_rn(sa);
    const bool fast = div2_rn_safe(sa);
    if (lane == 0) scale[row] = sa;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int c = (i * 32 + lane) * 4;
      if (c < w)
        *reinterpret_cast<uint32_t*>(q + row * ld_q + c) =
            quant4_i8(v[i].x, v[i].y, v[i].z, v[i].w, sa, rcp, fast);
    }
  }
}

template <bool IB, bool OB>
static void launch_ln_fp32(int grid, cudaStream_t st, const void* in, const float* gamma,
                           const float* beta, void* out, int64_t rows, int w, int64_t ld_in,
                           int64_t ld_out, float eps, void* const* out_ind) {
  const int nv = w > 16 * 128 ? 0 : ln_nv_bucket(w);
// (a failed launch is picked up by the caller's check_launch)
#define WX_LN_CASE(N)                                                                         \
  (void)launch_k(layernorm_fp32_kernel<IB, OB, N>, dim3(grid), dim3(256), 0, st, in, gamma,  \
                 beta, out, rows, w, ld_in, ld_out, eps, out_ind)
  switch (nv) {
    case 3: WX_LN_CASE(3); break;
    case 4: WX_LN_CASE(4); break;
    case 6: WX_LN_CASE(6); break;
    case 8: WX_LN_CASE(8); break;
    case 10: WX_LN_CASE(10); break;
    case 16: WX_LN_CASE(16); break;
    default: WX_LN_CASE(0);
  }
#undef WX_LN_CASE
}

static int grid_for(int64_t work_items, int per_block, int blocks_per_sm) {
  int64_t g = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int launch_gelu_poly4(const void* in, int in_dtype, void* out, int64_t rows, int64_t cols,
                      int64_t ld_in, int64_t ld_out, int rounding, cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(WX_ERR_INVALID, "gelu: negative shape");
  if (rows == 0 || cols == 0) return WX_OK;
  if (!in || !out) return fail(WX_ERR_INVALID, "gelu: NULL pointer");
  if (ld_in < cols || ld_out < cols) return fail(WX_ERR_INVALID, "gelu: row stride < cols");
  if (rounding != RND_TRUNC && rounding != RND_RNE)
    return fail(WX_ERR_INVALID, "gelu: rounding %d", rounding);
  if (in_dtype != WX_DTYPE_BF16 && in_dtype != WX_DTYPE_F32)
    return fail(WX_ERR_INVALID, "gelu: in_dtype %d", in_dtype);
  const bool f32 = in_dtype == WX_DTYPE_F32;
  const bool vec = cols % 8 == 0 && ld_in % 8 == 0 && ld_out % 8 == 0 && aligned16(in) &&
                   aligned16(out);
  const int64_t per_row = vec ? cols / 8 : cols;
  const int gx = (int)std::min<int64_t>((per_row + 127) / 128, 64);
  const int64_t want_y = ((int64_t)sm_count() * 16 + gx - 1) / gx;
  const dim3 grid(gx, (unsigned)std::min<int64_t>(std::min<int64_t>(rows, want_y), 65535));
  uint16_t* o = reinterpret_cast<uint16_t*>(out);
#define WX_GELU_LAUNCH(R, F, V) \
  gelu_poly4_kernel<R, F, V><<<grid, 128, 0, st>>>(in, o, rows, cols, ld_in, ld_out)
  if (rounding == RND_RNE) {
    if (f32) { if (vec) WX_GELU_LAUNCH(RND_RNE, true, 8); else WX_GELU_LAUNCH(RND_RNE, true, 1); }
    else { if (vec) WX_GELU_LAUNCH(RND_RNE, false, 8); else WX_GELU_LAUNCH(RND_RNE, false, 1); }
  } else {
    if (f32) { if (vec) WX_GELU_LAUNCH(RND_TRUNC, true, 8); else WX_GELU_LAUNCH(RND_TRUNC, true, 1); }
    else { if (vec) WX_GELU_LAUNCH(RND_TRUNC, false, 8); else WX_GELU_LAUNCH(RND_TRUNC, false, 1); }
  }
#undef WX_GELU_LAUNCH
  return check_launch("gelu_poly4");
}

// Warps per block for the row kernels: as many as the shared memory allows, up
// to 8.
static int row_warps(size_t fixed_bytes, size_t per_warp_bytes) {
  const size_t budget = 200 * 1024;
  int wps = 8;
  while (wps > 1 && fixed_bytes + wps * per_warp_bytes > budget) wps--;
  return wps;
}

int launch_softmax_rows(const void* in, void* out, int64_t rows, int64_t cols, int64_t valid,
                        int64_t ld_in, int64_t ld_out, float scale, int variant, int rounding,
                        cudaStream_t st) {
  if (rows < 0 || cols < 0) return fail(WX_ERR_INVALID, "softmax: negative shape");
  const int64_t w = valid > 0 ? valid : cols;
  if (w > cols) return fail(WX_ERR_INVALID, "softmax: window %lld > cols %lld", (long long)w, (long long)cols);
  if (rows == 0 || w == 0) return WX_OK;
  if (w > 65536) return fail(WX_ERR_UNSUPPORTED, "softmax: window %lld > 65536", (long long)w);
  if (!in || !out) return fail(WX_ERR_INVALID, "softmax: NULL pointer");
  if (ld_in < w || ld_out < w) return fail(WX_ERR_INVALID, "softmax: row stride < window");
  if (variant != 1 && variant != 3 && variant != 4)
    return fail(WX_ERR_INVALID, "softmax: variant %d (1, 3 or 4)", variant);
  if (rounding != RND_TRUNC && rounding != RND_RNE)
    return fail(WX_ERR_INVALID, "softmax: rounding %d", rounding);
  ExpTablesDev* tabs = nullptr;
  WX_TRY(exp_tables(&tabs));
  const uint16_t* i16 = reinterpret_cast<const uint16_t*>(in);
  uint16_t* o16 = reinterpret_cast<uint16_t*>(out);
  const bool even = (reinterpret_cast<uintptr_t>(in) & 1) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 1) == 0;
  if (variant != 3 && even && w <= 8 * 32 * 8 - 7) {
    const int chunks = (int)(((w + 7 + 7) / 8 + 31) / 32);
    const int nvc = chunks <= 2 ? chunks : chunks <= 4 ? 4 : chunks <= 6 ? 6 : 8;
    const int wps = kSmRegThreads / 32;
    const size_t smem = kExpTabBytes + (size_t)wps * nvc * 32 * 16;
    const int grid = grid_for(rows, wps, 2);
#define WX_SMR_LAUNCH(R, V, N)                                                                \
  do {                                                                                        \
    auto k = softmax_rows_reg_kernel<R, V, N>;                                                \
    WX_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k<<<grid, kSmRegThreads, smem, st>>>(i16, o16, rows, (int)w, ld_in, ld_out, scale,       \
                                         tabs->t16[R]);                                      \
  } while (0)
#define WX_SMR_NV(R, V)                       \
  do {                                        \
    if (nvc == 1) WX_SMR_LAUNCH(R, V, 1);     \
    else if (nvc == 2) WX_SMR_LAUNCH(R, V, 2); \
    else if (nvc == 4) WX_SMR_LAUNCH(R, V, 4); \
    else if (nvc == 6) WX_SMR_LAUNCH(R, V, 6); \
    else WX_SMR_LAUNCH(R, V, 8);              \
  } while (0)
    if (rounding == RND_RNE) {
      if (variant == 4) WX_SMR_NV(RND_RNE, 4); else WX_SMR_NV(RND_RNE, 1);
    } else {
      if (variant == 4) WX_SMR_NV(RND_TRUNC, 4); else WX_SMR_NV(RND_TRUNC, 1);
    }
#undef WX_SMR_NV
#undef WX_SMR_LAUNCH
    return check_launch("softmax_rows");
  }
  const int wpad = (int)((w + 7) / 8 * 8);
  const size_t fixed = ((kExpTabN * 2 + 15) / 16) * 16 + (variant == 3 ? kExpTabN * 4 : 0);
  const int wps = row_warps(fixed, (size_t)wpad * 2);
  const size_t smem = fixed + (size_t)wps * wpad * 2;
  const int vin = (w % 8 == 0 && ld_in % 8 == 0 && aligned16(in)) ? 1 : 0;
  const int vout = (w % 8 == 0 && ld_out % 8 == 0 && aligned16(out)) ? 1 : 0;
  const int grid = grid_for(rows, wps, 2);
#define WX_SM_LAUNCH(R, V)                                                                   \
  do {                                                                                       \
    auto k = softmax_rows_kernel<R, V>;                                                      \
    WX_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k<<<grid, wps * 32, smem, st>>>(i16, o16, rows, (int)w, ld_in, ld_out, scale,           \
                                    tabs->t16[R], tabs->t32, wpad, vin, vout);               \
  } while (0)
  if (rounding == RND_RNE) {
    if (variant == 4) WX_SM_LAUNCH(RND_RNE, 4); else if (variant == 1) WX_SM_LAUNCH(RND_RNE, 1); else WX_SM_LAUNCH(RND_RNE, 3);
  } else {
    if (variant == 4) WX_SM_LAUNCH(RND_TRUNC, 4); else if (variant == 1) WX_SM_LAUNCH(RND_TRUNC, 1); else WX_SM_LAUNCH(RND_TRUNC, 3);
  }
#undef WX_SM_LAUNCH
  return check_launch("softmax_rows");
}

int launch_layernorm_rows(const void* in, int in_dtype, const float* gamma, const float* beta,
                          void* out, int out_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                          int64_t ld_out, float eps, int mode, int rounding, cudaStream_t st,
                          void* const* out_ind) {
  if (rows < 0 || cols < 0) return fail(WX_ERR_INVALID, "layernorm: negative shape");
  if (out_ind && mode != WX_LN_FP32)
    return fail(WX_ERR_INVALID, "layernorm: an indirect output needs mode WX_LN_FP32");
  if (rows == 0 || cols == 0) return WX_OK;
  if (!in || !out) return fail(WX_ERR_INVALID, "layernorm: NULL pointer");
  if (ld_in < cols || ld_out < cols) return fail(WX_ERR_INVALID, "layernorm: row stride < cols");
  if (mode == WX_LN_AIE) {
    if (in_dtype != WX_DTYPE_BF16 || out_dtype != WX_DTYPE_BF16)
      return fail(WX_ERR_INVALID, "layernorm: WX_LN_AIE is bf16 in and out");
    if (rounding != RND_TRUNC && rounding != RND_RNE)
      return fail(WX_ERR_INVALID, "layernorm: rounding %d", rounding);
    if (cols > 65536) return fail(WX_ERR_UNSUPPORTED, "layernorm: cols %lld > 65536", (long long)cols);
    const bool even = (reinterpret_cast<uintptr_t>(in) & 1) == 0 &&
                      (reinterpret_cast<uintptr_t>(out) & 1) == 0;
    if (even && cols <= 8 * 32 * 8 - 7) {
      const int w = (int)cols;
      const int chunks = (w + 14) / 8;
      const int nvc = chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : chunks <= 192 ? 6 : 8;
      // per warp a lane-transposed copy of its row: 16 lane rows of
      // tstride = 8m + 4 >= ceil(w / 16) elements, padded to a multiple of 4
      const int kcols = (w + 15) / 16;
      const int tstride = ((kcols + 3) + 3) / 8 * 8 + 4;
      const size_t smem = (size_t)2 * ((w + 3) & ~3) * 4 + (size_t)8 * 16 * tstride * 2;
      const int grid = grid_for(rows, 8, 8);
      const uint16_t* i16 = reinterpret_cast<const uint16_t*>(in);
      uint16_t* o16 = reinterpret_cast<uint16_t*>(out);
#define WX_LNR_LAUNCH(R, N)                                                                   \
  do {                                                                                        \
    auto k = layernorm_aie_reg_kernel<R, N>;                                                  \
    WX_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k<<<grid, 256, smem, st>>>(i16, gamma, beta, o16, rows, w, ld_in, ld_out, eps, tstride);  \
  } while (0)
#define WX_LNR_NV(R)                           \
  do {                                         \
    if (nvc == 1) WX_LNR_LAUNCH(R, 1);         \
    else if (nvc == 2) WX_LNR_LAUNCH(R, 2);    \
    else if (nvc == 4) WX_LNR_LAUNCH(R, 4);    \
    else if (nvc == 6) WX_LNR_LAUNCH(R, 6);    \
    else WX_LNR_LAUNCH(R, 8);                  \
  } while (0)
      if (rounding == RND_RNE) WX_LNR_NV(RND_RNE); else WX_LNR_NV(RND_TRUNC);
#undef WX_LNR_NV
#undef WX_LNR_LAUNCH
      return check_launch("layernorm_aie");
    }
    const int wpad = (int)((cols + 7) / 8 * 8);
    const int wps = row_warps(0, (size_t)wpad * 2);
    const size_t smem = (size_t)wps * wpad * 2;
    const int vin = (cols % 8 == 0 && ld_in % 8 == 0 && aligned16(in)) ? 1 : 0;
    const int vout = (cols % 8 == 0 && ld_out % 8 == 0 && aligned16(out)) ? 1 : 0;
    const int grid = grid_for(rows, wps, 2);
    const uint16_t* i16 = reinterpret_cast<const uint16_t*>(in);
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out);
    if (rounding == RND_RNE) {
      auto k = layernorm_aie_kernel<RND_RNE>;
      WX_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k<<<grid, wps * 32, smem, st>>>(i16, gamma, beta, o16, rows, (int)cols, ld_in, ld_out, eps, wpad, vin, vout);
    } else {
      auto k = layernorm_aie_kernel<RND_TRUNC>;
      WX_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k<<<grid, wps * 32, smem, st>>>(i16, gamma, beta, o16, rows, (int)cols, ld_in, ld_out, eps, wpad, vin, vout);
    }
    return check_launch("layernorm_aie");
  }
  if (mode != WX_LN_FP32) return fail(WX_ERR_INVALID, "layernorm: mode %d", mode);
  if (cols % 4 != 0 || ld_in % 4 != 0 || ld_out % 4 != 0 || !aligned16(in) || !aligned16(out) ||
      (gamma && !aligned16(gamma)) || (beta && !aligned16(beta)))
    return fail(WX_ERR_INVALID, "layernorm fp32: cols and strides must be multiples of 4, "
                "pointers 16-byte aligned");
  const int grid = grid_for(rows, 8, 8);
  const bool ib = in_dtype == WX_DTYPE_BF16, ob = out_dtype == WX_DTYPE_BF16;
  const int w = (int)cols;
  if (ib && ob) launch_ln_fp32<true, true>(grid, st, in, gamma, beta, out, rows, w, ld_in, ld_out, eps,
                                             out_ind);
  else if (ib) launch_ln_fp32<true, false>(grid, st, in, gamma, beta, out, rows, w, ld_in, ld_out, eps,
                                             out_ind);
  else if (ob) launch_ln_fp32<false, true>(grid, st, in, gamma, beta, out, rows, w, ld_in, ld_out, eps,
                                             out_ind);
  else launch_ln_fp32<false, false>(grid, st, in, gamma, beta, out, rows, w, ld_in, ld_out, eps,
                                             out_ind);
  return check_launch("layernorm_fp32");
}

int launch_layernorm_quant_rows(const float* in, const float* gamma, const float* beta, int8_t* q,
                                float* scale, int64_t rows, int64_t cols, int64_t ld_in,
                                int64_t ld_q, float eps, cudaStream_t st) {
  if (rows == 0) return WX_OK;
  if (rows < 0 || cols <= 0) return fail(WX_ERR_INVALID, "layernorm_quant: rows >= 0 and cols > 0 required");
  if (!in || !q || !scale) return fail(WX_ERR_INVALID, "layernorm_quant: NULL pointer");
  if (cols % 4 != 0 || ld_in % 4 != 0 || ld_q % 4 != 0 || ld_in < cols || ld_q < cols ||
      !aligned16(in) || (reinterpret_cast<uintptr_t>(q) & 3) || (gamma && !aligned16(gamma)) ||
      (beta && !aligned16(beta)))
    return fail(WX_ERR_INVALID, "layernorm_quant: cols, ld_in and ld_q must be multiples of 4, "
                "in, gamma and beta 16-byte aligned, q 4-byte aligned");
  if (cols > 2048) return fail(WX_ERR_UNSUPPORTED, "layernorm_quant: rows wider than 2048");
  const int grid = grid_for(rows, 8, 8);
  const int w = (int)cols;
#define WX_LNQ_CASE(N)                                                                     \
  (void)launch_k(layernorm_quant_kernel<N>, dim3(grid), dim3(256), 0, st, in, gamma, beta, \
                 q, ld_q, scale, rows, w, ld_in, eps)
  switch (ln_nv_bucket(w)) {
    case 3: WX_LNQ_CASE(3); break;
    case 4: WX_LNQ_CASE(4); break;
    case 6: WX_LNQ_CASE(6); break;
    case 8: WX_LNQ_CASE(8); break;
    case 10: WX_LNQ_CASE(10); break;
    default: WX_LNQ_CASE(16);
  }
#undef WX_LNQ_CASE
  return check_launch("layernorm_quant");
}

}  // namespace wx

extern "C" {

int wx_layernorm_quant_rows(const float* in, const float* gamma, const float* beta, int8_t* q,
                            float* scale, int64_t rows, int64_t cols, int64_t ld_in, int64_t ld_q,
                            float eps, void* stream) {
  return wx::launch_layernorm_quant_rows(in, gamma, beta, q, scale, rows, cols, ld_in, ld_q, eps,
                                         wx::as_stream(stream));
}

int wx_gelu_poly4(const void* in, int in_dtype, void* out, int64_t rows, int64_t cols,
                  int64_t ld_in, int64_t ld_out, int rounding, void* stream) {
  return wx::launch_gelu_poly4(in, in_dtype, out, rows, cols, ld_in, ld_out, rounding,
                               wx::as_stream(stream));
}

int wx_softmax_rows(const void* in, void* out, int64_t rows, int64_t cols, int64_t valid,
                    int64_t ld_in, int64_t ld_out, float scale, int variant, int rounding,
                    void* stream) {
  return wx::launch_softmax_rows(in, out, rows, cols, valid, ld_in, ld_out, scale, variant,
                                 rounding, wx::as_stream(stream));
}

int wx_layernorm_rows(const void* in, int in_dtype, const float* gamma, const float* beta,
                      void* out, int out_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                      int64_t ld_out, float eps, int mode, int rounding, void* stream) {
  return wx::launch_layernorm_rows(in, in_dtype, gamma, beta, out, out_dtype, rows, cols, ld_in,
                                   ld_out, eps, mode, rounding, wx::as_stream(stream), nullptr);
}

int wx_softmax_exp_table(int rounding, uint16_t* out16, float* out32, int64_t n) {
  if (n < wx::kExpTabN) return wx::fail(WX_ERR_INVALID, "exp table needs %d entries", wx::kExpTabN);
  std::vector<uint16_t> a(wx::kExpTabN), b(wx::kExpTabN);
  std::vector<float> c(wx::kExpTabN);
  wx::host_exp_tables(a.data(), b.data(), c.data());
  for (int i = 0; i < wx::kExpTabN; i++) {
    if (out16) out16[i] = rounding == WX_ROUND_RNE ? b[i] : a[i];
    if (out32) out32[i] = c[i];
  }
  return wx::kExpTabN;
}

int wx_gelu4_table(int rounding, float* out, int64_t n) {
  if (n < 24) return wx::fail(WX_ERR_INVALID, "gelu table needs 24 floats");
  // The constants the kernels compile in (common.cuh), checked against the
  // decimal literals of the reference's table rounded in `rounding`.
  const wx::Gelu4Table t = wx::gelu4_table(rounding);
  const float kc[3][5] = WX_GELU4_COEF;
  const float brk[3] = {1.0f, 2.0f, 4.0f}, sh[3] = {0.5f, 1.5f, 3.0f}, sc[3] = {2.0f, 2.0f, 1.0f};
  for (int p = 0; p < 3; p++) {
    if (t.brk[p] != brk[p] || t.shift[p] != sh[p] || t.scale[p] != sc[p])
      return wx::fail(WX_ERR_INVALID, "gelu table: compiled piece bounds differ");
    for (int k = 0; k < 5; k++)
      if (t.c[p][k] != kc[p][k])
        return wx::fail(WX_ERR_INVALID, "gelu table: compiled coefficient %d,%d differs", p, k);
  }
  memcpy(out, brk, sizeof(brk));
  memcpy(out + 3, sh, sizeof(sh));
  memcpy(out + 6, sc, sizeof(sc));
  memcpy(out + 9, kc, sizeof(kc));
  return 24;
}

}  // extern "C"
