// int8 quantisation of activation and weight rows for the int8 GEMM.
//
// The reference's int8 mode (bench/probe_int8_decode.py:48-74, a numpy
// simulation that the encoder calls as its `mm`) quantises both operands of
// every projection and MLP GEMM:
//   sa = max|A[i, :]| / 127 per row (token), 1 where that is 0
//   sw = max|B[:, j]| / 127 per column (channel)       ("perchan")
//      = max|B| / 127 for the whole matrix              ("pertensor")
//   A_q = rint(A / sa), B_q = rint(B / sw)     (float32 divisions, half-even)
//   C = (float(A_q @ B_q) * sa) * sw  (+ bias)
// B there is the (K, N) transposed weight, so a column of B is a row of the
// torch weight (N, K) that the GEMM here takes: both operands are quantised
// per row of their row-major storage by the same kernel.
//
// One warp per row; 16-byte loads when the rows are aligned. The divisions are
// IEEE round-to-nearest (__fdiv_rn) and the rounding to an integer is
// half-to-even (__float2int_rn), so each quantised value equals numpy's. The
// kernels are HBM-bound: a bf16 row is read once (twice when the row maximum is
// computed here, the second time from L2) and written as int8.
//
// The same probe's unquantised control ("fp32") is the fp32 GEMM at the end.
#include <cstdint>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

constexpr int kQuantWarps = 8;

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float load_as_f32<uint16_t>(const uint16_t* p) {
  return __uint_as_float((uint32_t)*p << 16);
}

// 16 bytes of row elements as fp32: 4 floats or 8 bf16
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};
__device__ __forceinline__ void unpack16(const uint4& u, float (&v)[4]) {
  v[0] = __uint_as_float(u.x);
  v[1] = __uint_as_float(u.y);
  v[2] = __uint_as_float(u.z);
  v[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void unpack16(const uint4& u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// max |x| over one row, reduced over the warp (all lanes get it)
template <typename T, bool VEC>
__device__ __forceinline__ float row_absmax(const T* x, int64_t cols, int lane) {
  uint32_t m = 0;   // |x| bits: non-negative floats order as unsigned integers
  constexpr int V = Vec16<T>::N;
  int64_t c0 = 0;
  if (VEC) {
    const int64_t nv = cols / V;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int64_t i = lane; i < nv; i += 32) {
      float v[V];
      unpack16(__ldg(xv + i), v);
#pragma unroll
      for (int e = 0; e < V; e++) m = max(m, __float_as_uint(v[e]) & 0x7FFFFFFFu);
    }
    c0 = nv * V;
  }
  for (int64_t c = c0 + lane; c < cols; c += 32)
    m = max(m, __float_as_uint(load_as_f32<T>(x + c)) & 0x7FFFFFFFu);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  return __uint_as_float(m);
}

__device__ __forceinline__ uint32_t q8(float x, float sa) {
  return (uint32_t)(__float2int_rn(__fdiv_rn(x, sa)) & 0xFF);
}

// the per-row divisor and its reciprocal: scale = max / 127 (1 for a zero row)
struct RowScale {
  float s, rcp;
  bool fast;   // s in the range where quant4_i8's FMA division is exact
};
__device__ __forceinline__ RowScale row_scale(float m) {
  RowScale r;
  r.s = __fdiv_rn(m, 127.0f);
  if (r.s == 0.0f) r.s = 1.0f;
  r.rcp = __frcp_rn(r.s);
  r.fast = div2_rn_safe(r.s);
  return r;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(32 * kQuantWarps)
    absmax_rows_kernel(const T* __restrict__ in, int64_t rows, int64_t cols, int64_t ld,
                       float* __restrict__ out, int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float m = row_absmax<T, VEC>(in + row * ld, cols, lane);
  if (lane == 0 && m > 0.0f)
    atomicMax(reinterpret_cast<unsigned int*>(out) + row * out_stride, __float_as_uint(m));
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(32 * kQuantWarps)
    quantize_rows_kernel(const T* __restrict__ in, int64_t rows, int64_t cols, int64_t ld,
                         const float* __restrict__ rowmax, int64_t rowmax_stride,
                         int8_t* __restrict__ q, int64_t ld_q, float* __restrict__ scale) {
  pdl_launch_dependents();
  pdl_wait();   // the rows (and their maxima) come from the previous kernel
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* x = in + row * ld;
  const float m = rowmax ? rowmax[row * rowmax_stride] : row_absmax<T, VEC>(x, cols, lane);
  const RowScale rs = row_scale(m);
  if (lane == 0) scale[row] = rs.s;
  int8_t* qr = q + row * ld_q;
  constexpr int V = Vec16<T>::N;
  int64_t c0 = 0;
  if (VEC) {
    const int64_t nv = cols / V;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
#pragma unroll 4
    for (int64_t i = lane; i < nv; i += 32) {
      float v[V];
      unpack16(__ldg(xv + i), v);
      if constexpr (V == 8) {
        uint2 o;
        o.x = quant4_i8(v[0], v[1], v[2], v[3], rs.s, rs.rcp, rs.fast);
        o.y = quant4_i8(v[4], v[5], v[6], v[7], rs.s, rs.rcp, rs.fast);
        *reinterpret_cast<uint2*>(qr + i * 8) = o;
      } else {
        *reinterpret_cast<uint32_t*>(qr + i * 4) =
            quant4_i8(v[0], v[1], v[2], v[3], rs.s, rs.rcp, rs.fast);
      }
    }
    c0 = nv * V;
  }
  for (int64_t c = c0 + lane; c < cols; c += 32) qr[c] = (int8_t)q8(load_as_f32<T>(x + c), rs.s);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int launch_absmax_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld,
                       float* out, int64_t out_stride, cudaStream_t st) {
  if (rows == 0) return WX_OK;   // nothing to fold
  if (rows < 0 || cols <= 0) return fail(WX_ERR_INVALID, "absmax_rows: rows >= 0 and cols > 0 required");
  if (!in || !out) return fail(WX_ERR_INVALID, "absmax_rows: NULL pointer");
  if (ld < cols || out_stride < 0) return fail(WX_ERR_INVALID, "absmax_rows: bad ld or out_stride");
  if (in_dtype != WX_DTYPE_BF16 && in_dtype != WX_DTYPE_F32)
    return fail(WX_ERR_INVALID, "absmax_rows: dtype %d", in_dtype);
  const int es = in_dtype == WX_DTYPE_F32 ? 4 : 2;
  const bool vec = aligned16(in) && (ld * es) % 16 == 0;
  const unsigned grid = (unsigned)((rows + kQuantWarps - 1) / kQuantWarps);
  if (in_dtype == WX_DTYPE_F32) {
    const float* x = static_cast<const float*>(in);
    if (vec) absmax_rows_kernel<float, true><<<grid, 32 * kQuantWarps, 0, st>>>(x, rows, cols, ld, out, out_stride);
    else absmax_rows_kernel<float, false><<<grid, 32 * kQuantWarps, 0, st>>>(x, rows, cols, ld, out, out_stride);
  } else {
    const uint16_t* x = static_cast<const uint16_t*>(in);
    if (vec) absmax_rows_kernel<uint16_t, true><<<grid, 32 * kQuantWarps, 0, st>>>(x, rows, cols, ld, out, out_stride);
    else absmax_rows_kernel<uint16_t, false><<<grid, 32 * kQuantWarps, 0, st>>>(x, rows, cols, ld, out, out_stride);
  }
  return check_launch("absmax_rows");
}

int launch_quantize_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld,
                         const float* rowmax, int64_t rowmax_stride, int8_t* q, int64_t ld_q,
                         float* scale, cudaStream_t st) {
  if (rows == 0) return WX_OK;   // nothing to quantise
  if (rows < 0 || cols <= 0)
    return fail(WX_ERR_INVALID, "quantize_rows: rows >= 0 and cols > 0 required (an empty row has no scale)");
  if (!in || !q || !scale) return fail(WX_ERR_INVALID, "quantize_rows: NULL pointer");
  if (ld < cols || ld_q < cols || rowmax_stride < 0)
    return fail(WX_ERR_INVALID, "quantize_rows: bad ld, ld_q or rowmax_stride");
  if (in_dtype != WX_DTYPE_BF16 && in_dtype != WX_DTYPE_F32)
    return fail(WX_ERR_INVALID, "quantize_rows: dtype %d", in_dtype);
  const int es = in_dtype == WX_DTYPE_F32 ? 4 : 2;
  const bool vec = aligned16(in) && (ld * es) % 16 == 0 && aligned16(q) && ld_q % 16 == 0;
  const unsigned grid = (unsigned)((rows + kQuantWarps - 1) / kQuantWarps);
  if (in_dtype == WX_DTYPE_F32) {
    const float* x = static_cast<const float*>(in);
    // (a failed launch is picked up by check_launch below)
    if (vec)
      (void)launch_k(quantize_rows_kernel<float, true>, dim3(grid), dim3(32 * kQuantWarps), 0, st,
                     x, rows, cols, ld, rowmax, rowmax_stride, q, ld_q, scale);
    else
      (void)launch_k(quantize_rows_kernel<float, false>, dim3(grid), dim3(32 * kQuantWarps), 0,
                     st, x, rows, cols, ld, rowmax, rowmax_stride, q, ld_q, scale);
  } else {
    const uint16_t* x = static_cast<const uint16_t*>(in);
    if (vec)
      (void)launch_k(quantize_rows_kernel<uint16_t, true>, dim3(grid), dim3(32 * kQuantWarps), 0,
                     st, x, rows, cols, ld, rowmax, rowmax_stride, q, ld_q, scale);
    else
      (void)launch_k(quantize_rows_kernel<uint16_t, false>, dim3(grid), dim3(32 * kQuantWarps), 0,
                     st, x, rows, cols, ld, rowmax, rowmax_stride, q, ld_q, scale);
  }
  return check_launch("quantize_rows");
}

// ---------------------------------------------------------------- fp32 GEMM
// The unquantised control of q_matmul_factory ("fp32": A @ B + bias in numpy
// float32, bench/probe_int8_decode.py:58-60): C = A @ B^T (+ bias) on the FMA
// pipe. 128 x 128 tiles, 256 threads, each an 8 x 8 block of outputs (rows
// 4 ty + {0..3} and 64 + 4 ty + {0..3}, columns likewise from tx) so that its
// operands come from shared memory as float4; K in steps of 16, the next step
// loaded into registers while the current one is multiplied. Every output is
// one fp32 FMA chain over k in ascending order.
constexpr int kF32Tile = 128, kF32Step = 16;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       const float* __restrict__ bias,
                                                       float* __restrict__ C, int M, int N, int K,
                                                       int64_t lda, int64_t ldb, int64_t ldc) {
  __shared__ __align__(16) float sA[2][kF32Step][kF32Tile];
  __shared__ __align__(16) float sB[2][kF32Step][kF32Tile];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * kF32Tile, n0 = blockIdx.x * kF32Tile;
  // staging: element e = tid + 256 i of a 128 x 16 tile is row e / 16, k e % 16
  float ra[8], rb[8];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = tid + 256 * i, r = e >> 4, k = k0 + (e & 15);
      ra[i] = (m0 + r < M && k < K) ? A[(int64_t)(m0 + r) * lda + k] : 0.0f;
      rb[i] = (n0 + r < N && k < K) ? B[(int64_t)(n0 + r) * ldb + k] : 0.0f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = tid + 256 * i;
      sA[buf][e & 15][e >> 4] = ra[i];
      sB[buf][e & 15][e >> 4] = rb[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
  const int steps = (K + kF32Step - 1) / kF32Step;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int s = 0; s < steps; s++) {
    const int buf = s & 1;
    if (s + 1 < steps) fetch((s + 1) * kF32Step);
#pragma unroll
    for (int k = 0; k < kF32Step; k++) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sA[buf][k][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sA[buf][k][64 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sB[buf][k][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sB[buf][k][64 + 4 * tx]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    if (s + 1 < steps) {
      stash(buf ^ 1);   // the other buffer was last read before the previous barrier
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int m = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int n = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + j - 4);
      if (n < N) C[(int64_t)m * ldc + n] = bias ? __fadd_rn(acc[i][j], bias[n]) : acc[i][j];
    }
  }
}

int launch_gemm_f32(const float* A, const float* B, const float* bias, float* C, int64_t M,
                    int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0) return fail(WX_ERR_INVALID, "gemm_f32: negative shape");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(WX_ERR_UNSUPPORTED, "gemm_f32: dimension exceeds 2^31");
  if (M == 0 || N == 0) return WX_OK;
  if (!A || !B || !C) return fail(WX_ERR_INVALID, "gemm_f32: NULL operand");
  if (lda < K || ldb < K || ldc < N) return fail(WX_ERR_INVALID, "gemm_f32: leading dimension too small");
  const int64_t gx = (N + kF32Tile - 1) / kF32Tile, gy = (M + kF32Tile - 1) / kF32Tile;
  if (gy > 65535) return fail(WX_ERR_UNSUPPORTED, "gemm_f32: M above %d", 65535 * kF32Tile);
  (void)launch_k(gemm_f32_kernel, dim3((unsigned)gx, (unsigned)gy), dim3(256), 0, st, A, B, bias,
                 C, (int)M, (int)N, (int)K, lda, ldb, ldc);
  return check_launch("gemm_f32");
}

}  // namespace wx

extern "C" {

int wx_absmax_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                   float* out, int64_t out_stride, void* stream) {
  return wx::launch_absmax_rows(in, in_dtype, rows, cols, ld_in, out, out_stride,
                                wx::as_stream(stream));
}

int wx_quantize_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                     const float* rowmax, int64_t rowmax_stride, int8_t* q, int64_t ld_q,
                     float* scale, void* stream) {
  return wx::launch_quantize_rows(in, in_dtype, rows, cols, ld_in, rowmax, rowmax_stride, q, ld_q,
                                  scale, wx::as_stream(stream));
}

int wx_gemm_i8(const int8_t* A, const int8_t* B, const float* sa, const float* sw,
               const float* bias, const float* R, void* C, int64_t M, int64_t N, int64_t K,
               int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int epilogue, float* rowmax,
               void* stream) {
  if (epilogue < WX_EPI_F32 || epilogue > WX_EPI_BF16_GELU_ERF)
    return wx::fail(WX_ERR_INVALID, "gemm_i8: epilogue %d", epilogue);
  wx::GemmPlan p;
  WX_TRY(wx::gemm_plan_i8(&p, A, B, sa, sw, bias, R, C, M, N, K, lda, ldb, ldc, ldr, epilogue,
                          rowmax));
  return wx::gemm_run(p, wx::as_stream(stream));
}

int wx_gemm_f32(const float* A, const float* B, const float* bias, float* C, int64_t M,
                int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return wx::launch_gemm_f32(A, B, bias, C, M, N, K, lda, ldb, ldc, wx::as_stream(stream));
}

}  // extern "C"
