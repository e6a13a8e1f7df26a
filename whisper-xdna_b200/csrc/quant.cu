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

}  // extern "C"
