// One row of the encoder's fp32 LayerNorm (src/npu_whisper_encoder.py:278-281):
// mean, then the mean of the squared deviations, y = (x - mean) * rstd * gamma
// + beta with rstd = 1 / sqrt(var + eps), computed by one warp that holds the
// row in registers: lane l keeps columns 4*(32 i + l) .. +3 in v[i], zeros past
// the width w. The fp32 LayerNorm kernel and the LayerNorm + int8 quantise
// kernel (rowops.cu) both compute through these functions, so that a row
// normalised by either has the same bits.
#pragma once

#include "common.cuh"

namespace wx {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The four-wide groups of the row in registers: NV float4 per lane covers
// widths up to 128 * NV. The kernels instantiate these buckets.
__host__ __device__ constexpr int ln_nv_bucket(int w) {
  return (w + 127) / 128 <= 3    ? 3
         : (w + 127) / 128 <= 4  ? 4
         : (w + 127) / 128 <= 6  ? 6
         : (w + 127) / 128 <= 8  ? 8
         : (w + 127) / 128 <= 10 ? 10
                                 : 16;
}

template <int NV>
__device__ __forceinline__ void ln_row_stats(const float4 (&v)[NV], int w, int lane, float eps,
                                             float& mean, float& rstd) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; i++) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  mean = warp_sum(s) / (float)w;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c = (i * 32 + lane) * 4;
    if (c < w) {
      const float a = v[i].x - mean, b = v[i].y - mean, d = v[i].z - mean, e = v[i].w - mean;
      q += (a * a + b * b) + (d * d + e * e);
    }
  }
  rstd = 1.0f / sqrtf(warp_sum(q) / (float)w + eps);
}

// y for four columns given their gamma and beta
__device__ __forceinline__ float4 ln_affine4(float4 t, float mean, float rstd, float4 g,
                                             float4 b) {
  return make_float4((t.x - mean) * rstd * g.x + b.x, (t.y - mean) * rstd * g.y + b.y,
                     (t.z - mean) * rstd * g.z + b.z, (t.w - mean) * rstd * g.w + b.w);
}
__device__ __forceinline__ float4 ln_gamma4(const float* __restrict__ gamma, int c) {
  return gamma ? __ldg(reinterpret_cast<const float4*>(gamma + c))
               : make_float4(1.f, 1.f, 1.f, 1.f);
}
__device__ __forceinline__ float4 ln_beta4(const float* __restrict__ beta, int c) {
  return beta ? __ldg(reinterpret_cast<const float4*>(beta + c))
              : make_float4(0.f, 0.f, 0.f, 0.f);
}
// y for the four columns c .. c+3 (gamma / beta NULL: 1 / 0)
__device__ __forceinline__ float4 ln_affine4(float4 t, float mean, float rstd,
                                             const float* __restrict__ gamma,
                                             const float* __restrict__ beta, int c) {
  return ln_affine4(t, mean, rstd, ln_gamma4(gamma, c), ln_beta4(beta, c));
}

}  // namespace wx
