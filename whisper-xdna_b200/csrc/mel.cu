// whisper's log-mel frontend on the GPU: 16 kHz audio -> (n_mels, 3000)
// log-mel features, the encoder's input. The reference computes them on the
// CPU with openai-whisper's log_mel_spectrogram (serve/npu_stt_server.py:
// 334-336): a centred STFT (n_fft 400, hop 160, periodic Hann window, the
// 30 s window reflect-padded by 200 samples at both ends, last frame
// dropped), the power spectrum, a Slaney mel filterbank (0-8 kHz),
// log10(max(., 1e-10)), a floor 8 below the clip's maximum, then (x + 4) / 4.
//
// log_mel_kernel: one CTA per 32 frames of one clip. The DFT of the 32 frames
// is a small fp32 GEMM, (32 x 400 windowed samples) x (400 x 416 cos/sin
// columns), register-tiled: the frames are staged transposed in shared memory,
// the DFT matrix streams through a double buffer in slices of 16 samples
// (cp.async), and each of 208 threads accumulates 4 frames x 8 bins (cos and
// sin: 64 sums), reading one float4 of frames and four float4 of the matrix
// per sample for 64 FMAs. The matrix is laid out [sample][quarter][bin group]
// [4] so that the eight bin groups a warp reads sit in consecutive 16-byte
// units (no bank conflicts). The power spectrum goes to shared memory, each mel
// band sums its few nonzero filter weights, and the log10 values are written
// with the block's maximum.
// log_mel_finalize_kernel: the clip's maximum from the block maxima, then the
// floor and the affine map, elementwise.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace wx {

constexpr int kMelFFT = 400, kMelHop = 160, kMelBins = 201, kMelFrames = 3000;
constexpr int64_t kMelWindow = 480000;               // 30 s at 16 kHz
constexpr int kMelFB = 32;                           // frames per CTA
constexpr int kMelBlocks = (kMelFrames + kMelFB - 1) / kMelFB;   // 94 per clip
constexpr int kMelThreads = 224;                     // 7 warps; 208 compute threads
constexpr int kMelGroups = 26;                       // bin groups of 8 (208 >= 201 bins)
constexpr int kMelCompute = 8 * kMelGroups;          // 8 frame groups of 4 x 26 bin groups
constexpr int kMelKS = 16;                           // samples per DFT-matrix slice
constexpr int kMelXT = 36;                           // floats per transposed sample row
constexpr int kMelSlice = kMelKS * 4 * kMelGroups * 4;   // floats per slice (26.6 KB)
// shared memory: frames transposed [400][36], two matrix slices, 8 maxima; the
// power spectrum [32][201] reuses the slices after the GEMM
constexpr int kMelSmem = (kMelFFT * kMelXT + 2 * kMelSlice + 8) * 4;
static_assert(kMelFB * kMelBins <= 2 * kMelSlice, "power spectrum fits the slice buffers");
static_assert(kMelFFT % kMelKS == 0, "whole slices");

struct MelTables {
  int n_mels = 0, maxw = 0;
  float *dft = nullptr, *window = nullptr, *fw = nullptr;   // dft: [400][4][26][4]
  int *fstart = nullptr, *flen = nullptr;
};

// Slaney mel scale (linear below 1 kHz, logarithmic above), in double.
static double hz_to_mel(double f) {
  const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
  const double logstep = std::log(6.4) / 27.0;
  return f >= min_log_hz ? min_log_mel + std::log(f / min_log_hz) / logstep : f / f_sp;
}
static double mel_to_hz(double m) {
  const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
  const double logstep = std::log(6.4) / 27.0;
  return m >= min_log_mel ? min_log_hz * std::exp(logstep * (m - min_log_mel)) : f_sp * m;
}

// Triangles between consecutive mel-spaced edges, each scaled by 2 / bandwidth
// (Slaney area normalisation); row m of the (n_mels, 201) filterbank.
static std::vector<double> slaney_filters(int n_mels) {
  const double sr = 16000.0, fmax = sr / 2.0;
  std::vector<double> pts(n_mels + 2), w((size_t)n_mels * kMelBins, 0.0);
  const double m0 = hz_to_mel(0.0), m1 = hz_to_mel(fmax);
  for (int i = 0; i < n_mels + 2; i++) pts[i] = mel_to_hz(m0 + (m1 - m0) * i / (n_mels + 1));
  for (int m = 0; m < n_mels; m++) {
    const double enorm = 2.0 / (pts[m + 2] - pts[m]);
    for (int k = 0; k < kMelBins; k++) {
      const double f = fmax * k / (kMelBins - 1);
      const double lower = (f - pts[m]) / (pts[m + 1] - pts[m]);
      const double upper = (pts[m + 2] - f) / (pts[m + 2] - pts[m + 1]);
      w[(size_t)m * kMelBins + k] = std::max(0.0, std::min(lower, upper)) * enorm;
    }
  }
  return w;
}

static std::mutex g_mel_mu;
static MelTables g_mel[64][2];   // [device][80 mels, 128 mels]

static int mel_tables(int n_mels, MelTables** out) {
  if (n_mels != 80 && n_mels != 128)
    return fail(WX_ERR_UNSUPPORTED, "log_mel: n_mels %d (80 or 128)", n_mels);
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64) return fail(WX_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_mel_mu);
  MelTables& t = g_mel[dev][n_mels == 128];
  if (!t.dft) {
    // DFT matrix: element [n][q][g][e] is cos (q = 0, 1) or sin (q = 2, 3) of
    // 2 pi k n / 400 for bin k = 8 g + 4 (q & 1) + e; bins past 200 are zero
    std::vector<float> dft((size_t)kMelFFT * 4 * kMelGroups * 4, 0.0f), win(kMelFFT);
    const double two_pi = 6.283185307179586;
    for (int n = 0; n < kMelFFT; n++)
      for (int q = 0; q < 4; q++)
        for (int g = 0; g < kMelGroups; g++)
          for (int e = 0; e < 4; e++) {
            const int k = 8 * g + 4 * (q & 1) + e;
            if (k >= kMelBins) continue;
            const double a = two_pi * ((k * n) % kMelFFT) / kMelFFT;   // exact reduction
            dft[(((size_t)n * 4 + q) * kMelGroups + g) * 4 + e] =
                (float)(q < 2 ? std::cos(a) : std::sin(a));
          }
    for (int n = 0; n < kMelFFT; n++) win[n] = (float)(0.5 - 0.5 * std::cos(two_pi * n / kMelFFT));
    const std::vector<double> fb = slaney_filters(n_mels);
    std::vector<int> st(n_mels), len(n_mels);
    int maxw = 1;
    for (int m = 0; m < n_mels; m++) {
      int a = kMelBins, b = -1;
      for (int k = 0; k < kMelBins; k++)
        if (fb[(size_t)m * kMelBins + k] != 0.0) { a = std::min(a, k); b = std::max(b, k); }
      if (b < a) { a = 0; b = -1; }
      st[m] = a;
      len[m] = b - a + 1;
      maxw = std::max(maxw, len[m]);
    }
    std::vector<float> fw((size_t)n_mels * maxw, 0.0f);
    for (int m = 0; m < n_mels; m++)
      for (int i = 0; i < len[m]; i++) fw[(size_t)m * maxw + i] = (float)fb[(size_t)m * kMelBins + st[m] + i];
    MelTables nt;
    nt.n_mels = n_mels;
    nt.maxw = maxw;
    WX_CUDA_TRY(cudaMalloc(&nt.dft, dft.size() * 4));
    WX_CUDA_TRY(cudaMalloc(&nt.window, kMelFFT * 4));
    WX_CUDA_TRY(cudaMalloc(&nt.fw, fw.size() * 4));
    WX_CUDA_TRY(cudaMalloc(&nt.fstart, n_mels * 4));
    WX_CUDA_TRY(cudaMalloc(&nt.flen, n_mels * 4));
    WX_CUDA_TRY(cudaMemcpy(nt.dft, dft.data(), dft.size() * 4, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(nt.window, win.data(), kMelFFT * 4, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(nt.fw, fw.data(), fw.size() * 4, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(nt.fstart, st.data(), n_mels * 4, cudaMemcpyHostToDevice));
    WX_CUDA_TRY(cudaMemcpy(nt.flen, len.data(), n_mels * 4, cudaMemcpyHostToDevice));
    t = nt;
  }
  *out = &t;
  return WX_OK;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kMelThreads) log_mel_kernel(
    const float* __restrict__ audio, int64_t ld_audio, int64_t n_samples,
    const float* __restrict__ dft, const float* __restrict__ window,
    const int* __restrict__ fstart, const int* __restrict__ flen, const float* __restrict__ fw,
    int maxw, int n_mels, float* __restrict__ out, float* __restrict__ block_max) {
  extern __shared__ __align__(16) float msm[];
  float* xt = msm;                              // [400][36]: sample n, frame f
  float* slab = msm + kMelFFT * kMelXT;         // 2 slices of the DFT matrix
  float* power = slab;                          // [32][201], after the GEMM
  float* wmax = slab + 2 * kMelSlice;           // [7]
  const int b = blockIdx.y, f0 = blockIdx.x * kMelFB;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const float* a = audio + (int64_t)b * ld_audio;
  auto load_slice = [&](int sl, int buf) {
    const float4* src = reinterpret_cast<const float4*>(dft + (size_t)sl * kMelSlice);
    float4* dst = reinterpret_cast<float4*>(slab + buf * kMelSlice);
    for (int i = tid; i < kMelSlice / 4; i += kMelThreads) cp_async16(dst + i, src + i);
    cp_async_commit();
  };
  load_slice(0, 0);
  // windowed frames, transposed: sample j of the 30 s window is audio[j] below
  // n_samples and 0 above (pad_or_trim); positions outside the window reflect
  for (int i = tid; i < kMelFB * kMelFFT; i += kMelThreads) {
    const int f = i / kMelFFT, n = i - f * kMelFFT;
    float v = 0.0f;
    if (f0 + f < kMelFrames) {
      int64_t j = (int64_t)(f0 + f) * kMelHop + n - kMelFFT / 2;
      if (j < 0) j = -j;
      if (j >= kMelWindow) j = 2 * (kMelWindow - 1) - j;
      v = (j < n_samples ? __ldg(a + j) : 0.0f) * __ldg(window + n);
    }
    xt[n * kMelXT + f] = v;
  }
  // DFT: thread t < 208 takes frames 4 (t % 8) .. + 3 and bins 8 (t / 8) .. + 7
  const int fg = tid & 7, bg = tid >> 3;
  const bool active = tid < kMelCompute;
  float acc[4][16];
#pragma unroll
  for (int f = 0; f < 4; f++)
#pragma unroll
    for (int c = 0; c < 16; c++) acc[f][c] = 0.0f;
  constexpr int nsl = kMelFFT / kMelKS;
  for (int sl = 0; sl < nsl; sl++) {
    if (sl + 1 < nsl) {
      load_slice(sl + 1, (sl + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();   // slice sl (and, the first time, the frames) visible to all
    if (active) {
      const float* d = slab + (sl & 1) * kMelSlice + bg * 4;
#pragma unroll 4
      for (int kk = 0; kk < kMelKS; kk++) {
        const float4 x = *reinterpret_cast<const float4*>(xt + (sl * kMelKS + kk) * kMelXT + fg * 4);
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 w = *reinterpret_cast<const float4*>(d + (kk * 4 + q) * kMelGroups * 4);
#pragma unroll
          for (int f = 0; f < 4; f++) {
            acc[f][4 * q] = fmaf(xs[f], w.x, acc[f][4 * q]);
            acc[f][4 * q + 1] = fmaf(xs[f], w.y, acc[f][4 * q + 1]);
            acc[f][4 * q + 2] = fmaf(xs[f], w.z, acc[f][4 * q + 2]);
            acc[f][4 * q + 3] = fmaf(xs[f], w.w, acc[f][4 * q + 3]);
          }
        }
      }
    }
    __syncthreads();   // every thread is done with this slice before it is refilled
  }
  // |X|^2: cos sums in columns 0-7, sin sums in 8-15
  if (active) {
#pragma unroll
    for (int f = 0; f < 4; f++)
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int k = 8 * bg + e;
        if (k < kMelBins)
          power[(4 * fg + f) * kMelBins + k] = acc[f][e] * acc[f][e] + acc[f][8 + e] * acc[f][8 + e];
      }
  }
  __syncthreads();
  // mel bands, log10, the block's maximum
  float mx = -INFINITY;
  for (int m = warp; m < n_mels; m += kMelThreads / 32) {
    const int s0 = __ldg(fstart + m), len = __ldg(flen + m);
    const float* w = fw + (size_t)m * maxw;
    float acc = 0.0f;
    for (int i = 0; i < len; i++) acc = fmaf(__ldg(w + i), power[lane * kMelBins + s0 + i], acc);
    const float lv = log10f(fmaxf(acc, 1e-10f));
    if (f0 + lane < kMelFrames) {
      out[((int64_t)b * n_mels + m) * kMelFrames + f0 + lane] = lv;
      mx = fmaxf(mx, lv);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = wmax[0];
    for (int i = 1; i < kMelThreads / 32; i++) m = fmaxf(m, wmax[i]);
    block_max[(int64_t)b * kMelBlocks + blockIdx.x] = m;
  }
}

// floor at (clip maximum - 8), then (x + 4) / 4; grid (chunks, batch)
__global__ void __launch_bounds__(256) log_mel_finalize_kernel(float* __restrict__ out,
                                                               const float* __restrict__ block_max,
                                                               int n_mels) {
  __shared__ float clip_max;
  const int b = blockIdx.y;
  if (threadIdx.x < 32) {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < kMelBlocks; i += 32) m = fmaxf(m, block_max[(int64_t)b * kMelBlocks + i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) clip_max = m;
  }
  __syncthreads();
  const float lo = clip_max - 8.0f;
  float4* o4 = reinterpret_cast<float4*>(out + (int64_t)b * n_mels * kMelFrames);
  const int n4 = n_mels * kMelFrames / 4;       // 3000 frames: whole float4 per row
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    float4 v = o4[i];
    v.x = (fmaxf(v.x, lo) + 4.0f) * 0.25f;
    v.y = (fmaxf(v.y, lo) + 4.0f) * 0.25f;
    v.z = (fmaxf(v.z, lo) + 4.0f) * 0.25f;
    v.w = (fmaxf(v.w, lo) + 4.0f) * 0.25f;
    o4[i] = v;
  }
}

// per-device scratch for the block maxima, grown as batches grow
static std::mutex g_melsc_mu;
static float* g_melsc[64] = {nullptr};
static int64_t g_melsc_n[64] = {0};

static int mel_scratch(int64_t batch, float** out) {
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64) return fail(WX_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_melsc_mu);
  if (g_melsc_n[dev] < batch) {
    if (g_melsc[dev]) {
      WX_CUDA_TRY(cudaDeviceSynchronize());
      cudaFree(g_melsc[dev]);
      g_melsc[dev] = nullptr;
      g_melsc_n[dev] = 0;
    }
    WX_CUDA_TRY(cudaMalloc(&g_melsc[dev], (size_t)batch * kMelBlocks * 4));
    g_melsc_n[dev] = batch;
  }
  *out = g_melsc[dev];
  return WX_OK;
}

}  // namespace wx

extern "C" int wx_log_mel(const float* audio, int64_t batch, int64_t n_samples, int64_t ld_audio,
                          int n_mels, float* mel_out, void* stream) {
  using namespace wx;
  if (batch < 0 || n_samples < 0) return fail(WX_ERR_INVALID, "log_mel: negative size");
  if (batch == 0) return WX_OK;
  if (!mel_out || (n_samples > 0 && !audio)) return fail(WX_ERR_INVALID, "log_mel: NULL pointer");
  if (ld_audio < n_samples) return fail(WX_ERR_INVALID, "log_mel: ld_audio < n_samples");
  if (batch > 65535) return fail(WX_ERR_UNSUPPORTED, "log_mel: batch > 65535");
  if (reinterpret_cast<uintptr_t>(mel_out) & 15)
    return fail(WX_ERR_INVALID, "log_mel: mel_out must be 16-byte aligned");
  MelTables* t = nullptr;
  WX_TRY(mel_tables(n_mels, &t));
  float* bmax = nullptr;
  WX_TRY(mel_scratch(batch, &bmax));
  static bool attr[64] = {false};
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && !attr[dev]) {
    WX_CUDA_TRY(cudaFuncSetAttribute(log_mel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kMelSmem));
    attr[dev] = true;
  }
  cudaStream_t st = as_stream(stream);
  const int64_t n_used = std::min<int64_t>(n_samples, kMelWindow);
  log_mel_kernel<<<dim3(kMelBlocks, (unsigned)batch), kMelThreads, kMelSmem, st>>>(
      audio, ld_audio, n_used, t->dft, t->window, t->fstart, t->flen, t->fw, t->maxw, n_mels,
      mel_out, bmax);
  WX_TRY(check_launch("log_mel"));
  log_mel_finalize_kernel<<<dim3(16, (unsigned)batch), 256, 0, st>>>(mel_out, bmax, n_mels);
  return check_launch("log_mel_finalize");
}
