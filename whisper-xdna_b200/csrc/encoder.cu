// The Whisper encoder resident on one B200: bf16 weights, fp32 residual
// stream, and the forward pass as a fixed sequence of launches that is
// captured once per shape and replayed as a CUDA graph.
//
// Per clip batch (M = batch * T rows, T = n_frames / 2):
//   im2col(mel) -> conv1 GEMM + bias + GELU (bf16)         src/npu_whisper_encoder.py:444-448
//   im2col      -> conv2 GEMM + bias + GELU + positions    :450-458
//   per layer (:463-536):
//     LN (fp32 -> bf16)                  attn_ln
//     QKV GEMM + bias (bf16, fused [Wq; Wk; Wv])   the three bias-folded GEMMs :474-479
//     fused attention (bf16)             RawRT.attn_chain, src/rawxrt.py:813-891
//     out-proj GEMM + bias + residual    :512-514 (x updated in place, fp32)
//     LN (fp32 -> bf16)                  mlp_ln
//     fc1 GEMM + bias + GELU (bf16)      RawRT.mlp fc1 + g4f, src/rawxrt.py:459-544
//     fc2 GEMM + bias + residual         :525-527
//   ln_post (fp32 out)                   :538
// The reference's q * hd^-0.25 and k * hd^-0.25 scaling becomes one 1/sqrt(hd)
// on the scores inside the attention kernel.
//
// int8 mode (wx_encoder_set_quant; the reference's int8 probe,
// bench/probe_int8_decode.py:48-74 with :140-142): the conv, QKV, out-proj,
// fc1 and fc2 GEMMs take int8 operands on the int8 tensor cores. Weights are
// quantised once per output channel (or per weight matrix, per q/k/v and per
// fc1 column chunk of prepare_mlp_chunks for "pertensor"); each GEMM's
// activation rows are quantised per token right before it:
//   im2col (bf16) -> quantise -> conv GEMM          LN + quantise (one kernel) -> QKV
//   attention (bf16) -> quantise -> out-proj          LN + quantise (one kernel) -> fc1
//   fc1 + GELU (bf16, with max |row| by atomics) -> quantise -> fc2
// Attention itself stays bf16 (the probe keeps it in fp32: E.np_matmul).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

// ---------------------------------------------------------------- kernels

// fp32 -> bf16 (RNE), optionally with the conv2 column permutation
// dst[o][j*C + c] = src[o][c][j] (conv weight (O, C, 3) read j-major, so that
// an im2col row is three whole rows of the previous activation).
__global__ void convert_bf16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst,
                                    int64_t n, int conv_C) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t si = i;
    if (conv_C > 0) {  // i = o*(3C) + j*C + c  ->  src o*(3C) + c*3 + j
      const int64_t o = i / (3 * conv_C), rem = i % (3 * conv_C);
      const int64_t j = rem / conv_C, c = rem % conv_C;
      si = o * 3 * conv_C + c * 3 + j;
    }
    dst[i] = (uint16_t)bf16_bits<RND_RNE>(src[si]);
  }
}

// fp32 copy with the same optional conv2 column permutation (int8 weights are
// quantised from the permuted fp32 matrix)
__global__ void permute_f32_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                   int64_t n, int conv_C) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / (3 * conv_C), rem = i % (3 * conv_C);
    const int64_t j = rem / conv_C, c = rem % conv_C;
    dst[i] = src[o * 3 * conv_C + c * 3 + j];
  }
}

// conv1 im2col: mel (batch, C, F) fp32 -> A (batch*F, 3C) bf16 with column
// c*3 + j = mel[b, c, t + j - 1] (zero outside [0, F)); the column order of the
// conv weight reshaped (O, C*3) (src/npu_whisper_encoder.py:422-431). One block
// per 32 frames: the mel tile is staged in shared memory so reads run along
// time and writes along the row.
__global__ void __launch_bounds__(256) im2col_conv1_kernel(const float* __restrict__ mel,
                                                           uint16_t* __restrict__ A, int C, int F,
                                                           const float* const* __restrict__ mel_ind) {
  pdl_launch_dependents();
  pdl_wait();   // the input (and the graph's buffer pointers) come from earlier work
  if (mel_ind) mel = *mel_ind;   // graph replays read the current input from here
  extern __shared__ float tile[];  // C x 34
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * 32;
  const float* m = mel + (int64_t)b * C * F;
  for (int i = threadIdx.x; i < C * 34; i += blockDim.x) {
    const int c = i / 34, dt = i % 34;
    const int t = t0 - 1 + dt;
    tile[i] = (t >= 0 && t < F) ? m[(int64_t)c * F + t] : 0.0f;
  }
  __syncthreads();
  const int K = 3 * C;
  for (int i = threadIdx.x; i < 32 * K; i += blockDim.x) {
    const int r = i / K, col = i % K;
    const int t = t0 + r;
    if (t >= F) continue;
    const int c = col / 3, j = col % 3;
    A[((int64_t)b * F + t) * K + col] = (uint16_t)bf16_bits<RND_RNE>(tile[c * 34 + r + j]);
  }
}

// The input and output pointers of one graph replay, written on the replay's
// stream just before it: a captured forward reads mel and writes out through
// them, so one graph per (batch, frames) serves every pair of buffers.
struct IoPtrs {
  const float* mel;
  float* out;
};
__global__ void set_io_kernel(IoPtrs* io, const float* mel, float* out) {
  io->mel = mel;
  io->out = out;
}

// conv2 im2col with the j-major weight: A (batch*T, 3d) row t of clip b is
// [x1[2t-1], x1[2t], x1[2t+1]] (rows of the conv1 output, zero outside the
// clip), copied 16 bytes at a time.
__global__ void __launch_bounds__(256) im2col_conv2_kernel(const uint16_t* __restrict__ x1,
                                                           uint16_t* __restrict__ A, int64_t rows,
                                                           int T, int d) {
  pdl_launch_dependents();
  pdl_wait();   // the conv1 output comes from the previous kernel
  const int vpr = 3 * d / 8;  // 16-byte vectors per output row
  const int64_t total = rows * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vpr;
    const int v = (int)(i % vpr);
    const int j = (v * 8) / d, c = (v * 8) % d;
    const int64_t b = r / T;
    const int t = (int)(r % T);
    const int src_t = 2 * t + j - 1;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (src_t >= 0 && src_t < 2 * T)
      val = __ldg(reinterpret_cast<const uint4*>(x1 + ((b * 2 * T + src_t) * (int64_t)d + c)));
    reinterpret_cast<uint4*>(A + r * 3 * (int64_t)d)[v] = val;
  }
}

// ---------------------------------------------------------------- engine

struct LayerW {
  uint16_t *wqkv, *wo, *w1, *w2;                    // bf16, (out, in)
  float *bqkv, *bo, *b1, *b2;                       // fp32
  float *ln1_g, *ln1_b, *ln2_g, *ln2_b;             // fp32
  // int8 mode: the same weights quantised per output channel, and the scales
  int8_t *qqkv = nullptr, *qo = nullptr, *q1 = nullptr, *q2 = nullptr;
  float *sqkv = nullptr, *so = nullptr, *s1 = nullptr, *s2 = nullptr;
};

struct Plans {
  GemmPlan conv1, conv2;
  std::vector<GemmPlan> qkv, out, fc1, fc2;
  AttnPlan attn;
};

struct GraphKey {
  int64_t batch, frames;
  bool operator<(const GraphKey& o) const {
    return std::tie(batch, frames) < std::tie(o.batch, o.frames);
  }
};

}  // namespace wx

struct wx_encoder {
  int n_mels, d, nh, nl, ffn, n_ctx, max_batch, gelu_mode;
  int device;
  bool pdl = true;   // programmatic dependent launches in the forward (WXB200_PDL=0: off)
  std::vector<void*> allocs;
  int64_t bytes = 0;
  // weights
  uint16_t *conv1_w = nullptr, *conv2_w = nullptr;
  float *conv1_b = nullptr, *conv2_b = nullptr, *pos = nullptr;
  float *lnp_g = nullptr, *lnp_b = nullptr;
  std::vector<wx::LayerW> L;
  // workspace
  float* x = nullptr;         // (B*T, d) fp32 residual stream
  uint16_t* h = nullptr;      // (B*T, d) bf16 LN output
  uint16_t* qkv = nullptr;    // (B*T, 3d) bf16; also conv1 output (B*2T, d)
  uint16_t* o = nullptr;      // (B*T, d) bf16 attention output
  uint16_t* f = nullptr;      // (B*T, ffn) bf16; also the im2col buffers
  float* mel_dev = nullptr;   // (B, n_mels, 2*n_ctx) staging for host input
  float* out_dev = nullptr;   // (B, n_ctx, d) staging for host output
  wx::IoPtrs* io = nullptr;   // input / output pointers of the next graph replay
  float* stage = nullptr;     // fp32 upload staging for weights
  float* stage2 = nullptr;    // int8 mode: permuted fp32 weights
  int64_t stage_n = 0;
  // int8 mode (WX_QUANT_*)
  int quant = 0;
  int8_t *conv1_q = nullptr, *conv2_q = nullptr;
  float *conv1_s = nullptr, *conv2_s = nullptr;
  int8_t* aq = nullptr;       // (B*T, d) int8: the quantised LN / attention output
  int8_t* fq = nullptr;       // int8 fc1 output (B*T, ffn) and conv im2col rows
  float* sa = nullptr;        // per-row scales of aq / fq (2*B*T)
  float* rowmax = nullptr;    // (B*T) max |fc1 output| per row
  float* gmax = nullptr;      // one weight matrix's max |w| ("pertensor")
  bool set_front = false, set_post = false;
  std::vector<bool> set_layer;
  std::map<std::pair<int64_t, int64_t>, wx::Plans*> plans;
  std::map<wx::GraphKey, cudaGraphExec_t> graphs;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  // the host-buffer entry point's pipeline: copy-in, compute and copy-out
  // streams, and per-chunk events
  static constexpr int kHostChunks = 2;
  cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
  cudaEvent_t ev_start = nullptr, ev_end = nullptr;
  cudaEvent_t ev_h2d[kHostChunks] = {}, ev_done[kHostChunks] = {};
  // the pipelined host entry point (submit / wait): two staging slots, slot 0
  // is mel_dev / out_dev, slot 1 is allocated on first use
  float* mel_dev1 = nullptr;
  float* out_dev1 = nullptr;
  cudaEvent_t ev_q_in[2] = {}, ev_q_comp[2] = {}, ev_q_out[2] = {};
  bool q_busy[2] = {false, false};
  int q_next = 0;
  std::mutex mu;
};

namespace wx {

static int dalloc(wx_encoder* e, void** p, int64_t bytes) {
  cudaError_t r = cudaMalloc(p, (size_t)bytes);
  if (r != cudaSuccess) {
    *p = nullptr;
    cudaGetLastError();   // an allocation failure is not a launch error of a later kernel
    return fail(WX_ERR_NOMEM, "cudaMalloc(%lld) failed: %s", (long long)bytes, cudaGetErrorString(r));
  }
  e->allocs.push_back(*p);
  e->bytes += bytes;
  return WX_OK;
}

// release one of the encoder's allocations before the encoder itself goes
static void dfree(wx_encoder* e, void** p, int64_t bytes) {
  if (!*p) return;
  auto it = std::find(e->allocs.begin(), e->allocs.end(), *p);
  if (it != e->allocs.end()) {
    e->allocs.erase(it);
    e->bytes -= bytes;
  }
  cudaFree(*p);
  *p = nullptr;
}

static int upload_f32(wx_encoder* e, float* dst, const float* src, int64_t n) {
  if (!src) return fail(WX_ERR_INVALID, "encoder: NULL weight pointer");
  WX_CUDA_TRY(cudaMemcpy(dst, src, (size_t)n * 4, cudaMemcpyHostToDevice));
  (void)e;
  return WX_OK;
}

static int upload_bf16(wx_encoder* e, uint16_t* dst, const float* src, int64_t n, int conv_C) {
  if (!src) return fail(WX_ERR_INVALID, "encoder: NULL weight pointer");
  if (n > e->stage_n) return fail(WX_ERR_INVALID, "encoder: staging too small");
  WX_CUDA_TRY(cudaMemcpy(e->stage, src, (size_t)n * 4, cudaMemcpyHostToDevice));
  convert_bf16_kernel<<<1024, 256>>>(e->stage, dst, n, conv_C);
  WX_TRY(check_launch("convert_bf16"));
  WX_CUDA_TRY(cudaDeviceSynchronize());
  return WX_OK;
}

// int8 mode: quantise a weight (rows x cols fp32 on the host, conv_C > 0 for
// the conv2 column permutation) into dst with one scale per row (output
// channel). "pertensor" uses one scale per group of group_rows rows: the
// whole matrix, or one of q / k / v, or one fc1 column chunk.
static int upload_i8(wx_encoder* e, int8_t* dst, float* scale, const float* src, int64_t rows,
                     int64_t cols, int conv_C, int64_t group_rows) {
  if (!src) return fail(WX_ERR_INVALID, "encoder: NULL weight pointer");
  const int64_t n = rows * cols;
  if (n > e->stage_n) return fail(WX_ERR_INVALID, "encoder: staging too small");
  WX_CUDA_TRY(cudaMemcpy(e->stage, src, (size_t)n * 4, cudaMemcpyHostToDevice));
  const float* w = e->stage;
  if (conv_C > 0) {
    permute_f32_kernel<<<1024, 256>>>(e->stage, e->stage2, n, conv_C);
    WX_TRY(check_launch("permute_f32"));
    w = e->stage2;
  }
  if (e->quant == WX_QUANT_INT8_PERCHAN) {
    WX_TRY(launch_quantize_rows(w, WX_DTYPE_F32, rows, cols, cols, nullptr, 0, dst, cols, scale, 0));
  } else {
    for (int64_t g = 0; g < rows; g += group_rows) {
      const int64_t gr = std::min(group_rows, rows - g);
      WX_CUDA_TRY(cudaMemset(e->gmax, 0, 4));
      WX_TRY(launch_absmax_rows(w + g * cols, WX_DTYPE_F32, gr, cols, cols, e->gmax, 0, 0));
      WX_TRY(launch_quantize_rows(w + g * cols, WX_DTYPE_F32, gr, cols, cols, e->gmax, 0,
                                  dst + g * cols, cols, scale + g, 0));
    }
  }
  WX_CUDA_TRY(cudaDeviceSynchronize());
  return WX_OK;
}

// fc1's column chunk in the reference's prepare_mlp_chunks(W, n_layer, d, 0)
// (src/npu_whisper_encoder.py:383-398): the whole width up to 4096, else d
// when d divides it, else an even split.
static int64_t fc1_chunk(int64_t ffn, int64_t d) {
  if (ffn <= 4096) return ffn;
  if (ffn % d == 0) return d;
  return ffn / ((ffn + 4095) / 4096);
}

static int build_plans(wx_encoder* e, int64_t B, int64_t T, Plans** out) {
  auto it = e->plans.find({B, T});
  if (it != e->plans.end()) {
    *out = it->second;
    return WX_OK;
  }
  Plans* p = new Plans();
  const int64_t M = B * T, F2 = 2 * T, d = e->d, ffn = e->ffn;
  const int64_t K1 = 3 * (int64_t)e->n_mels;
  const int gelu_bf16 = e->gelu_mode == WX_GELU_ERF ? WX_EPI_BF16_GELU_ERF : WX_EPI_BF16_GELU;
  const int gelu_pos = e->gelu_mode == WX_GELU_ERF ? kEpiF32GeluErfPos : kEpiF32GeluPos;
  int s = WX_OK;
  if (e->quant) {
    // int8 GEMMs: conv inputs quantised into fq, LN / attention outputs into aq
    s = gemm_plan_i8(&p->conv1, e->fq, e->conv1_q, e->sa, e->conv1_s, e->conv1_b, nullptr, e->qkv,
                     B * F2, d, K1, K1, K1, d, 0, gelu_bf16, nullptr);
    if (s == WX_OK)
      s = gemm_plan_i8(&p->conv2, e->fq, e->conv2_q, e->sa, e->conv2_s, e->conv2_b, nullptr, e->x,
                       M, d, 3 * d, 3 * d, 3 * d, d, 0, gelu_pos, nullptr);
    if (s == WX_OK) gemm_set_pos(&p->conv2, e->pos, d, (int)T);
    p->qkv.resize(e->nl);
    p->out.resize(e->nl);
    p->fc1.resize(e->nl);
    p->fc2.resize(e->nl);
    for (int l = 0; s == WX_OK && l < e->nl; l++) {
      const LayerW& w = e->L[l];
      s = gemm_plan_i8(&p->qkv[l], e->aq, w.qqkv, e->sa, w.sqkv, w.bqkv, nullptr, e->qkv, M, 3 * d,
                       d, d, d, 3 * d, 0, WX_EPI_BF16, nullptr);
      if (s == WX_OK)
        s = gemm_plan_i8(&p->out[l], e->aq, w.qo, e->sa, w.so, w.bo, e->x, e->x, M, d, d, d, d, d,
                         d, WX_EPI_F32_RESID, nullptr);
      if (s == WX_OK)
        s = gemm_plan_i8(&p->fc1[l], e->aq, w.q1, e->sa, w.s1, w.b1, nullptr, e->f, M, ffn, d, d, d,
                         ffn, 0, gelu_bf16, e->rowmax);
      if (s == WX_OK)
        s = gemm_plan_i8(&p->fc2[l], e->fq, w.q2, e->sa, w.s2, w.b2, e->x, e->x, M, d, ffn, ffn, ffn,
                         d, d, WX_EPI_F32_RESID, nullptr);
    }
  }
  // conv1: A1 (B*2T, 3*n_mels) in f, out x1 (B*2T, d) in qkv
  if (s == WX_OK && !e->quant)
    s = gemm_plan(&p->conv1, e->f, e->conv1_w, e->conv1_b, nullptr, e->qkv, B * F2, d, K1, K1, K1,
                  d, 0, gelu_bf16, 0);
  // conv2: A2 (B*T, 3d) in f, out x fp32 (+ positions)
  if (s == WX_OK && !e->quant)
    s = gemm_plan(&p->conv2, e->f, e->conv2_w, e->conv2_b, nullptr, e->x, M, d, 3 * d, 3 * d,
                  3 * d, d, 0, gelu_pos, 0);
  if (s == WX_OK && !e->quant) gemm_set_pos(&p->conv2, e->pos, d, (int)T);
  if (!e->quant) {
    p->qkv.resize(e->nl);
    p->out.resize(e->nl);
    p->fc1.resize(e->nl);
    p->fc2.resize(e->nl);
  }
  for (int l = 0; s == WX_OK && !e->quant && l < e->nl; l++) {
    const LayerW& w = e->L[l];
    s = gemm_plan(&p->qkv[l], e->h, w.wqkv, w.bqkv, nullptr, e->qkv, M, 3 * d, d, d, d, 3 * d, 0,
                  WX_EPI_BF16, 0);
    if (s == WX_OK)
      s = gemm_plan(&p->out[l], e->o, w.wo, w.bo, e->x, e->x, M, d, d, d, d, d, d,
                    WX_EPI_F32_RESID, 0);
    if (s == WX_OK)
      s = gemm_plan(&p->fc1[l], e->h, w.w1, w.b1, nullptr, e->f, M, ffn, d, d, d, ffn, 0,
                    gelu_bf16, 0);
    if (s == WX_OK)
      s = gemm_plan(&p->fc2[l], e->f, w.w2, w.b2, e->x, e->x, M, d, ffn, ffn, ffn, d, d,
                    WX_EPI_F32_RESID, 0);
  }
  if (s == WX_OK)
    s = attn_plan(&p->attn, e->qkv, e->qkv + d, e->qkv + 2 * d, e->o, B, e->nh, T, d / e->nh,
                  3 * d, 3 * d, 3 * d, d, 1.0f / sqrtf((float)(d / e->nh)));
  if (s != WX_OK) {
    delete p;
    return s;
  }
  e->plans[{B, T}] = p;
  *out = p;
  return WX_OK;
}

// LayerNorm of the residual stream quantised per token into aq / sa: one
// fused kernel up to width 2048, else LN to fp32 (in h32) and a quantise pass.
static int ln_quant(wx_encoder* e, const float* x, const float* g, const float* b, float* h32,
                    int64_t M, cudaStream_t st) {
  const int64_t d = e->d;
  if (d <= 2048)
    return launch_layernorm_quant_rows(x, g, b, e->aq, e->sa, M, d, d, d, 1e-5f, st);
  WX_TRY(launch_layernorm_rows(x, WX_DTYPE_F32, g, b, h32, WX_DTYPE_F32, M, d, d, d, 1e-5f,
                               WX_LN_FP32, WX_ROUND_RNE, st));
  return launch_quantize_rows(h32, WX_DTYPE_F32, M, d, d, nullptr, 0, e->aq, d, e->sa, st);
}

// The launch sequence of one int8-mode forward pass.
static int forward_launches_i8(wx_encoder* e, Plans* p, const float* mel, float* out, int64_t B,
                               int64_t T, cudaStream_t st, const IoPtrs* io) {
  const int64_t M = B * T, F2 = 2 * T, d = e->d, ffn = e->ffn, K1 = 3 * (int64_t)e->n_mels;
  float* h32 = reinterpret_cast<float*>(e->f);   // fp32 LN output (f holds M*ffn bf16)
  {
    const size_t smem = (size_t)e->n_mels * 34 * 4;
    dim3 grid((unsigned)((F2 + 31) / 32), (unsigned)B);
    WX_CUDA_TRY(launch_k(im2col_conv1_kernel, grid, dim3(256), smem, st, mel, e->f, e->n_mels,
                         (int)F2, io ? &io->mel : nullptr));
    WX_TRY(check_launch("im2col_conv1"));
  }
  WX_TRY(launch_quantize_rows(e->f, WX_DTYPE_BF16, B * F2, K1, K1, nullptr, 0, e->fq, K1, e->sa, st));
  WX_TRY(gemm_run(p->conv1, st));
  {
    const int64_t total = M * (3 * d / 8);
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
    WX_CUDA_TRY(launch_k(im2col_conv2_kernel, dim3(grid), dim3(256), 0, st,
                         const_cast<const uint16_t*>(e->qkv), e->f, M, (int)T, (int)d));
    WX_TRY(check_launch("im2col_conv2"));
  }
  WX_TRY(launch_quantize_rows(e->f, WX_DTYPE_BF16, M, 3 * d, 3 * d, nullptr, 0, e->fq, 3 * d, e->sa,
                              st));
  WX_TRY(gemm_run(p->conv2, st));
  for (int l = 0; l < e->nl; l++) {
    const LayerW& w = e->L[l];
    WX_TRY(ln_quant(e, e->x, w.ln1_g, w.ln1_b, h32, M, st));
    WX_TRY(gemm_run(p->qkv[l], st));
    WX_TRY(attn_run(p->attn, st));
    WX_TRY(launch_quantize_rows(e->o, WX_DTYPE_BF16, M, d, d, nullptr, 0, e->aq, d, e->sa, st));
    WX_TRY(gemm_run(p->out[l], st));
    WX_TRY(ln_quant(e, e->x, w.ln2_g, w.ln2_b, h32, M, st));
    WX_CUDA_TRY(cudaMemsetAsync(e->rowmax, 0, (size_t)M * 4, st));
    {
      PdlScope after_memset(false);   // its predecessor is the memset, not a kernel
      WX_TRY(gemm_run(p->fc1[l], st));
    }
    WX_TRY(launch_quantize_rows(e->f, WX_DTYPE_BF16, M, ffn, ffn, e->rowmax, 1, e->fq, ffn, e->sa,
                                st));
    WX_TRY(gemm_run(p->fc2[l], st));
  }
  WX_TRY(launch_layernorm_rows(e->x, WX_DTYPE_F32, e->lnp_g, e->lnp_b, out, WX_DTYPE_F32, M, d, d,
                               d, 1e-5f, WX_LN_FP32, WX_ROUND_RNE, st,
                               io ? reinterpret_cast<void* const*>(&io->out) : nullptr));
  return WX_OK;
}

// The launch sequence of one forward pass.
// io: when not NULL (graph capture), the first kernel reads mel and the last
// writes out through it instead of the pointers given.
//
// For batches of up to kPdlMaxBatch clips every kernel is launched as a
// programmatic dependent of the one before it (PdlScope; WXB200_PDL=0 in the
// environment turns it off): its launch and prologue overlap the previous
// kernel's last wave, and it waits (pdl_wait) before touching memory. A
// forward is 229 launches; measured on a B200, large-v3 at one clip: 4.35 ->
// 4.25 ms per forward. At 64 clips the same launches measured 2% slower, so
// large batches launch plainly.
constexpr int64_t kPdlMaxBatch = 4;
static int forward_launches(wx_encoder* e, Plans* p, const float* mel, float* out, int64_t B,
                            int64_t T, cudaStream_t st, const IoPtrs* io) {
  PdlScope pdl(e->pdl && B <= kPdlMaxBatch);
  if (e->quant) return forward_launches_i8(e, p, mel, out, B, T, st, io);
  const int64_t M = B * T, F2 = 2 * T, d = e->d;
  {
    const size_t smem = (size_t)e->n_mels * 34 * 4;
    dim3 grid((unsigned)((F2 + 31) / 32), (unsigned)B);
    WX_CUDA_TRY(launch_k(im2col_conv1_kernel, grid, dim3(256), smem, st, mel, e->f, e->n_mels,
                         (int)F2, io ? &io->mel : nullptr));
    WX_TRY(check_launch("im2col_conv1"));
  }
  WX_TRY(gemm_run(p->conv1, st));
  {
    const int64_t total = M * (3 * d / 8);
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
    WX_CUDA_TRY(launch_k(im2col_conv2_kernel, dim3(grid), dim3(256), 0, st,
                         const_cast<const uint16_t*>(e->qkv), e->f, M, (int)T, (int)d));
    WX_TRY(check_launch("im2col_conv2"));
  }
  WX_TRY(gemm_run(p->conv2, st));
  for (int l = 0; l < e->nl; l++) {
    const LayerW& w = e->L[l];
    WX_TRY(launch_layernorm_rows(e->x, WX_DTYPE_F32, w.ln1_g, w.ln1_b, e->h, WX_DTYPE_BF16, M, d,
                                 d, d, 1e-5f, WX_LN_FP32, WX_ROUND_RNE, st));
    WX_TRY(gemm_run(p->qkv[l], st));
    WX_TRY(attn_run(p->attn, st));
    WX_TRY(gemm_run(p->out[l], st));
    WX_TRY(launch_layernorm_rows(e->x, WX_DTYPE_F32, w.ln2_g, w.ln2_b, e->h, WX_DTYPE_BF16, M, d,
                                 d, d, 1e-5f, WX_LN_FP32, WX_ROUND_RNE, st));
    WX_TRY(gemm_run(p->fc1[l], st));
    WX_TRY(gemm_run(p->fc2[l], st));
  }
  WX_TRY(launch_layernorm_rows(e->x, WX_DTYPE_F32, e->lnp_g, e->lnp_b, out, WX_DTYPE_F32, M, d, d,
                               d, 1e-5f, WX_LN_FP32, WX_ROUND_RNE, st,
                               io ? reinterpret_cast<void* const*>(&io->out) : nullptr));
  return WX_OK;
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_encoder_create(wx_encoder** out, int n_mels, int d_model, int n_head, int n_layer, int ffn,
                      int n_ctx, int max_batch, int gelu_mode) {
  if (!out) return fail(WX_ERR_INVALID, "encoder_create: out is NULL");
  *out = nullptr;
  if (n_mels <= 0 || d_model <= 0 || n_head <= 0 || n_layer <= 0 || ffn <= 0 || n_ctx <= 0 ||
      max_batch <= 0)
    return fail(WX_ERR_INVALID, "encoder_create: sizes must be > 0");
  if (d_model % n_head || d_model / n_head != 64)
    return fail(WX_ERR_UNSUPPORTED, "encoder_create: head dim must be 64");
  if (d_model % 64 || ffn % 64 || (3 * n_mels) % 8)
    return fail(WX_ERR_UNSUPPORTED, "encoder_create: d_model and ffn must be multiples of 64, "
                "3*n_mels a multiple of 8");
  if (gelu_mode != WX_GELU_POLY4 && gelu_mode != WX_GELU_ERF)
    return fail(WX_ERR_INVALID, "encoder_create: gelu_mode %d", gelu_mode);
  if (!device_error_word()) return fail(WX_ERR_CUDA, "encoder_create: no device");
  wx_encoder* e = new wx_encoder();
  e->n_mels = n_mels; e->d = d_model; e->nh = n_head; e->nl = n_layer; e->ffn = ffn;
  e->n_ctx = n_ctx; e->max_batch = max_batch; e->gelu_mode = gelu_mode;
  cudaGetDevice(&e->device);
  e->set_layer.assign(n_layer, false);
  if (const char* v = getenv("WXB200_PDL")) e->pdl = atoi(v) != 0;
  const int64_t d = d_model, B = max_batch, T = n_ctx;
  int s = WX_OK;
  auto A = [&](void** p, int64_t bytes) { if (s == WX_OK) s = dalloc(e, p, bytes); };
  A((void**)&e->conv1_w, d * 3 * n_mels * 2);
  A((void**)&e->conv2_w, d * 3 * d * 2);
  A((void**)&e->conv1_b, d * 4);
  A((void**)&e->conv2_b, d * 4);
  A((void**)&e->pos, T * d * 4);
  A((void**)&e->lnp_g, d * 4);
  A((void**)&e->lnp_b, d * 4);
  e->L.resize(n_layer);
  for (int l = 0; l < n_layer; l++) {
    LayerW& w = e->L[l];
    A((void**)&w.wqkv, 3 * d * d * 2);
    A((void**)&w.wo, d * d * 2);
    A((void**)&w.w1, (int64_t)ffn * d * 2);
    A((void**)&w.w2, (int64_t)ffn * d * 2);
    A((void**)&w.bqkv, 3 * d * 4);
    A((void**)&w.bo, d * 4);
    A((void**)&w.b1, (int64_t)ffn * 4);
    A((void**)&w.b2, d * 4);
    A((void**)&w.ln1_g, d * 4);
    A((void**)&w.ln1_b, d * 4);
    A((void**)&w.ln2_g, d * 4);
    A((void**)&w.ln2_b, d * 4);
  }
  const int64_t M = B * T;
  // f holds the MLP activation, the conv1 im2col (2T rows x 3*n_mels) and the
  // conv2 im2col (T rows x 3d); qkv also holds the conv1 output (2T x d).
  int64_t f_elems = std::max(M * ffn, std::max(B * 2 * T * 3 * (int64_t)n_mels, M * 3 * d));
  int64_t qkv_elems = std::max(M * 3 * d, B * 2 * T * d);
  A((void**)&e->x, M * d * 4);
  A((void**)&e->h, M * d * 2);
  A((void**)&e->qkv, qkv_elems * 2);
  A((void**)&e->o, M * d * 2);
  A((void**)&e->f, f_elems * 2);
  A((void**)&e->mel_dev, B * n_mels * 2 * T * 4);
  A((void**)&e->out_dev, M * d * 4);
  A((void**)&e->io, sizeof(IoPtrs));
  e->stage_n = std::max((int64_t)ffn * d, std::max(3 * d * d, T * d));
  A((void**)&e->stage, e->stage_n * 4);
  if (s == WX_OK) {
    bool good = cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking) == cudaSuccess &&
                cudaEventCreateWithFlags(&e->ev_in, cudaEventDisableTiming) == cudaSuccess &&
                cudaEventCreateWithFlags(&e->ev_out, cudaEventDisableTiming) == cudaSuccess &&
                cudaStreamCreateWithFlags(&e->s_in, cudaStreamNonBlocking) == cudaSuccess &&
                cudaStreamCreateWithFlags(&e->s_comp, cudaStreamNonBlocking) == cudaSuccess &&
                cudaStreamCreateWithFlags(&e->s_out, cudaStreamNonBlocking) == cudaSuccess &&
                cudaEventCreateWithFlags(&e->ev_start, cudaEventDisableTiming) == cudaSuccess &&
                cudaEventCreateWithFlags(&e->ev_end, cudaEventDisableTiming) == cudaSuccess;
    for (int k = 0; good && k < wx_encoder::kHostChunks; k++)
      good = cudaEventCreateWithFlags(&e->ev_h2d[k], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&e->ev_done[k], cudaEventDisableTiming) == cudaSuccess;
    for (int k = 0; good && k < 2; k++)
      good = cudaEventCreateWithFlags(&e->ev_q_in[k], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&e->ev_q_comp[k], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&e->ev_q_out[k], cudaEventDisableTiming) == cudaSuccess;
    if (!good) s = fail(WX_ERR_CUDA, "encoder_create: stream/event creation failed");
  }
  if (s != WX_OK) {
    wx_encoder_destroy(e);
    return s;
  }
  *out = e;
  return WX_OK;
}

int wx_encoder_destroy(wx_encoder* e) {
  if (!e) return WX_OK;
  DeviceGuard dg(e->device);
  // submitted batches finish writing their host buffers first
  for (int k = 0; k < 2; k++)
    if (e->q_busy[k]) cudaEventSynchronize(e->ev_q_out[k]);
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : e->plans) delete kv.second;
  for (void* p : e->allocs) cudaFree(p);
  if (e->side) cudaStreamDestroy(e->side);
  if (e->ev_in) cudaEventDestroy(e->ev_in);
  if (e->ev_out) cudaEventDestroy(e->ev_out);
  for (cudaStream_t x : {e->s_in, e->s_comp, e->s_out})
    if (x) cudaStreamDestroy(x);
  for (cudaEvent_t x : {e->ev_start, e->ev_end})
    if (x) cudaEventDestroy(x);
  for (int k = 0; k < wx_encoder::kHostChunks; k++) {
    if (e->ev_h2d[k]) cudaEventDestroy(e->ev_h2d[k]);
    if (e->ev_done[k]) cudaEventDestroy(e->ev_done[k]);
  }
  for (int k = 0; k < 2; k++)
    for (cudaEvent_t x : {e->ev_q_in[k], e->ev_q_comp[k], e->ev_q_out[k]})
      if (x) cudaEventDestroy(x);
  delete e;
  return WX_OK;
}

int wx_encoder_set_frontend(wx_encoder* e, const float* conv1_w, const float* conv1_b,
                            const float* conv2_w, const float* conv2_b, const float* pos) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  const int64_t d = e->d;
  if (e->quant) {
    const int64_t k1 = 3 * (int64_t)e->n_mels;
    WX_TRY(upload_i8(e, e->conv1_q, e->conv1_s, conv1_w, d, k1, 0, d));
    WX_TRY(upload_i8(e, e->conv2_q, e->conv2_s, conv2_w, d, 3 * d, (int)d, d));
  } else {
    WX_TRY(upload_bf16(e, e->conv1_w, conv1_w, d * 3 * e->n_mels, 0));
    WX_TRY(upload_bf16(e, e->conv2_w, conv2_w, d * 3 * d, (int)d));
  }
  WX_TRY(upload_f32(e, e->conv1_b, conv1_b, d));
  WX_TRY(upload_f32(e, e->conv2_b, conv2_b, d));
  WX_TRY(upload_f32(e, e->pos, pos, (int64_t)e->n_ctx * d));
  e->set_front = true;
  return WX_OK;
}

int wx_encoder_set_layer(wx_encoder* e, int layer, const float* attn_ln_w, const float* attn_ln_b,
                         const float* wq, const float* bq, const float* wk, const float* wv,
                         const float* bv, const float* wo, const float* bo, const float* mlp_ln_w,
                         const float* mlp_ln_b, const float* w1, const float* b1, const float* w2,
                         const float* b2) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  if (layer < 0 || layer >= e->nl) return fail(WX_ERR_INVALID, "encoder: layer %d", layer);
  const int64_t d = e->d, ffn = e->ffn;
  LayerW& w = e->L[layer];
  if (e->quant) {
    WX_TRY(upload_i8(e, w.qqkv, w.sqkv, wq, d, d, 0, d));
    WX_TRY(upload_i8(e, w.qqkv + d * d, w.sqkv + d, wk, d, d, 0, d));
    WX_TRY(upload_i8(e, w.qqkv + 2 * d * d, w.sqkv + 2 * d, wv, d, d, 0, d));
    WX_TRY(upload_i8(e, w.qo, w.so, wo, d, d, 0, d));
    WX_TRY(upload_i8(e, w.q1, w.s1, w1, ffn, d, 0, fc1_chunk(ffn, d)));
    WX_TRY(upload_i8(e, w.q2, w.s2, w2, d, ffn, 0, d));
  } else {
    WX_TRY(upload_bf16(e, w.wqkv, wq, d * d, 0));
    WX_TRY(upload_bf16(e, w.wqkv + d * d, wk, d * d, 0));
    WX_TRY(upload_bf16(e, w.wqkv + 2 * d * d, wv, d * d, 0));
    WX_TRY(upload_bf16(e, w.wo, wo, d * d, 0));
    WX_TRY(upload_bf16(e, w.w1, w1, ffn * d, 0));
    WX_TRY(upload_bf16(e, w.w2, w2, ffn * d, 0));
  }
  WX_TRY(upload_f32(e, w.bqkv, bq, d));
  WX_CUDA_TRY(cudaMemset(w.bqkv + d, 0, d * 4));  // the key projection has no bias
  WX_TRY(upload_f32(e, w.bqkv + 2 * d, bv, d));
  WX_TRY(upload_f32(e, w.bo, bo, d));
  WX_TRY(upload_f32(e, w.b1, b1, ffn));
  WX_TRY(upload_f32(e, w.b2, b2, d));
  WX_TRY(upload_f32(e, w.ln1_g, attn_ln_w, d));
  WX_TRY(upload_f32(e, w.ln1_b, attn_ln_b, d));
  WX_TRY(upload_f32(e, w.ln2_g, mlp_ln_w, d));
  WX_TRY(upload_f32(e, w.ln2_b, mlp_ln_b, d));
  e->set_layer[layer] = true;
  return WX_OK;
}

int wx_encoder_set_quant(wx_encoder* e, int mode) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  if (mode != WX_QUANT_NONE && mode != WX_QUANT_INT8_PERCHAN && mode != WX_QUANT_INT8_PERTENSOR)
    return fail(WX_ERR_INVALID, "encoder_set_quant: mode %d", mode);
  if (e->set_front || e->set_post || std::find(e->set_layer.begin(), e->set_layer.end(), true) !=
                                         e->set_layer.end())
    return fail(WX_ERR_INVALID, "encoder_set_quant: call before any weights are set");
  if (e->quant != WX_QUANT_NONE && mode != e->quant)
    return fail(WX_ERR_INVALID, "encoder_set_quant: the mode is already set");
  if (mode == WX_QUANT_NONE || e->quant == mode) return WX_OK;
  const int64_t d = e->d, ffn = e->ffn, B = e->max_batch, T = e->n_ctx, M = B * T;
  const int64_t k1 = 3 * (int64_t)e->n_mels;
  if (k1 % 16 || d % 16 || ffn % 16)
    return fail(WX_ERR_UNSUPPORTED, "encoder_set_quant: 3*n_mels, d and ffn must be multiples of 16");
  int s = WX_OK;
  auto A = [&](void** p, int64_t bytes) { if (s == WX_OK) s = dalloc(e, p, bytes); };
  A((void**)&e->conv1_q, d * k1);
  A((void**)&e->conv2_q, d * 3 * d);
  A((void**)&e->conv1_s, d * 4);
  A((void**)&e->conv2_s, d * 4);
  for (LayerW& w : e->L) {
    A((void**)&w.qqkv, 3 * d * d);
    A((void**)&w.qo, d * d);
    A((void**)&w.q1, ffn * d);
    A((void**)&w.q2, ffn * d);
    A((void**)&w.sqkv, 3 * d * 4);
    A((void**)&w.so, d * 4);
    A((void**)&w.s1, ffn * 4);
    A((void**)&w.s2, d * 4);
  }
  A((void**)&e->aq, M * d);
  A((void**)&e->fq, std::max(M * ffn, std::max(B * 2 * T * k1, M * 3 * d)));
  A((void**)&e->sa, 2 * M * 4);
  A((void**)&e->rowmax, M * 4);
  A((void**)&e->gmax, 16);
  A((void**)&e->stage2, e->stage_n * 4);
  if (s != WX_OK) return s;   // the allocations made are released with the encoder
  // the bf16 weights are not used in int8 mode
  dfree(e, (void**)&e->conv1_w, d * k1 * 2);
  dfree(e, (void**)&e->conv2_w, d * 3 * d * 2);
  for (LayerW& w : e->L) {
    dfree(e, (void**)&w.wqkv, 3 * d * d * 2);
    dfree(e, (void**)&w.wo, d * d * 2);
    dfree(e, (void**)&w.w1, ffn * d * 2);
    dfree(e, (void**)&w.w2, ffn * d * 2);
  }
  e->quant = mode;
  return WX_OK;
}

int wx_encoder_set_ln_post(wx_encoder* e, const float* w, const float* b) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  WX_TRY(upload_f32(e, e->lnp_g, w, e->d));
  WX_TRY(upload_f32(e, e->lnp_b, b, e->d));
  e->set_post = true;
  return WX_OK;
}

int64_t wx_encoder_device_bytes(const wx_encoder* e) { return e ? e->bytes : 0; }

int wx_encoder_forward(wx_encoder* e, const float* mel, float* out, int64_t batch,
                       int64_t n_frames, int use_graph, void* stream) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  if (!mel || !out) return fail(WX_ERR_INVALID, "encoder_forward: NULL buffer");
  if (batch <= 0 || batch > e->max_batch)
    return fail(WX_ERR_INVALID, "encoder_forward: batch %lld not in [1, %d]", (long long)batch, e->max_batch);
  if (n_frames <= 0 || n_frames % 2 || n_frames / 2 > e->n_ctx)
    return fail(WX_ERR_INVALID, "encoder_forward: n_frames %lld must be even and <= 2*n_ctx (%d)",
                (long long)n_frames, 2 * e->n_ctx);
  if (!e->set_front || !e->set_post)
    return fail(WX_ERR_INVALID, "encoder_forward: weights not set");
  for (int l = 0; l < e->nl; l++)
    if (!e->set_layer[l]) return fail(WX_ERR_INVALID, "encoder_forward: layer %d not set", l);
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(mel) & 3))
    return fail(WX_ERR_INVALID, "encoder_forward: out must be 16-byte aligned");
  std::lock_guard<std::mutex> lk(e->mu);
  const int64_t T = n_frames / 2;
  Plans* p = nullptr;
  WX_TRY(build_plans(e, batch, T, &p));
  cudaStream_t st = as_stream(stream);
  // Forwards share the workspace, so each one waits for the previous one
  // (ev_out marks the last forward's end) whatever stream either ran on.
  if (!use_graph) {
    WX_CUDA_TRY(cudaStreamWaitEvent(st, e->ev_out, 0));
    WX_TRY(forward_launches(e, p, mel, out, batch, T, st, nullptr));
    WX_CUDA_TRY(cudaEventRecord(e->ev_out, st));
    return WX_OK;
  }
  // Graphs are captured on a private stream fenced to the caller's stream by
  // events, so the legacy default stream works too. One graph per (batch,
  // frames): its first and last kernels take the buffers from e->io, which
  // set_io_kernel fills on the same stream right before each replay.
  GraphKey key{batch, T};
  auto it = e->graphs.find(key);
  cudaGraphExec_t exec = nullptr;
  if (it == e->graphs.end()) {
    cudaGraph_t g = nullptr;
    WX_CUDA_TRY(cudaStreamBeginCapture(e->side, cudaStreamCaptureModeThreadLocal));
    int s = forward_launches(e, p, mel, out, batch, T, e->side, e->io);
    cudaError_t ce = cudaStreamEndCapture(e->side, &g);
    if (s != WX_OK) {
      if (g) cudaGraphDestroy(g);
      return s;
    }
    if (ce != cudaSuccess) return fail(WX_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(WX_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(ce));
    e->graphs[key] = exec;
  } else {
    exec = it->second;
  }
  WX_CUDA_TRY(cudaEventRecord(e->ev_in, st));
  WX_CUDA_TRY(cudaStreamWaitEvent(e->side, e->ev_in, 0));
  WX_CUDA_TRY(cudaStreamWaitEvent(e->side, e->ev_out, 0));
  set_io_kernel<<<1, 1, 0, e->side>>>(e->io, mel, out);
  WX_TRY(check_launch("set_io"));
  WX_CUDA_TRY(cudaGraphLaunch(exec, e->side));
  WX_CUDA_TRY(cudaEventRecord(e->ev_out, e->side));
  WX_CUDA_TRY(cudaStreamWaitEvent(st, e->ev_out, 0));
  return WX_OK;
}

int wx_encoder_forward_host(wx_encoder* e, const float* mel_host, float* out_host, int64_t batch,
                            int64_t n_frames, int use_graph, void* stream) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  if (!mel_host || !out_host) return fail(WX_ERR_INVALID, "encoder_forward_host: NULL buffer");
  if (batch <= 0 || batch > e->max_batch || n_frames <= 0 || n_frames % 2 ||
      n_frames / 2 > e->n_ctx)
    return fail(WX_ERR_INVALID, "encoder_forward_host: bad batch or n_frames");
  WX_TRY(wx_encoder_wait_host(e));   // submitted batches share slot 0's staging
  cudaStream_t st = as_stream(stream);
  const int64_t T = n_frames / 2;
  const size_t in_clip = (size_t)e->n_mels * n_frames, out_clip = (size_t)T * e->d;
  // Batches of 32 clips or more run in two halves: the second half's mel goes
  // in on s_in while the first computes on s_comp, and the first half's
  // features come out on s_out while the second computes, so about half of
  // the copies hide behind compute. (Smaller chunks hide more of the copies
  // but cost more than they hide: at 16 clips the out-proj and fc2 GEMMs lose
  // ~9% to the last partial wave of tiles.) Chunks use disjoint parts of the
  // staging buffers and run one after the other through the shared workspace.
  const int64_t chunk = batch >= 32 ? (batch + 1) / 2 : batch;
  WX_CUDA_TRY(cudaEventRecord(e->ev_start, st));
  for (cudaStream_t x : {e->s_in, e->s_comp, e->s_out})
    WX_CUDA_TRY(cudaStreamWaitEvent(x, e->ev_start, 0));
  int k = 0;
  for (int64_t b0 = 0; b0 < batch; b0 += chunk, k++) {
    const int64_t nb = std::min(chunk, batch - b0);
    float* md = e->mel_dev + b0 * in_clip;
    float* od = e->out_dev + b0 * out_clip;
    WX_CUDA_TRY(cudaMemcpyAsync(md, mel_host + b0 * in_clip, nb * in_clip * 4,
                                cudaMemcpyHostToDevice, e->s_in));
    WX_CUDA_TRY(cudaEventRecord(e->ev_h2d[k], e->s_in));
    WX_CUDA_TRY(cudaStreamWaitEvent(e->s_comp, e->ev_h2d[k], 0));
    WX_TRY(wx_encoder_forward(e, md, od, nb, n_frames, use_graph, e->s_comp));
    WX_CUDA_TRY(cudaEventRecord(e->ev_done[k], e->s_comp));
    WX_CUDA_TRY(cudaStreamWaitEvent(e->s_out, e->ev_done[k], 0));
    WX_CUDA_TRY(cudaMemcpyAsync(out_host + b0 * out_clip, od, nb * out_clip * 4,
                                cudaMemcpyDeviceToHost, e->s_out));
  }
  WX_CUDA_TRY(cudaEventRecord(e->ev_end, e->s_out));
  WX_CUDA_TRY(cudaStreamWaitEvent(st, e->ev_end, 0));
  WX_CUDA_TRY(cudaStreamSynchronize(st));
  return WX_OK;
}

int wx_encoder_submit_host(wx_encoder* e, const float* mel_host, float* out_host, int64_t batch,
                           int64_t n_frames, int use_graph) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  if (!mel_host || !out_host) return fail(WX_ERR_INVALID, "encoder_submit_host: NULL buffer");
  if (batch <= 0 || batch > e->max_batch || n_frames <= 0 || n_frames % 2 ||
      n_frames / 2 > e->n_ctx)
    return fail(WX_ERR_INVALID, "encoder_submit_host: bad batch or n_frames");
  const int k = e->q_next;
  if (k == 1 && !e->mel_dev1)
    WX_TRY(dalloc(e, (void**)&e->mel_dev1, (int64_t)e->max_batch * e->n_mels * 2 * e->n_ctx * 4));
  if (k == 1 && !e->out_dev1)
    WX_TRY(dalloc(e, (void**)&e->out_dev1, (int64_t)e->max_batch * e->n_ctx * e->d * 4));
  // at most two batches in flight: the one submitted two calls ago has
  // finished with its host buffers before this one takes its slot
  if (e->q_busy[k]) {
    WX_CUDA_TRY(cudaEventSynchronize(e->ev_q_out[k]));
    e->q_busy[k] = false;
  }
  const int64_t T = n_frames / 2;
  const size_t in_bytes = (size_t)batch * e->n_mels * n_frames * 4;
  const size_t out_bytes = (size_t)batch * T * e->d * 4;
  float* md = k ? e->mel_dev1 : e->mel_dev;
  float* od = k ? e->out_dev1 : e->out_dev;
  // The copy-in waits for the compute that last read this slot; the compute
  // waits for its copy-in and for the copy-out that last read this slot's
  // features; computes follow one another on s_comp.
  WX_CUDA_TRY(cudaStreamWaitEvent(e->s_in, e->ev_q_comp[k], 0));
  WX_CUDA_TRY(cudaMemcpyAsync(md, mel_host, in_bytes, cudaMemcpyHostToDevice, e->s_in));
  WX_CUDA_TRY(cudaEventRecord(e->ev_q_in[k], e->s_in));
  WX_CUDA_TRY(cudaStreamWaitEvent(e->s_comp, e->ev_q_in[k], 0));
  WX_CUDA_TRY(cudaStreamWaitEvent(e->s_comp, e->ev_q_out[k], 0));
  WX_TRY(wx_encoder_forward(e, md, od, batch, n_frames, use_graph, e->s_comp));
  WX_CUDA_TRY(cudaEventRecord(e->ev_q_comp[k], e->s_comp));
  WX_CUDA_TRY(cudaStreamWaitEvent(e->s_out, e->ev_q_comp[k], 0));
  WX_CUDA_TRY(cudaMemcpyAsync(out_host, od, out_bytes, cudaMemcpyDeviceToHost, e->s_out));
  WX_CUDA_TRY(cudaEventRecord(e->ev_q_out[k], e->s_out));
  e->q_busy[k] = true;
  e->q_next = k ^ 1;
  return WX_OK;
}

int wx_encoder_wait_host(wx_encoder* e) {
  if (!e) return fail(WX_ERR_INVALID, "encoder: NULL handle");
  DeviceGuard dg(e->device);
  for (int k = 0; k < 2; k++) {
    if (!e->q_busy[k]) continue;
    e->q_busy[k] = false;
    WX_CUDA_TRY(cudaEventSynchronize(e->ev_q_out[k]));
  }
  return WX_OK;
}

}  // extern "C"
