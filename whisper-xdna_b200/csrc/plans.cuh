// Launch plans shared between the standalone entry points and the encoder:
// tensor maps and kernel arguments built once for fixed buffers.
#pragma once
#include "common.cuh"

namespace wx {

struct GemmArgs {
  int M, N, K;
  int num_n_blocks, num_tiles, num_k_blocks;
  void* C;
  int64_t ldc;
  const float* bias;
  const float* R;
  int64_t ldr;
  int* err;
  const float* pos;  // positional embedding (WX_EPI_*_POS), row (row % pos_T)
  int64_t ldp;
  int pos_T;
  // int8 GEMM: C = epilogue((float(A_q @ B_q^T) * sa[row]) * sw[col])
  const float* sa;   // per-row (token) scales of A
  const float* sw;   // per-column (channel) scales of B
  float* rowmax;     // bf16 outputs: max |value| of each row, atomically (or NULL)
  int resid_inplace; // WX_EPI_F32_RESID with C == R: the 2-SM kernel adds into C by TMA
};

// Epilogues used only inside the library (the conv2 step of the encoder):
//   C fp32 = GELU(acc + bias) + pos[row % pos_T]
constexpr int kEpiF32GeluPos = 16;     // GELU = poly4 RNE on rne(acc + bias)
constexpr int kEpiF32GeluErfPos = 17;  // GELU = exact erf form

struct GemmPlan {
  CUtensorMap tmA, tmB;
  CUtensorMap tmC, tmR;   // output / residual tiles of the 2-SM kernel's epilogue
  GemmArgs args;
  int bn;
  int grid;
  int epi;
  bool pair;   // 2-SM kernel (CTA pairs, 256 x 256 tiles)
  bool i8;     // int8 operands (tcgen05 kind::i8), dequantised in the epilogue
};

// force_bn: 0 = pick, else 128 or 256 (output columns per tile)
int gemm_plan(GemmPlan* p, const void* A, const void* B, const float* bias, const float* R,
              void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
              int64_t ldr, int epi, int force_bn);
// The int8 GEMM: A (M x K) and B (N x K) int8, row-major; sa (M) and sw (N) the
// dequantisation scales; rowmax (M floats, or NULL) collects max |C| per row
// for the bf16 epilogues.
int gemm_plan_i8(GemmPlan* p, const void* A, const void* B, const float* sa, const float* sw,
                 const float* bias, const float* R, void* C, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int epi, float* rowmax);
int gemm_run(const GemmPlan& p, cudaStream_t st);
// A bf16 plan whose kernels record wait timeouts into `err` (a word the
// caller owns) instead of the library's per-device error word.
int gemm_plan_err(GemmPlan* p, const void* A, const void* B, const float* bias, void* C,
                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int epi,
                  int* err);
// The allocation-free entry point's error word on the current device (if it
// has been set up there): OR it into *flags, and clear it when asked.
int noalloc_take_error(int* flags, bool clear);
// attach the positional embedding to a plan built with kEpiF32Gelu*Pos
void gemm_set_pos(GemmPlan* p, const float* pos, int64_t ldp, int pos_T);

struct AttnArgs {
  int T, H, num_q_tiles;
  int n_items;  // num_q_tiles * H * B work items (query tile pair, head, clip)
  void* O;
  int64_t ldo;
  float scale_log2;
  int* err;
};

struct AttnPlan {
  CUtensorMap tmQ, tmK, tmV;
  AttnArgs args;
  int B;
  int grid;      // persistent kernel: min(items, SMs) CTAs
  bool persist;  // run the persistent kernel (short items)
};

int attn_plan(AttnPlan* p, const void* q, const void* k, const void* v, void* o, int64_t B,
              int64_t H, int64_t T, int64_t hd, int64_t ldq, int64_t ldk, int64_t ldv,
              int64_t ldo, float scale);
int attn_run(const AttnPlan& p, cudaStream_t st);

// row ops (rowops.cu)
int launch_gelu_poly4(const void* in, int in_dtype, void* out, int64_t rows, int64_t cols,
                      int64_t ld_in, int64_t ld_out, int rounding, cudaStream_t st);
int launch_softmax_rows(const void* in, void* out, int64_t rows, int64_t cols, int64_t valid,
                        int64_t ld_in, int64_t ld_out, float scale, int variant, int rounding,
                        cudaStream_t st);
// out_ind (mode WX_LN_FP32 only): when not NULL the kernel reads its output
// pointer from this device address (out is then ignored)
int launch_layernorm_rows(const void* in, int in_dtype, const float* gamma, const float* beta,
                          void* out, int out_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                          int64_t ld_out, float eps, int mode, int rounding, cudaStream_t st,
                          void* const* out_ind = nullptr);

int launch_layernorm_quant_rows(const float* in, const float* gamma, const float* beta, int8_t* q,
                                float* scale, int64_t rows, int64_t cols, int64_t ld_in,
                                int64_t ld_q, float eps, cudaStream_t st);

// int8 quantisation (quant.cu)
int launch_absmax_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld,
                       float* out, int64_t out_stride, cudaStream_t st);
int launch_quantize_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld,
                         const float* rowmax, int64_t rowmax_stride, int8_t* q, int64_t ld_q,
                         float* scale, cudaStream_t st);

}  // namespace wx
