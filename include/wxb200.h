/*
 * wxb200.h -- C ABI of the B200 (sm_100a) Whisper-encoder hot path.
 *
 * One shared library, libwxb200.so, built from whisper-xdna_b200/csrc. Every
 * entry point is extern "C", takes plain pointers and sizes, returns a status
 * (WX_OK = 0, negative on error; wx_last_error() then gives the message) and
 * enqueues its work on the given CUDA stream (NULL = the legacy default
 * stream) without synchronizing, unless it says otherwise. Device pointers
 * are CUDA global-memory addresses; "host" pointers are ordinary CPU memory.
 * Matrices are row-major; ld* arguments are row strides in ELEMENTS.
 *
 * Each entry point names the reference interface it replaces
 * (drakosha/whisper-xdna, paths relative to the reference checkout).
 */
#ifndef WXB200_H
#define WXB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define WX_OK 0
#define WX_ERR_INVALID (-1)     /* bad argument: shape, stride, alignment, enum */
#define WX_ERR_CUDA (-2)        /* a CUDA runtime or driver call failed */
#define WX_ERR_UNSUPPORTED (-3) /* valid request this build does not handle */
#define WX_ERR_DEVICE (-4)      /* a kernel recorded a device-side error */
#define WX_ERR_NOMEM (-5)       /* device allocation failed */

/* bits of the device error word (wx_device_error) */
#define WX_DEVERR_TIMEOUT 1 /* a bounded wait inside a kernel gave up */

/* element types */
#define WX_DTYPE_BF16 0
#define WX_DTYPE_F32 1

/* bf16 rounding of the reference's AIE2 kernels */
#define WX_ROUND_TRUNC 0 /* the part's default: truncate toward zero */
#define WX_ROUND_RNE 1   /* aie::set_rounding(conv_even) */

/* ------------------------------------------------------------ library */

/* Library version, e.g. 100 for 0.1.0. */
int wx_version(void);

/* Copy the calling thread's last error message into buf (always
 * NUL-terminated when len > 0). Returns the message length. */
int wx_last_error(char* buf, int64_t len);

/* Synchronize the current device, read the device error word into *flags
 * (WX_DEVERR_* bits, 0 if none) and clear it when clear != 0. Kernels that
 * give up a bounded wait set a bit here instead of hanging the GPU.
 * Replaces the run-state check of src/rawxrt.py:319-324 (RawRT._await). */
int wx_device_error(int* flags, int clear);

/* ------------------------------------------------------------ row ops */

/* Polynomial erf-GELU, elementwise over a rows x cols window.
 *   in_dtype WX_DTYPE_BF16: g4 (rounding TRUNC, kernels/gelu_row4.cc:44) or g4r
 *     (RNE, kernels/gelu_row4_rne.cc:44);
 *   in_dtype WX_DTYPE_F32: g4f, the fp32 input is rounded to bf16 first
 *     (kernels/gelu_row4f.cc:58; the reference always uses RNE there).
 * out is bf16 with row stride ld_out, so a column band of a wider buffer can be
 * written (the out_cols banding of src/rowops.py:80-88, 306-313).
 * Replaces rowops.gelu_row4 / gelu_row4_rne / gelu_row4f (src/rowops.py:297-321)
 * and RawRT.rowop for g4* (src/rawxrt.py:384-400). */
int wx_gelu_poly4(const void* in, int in_dtype, void* out, int64_t rows, int64_t cols,
                  int64_t ld_in, int64_t ld_out, int rounding, void* stream);

/* Row softmax over the first `valid` columns (all cols if valid <= 0) of each
 * bf16 row; columns past the window are neither read nor written
 * (src/rowops.py:60-73). variant 4 = kernels/softmax_row4_body.inc:17-60
 * (rounding TRUNC: softmax_row4, RNE: softmax_row4r, kernels/softmax_row4_rne.cc:41),
 * variant 1 = kernels/softmax_row.cc:25, variant 3 = kernels/softmax_row3.cc:34.
 * scale != 1 multiplies the input by scale (rounded to bf16) first; the
 * reference kernels have no scale. Width limit: valid <= 65536.
 * Replaces rowops.softmax_row*, softmax_row*_win (src/rowops.py:227-330) and
 * RawRT.softmax_stack (src/rawxrt.py:569-585). */
int wx_softmax_rows(const void* in, void* out, int64_t rows, int64_t cols, int64_t valid,
                    int64_t ld_in, int64_t ld_out, float scale, int variant, int rounding,
                    void* stream);

/* LayerNorm over each row.
 *   mode WX_LN_AIE: the reference's device kernel (kernels/layer_norm_gb.cc:48-86):
 *     bf16 in and out, sums in 16 fp32 lanes, var = E[x^2] - mean^2, the
 *     bit-trick rsqrt with 3 Newton steps, bf16 mean and 1/std, then the
 *     optional affine (gamma/beta may be NULL) rounded once more.
 *   mode WX_LN_FP32: the encoder's host LayerNorm (src/npu_whisper_encoder.py:278-281):
 *     two-pass fp32 mean and variance, out = (x - mean) / sqrt(var + eps) * gamma
 *     + beta, in/out bf16 or fp32, output rounded RNE when bf16.
 * Replaces rowops.layer_norm (src/rowops.py:221-224). */
#define WX_LN_AIE 0
#define WX_LN_FP32 1
int wx_layernorm_rows(const void* in, int in_dtype, const float* gamma, const float* beta,
                      void* out, int out_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                      int64_t ld_out, float eps, int mode, int rounding, void* stream);

/* Host-only inspection (no GPU needed): the constant tables the row kernels
 * upload. wx_softmax_exp_table writes R(exp(x')) as bf16 bits (rounding mode
 * `rounding`) and/or the fp32 exponential for every bf16 x' in [-128, -0]
 * (bit patterns 0x8000 .. 0xC2FF), n >= 17152 entries; returns the count.
 * wx_gelu4_table writes the GELU table (kernels/gelu_poly4_coeffs.h:6-13)
 * rounded to bf16 in `rounding`: breaks[3], shifts[3], scales[3],
 * coefficients[3][5]; n >= 24; returns 24. */
int wx_softmax_exp_table(int rounding, uint16_t* out16, float* out32, int64_t n);
int wx_gelu4_table(int rounding, float* out, int64_t n);

/* ------------------------------------------------------------ GEMM */

/* C = epilogue(A @ B^T): A (M x K, bf16, row stride lda), B (N x K, bf16, row
 * stride ldb -- the torch Linear weight layout (out, in)), fp32 accumulation
 * in tensor memory (tcgen05). bias (N floats) may be NULL.
 *   WX_EPI_F32        C fp32 = acc + bias
 *   WX_EPI_BF16       C bf16 = rne(acc + bias)
 *   WX_EPI_F32_RESID  C fp32 = acc + bias + R (R fp32, row stride ldr; C may be R)
 *   WX_EPI_BF16_GELU  C bf16 = gelu_poly4_rne(rne(acc + bias))   (fc1 -> g4f)
 *   WX_EPI_BF16_GELU_ERF  C bf16 = rne(erf-GELU(acc + bias))
 * Alignment: A, B, C 16-byte aligned; lda, ldb multiples of 8; K >= 1.
 * Replaces RawRT.matmul / mm_start / mm_finish (src/rawxrt.py:926-996) and the
 * MLIR-AIE whole_array GEMM they drive; the bias fold of src/rawxrt.py:352-371
 * becomes the epilogue's bias. */
#define WX_EPI_F32 0
#define WX_EPI_BF16 1
#define WX_EPI_F32_RESID 2
#define WX_EPI_BF16_GELU 3
#define WX_EPI_BF16_GELU_ERF 4
int wx_gemm_bf16(const void* A, const void* B, const float* bias, const float* R, void* C,
                 int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                 int64_t ldr, int epilogue, void* stream);

/* ------------------------------------------------------------ int8 */

/* The reference's int8 projection/MLP mode (bench/probe_int8_decode.py:48-74,
 * q_matmul_factory; README.md "int8 on the wide GEMMs"), on int8 tensor cores.
 *
 * wx_absmax_rows: out[r * out_stride] = max(out[r * out_stride], max_c |in[r, c]|)
 * for r < rows (an atomic fold: out_stride 0 gives the maximum of the whole
 * matrix, the "pertensor" weight scale). in is bf16 or fp32 (in_dtype), row
 * stride ld_in elements. out must hold non-negative values (zero it first).
 *
 * wx_quantize_rows: per row r, m = rowmax[r * rowmax_stride] (or, with rowmax
 * NULL, max_c |in[r, c]|); scale[r] = m / 127 (1 where that is 0);
 * q[r, c] = rint(in[r, c] / scale[r]) as int8 (fp32 division rounded to
 * nearest, integer rounding half to even: numpy's np.rint(A / sa)). Quantises
 * activations per token and, applied to the torch weight (N, K), weights per
 * output channel. q has row stride ld_q bytes.
 *
 * wx_gemm_i8: C = epilogue((float(A @ B^T) * sa[m]) * sw[n]) with A (M x K) and
 * B (N x K) int8 row-major (lda, ldb multiples of 16, 16-byte aligned), s32
 * accumulation (exact), sa (M) and sw (N, 16-byte aligned) fp32 scales; the
 * two products are rounded separately, as (A_q @ B_q) * sa * sw in the
 * reference. Epilogues as wx_gemm_bf16 (bias added after the scaling). rowmax
 * (M floats, or NULL; bf16 epilogues only) receives max |C[m, :]| of the
 * stored bf16 values by an atomic fold, for quantising C as the next GEMM's A. */
int wx_absmax_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                   float* out, int64_t out_stride, void* stream);
/* The encoder's fp32 LayerNorm (wx_layernorm_rows, WX_LN_FP32, fp32 in) fused
 * with wx_quantize_rows of its output: q and scale equal those two calls in
 * sequence. cols <= 2048 and a multiple of 4; in, gamma, beta 16-byte aligned
 * (gamma/beta may be NULL), q 4-byte aligned with ld_q a multiple of 4. */
int wx_layernorm_quant_rows(const float* in, const float* gamma, const float* beta, int8_t* q,
                            float* scale, int64_t rows, int64_t cols, int64_t ld_in, int64_t ld_q,
                            float eps, void* stream);
int wx_quantize_rows(const void* in, int in_dtype, int64_t rows, int64_t cols, int64_t ld_in,
                     const float* rowmax, int64_t rowmax_stride, int8_t* q, int64_t ld_q,
                     float* scale, void* stream);
int wx_gemm_i8(const int8_t* A, const int8_t* B, const float* sa, const float* sw,
               const float* bias, const float* R, void* C, int64_t M, int64_t N, int64_t K,
               int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int epilogue, float* rowmax,
               void* stream);
/* The unquantised control of the same probe, q_matmul_factory("fp32")
 * (bench/probe_int8_decode.py:58-60, numpy float32 A @ B + bias): C = A @ B^T
 * (+ bias[n]) in fp32 on the FMA pipe, A (M x K) and B (N x K) fp32 row-major
 * with row strides lda, ldb, ldc (elements), bias NULL or N floats. Each
 * output is one fp32 FMA chain over k in ascending order. */
int wx_gemm_f32(const float* A, const float* B, const float* bias, float* C, int64_t M,
                int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* ------------------------------------------------------------ attention */

/* Fused attention, no mask: for every batch b < B and head h < H,
 *   O[b*T + t, h*hd : (h+1)*hd] = softmax_j(scale * q_t . k_j) v_j
 * with q_t = Q[b*T + t, h*hd : ...] and likewise K, V (bf16, row strides ldq,
 * ldk, ldv), O bf16 with row stride ldo. hd must be 64. QK^T and PV run on the
 * tensor cores with fp32 accumulation; the softmax is online in fp32 with the
 * row statistics of src/attn_fused.py / kernels/attn_fused.cc:13-17, and keys
 * past T are masked exactly (the reference pads with zeros; this does not).
 * Q, K, V may be column slices of one fused QKV buffer.
 * Replaces RawRT.attn_chain / attn_fused (src/rawxrt.py:761-891) and
 * attn_fused.attn_head (src/attn_fused.py:140-145). */
int wx_attention(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                 int64_t T, int64_t hd, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo,
                 float scale, void* stream);

/* ------------------------------------------------------------ no allocation */

/* The MLP block out = GELU(h @ w1^T + b1) @ w2^T + b2 for callers that cannot
 * allocate device memory -- processes whose device memory belongs to another
 * allocator (a framework's caching allocator, a fixed memory plan), and
 * callers that must not allocate after start-up. It has no counterpart in the
 * reference.
 * h (M x d, bf16, row stride ldh), w1 (ffn x d) and w2 (d x ffn) bf16 in the
 * torch Linear layout, b1 (ffn) and b2 (d) fp32 or NULL, out (M x d) fp32 with
 * row stride ldo; gelu_mode WX_GELU_POLY4 or WX_GELU_ERF. The fc1 activation
 * is kept in a fixed device array of 8M bf16 elements (16 MiB), so
 * M * ffn <= 8388608 (1638 rows at ffn 5120); larger calls are refused with
 * WX_ERR_INVALID. The library calls no cudaMalloc, cudaFree or allocating
 * library routine here. The array's device address is looked up on the first
 * call on each device (cudaGetSymbolAddress), so make that first call before
 * any stream capture. Every call shares the array: calls that overlap on the
 * GPU race on it. A device-side wait that gives up records WX_DEVERR_TIMEOUT
 * in an error word of this path (a file-scope device variable, not an
 * allocation), which wx_device_error reports and clears with the library's. */
int wx_mlp_bf16_noalloc(const void* h, const void* w1, const float* b1, const void* w2,
                        const float* b2, float* out, int64_t M, int64_t d, int64_t ffn,
                        int64_t ldh, int64_t ldo, int gelu_mode, void* stream);

/* ------------------------------------------------------------ encoder */

/* A Whisper encoder resident on the current device: bf16 weights, fp32 LN
 * parameters and biases, workspace for up to max_batch clips of n_ctx frames.
 * gelu_mode selects the GELU of the conv frontend and the MLP:
 *   WX_GELU_POLY4: the reference's device GELU (g4f / g4r, RNE poly4)
 *   WX_GELU_ERF:   exact erf-GELU in fp32 (the reference's numpy path)
 * Replaces the encoder loop of src/npu_whisper_encoder.py:436-541 driven by
 * RawRT (src/rawxrt.py) with register_weights (src/rawxrt.py:307-316). */
#define WX_GELU_POLY4 0
#define WX_GELU_ERF 1
typedef struct wx_encoder wx_encoder;

int wx_encoder_create(wx_encoder** out, int n_mels, int d_model, int n_head, int n_layer,
                      int ffn, int n_ctx, int max_batch, int gelu_mode);
int wx_encoder_destroy(wx_encoder* enc);

/* Weights from HOST fp32 arrays in the torch state_dict layouts:
 * conv1_w (d, n_mels, 3), conv2_w (d, d, 3), pos (n_ctx, d); Linear weights
 * (out, in). The key projection has no bias. */
int wx_encoder_set_frontend(wx_encoder* enc, const float* conv1_w, const float* conv1_b,
                            const float* conv2_w, const float* conv2_b, const float* pos);
int wx_encoder_set_layer(wx_encoder* enc, int layer, const float* attn_ln_w,
                         const float* attn_ln_b, const float* wq, const float* bq,
                         const float* wk, const float* wv, const float* bv, const float* wo,
                         const float* bo, const float* mlp_ln_w, const float* mlp_ln_b,
                         const float* w1, const float* b1, const float* w2, const float* b2);
int wx_encoder_set_ln_post(wx_encoder* enc, const float* w, const float* b);

/* int8 mode, the reference's int8 projection/MLP probe
 * (bench/probe_int8_decode.py:48-74, its encoder call :140-142): the conv,
 * QKV, out-proj, fc1 and fc2 GEMMs run on int8 operands (wx_gemm_i8), weights
 * quantised once per output channel (PERCHAN) or per weight matrix
 * (PERTENSOR: one scale for each of q, k, v, out, fc2, each conv, and each fc1
 * column chunk of prepare_mlp_chunks, src/npu_whisper_encoder.py:383-398),
 * activations per token right before each GEMM (wx_quantize_rows). Attention
 * stays bf16. Call after wx_encoder_create and before any wx_encoder_set_*
 * weight call; needs 3*n_mels, d_model and ffn multiples of 16. */
#define WX_QUANT_NONE 0
#define WX_QUANT_INT8_PERCHAN 1
#define WX_QUANT_INT8_PERTENSOR 2
int wx_encoder_set_quant(wx_encoder* enc, int mode);

/* Forward on DEVICE buffers: mel (batch, n_mels, n_frames) fp32 ->
 * out (batch, n_frames / 2, d_model) fp32. n_frames even, n_frames / 2 <= n_ctx
 * (a shortened mel is a reduced audio_ctx, bench/run_raw_encoder.py:63-65).
 * When use_graph != 0 the launch sequence is captured once per (batch,
 * n_frames) and replayed as a CUDA graph on any buffers and stream. */
int wx_encoder_forward(wx_encoder* enc, const float* mel, float* out, int64_t batch,
                       int64_t n_frames, int use_graph, void* stream);

/* Forward on HOST buffers (pinned memory gives asynchronous copies): copies
 * mel in, runs wx_encoder_forward, copies the result out, and synchronizes
 * the stream before returning. Batches submitted by wx_encoder_submit_host
 * are waited for first. */
int wx_encoder_forward_host(wx_encoder* enc, const float* mel_host, float* out_host,
                            int64_t batch, int64_t n_frames, int use_graph, void* stream);

/* Pipelined forward on HOST buffers, for a stream of batches (the server's
 * windows, serve/npu_stt_server.py:421-431, or the throughput loop of
 * bench/run_raw_encoder.py, each of which calls encoder(),
 * src/npu_whisper_encoder.py:436-541, once per input). Enqueues the copy-in,
 * the forward and the copy-out of one batch and returns; one batch's copies
 * overlap the neighbouring batches' compute. Two batches are in flight at
 * most: a call waits until the batch submitted two calls earlier is in its
 * host buffer. mel_host and out_host must stay valid, and unmodified, until
 * wx_encoder_wait_host returns (pinned memory for the overlap). One host
 * thread per handle. */
int wx_encoder_submit_host(wx_encoder* enc, const float* mel_host, float* out_host,
                           int64_t batch, int64_t n_frames, int use_graph);

/* Blocks until every submitted batch's features are in its host buffer. */
int wx_encoder_wait_host(wx_encoder* enc);

/* Device memory the encoder holds (weights + workspace), in bytes. */
int64_t wx_encoder_device_bytes(const wx_encoder* enc);

/* whisper's log-mel frontend: audio (batch clips, row stride ld_audio floats,
 * the first n_samples of each at 16 kHz, zero-padded or trimmed to 30 s) ->
 * mel_out (batch, n_mels, 3000) fp32, all device memory. Centred STFT (n_fft
 * 400, hop 160, periodic Hann, reflect padding), power spectrum, Slaney mel
 * filterbank (n_mels 80 or 128, 0-8 kHz), log10(max(., 1e-10)), floor at the
 * clip's maximum - 8, (x + 4) / 4. Replaces openai-whisper's
 * log_mel_spectrogram(pad_or_trim(audio), n_mels) as the reference server calls
 * it (serve/npu_stt_server.py:334-336). mel_out must be 16-byte aligned. */
int wx_log_mel(const float* audio, int64_t batch, int64_t n_samples, int64_t ld_audio,
               int n_mels, float* mel_out, void* stream);

/* Diagnostic: exercises the bounded-wait failure path of the kernels. One
 * thread waits, through the same helper every kernel wait uses, on an mbarrier
 * that nothing completes; after limit_ns (0 < limit_ns <= 2e9) it records
 * WX_DEVERR_TIMEOUT in the device error word and the kernel returns, leaving
 * the context usable. Read and clear the word with wx_device_error. Replaces
 * no reference interface (the reference's failure path is host-side:
 * serve/npu_stt_server.py:128-129 injects failures on the host). */
int wx_selftest_wait_timeout(uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* WXB200_H */
