// An entry point that allocates nothing: the MLP block fc2(GELU(fc1(h))) with
// its fc1 activation in a fixed, file-scope device array instead of memory the
// caller provides.
//
// Some callers cannot call cudaMalloc: processes whose device memory is owned
// by another allocator (a framework's caching allocator or a fixed memory
// plan), and embedded or real-time callers that must not allocate after
// start-up. They still pass inputs and outputs; the intermediate activation
// lives here.
//
// The scratch array is g_mlp_scratch below: kMlpScratchElems bf16 elements
// (16 MiB). Every GPU that loads the library holds it until the process
// exits. In host code its name is only a host-side stand-in, so its device
// address is taken with cudaGetSymbolAddress once per device, with that device
// current, on the entry point's first call there (that first call should come
// before any stream capture). Every call shares the array, and it keeps the
// last call's contents: fc1 overwrites every element fc2 reads, so nothing
// needs clearing, but calls that overlap on the GPU (different streams,
// without ordering between them) race on it.
//
// The GEMMs' bounded waits record a timeout into g_mlp_err, a file-scope
// word of this path (the library's own per-device error word is allocated on
// first use, so it is not used here); wx_device_error reports and clears it
// together with the library's word.
#include <mutex>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

constexpr int64_t kMlpScratchElems = 8ll * 1024 * 1024;  // bf16 elements: 16 MiB

static __device__ __align__(256) uint16_t g_mlp_scratch[kMlpScratchElems];
static __device__ int g_mlp_err;

static std::mutex g_scratch_mu;
static uint16_t* g_scratch_addr[64] = {nullptr};
static int* g_err_addr[64] = {nullptr};

// The device addresses of g_mlp_scratch and g_mlp_err on the current device.
static int mlp_scratch(uint16_t** out, int** err) {
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64) return fail(WX_ERR_UNSUPPORTED, "mlp_noalloc: device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    void* q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mlp_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_mlp_err);
    if (e != cudaSuccess || !p || !q)
      return fail(WX_ERR_CUDA, "mlp_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_err_addr[dev] = static_cast<int*>(q);
    g_scratch_addr[dev] = static_cast<uint16_t*>(p);
  }
  *out = g_scratch_addr[dev];
  *err = g_err_addr[dev];
  return WX_OK;
}

// Read (and clear) this path's error word on the current device, if the entry
// point has run there; the caller has synchronised the device.
int noalloc_take_error(int* flags, bool clear) {
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  int* w = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (dev < 64) w = g_err_addr[dev];
  }
  if (!w) return WX_OK;
  int v = 0;
  WX_CUDA_TRY(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  *flags |= v;
  if (clear && v) WX_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
  return WX_OK;
}

}  // namespace wx

extern "C" {

int wx_mlp_bf16_noalloc(const void* h, const void* w1, const float* b1, const void* w2,
                        const float* b2, float* out, int64_t M, int64_t d, int64_t ffn,
                        int64_t ldh, int64_t ldo, int gelu_mode, void* stream) {
  using namespace wx;
  if (M <= 0 || d <= 0 || ffn <= 0)
    return fail(WX_ERR_INVALID, "mlp_noalloc: M, d and ffn must be > 0");
  if (M > kMlpScratchElems / ffn)
    return fail(WX_ERR_INVALID,
                "mlp_noalloc: M*ffn = %lld exceeds the fixed scratch of %lld elements "
                "(%lld rows at ffn %lld); split the rows into smaller calls",
                (long long)(M * ffn), (long long)kMlpScratchElems,
                (long long)(kMlpScratchElems / ffn), (long long)ffn);
  if (ffn % 8) return fail(WX_ERR_INVALID, "mlp_noalloc: ffn must be a multiple of 8");
  if (gelu_mode != WX_GELU_POLY4 && gelu_mode != WX_GELU_ERF)
    return fail(WX_ERR_INVALID, "mlp_noalloc: gelu_mode %d", gelu_mode);
  uint16_t* f = nullptr;
  int* err = nullptr;
  WX_TRY(mlp_scratch(&f, &err));
  const int epi1 = gelu_mode == WX_GELU_ERF ? WX_EPI_BF16_GELU_ERF : WX_EPI_BF16_GELU;
  GemmPlan p1, p2;
  WX_TRY(gemm_plan_err(&p1, h, w1, b1, f, M, ffn, d, ldh, d, ffn, epi1, err));
  WX_TRY(gemm_plan_err(&p2, f, w2, b2, out, M, d, ffn, ffn, ffn, ldo, WX_EPI_F32, err));
  cudaStream_t st = as_stream(stream);
  WX_TRY(gemm_run(p1, st));
  return gemm_run(p2, st);
}

}  // extern "C"
