// Library-wide pieces of the C ABI: error reporting, the device error word,
// tensor-map encoding and device queries.
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "plans.cuh"
#include "wxb200_internal.h"

namespace wx {

static thread_local std::string g_last_error;
thread_local bool g_pdl = false;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(WX_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return WX_OK;
}

static std::mutex g_mu;
static std::vector<int*> g_err_words;  // per device

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_err_words.size() <= dev) g_err_words.resize(dev + 1, nullptr);
  if (!g_err_words[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_err_words[dev] = p;
  }
  return g_err_words[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encode_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                         int elem_bytes, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(WX_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(WX_ERR_INVALID, "tensor base address not 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    return fail(WX_ERR_INVALID, "row stride %llu bytes is not a multiple of 16",
                (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(WX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, box %u x %u",
                (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner,
                box_outer);
  (void)elem_bytes;
  return WX_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  if (dev < 64) cached[dev] = n;
  return n;
}

}  // namespace wx

extern "C" {

int wx_version(void) { return 100; }

int wx_last_error(char* buf, int64_t len) {
  const std::string& s = wx::g_last_error;
  if (buf && len > 0) {
    int64_t n = (int64_t)s.size() < len - 1 ? (int64_t)s.size() : len - 1;
    for (int64_t i = 0; i < n; i++) buf[i] = s[i];
    buf[n] = 0;
  }
  return (int)s.size();
}

int wx_device_error(int* flags, int clear) {
  if (!flags) return wx::fail(WX_ERR_INVALID, "wx_device_error: flags is NULL");
  int* w = wx::device_error_word();
  if (!w) return wx::fail(WX_ERR_CUDA, "device error word unavailable");
  WX_CUDA_TRY(cudaDeviceSynchronize());
  WX_CUDA_TRY(cudaMemcpy(flags, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) WX_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
  // the allocation-free entry point records into a word of its own
  return wx::noalloc_take_error(flags, clear != 0);
}

}  // extern "C"

// A kernel whose one waiting thread waits, through the same bounded-wait
// helper the kernels use, on an mbarrier that nothing ever completes: after
// limit_ns it records WX_DEVERR_TIMEOUT in the device error word and returns.
// It exercises the failure path of every kernel wait without a GPU fault; the
// context stays usable.
namespace wx {
__global__ void selftest_wait_timeout_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait_limit(&bar, 0, err, limit_ns);   // never completes
    if (ok) set_device_error(err, 0x40000000);                 // would be a logic error
  }
  __syncthreads();
}
}  // namespace wx

extern "C" int wx_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 2000000000ull)
    return wx::fail(WX_ERR_INVALID, "selftest: limit_ns must be in (0, 2e9]");
  int* w = wx::device_error_word();
  if (!w) return wx::fail(WX_ERR_CUDA, "device error word unavailable");
  wx::selftest_wait_timeout_kernel<<<1, 32, 0, wx::as_stream(stream)>>>(w, limit_ns);
  return wx::check_launch("selftest_wait_timeout");
}

