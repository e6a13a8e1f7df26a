// Internal host-side helpers shared by the .cu files of libwxb200.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/wxb200.h"

namespace wx {

// Record the calling thread's last error; returns `code` so call sites can
// `return fail(WX_ERR_INVALID, "...")`.
int fail(int code, const char* fmt, ...);

// Check a CUDA runtime status; on error record it and return WX_ERR_CUDA.
#define WX_CUDA_TRY(expr)                                                            \
  do {                                                                               \
    cudaError_t e_ = (expr);                                                         \
    if (e_ != cudaSuccess)                                                           \
      return ::wx::fail(WX_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                 \
                        cudaGetErrorString(e_), __FILE__, __LINE__);                 \
  } while (0)

#define WX_TRY(expr)         \
  do {                       \
    int s_ = (expr);         \
    if (s_ != WX_OK) return s_; \
  } while (0)

// After a kernel launch.
int check_launch(const char* what);

// The device error word kernels write into (one int per device).
int* device_error_word();

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda and loads on machines without a GPU.
int encode_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                         int elem_bytes, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

// Number of SMs of the current device.
int sm_count();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch (PDL) for the encoder's forward pass: while a
// PdlScope(true) is alive on the calling thread, launch_k gives each kernel the
// programmatic-stream-serialization attribute, so it may launch while the
// kernel before it on the stream finishes; the kernels launched this way call
// pdl_wait() (common.cuh) before touching global memory. Outside a scope
// launch_k is a plain launch.
extern thread_local bool g_pdl;
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(g_pdl) { g_pdl = on; }
  ~PdlScope() { g_pdl = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (g_pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Makes `dev` the calling thread's current device for a scope and restores
// the caller's device after: an engine's entry points run on the device the
// engine was created on, whichever device the calling thread has current.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess || prev == dev || cudaSetDevice(dev) != cudaSuccess)
      prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};

}  // namespace wx
