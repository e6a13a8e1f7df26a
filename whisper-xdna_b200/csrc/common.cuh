// Shared device helpers for the sm_100a kernels: bf16 rounding in the two AIE
// modes, bounded mbarrier waits, TMA loads and the tcgen05 (5th-generation
// tensor core) instructions, all as inline PTX.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "wxb200_internal.h"

namespace wx {

// ---------------------------------------------------------------- rounding
// Rounding modes of the reference's AIE2 kernels: RND_TRUNC is the part's
// default (truncate toward zero), RND_RNE is aie::set_rounding(conv_even).
enum { RND_TRUNC = 0, RND_RNE = 1 };

template <int R>
__device__ __forceinline__ uint32_t bf16_bits(float x) {
  if (R == RND_TRUNC) return __float_as_uint(x) >> 16;
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bits_f32(uint32_t b) { return __uint_as_float(b << 16); }

// Round an fp32 value to a bf16-representable fp32 value.
template <int R>
__device__ __forceinline__ float rbf(float x) {
  if (R == RND_TRUNC) return __uint_as_float(__float_as_uint(x) & 0xFFFF0000u);
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Two fp32 -> packed bf16x2 (lo in the low half), RNE.
__device__ __forceinline__ uint32_t pack_bf16x2_rne(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <int R>
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  if (R == RND_RNE) return pack_bf16x2_rne(lo, hi);
  return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
}

// ---------------------------------------------------------------- GELU poly4
// The piecewise degree-4 erf-GELU of the reference (kernels/gelu_poly4_eval.inc
// :27-65). Its table (kernels/gelu_poly4_coeffs.h:6-13) is used the way the
// kernels use it, every entry cast (bfloat16)float at its point of use; the
// decimal literals there round to the same bf16 values in both rounding
// modes, and those bf16 values are spelled out here exactly, so the device
// code selects between immediates. (rowops.cu rounds the decimal literals on
// the host and a CPU test checks both against the oracle.)
struct Gelu4Table {
  float brk[3], shift[3], scale[3], c[3][5];
};

// Host: the table rounded to bf16 in mode R from the decimal literals (rowops.cu).
Gelu4Table gelu4_table(int mode);

// breaks {1, 2, 4}, shifts {0.5, 1.5, 3}, scales {2, 2, 1}
#define WX_GELU4_COEF                                                                  \
  {{-0x1.0cp-9f, -0x1.aap-7f, 0x1.3cp-4f, -0x1.1p-4f, -0x1.3cp-3f},                    \
   {0x1.1ap-9f, -0x1.d6p-8f, -0x1.08p-8f, 0x1.06p-4f, -0x1.9ap-4f},                    \
   {-0x1.8p-9f, 0x1.5ep-7f, -0x1.04p-6f, 0x1.8ap-7f, -0x1.08p-8f}}

// Round two fp32 values to bf16-representable values (one packed conversion
// in RNE mode).
template <int R>
__device__ __forceinline__ void rbf2(float& a, float& b) {
  if (R == RND_TRUNC) {
    a = __uint_as_float(__float_as_uint(a) & 0xFFFF0000u);
    b = __uint_as_float(__float_as_uint(b) & 0xFFFF0000u);
  } else {
    const uint32_t p = pack_bf16x2_rne(a, b);
    a = __uint_as_float(p << 16);
    b = __uint_as_float(p & 0xFFFF0000u);
  }
}

// GELU-poly4 of two bf16 values (kernels/gelu_poly4_eval.inc:27-65). The
// piece is selected, not branched on, so the compiler can interleave the
// chains of many elements, and the selection runs on the FMA pipe (the ALU
// pipe, at half its rate, carries the bf16 roundings):
//  - the 0/1 indicators pa = [s < 1], [s < 2] and [s < 4] are saturating FMAs,
//    sat(256 - 256 s) and so on: for bf16 s below a break the product is at
//    least 1, at or above it at most 0 (NaN saturates to 0);
//  - with pb = [s < 2] - pa, every coefficient is C2 + pa*(C0 - C2) +
//    pb*(C1 - C2) by two FMAs (the differences of bf16 coefficients are exact
//    in fp32), the shift 3 - 2.5*pa - 1.5*pb likewise, and the scale
//    1 + pa + pb is 1 or 2, so u = R(s - shift) * scale needs no second
//    rounding;
//  - the chain runs on min(s, 4), which changes nothing where its value is
//    kept and keeps it finite where it is multiplied by [s < 4] = 0.
// Checked on every finite and infinite bf16 input, in both rounding modes,
// against the reference's evaluation order.
template <int R>
__device__ __forceinline__ void gelu_poly4_x2(float& x0, float& x1) {
  constexpr float kC[3][5] = WX_GELU4_COEF;
  const float s0 = fabsf(x0), s1 = fabsf(x1);    // s = max(x, 0 - x)
  const float pa0 = __saturatef(fmaf(s0, -256.0f, 256.0f));
  const float pa1 = __saturatef(fmaf(s1, -256.0f, 256.0f));
  const float pb0 = __saturatef(fmaf(s0, -128.0f, 256.0f)) - pa0;
  const float pb1 = __saturatef(fmaf(s1, -128.0f, 256.0f)) - pa1;
  const float in0 = __saturatef(fmaf(s0, -64.0f, 256.0f));
  const float in1 = __saturatef(fmaf(s1, -64.0f, 256.0f));
  float t0 = fminf(s0, 4.0f) - fmaf(pa0, -2.5f, fmaf(pb0, -1.5f, 3.0f));
  float t1 = fminf(s1, 4.0f) - fmaf(pa1, -2.5f, fmaf(pb1, -1.5f, 3.0f));
  rbf2<R>(t0, t1);                                // bf16 sub
  const float u0 = t0 * (1.0f + pa0 + pb0), u1 = t1 * (1.0f + pa1 + pb1);  // exact
  auto coef = [&](int k, float pa, float pb) {
    return fmaf(pa, kC[0][k] - kC[2][k], fmaf(pb, kC[1][k] - kC[2][k], kC[2][k]));
  };
  float acc0 = coef(0, pa0, pb0), acc1 = coef(0, pa1, pb1);
#pragma unroll
  for (int k = 1; k < 5; k++) {                   // Horner, fp32 MAC, bf16 state
    rbf2<R>(acc0, acc1);
    acc0 = fmaf(acc0, u0, coef(k, pa0, pb0));
    acc1 = fmaf(acc1, u1, coef(k, pa1, pb1));
  }
  rbf2<R>(acc0, acc1);
  float r0 = fmaxf(x0, 0.0f) + acc0 * in0;        // relu(x) + q
  float r1 = fmaxf(x1, 0.0f) + acc1 * in1;
  rbf2<R>(r0, r1);
  x0 = r0;
  x1 = r1;
}

// The same function in RNE mode on two bf16 values packed in a word, with
// bf16x2 arithmetic: every bf16x2 operation rounds its exact result once, and
// on every finite bf16 input this reproduces the reference's fp32-then-bf16
// steps bit for bit (checked exhaustively against the CPU restatement, and on
// the GPU by the every-input test). The indicators are bf16x2 compares
// (1.0 / 0.0), each coefficient is pa*C0 + pb*C1 + pc*C2 with exactly one term
// nonzero (exact), and relu(x) + q is one fma with q = acc * [s < 4].
// About 33 instructions per pair instead of about 76 for the fp32 form.
// Coefficient bit patterns: the bf16 values of WX_GELU4_COEF.
#define WX_GELU4_COEF_BITS                                  \
  {{0xBB06u, 0xBC55u, 0x3D9Eu, 0xBD88u, 0xBE1Eu},            \
   {0x3B0Du, 0xBBEBu, 0xBB84u, 0x3D83u, 0xBDCDu},            \
   {0xBB40u, 0x3C2Fu, 0xBC82u, 0x3C45u, 0xBB84u}}
__device__ __forceinline__ __nv_bfloat162 bf2_bits(uint32_t w) {
  return *reinterpret_cast<const __nv_bfloat162*>(&w);
}
__device__ __forceinline__ __nv_bfloat162 bf2_splat(uint32_t h) { return bf2_bits(h | (h << 16)); }
__device__ __forceinline__ uint32_t gelu_poly4_bf16x2_rne(uint32_t xw) {
  constexpr uint32_t kCb[3][5] = WX_GELU4_COEF_BITS;
  const __nv_bfloat162 x = bf2_bits(xw);
  const __nv_bfloat162 s = bf2_bits(xw & 0x7FFF7FFFu);      // |x|
  const __nv_bfloat162 one = bf2_splat(0x3F80u), four = bf2_splat(0x4080u);
  const __nv_bfloat162 pa = __hlt2(s, one);                  // [s < 1]
  const __nv_bfloat162 pab = __hlt2(s, bf2_splat(0x4000u));  // [s < 2]
  const __nv_bfloat162 in4 = __hlt2(s, four);                // [s < 4]
  const __nv_bfloat162 pb = __hsub2(pab, pa), pc = __hsub2(one, pab);
  const __nv_bfloat162 shift =
      __hfma2(pa, bf2_splat(0xC020u), __hfma2(pb, bf2_splat(0xBFC0u), bf2_splat(0x4040u)));
  const __nv_bfloat162 t = __hsub2(__hmin2(s, four), shift);    // bf16 sub
  const __nv_bfloat162 u = __hmul2(t, __hadd2(one, pab));        // exact (x1 or x2)
  auto coef = [&](int k) {
    return __hfma2(pa, bf2_splat(kCb[0][k]),
                   __hfma2(pb, bf2_splat(kCb[1][k]), __hmul2(pc, bf2_splat(kCb[2][k]))));
  };
  __nv_bfloat162 acc = coef(0);
#pragma unroll
  for (int k = 1; k < 5; k++) acc = __hfma2(acc, u, coef(k));   // Horner
  const __nv_bfloat162 r = __hfma2(acc, in4, __hmax2(x, bf2_splat(0u)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <int R>
__device__ __forceinline__ float gelu_poly4(float x) {
  float y = 0.0f;
  gelu_poly4_x2<R>(x, y);
  return x;
}

// max of three floats in one instruction (sm_100 three-input max.f32).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the SFU (MUFU.EX2), flushing denormal results; 2^-inf = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------- programmatic dependent launch
// The encoder's forward launches its kernels as programmatic dependents of the
// kernel before them (PdlScope in wxb200_internal.h), so that a kernel's launch
// and prologue (barrier set-up, tensor-memory allocation, descriptor prefetch)
// overlap the previous kernel's last wave. Every such kernel calls pdl_wait()
// before its first access to global memory: it returns once the previous
// kernel has completed and its writes are visible (at once for a kernel not
// launched as a dependent). pdl_launch_dependents() lets the next kernel's
// CTAs start launching once every CTA of this one has issued it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- timers
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every spin-wait in these kernels gives up after this long, records
// WX_DEVERR_TIMEOUT in the device error word and lets the kernel return.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ void set_device_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait with an explicit time limit and no error reporting (used to drain copies
// still in flight on a bail-out path).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > ns) return false;
  return true;
}

// Wait for the phase with the given parity to complete. Bounded: returns false
// (and records a timeout) if it has not after kWaitTimeoutNs, or at once if
// another thread of this kernel has already recorded an error.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* err,
                                                uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (err && *reinterpret_cast<volatile int*>(err) != 0) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      set_device_error(err, WX_DEVERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_limit(bar, parity, err, kWaitTimeoutNs);
}

// ---------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load into this CTA's shared memory, completing on an
// mbarrier. x is the innermost (contiguous) coordinate in elements; callers
// keep x * sizeof(element) a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor store from this CTA's shared memory (bulk-group
// completion). Elements of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x,
                                             int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// 2-D tiled bulk tensor reduction: global[box] += shared (fp32 add in L2, each
// element once), bulk-group completion. Elements outside the tensor are skipped.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x,
                                                  int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed bulk groups are still
// reading their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's committed bulk groups are incomplete
// (their global writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Bring one 128-byte line toward L2 ahead of use.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// generic-proxy shared-memory writes -> visible to the async proxy (tcgen05.mma)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16 in, fp32 accumulate.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row
// (lane base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand stored as TMA writes it
// with 128-byte swizzling: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused
// for swizzled K-major), stride byte offset >> 4 [32,46), version 1 [46,48),
// layout type SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// The same layout read MN-major (the contiguous 128-byte rows run along N):
// one 64-element atom along N, 8-row K groups 1024 bytes apart (stride byte
// offset); the leading byte offset would step between N atoms.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// The same descriptors as two 32-bit words. The high word (stride byte offset
// 1024, version 1, SWIZZLE_128B) is a constant of the layout; the low word is
// the start address >> 4 with the leading byte offset, so stepping along K (32
// bytes: +2) or between ring slots is one 32-bit add in the MMA issuer's loop.
constexpr uint32_t kSdescHiSw128 = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t sdesc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
// D[tmem] (+)= A[smem] * B[smem]^T with the descriptors given as low words
// (shared high word `hi`).
__device__ __forceinline__ void umma_bf16_ss_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                                uint32_t hi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 ad, {%1, %5};\n\t"
      "mov.b64 bd, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(hi)
      : "memory");
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A
// and B (bits 7-9, 10-12 = 1), A/B major (bits 15, 16), N >> 3 (bits 17-22),
// M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major,
                                                      int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- int8 quantisation
// x / s rounded to nearest (IEEE), for a per-row divisor s with rcp = RN(1/s)
// (__frcp_rn): q = RN(x * rcp) is within one ulp of x / s, the residual
// x - s*q is exact in one FMA, and RN(q + residual * rcp) is then the correctly
// rounded quotient (Markstein's theorem; P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990). It holds while nothing overflows or goes subnormal, so
// callers use it for s in [2^-100, 2^100] and |x| < 2^100 only.
__device__ __forceinline__ float2 div2_rn(float2 x, float2 s, float2 rcp) {
  const float2 q = __fmul2_rn(x, rcp);
  const float2 r = __ffma2_rn(make_float2(-q.x, -q.y), s, x);
  return __ffma2_rn(r, rcp, q);
}
__device__ __forceinline__ bool div2_rn_safe(float s) {
  return s >= 7.8886091e-31f && s <= 1.2676506e30f;   // 2^-100 .. 2^100
}
// rint(x / s) of four values as packed int8 (half to even; |x / s| <= 127.5)
__device__ __forceinline__ uint32_t quant4_i8(float x0, float x1, float x2, float x3, float s,
                                              float rcp, bool fast) {
  float q0, q1, q2, q3;
  if (fast) {
    const float2 s2 = make_float2(s, s), r2 = make_float2(rcp, rcp);
    const float2 a = div2_rn(make_float2(x0, x1), s2, r2);
    const float2 b = div2_rn(make_float2(x2, x3), s2, r2);
    q0 = a.x; q1 = a.y; q2 = b.x; q3 = b.y;
  } else {
    q0 = __fdiv_rn(x0, s); q1 = __fdiv_rn(x1, s); q2 = __fdiv_rn(x2, s); q3 = __fdiv_rn(x3, s);
  }
  return ((uint32_t)__float2int_rn(q0) & 0xFFu) | (((uint32_t)__float2int_rn(q1) & 0xFFu) << 8) |
         (((uint32_t)__float2int_rn(q2) & 0xFFu) << 16) |
         (((uint32_t)__float2int_rn(q3) & 0xFFu) << 24);
}

// Instruction descriptor, kind::i8: s32 accumulator (bits 4-5 = 2), signed
// 8-bit A and B (bits 7-9, 10-12 = 1), both K-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace wx
