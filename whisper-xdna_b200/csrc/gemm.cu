// bf16 GEMM with fp32 accumulation on the sm_100a tensor cores (tcgen05) and
// fused epilogues: the QKV / out-proj / fc1 / fc2 / conv GEMMs of the encoder.
//
//   C = epilogue(A @ B^T), A (M x K) bf16 row-major, B (N x K) bf16 row-major
//   (the torch Linear weight), fp32 accumulator in tensor memory.
//
// Design (one persistent CTA per SM, 10 warps):
//   warp 0     TMA producer: A and B tiles (128 x 64 and BN x 64 bf16, 128-byte
//              swizzle) into a STAGES-deep shared-memory ring
//   warp 1     allocates tensor memory and issues tcgen05.mma (M=128, N=BN,
//              K=16 per instruction) from one thread; tcgen05.commit frees the
//              ring slot and publishes the finished accumulator
//   warps 2-9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//              32*(w%4)...; warps 2-5 take the first half of the columns, 6-9
//              the second), bias / residual / GELU, bf16 or fp32 stores
// The accumulator is double-buffered in tensor memory (2 x BN columns), so the
// epilogue of one tile overlaps the MMAs of the next. Tiles are visited
// N-fastest so the CTAs in flight share A tiles through L2; the weights
// (<= 13 MB per GEMM) stay L2-resident.
//
// Large problems run gemm2_bf16_kernel on CTA pairs (tcgen05 cta_group::2,
// 256 x 256 tiles), whose epilogue goes through shared memory and TMA tensor
// stores (and TMA loads of the residual). Both kernels are templated on I8:
// int8 A and B (kind::i8, s32 accumulator) with the dequantising epilogue of
// the int8 mode, (float(acc) * sa[row]) * sw[col].
//
// It replaces the whole-array AIE GEMM the reference drives through
// RawRT.matmul / mm_start / mm_finish (src/rawxrt.py:926-996); its bias fold
// (ones column on A, bias row on B, src/rawxrt.py:352-371) becomes a bias
// added to the fp32 accumulator in the epilogue.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = kGemmBM * kGemmBK * 2;
  static constexpr int B_BYTES = BN * kGemmBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// int8 GEMM: accumulator columns n..n+31 of one row as fp32,
// (float(acc) * sa[row]) * sw[col], each product rounded on its own (the order
// of the reference's (A_q @ B_q) * sa * sw in fp32).
__device__ __forceinline__ void dequant32(const GemmArgs& a, float s_row, int n,
                                          const uint32_t (&acc)[32], float (&v)[32]) {
  if (n + 32 <= a.N) {
    // packed fp32 pairs: each product rounded on its own, as fmul.rn
    const float2 sr = make_float2(s_row, s_row);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(a.sw + n + j));
      const float2 p0 = __fmul2_rn(__fmul2_rn(make_float2(__int2float_rn((int)acc[j]),
                                                          __int2float_rn((int)acc[j + 1])), sr),
                                   make_float2(w.x, w.y));
      const float2 p1 = __fmul2_rn(__fmul2_rn(make_float2(__int2float_rn((int)acc[j + 2]),
                                                          __int2float_rn((int)acc[j + 3])), sr),
                                   make_float2(w.z, w.w));
      v[j] = p0.x; v[j + 1] = p0.y; v[j + 2] = p1.x; v[j + 3] = p1.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      v[j] = n + j < a.N ? __fmul_rn(__fmul_rn(__int2float_rn((int)acc[j]), s_row), a.sw[n + j])
                         : 0.0f;
  }
}

// max |x| over the bf16 pairs w[0..npairs) whose columns lie below `valid`
// (column 2i in the low half), as bf16 magnitude bits
template <int NP>
__device__ __forceinline__ uint32_t absmax_bf16x2(const uint32_t (&w)[NP], int valid) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < NP; i++) {
    const uint32_t lo = 2 * i < valid ? (w[i] & 0x7FFFu) : 0u;
    const uint32_t hi = 2 * i + 1 < valid ? ((w[i] >> 16) & 0x7FFFu) : 0u;
    m = max(m, max(lo, hi));
  }
  return m;
}
// fold a bf16 magnitude into rowmax[row] (fp32 bits of non-negative values
// order like unsigned integers)
__device__ __forceinline__ void rowmax_update(float* rowmax, int row, uint32_t bf16_mag) {
  if (bf16_mag) atomicMax(reinterpret_cast<unsigned int*>(rowmax) + row, bf16_mag << 16);
}

// Apply the epilogue to 32 consecutive accumulator columns of one row and
// store them. `full` = all 32 columns are inside N and the stores may be
// vectorized.
template <int EPI, bool I8>
__device__ __forceinline__ void epilogue_store32(const GemmArgs& a, int row, int n, bool full,
                                                 const uint32_t (&acc)[32]) {
  float v[32];
  if constexpr (I8) {
    dequant32(a, a.sa[row], n, acc, v);
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(acc[j]);
  }
  if (a.bias) {
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + n + j));
        v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n + j < a.N) v[j] += a.bias[n + j];
    }
  }
  if (EPI == WX_EPI_F32_RESID) {
    const float* r = a.R + (int64_t)row * a.ldr + n;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(r + j);
        v[j] += t.x; v[j + 1] += t.y; v[j + 2] += t.z; v[j + 3] += t.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n + j < a.N) v[j] += r[j];
    }
  }
  if (EPI == WX_EPI_BF16_GELU || EPI == kEpiF32GeluPos) {
    // g4f: input rounded to bf16 (RNE), then poly4 on packed pairs
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; j++)
      w[j] = gelu_poly4_bf16x2_rne(pack_bf16x2_rne(v[2 * j], v[2 * j + 1]));
    if constexpr (EPI == WX_EPI_BF16_GELU) {
      if (a.rowmax) rowmax_update(a.rowmax, row, absmax_bf16x2(w, a.N - n));
      uint16_t* c = reinterpret_cast<uint16_t*>(a.C) + (int64_t)row * a.ldc + n;
      if (full) {
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<uint4*>(c + 2 * j) = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (n + j < a.N) c[j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
      }
      return;
    } else {
#pragma unroll
      for (int j = 0; j < 16; j++) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
  if (EPI == WX_EPI_BF16_GELU_ERF || EPI == kEpiF32GeluErfPos) {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = gelu_erf(v[j]);
  }
  if (EPI == kEpiF32GeluPos || EPI == kEpiF32GeluErfPos) {
    const float* pp = a.pos + (int64_t)(row % a.pos_T) * a.ldp + n;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(pp + j));
        v[j] += t.x; v[j + 1] += t.y; v[j + 2] += t.z; v[j + 3] += t.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n + j < a.N) v[j] += pp[j];
    }
  }
  if (EPI == WX_EPI_F32 || EPI == WX_EPI_F32_RESID || EPI == kEpiF32GeluPos ||
      EPI == kEpiF32GeluErfPos) {
    float* c = reinterpret_cast<float*>(a.C) + (int64_t)row * a.ldc + n;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n + j < a.N) c[j] = v[j];
    }
  } else {
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; j++) w[j] = pack_bf16x2_rne(v[2 * j], v[2 * j + 1]);
    if (a.rowmax) rowmax_update(a.rowmax, row, absmax_bf16x2(w, a.N - n));
    uint16_t* c = reinterpret_cast<uint16_t*>(a.C) + (int64_t)row * a.ldc + n;
    if (full) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<uint4*>(c + 2 * j) = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n + j < a.N) c[j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
    }
  }
}

// Epilogues that the 2-SM kernel writes through shared memory and TMA stores:
// each epilogue warp stages 32 rows x 128 bytes of its share of the tile (32
// fp32 or 64 bf16 columns) and stores the box with one bulk tensor copy; the
// residual of WX_EPI_F32_RESID arrives in the same buffer by a TMA load two
// chunks ahead. Row-per-thread global accesses (one 16-byte piece of 32
// different rows per instruction) cost a wavefront per sector, which the
// short-K residual GEMMs could not hide behind their MMAs.
template <int EPI>
struct TmaEpi {
  static constexpr bool kOn = EPI == WX_EPI_F32 || EPI == WX_EPI_F32_RESID || EPI == WX_EPI_BF16 ||
                              EPI == WX_EPI_BF16_GELU || EPI == WX_EPI_BF16_GELU_ERF;
  static constexpr bool kF32 = EPI == WX_EPI_F32 || EPI == WX_EPI_F32_RESID;
  static constexpr int kCols = kF32 ? 32 : 64;   // columns of one 128-byte staged row
};
constexpr int kEpiBufBytes = 32 * 128;   // one warp's chunk: 32 rows x 128 bytes

__device__ __forceinline__ void add_bias32(const GemmArgs& a, int n, float (&v)[32]) {
  if (!a.bias) return;
  if (n + 32 <= a.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + n + j));
      const float2 s0 = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(b.x, b.y));
      const float2 s1 = __fadd2_rn(make_float2(v[j + 2], v[j + 3]), make_float2(b.z, b.w));
      v[j] = s0.x; v[j + 1] = s0.y; v[j + 2] = s1.x; v[j + 3] = s1.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (n + j < a.N) v[j] += a.bias[n + j];
  }
}

// One chunk of a warp's share of the tile into its staging buffer, thread =
// row: `rowp` is this thread's 128-byte row, whose 16-byte unit j sits at unit
// j ^ (row & 7) (the 128-byte swizzle of the tensor maps, so that the eight
// threads of each shared-memory phase hit eight different bank groups).
// t_col: tensor-memory address of the chunk's first column for this warp's
// lanes; n: its first output column. WX_EPI_F32_RESID finds the residual in
// the buffer and adds it. s_row: the row's int8 scale (I8). Returns, for the
// bf16 outputs, max |value| over the chunk's columns inside N as bf16
// magnitude bits (0 otherwise).
template <int EPI, bool I8, bool SEQ>
__device__ __forceinline__ uint32_t epi_chunk_to_smem(const GemmArgs& a, uint32_t t_col, int n,
                                                      uint8_t* rowp, int lane, float s_row) {
  const int sw = lane & 7;
  if constexpr (TmaEpi<EPI>::kF32) {
    uint32_t r[32];
    tmem_ld32(t_col, r);
    tmem_wait_ld();
    float v[32];
    if constexpr (I8) {
      dequant32(a, s_row, n, r, v);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
    }
    add_bias32(a, n, v);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float4* p = reinterpret_cast<float4*>(rowp + ((j ^ sw) << 4));
      if constexpr (EPI == WX_EPI_F32_RESID) {
        if (!a.resid_inplace) {
          const float4 t = *p;
          v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
        }
      }
      *p = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    return 0u;
  } else {
    // SEQ: one half's columns at a time (fewer live registers at 576 threads);
    // otherwise both halves' loads in flight together
    uint32_t r0[32], r1[32];
    if constexpr (!SEQ) {
      tmem_ld32(t_col, r0);
      tmem_ld32(t_col + 32, r1);
      tmem_wait_ld();
    }
    uint32_t mx = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      if constexpr (SEQ) {
        tmem_ld32(t_col + 32 * h, r0);
        tmem_wait_ld();
      }
      const uint32_t (&r)[32] = (SEQ || h == 0) ? r0 : r1;
      float v[32];
      if constexpr (I8) {
        dequant32(a, s_row, n + 32 * h, r, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
      }
      add_bias32(a, n + 32 * h, v);
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        if constexpr (EPI == WX_EPI_BF16_GELU)   // g4f: rne(x), then poly4 on packed pairs
          w[j] = gelu_poly4_bf16x2_rne(pack_bf16x2_rne(v[2 * j], v[2 * j + 1]));
        else if constexpr (EPI == WX_EPI_BF16_GELU_ERF)
          w[j] = pack_bf16x2_rne(gelu_erf(v[2 * j]), gelu_erf(v[2 * j + 1]));
        else
          w[j] = pack_bf16x2_rne(v[2 * j], v[2 * j + 1]);
      }
#pragma unroll
      for (int q = 0; q < 4; q++)
        *reinterpret_cast<uint4*>(rowp + (((4 * h + q) ^ sw) << 4)) =
            make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      if (a.rowmax) mx = max(mx, absmax_bf16x2(w, a.N - n - 32 * h));
    }
    return mx;
  }
}

// One K step of the MMA issuer: 4 instructions of K = 32 bytes (16 bf16 or
// 32 int8 elements); the descriptor address advances by 2 (16-byte units).
template <bool I8>
__device__ __forceinline__ void umma_ss_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                           uint32_t hi, uint32_t idesc, uint32_t accumulate) {
  if constexpr (I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "mov.b64 ad, {%1, %5};\n\t"
        "mov.b64 bd, {%2, %5};\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], ad, bd, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(hi)
        : "memory");
  } else {
    umma_bf16_ss_lo(d_tmem, a_lo, b_lo, hi, idesc, accumulate);
  }
}

constexpr int kGemmThreads = 320;
constexpr int kGemmEpiThreads = 256;

template <int BN, int EPI, bool I8>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  using Cfg = GemmCfg<BN>;
  constexpr int kKElems = I8 ? 2 * kGemmBK : kGemmBK;   // elements per 128-byte K step
  constexpr int S = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = warp_id(), lane = lane_id();
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpiThreads);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nnb = a.num_n_blocks, nkb = a.num_k_blocks;
  pdl_wait();   // the operands and the residual come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0, issued_phase = 0;  // per-slot bits
      for (int tile = blockIdx.x; ok && tile < a.num_tiles; tile += gridDim.x) {
        const int m0 = (tile / nnb) * kGemmBM, n0 = (tile % nnb) * BN;
        // the next kernel may start launching once every CTA is on its last tile
        if (tile + (int)gridDim.x >= a.num_tiles) pdl_launch_dependents();
        for (int kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, a.err)) { ok = false; break; }
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(&tmA, &full[stage], sA + stage * Cfg::A_BYTES, kb * kKElems, m0);
          tma_load_2d(&tmB, &full[stage], sB + stage * Cfg::B_BYTES, kb * kKElems, n0);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      // Loads still in flight land before the CTA retires: wait (1 ms at most
      // per slot) for the slots the MMA warp will no longer consume.
      if (!ok)
        for (int s = 0; s < S; s++)
          if (issued & (1u << s)) mbar_wait_for(&full[s], (issued_phase >> s) & 1u, 1000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = I8 ? idesc_s8_s32(kGemmBM, BN) : idesc_bf16_f32(kGemmBM, BN, 0, 0);
      const uint32_t hi = kSdescHiSw128;
      const uint32_t a_lo = sdesc_lo(smem_u32(sA), 16), b_lo = sdesc_lo(smem_u32(sB), 16);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < a.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, a.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(&full[stage], phase, a.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ad = a_lo + (uint32_t)(stage * (Cfg::A_BYTES >> 4));
          const uint32_t bd = b_lo + (uint32_t)(stage * (Cfg::B_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; k++)   // 32 bytes of K per MMA: +2
            umma_ss_lo<I8>(d_tmem, ad + 2 * k, bd + 2 * k, hi, idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // every MMA issued has completed before tensor memory is released
      umma_commit(done);
      mbar_wait_for(done, 0, kWaitTimeoutNs);
    }
  } else {
    // ---------------- epilogue: warps 2..9
    const int sub = warp & 3;  // TMEM lanes 32*sub .. 32*sub+31
    const int half = (warp - 2) >> 2;  // column half of the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x) {
      const int m0 = (tile / nnb) * kGemmBM, n0 = (tile % nnb) * BN;
      if (!mbar_wait(&tfull[acc], acc_phase, a.err)) break;
      tc_fence_after();
      if (EPI == WX_EPI_F32_RESID) {
        // the residual rows of this warp's next tile, into L2 while this tile drains
        const int nt = tile + gridDim.x;
        if (nt < a.num_tiles) {
          const int prow = (nt / nnb) * kGemmBM + sub * 32 + lane;
          const int pn = (nt % nnb) * BN + half * (BN / 2);
          if (prow < a.M) {
            const float* base = a.R + (int64_t)prow * a.ldr + pn;
#pragma unroll
            for (int q = 0; q < BN / 64; q++)
              if (pn + q * 32 < a.N) prefetch_l2(base + q * 32);
          }
        }
      }
      const int row = m0 + sub * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); c++) {
        const int n = n0 + c * 32;
        if (n >= a.N) break;  // uniform across the warp
        uint32_t r[32];
        tmem_ld32(t_row + (uint32_t)(c * 32), r);
        tmem_wait_ld();
        if (row < a.M) epilogue_store32<EPI, I8>(a, row, n, n + 32 <= a.N, r);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- 2-SM GEMM
// The same GEMM on CTA pairs (a cluster of two, tcgen05 cta_group::2): the
// pair computes 256 x 256 tiles with M=256, N=256 MMAs issued by the leader
// (cluster rank 0). Rank r stages rows [128 r, 128 r + 128) of the A tile and
// rows [128 r, 128 r + 128) of the B tile (32 KB per 64-wide K step instead
// of 48 KB for 128 x 256 on one SM, so six stages fit), and holds accumulator
// rows [128 r, 128 r + 128) x 256 columns in its own tensor memory; the
// tensor cores of the pair exchange the B halves themselves. Synchronisation:
//   full[s]    leader only: armed by the leader's producer with both CTAs'
//              bytes; both CTAs' TMA loads complete on it (cta_group::2 form)
//   empty[s]   both CTAs: the leader commits the MMAs of a step to its own
//              and to the peer's barrier (two commits, same offset)
//   tfull[b]   both CTAs, committed like empty
//   tempty[b]  leader only: one arrival per epilogue warp of either CTA
//   rfull[w][b] WX_EPI_F32_RESID: residual chunk landed in buffer b of
//              epilogue warp w
// Every wait is bounded; both CTAs always reach the final cluster barrier,
// after which the tensor memory of the pair is released. With the TMA
// epilogue the ring has five stages (160 KB) beside the 64 KB of staging
// buffers (8 warps x 2 x 4 KB); otherwise six.
constexpr int kGemm2ABytes = 128 * kGemmBK * 2;                   // 16 KB
constexpr int kGemm2BBytes = 128 * kGemmBK * 2;                   // 16 KB (half of N=256)
constexpr int kGemm2StageBytes = kGemm2ABytes + kGemm2BBytes;
constexpr int kGemm2EpiBytes = 64 * 1024;          // staging buffers of the TMA epilogue
constexpr int kGemm2BarBytes = 512;
template <int EPI, bool I8>
struct Gemm2Cfg {
  static constexpr int STAGES = TmaEpi<EPI>::kOn ? 5 : 6;
  // Epilogue warps: 8 (two per sub-partition, each 32 rows x 128 columns of a
  // tile, two 4 KB staging buffers each), or 16 for the int8 GELU epilogues
  // (32 rows x 64 columns, one buffer each): at the int8 MMA rate the GELU
  // epilogue of fc1 is latency-bound with two warps per sub-partition.
  static constexpr bool kGeluOut = EPI == WX_EPI_BF16_GELU || EPI == WX_EPI_BF16_GELU_ERF;
  static constexpr int EPI_WARPS = (I8 && kGeluOut) ? 16 : 8;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int NBUF = TmaEpi<EPI>::kOn ? kGemm2EpiBytes / (EPI_WARPS * kEpiBufBytes) : 0;
  static constexpr int EPI_BYTES = TmaEpi<EPI>::kOn ? kGemm2EpiBytes : 0;
  static constexpr int SMEM = STAGES * kGemm2StageBytes + EPI_BYTES + 1024 + kGemm2BarBytes;
  static_assert(SMEM <= 232448, "2-SM GEMM shared memory");
  static_assert(!TmaEpi<EPI>::kOn || NBUF >= 1, "a staging buffer per epilogue warp");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at local shared address `a` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// TMA tile load into this CTA's shared memory, completing on an mbarrier that
// may be the peer CTA's (the cta_group::2 form: one destination, this CTA)
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_cluster,
                                                 void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_local(uint64_t* bar, uint32_t bytes) {
  mbar_arrive_expect_tx(bar, bytes);
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void umma_bf16_ss_lo_pair(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                                     uint32_t hi, uint32_t idesc,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 ad, {%1, %5};\n\t"
      "mov.b64 bd, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], ad, bd, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(hi)
      : "memory");
}
template <bool I8>
__device__ __forceinline__ void umma_ss_lo_pair(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                                uint32_t hi, uint32_t idesc, uint32_t accumulate) {
  if constexpr (I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "mov.b64 ad, {%1, %5};\n\t"
        "mov.b64 bd, {%2, %5};\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], ad, bd, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(hi)
        : "memory");
  } else {
    umma_bf16_ss_lo_pair(d_tmem, a_lo, b_lo, hi, idesc, accumulate);
  }
}
// Arrive on the mbarrier at shared::cluster address `bar` (either CTA of the
// pair) once every cta_group::2 MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

template <int EPI, bool I8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2Cfg<EPI, I8>::THREADS, 1)
    gemm2_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC,
                      const __grid_constant__ CUtensorMap tmR, const GemmArgs a) {
  using Cfg = Gemm2Cfg<EPI, I8>;
  constexpr int S = Cfg::STAGES;
  constexpr int kKElems = I8 ? 2 * kGemmBK : kGemmBK;   // elements per 128-byte K step
  constexpr int BN = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kGemm2ABytes;
  uint8_t* sE = smem + S * kGemm2StageBytes;   // epilogue staging (TMA epilogues)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + Cfg::EPI_BYTES);
  uint64_t* full = bars;            // [S], used in the leader
  uint64_t* empty = bars + S;       // [S]
  uint64_t* tfull = bars + 2 * S;   // [2]
  uint64_t* tempty = tfull + 2;     // [2], used in the leader
  uint64_t* done = tempty + 2;
  constexpr int EW = Cfg::EPI_WARPS, NB = Cfg::NBUF > 0 ? Cfg::NBUF : 1;
  uint64_t* rfull = done + 1;       // [EW warps][NB buffers]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + EW * NB);
  static_assert((2 * S + 5 + EW * NB) * 8 + 4 <= kGemm2BarBytes, "barriers");

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EW);
    }
    mbar_init(done, 1);
    for (int i = 0; i < EW * NB; i++) mbar_init(&rfull[i], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (TmaEpi<EPI>::kOn) tma_prefetch_desc(&tmC);
    if constexpr (EPI == WX_EPI_F32_RESID) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();   // barriers of both CTAs initialised, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nnb = a.num_n_blocks, nkb = a.num_k_blocks;
  pdl_wait();   // the operands and the residual come from the previous kernel
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; ok && tile < a.num_tiles; tile += npairs) {
        const int m0 = (tile / nnb) * 256, n0 = (tile % nnb) * BN;
        // the next kernel may start launching once every CTA is on its last tile
        if (tile + npairs >= a.num_tiles) pdl_launch_dependents();
        for (int kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, a.err)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * kGemm2StageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(&tmA, fb, sA + stage * kGemm2ABytes, kb * kKElems, m0 + (int)rank * 128);
          tma_load_2d_pair(&tmB, fb, sB + stage * kGemm2BBytes, kb * kKElems, n0 + (int)rank * 128);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader)
      constexpr uint32_t idesc = I8 ? idesc_s8_s32(256, BN) : idesc_bf16_f32(256, BN, 0, 0);
      const uint32_t hi = kSdescHiSw128;
      const uint32_t a_lo = sdesc_lo(smem_u32(sA), 16), b_lo = sdesc_lo(smem_u32(sB), 16);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int tile = pair; ok && tile < a.num_tiles; tile += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, a.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nkb; kb++) {
          if (!mbar_wait(&full[stage], phase, a.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ad = a_lo + (uint32_t)(stage * (kGemm2ABytes >> 4));
          const uint32_t bd = b_lo + (uint32_t)(stage * (kGemm2BBytes >> 4));
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; k++)   // 32 bytes of K per MMA: +2
            umma_ss_lo_pair<I8>(d_tmem, ad + 2 * k, bd + 2 * k, hi, idesc, (kb | k) != 0);
          umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 0));
        umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // every MMA issued has completed before the pair's tensor memory is released
      umma_commit_pair(mapa_shared(smem_u32(done), 0));
      mbar_wait_for(done, 0, kWaitTimeoutNs);
    }
  } else if constexpr (TmaEpi<EPI>::kOn) {
    // ---------------- epilogue through shared memory + TMA stores: warps 2..17
    constexpr int kCols = TmaEpi<EPI>::kCols;      // columns per staged chunk
    constexpr int kPartCols = BN / (EW / 4);       // columns per warp: 64
    constexpr int kChunks = kPartCols / kCols;     // 1 (bf16) or 2 (fp32) per tile
    const int sub = warp & 3;                      // TMEM lanes 32*sub .. 32*sub+31
    const int part = (warp - 2) >> 2;              // column part of the tile
    uint8_t* ebuf = sE + (warp - 2) * NB * kEpiBufBytes;
    uint64_t* rf = rfull + NB * (warp - 2);
    const int row_off = (int)rank * 128 + sub * 32;
    // this warp's chunks of a tile: a prefix of kChunks (none past M or N)
    auto chunks_of = [&](int tile) -> int {
      const int r0 = (tile / nnb) * 256 + row_off, c0 = (tile % nnb) * BN + part * kPartCols;
      if (r0 >= a.M || c0 >= a.N) return 0;
      return min(kChunks, (a.N - c0 + kCols - 1) / kCols);
    };
    // residual loads (lane 0) run NB chunks ahead, across tiles
    int lt = pair, lc = 0;
    uint32_t lk = 0;
    auto load_next = [&]() {
      while (lt < a.num_tiles && lc >= chunks_of(lt)) { lt += npairs; lc = 0; }
      if (lt >= a.num_tiles) return;
      const uint32_t b = lk % NB;
      mbar_arrive_expect_tx(&rf[b], kEpiBufBytes);
      tma_load_2d(&tmR, &rf[b], ebuf + b * kEpiBufBytes,
                  (lt % nnb) * BN + part * kPartCols + lc * kCols, (lt / nnb) * 256 + row_off);
      lc++;
      lk++;
    };
    // residual in place (C == R): the epilogue writes acc + bias and a TMA
    // reduce-add folds it into C, so no residual is loaded
    const bool resid_ld = EPI == WX_EPI_F32_RESID && !a.resid_inplace;
    if (resid_ld && lane == 0)
      for (int i = 0; i < NB; i++) load_next();
    int acc = 0;
    uint32_t acc_phase = 0, k = 0;
    for (int tile = pair; ok && tile < a.num_tiles; tile += npairs) {
      ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, a.err));
      if (!ok) break;
      tc_fence_after();
      const int nc = chunks_of(tile);
      const int r0 = (tile / nnb) * 256 + row_off, c0 = (tile % nnb) * BN + part * kPartCols;
      const uint32_t t_row = tmem_base + ((uint32_t)(sub * 32) << 16) +
                             (uint32_t)(acc * BN + part * kPartCols);
      const int row = r0 + lane;
      float s_row = 0.0f;
      if constexpr (I8) s_row = row < a.M ? a.sa[row] : 0.0f;
      uint32_t mx = 0;
      for (int c = 0; c < nc; c++, k++) {
        uint8_t* buf = ebuf + (k % NB) * kEpiBufBytes;
        if (resid_ld) {
          ok = __all_sync(0xffffffffu, mbar_wait(&rf[k % NB], (k / NB) & 1, a.err));
          if (!ok) break;
        } else {
          if (lane == 0) bulk_wait_group_read<NB - 1>();   // the store of chunk k-NB has read buf
          __syncwarp();
        }
        mx = max(mx, epi_chunk_to_smem<EPI, I8, (EW > 8)>(a, t_row + (uint32_t)(c * kCols),
                                                           c0 + c * kCols, buf + lane * 128,
                                                           lane, s_row));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (EPI == WX_EPI_F32_RESID && a.resid_inplace)
            tma_reduce_add_2d(&tmC, buf, c0 + c * kCols, r0);
          else
            tma_store_2d(&tmC, buf, c0 + c * kCols, r0);
          bulk_commit_group();
          if (resid_ld) {
            bulk_wait_group_read<0>();   // the store has read buf: refill it
            load_next();
          }
        }
      }
      if (!ok) break;
      if (!TmaEpi<EPI>::kF32 && a.rowmax && row < a.M) rowmax_update(a.rowmax, row, mx);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait_group<0>();   // stores complete before the CTA retires
  } else {
    // ---------------- epilogue: warps 2..9 of both CTAs
    const int sub = warp & 3;          // TMEM lanes 32*sub .. 32*sub+31
    const int half = (warp - 2) >> 2;  // column half of the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < a.num_tiles; tile += npairs) {
      const int m0 = (tile / nnb) * 256 + (int)rank * 128, n0 = (tile % nnb) * BN;
      if (!mbar_wait(&tfull[acc], acc_phase, a.err)) { ok = false; break; }
      tc_fence_after();
      if (EPI == WX_EPI_F32_RESID) {
        // the residual rows of this warp's next tile, into L2 while this tile drains
        const int nt = tile + npairs;
        if (nt < a.num_tiles) {
          const int prow = (nt / nnb) * 256 + (int)rank * 128 + sub * 32 + lane;
          const int pn = (nt % nnb) * BN + half * (BN / 2);
          if (prow < a.M) {
            const float* base = a.R + (int64_t)prow * a.ldr + pn;
#pragma unroll
            for (int q = 0; q < BN / 64; q++)
              if (pn + q * 32 < a.N) prefetch_l2(base + q * 32);
          }
        }
      }
      const int row = m0 + sub * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); c++) {
        const int n = n0 + c * 32;
        if (n >= a.N) break;  // uniform across the warp
        uint32_t r[32];
        tmem_ld32(t_row + (uint32_t)(c * 32), r);
        tmem_wait_ld();
        if (row < a.M) epilogue_store32<EPI, I8>(a, row, n, n + 32 <= a.N, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  // On a failed wait, loads this CTA issued may still be landing in its
  // shared memory: give them 50 us before the pair retires.
  if (!ok || (a.err && *reinterpret_cast<volatile int*>(a.err) != 0)) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 50000ull) __nanosleep(1000);
  }
  tc_fence_before();
  cluster_sync_all();   // no MMA reads this CTA's shared memory or tensor memory any more
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

static int gemm_prepare(int bn, int epi, bool pair, bool i8);

// CTA pairs (the 2-SM kernel) when the 256 x 256 tiles fill every SM pair at
// least once; smaller problems spread better over single-SM tiles.
static bool use_pair(int64_t M, int64_t N, int nsm) {
  return N > 128 && ((M + 255) / 256) * ((N + 255) / 256) >= nsm / 2;
}

// Tensor maps of the 2-SM kernel's TMA epilogue: C (and the residual) in
// boxes of 32 rows x 128 bytes with the 128-byte swizzle; left zeroed for the
// epilogues that store from registers.
static int encode_epilogue_maps(GemmPlan* p, void* C, const float* R, int64_t M, int64_t N,
                                int64_t ldc, int64_t ldr, int epi) {
  memset(&p->tmC, 0, sizeof(p->tmC));
  memset(&p->tmR, 0, sizeof(p->tmR));
  const bool f32 = epi == WX_EPI_F32 || epi == WX_EPI_F32_RESID;
  const bool bf16 = epi == WX_EPI_BF16 || epi == WX_EPI_BF16_GELU || epi == WX_EPI_BF16_GELU_ERF;
  if (!p->pair || !(f32 || bf16)) return WX_OK;
  if (f32)
    WX_TRY(encode_tensor_map_2d(&p->tmC, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)N,
                                (uint64_t)M, (uint64_t)ldc * 4, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B));
  else
    WX_TRY(encode_tensor_map_2d(&p->tmC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)N,
                                (uint64_t)M, (uint64_t)ldc * 2, 64, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B));
  if (epi == WX_EPI_F32_RESID)
    WX_TRY(encode_tensor_map_2d(&p->tmR, R, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)N,
                                (uint64_t)M, (uint64_t)ldr * 4, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B));
  return WX_OK;
}

// err: the error word the kernels' bounded waits record into; NULL takes the
// library's per-device word (device_error_word(), allocated on first use).
static int gemm_plan_impl(GemmPlan* p, const void* A, const void* B, const float* bias,
                          const float* R, void* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                          int64_t ldb, int64_t ldc, int64_t ldr, int epi, int force_bn, bool i8,
                          const float* sa, const float* sw, float* rowmax, int* err) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(WX_ERR_INVALID, "gemm: M, N, K must be > 0");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(WX_ERR_UNSUPPORTED, "gemm: dimension exceeds 2^31");
  if (!A || !B || !C) return fail(WX_ERR_INVALID, "gemm: NULL operand");
  const bool pos_epi = epi == kEpiF32GeluPos || epi == kEpiF32GeluErfPos;
  if ((epi < WX_EPI_F32 || epi > WX_EPI_BF16_GELU_ERF) && !pos_epi)
    return fail(WX_ERR_INVALID, "gemm: epilogue %d", epi);
  if (epi == WX_EPI_F32_RESID && !R) return fail(WX_ERR_INVALID, "gemm: residual is NULL");
  if (lda < K || ldb < K || ldc < N) return fail(WX_ERR_INVALID, "gemm: leading dimension too small");
  const int a_align = i8 ? 16 : 8;   // elements per 16 bytes
  if (lda % a_align || ldb % a_align)
    return fail(WX_ERR_INVALID, "gemm: lda and ldb must keep rows 16-byte aligned");
  const bool f32_out = epi == WX_EPI_F32 || epi == WX_EPI_F32_RESID || pos_epi;
  if (ldc % (f32_out ? 4 : 8)) return fail(WX_ERR_INVALID, "gemm: ldc must keep rows 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(C) & 15) || (bias && (reinterpret_cast<uintptr_t>(bias) & 15)))
    return fail(WX_ERR_INVALID, "gemm: C and bias must be 16-byte aligned");
  if (R && ((reinterpret_cast<uintptr_t>(R) & 15) || ldr % 4 || ldr < N))
    return fail(WX_ERR_INVALID, "gemm: residual must be 16-byte aligned with ldr a multiple of 4");
  if (i8 && (!sa || !sw || (reinterpret_cast<uintptr_t>(sw) & 15)))
    return fail(WX_ERR_INVALID, "gemm: int8 needs row scales and 16-byte aligned column scales");
  if (rowmax && f32_out)
    return fail(WX_ERR_INVALID, "gemm: row maxima are collected for bf16 outputs only");
  const int nsm = sm_count();
  const int64_t mb = (M + kGemmBM - 1) / kGemmBM;
  int bn = force_bn;
  if (bn == 0) bn = (mb * ((N + 255) / 256) >= nsm && N > 128) ? 256 : 128;
  if (bn != 128 && bn != 256) return fail(WX_ERR_INVALID, "gemm: BN %d", bn);
  const bool pair = force_bn == 0 && use_pair(M, N, nsm);
  if (!err) err = device_error_word();
  if (!err) return fail(WX_ERR_CUDA, "gemm: device error word unavailable");
  // one K step is 128 bytes of every row: 64 bf16 or 128 int8 elements
  const CUtensorMapDataType dt = i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int es = i8 ? 1 : 2;
  const uint32_t kstep = (uint32_t)(128 / es);
  WX_TRY(encode_tensor_map_2d(&p->tmA, A, dt, es, (uint64_t)K, (uint64_t)M, (uint64_t)lda * es,
                              kstep, kGemmBM, CU_TENSOR_MAP_SWIZZLE_128B));
  WX_TRY(encode_tensor_map_2d(&p->tmB, B, dt, es, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * es,
                              kstep, pair ? 128u : (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B));
  GemmArgs& g = p->args;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.num_n_blocks = (int)((N + bn - 1) / bn);
  g.num_tiles = (int)((pair ? (M + 255) / 256 : mb) * g.num_n_blocks);
  g.num_k_blocks = (int)((K + kstep - 1) / kstep);
  g.C = C;
  g.ldc = ldc;
  g.bias = bias;
  g.R = R;
  g.ldr = ldr;
  g.err = err;
  g.pos = nullptr;
  g.ldp = 0;
  g.pos_T = 1;
  g.sa = sa;
  g.sw = sw;
  g.rowmax = rowmax;
  // In-place residual by TMA reduce-add (the same single rounding of
  // x + (acc + bias) as adding a loaded residual): int8 plans, and bf16 plans
  // with a long K. Measured on B200 at 64 clips: int8 fc2 2.6% faster, bf16
  // fc2 (K = 5120) 907 against 922 us, bf16 out-proj (K = 1280) 2.3% slower.
  g.resid_inplace =
      (epi == WX_EPI_F32_RESID && (i8 || K >= 4096) && pair && R == C && ldr == ldc) ? 1 : 0;
  p->bn = bn;
  p->epi = epi;
  p->pair = pair;
  p->i8 = i8;
  p->grid = pair ? 2 * std::min(g.num_tiles, nsm / 2) : std::min(g.num_tiles, nsm);
  WX_TRY(encode_epilogue_maps(p, C, R, M, N, ldc, ldr, epi));
  return gemm_prepare(bn, epi, pair, i8);
}

// Build the tensor maps and launch arguments once; the encoder keeps plans for
// its fixed buffers, the standalone entry point builds one per call.
int gemm_plan(GemmPlan* p, const void* A, const void* B, const float* bias, const float* R,
              void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
              int64_t ldr, int epi, int force_bn) {
  return gemm_plan_impl(p, A, B, bias, R, C, M, N, K, lda, ldb, ldc, ldr, epi, force_bn, false,
                        nullptr, nullptr, nullptr, nullptr);
}

int gemm_plan_i8(GemmPlan* p, const void* A, const void* B, const float* sa, const float* sw,
                 const float* bias, const float* R, void* C, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int epi, float* rowmax) {
  return gemm_plan_impl(p, A, B, bias, R, C, M, N, K, lda, ldb, ldc, ldr, epi, 0, true, sa, sw,
                        rowmax, nullptr);
}

// The same bf16 plan recording its kernels' wait timeouts into `err`, a word
// the caller owns (the allocation-free entry point's, in noalloc.cu), instead
// of the library's per-device word, whose first use on a device allocates it.
int gemm_plan_err(GemmPlan* p, const void* A, const void* B, const float* bias, void* C,
                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int epi,
                  int* err) {
  if (!err) return fail(WX_ERR_INVALID, "gemm: NULL error word");
  return gemm_plan_impl(p, A, B, bias, nullptr, C, M, N, K, lda, ldb, ldc, 0, epi, 0, false,
                        nullptr, nullptr, nullptr, err);
}

template <int BN, int EPI, bool I8>
static int set_attr_t() {
  static bool done[64] = {false};
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && done[dev]) return WX_OK;
  WX_CUDA_TRY(cudaFuncSetAttribute(gemm_bf16_kernel<BN, EPI, I8>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM));
  if (dev < 64) done[dev] = true;
  return WX_OK;
}

template <int EPI, bool I8>
static int set_attr_pair_t() {
  static bool done[64] = {false};
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && done[dev]) return WX_OK;
  WX_CUDA_TRY(cudaFuncSetAttribute(gemm2_bf16_kernel<EPI, I8>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Gemm2Cfg<EPI, I8>::SMEM));
  if (dev < 64) done[dev] = true;
  return WX_OK;
}

template <int EPI, bool I8>
static int prepare_t(int bn, bool pair) {
  return pair ? set_attr_pair_t<EPI, I8>() : bn == 256 ? set_attr_t<256, EPI, I8>()
                                                       : set_attr_t<128, EPI, I8>();
}

template <int BN, int EPI, bool I8>
static int launch_t(const GemmPlan& p, cudaStream_t st) {
  if (p.pair) {
    WX_CUDA_TRY(launch_k(gemm2_bf16_kernel<EPI, I8>, dim3(p.grid), dim3(Gemm2Cfg<EPI, I8>::THREADS),
                         Gemm2Cfg<EPI, I8>::SMEM, st, p.tmA, p.tmB, p.tmC, p.tmR, p.args));
    return check_launch(I8 ? "gemm_i8_pair" : "gemm_bf16_pair");
  }
  WX_CUDA_TRY(launch_k(gemm_bf16_kernel<BN, EPI, I8>, dim3(p.grid), dim3(kGemmThreads),
                       GemmCfg<BN>::SMEM, st, p.tmA, p.tmB, p.args));
  return check_launch(I8 ? "gemm_i8" : "gemm_bf16");
}

template <int EPI, bool I8>
static int run_t(const GemmPlan& p, cudaStream_t st) {
  return p.bn == 256 ? launch_t<256, EPI, I8>(p, st) : launch_t<128, EPI, I8>(p, st);
}

// Kernel attributes are set when a plan is made, so that a captured launch
// sequence contains nothing but launches.
static int gemm_prepare(int bn, int epi, bool pair, bool i8) {
#define WX_GEMM_PREP(E) \
  case E:               \
    return i8 ? prepare_t<E, true>(bn, pair) : prepare_t<E, false>(bn, pair);
  switch (epi) {
    WX_GEMM_PREP(WX_EPI_F32)
    WX_GEMM_PREP(WX_EPI_BF16)
    WX_GEMM_PREP(WX_EPI_F32_RESID)
    WX_GEMM_PREP(WX_EPI_BF16_GELU)
    WX_GEMM_PREP(WX_EPI_BF16_GELU_ERF)
    WX_GEMM_PREP(kEpiF32GeluPos)
    WX_GEMM_PREP(kEpiF32GeluErfPos)
    default:
      return fail(WX_ERR_INVALID, "gemm: epilogue %d", epi);
  }
#undef WX_GEMM_PREP
}

int gemm_run(const GemmPlan& p, cudaStream_t st) {
#define WX_GEMM_CASE(E) \
  case E:               \
    return p.i8 ? run_t<E, true>(p, st) : run_t<E, false>(p, st);
  switch (p.epi) {
    WX_GEMM_CASE(WX_EPI_F32)
    WX_GEMM_CASE(WX_EPI_BF16)
    WX_GEMM_CASE(WX_EPI_F32_RESID)
    WX_GEMM_CASE(WX_EPI_BF16_GELU)
    WX_GEMM_CASE(WX_EPI_BF16_GELU_ERF)
    WX_GEMM_CASE(kEpiF32GeluPos)
    WX_GEMM_CASE(kEpiF32GeluErfPos)
    default:
      return fail(WX_ERR_INVALID, "gemm: epilogue %d", p.epi);
  }
#undef WX_GEMM_CASE
}

void gemm_set_pos(GemmPlan* p, const float* pos, int64_t ldp, int pos_T) {
  p->args.pos = pos;
  p->args.ldp = ldp;
  p->args.pos_T = pos_T;
}

}  // namespace wx

extern "C" {

int wx_gemm_bf16(const void* A, const void* B, const float* bias, const float* R, void* C,
                 int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                 int64_t ldr, int epilogue, void* stream) {
  wx::GemmPlan p;
  WX_TRY(wx::gemm_plan(&p, A, B, bias, R, C, M, N, K, lda, ldb, ldc, ldr, epilogue, 0));
  return wx::gemm_run(p, wx::as_stream(stream));
}

}  // extern "C"
