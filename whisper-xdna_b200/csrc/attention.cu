// Fused multi-head attention on the sm_100a tensor cores (tcgen05), head dim
// 64, no mask: O = softmax(scale * Q K^T) V per (clip, head), the whole
// QK -> softmax -> AV chain of the reference in one kernel, with the scores
// never leaving the SM.
//
// One CTA per (pair of 128-query tiles A and B, head, clip); 18 warps:
//   warp 0     TMA: the two Q tiles once, then K and V tiles (128 keys x 64)
//              into two-slot rings with separate K and V barriers
//   warp 1     allocates tensor memory and issues, per key block j,
//              S_A = Q_A K_j^T, O_A += P_A V_j, S_B = Q_B K_j^T, O_B += P_B V_j
//              (M=128; S: N=128, K=64; PV: N=64, K=128 with V read MN-major
//              straight from its row-major tile), O accumulating in tensor
//              memory across blocks
//   warps 2-9  softmax of tile A, warps 10-17 of tile B. A query row is split
//              over two warps of one tensor-memory sub-partition (keys 0-63
//              and 64-127 of each block; O columns 0-31 and 32-63), which puts
//              four softmax warps on every SM sub-partition; the two halves
//              exchange their partial row maxima through shared memory at a
//              64-thread named barrier once per block and their row sums once
//              at the end. Each S half-row is loaded from tensor memory once
//              and the buffer released at once, so the next QK^T overlaps this
//              block's exponentials; P = exp2(s*c - m) goes to shared memory as
//              bf16 in the 128-byte-swizzled K-major layout the PV MMA reads.
// The two tiles' softmax warpgroups alternate with each other's MMAs.
//
// Online softmax with lazy rescaling: the running max m only moves when a
// block's row max exceeds it by more than 8 (in log2 units); then O (read and
// written back in tensor memory) and the row sum l are scaled by
// exp2(m_old - m_new). Otherwise P is taken against the stale max, which keeps
// every p <= 2^8 -- exact in the final O / l because O and l share the max.
// The recurrence is the one of the reference's fused head kernel
// (kernels/attn_fused.cc:13-17, src/attn_fused.py): m' = max(m, rowmax S),
// c = exp(m - m'), l' = c l + rowsum exp(S - m'), O' = c O + exp(S - m') V.
// Keys past T are masked exactly (p = 0); the reference's zero-padded keys
// took probability mass (src/rawxrt.py:618-623), which is not reproduced.
#include <type_traits>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

constexpr int kAttBQ = 128;                       // rows per Q tile (2 tiles per CTA)
constexpr int kAttBK = 128;                       // keys per block
constexpr int kAttHD = 64;
constexpr int kAttThreads = 576;   // 2 control warps + 16 softmax warps
constexpr int kTileBytes = 128 * kAttHD * 2;      // 16 KB: Q, K or V tile
constexpr int kPBytes = kAttBQ * kAttBK * 2;      // 32 KB: P tile
// Q_A, Q_B, K x2, V x2, P_A, P_B, barriers, the row-max exchange (2 tiles x 2
// parities x 2 halves x 128 rows of fp32)
constexpr int kAttSmem = 1024 + kTileBytes * 6 + kPBytes * 2 + 256 + 2 * 2 * 2 * 128 * 4;
constexpr int kAttTmemCols = 512;
constexpr int kSCol = 0;      // S_A at 0, S_B at 128
constexpr int kOCol = 256;    // O_A at 256, O_B at 320
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 18 warps: five share a sub-partition's 16K registers, so at most 96 each.
__global__ void __launch_bounds__(kAttThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // 2 tiles
  uint8_t* sK = smem + 2 * kTileBytes;         // 2 slots
  uint8_t* sV = smem + 4 * kTileBytes;         // 2 slots
  uint8_t* sP = smem + 6 * kTileBytes;         // 2 tiles of 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2] per slot
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per tile
  uint64_t* s_empty = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;   // [2]
  uint64_t* o_done = bars + 15;   // [2]
  uint64_t* done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  const int warp = warp_id(), lane = lane_id();
  const int h = blockIdx.y, b = blockIdx.z;
  const int T = a.T;
  const int q0 = blockIdx.x * 2 * kAttBQ;
  const int row0 = b * T;
  const int nkv = (T + kAttBK - 1) / kAttBK;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kAttTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      tma_load_2d(&tmQ, q_full, sQ, h * kAttHD, row0 + q0);
      tma_load_2d(&tmQ, q_full, sQ + kTileBytes, h * kAttHD, row0 + q0 + kAttBQ);
      uint32_t issued_k = 0, issued_v = 0;
      uint32_t last_k_phase = 0, last_v_phase = 0;
      bool ok = true;
      for (int j = 0; ok && j < nkv; j++) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_2d(&tmK, &k_full[s], sK + s * kTileBytes, h * kAttHD, row0 + j * kAttBK);
        issued_k |= 1u << s;
        last_k_phase = (last_k_phase & ~(1u << s)) | (ph << s);
        if (!mbar_wait(&v_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_2d(&tmV, &v_full[s], sV + s * kTileBytes, h * kAttHD, row0 + j * kAttBK);
        issued_v |= 1u << s;
        last_v_phase = (last_v_phase & ~(1u << s)) | (ph << s);
      }
      if (!ok) {  // drain copies in flight (1 ms at most each)
        mbar_wait_for(q_full, 0, 1000000ull);
        for (int s = 0; s < 2; s++) {
          if (issued_k & (1u << s)) mbar_wait_for(&k_full[s], (last_k_phase >> s) & 1u, 1000000ull);
          if (issued_v & (1u << s)) mbar_wait_for(&v_full[s], (last_v_phase >> s) & 1u, 1000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer. Order per block j: S_A(j+1), PV_A(j),
      // S_B(j+1), PV_B(j). The waits are blocking mbarrier try-waits, which
      // suspend the warp instead of taking issue slots from the softmax warps
      // that share its sub-partition (a polling scheduler measured slower).
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kAttBQ, kAttBK, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kAttBQ, kAttHD, 0, 1);
      bool ok = mbar_wait(q_full, 0, a.err);
      // S_t(j) = Q_t K_j^T; the K slot frees once tile B's product is done
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (t == 0 && !mbar_wait(&k_full[s], (j >> 1) & 1, a.err)) return false;
        if (j > 0 && !mbar_wait(&s_empty[t], (j - 1) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + t * kTileBytes);
        const uint32_t k_addr = smem_u32(sK + s * kTileBytes);
        const uint32_t d = tmem + kSCol + t * kAttBK;
#pragma unroll
        for (int kk = 0; kk < kAttHD / 16; kk++)
          umma_bf16_ss(d, sdesc_kmajor_sw128(q_addr + kk * 32),
                       sdesc_kmajor_sw128(k_addr + kk * 32), idesc_qk, kk != 0);
        umma_commit(&s_full[t]);
        if (t == 1) umma_commit(&k_empty[s]);
        return true;
      };
      // O_t += P_t V_j; the V slot frees once tile B's product is done
      auto issue_pv = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&p_full[t], j & 1, a.err)) return false;
        if (t == 0 && !mbar_wait(&v_full[s], (j >> 1) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + t * kPBytes);
        const uint32_t v_addr = smem_u32(sV + s * kTileBytes);
        const uint32_t d = tmem + kOCol + t * kAttHD;
#pragma unroll
        for (int kk = 0; kk < kAttBK / 16; kk++)
          umma_bf16_ss(d, sdesc_kmajor_sw128(p_addr + (kk >> 2) * (kPBytes / 2) + (kk & 3) * 32),
                       sdesc_mnmajor_sw128(v_addr + kk * 2048, kTileBytes), idesc_pv,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
        if (t == 1) umma_commit(&v_empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      for (int j = 0; ok && j < nkv; j++) {
        const bool more = j + 1 < nkv;
        if (more && !issue_s(0, j + 1)) { ok = false; break; }
        if (!issue_pv(0, j)) { ok = false; break; }
        if (more && !issue_s(1, j + 1)) { ok = false; break; }
        if (!issue_pv(1, j)) { ok = false; break; }
      }
      umma_commit(done);
      mbar_wait_for(done, 0, kWaitTimeoutNs);
    }
  } else {
    // ---------------- softmax: warps 2-9 tile A, 10-17 tile B. Each query row
    // is split over two warps of the same TMEM sub-partition: half 0 takes keys
    // 0-63 of every block and O columns 0-31, half 1 keys 64-127 and O 32-63.
    const int t = (warp - 2) >> 3;
    const int half = ((warp - 2) & 7) >> 2;
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t t_s = t_lane + kSCol + t * kAttBK + half * 64;
    const uint32_t t_o = t_lane + kOCol + t * kAttHD + half * 32;
    uint8_t* prow = sP + t * kPBytes + half * (kPBytes / 2) + r * 128;
    // partial row maxima of the two halves, double-buffered by block parity
    float* xchg = reinterpret_cast<float*>(bars + 20) + t * 2 * 2 * 128;  // [parity][half][row]
    const int bar_id = 1 + t * 4 + sub;  // named barrier of the warp pair
    const float c = a.scale_log2;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; j++) {
      const int kvalid = min(kAttBK, T - j * kAttBK) - half * 64;  // valid keys of this half
      // A failed wait never leaves the loop: the two halves of a row meet at
      // named barriers (which have no time limit) once per block, so both run
      // every iteration; once the error word is set the remaining waits return
      // at once.
      if (!mbar_wait(&s_full[t], j & 1, a.err)) ok = false;
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32(t_s + 0, s0);
      tmem_ld32(t_s + 32, s1);
      tmem_wait_ld();
      // S is in registers: the next QK^T may overwrite the buffer
      tc_fence_before();
      mbar_arrive(&s_empty[t]);
      auto chunk_max = [&](const uint32_t (&v)[32], int base) -> float {
        float mm[8];
        if (kvalid >= base + 32) {
#pragma unroll
          for (int i = 0; i < 8; i++)
            mm[i] = fmaxf(fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 8])),
                          fmaxf(__uint_as_float(v[i + 16]), __uint_as_float(v[i + 24])));
        } else {
#pragma unroll
          for (int i = 0; i < 8; i++) {
            mm[i] = -INFINITY;
#pragma unroll
            for (int k = 0; k < 4; k++)
              if (base + i + 8 * k < kvalid) mm[i] = fmaxf(mm[i], __uint_as_float(v[i + 8 * k]));
          }
        }
        return fmaxf(fmaxf(fmaxf(mm[0], mm[1]), fmaxf(mm[2], mm[3])),
                     fmaxf(fmaxf(mm[4], mm[5]), fmaxf(mm[6], mm[7])));
      };
      float mx = fmaxf(chunk_max(s0, 0), chunk_max(s1, 32));
      // combine with the other half of the row
      float* slot = xchg + (j & 1) * 256;
      slot[half * 128 + r] = mx;
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
      mx = fmaxf(mx, slot[(half ^ 1) * 128 + r]) * c;
      const bool grow = mx > m + kRescaleThreshold;  // includes the first block
      const float m_use = grow ? mx : m;
      const float corr = fast_exp2(m - m_use);        // 1 when m stays, 0 on block 0
      // P_t(j-1) V must have been consumed before P is rewritten (and before
      // O is rescaled)
      if (j > 0 && !mbar_wait(&o_done[t], (j - 1) & 1, a.err)) ok = false;
      m = m_use;
      float sums[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // independent accumulators
      const float negm = -m;
      // 32 keys = 4 chunks of 8 keys (16 bytes each) of the swizzled P row;
      // MASKED only for the last, partial key block
      auto chunk_p = [&](const uint32_t (&v)[32], int base, auto masked) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int i = q * 8 + 2 * e;
            float p0 = fast_exp2(fmaf(__uint_as_float(v[i]), c, negm));
            float p1 = fast_exp2(fmaf(__uint_as_float(v[i + 1]), c, negm));
            if (decltype(masked)::value) {
              p0 = (base + i < kvalid) ? p0 : 0.0f;
              p1 = (base + i + 1 < kvalid) ? p1 : 0.0f;
            }
            w[e] = pack_bf16x2_rne(p0, p1);
            sums[e] += p0 + p1;
          }
          const int chunk = base / 8 + q;  // 16-byte chunk within this half's 128-byte row
          uint8_t* dst = prow + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      };
      if (kvalid >= 64) {
        chunk_p(s0, 0, std::false_type());
        chunk_p(s1, 32, std::false_type());
      } else {
        chunk_p(s0, 0, std::true_type());
        chunk_p(s1, 32, std::true_type());
      }
      // O rescale after P is written, so the S registers are free; PV(j) reads
      // O only after p_full below
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        tc_fence_after();
        uint32_t ov[32];
        tmem_ld32(t_o, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
        tmem_st32(t_o, ov);
        tmem_wait_st();
      }
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&p_full[t]);
      l = l * corr + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
    }
    if (ok) ok = mbar_wait(&o_done[t], (nkv - 1) & 1, a.err);
    // the row sum is the sum of the two halves' sums
    float* lslot = xchg + (nkv & 1) * 256;
    lslot[half * 128 + r] = l;
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
    l += lslot[(half ^ 1) * 128 + r];
    if (ok) {
      tc_fence_after();
      uint32_t o0[32];
      tmem_ld32(t_o, o0);
      tmem_wait_ld();
      const int qrow = q0 + t * kAttBQ + r;
      if (qrow < T) {
        const float inv = 1.0f / l;
        uint16_t* dst = reinterpret_cast<uint16_t*>(a.O) + (int64_t)(row0 + qrow) * a.ldo +
                        h * kAttHD + half * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w0;
          w0.x = pack_bf16x2_rne(__uint_as_float(o0[i]) * inv, __uint_as_float(o0[i + 1]) * inv);
          w0.y = pack_bf16x2_rne(__uint_as_float(o0[i + 2]) * inv, __uint_as_float(o0[i + 3]) * inv);
          w0.z = pack_bf16x2_rne(__uint_as_float(o0[i + 4]) * inv, __uint_as_float(o0[i + 5]) * inv);
          w0.w = pack_bf16x2_rne(__uint_as_float(o0[i + 6]) * inv, __uint_as_float(o0[i + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + i) = w0;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttTmemCols);
  }
}

int attn_plan(AttnPlan* p, const void* q, const void* k, const void* v, void* o, int64_t B,
              int64_t H, int64_t T, int64_t hd, int64_t ldq, int64_t ldk, int64_t ldv,
              int64_t ldo, float scale) {
  if (hd != kAttHD) return fail(WX_ERR_UNSUPPORTED, "attention: head dim %lld (only 64)", (long long)hd);
  if (B <= 0 || H <= 0 || T <= 0) return fail(WX_ERR_INVALID, "attention: B, H, T must be > 0");
  if (B > 65535 || H > 65535) return fail(WX_ERR_UNSUPPORTED, "attention: B or H > 65535");
  if (B * T > INT32_MAX) return fail(WX_ERR_UNSUPPORTED, "attention: B*T exceeds 2^31");
  if (!q || !k || !v || !o) return fail(WX_ERR_INVALID, "attention: NULL pointer");
  const int64_t need = H * hd;
  if (ldq < need || ldk < need || ldv < need || ldo < need)
    return fail(WX_ERR_INVALID, "attention: row stride < H*hd");
  if (ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(o) & 15))
    return fail(WX_ERR_INVALID, "attention: strides must be multiples of 8, O 16-byte aligned");
  if (!(scale > 0.0f)) return fail(WX_ERR_INVALID, "attention: scale must be > 0");
  int* err = device_error_word();
  if (!err) return fail(WX_ERR_CUDA, "attention: device error word unavailable");
  const uint64_t rows = (uint64_t)(B * T);
  // Columns beyond H*hd are outside the map: a box never reaches them. Rows
  // past B*T read as zeros.
  WX_TRY(encode_tensor_map_2d(&p->tmQ, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldq * 2, kAttHD, kAttBQ, CU_TENSOR_MAP_SWIZZLE_128B));
  WX_TRY(encode_tensor_map_2d(&p->tmK, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldk * 2, kAttHD, kAttBK, CU_TENSOR_MAP_SWIZZLE_128B));
  WX_TRY(encode_tensor_map_2d(&p->tmV, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldv * 2, kAttHD, kAttBK, CU_TENSOR_MAP_SWIZZLE_128B));
  AttnArgs& g = p->args;
  g.T = (int)T;
  g.H = (int)H;
  g.num_q_tiles = (int)((T + 2 * kAttBQ - 1) / (2 * kAttBQ));  // tile pairs
  g.O = o;
  g.ldo = ldo;
  g.scale_log2 = scale * 1.4426950408889634f;
  g.err = err;
  p->B = (int)B;
  // set when the plan is made, so a captured launch sequence holds only launches
  static bool attr_set[64] = {false};
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !attr_set[dev]) {
    WX_CUDA_TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kAttSmem));
    if (dev < 64) attr_set[dev] = true;
  }
  return WX_OK;
}

int attn_run(const AttnPlan& p, cudaStream_t st) {
  dim3 grid(p.args.num_q_tiles, p.args.H, p.B);
  attention_kernel<<<grid, kAttThreads, kAttSmem, st>>>(p.tmQ, p.tmK, p.tmV, p.args);
  return check_launch("attention");
}

}  // namespace wx

extern "C" {

int wx_attention(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
                 int64_t T, int64_t hd, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo,
                 float scale, void* stream) {
  wx::AttnPlan p;
  WX_TRY(wx::attn_plan(&p, q, k, v, o, B, H, T, hd, ldq, ldk, ldv, ldo, scale));
  return wx::attn_run(p, wx::as_stream(stream));
}

}  // extern "C"
