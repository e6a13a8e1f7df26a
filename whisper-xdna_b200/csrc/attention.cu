// Fused multi-head attention on the sm_100a tensor cores (tcgen05), head dim
// 64, no mask: O = softmax(scale * Q K^T) V per (clip, head), the whole
// QK -> softmax -> AV chain of the reference in one kernel, with the scores
// never leaving the SM.
//
// One CTA per (128-query tile, head, clip); 6 warps:
//   warp 0     TMA: the Q tile once, then K and V tiles (128 keys x 64) into
//              two-slot rings (separate K and V barriers, so a K slot frees as
//              soon as its QK^T is done)
//   warp 1     allocates tensor memory, issues S = Q K^T (M=128, N=128, K=64)
//              into one of two S buffers and O_j = P_j V_j (M=128, N=64, K=128,
//              V read MN-major straight from its row-major tile) into one of
//              two O buffers
//   warps 2-5  online softmax, one query row per thread: tcgen05.ld of the S
//              row, running max in the exp2 domain, P = exp2(s*c - m) written
//              as bf16 into shared memory in the 128-byte-swizzled K-major
//              layout the PV MMA reads, and the fp32 output row kept in
//              registers: O = O * exp2(m_old - m_new) + P_j V_j, divided by the
//              row sum at the end.
// The recurrence is the one of the reference's fused head kernel
// (kernels/attn_fused.cc:13-17, src/attn_fused.py): m' = max(m, rowmax S),
// c = exp(m - m'), l' = c l + rowsum exp(S - m'), O' = c O + exp(S - m') V.
// Keys past T are masked exactly (p = 0); the reference's zero-padded keys
// took probability mass (src/rawxrt.py:618-623), which is not reproduced.
#include "common.cuh"
#include "plans.cuh"

namespace wx {

constexpr int kAttBQ = 128;
constexpr int kAttBK = 128;
constexpr int kAttHD = 64;
constexpr int kTileBytes = 128 * kAttHD * 2;     // 16 KB: Q, K or V tile
constexpr int kPBytes = kAttBQ * kAttBK * 2;     // 32 KB: P tile
constexpr int kAttSmem = 1024 + kTileBytes * 5 + kPBytes * 2 + 512;
constexpr int kAttTmemCols = 512;                // S: 2 x 128, O: 2 x 64
constexpr int kSCol = 0;
constexpr int kOCol = 256;

__global__ void __launch_bounds__(192, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;            // 2 slots
  uint8_t* sV = smem + 3 * kTileBytes;        // 2 slots
  uint8_t* sP = smem + 5 * kTileBytes;        // 2 slots of 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;  // [2]
  uint64_t* p_empty = bars + 15; // [2]
  uint64_t* o_full = bars + 17;  // [2]
  uint64_t* o_empty = bars + 19; // [2]
  uint64_t* done = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);

  const int warp = warp_id(), lane = lane_id();
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = a.T;
  const int q0 = qt * kAttBQ;
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
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
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
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(&tmQ, q_full, sQ, h * kAttHD, row0 + q0);
      uint32_t issued_k = 0, issued_v = 0;
      int last_k_phase[2] = {0, 0}, last_v_phase[2] = {0, 0};
      bool ok = true;
      for (int j = 0; ok && j < nkv; j++) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_2d(&tmK, &k_full[s], sK + s * kTileBytes, h * kAttHD, row0 + j * kAttBK);
        issued_k |= 1u << s;
        last_k_phase[s] = ph;
        if (!mbar_wait(&v_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_2d(&tmV, &v_full[s], sV + s * kTileBytes, h * kAttHD, row0 + j * kAttBK);
        issued_v |= 1u << s;
        last_v_phase[s] = ph;
      }
      if (!ok) {  // drain copies in flight (1 ms at most each)
        mbar_wait_for(q_full, 0, 1000000ull);
        for (int s = 0; s < 2; s++) {
          if (issued_k & (1u << s)) mbar_wait_for(&k_full[s], last_k_phase[s], 1000000ull);
          if (issued_v & (1u << s)) mbar_wait_for(&v_full[s], last_v_phase[s], 1000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kAttBQ, kAttBK, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kAttBQ, kAttHD, 0, 1);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[s], ph, a.err)) return false;
        if (!mbar_wait(&s_empty[s], ph ^ 1, a.err)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * kTileBytes);
        const uint32_t d = tmem + kSCol + s * kAttBK;
#pragma unroll
        for (int kk = 0; kk < kAttHD / 16; kk++)
          umma_bf16_ss(d, sdesc_kmajor_sw128(q_addr + kk * 32),
                       sdesc_kmajor_sw128(k_addr + kk * 32), idesc_qk, kk != 0);
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; j++) {
        if (j + 1 < nkv && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&p_full[s], ph, a.err)) { ok = false; break; }
        if (!mbar_wait(&v_full[s], ph, a.err)) { ok = false; break; }
        if (!mbar_wait(&o_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + s * kPBytes);
        const uint32_t v_addr = smem_u32(sV + s * kTileBytes);
        const uint32_t d = tmem + kOCol + s * kAttHD;
#pragma unroll
        for (int kk = 0; kk < kAttBK / 16; kk++)
          umma_bf16_ss(d, sdesc_kmajor_sw128(p_addr + (kk >> 2) * (kPBytes / 2) + (kk & 3) * 32),
                       sdesc_mnmajor_sw128(v_addr + kk * 2048, kTileBytes), idesc_pv, kk != 0);
        umma_commit(&o_full[s]);
        umma_commit(&v_empty[s]);
        umma_commit(&p_empty[s]);
      }
      umma_commit(done);
      mbar_wait_for(done, 0, kWaitTimeoutNs);
    }
  } else {
    // ---------------- softmax: warps 2..5, thread <-> query row
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(sub * 32) << 16);
    const float c = a.scale_log2;
    float m = -INFINITY, l = 0.0f, corr_prev = 0.0f;
    float o[kAttHD];
#pragma unroll
    for (int i = 0; i < kAttHD; i++) o[i] = 0.0f;
    bool ok = true;
    auto fold = [&](int j, float corr) -> bool {  // O = O * corr + P_j V_j
      const int s = j & 1;
      if (!mbar_wait(&o_full[s], (j >> 1) & 1, a.err)) return false;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld32(t_lane + kOCol + s * kAttHD, v0);
      tmem_ld32(t_lane + kOCol + s * kAttHD + 32, v1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&o_empty[s]);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        o[i] = fmaf(o[i], corr, __uint_as_float(v0[i]));
        o[32 + i] = fmaf(o[32 + i], corr, __uint_as_float(v1[i]));
      }
      return true;
    };
    for (int j = 0; j < nkv; j++) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      const int kvalid = min(kAttBK, T - j * kAttBK);
      if (!mbar_wait(&s_full[s], ph, a.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t t_s = t_lane + kSCol + s * kAttBK;
      // pass A: row max of the valid keys
      float mx = -INFINITY;
#pragma unroll 1
      for (int ch = 0; ch < kAttBK / 32; ch++) {
        uint32_t v[32];
        tmem_ld32(t_s + ch * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (ch * 32 + i < kvalid) mx = fmaxf(mx, __uint_as_float(v[i]));
      }
      const float m_new = fmaxf(m, mx * c);
      const float corr = fast_exp2(m - m_new);
      // P must not be overwritten while the PV MMA of two blocks ago reads it
      if (!mbar_wait(&p_empty[s], ph ^ 1, a.err)) { ok = false; break; }
      uint8_t* prow = sP + s * kPBytes + r * 128;
      float sum = 0.0f;
#pragma unroll 1
      for (int ch = 0; ch < kAttBK / 32; ch++) {
        uint32_t v[32];
        tmem_ld32(t_s + ch * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const bool in0 = ch * 32 + i < kvalid, in1 = ch * 32 + i + 1 < kvalid;
          const float p0 = in0 ? fast_exp2(fmaf(__uint_as_float(v[i]), c, -m_new)) : 0.0f;
          const float p1 = in1 ? fast_exp2(fmaf(__uint_as_float(v[i + 1]), c, -m_new)) : 0.0f;
          const uint32_t w = pack_bf16x2_rne(p0, p1);
          pk[i >> 1] = w;
          // the row sum takes the bf16 values the PV product uses
          sum += __uint_as_float(w << 16) + __uint_as_float(w & 0xFFFF0000u);
        }
        // 32 keys = 4 chunks of 16 bytes; key block half = ch / 2
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int chunk = (ch & 1) * 4 + q;                  // 16-byte chunk in the row
          uint8_t* dst = prow + (ch >> 1) * (kPBytes / 2) + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      // S buffer fully read; P visible to the tensor core
      tc_fence_before();
      mbar_arrive(&s_empty[s]);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[s]);
      l = l * corr + sum;
      if (j >= 1 && !fold(j - 1, corr_prev)) { ok = false; break; }
      corr_prev = corr;
      m = m_new;
    }
    if (ok) ok = fold(nkv - 1, corr_prev);
    if (ok && q0 + r < T) {
      const float inv = 1.0f / l;
      uint16_t* dst = reinterpret_cast<uint16_t*>(a.O) + (int64_t)(row0 + q0 + r) * a.ldo +
                      h * kAttHD;
#pragma unroll
      for (int i = 0; i < kAttHD; i += 8) {
        uint4 w;
        w.x = pack_bf16x2_rne(o[i] * inv, o[i + 1] * inv);
        w.y = pack_bf16x2_rne(o[i + 2] * inv, o[i + 3] * inv);
        w.z = pack_bf16x2_rne(o[i + 4] * inv, o[i + 5] * inv);
        w.w = pack_bf16x2_rne(o[i + 6] * inv, o[i + 7] * inv);
        *reinterpret_cast<uint4*>(dst + i) = w;
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
  // Columns beyond H*hd are outside the map: a box never reaches them.
  WX_TRY(encode_tensor_map_2d(&p->tmQ, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldq * 2, kAttHD, kAttBQ, CU_TENSOR_MAP_SWIZZLE_128B));
  WX_TRY(encode_tensor_map_2d(&p->tmK, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldk * 2, kAttHD, kAttBK, CU_TENSOR_MAP_SWIZZLE_128B));
  WX_TRY(encode_tensor_map_2d(&p->tmV, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)need,
                              rows, (uint64_t)ldv * 2, kAttHD, kAttBK, CU_TENSOR_MAP_SWIZZLE_128B));
  AttnArgs& g = p->args;
  g.T = (int)T;
  g.H = (int)H;
  g.num_q_tiles = (int)((T + kAttBQ - 1) / kAttBQ);
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
  attention_kernel<<<grid, 192, kAttSmem, st>>>(p.tmQ, p.tmK, p.tmV, p.args);
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
