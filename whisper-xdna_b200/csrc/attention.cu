// Fused multi-head attention on the sm_100a tensor cores (tcgen05), head dim
// 64, no mask: O = softmax(scale * Q K^T) V per (clip, head), the whole
// QK -> softmax -> AV chain of the reference in one kernel, with the scores
// and probabilities never leaving the SM.
//
// A work item is (pair of 128-query tiles A and B, head, clip). Two kernels:
//   attention_kernel             one CTA per item (the hardware hands items to
//                                SMs as they free up);
//   attention_persistent_kernel  one CTA per SM walking the items c, c + grid,
//                                ...; every role runs straight on from one item
//                                to the next -- the TMA warp loads the next
//                                item's Q into the other of two Q buffers, the
//                                issuers compute its first two S blocks while
//                                the softmax warps finish the current one -- so
//                                a CTA's start-up, its first loads and the
//                                pipeline ramp (about 4 us, measured) are paid
//                                once per SM instead of once per item.
// The persistent kernel keeps a few more registers live in the softmax key
// loop (at the 96-register cap of 19 warps some spill), which costs a little
// per key block, so it runs only short items, where the fixed cost dominates
// (kAttPersistMaxBlocks; measured at 64 clips x 20 heads: T 512 +15%, 768
// +10%, 1024 +3.5%, 1152 +2%, 1280 +1.5%, 1344 even; at 1500 the per-item
// kernel is 1% faster).
// Both compute the same arithmetic in the same order: outputs are identical.
// They are two functions rather than one template on purpose: a template whose
// per-item instance folds the item loops away compiled spill-free but ran 5-6%
// slower than this per-item source at T >= 1280 (the kernel sits at the
// register cap, where small code changes move its schedule), so the per-item
// kernel keeps its own code. 19 warps in both:
//   warp 0     TMA: the two Q tiles of an item, then K and V tiles (96 keys
//              x 64) into three-slot rings with separate K and V barriers
//   warps 1-2  MMA issuers, one per query tile (warp 1 also allocates tensor
//              memory): per key block j, O_t += P_t(j) V_j, then S_t(j+2) =
//              Q_t K_{j+2}^T, which in the persistent kernel may be the next
//              item's (M=128; S: N=96, K=64; PV: N=64, K=96 with P read
//              from tensor memory and V MN-major straight from its row-major
//              tile). One issuer per tile lets the two tiles' S -> softmax ->
//              PV round trips overlap instead of queueing in one program order.
//   warps 3-10 softmax of tile A, warps 11-18 of tile B. A query row is split
//              over two warps of one tensor-memory sub-partition (keys 0-47
//              and 48-95 of each block; O columns 0-31 and 32-63), which puts
//              four softmax warps on every SM sub-partition; the two halves
//              exchange their partial row maxima through shared memory at a
//              64-thread named barrier once per block and their row sums once
//              at the end. Three exponential pairs in four run on the SFU and
//              one on the FMA pipe (exp2_poly2), and the two tiles' warps
//              share each sub-partition freely. (Making the tiles take turns
//              on the SFU paid while every exponential was an SFU one; with a
//              quarter on the FMA pipe it costs 5%.)
//
// Tensor memory (512 columns): S_A double-buffered at columns 0 and 96, S_B at
// 192 and 288, O_A at 384, O_B at 448. P = exp2(s*c - m) is written back as
// packed bf16 pairs over the S buffer it came from (keys 0-47 at columns
// 0-23, keys 48-95 at 64-87: each half overwrites only columns it has already
// read), and the PV MMA takes its A operand from there. The tensor core runs
// one thread's MMAs in issue order, so S_t(j+2), issued by tile t's issuer
// after PV_t(j), overwrites the buffer only after PV_t(j) has read P_t(j): the
// softmax warps never wait for a PV except to rescale O (and, persistent, at
// the end of an item), and S(j+1) is being computed while they work on S(j).
// In the persistent kernel the first PV of an item overwrites O (no
// accumulate); it waits for that block's P, which the softmax warps publish
// only after they have read the previous item's O out.
//
// Online softmax with lazy rescaling: the running max m only moves when a
// block's row max exceeds it by more than 8 (in log2 units); then O (read and
// written back in tensor memory, after PV(j-1) has landed) and the row sum l
// are scaled by exp2(m_old - m_new). Otherwise P is taken against the stale
// max, which keeps every p <= 2^8 -- exact in the final O / l because O and l
// share the max. The recurrence is the one of the reference's fused head
// kernel (kernels/attn_fused.cc:13-17, src/attn_fused.py): m' = max(m, rowmax
// S), c = exp(m - m'), l' = c l + rowsum exp(S - m'), O' = c O + exp(S - m') V.
// Keys past T are masked exactly (p = 0); the reference's zero-padded keys
// took probability mass (src/rawxrt.py:618-623), which is not reproduced.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "plans.cuh"

namespace wx {

// 2^x of a pair on the FMA pipe: x = n + f with n = round(x), |f| <= 1/2;
// 2^f by a degree-3 polynomial fitted here for minimum maximum relative error
// on [-1/2, 1/2] (7.5e-5, against the 2^-9 of the bf16 P it feeds), 2^n added
// to the exponent field. One pair in four of the softmax takes this path so
// that the SFU, which bounds the exponentials, carries three quarters of them.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.0f, 12582912.0f));
  const float2 j = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(0.0551716573536396f, 0.0551716573536396f), f,
                        make_float2(0.2426111400127411f, 0.2426111400127411f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  return make_float2(__int_as_float(__float_as_int(t.x) * 8388608 + __float_as_int(p.x)),
                     __int_as_float(__float_as_int(t.y) * 8388608 + __float_as_int(p.y)));
}

constexpr int kAttBQ = 128;                       // rows per Q tile (2 tiles per CTA)
constexpr int kAttBK = 96;                        // keys per block
constexpr int kAttHD = 64;
constexpr int kAttHalf = kAttBK / 2;              // keys per half-row warp
constexpr int kAttThreads = 608;                  // 3 control warps + 16 softmax warps
constexpr int kAttStages = 3;                     // K and V ring slots
constexpr int kQBytes = kAttBQ * kAttHD * 2;      // 16 KB Q tile
constexpr int kKVBytes = kAttBK * kAttHD * 2;     // 12 KB K or V tile
// Q_A, Q_B, the K and V rings, barriers, the row-max exchange (2 tiles x 2
// parities x 2 halves x 128 rows of fp32)
constexpr int kAttBarBytes = 512;                // up to 30 mbarriers and the TMEM address
constexpr int kAttSmem = 1024 + 2 * kQBytes + 2 * kAttStages * kKVBytes + kAttBarBytes +
                         2 * 2 * 2 * 128 * 4;
// the persistent kernel: a second Q buffer
constexpr int kAttSmemPersist = kAttSmem + 2 * kQBytes;
// the persistent kernel for items of at most this many key blocks (T <= 1344)
constexpr int kAttPersistMaxBlocks = 14;
constexpr int kAttTmemCols = 512;
constexpr int kSBufCols = kAttBK;                 // one S buffer: 96 fp32 columns
constexpr int kOCol = 4 * kSBufCols;              // O_A at 384, O_B at 448
// P of half 0 (keys 0-47) at column 0 of its S buffer, of half 1 at column 64
__host__ __device__ constexpr int p_col(int half) { return half ? 64 : 0; }
constexpr float kRescaleThreshold = 8.0f;         // log2 units
// Tile B's issuer starts its first S this many SM cycles after tile A's. The
// two tiles' softmax warps share each sub-partition's SFU; started together
// they run their exponentials (SFU-bound) and their max / load phases (SFU
// idle) in step. Measured at 64 clips x 20 heads x 1500 frames: 1128 us
// without an offset, 1091-1095 us at 700-1,000 cycles, 1107 us at 400,
// 1140-1154 us at 1,300-1,600.
constexpr long long kTileBOffsetCycles = 800;
static_assert(kOCol + 2 * kAttHD <= kAttTmemCols, "tensor memory budget");
static_assert((1 + 4 * kAttStages + 4 + 4 + 4 + 2) * 8 + 4 <= kAttBarBytes, "barrier area");
static_assert((2 + 2 + 4 * kAttStages + 4 + 4 + 4 + 2) * 8 + 4 <= kAttBarBytes,
              "barrier area (persistent)");
static_assert(kAttSmemPersist <= 227 * 1024, "shared memory per CTA");
static_assert(2 * kQBytes % 1024 == 0 && kKVBytes % 1024 == 0, "SW128 tiles 1024-aligned");

// a busy wait of n SM cycles (one thread; the clock only moves forward)
__device__ __forceinline__ void spin_cycles(long long n) {
  const long long t0 = clock64();
  while (clock64() - t0 < n) {
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  static_assert(N == 16, "x16 only");
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
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
// D[tmem] (+)= A[tmem] * B[smem]: A is M rows (lanes) x K bf16 packed in pairs
// along the columns; B's descriptor as its low word with high word `hi`.
__device__ __forceinline__ void umma_bf16_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                                uint32_t hi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 bd;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 bd, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(hi)
      : "memory");
}

// 19 warps: up to five share a sub-partition's 16K registers, so at most 96 each.
__global__ void __launch_bounds__(kAttThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 tiles
  uint8_t* sK = smem + 2 * kQBytes;                    // kAttStages slots
  uint8_t* sV = sK + kAttStages * kKVBytes;            // kAttStages slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kAttStages * kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                         // [kAttStages]
  uint64_t* k_empty = k_full + kAttStages;             // [kAttStages]
  uint64_t* v_full = k_empty + kAttStages;             // [kAttStages]
  uint64_t* v_empty = v_full + kAttStages;             // [kAttStages]
  // Every barrier below is waited on by parity, which tells apart only the
  // current phase and the one before: S(j+2) is issued after PV(j), so no
  // barrier gets two phases ahead of its waiter (the softmax warps of a tile
  // may finish block j+1 before PV(j) is issued, hence p_full per block parity)
  uint64_t* s_full = v_empty + kAttStages;             // [tile][buffer]
  uint64_t* p_full = s_full + 4;                       // [tile][block parity]
  uint64_t* o_done = p_full + 4;                       // [tile][PV parity]
  uint64_t* done = o_done + 4;                         // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
  float* xchg_base = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kAttBarBytes);

  const int warp = warp_id(), lane = lane_id();
  const int h = blockIdx.y, b = blockIdx.z;
  const int T = a.T;
  const int q0 = blockIdx.x * 2 * kAttBQ;
  const int row0 = b * T;
  const int nkv = (T + kAttBK - 1) / kAttBK;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kAttStages; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 2);   // released by both tiles' issuers
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 2);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
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
  pdl_launch_dependents();
  pdl_wait();   // Q, K and V come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(q_full, 2 * kQBytes);
      tma_load_2d(&tmQ, q_full, sQ, h * kAttHD, row0 + q0);
      tma_load_2d(&tmQ, q_full, sQ + kQBytes, h * kAttHD, row0 + q0 + kAttBQ);
      uint32_t issued_k = 0, issued_v = 0, last_k_phase = 0, last_v_phase = 0;
      bool ok = true;
      for (int j = 0; ok && j < nkv; j++) {
        const int s = j % kAttStages;
        const uint32_t ph = (uint32_t)(j / kAttStages) & 1u;
        if (!mbar_wait(&k_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        tma_load_2d(&tmK, &k_full[s], sK + s * kKVBytes, h * kAttHD, row0 + j * kAttBK);
        issued_k |= 1u << s;
        last_k_phase = (last_k_phase & ~(1u << s)) | (ph << s);
        if (!mbar_wait(&v_empty[s], ph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        tma_load_2d(&tmV, &v_full[s], sV + s * kKVBytes, h * kAttHD, row0 + j * kAttBK);
        issued_v |= 1u << s;
        last_v_phase = (last_v_phase & ~(1u << s)) | (ph << s);
      }
      if (!ok) {  // drain copies in flight (1 ms at most each)
        mbar_wait_for(q_full, 0, 1000000ull);
        for (int s = 0; s < kAttStages; s++) {
          if (issued_k & (1u << s)) mbar_wait_for(&k_full[s], (last_k_phase >> s) & 1u, 1000000ull);
          if (issued_v & (1u << s)) mbar_wait_for(&v_full[s], (last_v_phase >> s) & 1u, 1000000ull);
        }
      }
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      // ---------------- MMA issuers: warp 1 for tile A, warp 2 for tile B, so
      // each tile's S -> softmax -> PV round trip runs on its own and the two
      // overlap. The tensor core runs one thread's MMAs in issue order.
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kAttBQ, kAttBK, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kAttBQ, kAttHD, 0, 1);
      // The ring slot and S buffer are fixed at compile time (the block loop is
      // unrolled by six = three slots x two buffers), so each operand is one
      // constant offset from these bases and each group of MMAs is one asm
      // statement with a single pair of predicates.
      const uint64_t q_desc = sdesc_kmajor_sw128(smem_u32(sQ));
      const uint64_t k_desc = sdesc_kmajor_sw128(smem_u32(sK));
      const uint64_t v_desc = sdesc_mnmajor_sw128(smem_u32(sV), kKVBytes);
      // S_t(j) = Q_t K_j^T into buffer B from ring slot SL (K = 64: four MMAs,
      // 32 bytes of K apart)
      auto mma_s = [&](auto t_c, auto b_c, auto sl_c) {
        constexpr int t = decltype(t_c)::value, b = decltype(b_c)::value,
                      sl = decltype(sl_c)::value;
        const uint32_t d = tmem + (uint32_t)((2 * t + b) * kSBufCols);
        const uint64_t qa = q_desc + (uint64_t)(t * (kQBytes >> 4));
        const uint64_t kb = k_desc + (uint64_t)(sl * (kKVBytes >> 4));
        asm volatile(
            "{\n\t.reg .pred pf, pt;\n\t"
            "setp.ne.b32 pf, %1, %1;\n\t"
            "setp.eq.b32 pt, %1, %1;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %3, %1, pf;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %5, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %7, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %9, %1, pt;\n\t}\n" ::"r"(d),
            "r"(idesc_qk), "l"(qa), "l"(kb), "l"(qa + 2), "l"(kb + 2), "l"(qa + 4), "l"(kb + 4),
            "l"(qa + 6), "l"(kb + 6)
            : "memory");
      };
      // O_t += P_t V from buffer B and ring slot SL: six MMAs of 16 keys, P
      // read from tensor memory (keys 0-47 at columns 0-23, 48-95 at 64-87),
      // V MN-major 2048 bytes (16 rows) apart; acc = 0 only for the first block
      auto mma_pv = [&](auto t_c, auto b_c, auto sl_c, uint32_t acc) {
        constexpr int t = decltype(t_c)::value, b = decltype(b_c)::value,
                      sl = decltype(sl_c)::value;
        const uint32_t d = tmem + (uint32_t)(kOCol + t * kAttHD);
        const uint32_t pa = tmem + (uint32_t)((2 * t + b) * kSBufCols);
        const uint64_t vb = v_desc + (uint64_t)(sl * (kKVBytes >> 4));
        asm volatile(
            "{\n\t.reg .pred p0, pt;\n\t"
            "setp.ne.b32 p0, %2, 0;\n\t"
            "setp.eq.b32 pt, %1, %1;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %9, %1, p0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %10, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %11, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %12, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %13, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %14, %1, pt;\n\t}\n" ::"r"(d),
            "r"(idesc_pv), "r"(acc), "r"(pa + p_col(0)), "r"(pa + p_col(0) + 8),
            "r"(pa + p_col(0) + 16), "r"(pa + p_col(1)), "r"(pa + p_col(1) + 8),
            "r"(pa + p_col(1) + 16), "l"(vb), "l"(vb + 128), "l"(vb + 256), "l"(vb + 384),
            "l"(vb + 512), "l"(vb + 640)
            : "memory");
      };
      auto run = [&](auto t_c) {
        constexpr int t = decltype(t_c)::value;
        bool ok = mbar_wait(q_full, 0, a.err);
        // S of block j (j % 6 == M) into buffer M % 2 from slot M % 3; the K
        // slot frees once both tiles' products are done (count 2)
        auto issue_s = [&](int j, auto mc) -> bool {
          constexpr int m = decltype(mc)::value;
          if (!mbar_wait(&k_full[m % 3], (uint32_t)(j / kAttStages) & 1u, a.err)) return false;
          tc_fence_after();
          mma_s(t_c, std::integral_constant<int, m % 2>(), std::integral_constant<int, m % 3>());
          umma_commit(&s_full[2 * t + m % 2]);
          umma_commit(&k_empty[m % 3]);
          return true;
        };
        // Block j: PV_t(j), then S_t(j + 2) into the buffer PV_t(j) has read P from
        auto step = [&](int j, auto mc) -> bool {
          constexpr int m = decltype(mc)::value;
          if (!mbar_wait(&p_full[2 * t + m % 2], (uint32_t)(j >> 1) & 1u, a.err)) return false;
          if (!mbar_wait(&v_full[m % 3], (uint32_t)(j / kAttStages) & 1u, a.err)) return false;
          tc_fence_after();
          mma_pv(t_c, std::integral_constant<int, m % 2>(), std::integral_constant<int, m % 3>(),
                 j > 0 ? 1u : 0u);
          umma_commit(&o_done[2 * t + m % 2]);
          umma_commit(&v_empty[m % 3]);
          if (j + 2 < nkv) return issue_s(j + 2, std::integral_constant<int, (m + 2) % 6>());
          return true;
        };
        if (t == 1) spin_cycles(kTileBOffsetCycles);
        if (ok) ok = issue_s(0, std::integral_constant<int, 0>());
        if (ok && nkv > 1) ok = issue_s(1, std::integral_constant<int, 1>());
        for (int j = 0; ok && j < nkv; j += 6) {
          ok = step(j, std::integral_constant<int, 0>());
          if (ok && j + 1 < nkv) ok = step(j + 1, std::integral_constant<int, 1>());
          if (ok && j + 2 < nkv) ok = step(j + 2, std::integral_constant<int, 2>());
          if (ok && j + 3 < nkv) ok = step(j + 3, std::integral_constant<int, 3>());
          if (ok && j + 4 < nkv) ok = step(j + 4, std::integral_constant<int, 4>());
          if (ok && j + 5 < nkv) ok = step(j + 5, std::integral_constant<int, 5>());
        }
        // every MMA of this issuer has completed before tensor memory is released
        umma_commit(&done[t]);
        mbar_wait_for(&done[t], 0, kWaitTimeoutNs);
      };
      if (warp == 1) run(std::integral_constant<int, 0>());
      else run(std::integral_constant<int, 1>());
    }
  } else {
    // ---------------- softmax: warps 2-9 tile A, 10-17 tile B. Each query row
    // is split over two warps of the same TMEM sub-partition: half 0 takes keys
    // 0-47 of every block and O columns 0-31, half 1 keys 48-95 and O 32-63.
    const int t = (warp - 3) >> 3;
    const int half = ((warp - 3) & 7) >> 2;
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t t_o = t_lane + (uint32_t)(kOCol + t * kAttHD + half * 32);
    // partial row maxima of the two halves, double-buffered by block parity
    float* xchg = xchg_base + t * 2 * 2 * 128;  // [parity][half][row]
    const int bar_id = 1 + t * 4 + sub;          // named barrier of the warp pair
    const float c = a.scale_log2;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; j++) {
      const int kvalid = min(kAttBK, T - j * kAttBK) - half * kAttHalf;  // valid keys of this half
      const uint32_t t_buf = t_lane + (uint32_t)((2 * t + (j & 1)) * kSBufCols);
      // A failed wait never leaves the loop: the two halves of a row meet at
      // named barriers (which have no time limit) once per block, so both run
      // every iteration; once the error word is set the remaining waits return
      // at once.
      if (!mbar_wait(&s_full[2 * t + (j & 1)], (uint32_t)(j >> 1) & 1u, a.err)) ok = false;
      tc_fence_after();
      uint32_t s[kAttHalf];
      tmem_ld16<16>(t_buf + half * kAttHalf, s);
      tmem_ld16<16>(t_buf + half * kAttHalf + 16, s + 16);
      tmem_ld16<16>(t_buf + half * kAttHalf + 32, s + 32);
      tmem_wait_ld();
      float mx;
      if (kvalid >= kAttHalf) {
        float mm[8];   // three-input max: 24 instructions for 48 values
#pragma unroll
        for (int i = 0; i < 8; i++)
          mm[i] = fmax3(fmax3(__uint_as_float(s[i]), __uint_as_float(s[i + 8]),
                              __uint_as_float(s[i + 16])),
                        __uint_as_float(s[i + 24]),
                        fmaxf(__uint_as_float(s[i + 32]), __uint_as_float(s[i + 40])));
        mx = fmax3(fmax3(mm[0], mm[1], mm[2]), fmax3(mm[3], mm[4], mm[5]), fmaxf(mm[6], mm[7]));
      } else {
        mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < kAttHalf; i++)
          if (i < kvalid) mx = fmaxf(mx, __uint_as_float(s[i]));
      }
      // combine with the other half of the row
      float* slot = xchg + (j & 1) * 256;
      slot[half * 128 + r] = mx;
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
      mx = fmaxf(mx, slot[(half ^ 1) * 128 + r]) * c;
      const bool grow = mx > m + kRescaleThreshold;  // includes the first block
      const float m_use = grow ? mx : m;
      const float corr = fast_exp2(m - m_use);        // 1 when m stays, 0 on block 0
      m = m_use;
      // packed fp32 pairs (fma/add .f32x2): one instruction for two elements
      float2 sums[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      const float2 c2 = make_float2(c, c), negm2 = make_float2(-m, -m);
      uint32_t pw[kAttHalf / 2];
      auto make_p = [&](auto masked) {
#pragma unroll
        for (int i = 0; i < kAttHalf; i += 2) {
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1])),
                                      c2, negm2);
          float p0, p1;
          if (((i / 2) % 4) == 3) {
            const float2 e = exp2_poly2(x);
            p0 = e.x;
            p1 = e.y;
          } else {
            p0 = fast_exp2(x.x);
            p1 = fast_exp2(x.y);
          }
          if (decltype(masked)::value) {
            p0 = (i < kvalid) ? p0 : 0.0f;
            p1 = (i + 1 < kvalid) ? p1 : 0.0f;
          }
          pw[i / 2] = pack_bf16x2_rne(p0, p1);
          sums[(i / 2) & 1] = __fadd2_rn(sums[(i / 2) & 1], make_float2(p0, p1));
        }
      };
      if (kvalid >= kAttHalf) make_p(std::false_type());
      else make_p(std::true_type());

      const uint32_t t_p = t_buf + (uint32_t)p_col(half);
      tmem_st16(t_p, pw);
      tmem_st8(t_p + 16, pw + 16);
      // O rescale: PV(j-1) must have landed (o_done of its parity; the wait is
      // unambiguous because S(j) arriving implies PV(j-2) has completed)
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        if (!mbar_wait(&o_done[2 * t + ((j - 1) & 1)], (uint32_t)((j - 1) >> 1) & 1u, a.err))
          ok = false;
        tc_fence_after();
        uint32_t ov[32];
        tmem_ld32(t_o, ov);
        tmem_wait_ld();
        const float2 corr2 = make_float2(corr, corr);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 o2 = __fmul2_rn(make_float2(__uint_as_float(ov[i]), __uint_as_float(ov[i + 1])),
                                       corr2);
          ov[i] = __float_as_uint(o2.x);
          ov[i + 1] = __float_as_uint(o2.y);
        }
        tmem_st32(t_o, ov);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[2 * t + (j & 1)]);
      l = l * corr + ((sums[0].x + sums[1].x) + (sums[0].y + sums[1].y));
    }
    // tile B's last turn is consumed, so no phase is left pending at exit

    if (ok) ok = mbar_wait(&o_done[2 * t + ((nkv - 1) & 1)], (uint32_t)((nkv - 1) >> 1) & 1u, a.err);
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

// The persistent form of attention_kernel for short items (see the file head).
__global__ void __launch_bounds__(kAttThreads, 1)
    attention_persistent_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 buffers of (Q_A, Q_B)
  uint8_t* sK = smem + 4 * kQBytes;                    // kAttStages slots
  uint8_t* sV = sK + kAttStages * kKVBytes;            // kAttStages slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kAttStages * kKVBytes);
  uint64_t* q_full = bars;                             // [Q buffer]
  uint64_t* q_empty = bars + 2;                        // [Q buffer]
  uint64_t* k_full = bars + 4;                         // [kAttStages]
  uint64_t* k_empty = k_full + kAttStages;             // [kAttStages]
  uint64_t* v_full = k_empty + kAttStages;             // [kAttStages]
  uint64_t* v_empty = v_full + kAttStages;             // [kAttStages]
  // Every barrier below is waited on by parity, which tells apart only the
  // current phase and the one before: S(g+2) is issued after PV(g), so no
  // barrier gets two phases ahead of its waiter (the softmax warps of a tile
  // may finish block g+1 before PV(g) is issued, hence p_full per block parity)
  uint64_t* s_full = v_empty + kAttStages;             // [tile][buffer]
  uint64_t* p_full = s_full + 4;                       // [tile][block parity]
  uint64_t* o_done = p_full + 4;                       // [tile][PV parity]
  uint64_t* done = o_done + 4;                         // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
  float* xchg_base = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kAttBarBytes);

  const int warp = warp_id(), lane = lane_id();
  const int T = a.T;
  const int nkv = (T + kAttBK - 1) / kAttBK;
  // This CTA's items are blockIdx.x + it * gridDim.x for it < n_my (the grid is
  // never larger than the item count, so n_my >= 1). Item -> (query tile pair,
  // head, clip) with the tile pair fastest, so the CTAs working at one time
  // share each head's K and V in L2.
  const int n_my = (a.n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto item_coords = [&](int it, int& q0, int& h, int& row0) {
    const int item = (int)blockIdx.x + it * (int)gridDim.x;
    const int rest = item / a.num_q_tiles;
    q0 = (item - rest * a.num_q_tiles) * 2 * kAttBQ;
    h = rest % a.H;
    row0 = (rest / a.H) * T;
  };

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);   // released by both tiles' issuers
    }
    for (int i = 0; i < kAttStages; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 2);   // released by both tiles' issuers
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 2);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
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
  pdl_launch_dependents();
  pdl_wait();   // Q, K and V come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: per item its Q tile pair into Q buffer
      // it % 2 (free once both issuers' last S of item it - 2 has completed),
      // then its K and V blocks; g numbers the key blocks across items and
      // picks the ring slot and phase.
      uint32_t issued_q = 0, issued_k = 0, issued_v = 0;
      uint32_t last_q_phase = 0, last_k_phase = 0, last_v_phase = 0;
      bool ok = true;
      int g = 0;
      for (int it = 0; ok && it < n_my; it++) {
        int q0, h, row0;
        item_coords(it, q0, h, row0);
        const int qb = it & 1;
        const uint32_t qph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&q_empty[qb], qph ^ 1, a.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&q_full[qb], 2 * kQBytes);
        uint8_t* q_dst = sQ + qb * 2 * kQBytes;
        tma_load_2d(&tmQ, &q_full[qb], q_dst, h * kAttHD, row0 + q0);
        tma_load_2d(&tmQ, &q_full[qb], q_dst + kQBytes, h * kAttHD, row0 + q0 + kAttBQ);
        issued_q |= 1u << qb;
        last_q_phase = (last_q_phase & ~(1u << qb)) | (qph << qb);
        for (int j = 0; j < nkv; j++, g++) {
          const int s = g % kAttStages;
          const uint32_t ph = (uint32_t)(g / kAttStages) & 1u;
          if (!mbar_wait(&k_empty[s], ph ^ 1, a.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], kKVBytes);
          tma_load_2d(&tmK, &k_full[s], sK + s * kKVBytes, h * kAttHD, row0 + j * kAttBK);
          issued_k |= 1u << s;
          last_k_phase = (last_k_phase & ~(1u << s)) | (ph << s);
          if (!mbar_wait(&v_empty[s], ph ^ 1, a.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[s], kKVBytes);
          tma_load_2d(&tmV, &v_full[s], sV + s * kKVBytes, h * kAttHD, row0 + j * kAttBK);
          issued_v |= 1u << s;
          last_v_phase = (last_v_phase & ~(1u << s)) | (ph << s);
        }
      }
      if (!ok) {  // drain copies in flight (1 ms at most each)
        for (int i = 0; i < 2; i++)
          if (issued_q & (1u << i)) mbar_wait_for(&q_full[i], (last_q_phase >> i) & 1u, 1000000ull);
        for (int s = 0; s < kAttStages; s++) {
          if (issued_k & (1u << s)) mbar_wait_for(&k_full[s], (last_k_phase >> s) & 1u, 1000000ull);
          if (issued_v & (1u << s)) mbar_wait_for(&v_full[s], (last_v_phase >> s) & 1u, 1000000ull);
        }
      }
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      // ---------------- MMA issuers: warp 1 for tile A, warp 2 for tile B, so
      // each tile's S -> softmax -> PV round trip runs on its own and the two
      // overlap. The tensor core runs one thread's MMAs in issue order.
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kAttBQ, kAttBK, 0, 0);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kAttBQ, kAttHD, 0, 1);
      // The ring slot and S buffer are fixed at compile time (the block loop is
      // unrolled by six = three slots x two buffers), so each operand is one
      // constant offset from these bases and each group of MMAs is one asm
      // statement with a single pair of predicates.
      const uint64_t q_desc = sdesc_kmajor_sw128(smem_u32(sQ));
      const uint64_t k_desc = sdesc_kmajor_sw128(smem_u32(sK));
      const uint64_t v_desc = sdesc_mnmajor_sw128(smem_u32(sV), kKVBytes);
      // S_t(g) = Q_t K_g^T into buffer B from ring slot SL and Q buffer qb
      // (K = 64: four MMAs, 32 bytes of K apart)
      auto mma_s = [&](auto t_c, auto b_c, auto sl_c, uint32_t qb) {
        constexpr int t = decltype(t_c)::value, b = decltype(b_c)::value,
                      sl = decltype(sl_c)::value;
        const uint32_t d = tmem + (uint32_t)((2 * t + b) * kSBufCols);
        const uint64_t qa = q_desc + (uint64_t)((2 * qb + t) * (kQBytes >> 4));
        const uint64_t kb = k_desc + (uint64_t)(sl * (kKVBytes >> 4));
        asm volatile(
            "{\n\t.reg .pred pf, pt;\n\t"
            "setp.ne.b32 pf, %1, %1;\n\t"
            "setp.eq.b32 pt, %1, %1;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %3, %1, pf;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %5, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %7, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %9, %1, pt;\n\t}\n" ::"r"(d),
            "r"(idesc_qk), "l"(qa), "l"(kb), "l"(qa + 2), "l"(kb + 2), "l"(qa + 4), "l"(kb + 4),
            "l"(qa + 6), "l"(kb + 6)
            : "memory");
      };
      // O_t += P_t V from buffer B and ring slot SL: six MMAs of 16 keys, P
      // read from tensor memory (keys 0-47 at columns 0-23, 48-95 at 64-87),
      // V MN-major 2048 bytes (16 rows) apart; acc = 0 for an item's first block
      auto mma_pv = [&](auto t_c, auto b_c, auto sl_c, uint32_t acc) {
        constexpr int t = decltype(t_c)::value, b = decltype(b_c)::value,
                      sl = decltype(sl_c)::value;
        const uint32_t d = tmem + (uint32_t)(kOCol + t * kAttHD);
        const uint32_t pa = tmem + (uint32_t)((2 * t + b) * kSBufCols);
        const uint64_t vb = v_desc + (uint64_t)(sl * (kKVBytes >> 4));
        asm volatile(
            "{\n\t.reg .pred p0, pt;\n\t"
            "setp.ne.b32 p0, %2, 0;\n\t"
            "setp.eq.b32 pt, %1, %1;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %9, %1, p0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %10, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %11, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %12, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %13, %1, pt;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %14, %1, pt;\n\t}\n" ::"r"(d),
            "r"(idesc_pv), "r"(acc), "r"(pa + p_col(0)), "r"(pa + p_col(0) + 8),
            "r"(pa + p_col(0) + 16), "r"(pa + p_col(1)), "r"(pa + p_col(1) + 8),
            "r"(pa + p_col(1) + 16), "l"(vb), "l"(vb + 128), "l"(vb + 256), "l"(vb + 384),
            "l"(vb + 512), "l"(vb + 640)
            : "memory");
      };
      auto run = [&](auto t_c) {
        constexpr int t = decltype(t_c)::value;
        const int G = n_my * nkv;   // key blocks of all this CTA's items
        bool ok = true;
        // S of block g (g % 6 == M) into buffer M % 2 from slot M % 3. The K
        // slot frees once both tiles' products are done (count 2); after an
        // item's last S, so does its Q buffer. s_item / s_j: the item of the
        // next S and its block within the item.
        int s_item = 0, s_j = 0;
        auto issue_s = [&](int g, auto mc) -> bool {
          constexpr int m = decltype(mc)::value;
          const uint32_t qb = (uint32_t)s_item & 1u;
          if (s_j == 0 && !mbar_wait(&q_full[qb], (uint32_t)(s_item >> 1) & 1u, a.err))
            return false;
          if (!mbar_wait(&k_full[m % 3], (uint32_t)(g / kAttStages) & 1u, a.err)) return false;
          tc_fence_after();
          mma_s(t_c, std::integral_constant<int, m % 2>(), std::integral_constant<int, m % 3>(),
                qb);
          umma_commit(&s_full[2 * t + m % 2]);
          umma_commit(&k_empty[m % 3]);
          if (++s_j == nkv) {
            umma_commit(&q_empty[qb]);
            s_j = 0;
            s_item++;
          }
          return true;
        };
        // Block g: PV_t(g), then S_t(g + 2) into the buffer PV_t(g) has read P
        // from. pv_j: block of this PV within its item.
        int pv_j = 0;
        auto step = [&](int g, auto mc) -> bool {
          constexpr int m = decltype(mc)::value;
          if (!mbar_wait(&p_full[2 * t + m % 2], (uint32_t)(g >> 1) & 1u, a.err)) return false;
          if (!mbar_wait(&v_full[m % 3], (uint32_t)(g / kAttStages) & 1u, a.err)) return false;
          tc_fence_after();
          mma_pv(t_c, std::integral_constant<int, m % 2>(), std::integral_constant<int, m % 3>(),
                 pv_j > 0 ? 1u : 0u);
          if (++pv_j == nkv) pv_j = 0;
          umma_commit(&o_done[2 * t + m % 2]);
          umma_commit(&v_empty[m % 3]);
          if (g + 2 < G) return issue_s(g + 2, std::integral_constant<int, (m + 2) % 6>());
          return true;
        };
        if (t == 1) spin_cycles(kTileBOffsetCycles);
        ok = issue_s(0, std::integral_constant<int, 0>());
        if (ok && G > 1) ok = issue_s(1, std::integral_constant<int, 1>());
        for (int g = 0; ok && g < G; g += 6) {
          ok = step(g, std::integral_constant<int, 0>());
          if (ok && g + 1 < G) ok = step(g + 1, std::integral_constant<int, 1>());
          if (ok && g + 2 < G) ok = step(g + 2, std::integral_constant<int, 2>());
          if (ok && g + 3 < G) ok = step(g + 3, std::integral_constant<int, 3>());
          if (ok && g + 4 < G) ok = step(g + 4, std::integral_constant<int, 4>());
          if (ok && g + 5 < G) ok = step(g + 5, std::integral_constant<int, 5>());
        }
        // every MMA of this issuer has completed before tensor memory is released
        umma_commit(&done[t]);
        mbar_wait_for(&done[t], 0, kWaitTimeoutNs);
      };
      if (warp == 1) run(std::integral_constant<int, 0>());
      else run(std::integral_constant<int, 1>());
    }
  } else {
    // ---------------- softmax: warps 3-10 tile A, 11-18 tile B. Each query row
    // is split over two warps of the same TMEM sub-partition: half 0 takes keys
    // 0-47 of every block and O columns 0-31, half 1 keys 48-95 and O 32-63.
    const int t = (warp - 3) >> 3;
    const int half = ((warp - 3) & 7) >> 2;
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // row within the tile
    const uint32_t t_lane = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t t_o = t_lane + (uint32_t)(kOCol + t * kAttHD + half * 32);
    // partial row maxima (and the final row sums) of the two halves, in two
    // slots used in turn. Item `it` makes nkv + 1 exchanges, so g + it of them
    // come before block g's and g + it (g one past the item) before its row-sum
    // exchange; consecutive exchanges therefore alternate slots, across items.
    float* xchg = xchg_base + t * 2 * 2 * 128;  // [slot][half][row]
    const int bar_id = 1 + t * 4 + sub;          // named barrier of the warp pair
    const float c = a.scale_log2;
    bool ok = true;
    int g = 0;  // key block across this CTA's items
    for (int it = 0; it < n_my; it++) {
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < nkv; j++, g++) {
        const int kvalid = min(kAttBK, T - j * kAttBK) - half * kAttHalf;  // valid keys of this half
        const uint32_t t_buf = t_lane + (uint32_t)((2 * t + (g & 1)) * kSBufCols);
        // A failed wait never leaves the loops: the two halves of a row meet at
        // named barriers (which have no time limit) once per block, so both run
        // every iteration; once the error word is set the remaining waits return
        // at once.
        if (!mbar_wait(&s_full[2 * t + (g & 1)], (uint32_t)(g >> 1) & 1u, a.err)) ok = false;
        tc_fence_after();
        uint32_t s[kAttHalf];
        tmem_ld16<16>(t_buf + half * kAttHalf, s);
        tmem_ld16<16>(t_buf + half * kAttHalf + 16, s + 16);
        tmem_ld16<16>(t_buf + half * kAttHalf + 32, s + 32);
        tmem_wait_ld();
        float mx;
        if (kvalid >= kAttHalf) {
          float mm[8];   // three-input max: 24 instructions for 48 values
#pragma unroll
          for (int i = 0; i < 8; i++)
            mm[i] = fmax3(fmax3(__uint_as_float(s[i]), __uint_as_float(s[i + 8]),
                                __uint_as_float(s[i + 16])),
                          __uint_as_float(s[i + 24]),
                          fmaxf(__uint_as_float(s[i + 32]), __uint_as_float(s[i + 40])));
          mx = fmax3(fmax3(mm[0], mm[1], mm[2]), fmax3(mm[3], mm[4], mm[5]), fmaxf(mm[6], mm[7]));
        } else {
          mx = -INFINITY;
#pragma unroll
          for (int i = 0; i < kAttHalf; i++)
            if (i < kvalid) mx = fmaxf(mx, __uint_as_float(s[i]));
        }
        // combine with the other half of the row
        float* slot = xchg + ((g + it) & 1) * 256;
        slot[half * 128 + r] = mx;
        asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
        mx = fmaxf(mx, slot[(half ^ 1) * 128 + r]) * c;
        const bool grow = mx > m + kRescaleThreshold;  // includes the first block
        const float m_use = grow ? mx : m;
        const float corr = fast_exp2(m - m_use);        // 1 when m stays, 0 on block 0
        m = m_use;
        // packed fp32 pairs (fma/add .f32x2): one instruction for two elements
        float2 sums[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
        const float2 c2 = make_float2(c, c), negm2 = make_float2(-m, -m);
        uint32_t pw[kAttHalf / 2];
        auto make_p = [&](auto masked) {
#pragma unroll
          for (int i = 0; i < kAttHalf; i += 2) {
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1])),
                                        c2, negm2);
            float p0, p1;
            if (((i / 2) % 4) == 3) {
              const float2 e = exp2_poly2(x);
              p0 = e.x;
              p1 = e.y;
            } else {
              p0 = fast_exp2(x.x);
              p1 = fast_exp2(x.y);
            }
            if (decltype(masked)::value) {
              p0 = (i < kvalid) ? p0 : 0.0f;
              p1 = (i + 1 < kvalid) ? p1 : 0.0f;
            }
            pw[i / 2] = pack_bf16x2_rne(p0, p1);
            sums[(i / 2) & 1] = __fadd2_rn(sums[(i / 2) & 1], make_float2(p0, p1));
          }
        };
        if (kvalid >= kAttHalf) make_p(std::false_type());
        else make_p(std::true_type());

        const uint32_t t_p = t_buf + (uint32_t)p_col(half);
        tmem_st16(t_p, pw);
        tmem_st8(t_p + 16, pw + 16);
        // O rescale: PV(g-1) must have landed (o_done of its parity; the wait is
        // unambiguous because S(g) arriving implies PV(g-2) has completed)
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          if (!mbar_wait(&o_done[2 * t + ((g - 1) & 1)], (uint32_t)((g - 1) >> 1) & 1u, a.err))
            ok = false;
          tc_fence_after();
          uint32_t ov[32];
          tmem_ld32(t_o, ov);
          tmem_wait_ld();
          const float2 corr2 = make_float2(corr, corr);
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 o2 = __fmul2_rn(make_float2(__uint_as_float(ov[i]), __uint_as_float(ov[i + 1])),
                                         corr2);
            ov[i] = __float_as_uint(o2.x);
            ov[i + 1] = __float_as_uint(o2.y);
          }
          tmem_st32(t_o, ov);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[2 * t + (g & 1)]);
        l = l * corr + ((sums[0].x + sums[1].x) + (sums[0].y + sums[1].y));
      }
      // The item's last PV (block g - 1) must have landed before O is read; the
      // next item's first PV, which overwrites O, waits for this warp's next
      // p_full arrival, which comes after the read.
      const int gl = g - 1;
      if (ok) ok = mbar_wait(&o_done[2 * t + (gl & 1)], (uint32_t)(gl >> 1) & 1u, a.err);
      // the row sum is the sum of the two halves' sums
      float* lslot = xchg + ((g + it) & 1) * 256;
      lslot[half * 128 + r] = l;
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
      l += lslot[(half ^ 1) * 128 + r];
      if (ok) {
        tc_fence_after();
        uint32_t o0[32];
        tmem_ld32(t_o, o0);
        tmem_wait_ld();
        int q0, h, row0;
        item_coords(it, q0, h, row0);
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
  const int64_t nq = (T + 2 * kAttBQ - 1) / (2 * kAttBQ);      // tile pairs per (head, clip)
  if (nq * H * B > INT32_MAX) return fail(WX_ERR_UNSUPPORTED, "attention: more than 2^31 tile pairs");
  g.num_q_tiles = (int)nq;
  g.n_items = (int)(nq * H * B);
  g.O = o;
  g.ldo = ldo;
  g.scale_log2 = scale * 1.4426950408889634f;
  g.err = err;
  p->B = (int)B;
  // Short items run persistent: one CTA per SM, or per item when there are
  // fewer items than SMs.
  p->persist = (T + kAttBK - 1) / kAttBK <= kAttPersistMaxBlocks;
  p->grid = std::min(g.n_items, sm_count());
  // set when the plan is made, so a captured launch sequence holds only launches
  static bool attr_set[64] = {false};
  int dev = 0;
  WX_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !attr_set[dev]) {
    WX_CUDA_TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kAttSmem));
    WX_CUDA_TRY(cudaFuncSetAttribute(attention_persistent_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kAttSmemPersist));
    if (dev < 64) attr_set[dev] = true;
  }
  return WX_OK;
}

int attn_run(const AttnPlan& p, cudaStream_t st) {
  if (p.persist) {
    WX_CUDA_TRY(launch_k(attention_persistent_kernel, dim3(p.grid), dim3(kAttThreads),
                         kAttSmemPersist, st, p.tmQ, p.tmK, p.tmV, p.args));
  } else {
    dim3 grid(p.args.num_q_tiles, p.args.H, p.B);
    WX_CUDA_TRY(launch_k(attention_kernel, grid, dim3(kAttThreads), kAttSmem, st, p.tmQ, p.tmK,
                         p.tmV, p.args));
  }
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
