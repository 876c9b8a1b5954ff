// flashb: causal GQA prefill attention on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces the backbone prefill attention of the reference (flash/prefill_attn.py:15-46, bz_prefill_attention, which
// trims K/V/mask to the prefill length L and calls the eager transformers attention, UP/models/breeze.py:259-286):
//     s = bf16(bf16(q k^T) * scaling) ; s = bf16(s + mask) ; p = bf16(softmax_fp32(s)) ; out = bf16(p v)
// with q [B, NH, L, D], k/v [B, NKV, S, D] (GQA: q head h reads kv head h / (NH / NKV)), an additive mask
// [B | 1, 1, L, S] (bf16 or fp32) and out [B, L, NH, D] (the eager transpose(1, 2)).
//
// One CTA per (128-query tile, q head, batch row); 16 warps: warp w reads TMEM lanes 32 (w % 4) .. (query rows) and
// owns key / output columns [32 (w / 4), 32 (w / 4) + 32) of every tile, so four threads share a row.
//   * Q, K and V tiles (128 x 128 bf16, 32 KB each) sit in canonical no-swizzle UMMA layouts (8-row x 16-byte core
//     matrices) and arrive by one TMA tensor copy each (fbh::tmap_heads: a box of [16 chunks of 8 dims][128 rows]
//     [16 B], rows past L or S zero-filled): Q (once per CTA) and K as K-major tiles with LBO = 2048 B between K
//     chunks and SBO = 128 B between 8-row groups, V as an MN-major tile (8-key x 8-dim core matrices, LBO = 128 B
//     between key groups, SBO = 2048 B between dimension groups).  P (written by the threads) is K-major with
//     LBO = 128 B and SBO = 2048 B.
//   * Thread 0 issues tcgen05.mma.cta_group::1.kind::f16 (bf16 x bf16 -> fp32, M = N = 128, K = 16 per
//     instruction) and tcgen05.commit to an mbarrier; the others wait on it (bounded).
//   * Copies run one key tile ahead: K(t + 1) and its mask (two mask buffers) while tile t's scores are read,
//     V(t + 1) once P(t) V(t) is done; S(t + 1) is issued as soon as K(t + 1) has landed.
//   * Pass 1: S = Q K^T per key tile into TMEM columns [0, 128); every thread reads its 32 scores (tcgen05.ld
//     32x32b), applies the eager rounding points and the mask, and keeps a running max and fp32 sum of
//     exp(s - max) (rescaled when the max grows); the four quarters of a row are merged after the pass.
//   * Pass 1 also keeps the rounded, masked scores of the first PF_KEEP key tiles in TMEM columns [256, 512) as bf16
//     pairs (they are bf16 values; not with an fp32 mask).
//   * Pass 2: per tile, the kept scores read back from TMEM, or S again; p = bf16(exp(s - max) / sum) exactly as
//     the eager softmax forms it, written to shared memory as the K-major A operand; O += P V on tcgen05 into TMEM
//     columns [128, 256).  Keeping the scores saves pass 2 the K copy, the S MMAs and the fp32 score rounding of
//     those tiles (all of them at prompts up to 512 tokens).
//   * Epilogue: O row -> bf16 -> out.  Rows whose every key is masked (left padding) are written as 0 (their
//     outputs never reach a live row; the oracle uses the same convention).
// With `causal` the key tiles entirely above the diagonal are skipped: the mask gives them probability exactly 0.
#include "fb_common.cuh"
#include "fb_norm.cuh"

namespace fb {

constexpr int PF_TILE = 128;                       // queries per CTA = keys per tile = TMEM lanes
constexpr int PF_D = 128;                          // head dim
constexpr int PF_QUARTERS = 4;                     // column quarters per row (one warp per lane quarter each)
constexpr int PF_THREADS = 128 * PF_QUARTERS;     // 16 warps
constexpr int PF_OPND = PF_TILE * PF_D * 2;        // 32 KB per operand tile
constexpr int PF_MPITCH = PF_TILE * 2 + 16;       // bytes per staged bf16 mask row (padded: fewer bank conflicts)
constexpr int PF_MASK = PF_TILE * PF_MPITCH;       // the bf16 mask tile of the current key tile
constexpr int PF_SMEM = 4 * PF_OPND + 2 * PF_MASK + 64;  // Q, K, V, P, two mask tiles, four mbarriers, TMEM slot
constexpr uint32_t PF_TMEM_COLS = 512;             // S: columns [0, 128); O: [128, 256); kept scores: [256, 512)
constexpr int PF_KEEP = 4;                         // key tiles whose pass-1 scores stay in TMEM (bf16 pairs, 64 columns each)

struct alignas(64) PFArgs {
  CUtensorMap tq, tk, tv;  // Q of every (batch row, q head), K and V of every (batch row, KV head): fbh::tmap_heads
  const bf16 *q, *k, *v;
  long q_sb, q_sh, q_sl, k_sb, k_sh, k_sl, v_sb, v_sh, v_sl;
  const void* mask;
  int mask_bf16;
  long m_sb, m_sl;
  bf16* out;
  long o_sb, o_sl, o_sh;
  int B, NH, NKV, L, S, h0, causal;
  int t0;              // first query tile of the launch (a query-row shard computes tiles [t0, t0 + gridDim.x))
  float scaling;
  unsigned* err;
};

// Shared-memory matrix descriptor, no swizzle: start >> 4 in [0, 14), LBO >> 4 in [16, 30), SBO >> 4 in [32, 46),
// descriptor version 1 in [46, 48), layout type 0 (none) in [61, 64).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: D fp32 (bits 4-5 = 1), A bf16 (7-9 = 1), B bf16 (10-12 = 1), A K-major
// (bit 15 = 0), B major given (bit 16), N >> 3 in [17, 23), M >> 4 in [24, 29); M = N = 128.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_128(uint32_t b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void cp_async16_pf(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all_pf() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_commit_pf() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_pf() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32w .. 32w + 31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&f)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
}

// 16 consecutive 32-bit TMEM columns of this thread's lane: store (then wait for the store), load (then wait).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte chunk c (elements 8c .. 8c+7 along K) of row r in a K-major no-swizzle tile of 128 x 128.
__device__ __forceinline__ uint32_t kmaj_off(int r, int c) { return (((r >> 3) << 4) + c) * 128 + (r & 7) * 16; }
// TMA tensor copy of a 5-D box into shared memory, completion counted on an mbarrier (no multicast).
__device__ __forceinline__ void tma_load_5d(void* dst, const void* tmap, int c0, int c1, int c2, int c3, int c4,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// Stage the bf16 mask tile of key tile t (rows q0.., columns 128 t..) into smem rows of PF_MPITCH bytes: 16-byte
// cp.async chunks where aligned and in range, element loads at ragged edges.
__device__ __forceinline__ void stage_mask(const PFArgs& a, int b, int q0, int t, unsigned char* sm) {
  const bf16* mb = reinterpret_cast<const bf16*>(a.mask) + (size_t)b * a.m_sb;
  for (int i = threadIdx.x; i < PF_TILE * 16; i += PF_THREADS) {
    const int r = i >> 4, c = i & 15, row = q0 + r, col = t * PF_TILE + c * 8;
    unsigned char* dst = sm + r * PF_MPITCH + c * 16;
    const bf16* src = mb + (size_t)(row < a.L ? row : 0) * a.m_sl + col;
    if (row < a.L && col + 8 <= a.S && (((uintptr_t)src) & 15) == 0) {
      cp_async16_pf(dst, src);
    } else {
      bf16* d = reinterpret_cast<bf16*>(dst);
#pragma unroll
      for (int e = 0; e < 8; ++e) d[e] = (row < a.L && col + e < a.S) ? src[e] : __float2bfloat16_rn(0.f);
    }
  }
}

// Mask values of this thread's row for key columns [col0, col0 + 32) (absolute key index), or 0 without a mask.
// bf16 masks come from the staged tile (`srow` = this thread's row, `c0` = column offset in the tile).
__device__ __forceinline__ void load_mask32(const PFArgs& a, int b, int row, int col0, const unsigned char* srow,
                                            int c0, float (&mv)[32]) {
  if (!a.mask) {
#pragma unroll
    for (int i = 0; i < 32; ++i) mv[i] = 0.f;
    return;
  }
  if (a.mask_bf16) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float f[8];
      cvt8(*reinterpret_cast<const uint4*>(srow + (c0 + c * 8) * 2), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) mv[c * 8 + e] = f[e];
    }
  } else {
    const float* p = reinterpret_cast<const float*>(a.mask) + (size_t)b * a.m_sb + (size_t)row * a.m_sl + col0;
#pragma unroll
    for (int i = 0; i < 32; ++i) mv[i] = (col0 + i < a.S) ? p[i] : 0.f;
  }
}

__global__ void __launch_bounds__(PF_THREADS, 1) prefill_attn_kernel(const __grid_constant__ PFArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* sq = smem;
  unsigned char* sk = smem + PF_OPND;
  unsigned char* sv = smem + 2 * PF_OPND;
  unsigned char* sp = smem + 3 * PF_OPND;
  unsigned char* smb[2] = {smem + 4 * PF_OPND, smem + 4 * PF_OPND + PF_MASK};   // mask tiles of even / odd key tiles
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + 4 * PF_OPND + 2 * PF_MASK);
  uint64_t* bar_o = bar_s + 1;
  uint64_t* bar_k = bar_s + 2;           // K tile landed (TMA)
  uint64_t* bar_v = bar_s + 3;           // V tile landed (TMA)
  uint64_t* bar_q = bar_s + 4;           // Q tile landed (TMA)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_s + 5);
  __shared__ float s_stat[2][PF_QUARTERS][PF_TILE];   // per (column quarter, row): running max, sum

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // TMEM lane quarter (warp % 4) x column quarter (warp / 4): this thread owns row r, columns [32 cq, 32 cq + 32)
  const int r = (warp & 3) * 32 + lane, cq = warp >> 2;
  const int q0 = (a.t0 + (int)blockIdx.x) * PF_TILE, h = a.h0 + blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.NH / a.NKV);
  const int row = q0 + r;
  const bool row_ok = row < a.L;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_k, 1);
    mbar_init(bar_v, 1);
    mbar_init(bar_q, 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tq) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tv) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(PF_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t t_s = tmem, t_o = tmem + 128, t_keep = tmem + 256;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;   // this warp's TMEM lane quarter
  const uint32_t my_taddr = lane_base + cq * 32;

  // Q tile -> K-major A operand, [16 chunks of 8 dims][128 rows][16 B] by one TMA copy (rows beyond L are zero);
  // the first S waits for it
  bool q_in = false;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_q, (unsigned)PF_OPND);
    tma_load_5d(sq, &a.tq, 0, q0, 0, h, b, bar_q);
  }
  const int ntile_all = (a.S + PF_TILE - 1) / PF_TILE;
  int ntile = ntile_all;
  if (a.causal) {
    const int last_q = min(q0 + PF_TILE, a.L) - 1;
    ntile = min(ntile_all, last_q / PF_TILE + 1);
  }
  const uint32_t idesc_s = umma_idesc_bf16_128(0u), idesc_o = umma_idesc_bf16_128(1u);
  const uint32_t aq = smem_u32(sq), ak = smem_u32(sk), av = smem_u32(sv), ap = smem_u32(sp);
  unsigned ph_s = 0, ph_o = 0;
  float mx = -INFINITY, sum = 0.f;
  bool fail = false;
  const bool mask_smem = a.mask && a.mask_bf16;
  // pass-1 scores kept in TMEM for pass 2 (tiles [0, nkeep)): they are bf16 values unless an fp32 mask is added
  const int nkeep = (!a.mask || a.mask_bf16) ? min(ntile, PF_KEEP) : 0;

  // Staging of key tile t: K (K-major B operand of S = Q K^T) and V (MN-major B operand of O += P V) by one TMA
  // tensor copy each (thread 0, an mbarrier per operand; rows past S arrive as zeros), both as [16 chunks of 8 dims]
  // [128 keys][16 B]; the tile's bf16 mask rows by cp.async from every thread (one group, the caller commits).
  // At most one copy of each operand is in flight; for thread 0, kpend / vpend count them and kpar / vpar hold the
  // parity their wait uses (the waits come in copy order).
  unsigned ph_k = 0, ph_v = 0, kpar = 0, vpar = 0;
  int kpend = 0, vpend = 0;
  auto stage_k = [&](int t) {
    if (mask_smem) stage_mask(a, b, q0, t, smb[t & 1]);
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_k, (unsigned)PF_OPND);
      tma_load_5d(sk, &a.tk, 0, t * PF_TILE, 0, kvh, b, bar_k);
      ++kpend;
      kpar = ph_k;
    }
  };
  auto stage_v = [&](int t) {
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_v, (unsigned)PF_OPND);
      tma_load_5d(sv, &a.tv, 0, t * PF_TILE, 0, kvh, b, bar_v);
      ++vpend;
      vpar = ph_v;
    }
  };
  // Issue S = Q K^T once K has landed and this tile's mask chunks are in (8 MMAs of K = 16, Q's and K's start
  // advancing 4096 B, two 2048-byte chunks, per step); false if a wait gave up.
  auto issue_s = [&]() -> bool {
    cp_wait_pf<0>();
    bool ok = true;
    if (tid == 0) {
      if (!q_in) ok = q_in = mbar_wait(bar_q, 0, a.err);
      ok = ok && mbar_wait(bar_k, ph_k, a.err);
      if (ok) --kpend;
    }
    ph_k ^= 1u;
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) return false;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < PF_D / 16; ++s)
        umma_bf16(t_s, umma_desc(aq + 4096 * s, 2048, 128), umma_desc(ak + 4096 * s, 2048, 128), idesc_s, s > 0);
      umma_commit(bar_s);
    }
    return true;
  };
  // Wait for V(t), then O += P(t) V(t) (P written by every thread before); false if the wait gave up.
  auto issue_o = [&](int t) -> bool {
    bool ok = true;
    if (tid == 0) {
      ok = mbar_wait(bar_v, ph_v, a.err);
      if (ok) --vpend;
    }
    ph_v ^= 1u;
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) return false;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < PF_TILE / 16; ++s)
        umma_bf16(t_o, umma_desc(ap + 256 * s, 128, 2048), umma_desc(av + 256 * s, 128, 2048), idesc_o,
                  (t > 0 || s > 0) ? 1u : 0u);
      umma_commit(bar_o);
    }
    return true;
  };
  auto wait_s = [&]() {
    const bool ok = mbar_wait(bar_s, ph_s, a.err);
    ph_s ^= 1u;
    if (__syncthreads_or(!ok)) return false;
    tc_fence_after();
    return true;
  };
  auto wait_o = [&]() {
    const bool ok = mbar_wait(bar_o, ph_o, a.err);
    ph_o ^= 1u;
    if (__syncthreads_or(!ok)) return false;
    tc_fence_after();
    return true;
  };
  // this thread's 32 scores of key tile t with the eager rounding points; -inf for keys that do not exist
  auto scores32 = [&](int t, float (&sc)[32], uint32_t scol) {   // scol: TMEM column of the tile's S
    float acc[32], mv[32];
    tmem_ld32(scol + my_taddr, acc);
    const int col0 = t * PF_TILE + cq * 32;
    load_mask32(a, b, row_ok ? row : 0, col0, smb[t & 1] + r * PF_MPITCH, cq * 32, mv);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float s = rbf(rbf(acc[i]) * a.scaling);
      s = a.mask_bf16 ? rbf(s + mv[i]) : s + mv[i];
      const bool exists = (col0 + i < a.S) && !(a.causal && !a.mask && col0 + i > row);
      sc[i] = exists ? s : -INFINITY;
    }
  };

  // ---------------------------------------------------------------- pass 1: row max and sum of exp
  // S and K are double-buffered: S(t) in TMEM columns 128 (t % 2) (O's columns are free until pass 2), K(t) in sk
  // or sv (V's tile is free until pass 2), S(t) signalled on bar_s or bar_o.  At the start of tile t (S(t) done,
  // every thread past tile t - 1) thread 0 issues S(t + 1) on K(t + 1), copied one tile earlier, and copies
  // K(t + 2) into the buffer S(t) has released; the mask of tile t + 1 is copied into the buffer tile t - 1 used.
  // So the tensor core and the copies run while tile t's scores are read.  Only thread 0 waits on bar_k.
  bool kfail = false;                  // thread 0: a K or Q wait gave up (reported at the next barrier)
  auto stage_k1 = [&](int t) {         // thread 0
    mbar_arrive_expect_tx(bar_k, (unsigned)PF_OPND);
    tma_load_5d((t & 1) ? sv : sk, &a.tk, 0, t * PF_TILE, 0, kvh, b, bar_k);
    ++kpend;
    kpar = ph_k;
  };
  auto issue_s1 = [&](int t) {         // thread 0: S(t) once Q and K(t) are in
    bool ok = true;
    if (!q_in) ok = q_in = mbar_wait(bar_q, 0, a.err);
    ok = ok && mbar_wait(bar_k, ph_k, a.err);
    ph_k ^= 1u;
    if (!ok) {
      kfail = true;
      return;
    }
    --kpend;
    tc_fence_after();
    const uint32_t kb = (t & 1) ? av : ak;
#pragma unroll
    for (int s = 0; s < PF_D / 16; ++s)
      umma_bf16(t_s + 128u * (uint32_t)(t & 1), umma_desc(aq + 4096 * s, 2048, 128),
                umma_desc(kb + 4096 * s, 2048, 128), idesc_s, s > 0);
    umma_commit((t & 1) ? bar_o : bar_s);
  };
  if (ntile > 0) {
    if (mask_smem) stage_mask(a, b, q0, 0, smb[0]);
    cp_commit_pf();
    if (tid == 0) {
      stage_k1(0);
      issue_s1(0);
      if (ntile > 1 && !kfail) stage_k1(1);
    }
  }
  for (int t = 0; t < ntile && !fail; ++t) {
    cp_wait_pf<0>();                   // this thread's chunks of mask tile t
    tc_fence_before();
    {
      const bool odd = (t & 1) != 0;
      const bool ok = mbar_wait(odd ? bar_o : bar_s, odd ? ph_o : ph_s, a.err);
      if (odd) ph_o ^= 1u;
      else ph_s ^= 1u;
      if (__syncthreads_or(!ok || kfail)) {
        fail = true;
        break;
      }
      tc_fence_after();
    }
    if (t + 1 < ntile) {
      if (mask_smem) stage_mask(a, b, q0, t + 1, smb[(t + 1) & 1]);
      cp_commit_pf();
      if (tid == 0) {
        issue_s1(t + 1);
        if (t + 2 < ntile && !kfail) stage_k1(t + 2);
      }
    }
    float sc[32];
    scores32(t, sc, t_s + 128u * (uint32_t)(t & 1));
    if (t < nkeep) {
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = pack2(sc[2 * i], sc[2 * i + 1]);
      tmem_st16(t_keep + lane_base + (uint32_t)(t * 64 + cq * 16), pk);
    }
    float tm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) tm = fmaxf(tm, sc[i]);
    const float nm = fmaxf(mx, tm);
    if (nm > -INFINITY) {
      float add = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) add += __expf(sc[i] - nm);
      sum = (mx > -INFINITY ? sum * __expf(mx - nm) : 0.f) + add;
      mx = nm;
    }
  }
  tc_fence_before();
  // merge the four column quarters of every row (the same result in all four threads of a row)
  s_stat[0][cq][r] = mx;
  s_stat[1][cq][r] = sum;
  __syncthreads();
  {
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < PF_QUARTERS; ++k) m = fmaxf(m, s_stat[0][k][r]);
    float l = 0.f;
    if (m > -INFINITY) {
#pragma unroll
      for (int k = 0; k < PF_QUARTERS; ++k) {
        const float mk = s_stat[0][k][r];
        if (mk > -INFINITY) l += s_stat[1][k][r] * __expf(mk - m);
      }
    }
    mx = m;
    sum = l;
  }
  const bool dead = !(mx > -1e30f);
  const float inv = 1.0f / sum;

  // ---------------------------------------------------------------- pass 2: P = softmax, O += P V
  // Tiles [0, nkeep) read their scores back from TMEM; later tiles recompute S = Q K^T.  Per tile t: the scores
  // (for a recomputed tile: wait for S(t), then copy K(t + 1) and its mask, K being free once S(t) is done); P(t);
  // once V(t) has landed, O += P(t) V(t); when that MMA is done, copy V(t + 1) (and K(t + 1) for the first
  // recomputed tile) and issue S(t + 1) as soon as K(t + 1) is in.
  if (!fail && ntile > 0) {
    if (nkeep == 0) {
      stage_k(0);
      cp_commit_pf();
    }
    stage_v(0);
    if (nkeep == 0) fail = !issue_s();
  }
  for (int t = 0; t < ntile && !fail; ++t) {
    const bool kept = t < nkeep;
    float sc[32];
    if (kept) {
      uint32_t pk[16];
      tmem_ld16(t_keep + lane_base + (uint32_t)(t * 64 + cq * 16), pk);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sc[2 * i] = lo_f(pk[i]);
        sc[2 * i + 1] = hi_f(pk[i]);
      }
    } else {
      if (!wait_s()) {
        fail = true;
        break;
      }
      if (t + 1 < ntile) {
        stage_k(t + 1);
        cp_commit_pf();
      }
      scores32(t, sc, t_s);
    }
    // p = bf16(e^(s - max) / sum) with the fast exponential and one reciprocal per row: a few fp32 ulps, below the
    // bf16 rounding of p except at rare ties (the exact expf and IEEE division per score serialise on their
    // special-case branches and cost several microseconds per tile)
    float p[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) p[i] = (dead || !row_ok) ? 0.f : rbf(__expf(sc[i] - mx) * inv);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 w;
      w.x = pack2(p[c * 8 + 0], p[c * 8 + 1]);
      w.y = pack2(p[c * 8 + 2], p[c * 8 + 3]);
      w.z = pack2(p[c * 8 + 4], p[c * 8 + 5]);
      w.w = pack2(p[c * 8 + 6], p[c * 8 + 7]);
      *reinterpret_cast<uint4*>(sp + kmaj_off(r, cq * 4 + c)) = w;
    }
    if (!issue_o(t)) {
      fail = true;
      break;
    }
    // P and V are free again once this P V is done; the last one is waited for after the loop
    if (t + 1 < ntile) {
      if (!wait_o()) {
        fail = true;
        break;
      }
      const bool next_s = t + 1 >= nkeep;
      if (next_s && kept) {            // the first recomputed tile: its K has not been copied yet
        stage_k(t + 1);
        cp_commit_pf();
      }
      stage_v(t + 1);
      if (next_s && !issue_s()) {
        fail = true;
        break;
      }
    }
  }
  if (!fail && ntile > 0) {
    if (!wait_o()) fail = true;
  }
  cp_async_wait_all_pf();              // nothing may land in shared memory after this point (failure paths)
  if (tid == 0) {                      // a copy a failure path left in flight lands before the CTA ends
    if (!q_in) mbar_wait(bar_q, 0, nullptr);
    if (kpend) mbar_wait(bar_k, kpar, nullptr);
    if (vpend) mbar_wait(bar_v, vpar, nullptr);
  }

  // ---------------------------------------------------------------- epilogue: O -> bf16 -> out [B, L, NH, D]
  if (!fail) {
    float o[32];
    if (ntile > 0) tmem_ld32(t_o + my_taddr, o);
    if (row_ok) {
      bf16* og = a.out + (size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)row * a.o_sl + cq * 32;
      const bool z = dead || ntile == 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        const float* f = o + c * 8;
        w.x = z ? 0u : pack2(f[0], f[1]);
        w.y = z ? 0u : pack2(f[2], f[3]);
        w.z = z ? 0u : pack2(f[4], f[5]);
        w.w = z ? 0u : pack2(f[6], f[7]);
        *reinterpret_cast<uint4*>(og + c * 8) = w;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS) : "memory");
  }
}

}  // namespace fb

// ------------------------------------------------------------------------------------------------ host API
using namespace fb;

extern "C" int flashb_prefill_attn_tiles(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sl, const void* k,
                                         int64_t k_sb, int64_t k_sh, int64_t k_sl, const void* v, int64_t v_sb,
                                         int64_t v_sh, int64_t v_sl, const void* mask, int mask_is_bf16, int64_t m_sb,
                                         int64_t m_sl, int B, int NH, int NKV, int L, int S, int D, float scaling,
                                         int causal, int h0, int h1, int tile0, int tile1, void* out, int64_t o_sb,
                                         int64_t o_sl, int64_t o_sh, void* stream) {
  FB_CHECK_ARG(q && k && v && out, "prefill_attn: null pointer argument");
  FB_CHECK_ARG(D == PF_D, "prefill_attn: head_dim must be 128 (got %d)", D);
  FB_CHECK_ARG(B >= 1 && NH >= 1 && NKV >= 1 && NH % NKV == 0 && L >= 1 && S >= 1 && L <= 65535 * PF_TILE,
               "prefill_attn: bad shape B=%d NH=%d NKV=%d L=%d S=%d", B, NH, NKV, L, S);
  FB_CHECK_ARG(0 <= h0 && h0 < h1 && h1 <= NH, "prefill_attn: head range [%d, %d) outside [0, %d)", h0, h1, NH);
  const int ntile = (L + PF_TILE - 1) / PF_TILE;
  FB_CHECK_ARG(0 <= tile0 && tile0 < tile1 && tile1 <= ntile, "prefill_attn: query tiles [%d, %d) outside [0, %d)",
               tile0, tile1, ntile);
  const uintptr_t align = (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out;
  const int64_t strides = q_sb | q_sh | q_sl | k_sb | k_sh | k_sl | v_sb | v_sh | v_sl | o_sb | o_sl | o_sh;
  FB_CHECK_ARG((align & 15) == 0 && (strides & 7) == 0,
               "prefill_attn: q/k/v/out must be 16-byte aligned with strides that are multiples of 8 elements");
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
    if (e != cudaSuccess) {
      fbh::set_msg("prefill_attn: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = 1;
  }
  PFArgs a{};
  int rc = fbh::tmap_heads(&a.tq, q, B, NH, L, (long long)q_sl, (long long)q_sh, (long long)q_sb);
  if (rc == FB_OK) rc = fbh::tmap_heads(&a.tk, k, B, NKV, S, (long long)k_sl, (long long)k_sh, (long long)k_sb);
  if (rc == FB_OK) rc = fbh::tmap_heads(&a.tv, v, B, NKV, S, (long long)v_sl, (long long)v_sh, (long long)v_sb);
  if (rc != FB_OK) return rc;
  a.q = (const bf16*)q; a.k = (const bf16*)k; a.v = (const bf16*)v;
  a.q_sb = (long)q_sb; a.q_sh = (long)q_sh; a.q_sl = (long)q_sl;
  a.k_sb = (long)k_sb; a.k_sh = (long)k_sh; a.k_sl = (long)k_sl;
  a.v_sb = (long)v_sb; a.v_sh = (long)v_sh; a.v_sl = (long)v_sl;
  a.mask = mask; a.mask_bf16 = mask_is_bf16; a.m_sb = (long)m_sb; a.m_sl = (long)m_sl;
  a.out = (bf16*)out; a.o_sb = (long)o_sb; a.o_sl = (long)o_sl; a.o_sh = (long)o_sh;
  a.B = B; a.NH = NH; a.NKV = NKV; a.L = L; a.S = S; a.h0 = h0; a.causal = causal; a.scaling = scaling;
  a.t0 = tile0;
  a.err = fbh::device_err_ptr();
  void* args[] = {(void*)&a};
  const dim3 grid(tile1 - tile0, h1 - h0, B);
  cudaError_t e = cudaLaunchKernel((const void*)prefill_attn_kernel, grid, dim3(PF_THREADS), args, PF_SMEM,
                                   (cudaStream_t)stream);
  if (e != cudaSuccess) {
    fbh::set_msg("prefill_attn launch: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

extern "C" int flashb_prefill_attn(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sl, const void* k,
                                   int64_t k_sb, int64_t k_sh, int64_t k_sl, const void* v, int64_t v_sb,
                                   int64_t v_sh, int64_t v_sl, const void* mask, int mask_is_bf16, int64_t m_sb,
                                   int64_t m_sl, int B, int NH, int NKV, int L, int S, int D, float scaling,
                                   int causal, int h0, int h1, void* out, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                                   void* stream) {
  const int ntile = L >= 1 ? (L + PF_TILE - 1) / PF_TILE : 1;
  return flashb_prefill_attn_tiles(q, q_sb, q_sh, q_sl, k, k_sb, k_sh, k_sl, v, v_sb, v_sh, v_sl, mask, mask_is_bf16,
                                   m_sb, m_sl, B, NH, NKV, L, S, D, scaling, causal, h0, h1, 0, ntile, out, o_sb,
                                   o_sl, o_sh, stream);
}


// ------------------------------------------------------------------------------------------------ prefill q|k|v tail
// The attention's projection tail for every prompt token, as transformers Qwen3Attention.forward runs it inside the
// reference prefill (BackbonePrefillGraphCache._forward, UP/models/cudagraph/backbone_prefill_graph.py:95-112):
// q = RoPE(q_norm(q)), k = RoPE(k_norm(k)) at the token's position, then the StaticCache update at cache_position
// (keys[:, :, cache_position] = k, values likewise).  One warp per (token, head) of the q|k|v GEMM output, in the
// rotary-pair view of fb_norm.cuh: q heads are rewritten in place (the attention reads them there), k heads go to
// the key cache, v heads are copied to the value cache.  Positions outside the rotary tables and cache slots outside
// the cache are skipped (the host checks the shapes; the device never writes out of bounds).
namespace fb {

struct PQArgs {
  bf16* qkv;
  long ldq;
  int B, L, NH, NKV;
  const bf16 *qn_w, *kn_w;
  float eps;
  const bf16 *cos_tab, *sin_tab;
  int P;
  const long long *pos, *slot;
  bf16 *kc, *vc;
  long c_sb, c_sh;
  int S;
};

__global__ void __launch_bounds__(256) prefill_qkv_kernel(const PQArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int HH = a.NH + 2 * a.NKV;
  const long w = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (long)a.B * a.L * HH) return;
  const int t = (int)(w / HH), h = (int)(w - (long)t * HH);
  const int b = t / a.L, l = t - b * a.L;
  bf16* x = a.qkv + (size_t)t * a.ldq + (size_t)h * 128;
  const long long slot = a.slot[l];
  if (h >= a.NH + a.NKV) {                                 // v head: copy to the value cache
    if (slot < 0 || slot >= a.S) return;
    const int j = h - a.NH - a.NKV;
    bf16* dst = a.vc + (size_t)b * a.c_sb + (size_t)j * a.c_sh + (size_t)slot * 128;
    reinterpret_cast<uint2*>(dst)[lane] = reinterpret_cast<const uint2*>(x)[lane];
    return;
  }
  const long long p = a.pos[(size_t)b * a.L + l];
  if (p < 0 || p >= a.P) return;
  const bool is_q = h < a.NH;
  const HeadPair wv = head_load(is_q ? a.qn_w : a.kn_w, lane);
  const HeadPair cs = head_load(a.cos_tab + (size_t)p * 128, lane);
  const HeadPair sn = head_load(a.sin_tab + (size_t)p * 128, lane);
  const HeadPair y = head_norm_rope(x, wv, cs, sn, a.eps, lane);
  if (is_q) {
    head_store(x, y, lane);
  } else if (slot >= 0 && slot < a.S) {
    head_store(a.kc + (size_t)b * a.c_sb + (size_t)(h - a.NH) * a.c_sh + (size_t)slot * 128, y, lane);
  }
}

}  // namespace fb

extern "C" int flashb_prefill_qkv(void* qkv, int64_t ldq, int B, int L, int NH, int NKV, const void* qn_w,
                                  const void* kn_w, float eps, const void* cos_tab, const void* sin_tab, int P,
                                  const int64_t* position_ids, const int64_t* cache_position, void* kc, void* vc,
                                  int64_t c_sb, int64_t c_sh, int S, void* stream) {
  FB_CHECK_ARG(qkv && qn_w && kn_w && cos_tab && sin_tab && position_ids && cache_position && kc && vc,
               "prefill_qkv: null pointer argument");
  FB_CHECK_ARG(B >= 1 && L >= 1 && NH >= 1 && NKV >= 1 && NH % NKV == 0 && P >= 1 && S >= 1,
               "prefill_qkv: bad shape B=%d L=%d NH=%d NKV=%d P=%d S=%d", B, L, NH, NKV, P, S);
  FB_CHECK_ARG(ldq >= (int64_t)(NH + 2 * NKV) * 128 && ldq % 8 == 0 && c_sh >= (int64_t)S * 128 &&
                   c_sb >= (int64_t)NKV * c_sh && ((uintptr_t)qkv & 15) == 0 && ((uintptr_t)kc & 15) == 0 &&
                   ((uintptr_t)vc & 15) == 0,
               "prefill_qkv: bad strides or alignment");
  fb::PQArgs a{};
  a.qkv = (bf16*)qkv; a.ldq = (long)ldq; a.B = B; a.L = L; a.NH = NH; a.NKV = NKV;
  a.qn_w = (const bf16*)qn_w; a.kn_w = (const bf16*)kn_w; a.eps = eps;
  a.cos_tab = (const bf16*)cos_tab; a.sin_tab = (const bf16*)sin_tab; a.P = P;
  a.pos = (const long long*)position_ids; a.slot = (const long long*)cache_position;
  a.kc = (bf16*)kc; a.vc = (bf16*)vc; a.c_sb = (long)c_sb; a.c_sh = (long)c_sh; a.S = S;
  const long warps = (long)B * L * (NH + 2 * NKV);
  void* args[] = {(void*)&a};
  return fbh::launch_pdl((const void*)fb::prefill_qkv_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0,
                         (cudaStream_t)stream, args, true);
}
