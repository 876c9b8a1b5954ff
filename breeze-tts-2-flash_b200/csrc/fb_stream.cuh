// flashb: the weight-streaming GEMV core shared by the standalone GEMV kernels and the persistent step kernels.
//
// A skinny GEMV y[m, n] = sum_k x[m, k] W[n, k] (M <= 8 activation rows) is an HBM stream of W.  The core splits
// the work into stages of 16 weight rows x 2048 columns (64 KB):
//   * a producer warp moves each row slice into a shared-memory ring with one 1-D bulk copy (cp.async.bulk, the TMA
//     engine; no tensor map, no multicast) completing on the stage's mbarrier.  Rows sit at a 4112-byte pitch (one
//     16-byte pad per row) so that ldmatrix reads of 8 consecutive rows fall in distinct banks.  Measured on B200:
//     the per-SM rate is set by the consumers' per-stage overhead, so stages are large (64 KB stages stream a
//     400 MB matrix at 6.4 TB/s; 32 KB stages at 4.9 TB/s; a 16-byte cp.async staging variant at 2.3 TB/s);
//   * 8 consumer warps split the stage's 64 k-steps; each k-step is one tensor-core mma.sync m16n8k16
//     (bf16 x bf16 -> fp32): A = 16 weight rows x 16 columns via ldmatrix.x4, B = the 8-row activation tile (rows
//     >= M read a zero block) via ldmatrix.x2.  One mma replaces 256 scalar FMAs plus their bf16 unpacking, so the
//     consumer issue rate stays far below the HBM rate even with one CTA per SM;
//   * at the end of a row group the 8 warps' fp32 accumulators are summed in shared memory in a fixed order
//     (deterministic), and a task-specific epilogue turns the 16 x M sums into outputs.
// Both sides walk the same static stage sequence, so the producer runs ahead of the consumers by the ring depth,
// across task boundaries and grid barriers (weights never depend on activations).
#pragma once
#include "fb_norm.cuh"

// The stage width (FB_ST_KC, default 2048 columns) and the stage layout (FB_ST_TMA) are per-translation-unit
// choices; everything that depends on them lives in an inline namespace named after them, so units built
// differently never share a definition.
//   FB_ST_TMA 0: each of the 16 rows arrives by its own 1-D bulk copy at a padded pitch (ST_KC * 2 + 16 bytes).
//   FB_ST_TMA 1: two TMA tensor copies per stage (cp.async.bulk.tensor.3d, a tensor map per weight matrix viewed as
//     [K / 64 column blocks][rows][64 columns]), each bringing 8 rows x ST_KC columns as [ST_KC / 64][8 rows][128 B]
//     with the 128-byte swizzle (16-byte unit j of row r lands at unit j ^ (r % 8)), so ldmatrix reads of 8 rows
//     hit 8 distinct bank groups without padding.  Measured on B200, one SM streams 82 GB/s with two such copies
//     per 32 KB stage and 154 GB/s per 64 KB stage, against 47 and 92 GB/s with 16 row copies: the TMA engine's
//     per-copy cost, not the bytes, bounds a ring of row copies.
#ifndef FB_ST_KC
#define FB_ST_KC 2048
#endif
#ifndef FB_ST_TMA
#define FB_ST_TMA 0
#endif
#define FB_ST_NS_CAT2(a, b) a##b
#define FB_ST_NS_CAT(a, b) FB_ST_NS_CAT2(a, b)
#if FB_ST_TMA
#define FB_ST_NS FB_ST_NS_CAT(FB_ST_NS_CAT(kc, FB_ST_KC), t)
#else
#define FB_ST_NS FB_ST_NS_CAT(kc, FB_ST_KC)
#endif

namespace fb {
inline namespace FB_ST_NS {

constexpr int ST_ROWS = 16;                       // weight rows per stage (one mma M tile)
constexpr int ST_KC = FB_ST_KC;                   // columns per stage
#if FB_ST_TMA
constexpr int ST_PITCH = 128;                     // bytes per row within a 64-column block
constexpr int ST_BYTES = ST_ROWS * ST_KC * 2;     // 65536 bytes per stage at 2048 columns
constexpr int ST_HALF = ST_BYTES / 2;             // rows 8..15 start here
constexpr int ST_ALIGN = 1024;                    // stage alignment the 128-byte swizzle pattern assumes
#else
constexpr int ST_PITCH = ST_KC * 2 + 16;          // bytes per staged row
constexpr int ST_BYTES = ST_ROWS * ST_PITCH;      // 65792 bytes per stage at 2048 columns
constexpr int ST_ALIGN = 128;
#endif
constexpr int ST_CWARPS = 8;                      // consumer warps
constexpr int ST_KSTEPS_PER_WARP = ST_KC / 16 / ST_CWARPS;  // 16 at 2048 columns

// ldmatrix.x4 row address of the A fragment: lane l supplies row (l % 8) + 8 * ((l / 8) % 2), columns
// 16 ks + 8 (l / 16) .. + 7 of the stage.  a_base() is the per-lane part for the warp's first k-step ks0 (a
// multiple of 4), a_addr() adds k-step ks0 + i; with i a compile-time constant the swizzle terms are 4 per-lane
// values the compiler keeps in registers.
__device__ __forceinline__ uint32_t a_base(const unsigned char* stage, int lane, int ks0) {
#if FB_ST_TMA
  return smem_u32(stage) + ((lane >> 3) & 1) * ST_HALF + (lane & 7) * 128 + ((ks0 >> 2) << 10);
#else
  return smem_u32(stage) + ((lane & 7) + ((lane >> 3) & 1) * 8) * ST_PITCH + (lane >> 4) * 16 + ks0 * 32;
#endif
}
__device__ __forceinline__ uint32_t a_addr(uint32_t abase, int i, int lane) {
#if FB_ST_TMA
  return abase + ((i >> 2) << 10) + (((((i & 3) << 1) | (lane >> 4)) ^ (lane & 7)) << 4);
#else
  return abase + i * 32;
#endif
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Consumer side of one stage: this warp's share of the k-steps of a [16 x kw] weight tile against the activation
// rows xs (M rows at byte pitch x_pitch, columns k0.. of the full K), accumulated into the C fragment c:
// c[0], c[1] = rows lane/4, activation rows (lane%4)*2 + {0,1}; c[2], c[3] = rows lane/4 + 8, same columns.
__device__ __forceinline__ void stage_mma(const unsigned char* stage, int kw, const unsigned char* xs, int x_pitch,
                                          int M, int k0, const unsigned char* zero16, float (&c)[4]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nks = kw >> 4;
  const int ks0 = warp * ST_KSTEPS_PER_WARP;
  const int ks1 = min(nks, ks0 + ST_KSTEPS_PER_WARP);
  const uint32_t abase = a_base(stage, lane, ks0);
  // B: lanes 0-7 supply activation row n = lane at column offset 0, lanes 8-15 row lane-8 at offset 8
  const int bn = lane & 7;
  const bool breal = bn < M && lane < 16;
  const uint32_t bbase = breal ? smem_u32(xs) + bn * x_pitch + (size_t)k0 * 2 + ((lane >> 3) & 1) * 16 : smem_u32(zero16);
  const uint32_t bstep = breal ? 32u : 0u;
#ifndef FB_MMA_NACC
#define FB_MMA_NACC 4
#endif
#if FB_MMA_NACC > 1
  // independent accumulator chains (one mma latency per NACC k-steps), summed at the end in a fixed order
  float cc[FB_MMA_NACC][4];
#pragma unroll
  for (int i = 0; i < FB_MMA_NACC; ++i) cc[i][0] = cc[i][1] = cc[i][2] = cc[i][3] = 0.f;
#pragma unroll
  for (int i = 0; i < ST_KSTEPS_PER_WARP; ++i) {
    const int ks = ks0 + i;
    if (ks < ks1) {
      uint32_t a0, a1, a2, a3, b0, b1;
      ldsm_x4(a_addr(abase, i, lane), a0, a1, a2, a3);
      ldsm_x2(bbase + ks * bstep, b0, b1);
      mma_bf16_16816(cc[i % FB_MMA_NACC], a0, a1, a2, a3, b0, b1);
    }
  }
#pragma unroll
  for (int i = 0; i < FB_MMA_NACC; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j] += cc[i][j];
#else
#pragma unroll 4
  for (int ks = ks0; ks < ks1; ++ks) {
    uint32_t a0, a1, a2, a3, b0, b1;
    ldsm_x4(a_addr(abase, ks - ks0, lane), a0, a1, a2, a3);
    ldsm_x2(bbase + ks * bstep, b0, b1);
    mma_bf16_16816(c, a0, a1, a2, a3, b0, b1);
  }
#endif
}

// Sum the 8 warps' C fragments (fixed order) into sums[16][8] (shared).  Called by all 256 consumer threads.
__device__ __forceinline__ void reduce_warps(const float (&c)[4], float* red /* [8][16][8] */, float* sums /* [16][8] */,
                                             int bar_id) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, m = (lane & 3) * 2;
  float* w = red + warp * 128;
  w[r * 8 + m] = c[0];
  w[r * 8 + m + 1] = c[1];
  w[(r + 8) * 8 + m] = c[2];
  w[(r + 8) * 8 + m + 1] = c[3];
  named_sync(bar_id, ST_CWARPS * 32);
  if (threadIdx.x < 128) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < ST_CWARPS; ++i) s += red[i * 128 + threadIdx.x];
    sums[threadIdx.x] = s;
  }
  named_sync(bar_id, ST_CWARPS * 32);
}

// NT tiles of 8 activation rows (M <= 8 NT): each k-step's weight fragment (ldmatrix.x4) is loaded once and
// multiplied by every tile's activation fragment; tile t covers activation rows 8t .. 8t+7 (rows >= M read zeros).
// Two independent accumulator chains per tile, summed at the end in a fixed order.
template <int NT>
__device__ __forceinline__ void stage_mma_nt(const unsigned char* stage, int kw, const unsigned char* xs, int x_pitch,
                                             int M, int k0, const unsigned char* zero16, float (&c)[NT][4]) {
  if constexpr (NT == 1) {
    stage_mma(stage, kw, xs, x_pitch, M, k0, zero16, c[0]);
  } else {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nks = kw >> 4;
    const int ks0 = warp * ST_KSTEPS_PER_WARP;
    const int ks1 = min(nks, ks0 + ST_KSTEPS_PER_WARP);
    const uint32_t abase = a_base(stage, lane, ks0);
    const int bn = lane & 7;
    uint32_t bbase[NT], bstep[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const bool breal = bn + 8 * t < M && lane < 16;
      bbase[t] = breal ? smem_u32(xs) + (bn + 8 * t) * x_pitch + (size_t)k0 * 2 + ((lane >> 3) & 1) * 16
                       : smem_u32(zero16);
      bstep[t] = breal ? 32u : 0u;
    }
    float cc[2][NT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int t = 0; t < NT; ++t) cc[h][t][0] = cc[h][t][1] = cc[h][t][2] = cc[h][t][3] = 0.f;
#pragma unroll
    for (int i = 0; i < ST_KSTEPS_PER_WARP; ++i) {
      const int ks = ks0 + i;
      if (ks < ks1) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a_addr(abase, i, lane), a0, a1, a2, a3);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          uint32_t b0, b1;
          ldsm_x2(bbase[t] + ks * bstep[t], b0, b1);
          mma_bf16_16816(cc[i & 1][t], a0, a1, a2, a3, b0, b1);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int j = 0; j < 4; ++j) c[t][j] += cc[0][t][j] + cc[1][t][j];
  }
}

// Sum the 8 warps' fragments of NT tiles (fixed order) into sums[16][8 NT] (row r, activation row m at
// sums[r * 8 NT + m]).  red holds [8 warps][16][8 NT] floats.  Called by all 256 consumer threads.
template <int NT>
__device__ __forceinline__ void reduce_warps_nt(const float (&c)[NT][4], float* red, float* sums, int bar_id) {
  if constexpr (NT == 1) {
    reduce_warps(c[0], red, sums, bar_id);
  } else {
    constexpr int MS = 8 * NT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, m = (lane & 3) * 2;
    float* w = red + warp * 16 * MS;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      w[r * MS + 8 * t + m] = c[t][0];
      w[r * MS + 8 * t + m + 1] = c[t][1];
      w[(r + 8) * MS + 8 * t + m] = c[t][2];
      w[(r + 8) * MS + 8 * t + m + 1] = c[t][3];
    }
    named_sync(bar_id, ST_CWARPS * 32);
    for (int i = threadIdx.x; i < 16 * MS; i += ST_CWARPS * 32) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < ST_CWARPS; ++k) s += red[k * 16 * MS + i];
      sums[i] = s;
    }
    named_sync(bar_id, ST_CWARPS * 32);
  }
}

__device__ __forceinline__ void cp_async_wait_dyn(int n) {  // n in [0, 7]
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}

#if !FB_ST_TMA
// Stage load by all `nthreads` consumer threads: rows[i] (i < nrows) -> stage row i, columns [0, kw) (kw % 8 == 0).
// 16-byte chunks are spread across threads so consecutive threads read consecutive chunks of a row.
template <typename RowFn>
__device__ __forceinline__ void stage_load(unsigned char* stage, int nrows, int kw, int tid, int nthreads,
                                           RowFn row) {
  const int cpr = kw >> 3;  // 16-byte chunks per row
  const int total = nrows * cpr;
  for (int c = tid; c < total; c += nthreads) {
    const int r = c / cpr, j = c - r * cpr;
    const bf16* src = row(r);
    if (src) cp_async16(stage + r * ST_PITCH + j * 16, src + j * 8);
  }
}
#endif

#if FB_ST_TMA
// One TMA tensor copy of a 3-D box (coordinates c0 innermost) into shared memory, completing on bar.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
// Pull a tensor map into the TMA unit's descriptor cache ahead of its first copy.
__device__ __forceinline__ void tma_prefetch_map(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Source of 8 stage rows: rows row .. row + 7 of the matrix behind tensor map `map` (nullptr: nothing to load).
struct TmaRows {
  const void* map;
  int row;
};
// Stage s <- column chunk kc (ST_KC columns) of two 8-row sources (rows 0..7, rows 8..15).  Issued by one thread.
__device__ __forceinline__ void tma_stage(unsigned char* stage, TmaRows lo, TmaRows hi, int kc, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, (unsigned)((lo.map ? ST_HALF : 0) + (hi.map ? ST_HALF : 0)));
  if (lo.map) tma_load_3d(stage, lo.map, 0, lo.row, kc * (ST_KC / 64), bar);
  if (hi.map) tma_load_3d(stage + ST_HALF, hi.map, 0, hi.row, kc * (ST_KC / 64), bar);
}
#endif

}  // inline namespace
}  // namespace fb
