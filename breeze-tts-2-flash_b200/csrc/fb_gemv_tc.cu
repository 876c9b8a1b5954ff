// flashb: skinny GEMV / small GEMM on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), for up to
// 128 activation rows and K % 64 == 0.  Same semantics as the mma.sync kernel of fb_gemv_core.cuh (see fb_gemv.cu):
//   y[m, n] = sum_k xin[m, k] W[n, k] (fp32), NORM: xin = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))),
//   EPI 0: bf16(acc)   EPI 1: bf16(res + bf16(acc))   EPI 2: bf16(bf16(silu(bf16(acc_gate))) * bf16(acc_up)).
//
// B200 design.  The GEMV is turned around so that the weights are the MMA's M side: D[128 weight rows x MT] +=
// W[128 x 16 k] . x^T[16 k x MT activation rows] (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = MT, K = 16), MT
// = the activation rows rounded up to 16, 32, 64 or 128, rows >= M being zeros.  More rows than MT form row groups
// (blockIdx.y): each group is the same GEMV over MT rows on its share of the grid, and the groups, launched together,
// stream each weight tile from HBM about once and from L2 for the others.  A CTA owns whole blocks of 128 output
// units and walks K in stages:
//   * warp 0 (one lane) streams each stage with TMA tensor copies in the canonical K-major 128-byte-swizzle operand
//     layout (8-row groups 1024 B apart): EPI 0/1 one 128-row x 128-column box of W; EPI 2 one 128-row x 64-column
//     box of the gate rows and one of the up rows; plus the activation tile x[MT rows x the stage's columns] in the
//     same layout.  One large box per matrix and stage matters: measured on B200, one SM streams 93 GB/s with a
//     128 x 128 box per 32 KB stage, 67 GB/s with four 64 x 64 boxes, 35 GB/s with 8-row boxes.  Weights are
//     independent of the previous kernel, so the first ring's worth of weight copies is issued before
//     griddepcontrol.wait, the activation copies after;
//   * warp 1 (one lane) issues the stage's MMAs (EPI 2: gate and up into two accumulators, so that a unit's gate
//     and up sums land in the same TMEM lane) and commits them to the stage's "empty" barrier (the ring slot is
//     free once the tensor core has read it) and, after a block's last stage, to the block's accumulator barrier.
//     The accumulators are double-buffered in TMEM, so block i + 1 accumulates while the epilogue of block i runs.
//     With few activation rows (N = 16 or 32) consecutive k-steps go to independent accumulator chains, summed in a
//     fixed order in the epilogue: a single chain of small dependent MMAs kept every ring slot busy about twice as
//     long (measured);
//   * warps 2-5 (one TMEM lane quarter each) read a block's accumulators (tcgen05.ld 32x32b.x16: row = lane,
//     16 activation columns at a time), release them, and write the outputs.  With NORM they first rescale every
//     activation tile in shared memory (the RMS factors of the M rows are computed once per CTA) and hand it to the
//     MMA warp through a second barrier.
// Split K (a matrix with too few 128-row blocks to fill the grid, e.g. 16 blocks on 148 SMs): the grid becomes one
// thread-block cluster of S <= 8 CTAs per block, CTA r of a cluster takes the r-th of S column ranges, and the S
// partial sums meet through distributed shared memory: every CTA copies its fp32 accumulators into its own (now
// idle) ring, a cluster barrier, then CTA r sums units [128 r / S, 128 (r + 1) / S) of the block over the S CTAs in
// rank order (deterministic) and writes them, and a second cluster barrier keeps every CTA's shared memory alive
// until its peers have read it.  No global workspace, no atomics, no second launch.
// There is no cross-warp reduction and no mma.sync: one thread drives the tensor core, the fp32 sums stay in TMEM
// across the whole K loop.  Every wait is bounded (fb_common.cuh); on expiry the error word is set and the CTA
// winds down (the producer waits for its own copies, the cluster barriers are still reached, the TMEM is freed).
#define FB_ST_TMA 1
#include <cooperative_groups.h>

#include <cstdlib>

#include "fb_gemv_core.cuh"
#include "fb_tc.cuh"

namespace cg = cooperative_groups;

namespace fb {
namespace {

constexpr int TC_BR = 128;                      // output units per block (the MMA's M)
constexpr int TC_WBYTES = 32768;                // weight tile per stage: 128 rows x 128 columns (EPI 2: x 2 x 64)
// columns per stage: 128, or 64 for EPI 2 (gate and up tiles share the stage)
template <int EPI>
constexpr int tc_cols() { return EPI == 2 ? 64 : 128; }
template <int EPI, int MT>
constexpr int tc_xbytes() { return MT * tc_cols<EPI>() * 2; }    // activation tile per stage
// independent accumulator chains per matrix
template <int EPI, int MT>
constexpr int tc_nch() { return EPI == 2 ? (MT == 16 ? 2 : 1) : (MT == 16 ? 4 : (MT == 32 ? 2 : 1)); }
// TMEM columns of one accumulator buffer (x 2 buffers; at most 256)
template <int EPI, int MT>
constexpr int tc_dcols() { return (EPI == 2 ? 2 : 1) * tc_nch<EPI, MT>() * MT; }
// split K: row pitch (floats) of the partial sums [unit][MT (+ MT up)]: 16-byte rows, and 4 banks apart so that
// a warp's float4 writes of 32 rows are conflict-free
template <int EPI, int MT>
constexpr int tc_rp() { return (EPI == 2 ? 2 : 1) * MT + 4; }
constexpr int TC_MAX_STAGES = 6;
constexpr int TC_MAX_SPLIT = 8;                 // CTAs per cluster (portable cluster size)
constexpr int TC_THREADS = 6 * 32;
constexpr int TC_EPI_THREADS = 4 * 32;

// Split phases of a cluster barrier (every thread of every CTA of the cluster arrives once per phase, then waits).
__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

struct alignas(64) TcArgs {
  CUtensorMap tw[3];   // weight segments (EPI 2: gate, up) as [K / 64][rows][64], boxes of 128 rows x the stage
  CUtensorMap tx;      // x [M, K] as [K / 64][M][64], one box = MT rows x the stage (both 128-byte swizzle)
  const bf16* x;
  long ldx;
  const bf16* nw;
  float eps;
  int N0, N1, N, K, M;
  bf16* y;
  long ldy;
  const bf16* res;
  long ldr;
  int nst;
  int split;           // CTAs per cluster sharing one block's K range (1: no split)
  unsigned* err;
  unsigned long long* trace;   // optional per-CTA timeline (TC_TRACE_SLOTS %globaltimer stamps), or null
};

// Optional timeline of one launch: CTA c (blockIdx.y * gridDim.x + blockIdx.x) writes TC_TRACE_SLOTS values at
// trace[c * TC_TRACE_SLOTS]: entry, producer past griddepcontrol.wait, first stage in (MMA warp), last MMA committed,
// epilogue done, split-K reduction done, exit (ns), and the SM id.
constexpr int TC_TRACE_SLOTS = 8;
#define TC_STAMP(i)                                                                                         \
  do {                                                                                                      \
    if (a.trace) a.trace[(blockIdx.y * gridDim.x + blockIdx.x) * TC_TRACE_SLOTS + (i)] = globaltimer();   \
  } while (0)

// Tensor map and first row of 128 weight rows starting at block row r (EPI 0/1: segments are multiples of 128).
// Rows past the last row stay with the last segment (an out-of-range box reads zeros), never with an empty one.
__device__ __forceinline__ TmaRows tc_rows(const TcArgs& a, int r) {
  const int n2 = a.N - a.N0 - a.N1;
  if (r < a.N0 || (a.N1 == 0 && n2 == 0)) return TmaRows{&a.tw[0], r};
  if (r < a.N0 + a.N1 || n2 == 0) return TmaRows{&a.tw[1], r - a.N0};
  return TmaRows{&a.tw[2], r - a.N0 - a.N1};
}

// The epilogue of one output: fp32 sum(s) -> the output value of unit n, row m (before the bf16 store).
template <int EPI>
__device__ __forceinline__ float tc_out(const TcArgs& a, float v, float u, int m, int n) {
  if (EPI == 2) {
    const float gg = rbf(v);
    return silu_rbf(gg) * rbf(u);
  }
  if (EPI == 1) return b2f(a.res[(size_t)m * a.ldr + n]) + rbf(v);
  return v;
}

template <int EPI, bool NORM, int MT>
__global__ void __launch_bounds__(TC_THREADS, 1) gemv_tc_kernel(const __grid_constant__ TcArgs a) {
  constexpr int TC_C = tc_cols<EPI>();
  constexpr int XB = tc_xbytes<EPI, MT>();
  constexpr int UB = TC_BR;                           // output units per block
  constexpr int NCH = tc_nch<EPI, MT>();
  constexpr int DCOLS = tc_dcols<EPI, MT>();          // TMEM columns per accumulator buffer (x 2 buffers)
  constexpr int RP = tc_rp<EPI, MT>();
  constexpr uint32_t IDESC = tc_idesc(MT);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = a.nst;
  unsigned char* wring = smem;                                   // [NST][TC_WBYTES], 1024-aligned
  unsigned char* xring = smem + (size_t)NST * TC_WBYTES;         // [NST][XB]
  uint64_t* full = reinterpret_cast<uint64_t*>(xring + (size_t)NST * XB);
  uint64_t* empty = full + TC_MAX_STAGES;
  uint64_t* xok = empty + TC_MAX_STAGES;
  uint64_t* dfull = xok + TC_MAX_STAGES;                          // [2]
  uint64_t* dempty = dfull + 2;                                   // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dempty + 2);
  float* rs = reinterpret_cast<float*>(tslot + 4);                // [MT] RMS factors
  float* psum = rs + MT;                                          // [MT] sums of squares (split K: this CTA's)
  float* red = reinterpret_cast<float*>(smem);                    // split K: partial sums, over the idle ring

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) TC_STAMP(0);
  // row group blockIdx.y: activation rows [r0, r0 + M) of the launch's a.M
  const int r0 = blockIdx.y * MT;
  const int K = a.K, M = min(MT, a.M - r0);
  const int nkc_all = (K + TC_C - 1) / TC_C;
  const int units = a.N;
  const int nb_all = (units + UB - 1) / UB;
  // split K: cluster c takes block c and its rank r the r-th column range; else CTA c takes blocks [b0, b1)
  const int S = a.split;
  const int rank = (int)(blockIdx.x % S);
  const int nclu = gridDim.x / S;
  const int cid = blockIdx.x / S;
  const int b0 = (int)((long long)nb_all * cid / nclu);
  const int b1 = (int)((long long)nb_all * (cid + 1) / nclu);
  const int kc0 = (int)((long long)nkc_all * rank / S);
  const int nkc = (int)((long long)nkc_all * (rank + 1) / S) - kc0;
  const int nblk = b1 - b0;
  const int T = nblk * nkc;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&xok[s], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tc_alloc(tslot, 2 * DCOLS);
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  // split K, phase 0 of the cluster barrier: with NORM the epilogue warps exchange the RMS partial sums of their K
  // ranges; every other thread arrives now and waits at the end
  const bool early = S > 1 && !(NORM && warp >= 2);
  if (early) cl_arrive();

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    int issued = 0;
    auto issue_w = [&](int t) {
      const int s = t % NST, kc = kc0 + t % nkc, blk = b0 + t / nkc;
      unsigned char* wt = wring + (size_t)s * TC_WBYTES;
      if (EPI == 2) {
        // [gate 128 rows x 128 B][up 128 rows x 128 B]
        tma_load_3d(wt, &a.tw[0], 0, blk * UB, kc, &full[s]);
        tma_load_3d(wt + TC_BR * 128, &a.tw[1], 0, blk * UB, kc, &full[s]);
      } else {
        // [2 column blocks][128 rows x 128 B]
        const TmaRows h = tc_rows(a, blk * TC_BR);
        tma_load_3d(wt, h.map, 0, h.row, kc * 2, &full[s]);
      }
    };
    auto issue_x = [&](int t) {
      const int s = t % NST, kc = kc0 + t % nkc;
      tma_load_3d(xring + (size_t)s * XB, &a.tx, 0, r0, kc * (TC_C / 64), &full[s]);
    };
    constexpr unsigned STAGE_TX = (unsigned)(TC_WBYTES + XB);
    if (lane < 4) tma_prefetch_map(lane < 3 ? (const void*)&a.tw[lane] : (const void*)&a.tx);
    bool ok = true;
    const int pre = min(T, NST);
    if (lane == 0) {
      for (int t = 0; t < pre; ++t) {       // weights of the first ring's worth, before the previous kernel ends
        mbar_arrive_expect_tx(&full[t], STAGE_TX);
        issue_w(t);
      }
    }
    __syncwarp();
    issued = pre;
    pdl_wait();
    if (lane == 0) TC_STAMP(1);
    if (lane == 0)
      for (int t = 0; t < pre; ++t) issue_x(t);
    __syncwarp();
    for (int t = pre; t < T && ok; ++t) {
      const int s = t % NST;
      if (!mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1, a.err)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], STAGE_TX);
        issue_w(t);
        issue_x(t);
      }
      __syncwarp();
      issued = t + 1;
    }
    // never leave with copies in flight into this CTA's shared memory
    for (int t = max(0, issued - NST); t < issued; ++t)
      if (!mbar_wait_warp(&full[t % NST], (t / NST) & 1, a.err)) break;
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue (one lane)
    bool ok = true;
    int committed = -1;
    for (int i = 0; i < nblk && ok; ++i) {
      const uint32_t td = tmem + (uint32_t)((i & 1) * DCOLS);
      if (i >= 2 && !mbar_wait_warp(&dempty[i & 1], ((i >> 1) - 1) & 1, a.err)) {
        ok = false;
        break;
      }
      for (int kc = 0; kc < nkc; ++kc) {
        const int t = i * nkc + kc, s = t % NST;
        if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err) ||
            (NORM && !mbar_wait_warp(&xok[s], (t / NST) & 1, a.err))) {
          ok = false;
          break;
        }
        tc_after();
        if (lane == 0 && t == 0) TC_STAMP(2);
        if (lane == 0) {
          // descriptors as base + offset in 16-byte units (one add per MMA)
          const uint64_t wd = tc_desc_sw128(smem_u32(wring + (size_t)s * TC_WBYTES));
          const uint64_t xd = tc_desc_sw128(smem_u32(xring + (size_t)s * XB));
#pragma unroll
          for (int j = 0; j < TC_C / 16; ++j) {
            const uint64_t bd = xd + (uint64_t)((j >> 2) * (MT * 128 / 16) + ((j & 3) << 1));
            const uint32_t acc = (kc > 0 || j >= NCH) ? 1u : 0u;
            const uint32_t ch = (uint32_t)((j % NCH) * MT);
            if (EPI == 2) {
              // gate chains in columns [0, NCH MT), up chains in [NCH MT, 2 NCH MT)
              tc_mma(td + ch, wd + (uint64_t)((j & 3) << 1), bd, acc, IDESC);
              tc_mma(td + NCH * MT + ch, wd + (uint64_t)(TC_BR * 128 / 16 + ((j & 3) << 1)), bd, acc, IDESC);
            } else {
              tc_mma(td + ch, wd + (uint64_t)((j >> 2) * (TC_BR * 128 / 16) + ((j & 3) << 1)), bd, acc, IDESC);
            }
          }
          tc_commit(&empty[s]);
          if (kc == nkc - 1) tc_commit(&dfull[i & 1]);
        }
        __syncwarp();
        committed = t;
      }
    }
    if (lane == 0) TC_STAMP(3);
    // the ring's last slots must not be overwritten by a later CTA while the tensor core still reads them
    if (committed >= 0) mbar_wait_warp(&empty[committed % NST], (committed / NST) & 1, a.err);
  } else {
    // ------------------------------------------------------------------ epilogue (and NORM rescaling) warps
    const int q = warp & 3;              // TMEM lane quarter
    const int etid = tid - 64;           // 0..127
    const int row = q * 32 + lane;       // accumulator row of this thread
    pdl_wait();
    pdl_trigger();
    bool ok = true;
    if (NORM) {
      // sums of squares of the rows over their 16-byte chunks [jb, je) -> psum[m]: warp q takes rows q, q + 4, ...,
      // RB of them at a time (RB loads in flight per lane), each lane its chunks in order, then a butterfly
      constexpr int RB = MT / 4 < 8 ? MT / 4 : 8;
      const int jb = S > 1 ? kc0 * TC_C / 8 : 0;
      const int je = S > 1 ? min(K, (kc0 + nkc) * TC_C) / 8 : K / 8;
      for (int i0 = 0; i0 < MT / 4; i0 += RB) {
        float ss[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r) ss[r] = 0.f;
        for (int j = jb + lane; j < je; j += 32) {
          uint4 v[RB];
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            const int m = q + 4 * (i0 + r);
            v[r] = m < M ? *reinterpret_cast<const uint4*>(a.x + (size_t)(r0 + m) * a.ldx + (size_t)j * 8)
                         : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            float f[8];
            cvt8(v[r], f);
#pragma unroll
            for (int u = 0; u < 8; ++u) ss[r] = fmaf(f[u], f[u], ss[r]);
          }
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const float t = warp_sum(ss[r]);
          if (lane == 0) psum[q + 4 * (i0 + r)] = t;
        }
      }
      if (S > 1) {
        // the cluster's partial sums, added in rank order
        cl_arrive();
        cl_wait();
        cg::cluster_group cluster = cg::this_cluster();
        for (int m = etid; m < MT; m += TC_EPI_THREADS) {
          float t = 0.f;
          for (int p = 0; p < S; ++p) t += *cluster.map_shared_rank(psum + m, p);
          rs[m] = rms_factor(t, K, a.eps);
        }
      } else {
        __syncwarp();
        for (int m = lane; m < MT; m += 32)
          if ((m & 3) == q) rs[m] = rms_factor(psum[m], K, a.eps);
      }
      named_sync(1, TC_EPI_THREADS);
    }
    auto fix = [&](int t) -> bool {       // rescale stage t's activation tile in place
      const int s = t % NST, kc = kc0 + t % nkc;
      if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err)) return false;
      unsigned char* xt = xring + (size_t)s * XB;
      for (int i = etid; i < XB / 16; i += TC_EPI_THREADS) {
        // [64-column block c][row m][16-byte unit jp], unit jp holding columns 8 (jp ^ (m % 8)) .. of the block
        const int c = i / (MT * 8), m = (i >> 3) % MT, jp = i & 7;
        const int k = kc * TC_C + c * 64 + ((jp ^ (m & 7)) << 3);
        if (m >= M || k >= K) continue;
        uint4* p = reinterpret_cast<uint4*>(xt + (size_t)i * 16);
        *p = rms_unit(*p, *reinterpret_cast<const uint4*>(a.nw + k), rs[m]);
      }
      fence_proxy_async();                 // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&xok[s]);
      return true;
    };
    // activation columns c16 .. c16 + 15 of this thread's row: the chains of matrix mat summed in a fixed order
    auto load16 = [&](uint32_t tq, int mat, int c16, float (&v)[16]) {
      tc_ld16(tq + (uint32_t)(mat * NCH * MT + c16), v);
#pragma unroll
      for (int ch = 1; ch < NCH; ++ch) {
        float c[16];
        tc_ld16(tq + (uint32_t)(mat * NCH * MT + ch * MT + c16), c);
#pragma unroll
        for (int m = 0; m < 16; ++m) v[m] += c[m];
      }
    };
    auto epilogue = [&](int i) -> bool {
      if (!mbar_wait(&dfull[i & 1], (i >> 1) & 1, a.err)) return false;
      tc_after();
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((i & 1) * DCOLS);
      const int n = (b0 + i) * UB + row;
#pragma unroll 1
      for (int c16 = 0; c16 < MT; c16 += 16) {
        float v[16], u[16];
        load16(tq, 0, c16, v);
        if (EPI == 2) load16(tq, 1, c16, u);
        if (n < units) {
#pragma unroll
          for (int m = 0; m < 16; ++m)
            if (c16 + m < M)
              a.y[(size_t)(r0 + c16 + m) * a.ldy + n] =
                  __float2bfloat16_rn(tc_out<EPI>(a, v[m], EPI == 2 ? u[m] : 0.f, r0 + c16 + m, n));
        }
      }
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[i & 1]);
      return true;
    };
    // split K: this CTA's partial sums of its one block -> red[unit][MT (+ MT up)]
    auto dump = [&]() -> bool {
      if (!mbar_wait(&dfull[0], 0, a.err)) return false;
      tc_after();
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c16 = 0; c16 < MT; c16 += 16) {
        float v[16];
        load16(tq, 0, c16, v);
        float4* d = reinterpret_cast<float4*>(red + row * RP + c16);
#pragma unroll
        for (int m = 0; m < 4; ++m) d[m] = make_float4(v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3]);
        if (EPI == 2) {
          load16(tq, 1, c16, v);
          d = reinterpret_cast<float4*>(red + row * RP + MT + c16);
#pragma unroll
          for (int m = 0; m < 4; ++m) d[m] = make_float4(v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3]);
        }
      }
      tc_before();
      return true;
    };
    if (S > 1) {
      if (nblk == 1) {
        if (NORM)
          for (int kc = 0; kc < nkc && ok; ++kc) ok = fix(kc);
        if (ok) ok = dump();
      }
    } else if (NORM) {
      // rescale block i's tiles, then write block i - 1 (its accumulator fills while block i is rescaled)
      for (int i = 0; i < nblk && ok; ++i) {
        for (int kc = 0; kc < nkc && ok; ++kc) ok = fix(i * nkc + kc);
        if (ok && i > 0) ok = epilogue(i - 1);
      }
      if (ok && nblk > 0) ok = epilogue(nblk - 1);
    } else {
      for (int i = 0; i < nblk && ok; ++i) ok = epilogue(i);
    }
  }
  __syncwarp();
  if (tid == 64) TC_STAMP(4);
  if (early) cl_wait();
  if (S > 1) {
    // every thread of every CTA of the cluster reaches both barriers, whatever happened above
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (warp >= 2 && nblk == 1) {
      // unit uu, rows 4 mq .. 4 mq + 3: the S partial sums (all requested together), added in rank order
      const int u0 = UB * rank / S, nu = UB * (rank + 1) / S - u0;
      const int nq = (M + 3) / 4;
      for (int idx = tid - 64; idx < nu * nq; idx += TC_EPI_THREADS) {
        const int mq = idx / nu, uu = u0 + idx % nu;
        const int n = b0 * UB + uu;
        float4 pv[TC_MAX_SPLIT], pu[TC_MAX_SPLIT];
#pragma unroll
        for (int p = 0; p < TC_MAX_SPLIT; ++p)
          if (p < S) {
            const float* rp = cluster.map_shared_rank(red, p) + uu * RP + mq * 4;
            pv[p] = *reinterpret_cast<const float4*>(rp);
            if (EPI == 2) pu[p] = *reinterpret_cast<const float4*>(rp + MT);
          }
        float v[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < TC_MAX_SPLIT; ++p)
          if (p < S) {
            v[0] += pv[p].x; v[1] += pv[p].y; v[2] += pv[p].z; v[3] += pv[p].w;
            if (EPI == 2) {
              u[0] += pu[p].x; u[1] += pu[p].y; u[2] += pu[p].z; u[3] += pu[p].w;
            }
          }
        if (n < units) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int m = mq * 4 + r;
            if (m < M) a.y[(size_t)(r0 + m) * a.ldy + n] = __float2bfloat16_rn(tc_out<EPI>(a, v[r], u[r], r0 + m, n));
          }
        }
      }
    }
    cluster.sync();
  }
  if (tid == 64) TC_STAMP(5);
  tc_before();
  __syncthreads();
  tc_after();
  if (warp == 1) tc_dealloc(tmem, 2 * DCOLS);
  if (tid == 0) {
    TC_STAMP(6);
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    if (a.trace) a.trace[(blockIdx.y * gridDim.x + blockIdx.x) * TC_TRACE_SLOTS + 7] = sm;
  }
}

thread_local int t_split = 1;
unsigned long long* g_tc_trace = nullptr;
// split K also for M <= 16 (FLASHB_TC_SPLIT=1 or flashb_set_gemv_split(1)).  Off by default: measured on B200 at 148 SMs and M = 2, the
// mma.sync kernel's 8-row split takes 3.6 / 7.8 / 7.9 / 14.7 us for the backbone's o / q|k|v / down / gate|up
// matrices, the cluster split 9.2 / 17.2 / 14.6 / 27.4 us (a cluster of 8 large-smem CTAs waits for whole free SMs
// of one GPC, so it cannot start while the previous kernel drains).
int g_split_small = -1;
// rows per row group for M > 16: 64 (default), or 16 / 32 / 128.  Measured on B200 in the shared backbone step
// (128 rows, 148 SMs): 16 -> 5.92 ms, 32 -> 5.71, 64 -> 5.32, 128 -> 7.04 ms per step.
int g_group_rows = 64;

template <int EPI, bool NORM, int MT>
int launch_tc(const GemvArgs& g, int split, cudaStream_t st) {
  TcArgs a{};
  a.x = g.x; a.ldx = g.ldx; a.nw = g.nw; a.eps = g.eps;
  a.N0 = g.N0; a.N1 = g.N1; a.N = g.N; a.K = g.K; a.M = g.M;
  a.y = g.y; a.ldy = g.ldy; a.res = g.res; a.ldr = g.ldr; a.err = g.err;
  a.split = split;
  a.trace = g_tc_trace;
  const int nseg[3] = {EPI == 2 ? g.N : g.N0, EPI == 2 ? g.N : g.N1, EPI == 2 ? 0 : g.N - g.N0 - g.N1};
  const bf16* wseg[3] = {g.W0, g.W1, g.W2};
  for (int i = 0; i < 3; ++i) {
    if (nseg[i] <= 0) continue;
    if (fbh::tmap_box(&a.tw[i], wseg[i], nseg[i], g.K, 64, TC_BR, tc_cols<EPI>() / 64, true) != FB_OK)
      return FB_ERR_UNSUPPORTED;
  }
  // x [M rows, K] viewed as [K / 64 blocks][M rows][64]: one box = MT rows x the stage (rows >= M read zeros)
  if (fbh::tmap_box(&a.tx, g.x, g.M, g.K, 64, MT, tc_cols<EPI>() / 64, true, (long long)g.ldx) != FB_OK)
    return FB_ERR_UNSUPPORTED;
  constexpr int XB = tc_xbytes<EPI, MT>();
  const size_t fixed = 1024 + (size_t)TC_MAX_STAGES * 3 * 8 + 4 * 8 + 16 + 2 * MT * 4;
  int nst = (int)((227 * 1024 - fixed) / (TC_WBYTES + XB));
  if (nst > TC_MAX_STAGES) nst = TC_MAX_STAGES;
  a.nst = nst;
  // split K: the partial sums [128][RP] fp32 must fit over the ring
  if (split > 1 && (size_t)TC_BR * tc_rp<EPI, MT>() * 4 > (size_t)nst * (TC_WBYTES + XB)) return FB_ERR_UNSUPPORTED;
  const size_t smem = fixed + (size_t)nst * (TC_WBYTES + XB);
  auto kern = gemv_tc_kernel<EPI, NORM, MT>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_done[dev] < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("gemv_tc: cudaFuncSetAttribute(%zu bytes): %s", smem, cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = (int)smem;
  }
  const int nb = (g.N + TC_BR - 1) / TC_BR;
  const int groups = (g.M + MT - 1) / MT;
  int gsm = fbh::grid_sms() / groups;
  if (gsm < 1) gsm = 1;
  const int grid = split > 1 ? nb * split : (nb < gsm ? nb : gsm);
  void* args[] = {(void*)&a};
  t_split = split;
  return fbh::launch_pdl((const void*)kern, dim3(grid, groups), dim3(TC_THREADS), smem, st, args, true,
                         split > 1 ? split : 0);
}

template <int EPI, bool NORM>
int launch_mt(const GemvArgs& g, int mt, int split, cudaStream_t st) {
  if (mt == 16) return launch_tc<EPI, NORM, 16>(g, split, st);
  if (mt == 32) return launch_tc<EPI, NORM, 32>(g, split, st);
  if (mt == 64) return launch_tc<EPI, NORM, 64>(g, split, st);
  return launch_tc<EPI, NORM, 128>(g, split, st);
}

}  // namespace

// The tensor-core (tcgen05) GEMV when it applies: 1 <= M <= 128, K % 64 == 0, segment boundaries at multiples of
// 128.  M > 16 rows run as row groups of 64 rows (or of the width set by gemv_tc_set_group_rows), each on an equal
// share of the grid.  With at least a third of a group's CTAs in 128-row blocks, each CTA takes whole blocks; with
// fewer blocks the K range of each block is split over a cluster of S = min(8, CTAs / blocks, column stages) CTAs.  For M <= 16
// it then returns FB_ERR_UNSUPPORTED (the mma.sync kernel's 8-row split over every SM is faster) unless
// FLASHB_TC_SPLIT=1.
int gemv_tc(GemvArgs& g, int epi, bool norm, cudaStream_t st) {
  if (g.M < 1 || g.M > 128 || g.K % 64 != 0) return FB_ERR_UNSUPPORTED;
  const int n2 = g.N - g.N0 - g.N1;
  if (epi != 2 && (((g.N1 || n2) && g.N0 % TC_BR) || (n2 && (g.N0 + g.N1) % TC_BR))) return FB_ERR_UNSUPPORTED;
  if (g_split_small < 0) {
    const char* e = getenv("FLASHB_TC_SPLIT");
    g_split_small = (e && e[0] == '1') ? 1 : 0;
  }
  int mt = 16;                             // rows per group
  if (g.M > 16) {
    mt = g_group_rows;
    while (mt > 16 && mt / 2 >= g.M) mt /= 2;    // no wider than the rows need
  }
  const int groups = (g.M + mt - 1) / mt;
  const int nb = (g.N + TC_BR - 1) / TC_BR;
  int G = fbh::grid_sms() / groups;        // SMs per row group
  if (G < 1) G = 1;
  const int mrows = g.M < mt ? g.M : mt;   // rows of a group
  int split = 1;
  if (nb * 3 < G) {
    const int nkc = g.K / (epi == 2 ? 64 : 128);
    split = G / nb;
    if (split > TC_MAX_SPLIT) split = TC_MAX_SPLIT;
    if (split > nkc) split = nkc;
    if (split < 2) split = 1;
    if (mrows <= 16 && (split == 1 || !g_split_small)) return FB_ERR_UNSUPPORTED;
  }
  if (epi == 0 && norm) return launch_mt<0, true>(g, mt, split, st);
  if (epi == 0) return launch_mt<0, false>(g, mt, split, st);
  if (epi == 1) return launch_mt<1, false>(g, mt, split, st);
  if (epi == 2 && norm) return launch_mt<2, true>(g, mt, split, st);
  if (epi == 2) return launch_mt<2, false>(g, mt, split, st);
  return FB_ERR_UNSUPPORTED;
}

int gemv_tc_last_split() { return t_split; }
void gemv_tc_set_trace(void* buf) { g_tc_trace = static_cast<unsigned long long*>(buf); }
unsigned long long* gemv_trace_buf() { return g_tc_trace; }
void gemv_tc_set_split_small(int on) { g_split_small = on ? 1 : 0; }
int gemv_tc_set_group_rows(int rows) {
  if (rows != 16 && rows != 32 && rows != 64 && rows != 128) return FB_ERR_ARG;
  g_group_rows = rows;
  return FB_OK;
}

}  // namespace fb
