// flashb: skinny GEMV on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), for M <= 16 activation
// rows and K % 64 == 0.  Same semantics as the mma.sync kernel of fb_gemv_core.cuh (see fb_gemv.cu):
//   y[m, n] = sum_k xin[m, k] W[n, k] (fp32), NORM: xin = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))),
//   EPI 0: bf16(acc)   EPI 1: bf16(res + bf16(acc))   EPI 2: bf16(bf16(silu(bf16(acc_gate))) * bf16(acc_up)).
//
// B200 design.  The GEMV is turned around so that the weights are the MMA's M side: D[128 weight rows x 16] +=
// W[128 x 16 k] . x^T[16 k x 16 activation rows] (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 16, K = 16),
// activation rows >= M being zeros.  A CTA owns whole blocks of 128 output units and walks K in stages:
//   * warp 0 (one lane) streams each stage with TMA tensor copies in the canonical K-major 128-byte-swizzle operand
//     layout (8-row groups 1024 B apart): EPI 0/1 one 128-row x 128-column box of W; EPI 2 one 128-row x 64-column
//     box of the gate rows and one of the up rows; plus the activation tile x[16 rows x the stage's columns] in the
//     same layout.  One large box per matrix and stage matters: measured on B200, one SM streams 93 GB/s with a
//     128 x 128 box per 32 KB stage, 67 GB/s with four 64 x 64 boxes, 35 GB/s with 8-row boxes.  Weights are
//     independent of the previous kernel, so the first ring's worth of weight copies is issued before
//     griddepcontrol.wait, the activation copies after;
//   * warp 1 (one lane) issues the stage's MMAs (EPI 2: gate and up into two accumulators, so that a unit's gate
//     and up sums land in the same TMEM lane) and commits them to the stage's "empty" barrier (the ring slot is
//     free once the tensor core has read it) and, after a block's last stage, to the block's accumulator barrier.
//     The accumulators are double-buffered in TMEM, so block i + 1 accumulates while the epilogue of block i runs;
//   * warps 2-5 (one TMEM lane quarter each) read a block's accumulators (tcgen05.ld 32x32b.x16: row = lane,
//     16 activation columns), release them, and write the outputs.  With NORM they first rescale every activation
//     tile in shared memory (the RMS factors of the M rows are computed once per CTA) and hand it to the MMA warp
//     through a second barrier.
// There is no cross-warp reduction and no mma.sync: one thread drives the tensor core, the fp32 sums stay in TMEM
// across the whole K loop.  Every wait is bounded (fb_common.cuh); on expiry the error word is set and the CTA
// winds down (the producer waits for its own copies, the TMEM is freed).
#define FB_ST_TMA 1
#include "fb_gemv_core.cuh"
#include "fb_tc.cuh"

namespace fb {
namespace {

constexpr int TC_BR = 128;                      // output units per block (the MMA's M)
constexpr int TC_WBYTES = 32768;                // weight tile per stage: 128 rows x 128 columns (EPI 2: x 2 x 64)
constexpr int TC_XBYTES = 16 * 128 * 2;         // activation tile (16 rows x up to 128 columns)
// columns per stage: 128, or 64 for EPI 2 (gate and up tiles share the stage)
template <int EPI>
constexpr int tc_cols() { return EPI == 2 ? 64 : 128; }
constexpr int TC_MAX_STAGES = 6;
constexpr int TC_THREADS = 6 * 32;
constexpr int TC_EPI_THREADS = 4 * 32;

struct alignas(64) TcArgs {
  CUtensorMap tw[3];   // weight segments (EPI 2: gate, up) as [K / 64][rows][64], boxes of 128 rows x the stage
  CUtensorMap tx;      // x [M, K] as [K / 64][M][64], one box = 16 rows x the stage (both 128-byte swizzle)
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
  unsigned* err;
};

// Tensor map and first row of 128 weight rows starting at block row r (EPI 0/1: segments are multiples of 128).
// Rows past the last row stay with the last segment (an out-of-range box reads zeros), never with an empty one.
__device__ __forceinline__ TmaRows tc_rows(const TcArgs& a, int r) {
  const int n2 = a.N - a.N0 - a.N1;
  if (r < a.N0 || (a.N1 == 0 && n2 == 0)) return TmaRows{&a.tw[0], r};
  if (r < a.N0 + a.N1 || n2 == 0) return TmaRows{&a.tw[1], r - a.N0};
  return TmaRows{&a.tw[2], r - a.N0 - a.N1};
}

template <int EPI, bool NORM>
__global__ void __launch_bounds__(TC_THREADS, 1) gemv_tc_kernel(const __grid_constant__ TcArgs a) {
  constexpr int TC_C = tc_cols<EPI>();
  constexpr int UB = TC_BR;                           // output units per block
  // Accumulator chains: consecutive k-steps of a stage go to NCH independent accumulators (EPI 2: gate and up get
  // two each), summed in a fixed order in the epilogue.  The tensor core then overlaps them instead of running one
  // dependent chain of 8 small MMAs per stage, which kept every ring slot busy about twice as long (measured).
  constexpr int NCH = 4;
  constexpr int DCOLS = NCH * 16;                     // TMEM columns per accumulator buffer (x 2 buffers)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = a.nst;
  unsigned char* wring = smem;                                   // [NST][TC_WBYTES], 1024-aligned
  unsigned char* xring = smem + (size_t)NST * TC_WBYTES;         // [NST][TC_XBYTES]
  uint64_t* full = reinterpret_cast<uint64_t*>(xring + (size_t)NST * TC_XBYTES);
  uint64_t* empty = full + TC_MAX_STAGES;
  uint64_t* xok = empty + TC_MAX_STAGES;
  uint64_t* dfull = xok + TC_MAX_STAGES;                          // [2]
  uint64_t* dempty = dfull + 2;                                   // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dempty + 2);
  float* rs = reinterpret_cast<float*>(tslot + 4);                // [16] RMS factors

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, M = a.M;
  const int nkc = (K + TC_C - 1) / TC_C;
  const int units = a.N;
  const int nb_all = (units + UB - 1) / UB;
  const int b0 = (int)((long long)nb_all * blockIdx.x / gridDim.x);
  const int b1 = (int)((long long)nb_all * (blockIdx.x + 1) / gridDim.x);
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
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(2 * DCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    int issued = 0;
    auto issue_w = [&](int t) {
      const int s = t % NST, kc = t % nkc, blk = b0 + t / nkc;
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
      const int s = t % NST, kc = t % nkc;
      tma_load_3d(xring + (size_t)s * TC_XBYTES, &a.tx, 0, 0, kc * (TC_C / 64), &full[s]);
    };
    constexpr unsigned STAGE_TX = (unsigned)(TC_WBYTES + 16 * TC_C * 2);
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
        if (lane == 0) {
          const uint32_t wa = smem_u32(wring + (size_t)s * TC_WBYTES);
          const uint32_t xa = smem_u32(xring + (size_t)s * TC_XBYTES);
#pragma unroll
          for (int j = 0; j < TC_C / 16; ++j) {
            const uint64_t bd = tc_desc_sw128(xa + (j >> 2) * (16 * 128) + (j & 3) * 32);
            if (EPI == 2) {
              // gate chains in columns [0, 32), up chains in [32, 64)
              const uint32_t acc = (kc > 0 || j >= 2) ? 1u : 0u;
              const uint32_t ch = (uint32_t)((j & 1) * 16);
              tc_mma16(td + ch, tc_desc_sw128(wa + (j & 3) * 32), bd, acc);
              tc_mma16(td + 32 + ch, tc_desc_sw128(wa + TC_BR * 128 + (j & 3) * 32), bd, acc);
            } else {
              const uint32_t acc = (kc > 0 || j >= NCH) ? 1u : 0u;
              tc_mma16(td + (uint32_t)((j % NCH) * 16),
                     tc_desc_sw128(wa + (j >> 2) * (TC_BR * 128) + (j & 3) * 32), bd, acc);
            }
          }
          tc_commit(&empty[s]);
          if (kc == nkc - 1) tc_commit(&dfull[i & 1]);
        }
        __syncwarp();
        committed = t;
      }
    }
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
      // RMS factor of each activation row: warp q reduces rows q, q + 4, ...
      for (int m = q; m < 16; m += 4) {
        float ss = 0.f;
        if (m < M)
          for (int j = lane; j < (K >> 3); j += 32) {
            float f[8];
            cvt8(*reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + j * 8), f);
#pragma unroll
            for (int u = 0; u < 8; ++u) ss = fmaf(f[u], f[u], ss);
          }
        ss = warp_sum(ss);
        if (lane == 0) rs[m] = 1.0f / sqrtf(ss / (float)K + a.eps);
      }
      named_sync(1, TC_EPI_THREADS);
    }
    auto fix = [&](int t) -> bool {       // rescale stage t's activation tile in place
      const int s = t % NST, kc = t % nkc;
      if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err)) return false;
      unsigned char* xt = xring + (size_t)s * TC_XBYTES;
      for (int i = etid; i < 16 * TC_C * 2 / 16; i += TC_EPI_THREADS) {
        // [64-column block c][row m][16-byte unit jp], unit jp holding columns 8 (jp ^ (m % 8)) .. of the block
        const int c = i >> 7, m = (i >> 3) & 15, jp = i & 7;
        const int k = kc * TC_C + c * 64 + ((jp ^ (m & 7)) << 3);
        if (m >= M || k >= K) continue;
        uint4* p = reinterpret_cast<uint4*>(xt + (size_t)i * 16);
        float f[8], w[8];
        cvt8(*p, f);
        cvt8(*reinterpret_cast<const uint4*>(a.nw + k), w);
        const float r = rs[m];
        uint4 o;
        o.x = pack2(w[0] * rbf(f[0] * r), w[1] * rbf(f[1] * r));
        o.y = pack2(w[2] * rbf(f[2] * r), w[3] * rbf(f[3] * r));
        o.z = pack2(w[4] * rbf(f[4] * r), w[5] * rbf(f[5] * r));
        o.w = pack2(w[6] * rbf(f[6] * r), w[7] * rbf(f[7] * r));
        *p = o;
      }
      fence_proxy_async();                 // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&xok[s]);
      return true;
    };
    auto epilogue = [&](int i) -> bool {
      if (!mbar_wait(&dfull[i & 1], (i >> 1) & 1, a.err)) return false;
      tc_after();
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((i & 1) * DCOLS);
      float v[16], u[16];
      {
        float c0[16], c1[16];
        tc_ld16(tq, c0);
        tc_ld16(tq + 16, c1);
#pragma unroll
        for (int m = 0; m < 16; ++m) v[m] = c0[m] + c1[m];
        tc_ld16(tq + 32, c0);
        tc_ld16(tq + 48, c1);
        if (EPI == 2) {
#pragma unroll
          for (int m = 0; m < 16; ++m) u[m] = c0[m] + c1[m];
        } else {
#pragma unroll
          for (int m = 0; m < 16; ++m) v[m] = (v[m] + c0[m]) + c1[m];
        }
      }
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[i & 1]);
      const int n = (b0 + i) * UB + row;
      if (n < units) {
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          if (m < M) {
            float o;
            if (EPI == 2) {
              const float gg = rbf(v[m]);
              o = rbf(gg / (1.0f + expf(-gg))) * rbf(u[m]);
            } else if (EPI == 1) {
              o = b2f(a.res[(size_t)m * a.ldr + n]) + rbf(v[m]);
            } else {
              o = v[m];
            }
            a.y[(size_t)m * a.ldy + n] = __float2bfloat16_rn(o);
          }
        }
      }
      return true;
    };
    if (NORM) {
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
  tc_before();
  __syncthreads();
  tc_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * DCOLS) : "memory");
}

template <int EPI, bool NORM>
int launch_tc(const GemvArgs& g, cudaStream_t st) {
  TcArgs a{};
  a.x = g.x; a.ldx = g.ldx; a.nw = g.nw; a.eps = g.eps;
  a.N0 = g.N0; a.N1 = g.N1; a.N = g.N; a.K = g.K; a.M = g.M;
  a.y = g.y; a.ldy = g.ldy; a.res = g.res; a.ldr = g.ldr; a.err = g.err;
  const int nseg[3] = {EPI == 2 ? g.N : g.N0, EPI == 2 ? g.N : g.N1, EPI == 2 ? 0 : g.N - g.N0 - g.N1};
  const bf16* wseg[3] = {g.W0, g.W1, g.W2};
  for (int i = 0; i < 3; ++i) {
    if (nseg[i] <= 0) continue;
    if (fbh::tmap_box(&a.tw[i], wseg[i], nseg[i], g.K, 64, TC_BR, tc_cols<EPI>() / 64, true) != FB_OK)
      return FB_ERR_UNSUPPORTED;
  }
  // x [M rows, K] viewed as [K / 64 blocks][M rows][64]: one box = 16 rows x the stage (rows >= M read zeros)
  if (fbh::tmap_box(&a.tx, g.x, g.M, g.K, 64, 16, tc_cols<EPI>() / 64, true, (long long)g.ldx) != FB_OK)
    return FB_ERR_UNSUPPORTED;
  const size_t fixed = 1024 + (size_t)TC_MAX_STAGES * 3 * 8 + 4 * 8 + 16 + 16 * 4;
  int nst = (int)((227 * 1024 - fixed) / (TC_WBYTES + TC_XBYTES));
  if (nst > TC_MAX_STAGES) nst = TC_MAX_STAGES;
  a.nst = nst;
  const size_t smem = fixed + (size_t)nst * (TC_WBYTES + TC_XBYTES);
  auto kern = gemv_tc_kernel<EPI, NORM>;
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
  const int grid = nb < fbh::grid_sms() ? nb : fbh::grid_sms();
  void* args[] = {(void*)&a};
  return fbh::launch_pdl((const void*)kern, dim3(grid), dim3(TC_THREADS), smem, st, args, true);
}

}  // namespace

// The tensor-core (tcgen05) GEMV when it applies: M <= 16, K % 64 == 0, segment boundaries at multiples of 128,
// and enough 128-unit blocks to keep at least a third of the grid busy (fewer, and the mma.sync kernel's finer
// split over every SM is faster).  Returns FB_ERR_UNSUPPORTED when it does not apply.
int gemv_tc(GemvArgs& g, int epi, bool norm, cudaStream_t st) {
  if (g.M < 1 || g.M > 16 || g.K % 64 != 0) return FB_ERR_UNSUPPORTED;
  const int n2 = g.N - g.N0 - g.N1;
  if (epi != 2 && (((g.N1 || n2) && g.N0 % TC_BR) || (n2 && (g.N0 + g.N1) % TC_BR))) return FB_ERR_UNSUPPORTED;
  const int nb = (g.N + TC_BR - 1) / TC_BR;
  if (nb * 3 < fbh::grid_sms()) return FB_ERR_UNSUPPORTED;
  if (epi == 0 && norm) return launch_tc<0, true>(g, st);
  if (epi == 0) return launch_tc<0, false>(g, st);
  if (epi == 1) return launch_tc<1, false>(g, st);
  if (epi == 2 && norm) return launch_tc<2, true>(g, st);
  if (epi == 2) return launch_tc<2, false>(g, st);
  return FB_ERR_UNSUPPORTED;
}

}  // namespace fb
