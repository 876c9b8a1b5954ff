// flashb: the GEMV of many activation rows (17 .. 128 for the shared backbone step of many streams; any number in
// tiles of 128 rows for the prefill's dense GEMMs) on the 5th-generation tensor cores.  Same semantics as the other GEMV kernels (fb_gemv.cu), without the RMSNorm (the
// caller normalises the rows first, flashb_rmsnorm):
//   y[m, n] = sum_k x[m, k] W[n, k] (fp32),  EPI 0: bf16(acc)   EPI 1: bf16(res + bf16(acc))
//   EPI 2: bf16(bf16(silu(bf16(acc_gate))) * bf16(acc_up)).
//
// B200 design.  The activation rows are the MMA's M side and the weights its N side: D[128 rows x BN units] +=
// x[128 rows x 16 k] . W[BN units x 16 k]^T (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 128, or 256 for the
// gate|up pair whose 128 gate and 128 up rows sit in one operand).  Rows >= M are the zeros of the x tensor map's
// out-of-range fill.  All rows in one MMA means every weight byte crosses HBM once, and D's layout (TMEM lane = row,
// column = unit) gives each epilogue thread 16 consecutive units of one row per TMEM load: 32-byte row segments
// written straight to y, a residual read the same way, and the gate and up sums of a unit in the same thread.
//
// A tile is 128 output units (EPI 2: 128 gate + 128 up units) over the whole K, for 128 activation rows (row tile
// blockIdx.y when there are more).  A decode step has few tiles (16 for a 2048-row matrix), so K is split over a
// thread-block cluster of S CTAs (S <= 8): rank r takes the r-th of S ranges of 64-column chunks.  S is chosen on the host from the occupancy API so that every cluster of the launch is
// resident at once and the most SMs stream.  Per CTA:
//   * warp 0 (one lane) streams the K range through a ring of stages [x 128 rows x 64 columns | W BN rows x 64
//     columns] with TMA tensor copies in the K-major 128-byte-swizzle layout.  The weight copies of the first ring's
//     worth are issued before griddepcontrol.wait (weights do not depend on the previous kernel), x after it;
//   * warp 1 (one lane) issues four MMAs per stage into one TMEM accumulator and commits them to the stage's
//     "empty" barrier and, after the last stage, to the accumulator barrier;
//   * warps 2-9 (TMEM lane quarter = warp % 4, so thread = row; two warps per quarter take alternate groups) run the
//     reduction and the epilogue.
// Split-K reduction through distributed shared memory, pushed rather than pulled: the tile's 16-unit groups are
// divided among the ranks; after a cluster barrier (every CTA's MMAs complete, so every ring is free) each thread
// reads from TMEM the groups other ranks own and stores them into the owner's receive area (the owner's ring; rank
// r + 1 first, so that the cluster's senders spread over the receivers), a
// second cluster barrier publishes the stores, and each owner adds the S partial sums of its groups in rank order
// (deterministic) and writes them.  No global workspace, no atomics, no dependent remote loads.
// Every mbarrier wait is bounded (fb_common.cuh); on expiry the error word is set and every thread still reaches
// both cluster barriers, so the CTA winds down.
#include "fb_gemv_core.cuh"
#include "fb_tc.cuh"

#include <map>
#include <mutex>
#include <tuple>

namespace fb {
namespace {

constexpr int GR_BN = 128;                  // output units per tile (per matrix for EPI 2)
constexpr int GR_GROUPS = GR_BN / 16;       // 16-unit groups of a tile (the split-K reduction's unit of work)
constexpr int GR_XB = 128 * 128;            // x per stage: 128 rows x 64 columns bf16
constexpr int GR_THREADS = 10 * 32;          // producer, MMA, 8 epilogue warps (two per TMEM lane quarter)
constexpr int GR_MAX_STAGES = 8;
constexpr int GR_MAX_SPLIT = 8;
template <int EPI>
constexpr int gr_wbytes() { return (EPI == 2 ? 2 : 1) * GR_BN * 128; }   // weights per stage
template <int EPI>
constexpr int gr_sbytes() { return GR_XB + gr_wbytes<EPI>(); }             // stage
template <int EPI>
constexpr int gr_ncols() { return (EPI == 2 ? 2 : 1) * GR_BN; }            // MMA N = TMEM columns
constexpr int gr_mats(int epi) { return epi == 2 ? 2 : 1; }

struct alignas(64) RowsArgs {
  CUtensorMap tw[3];   // weight segments (EPI 2: gate, up) as [K / 64][rows][64], boxes of 128 rows x 64 columns
  CUtensorMap tx;      // x [M, K] as [K / 64][M][64], boxes of 128 rows x 64 columns (rows >= M read zeros)
  int N0, N1, N, K, M;
  bf16* y;
  long ldy;
  const bf16* res;
  long ldr;
  int nst;             // ring stages
  int split;           // CTAs per cluster (1: no split)
  int pitch;           // columns of a receive slot per sender (column-major over the 128 rows)
  int area;            // bytes of the ring / receive area (the mbarriers follow it)
  unsigned* err;
  unsigned long long* trace;   // optional per-CTA timeline (flashb_set_gemv_trace), or null
};

// Timeline stamps (flashb_set_gemv_trace): entry, producer past griddepcontrol.wait, first stage in, last MMA
// committed, accumulators complete, split-K exchange done, exit (ns), SM id.
#define GR_STAMP(i, v)                                                                  \
  do {                                                                                  \
    if (a.trace) a.trace[(blockIdx.y * gridDim.x + blockIdx.x) * 16 + (i)] = (unsigned long long)(v); \
  } while (0)

__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t cl_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cl_st1(uint32_t addr, float a) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(a) : "memory");
}
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_plain(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// First 16-unit group owned by rank r of S (ranks own [gr_first(r), gr_first(r + 1))).
__device__ __forceinline__ int gr_first(int r, int S) { return GR_GROUPS * r / S; }

// Tensor map and first row of the 128 weight rows of tile t (EPI 0/1: segments are multiples of 128 rows).
__device__ __forceinline__ TmaRows gr_rows(const RowsArgs& a, int r) {
  const int n2 = a.N - a.N0 - a.N1;
  if (r < a.N0 || (a.N1 == 0 && n2 == 0)) return TmaRows{&a.tw[0], r};
  if (r < a.N0 + a.N1 || n2 == 0) return TmaRows{&a.tw[1], r - a.N0};
  return TmaRows{&a.tw[2], r - a.N0 - a.N1};
}

// Epilogue of 16 units n0 .. n0 + 15 of row m (N % 16 == 0): v = sums (EPI 2: gate), u = up sums, r0 / r1 = the
// residual's 16 values (EPI 1).
template <int EPI>
__device__ __forceinline__ void gr_store(const RowsArgs& a, int m, int n0, const float (&v)[16], const float (&u)[16],
                                         const uint4& r0, const uint4& r1) {
  float o[16];
  if (EPI == 1) {
    float r[16];
    cvt8(r0, r);
    cvt8(r1, r + 8);
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = r[i] + rbf(v[i]);
  } else if (EPI == 2) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float g = rbf(v[i]);
      o[i] = silu_rbf(g) * rbf(u[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = v[i];
  }
  uint4* yp = reinterpret_cast<uint4*>(a.y + (size_t)m * a.ldy + n0);
  yp[0] = make_uint4(pack2(o[0], o[1]), pack2(o[2], o[3]), pack2(o[4], o[5]), pack2(o[6], o[7]));
  yp[1] = make_uint4(pack2(o[8], o[9]), pack2(o[10], o[11]), pack2(o[12], o[13]), pack2(o[14], o[15]));
}

template <int EPI>
__global__ void __launch_bounds__(GR_THREADS, 1) gemv_rows_kernel(const __grid_constant__ RowsArgs a) {
  constexpr int WB = gr_wbytes<EPI>();
  constexpr int SB = gr_sbytes<EPI>();
  constexpr int NC = gr_ncols<EPI>();
  constexpr int MATS = gr_mats(EPI);
  constexpr uint32_t IDESC = tc_idesc(NC, 128);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = a.nst, S = a.split;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.area);
  uint64_t* empty = full + GR_MAX_STAGES;
  uint64_t* dfull = empty + GR_MAX_STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dfull + 1);
  float* recv = reinterpret_cast<float*>(smem);     // split K: [S senders][pitch columns][128 rows], over the idle ring

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) GR_STAMP(0, globaltimer());
  const int rank = (int)(blockIdx.x % S), tile = (int)(blockIdx.x / S);
  const int r0 = (int)blockIdx.y * 128;      // first activation row of this row tile
  const int nkc_all = a.K / 64;
  const int kc0 = nkc_all * rank / S;
  const int nkc = nkc_all * (rank + 1) / S - kc0;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(dfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tc_alloc(tslot, NC);
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const uint64_t wpol = policy_evict_first();    // weights are read once per step
    auto issue_w = [&](int t) {
      unsigned char* wt = smem + (size_t)(t % NST) * SB + GR_XB;
      const int kc = kc0 + t;
      if (EPI == 2) {
        tma_load_3d_hint(wt, &a.tw[0], 0, tile * GR_BN, kc, &full[t % NST], wpol);
        tma_load_3d_hint(wt + GR_BN * 128, &a.tw[1], 0, tile * GR_BN, kc, &full[t % NST], wpol);
      } else {
        const TmaRows h = gr_rows(a, tile * GR_BN);
        tma_load_3d_hint(wt, h.map, 0, h.row, kc, &full[t % NST], wpol);
      }
    };
    auto issue_x = [&](int t) {
      tma_load_3d_plain(smem + (size_t)(t % NST) * SB, &a.tx, 0, r0, kc0 + t, &full[t % NST]);
    };
    if (lane < 4) tma_prefetch_map(lane < 3 ? (const void*)&a.tw[lane] : (const void*)&a.tx);
    const int pre = min(nkc, NST);
    if (lane == 0)
      for (int t = 0; t < pre; ++t) {
        mbar_arrive_expect_tx(&full[t], (unsigned)SB);
        issue_w(t);
      }
    __syncwarp();
    pdl_wait();
    if (lane == 0) GR_STAMP(1, globaltimer());
    if (lane == 0)
      for (int t = 0; t < pre; ++t) issue_x(t);
    __syncwarp();
    int issued = pre;
    for (int t = pre; t < nkc; ++t) {
      if (!mbar_wait_warp(&empty[t % NST], ((t / NST) - 1) & 1, a.err)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[t % NST], (unsigned)SB);
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
    for (int t = 0; t < nkc; ++t) {
      const int s = t % NST;
      if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err)) {
        ok = false;
        break;
      }
      tc_after();
      if (lane == 0 && t == 0) GR_STAMP(2, globaltimer());
      if (lane == 0) {
        const uint64_t xd = tc_desc_sw128(smem_u32(smem + (size_t)s * SB));
        const uint64_t wd = xd + (uint64_t)(GR_XB / 16);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc_mma(tmem, xd + (uint64_t)(j << 1), wd + (uint64_t)(j << 1), (t > 0 || j > 0) ? 1u : 0u, IDESC);
        tc_commit(&empty[s]);
        if (t == nkc - 1) tc_commit(dfull);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) tc_commit(dfull);   // the epilogue's wait ends (the sums are void; the error is set)
    if (lane == 0) GR_STAMP(3, globaltimer());
    __syncwarp();
  }
  // ------------------------------------------------------------------ reduction and epilogue (warps 2-9)
  // Two warps per TMEM lane quarter (warp % 4); the quarter's work items alternate between them.
  const bool epi = warp >= 2;
  const int q = warp & 3;                    // TMEM lane quarter
  const int eh = (warp - 2) >> 2;            // 0 / 1: which of the quarter's two warps
  const int row = q * 32 + lane;             // the accumulator row of this thread (activation row r0 + row)
  const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
  if (epi) {
    pdl_wait();                              // res / y belong to earlier kernels of the stream
    pdl_trigger();
    mbar_wait(dfull, 0, a.err);
    tc_after();
    if (tid == 64) GR_STAMP(4, globaltimer());
  }
  const int g0 = gr_first(rank, S), g1 = gr_first(rank + 1, S);
  if (S > 1) {
    // every CTA of the cluster: its MMAs are complete, so its ring may receive
    __syncwarp();
    cl_arrive();
    cl_wait();
    if (tid == 64) GR_STAMP(8, globaltimer());
    if (epi) {
      // the groups other ranks own, rank + 1's first (so that the senders of a cluster spread over the receivers)
      // column-major slots: for each column the 32 lanes of a warp (consecutive rows) write 128 contiguous bytes
      const uint32_t mine = smem_u32(recv) + (uint32_t)(rank * a.pitch * 128 + row) * 4u;
      int item = 0;
      for (int j = 1; j < S; ++j) {
        const int o = (rank + j) % S, f0 = gr_first(o, S), f1 = gr_first(o + 1, S);
        const uint32_t base = cl_map(mine, (uint32_t)o);
        for (int g = f0; g < f1; ++g, ++item) {
          if ((item & 1) != eh) continue;
          float v[16], w[16];
          if (EPI == 2) {
            tc_ld16x2(tq + (uint32_t)(g * 16), tq + (uint32_t)(GR_BN + g * 16), v, w);
          } else {
            tc_ld16(tq + (uint32_t)(g * 16), v);
          }
          const uint32_t dst = base + (uint32_t)((g - f0) * 16 * MATS * 128) * 4u;
#pragma unroll
          for (int i = 0; i < 16; ++i) cl_st1(dst + (uint32_t)(i * 128) * 4u, v[i]);
          if (EPI == 2) {
#pragma unroll
            for (int i = 0; i < 16; ++i) cl_st1(dst + (uint32_t)((16 + i) * 128) * 4u, w[i]);
          }
        }
      }
    }
    if (tid == 64) GR_STAMP(9, globaltimer());
    __syncwarp();
    cl_arrive();
    cl_wait();
  }
  if (tid == 64) GR_STAMP(5, globaltimer());
  if (epi) {
    // own groups: this CTA's sums (TMEM) plus the other ranks' (received) in increasing rank order
    const int ga = S > 1 ? g0 : 0, gb = S > 1 ? g1 : GR_GROUPS;
    for (int g = ga + eh; g < gb; g += 2) {
      const int n0 = tile * GR_BN + g * 16;
      const int m = r0 + row;
      const bool live = m < a.M && n0 < a.N;
      uint4 rr0 = make_uint4(0u, 0u, 0u, 0u), rr1 = rr0;
      if (EPI == 1 && live) {                // the residual first: its latency overlaps the reads below
        const uint4* rp = reinterpret_cast<const uint4*>(a.res + (size_t)m * a.ldr + n0);
        rr0 = rp[0];
        rr1 = rp[1];
      }
      float v[16], u[16];
      if (EPI == 2) {
        tc_ld16x2(tq + (uint32_t)(g * 16), tq + (uint32_t)(GR_BN + g * 16), v, u);
      } else {
        tc_ld16(tq + (uint32_t)(g * 16), v);
      }
      for (int p = 0; p < S; ++p) {
        if (p == rank) continue;
        const float* src = recv + ((size_t)p * a.pitch + (g - g0) * 16 * MATS) * 128 + row;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] += src[i * 128];
          if (EPI == 2) u[i] += src[(16 + i) * 128];
        }
      }
      if (live) gr_store<EPI>(a, m, n0, v, u, rr0, rr1);
    }
    if (tid == 64) GR_STAMP(10, globaltimer());
  }
  tc_before();
  __syncthreads();
  tc_after();
  if (warp == 1) tc_dealloc(tmem, NC);
  if (tid == 0) {
    GR_STAMP(6, globaltimer());
    unsigned sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    GR_STAMP(7, sm);
  }
}

// ------------------------------------------------------------------------------------------------ host side
std::mutex g_rows_mu;
std::map<std::tuple<int, int, int, size_t>, int> g_rows_occ;   // (device, EPI, S, smem) -> clusters resident at once

template <int EPI>
size_t rows_area(int nst, int S, int pitch) {
  const size_t ring = (size_t)nst * gr_sbytes<EPI>();
  const size_t recv = S > 1 ? (size_t)S * 128 * pitch * 4 : 0;
  return ring > recv ? ring : recv;
}
// At least 116 KB, so that two CTAs never share an SM: a CTA waiting for TMEM held by another cluster's CTA on its
// SM, while that cluster waits at a cluster barrier for a CTA in the same position elsewhere, could wait for good.
template <int EPI>
size_t rows_smem(int nst, int S, int pitch) {
  const size_t s = 1024 + rows_area<EPI>(nst, S, pitch) + (2 * GR_MAX_STAGES + 1) * 8 + 16;
  return s < 116 * 1024 ? 116 * 1024 : s;
}

template <int EPI>
int rows_pitch(int S) {
  return (GR_GROUPS + S - 1) / S * 16 * gr_mats(EPI);      // columns a rank owns (its receive slot per sender)
}

template <int EPI>
int rows_stages(int nkc_cta) {
  int nst = (200 * 1024) / gr_sbytes<EPI>();
  if (nst > GR_MAX_STAGES) nst = GR_MAX_STAGES;
  if (nst > nkc_cta) nst = nkc_cta;
  return nst < 1 ? 1 : nst;
}

// Clusters of S CTAs of this kernel resident at once (occupancy API, cached per device and shape).
template <int EPI>
int rows_occupancy(int dev, int S, size_t smem, int tiles) {
  const auto key = std::make_tuple(dev, EPI, S, smem);
  {
    std::lock_guard<std::mutex> lk(g_rows_mu);
    auto it = g_rows_occ.find(key);
    if (it != g_rows_occ.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * S);
  cfg.blockDim = dim3(GR_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (S == 1) {
    int per = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, gemv_rows_kernel<EPI>, GR_THREADS, smem) != cudaSuccess)
      per = 0;
    n = per * fbh::num_sms();
  } else if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemv_rows_kernel<EPI>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(g_rows_mu);
  g_rows_occ[key] = n;
  return n;
}

thread_local int t_rows_split = 1;

template <int EPI>
int launch_rows(const GemvArgs& g, cudaStream_t st) {
  const int N = g.N, K = g.K;
  const int tiles = (N + GR_BN - 1) / GR_BN;
  const int rtiles = (g.M + 127) / 128;      // row tiles (blockIdx.y)
  const int nkc = K / 64;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_done[64] = {false};
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_rows_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) {
      fbh::set_msg("gemv_rows: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = true;
  }
  // the split with the most streaming CTAs that all fit at once (ties: the smaller split)
  const int sms = fbh::grid_sms();
  int best = 1, best_ctas = 0;
  for (int S = 1; S <= GR_MAX_SPLIT; ++S) {
    if (S > 1 && nkc / S < 2) break;              // at least two chunks per CTA
    if (S > 1 && tiles * rtiles * S > sms) break; // enough tiles already: no split
    const int nst = rows_stages<EPI>((nkc + S - 1) / S);
    const size_t smem = rows_smem<EPI>(nst, S, rows_pitch<EPI>(S));
    if (smem > 227 * 1024) continue;
    const int fit = rows_occupancy<EPI>(dev, S, smem, tiles);
    if (S > 1 && fit < tiles * rtiles) continue;
    if (tiles * S > best_ctas) {
      best = S;
      best_ctas = tiles * S;
    }
  }
  const int S = best;
  RowsArgs a{};
  a.N0 = g.N0; a.N1 = g.N1; a.N = N; a.K = K; a.M = g.M;
  a.y = g.y; a.ldy = g.ldy; a.res = g.res; a.ldr = g.ldr; a.err = g.err;
  a.split = S;
  a.trace = gemv_trace_buf();
  a.pitch = rows_pitch<EPI>(S);
  a.nst = rows_stages<EPI>((nkc + S - 1) / S);
  a.area = (int)rows_area<EPI>(a.nst, S, a.pitch);
  const int nseg[3] = {EPI == 2 ? N : g.N0, EPI == 2 ? N : g.N1, EPI == 2 ? 0 : N - g.N0 - g.N1};
  const bf16* wseg[3] = {g.W0, g.W1, g.W2};
  for (int i = 0; i < 3; ++i) {
    if (nseg[i] <= 0) continue;
    if (fbh::tmap_box(&a.tw[i], wseg[i], nseg[i], K, 64, GR_BN, 1, true) != FB_OK) return FB_ERR_UNSUPPORTED;
  }
  if (fbh::tmap_box(&a.tx, g.x, g.M, K, 64, 128, 1, true, (long long)g.ldx) != FB_OK) return FB_ERR_UNSUPPORTED;
  const size_t smem = rows_smem<EPI>(a.nst, S, a.pitch);
  void* args[] = {(void*)&a};
  t_rows_split = S;
  return fbh::launch_pdl((const void*)gemv_rows_kernel<EPI>, dim3(tiles * S, rtiles), dim3(GR_THREADS), smem, st, args,
                         true, S > 1 ? S : 0);
}

}  // namespace

// The many-rows tensor-core GEMV when it applies: M >= 17 (tiles of 128 rows), no RMSNorm, K % 64 == 0, segment
// boundaries (EPI 0/1) at multiples of 128 rows, N % 16 == 0, y / res rows 16-byte aligned.  Else
// FB_ERR_UNSUPPORTED.
int gemv_rows(GemvArgs& g, int epi, cudaStream_t st) {
  if (g.M < 17 || g.M > 65535 * 128 || g.K % 64 != 0 || g.K < 128 || g.N % 16 != 0) return FB_ERR_UNSUPPORTED;
  const int n2 = g.N - g.N0 - g.N1;
  if (epi != 2 && (((g.N1 || n2) && g.N0 % GR_BN) || (n2 && (g.N0 + g.N1) % GR_BN))) return FB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(g.y) & 15) || g.ldy % 8) return FB_ERR_UNSUPPORTED;
  if (epi == 1 && ((reinterpret_cast<uintptr_t>(g.res) & 15) || g.ldr % 8)) return FB_ERR_UNSUPPORTED;
  if (epi == 0) return launch_rows<0>(g, st);
  if (epi == 1) return launch_rows<1>(g, st);
  if (epi == 2) return launch_rows<2>(g, st);
  return FB_ERR_UNSUPPORTED;
}

int gemv_rows_last_split() { return t_rows_split; }

}  // namespace fb
