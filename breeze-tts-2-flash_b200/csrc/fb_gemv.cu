// flashb: skinny bf16 GEMVs for the backbone decode step (M = 1..8 activation rows, nn.Linear weights [N, K]).
//
// Semantics (the eager rounding points the reference restates in flash/csrc/bb_fused.cu:1-7):
//   y[m, n] = sum_k xin[m, k] * W[n, k]           fp32 accumulation
//   prologue NORM: xin = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))   (Qwen3RMSNorm, per CTA, redundant)
//   EPI 0: bf16(acc)   EPI 1: bf16(res + bf16(acc))   EPI 2: bf16(bf16(silu(bf16(acc_gate))) * bf16(acc_up))
//
// B200 design: the kernel is an HBM stream of the weight matrix.  Each CTA owns a contiguous range of output rows
// (grid = #SMs, so every SM streams ~N/148 rows) and a producer warp moves the rows into a shared-memory ring with
// 1-D bulk copies (cp.async.bulk, the TMA engine; no tensor map, no multicast) completing on mbarriers, while 8
// consumer warps do the dot products from shared memory (one weight row per warp per stage, x staged once).  The
// weights never depend on the previous kernel, so the producer fills the whole ring BEFORE griddepcontrol.wait: with
// programmatic dependent launch the weight stream of GEMV i+1 starts while kernel i drains.  The ring is sized so
// two CTAs fit on an SM (<= ~112 KB each), letting the next kernel's CTAs co-reside and prefetch.
#include "fb_gemv_core.cuh"

#ifndef FB_GEMV_NARROW_MIN
#define FB_GEMV_NARROW_MIN 4
#endif

namespace fb {

// Kernel the calling thread's last GEMV launch used: 0 FMA, 1 mma.sync stream, 2 tcgen05 (flashb_gemv_last_path).
thread_local int t_gemv_path = -1;
int g_rows_path = 1;   // the many-rows kernel (fb_gemv_rows.cu) for 17..128 rows without norm; 0: off

constexpr int GV_CWARPS = 8;
constexpr int GV_MAX_ROWS = 1 << 20;   // activation rows of one call (a prefill: batch x prompt tokens)
constexpr int GV_THREADS = (GV_CWARPS + 1) * 32;
constexpr int GV_STAGE_BYTES = 32768;
constexpr int GV_MAX_STAGES = 12;
constexpr int GV_SMEM_BUDGET = 112 * 1024;

// Fallback for K % 8 == 0 but K % 64 != 0 (the tensor path's column blocks are 64 wide): scalar FMA from shared
// memory.
// A stage holds RS consecutive output rows (x NMAT matrices) in full (all K columns), copied as contiguous runs:
// one bulk copy per matrix and segment (<= 3 per stage), each up to 32 KB.  Warps take rows round-robin; when a
// stage has fewer rows than warps, 2 or 4 warps split each row's K range and combine their partial sums through
// shared memory in a fixed order (deterministic results).
template <int M, int EPI, bool NORM>
__global__ void __launch_bounds__(GV_THREADS) gemv_fma_kernel(const GemvArgs a) {
  constexpr int NMAT = EPI == 2 ? 2 : 1;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* xs = reinterpret_cast<bf16*>(smem);
  unsigned char* ring = smem + a.xs_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)a.nstages * GV_STAGE_BYTES);
  uint64_t* empty = full + GV_MAX_STAGES;
  __shared__ float rfac[M];
  __shared__ float part[GV_CWARPS][NMAT][M];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, bid = blockIdx.x;
  const int r0 = (int)((long long)a.N * bid / G), r1 = (int)((long long)a.N * (bid + 1) / G);
  const int RS = a.RS;
  const int T = (r1 - r0 + RS - 1) / RS;
  const int NST = a.nstages;
  const int K = a.K;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CWARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == GV_CWARPS) {
    // ------------------------------------------------------------ producer: weights only, may run before pdl_wait
    int issued = 0;
    for (int t = 0; t < T; ++t) {
      const int s = t % NST;
      if (t >= NST) {
        if (!mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1, a.err)) break;
      }
      const int n0 = r0 + t * RS;
      const int nr = min(RS, r1 - n0);
      bf16* st = reinterpret_cast<bf16*>(ring + (size_t)s * GV_STAGE_BYTES);
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], (unsigned)(nr * NMAT * K * 2));
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat) {
          int n = n0;
          while (n < n0 + nr) {
            const int e = min(n0 + nr, gv_seg_end<EPI>(a, n));
            bulk_g2s(st + ((size_t)mat * RS + (n - n0)) * K, gv_row<EPI>(a, n, mat), (unsigned)((e - n) * K * 2),
                     &full[s]);
            n = e;
          }
        }
      }
      __syncwarp();
      ++issued;
    }
    // never leave with copies in flight into this CTA's shared memory
    for (int t = max(0, issued - NST); t < issued; ++t) {
      if (!mbar_wait_warp(&full[t % NST], (t / NST) & 1, a.err)) break;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  pdl_trigger();
  const int ctid = threadIdx.x;  // 0..255
  {
    // stage x (rows at a pitch of K elements), then the row factors and the norm in place
    const int nu = K >> 3;
    for (int i = ctid; i < M * nu; i += GV_CWARPS * 32) {
      const int m = i / nu, u = i - m * nu;
      reinterpret_cast<uint4*>(xs)[i] = *reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + (size_t)u * 8);
    }
    named_sync(1, GV_CWARPS * 32);
    if (NORM) {
      const PitchOff off{K * 2};
      rms_row_factors(smem, off, M, K, a.eps, rfac, warp, GV_CWARPS);
      named_sync(1, GV_CWARPS * 32);
      rms_rows_apply(smem, off, M, K, a.nw, rfac, ctid, GV_CWARPS * 32);
      named_sync(1, GV_CWARPS * 32);
    }
  }

  for (int t = 0; t < T; ++t) {
    const int s = t % NST;
    if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err)) return;
    const int n0 = r0 + t * RS;
    const int nr = min(RS, r1 - n0);
    // warps per row: split K when the stage has fewer rows than warps
    const int wpr = nr >= GV_CWARPS ? 1 : (nr >= 4 ? 2 : (nr >= 2 ? 4 : 8));
    const int kslice = ((K + 8 * wpr - 1) / (8 * wpr)) * 8;
    const bf16* st = reinterpret_cast<const bf16*>(ring + (size_t)s * GV_STAGE_BYTES);
    const int rows_per_pass = GV_CWARPS / wpr;
    for (int rb = 0; rb < nr; rb += rows_per_pass) {
      const int r = rb + warp / wpr;
      const int ks = (warp % wpr) * kslice;
      const int ke = min(ks + kslice, K);
      float acc[NMAT][M];
#pragma unroll
      for (int q = 0; q < NMAT; ++q)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[q][m] = 0.f;
      if (r < nr) {
        const bf16* wr[NMAT];
#pragma unroll
        for (int q = 0; q < NMAT; ++q) wr[q] = st + ((size_t)q * RS + r) * K;
#pragma unroll 2
        for (int c = ks + lane * 8; c < ke; c += 256) {
          float wf[NMAT][8];
#pragma unroll
          for (int q = 0; q < NMAT; ++q) cvt8(*reinterpret_cast<const uint4*>(wr[q] + c), wf[q]);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float xf[8];
            cvt8(*reinterpret_cast<const uint4*>(xs + (size_t)m * K + c), xf);
#pragma unroll
            for (int q = 0; q < NMAT; ++q)
#pragma unroll
              for (int j = 0; j < 8; ++j) acc[q][m] = fmaf(wf[q][j], xf[j], acc[q][m]);
          }
        }
#pragma unroll
        for (int q = 0; q < NMAT; ++q)
#pragma unroll
          for (int m = 0; m < M; ++m) acc[q][m] = warp_sum(acc[q][m]);
      }
      if (wpr > 1) {
        if (lane == 0) {
#pragma unroll
          for (int q = 0; q < NMAT; ++q)
#pragma unroll
            for (int m = 0; m < M; ++m) part[warp][q][m] = acc[q][m];
        }
        named_sync(1, GV_CWARPS * 32);
        if (warp % wpr == 0 && r < nr) {
#pragma unroll
          for (int q = 0; q < NMAT; ++q)
#pragma unroll
            for (int m = 0; m < M; ++m) {
              float v = part[warp][q][m];
              for (int i = 1; i < wpr; ++i) v += part[warp + i][q][m];
              acc[q][m] = v;
            }
        }
        named_sync(1, GV_CWARPS * 32);
      }
      if (warp % wpr == 0 && r < nr) {
        const int n = n0 + r;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          if (lane == m) {
            float v;
            if (EPI == 0) {
              v = acc[0][m];
            } else if (EPI == 1) {
              v = b2f(a.res[(size_t)m * a.ldr + n]) + rbf(acc[0][m]);
            } else {
              const float g = rbf(acc[0][m]);
              const float u = rbf(acc[NMAT - 1][m]);
              v = silu_rbf(g) * u;
            }
            a.y[(size_t)m * a.ldy + n] = __float2bfloat16_rn(v);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}


// Standalone Qwen3 RMSNorm: one warp per row, 4 rows per CTA.  A lane keeps its units of the row in registers
// (RN_UNITS per lane covers K <= 32 * 8 * RN_UNITS columns) so the row is read from global memory once.
constexpr int RN_WARPS = 4, RN_UNITS = 16;
__global__ void __launch_bounds__(RN_WARPS * 32) rmsnorm_rows_kernel(const bf16* __restrict__ x, long ldx,
                                                                     const bf16* __restrict__ w, float eps,
                                                                     bf16* __restrict__ y, long ldy, int M, int K) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * RN_WARPS + (threadIdx.x >> 5);
  if (m >= M) return;
  const int nu = K >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)m * ldx);
  uint4 v[RN_UNITS];
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < RN_UNITS; ++i) {
    const int u = lane + 32 * i;
    if (u < nu) {
      v[i] = xr[u];
      acc = sumsq8(v[i], acc);
    }
  }
  const float r = rms_factor(warp_sum(acc), K, eps);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)m * ldy);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int i = 0; i < RN_UNITS; ++i) {
    const int u = lane + 32 * i;
    if (u < nu) yr[u] = rms_unit(v[i], wr[u], r);
  }
}

}  // namespace fb

namespace {
using namespace fb;

bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <int M, int EPI, bool NORM>
int launch_gemv_t(GemvArgs& a, cudaStream_t st) {
  auto kern = gemv_fma_kernel<M, EPI, NORM>;
  const size_t smem = (size_t)a.xs_bytes + (size_t)a.nstages * GV_STAGE_BYTES + 2 * GV_MAX_STAGES * 8 + 128;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_done[dev] < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("gemv: cudaFuncSetAttribute(%zu bytes): %s", smem, cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = (int)smem;
  }
  const int grid = a.N < fbh::grid_sms() ? a.N : fbh::grid_sms();
  void* args[] = {(void*)&a};
  return fbh::launch_pdl((const void*)kern, dim3(grid), dim3(GV_THREADS), smem, st, args, true);
}

template <int EPI, bool NORM>
int dispatch_m(GemvArgs& a, int M, cudaStream_t st) {
  a.M = M;
  if (M > 128) {
    // the prefill's dense GEMMs: the many-rows kernel in tiles of 128 rows, else blocks of 128 rows
    if (a.K % 64 == 0 && !NORM && g_rows_path) {
      const int rt = gemv_rows(a, EPI, st);
      if (rt != FB_ERR_UNSUPPORTED) {
        t_gemv_path = 3;
        return rt;
      }
    }
    for (int r0 = 0; r0 < M; r0 += 128) {
      GemvArgs b = a;
      b.x += (size_t)r0 * a.ldx;
      b.y += (size_t)r0 * a.ldy;
      if (b.res) b.res += (size_t)r0 * a.ldr;
      const int rc = dispatch_m<EPI, NORM>(b, M - r0 < 128 ? M - r0 : 128, st);
      if (rc) return rc;
    }
    return FB_OK;
  }
  if (M > 16) {
    // up to 128 rows: the tcgen05 kernel (MMA N = the rows); else row blocks through the paths below (16 rows, or
    // 8 / 4 / 2 / 1 for K % 64 != 0), each block streaming the weights again
    if (a.K % 64 == 0 && !NORM && g_rows_path) {
      const int rt = gemv_rows(a, EPI, st);
      if (rt != FB_ERR_UNSUPPORTED) {
        t_gemv_path = 3;
        return rt;
      }
    }
    if (a.K % 64 == 0) {
      const int rt = gemv_tc(a, EPI, NORM, st);
      if (rt != FB_ERR_UNSUPPORTED) {
        t_gemv_path = 2;
        return rt;
      }
    }
    for (int r0 = 0; r0 < M;) {
      int m = M - r0 < 16 ? M - r0 : 16;
      if (a.K % 64 != 0) {   // the scalar kernel's row counts: 8, 4, 2, 1
        m = 8;
        while (m > M - r0) m >>= 1;
      }
      GemvArgs b = a;
      b.x += (size_t)r0 * a.ldx;
      b.y += (size_t)r0 * a.ldy;
      if (b.res) b.res += (size_t)r0 * a.ldr;
      const int rc = dispatch_m<EPI, NORM>(b, m, st);
      if (rc) return rc;
      r0 += m;
    }
    return FB_OK;
  }
  if (a.K % 64 == 0) {
    int rt = gemv_tc(a, EPI, NORM, st);       // tcgen05 kernel (fb_gemv_tc.cu) when the shape suits it
    if (rt != FB_ERR_UNSUPPORTED) {
      t_gemv_path = 2;
      return rt;
    }
    t_gemv_path = 1;
    // x staged whole: 64 KB stages if three fit, else 32 KB stages if four fit (bytes in flight per SM set the
    // streaming rate of a small grid), else whichever fits; else (no norm) x in double-buffered column chunks,
    // 64 KB stages then 32 KB stages
    int rc = launch_mma_t<EPI, NORM>(a, st, 0, 3);
    if (rc == FB_ERR_UNSUPPORTED) rc = gemv_mma_narrow(a, EPI, NORM, st, 0, FB_GEMV_NARROW_MIN);
    if (rc == FB_ERR_UNSUPPORTED) rc = launch_mma_t<EPI, NORM>(a, st, 0, 2);
    if (rc == FB_ERR_UNSUPPORTED) rc = gemv_mma_narrow(a, EPI, NORM, st, 0, 2);
    if (rc == FB_ERR_UNSUPPORTED && !NORM) rc = launch_mma_t<EPI, NORM>(a, st, 1, 2);
    if (rc == FB_ERR_UNSUPPORTED && !NORM) rc = gemv_mma_narrow(a, EPI, NORM, st, 1, 2);
    return rc;
  }
  t_gemv_path = 0;
  switch (M) {
    case 1: return launch_gemv_t<1, EPI, NORM>(a, st);
    case 2: return launch_gemv_t<2, EPI, NORM>(a, st);
    case 3: return launch_gemv_t<3, EPI, NORM>(a, st);
    case 4: return launch_gemv_t<4, EPI, NORM>(a, st);
    case 8: return launch_gemv_t<8, EPI, NORM>(a, st);
    default: fbh::set_msg("gemv: M=%d rows not built for K %% 64 != 0 (1, 2, 3, 4, 8)", M); return FB_ERR_UNSUPPORTED;
  }
}

int common_checks(const void* x, int64_t ldx, int M, int K, const void* y, int64_t ldy) {
  FB_CHECK_ARG(x && y, "gemv: null x or y");
  FB_CHECK_ARG(M >= 1 && M <= GV_MAX_ROWS, "gemv: M=%d out of range 1..%d", M, GV_MAX_ROWS);
  FB_CHECK_ARG(K > 0 && K % 8 == 0, "gemv: K=%d must be a positive multiple of 8", K);
  FB_CHECK_ARG(ldx % 8 == 0 && ldy >= 1 && al16(x), "gemv: x row stride %lld must be a multiple of 8 and x 16B aligned",
               (long long)ldx);
  return FB_OK;
}

int setup_ring(GemvArgs& a, int M, int nmat) {
  a.err = fbh::device_err_ptr();
  if (a.K % 64 == 0) return FB_OK;  // tensor-core path: its ring is sized at launch
  const int row_bytes = nmat * a.K * 2;
  if (row_bytes > GV_STAGE_BYTES) {
    fbh::set_msg("gemv: K=%d too large for one stage (max %d)", a.K, GV_STAGE_BYTES / (2 * nmat));
    return FB_ERR_UNSUPPORTED;
  }
  a.RS = GV_STAGE_BYTES / row_bytes;
  if (a.RS > 16) a.RS = 16;
  if (M > 16) M = 16;   // more rows go through the tcgen05 kernel or in row blocks of 16
  a.xs_bytes = ((M * a.K * 2) + 127) / 128 * 128;
  int nst = (GV_SMEM_BUDGET - a.xs_bytes) / GV_STAGE_BYTES;
  if (nst < 2) nst = (200 * 1024 - a.xs_bytes) / GV_STAGE_BYTES;
  if (nst > GV_MAX_STAGES) nst = GV_MAX_STAGES;
  if (nst < 2) {
    fbh::set_msg("gemv: M*K = %d activations do not fit the shared-memory budget", M * a.K);
    return FB_ERR_UNSUPPORTED;
  }
  a.nstages = nst;
  a.err = fbh::device_err_ptr();
  return FB_OK;
}

}  // namespace

extern "C" int flashb_gemv_seg(const void* x, int64_t ldx, int M, int K, const void* nw, float eps, const void* W0,
                               int N0, const void* W1, int N1, const void* W2, int N2, void* y, int64_t ldy,
                               void* stream) {
  int rc = common_checks(x, ldx, M, K, y, ldy);
  if (rc) return rc;
  FB_CHECK_ARG(W0 && N0 > 0 && al16(W0), "gemv_seg: W0 missing or misaligned");
  FB_CHECK_ARG(N1 >= 0 && N2 >= 0 && (N1 == 0 || (W1 && al16(W1))) && (N2 == 0 || (W2 && al16(W2))),
               "gemv_seg: bad W1/W2 segment");
  FB_CHECK_ARG(!nw || al16(nw), "gemv_seg: norm weight misaligned");
  if (K % 64 == 0 && ((N1 && N0 % 8) || (N2 && (N0 + N1) % 8))) {
    // the tensor path's 8-row copies need segment boundaries at multiples of 8: one launch per segment instead
    bf16* yb = (bf16*)y;
    rc = flashb_gemv_seg(x, ldx, M, K, nw, eps, W0, N0, nullptr, 0, nullptr, 0, yb, ldy, stream);
    if (!rc && N1) rc = flashb_gemv_seg(x, ldx, M, K, nw, eps, W1, N1, nullptr, 0, nullptr, 0, yb + N0, ldy, stream);
    if (!rc && N2)
      rc = flashb_gemv_seg(x, ldx, M, K, nw, eps, W2, N2, nullptr, 0, nullptr, 0, yb + N0 + N1, ldy, stream);
    return rc;
  }
  GemvArgs a{};
  a.x = (const bf16*)x; a.ldx = (long)ldx; a.nw = (const bf16*)nw; a.eps = eps;
  a.W0 = (const bf16*)W0; a.W1 = N1 ? (const bf16*)W1 : a.W0; a.W2 = N2 ? (const bf16*)W2 : a.W0;
  a.N0 = N0; a.N1 = N1; a.K = K; a.N = N0 + N1 + N2;
  a.y = (bf16*)y; a.ldy = (long)ldy;
  if ((rc = setup_ring(a, M, 1))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return nw ? dispatch_m<0, true>(a, M, st) : dispatch_m<0, false>(a, M, st);
}

extern "C" int flashb_gemv_last_path(void) { return t_gemv_path; }

extern "C" int flashb_gemv_last_split(void) {
  return t_gemv_path == 2 ? fb::gemv_tc_last_split() : (t_gemv_path == 3 ? fb::gemv_rows_last_split() : 1);
}

extern "C" void flashb_set_gemv_rows_path(int enable) { g_rows_path = enable ? 1 : 0; }

extern "C" void flashb_set_gemv_split(int enable) { fb::gemv_tc_set_split_small(enable); }

extern "C" void flashb_set_gemv_trace(void* buf) { fb::gemv_tc_set_trace(buf); }

extern "C" int flashb_set_gemv_group_rows(int rows) {
  FB_CHECK_ARG(rows == 16 || rows == 32 || rows == 64 || rows == 128, "gemv: group rows %d not 16, 32, 64 or 128", rows);
  return fb::gemv_tc_set_group_rows(rows);
}

extern "C" int flashb_gemv_resid(const void* x, int64_t ldx, int M, int K, const void* W, int N, const void* res,
                                 int64_t ldr, void* y, int64_t ldy, void* stream) {
  int rc = common_checks(x, ldx, M, K, y, ldy);
  if (rc) return rc;
  FB_CHECK_ARG(W && N > 0 && al16(W) && res, "gemv_resid: bad W or res");
  GemvArgs a{};
  a.x = (const bf16*)x; a.ldx = (long)ldx;
  a.W0 = a.W1 = a.W2 = (const bf16*)W; a.N0 = N; a.N1 = 0; a.K = K; a.N = N;
  a.y = (bf16*)y; a.ldy = (long)ldy; a.res = (const bf16*)res; a.ldr = (long)ldr;
  if ((rc = setup_ring(a, M, 1))) return rc;
  return dispatch_m<1, false>(a, M, (cudaStream_t)stream);
}

extern "C" int flashb_gemv_gateup(const void* x, int64_t ldx, int M, int K, const void* nw, float eps, const void* Wg,
                                  const void* Wu, int N, void* y, int64_t ldy, void* stream) {
  int rc = common_checks(x, ldx, M, K, y, ldy);
  if (rc) return rc;
  FB_CHECK_ARG(Wg && Wu && N > 0 && al16(Wg) && al16(Wu), "gemv_gateup: bad Wg/Wu");
  FB_CHECK_ARG(!nw || al16(nw), "gemv_gateup: norm weight not 16B aligned");
  GemvArgs a{};
  a.x = (const bf16*)x; a.ldx = (long)ldx; a.nw = (const bf16*)nw; a.eps = eps;
  a.W0 = (const bf16*)Wg; a.W1 = (const bf16*)Wu; a.W2 = a.W0; a.N0 = N; a.N1 = 0; a.K = K; a.N = N;
  a.y = (bf16*)y; a.ldy = (long)ldy;
  if ((rc = setup_ring(a, M, 2))) return rc;
  return nw ? dispatch_m<2, true>(a, M, (cudaStream_t)stream) : dispatch_m<2, false>(a, M, (cudaStream_t)stream);
}

extern "C" int flashb_rmsnorm(const void* x, int64_t ldx, int M, int K, const void* w, float eps, void* y,
                              int64_t ldy, void* stream) {
  int rc = common_checks(x, ldx, M, K, y, ldy);
  if (rc) return rc;
  FB_CHECK_ARG(w && al16(w) && ldy % 8 == 0 && al16(y), "rmsnorm: bad weight or output stride");
  FB_CHECK_ARG(K <= 32 * 8 * RN_UNITS, "rmsnorm: K %d above %d", K, 32 * 8 * RN_UNITS);
  const bf16* xp = (const bf16*)x;
  const bf16* wp = (const bf16*)w;
  bf16* yp = (bf16*)y;
  long lx = (long)ldx, ly = (long)ldy;
  void* args[] = {(void*)&xp, (void*)&lx, (void*)&wp, (void*)&eps, (void*)&yp, (void*)&ly, (void*)&M, (void*)&K};
  return fbh::launch_pdl((const void*)rmsnorm_rows_kernel, dim3((M + RN_WARPS - 1) / RN_WARPS), dim3(RN_WARPS * 32),
                         0, (cudaStream_t)stream, args, true);
}
