// flashb: the tensor-core GEMV kernel (see fb_gemv.cu for the semantics), shared by two translation units that
// build it for two stage widths: fb_gemv.cu (FB_ST_KC = 2048, 64 KB stages) and fb_gemv_narrow.cu (1024, 32 KB
// stages, used when the activation rows leave no room for two 64 KB stages).  Both use TMA stages (FB_ST_TMA 1):
// the weight matrices reach the kernel as tensor maps inside the argument block.  The kernel and its launcher live
// in the stage inline namespace of fb_stream.cuh; the argument block and the row helpers do not depend on it.
#pragma once
#define FB_ST_TMA 1
#include "fb_stream.cuh"

namespace fb {

#ifndef FB_GEMV_ARGS_DEFINED
#define FB_GEMV_ARGS_DEFINED
struct alignas(64) GemvArgs {
  CUtensorMap tm[3];   // W0, W1, W2 as [K / 64][rows][64] bf16, 8-row boxes of ST_KC columns (tensor path)
  const bf16* x;
  long ldx;
  const bf16* nw;
  float eps;
  const bf16* W0;
  const bf16* W1;
  const bf16* W2;
  int N0, N1;  // segment boundaries (EPI 0/1); EPI 2: W0 = gate, W1 = up
  int K, N;
  bf16* y;
  long ldy;
  const bf16* res;
  long ldr;
  int M;        // activation rows (tensor-core path)
  int RS;       // units (output rows) per stage
  int nstages;  // ring depth
  int xs_bytes; // shared bytes reserved for x
  int xchunk;   // 1: x staged per column chunk (too large to stage whole)
  unsigned* err;
};

// Row n of matrix `mat` (EPI 2: 0 = gate, 1 = up; else the q|k|v-style segment holding row n).
template <int EPI>
__device__ __forceinline__ const bf16* gv_row(const GemvArgs& a, int n, int mat) {
  if (EPI == 2) return (mat == 0 ? a.W0 : a.W1) + (size_t)n * a.K;
  if (n < a.N0) return a.W0 + (size_t)n * a.K;
  if (n < a.N0 + a.N1) return a.W1 + (size_t)(n - a.N0) * a.K;
  return a.W2 + (size_t)(n - a.N0 - a.N1) * a.K;
}
// First row index after n at which the segment (and so the contiguous source range) changes.
template <int EPI>
__device__ __forceinline__ int gv_seg_end(const GemvArgs& a, int n) {
  if (EPI == 2) return a.N;
  if (n < a.N0) return a.N0;
  if (n < a.N0 + a.N1) return a.N0 + a.N1;
  return a.N;
}


#endif

// The tcgen05 GEMV (fb_gemv_tc.cu); FB_ERR_UNSUPPORTED when the shape does not suit it.  gemv_tc_last_split: the
// CTAs per block (split K) of this thread's last tcgen05 launch.
int gemv_tc(GemvArgs& a, int epi, bool norm, cudaStream_t st);
int gemv_tc_last_split();
void gemv_tc_set_split_small(int on);
int gemv_tc_set_group_rows(int rows);
void gemv_tc_set_trace(void* buf);
unsigned long long* gemv_trace_buf();   // the timeline buffer of flashb_set_gemv_trace, or null
// The many-rows tcgen05 GEMV (fb_gemv_rows.cu, 17..128 rows, no norm); FB_ERR_UNSUPPORTED when the shape does not
// suit it.  gemv_rows_last_split: the cluster size of this thread's last launch of it.
int gemv_rows(GemvArgs& a, int epi, cudaStream_t st);
int gemv_rows_last_split();

// Launches the 32 KB-stage build (fb_gemv_narrow.cu); epi / norm select the instantiation, xchunk the staging.
int gemv_mma_narrow(GemvArgs& a, int epi, bool norm, cudaStream_t st, int xchunk, int min_nst);

inline namespace FB_ST_NS {

// Tensor-core path (K % 64 == 0): a producer warp streams stages of 16 weight rows x ST_KC columns, two 8-row TMA
// tensor copies each, into a ring of mbarrier-tracked slots; 8 consumer warps run mma.sync m16n8k16 on them
// (fb_stream.cuh).  NMAT = 2 (gate/up): rows 0..7 of a stage are gate rows of 8 output units, rows 8..15 the
// matching up rows, so a unit's gate and up sums land in the same reduction slots.  A CTA's output rows start at a
// multiple of 8, so no 8-row copy straddles a segment boundary (the host keeps those multiples of 8).
constexpr int GM_MAX_STAGES = 6;
constexpr int GM_THREADS = (ST_CWARPS + 1) * 32;

// Tensor map and first row of output rows n .. n + 7 (n a multiple of 8; segment boundaries are multiples of 8).
__device__ __forceinline__ TmaRows gv_tma_rows(const GemvArgs& a, int n) {
  if (n < a.N0) return TmaRows{&a.tm[0], n};
  if (n < a.N0 + a.N1) return TmaRows{&a.tm[1], n - a.N0};
  return TmaRows{&a.tm[2], n - a.N0 - a.N1};
}

// NT tiles of 8 activation rows (M <= 8 NT).  a.xchunk: x does not fit whole, so it is staged per column chunk
// (ST_KC columns, double-buffered, the next chunk in flight while this one is multiplied); only without NORM.
template <int EPI, bool NORM, int NT>
__global__ void __launch_bounds__(GM_THREADS) gemv_mma_kernel(const __grid_constant__ GemvArgs a) {
  constexpr int NMAT = EPI == 2 ? 2 : 1;
  constexpr int UG = ST_ROWS / NMAT;  // output units per row group
  constexpr int MS = 8 * NT;          // activation-row slots per reduced output row
  extern __shared__ __align__(128) unsigned char smem[];
  const int M = a.M, K = a.K, NST = a.nstages;
  const int x_pitch = a.xchunk ? ST_KC * 2 + 16 : K * 2 + 16;
  unsigned char* xs = smem;
  unsigned char* zero16 = smem + a.xs_bytes;
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(zero16 + 128) + (ST_ALIGN - 1)) & ~uintptr_t(ST_ALIGN - 1));
  float* red = reinterpret_cast<float*>(ring + (size_t)NST * ST_BYTES);
  float* sums = red + ST_CWARPS * 128 * NT;
  uint64_t* full = reinterpret_cast<uint64_t*>(sums + 128 * NT);
  uint64_t* empty = full + GM_MAX_STAGES;
  __shared__ float rfac[MS];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, bid = blockIdx.x;
  const int n8 = (a.N + 7) >> 3;
  const int u0 = min(a.N, 8 * (int)((long long)n8 * bid / G));
  const int u1 = min(a.N, 8 * (int)((long long)n8 * (bid + 1) / G));
  const int ngroups = (u1 - u0 + UG - 1) / UG;
  const int nkc = (K + ST_KC - 1) / ST_KC;
  const int T = ngroups * nkc;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ST_CWARPS);
    }
    fence_mbar_init();
  }
  if (tid < 32) reinterpret_cast<uint32_t*>(zero16)[tid] = 0u;
  __syncthreads();

  if (warp == ST_CWARPS) {
    // ------------------------------------------------------------ producer: weights only, runs before pdl_wait
    if (lane < 3) tma_prefetch_map(&a.tm[lane]);
    int issued = 0;
    for (int t = 0; t < T; ++t) {
      const int s = t % NST;
      if (t >= NST && !mbar_wait_warp(&empty[s], ((t / NST) - 1) & 1, a.err)) break;
      const int g = t / nkc, kc = t % nkc;
      const int n0 = u0 + g * UG;
      const int nu = min(UG, u1 - n0);
      if (lane == 0) {
        TmaRows lo, hi;
        if (EPI == 2) {
          lo = TmaRows{&a.tm[0], n0};
          hi = TmaRows{&a.tm[1], n0};
        } else {
          lo = gv_tma_rows(a, n0);
          hi = nu > 8 ? gv_tma_rows(a, n0 + 8) : TmaRows{nullptr, 0};
        }
        tma_stage(ring + (size_t)s * ST_BYTES, lo, hi, kc, &full[s]);
      }
      __syncwarp();
      ++issued;
    }
    for (int t = max(0, issued - NST); t < issued; ++t)
      if (!mbar_wait_warp(&full[t % NST], (t / NST) & 1, a.err)) break;
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  pdl_trigger();
  const int ctid = tid;
  if (!a.xchunk) {
    // stage every x row, then the row factors and the norm in place
    const int nu = K >> 3;
    const PitchOff off{x_pitch};
    for (int i = ctid; i < M * nu; i += ST_CWARPS * 32) {
      const int m = i / nu, u = i - m * nu;
      *reinterpret_cast<uint4*>(xs + off(m, u)) =
          *reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + (size_t)u * 8);
    }
    named_sync(1, ST_CWARPS * 32);
    if (NORM) {
      rms_row_factors(xs, off, M, K, a.eps, rfac, warp, ST_CWARPS);
      named_sync(1, ST_CWARPS * 32);
      rms_rows_apply(xs, off, M, K, a.nw, rfac, ctid, ST_CWARPS * 32);
      named_sync(1, ST_CWARPS * 32);
    }
  }

  int t = 0;
  const int cbuf = M * x_pitch;                 // bytes of one x chunk buffer (chunked mode)
  auto load_chunk = [&](int kc) {               // x[:, kc * ST_KC ..] -> chunk buffer kc & 1 (chunked mode)
    const int k0 = kc * ST_KC, kvc = min(ST_KC, K - k0) >> 3;
    unsigned char* dst = xs + (size_t)(kc & 1) * cbuf;
    for (int i = ctid; i < M * kvc; i += ST_CWARPS * 32) {
      const int m = i / kvc, j = i - m * kvc;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + (size_t)m * x_pitch + j * 16)),
                   "l"(a.x + (size_t)m * a.ldx + k0 + (size_t)j * 8)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int g = 0; g < ngroups; ++g) {
    const int n0 = u0 + g * UG;
    const int nu = min(UG, u1 - n0);
    float c[NT][4];
#pragma unroll
    for (int q = 0; q < NT; ++q) c[q][0] = c[q][1] = c[q][2] = c[q][3] = 0.f;
    if (a.xchunk) load_chunk(0);
    for (int kc = 0; kc < nkc; ++kc, ++t) {
      const int s = t % NST;
      const unsigned char* xk = xs;
      int kx = kc * ST_KC;
      if (a.xchunk) {
        if (kc + 1 < nkc) {
          load_chunk(kc + 1);
          asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
          asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        named_sync(1, ST_CWARPS * 32);
        xk = xs + (size_t)(kc & 1) * cbuf;
        kx = 0;
      }
      if (!mbar_wait_warp(&full[s], (t / NST) & 1, a.err)) return;
      stage_mma_nt<NT>(ring + (size_t)s * ST_BYTES, min(ST_KC, K - kc * ST_KC), xk, x_pitch, M, kx, zero16, c);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (a.xchunk) named_sync(1, ST_CWARPS * 32);   // chunk buffer kc & 1 is refilled two chunks later
    }
    reduce_warps_nt<NT>(c, red, sums, 1);
    if (ctid < nu * M) {
      const int i = ctid / M, m = ctid - i * M;
      const int n = n0 + i;
      float v;
      if (EPI == 0) {
        v = sums[i * MS + m];
      } else if (EPI == 1) {
        v = b2f(a.res[(size_t)m * a.ldr + n]) + rbf(sums[i * MS + m]);
      } else {
        const float gg = rbf(sums[i * MS + m]);
        const float uu = rbf(sums[(i + 8) * MS + m]);
        v = silu_rbf(gg) * uu;
      }
      a.y[(size_t)m * a.ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

// Ring depth and launch for this stage width: x whole (xchunk = 0) or in double-buffered column chunks (1, only
// without NORM).  Returns FB_ERR_UNSUPPORTED when fewer than two ring stages fit.
template <int EPI, bool NORM, int NT>
inline int launch_mma_nt(GemvArgs& a, cudaStream_t st, int xchunk, int min_nst) {
  auto kern = gemv_mma_kernel<EPI, NORM, NT>;
  a.xchunk = xchunk;
  a.xs_bytes = xchunk ? ((2 * a.M * (ST_KC * 2 + 16)) + 127) / 128 * 128 : ((a.M * (a.K * 2 + 16)) + 127) / 128 * 128;
  const size_t fixed = (size_t)a.xs_bytes + 128 + ST_ALIGN + ST_CWARPS * 128 * 4 * NT + 128 * 4 * NT +
                       2 * GM_MAX_STAGES * 8;
#ifndef FB_GM_BUDGET
#define FB_GM_BUDGET 220000
#endif
  int nst = fixed < FB_GM_BUDGET ? (int)((FB_GM_BUDGET - fixed) / ST_BYTES) : 0;
  if (nst < 3 && fixed < 210 * 1024) nst = (int)((210 * 1024 - fixed) / ST_BYTES);
  if (nst > GM_MAX_STAGES) nst = GM_MAX_STAGES;
  if (nst < min_nst) {
    fbh::set_msg("gemv: M*K = %d activations leave fewer than %d ring stages", a.M * a.K, min_nst);
    return FB_ERR_UNSUPPORTED;
  }
  a.nstages = nst;
  const size_t smem = fixed + (size_t)nst * ST_BYTES;
  // tensor maps of the weight matrices (EPI 2: gate, up; else the q|k|v-style segments)
  const int nseg[3] = {EPI == 2 ? a.N : a.N0, EPI == 2 ? a.N : a.N1, EPI == 2 ? 0 : a.N - a.N0 - a.N1};
  const bf16* wseg[3] = {a.W0, a.W1, a.W2};
  for (int i = 0; i < 3; ++i) {
    if (nseg[i] <= 0) continue;
    const int rc = fbh::tmap_rows(&a.tm[i], wseg[i], nseg[i], a.K, ST_KC);
    if (rc != FB_OK) return rc;
  }
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
  return fbh::launch_pdl((const void*)kern, dim3(grid), dim3(GM_THREADS), smem, st, args, true);
}

// This build's launch for M <= 16 rows: one or two activation tiles, x whole or chunked.
template <int EPI, bool NORM>
inline int launch_mma_t(GemvArgs& a, cudaStream_t st, int xchunk = 0, int min_nst = 2) {
  if (xchunk && NORM) {
    fbh::set_msg("gemv: chunked activations need the norm-free kernel");
    return FB_ERR_UNSUPPORTED;
  }
  if (a.M <= 8) return launch_mma_nt<EPI, NORM, 1>(a, st, xchunk, min_nst);
  return launch_mma_nt<EPI, NORM, 2>(a, st, xchunk, min_nst);
}

}  // inline namespace
}  // namespace fb
