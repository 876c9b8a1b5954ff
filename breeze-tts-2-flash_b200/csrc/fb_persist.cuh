// flashb: building blocks of the persistent (one launch per step) kernels: a bounded grid barrier and the
// producer / consumer halves of a streamed GEMV task over the fb_stream.cuh ring.
//
// A persistent kernel runs one CTA per SM (cooperative launch, so all CTAs are resident).  Warps 0..7 consume, warp
// 8 produces: it walks the kernel's static list of GEMV tasks and streams this CTA's row slice of every weight
// matrix into the ring, stopping only when the ring is full.  Weights never depend on activations, so the producer
// keeps streaming while the consumers wait at a grid barrier; the ring depth (up to ~200 KB per SM) covers the
// barrier latency.
#pragma once
#include "fb_stream.cuh"

#ifndef FB_PK_MAX_STAGES
#define FB_PK_MAX_STAGES 4
#endif

namespace fb {
inline namespace FB_ST_NS {

constexpr int PK_MAX_STAGES = FB_PK_MAX_STAGES;
constexpr int PK_CONSUMERS = ST_CWARPS * 32;        // 256
constexpr int PK_THREADS = PK_CONSUMERS + 32;       // + producer warp

// Grid barrier state (zero-initialised by the caller).  `count` only grows during a launch; the last CTA to leave the
// kernel resets it (grid_exit), so every launch starts from zero.
struct GridBar {
  unsigned count;
  unsigned exitc;
  unsigned abort;
  unsigned pad;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier over the consumer warps of every CTA: arrival is one fire-and-forget release-add on a monotonic counter,
// completion of barrier number `epoch` is count >= epoch * gridDim.x (observed with acquire loads).  The critical
// path is one add plus one poll round trip through L2.  Waits are bounded (`limit` ns); on expiry the waiter records
// FB_ERR_TIMEOUT and sets the abort flag; a waiter that finds the flag set (another CTA's expiry, or the host's
// request) records FB_ERR_ABORTED.  Either way every CTA returns false and the kernel winds down (the host then
// re-zeroes the state).
__device__ __noinline__ bool grid_sync_n(GridBar* gb, unsigned epoch, unsigned* err, int* s_flag, uint64_t limit) {
  named_sync(2, PK_CONSUMERS);
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = epoch * gridDim.x;
    __threadfence();
    red_release_add(&gb->count, 1u);
    // the abort word is read at every barrier (both loads in flight together), so a request that arrives before
    // the waits are long still stops the frame at its next barrier
    const unsigned cnt = ld_acquire_u32(&gb->count), ab = ld_acquire_u32(&gb->abort);
    if (ab) {
      set_error(err, FB_ERR_ABORTED);
      ok = 0;
    } else if (cnt < target) {
      const uint64_t t0 = globaltimer();
      int spins = 0;
      while (ld_acquire_u32(&gb->count) < target) {
        if (++spins == 256) {
          spins = 0;
          if (ld_acquire_u32(&gb->abort)) {
            set_error(err, FB_ERR_ABORTED);
            ok = 0;
            break;
          }
          if (globaltimer() - t0 > limit) {
            set_error(err, FB_ERR_TIMEOUT);
            atomicExch(&gb->abort, 1u);
            ok = 0;
            break;
          }
        }
      }
    }
    *s_flag = ok;
  }
  named_sync(2, PK_CONSUMERS);
  return *s_flag != 0;
}
// Not inlined: a persistent kernel calls it at ~20 sites, and its code must stay small enough to remain in the
// instruction cache across a whole step (cold code re-fetched from L2 costs microseconds per phase).
__device__ __forceinline__ bool grid_sync(GridBar* gb, unsigned& epoch, unsigned* err, int* s_flag,
                                          uint64_t limit = WAIT_LIMIT_NS) {
  ++epoch;
  return grid_sync_n(gb, epoch, err, s_flag, limit);
}

// Called once by consumer thread 0 of every CTA after its last barrier: the last CTA out resets the barrier.
// Every CTA increments `exitc` only after it has observed the final barrier, so the reset races with no waiter.
__device__ __forceinline__ void grid_exit(GridBar* gb) {
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&gb->exitc, 1u) == gridDim.x - 1) {
      atomicExch(&gb->count, 0u);
      atomicExch(&gb->exitc, 0u);
    }
  }
}

__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The ring of one persistent CTA.  `quit` (shared memory, may be null): set by the consumers when they stop early
// (a barrier gave up); the producer then abandons its wait for a free slot without recording an error.
struct Ring {
  unsigned char* base;
  uint64_t* full;
  uint64_t* empty;
  int nst;
  volatile int* quit;
};

// The producer's wait for a free ring slot (warp-uniform): bounded like every wait, and abandoned once the
// consumers have stopped.
__device__ __forceinline__ bool ring_wait_empty(const Ring& rg, int s, unsigned parity, unsigned* err) {
  bool ok = mbar_try_wait(&rg.empty[s], parity);
  if (!ok) {
    const uint64_t t0 = globaltimer();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 64 && !ok; ++i) ok = mbar_try_wait(&rg.empty[s], parity);
      if (ok || (rg.quit && *rg.quit)) break;
      if (globaltimer() - t0 > WAIT_LIMIT_NS) {
        set_error(err, FB_ERR_TIMEOUT);
        break;
      }
    }
  }
  return __all_sync(FULL, ok);
}

// A streamed GEMV task: `units` output units over K columns; NMAT = 2 pairs each unit with a second weight row
// (gate/up, or the two rotary halves of a q/k head dimension).  Row pointers come from a functor row(n, mat).
// CTA c owns units [units * c / G, units * (c + 1) / G); with TMA stages the split is in blocks of 8 units, so
// every 8-row tensor copy starts at a multiple of 8 and never straddles a segment or head boundary that is one.
__device__ __forceinline__ void task_range(int units, int& u0, int& u1) {
#if FB_ST_TMA
  const int n8 = (units + 7) >> 3;
  u0 = min(units, 8 * (int)((long long)n8 * blockIdx.x / gridDim.x));
  u1 = min(units, 8 * (int)((long long)n8 * (blockIdx.x + 1) / gridDim.x));
#else
  u0 = (int)((long long)units * blockIdx.x / gridDim.x);
  u1 = (int)((long long)units * (blockIdx.x + 1) / gridDim.x);
#endif
}

#if !FB_ST_TMA
// Producer half of one 16-row group: stream its nkc column chunks; `row` is this lane's weight row (lanes < nrows,
// others pass nullptr).  Returns the new stage counter, or -1 on timeout.  Not inlined (one copy for every task).
__device__ __noinline__ int produce_group(Ring rg, int t, const bf16* row, int nrows, int K, unsigned* err) {
  const int lane = threadIdx.x & 31;
  const int nkc = (K + ST_KC - 1) / ST_KC;
  for (int kc = 0; kc < nkc; ++kc, ++t) {
    const int s = t % rg.nst;
    if (t >= rg.nst && !ring_wait_empty(rg, s, ((t / rg.nst) - 1) & 1, err)) return -1;
    const int k0 = kc * ST_KC;
    const int kw = min(ST_KC, K - k0);
    unsigned char* st = rg.base + (size_t)s * ST_BYTES;
    if (lane == 0) mbar_arrive_expect_tx(&rg.full[s], (unsigned)(nrows * kw * 2));
    __syncwarp();
    if (row) bulk_g2s(st + lane * ST_PITCH, row + k0, (unsigned)(kw * 2), &rg.full[s]);
  }
  return t;
}

// Producer half: stream this CTA's stages of the task; t is the running stage counter.  Returns false on timeout.
// NMAT = 2 pairs each unit with a second matrix row: lanes 0-7 carry matrix 0, lanes 8-15 matrix 1.
template <int NMAT, typename RowFn>
__device__ __forceinline__ bool produce_task(Ring& rg, int& t, int units, int K, RowFn row, unsigned* err) {
  constexpr int UG = ST_ROWS / NMAT;
  const int lane = threadIdx.x & 31;
  int u0, u1;
  task_range(units, u0, u1);
  for (int n0 = u0; n0 < u1; n0 += UG) {
    const int nu = min(UG, u1 - n0);
    const int i = lane % UG, mat = lane / UG;
    const bf16* r = (lane < ST_ROWS && i < nu) ? row(n0 + i, mat) : nullptr;
    t = produce_group(rg, t, r, nu * NMAT, K, err);
    if (t < 0) return false;
  }
  return true;
}

#endif

#if FB_ST_TMA
// Producer half of one 16-row group with TMA stages: rows 0..7 from `lo`, rows 8..15 from `hi` (either may be
// empty), every ST_KC column chunk.  Lane 0 issues; returns the new stage counter, or -1 on timeout.
__device__ __noinline__ int produce_group_tma(Ring rg, int t, TmaRows lo, TmaRows hi, int K, unsigned* err) {
  const int lane = threadIdx.x & 31;
  const int nkc = (K + ST_KC - 1) / ST_KC;
  for (int kc = 0; kc < nkc; ++kc, ++t) {
    const int s = t % rg.nst;
    if (t >= rg.nst && !ring_wait_empty(rg, s, ((t / rg.nst) - 1) & 1, err)) return -1;
    if (lane == 0) tma_stage(rg.base + (size_t)s * ST_BYTES, lo, hi, kc, &rg.full[s]);
    __syncwarp();
  }
  return t;
}

// Producer half with TMA stages.  src(n, mat) is the tensor map and first row of the 8 rows of units n .. n + 7 of
// matrix mat (n a multiple of 8).  NMAT = 1: a group is 16 units, rows 0..7 units n0.., rows 8..15 units n0 + 8..;
// NMAT = 2: a group is 8 units, rows 0..7 from matrix 0, rows 8..15 the same units of matrix 1.
template <int NMAT, typename SrcFn>
__device__ __forceinline__ bool produce_task_tma(Ring& rg, int& t, int units, int K, SrcFn src, unsigned* err) {
  constexpr int UG = ST_ROWS / NMAT;
  int u0, u1;
  task_range(units, u0, u1);
  for (int n0 = u0; n0 < u1; n0 += UG) {
    const int nu = min(UG, u1 - n0);
    const TmaRows lo = src(n0, 0);
    const TmaRows hi = NMAT == 2 ? src(n0, 1) : (nu > 8 ? src(n0 + 8, 0) : TmaRows{nullptr, 0});
    t = produce_group_tma(rg, t, lo, hi, K, err);
    if (t < 0) return false;
  }
  return true;
}
#endif

// L2 prefetch of this CTA's slice of a task (one bulk prefetch per weight row).  Measured on the backbone step it
// does not pay off (the critical path is latency, not bandwidth), so the step kernels do not call it; kept as a tool.
template <int NMAT, typename RowFn>
__device__ __forceinline__ void prefetch_task(int units, int K, RowFn row) {
  const int lane = threadIdx.x & 31;
  int u0, u1;
  task_range(units, u0, u1);
  const int n = (u1 - u0) * NMAT;
  for (int i = lane; i < n; i += 32) prefetch_l2(row(u0 + i / NMAT, i % NMAT), (unsigned)(K * 2));
}

// Consumer half of one 16-row group: multiply its nkc stages by the activation rows xs (M <= 8 NT rows, byte pitch
// x_pitch), release them, and sum the 8 warps' partials into sums[r * 8 NT + m] (r < 16).  With xg != nullptr the
// activations are too large to stage whole: each ST_KC-column chunk of the global rows xg (row stride ldx) is
// brought into one of two chunk buffers at xs (pitch x_pitch = ST_KC * 2 + 16), the next one in flight while this
// one is multiplied.  Returns the new stage counter, or -1 on timeout.  Not inlined: one copy per NT.
template <int NT>
__device__ __noinline__ int consume_group_nt(Ring rg, int t, int K, const unsigned char* xs, int x_pitch, int M,
                                             const unsigned char* zero16, float* red, float* sums, unsigned* err,
                                             const bf16* xg, long ldx) {
  const int lane = threadIdx.x & 31;
  const int nkc = (K + ST_KC - 1) / ST_KC;
  const int cbuf = M * x_pitch;
  auto load_chunk = [&](int kc) {
    const int k0 = kc * ST_KC, kvc = min(ST_KC, K - k0) >> 3;
    unsigned char* dst = const_cast<unsigned char*>(xs) + (size_t)(kc & 1) * cbuf;
    for (int i = threadIdx.x; i < M * kvc; i += PK_CONSUMERS) {
      const int m = i / kvc, j = i - m * kvc;
      cp_async16(dst + (size_t)m * x_pitch + j * 16, xg + (size_t)m * ldx + k0 + (size_t)j * 8);
    }
    cp_async_commit();
  };
  float c[NT][4];
#pragma unroll
  for (int q = 0; q < NT; ++q) c[q][0] = c[q][1] = c[q][2] = c[q][3] = 0.f;
  if (xg) load_chunk(0);
  for (int kc = 0; kc < nkc; ++kc, ++t) {
    const int s = t % rg.nst;
    const unsigned char* xk = xs;
    int kx = kc * ST_KC;
    if (xg) {
      if (kc + 1 < nkc) {
        load_chunk(kc + 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      named_sync(1, PK_CONSUMERS);
      xk = xs + (size_t)(kc & 1) * cbuf;
      kx = 0;
    }
    if (!mbar_wait_warp(&rg.full[s], (t / rg.nst) & 1, err)) return -1;
    stage_mma_nt<NT>(rg.base + (size_t)s * ST_BYTES, min(ST_KC, K - kc * ST_KC), xk, x_pitch, M, kx, zero16, c);
    __syncwarp();
    if (lane == 0) mbar_arrive(&rg.empty[s]);
    if (xg) named_sync(1, PK_CONSUMERS);        // chunk buffer kc & 1 is refilled two chunks later
  }
  reduce_warps_nt<NT>(c, red, sums, 1);
  return t;
}

// Consumer half: every 16-row group of the task through consume_group_nt, then epi(n0, nu, sums, tid).  All 256
// consumer threads call it.  Chunked activations (xg) need a task of one row group per CTA or accept re-loading.
template <int NMAT, int NT = 1, typename EpiFn>
__device__ __forceinline__ bool consume_task(Ring& rg, int& t, int units, int K, const unsigned char* xs, int x_pitch,
                                             int M, const unsigned char* zero16, float* red, float* sums, EpiFn epi,
                                             unsigned* err, const bf16* xg = nullptr, long ldx = 0) {
  constexpr int UG = ST_ROWS / NMAT;
  int u0, u1;
  task_range(units, u0, u1);
  for (int n0 = u0; n0 < u1; n0 += UG) {
    const int nu = min(UG, u1 - n0);
    t = consume_group_nt<NT>(rg, t, K, xs, x_pitch, M, zero16, red, sums, err, xg, ldx);
    if (t < 0) return false;
    epi(n0, nu, sums, (int)threadIdx.x);
  }
  return true;
}

// Byte offset of 16-byte unit j (columns 8 j .. 8 j + 7) of staged activation row m.  x_pitch > 0: rows at that
// pitch.  x_pitch == 0: the tcgen05 B-operand layout (canonical K-major, 128-byte swizzle): 64-column blocks of
// 16 rows x 128 B, unit j of row m at unit (j % 8) ^ (m % 8) of its 128-byte row.
__device__ __forceinline__ uint32_t xs_off(int m, int j, int x_pitch) {
  if (x_pitch) return (uint32_t)(m * x_pitch + j * 16);
  return (uint32_t)(((j >> 3) << 11) + (m << 7) + (((j & 7) ^ (m & 7)) << 4));
}

// Offset functor for xs_off (either staged layout).
struct StagedOff {
  int pitch;
  __device__ __forceinline__ uint32_t operator()(int m, int u) const { return xs_off(m, u, pitch); }
};

// Per-row RMS factors of M <= 16 staged rows (one warp per row over the consumer warps), then a consumer barrier.
__device__ __noinline__ void row_rms(const unsigned char* xs, int x_pitch, int M, int K, float eps, float* rs) {
  rms_row_factors(xs, StagedOff{x_pitch}, M, K, eps, rs, threadIdx.x >> 5, ST_CWARPS);
  named_sync(1, PK_CONSUMERS);
}

// The eager Qwen3 RMSNorm in place on staged rows, factors from row_rms.
__device__ __forceinline__ void apply_rms(unsigned char* xs, int x_pitch, int M, int K, const bf16* nw,
                                          const float* rs) {
  rms_rows_apply(xs, StagedOff{x_pitch}, M, K, nw, rs, threadIdx.x, PK_CONSUMERS);
}

// Stage rows [0, M) (M <= 16) of a global bf16 activation matrix (row stride ld) into xs, optionally applying the
// eager Qwen3 RMSNorm with weight nw.  Cross-CTA data: copied with cp.async.cg (L2 only), every chunk in flight at
// once (one round trip).  nred holds at least 16 floats.
__device__ __noinline__ void load_x(unsigned char* xs, int x_pitch, const bf16* x, long ld, int M, int K,
                                    const bf16* nw, float eps, float* nred) {
  const int kv = K >> 3;
  if (kv <= PK_CONSUMERS && PK_CONSUMERS % kv == 0) {
    // one unit column per thread, the rows without divisions
    const int j = threadIdx.x % kv, dm = PK_CONSUMERS / kv;
#pragma unroll 4
    for (int m = threadIdx.x / kv; m < M; m += dm) cp_async16(xs + xs_off(m, j, x_pitch), x + (size_t)m * ld + (size_t)j * 8);
  } else {
    for (int i = threadIdx.x; i < M * kv; i += PK_CONSUMERS) {
      const int m = i / kv, j = i - m * kv;
      cp_async16(xs + xs_off(m, j, x_pitch), x + (size_t)m * ld + (size_t)j * 8);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  named_sync(1, PK_CONSUMERS);
  if (nw) {
    row_rms(xs, x_pitch, M, K, eps, nred);
    apply_rms(xs, x_pitch, M, K, nw, nred);
    named_sync(1, PK_CONSUMERS);
  }
}

}  // inline namespace
}  // namespace fb
