// flashb: shared device helpers for the sm_100a kernels (bf16 conversion, bulk-copy/mbarrier pipeline, PDL,
// bounded waits, the device error word).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "flashb.h"

namespace fb {

typedef __nv_bfloat16 bf16;
constexpr unsigned FULL = 0xffffffffu;

// ------------------------------------------------------------------------------------------------ bf16 helpers
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// bf16(silu(g)) for the SwiGLU activations, g on the bf16 grid: g / (1 + e^-g) with the fast exponential and
// division intrinsics (a few fp32 ulps, below the bf16 rounding of the result except at rare ties).  The exact
// expf and IEEE division cost about 55 ns per value per thread on B200 (their special-case branches defeat
// interleaving), which made the SiLU the longest part of the many-rows GEMV epilogues.
__device__ __forceinline__ float silu_rbf(float g) { return rbf(__fdividef(g, 1.0f + __expf(-g))); }
__device__ __forceinline__ float b2f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float lo_f(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float hi_f(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ void cvt8(const uint4& v, float* f) {
  f[0] = lo_f(v.x); f[1] = hi_f(v.x); f[2] = lo_f(v.y); f[3] = hi_f(v.y);
  f[4] = lo_f(v.z); f[5] = hi_f(v.z); f[6] = lo_f(v.w); f[7] = hi_f(v.w);
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// ------------------------------------------------------------------------------------------------ memory ops
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {  // read-only, do not allocate in L1
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// mbarrier (CTA scope)
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Every device-side wait in this library is bounded in time.  On expiry the waiter records FB_ERR_TIMEOUT in the
// library's device error word (read by flashb_device_error) and its caller abandons the work.
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s

__device__ __forceinline__ void set_error(unsigned* err, unsigned code) {
  if (err) atomicCAS(err, 0u, code);
}

// Non-blocking test of a phase (no suspension window): the fast path of a wait whose phase is usually complete.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* err) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > WAIT_LIMIT_NS) {
      set_error(err, FB_ERR_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform bounded wait: every lane polls, the verdict is agreed by vote so the warp never splits.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, unsigned parity, unsigned* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(FULL, ok);
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast).  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch.  pdl_wait blocks until the preceding kernel in the stream has completed and its
// writes are visible; code before it may only read data that the preceding kernel does not write (weights, old KV
// slots).  pdl_trigger lets the next kernel's CTAs be scheduled; every kernel here issues it after its own pdl_wait,
// so when kernel N+1 starts, kernel N-1 has completed.  Both are no-ops for a launch without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// cp.async 16-byte global -> shared copy (bypasses L1), group commit / wait.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Named barrier over `nthreads` threads (multiple of 32).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace fb

// ------------------------------------------------------------------------------------------------ host side
namespace fbh {
// Thread-local last error message and the per-device error-word address (fb_api.cu).
void set_msg(const char* fmt, ...);
unsigned* device_err_ptr();  // error word of the current device (nullptr if unavailable)
int launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args, bool pdl,
               int cluster_x = 0);
bool pdl_enabled();
int num_sms();
int grid_sms();
// Tensor map of a row-major bf16 matrix [rows, K] (K % 64 == 0, base 16-byte aligned) viewed as
// [K / 64 column blocks][rows][64 columns], for 8-row boxes of kc columns with the 128-byte swizzle (fb_stream.cuh
// TMA stages).  Encoded through the driver's cuTensorMapEncodeTiled (fetched once, no link to libcuda) and cached
// per (base, rows, K, kc).  Returns FB_OK, or FB_ERR_ARG / FB_ERR_CUDA with the message set.
int tmap_rows(CUtensorMap* out, const void* base, long long rows, int K, int kc);
// General form: [rows, K] bf16 with row stride ld elements (0: K), viewed as [K / inner][rows][inner]; boxes of
// box_rows rows x box_blocks blocks of `inner` columns, 128-byte swizzle (inner = 64) or none.
int tmap_box(CUtensorMap* out, const void* base, long long rows, int K, int inner, int box_rows, int box_blocks,
             bool swizzle128, long long ld = 0);  // num_sms(), or the calling thread's SM budget when one is set (flashb_set_sm_budget)
// Tensor map of an LN12 matrix's data bytes (N rows, K % 1024 == 0): per row and 1024-column group three 512-byte
// slots (low bytes of chunks 0-1, of chunks 2-3, the nibble words), viewed as [N][K / 1024][3][512 B]; boxes of
// box_rows rows x 3 slots x 128 bytes (the 8 lanes of one lane octet: 256 columns of the group).  Cached per
// (base, N, K, box_rows).
int tmap_ln12(CUtensorMap* out, const void* data, long long N, int K, int box_rows);
// Tensor map of a head-major bf16 cache [B][NH][S][128] (element strides sl between rows, sh between heads, sb
// between batch rows; sl, sh, sb multiples of 8) viewed as [B][NH][16 chunks of 8 dims][S][8], boxes of 128 rows x
// all 16 chunks of one (batch row, head): shared memory [chunk][row][16 B], the canonical no-swizzle core-matrix
// layout of a K-major tile with 2048 bytes between K chunks (or of an MN-major one, 2048 bytes between dimension
// groups).  Rows past S read as zeros.  Cached per (base, shape, strides).
int tmap_heads(CUtensorMap* out, const void* base, int B, int NH, long long S, long long sl, long long sh,
               long long sb);
}  // namespace fbh

#define FB_CHECK_ARG(cond, ...)          \
  do {                                   \
    if (!(cond)) {                       \
      fbh::set_msg(__VA_ARGS__);         \
      return FB_ERR_ARG;                 \
    }                                    \
  } while (0)
