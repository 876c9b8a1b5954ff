// flashb: tcgen05 building blocks shared by the tensor-core GEMV (fb_gemv_tc.cu) and the depth frame's tcgen05
// build (fb_depth.cu): shared-memory matrix descriptors, the kind::f16 MMA issued by one thread, commit to an
// mbarrier, TMEM loads, allocation, and the fences between the generic and async proxies.
#pragma once
#include "fb_common.cuh"

namespace fb {

// Shared-memory matrix descriptor: start >> 4 in [0, 14), LBO >> 4 in [16, 30), SBO >> 4 in [32, 46), version 1 in
// [46, 48), layout type in [61, 64) (0: no swizzle, 2: 128-byte swizzle).  For the K-major 128-byte-swizzle layout
// used here (8-row groups of 128-byte rows, 1024 B apart) SBO = 1024 and LBO is unused; a k-step of 16 bf16
// advances the start address by 32 B inside the swizzle atom.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) { return tc_desc(saddr, 16, 1024, 2); }
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M = m (64 or 128), N = n.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t n, uint32_t m = 128) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// D[tmem] (+)= A . B^T, M = 128 (or M = 64 with tc_mma16_m64), N = 16, K = 16 (accumulate != 0 adds to D).
// M = 64 puts D row r in TMEM lane (r % 16) + 32 (r / 16): the first 16 lanes of each warp's quarter.
__device__ __forceinline__ void tc_mma16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(tc_idesc(16)));
}
__device__ __forceinline__ void tc_mma16_m64(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(tc_idesc(16, 64)));
}
// Any N (a multiple of 16 up to 256 for M = 128): idesc = tc_idesc(n, m).
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate,
                                       uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(idesc));
}
// The mbarrier receives one arrival once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Generic-proxy shared-memory writes (st.shared, cp.async) -> visible to the tensor core's operand reads.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) .. + 31).
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&f)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
}
// Two 16-column loads (addresses ta, tb) and one wait, as one statement so no use of the values precedes the wait.
__device__ __forceinline__ void tc_ld16x2(uint32_t ta, uint32_t tb, float (&fa)[16], float (&fb)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    fa[i] = __uint_as_float(r[i]);
    fb[i] = __uint_as_float(r[16 + i]);
  }
}
// Whole-warp TMEM allocation of ncols (a power of two >= 32); the base address lands in *slot.
__device__ __forceinline__ void tc_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t tmem, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
}

}  // namespace fb
