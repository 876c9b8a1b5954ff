// flashb: the sampler arithmetic shared by the depth frame and the backbone sampler: an exponential and a lane scan
// whose exact operation sequences the CPU oracle (oracle/sampler.c) repeats, so CPU and GPU tokens agree bit for bit,
// and the order-preserving float <-> uint32 map of the composite sort keys.
#pragma once
#include "fb_common.cuh"

namespace fb {

// exp(x) by Cody-Waite reduction and a degree-7 Taylor polynomial (Horner, fused multiply-adds); the exact operation
// sequence of fb_exp in oracle/sampler.c, so CPU and GPU agree bit for bit.
__device__ __forceinline__ float exp2i_dev(int n) { return __uint_as_float((unsigned)(n + 127) << 23); }
__device__ __forceinline__ float fb_exp_dev(float x) {
  if (!(x > -103.0f)) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float n = rintf(__fmul_rn(x, 0x1.715476p+0f));
  float r = fmaf(-n, 0x1.62e4p-1f, x);
  r = fmaf(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1.0p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = (int)n;
  if (ni < -125) return __fmul_rn(__fmul_rn(p, exp2i_dev(ni + 100)), exp2i_dev(-100));
  return __fmul_rn(p, exp2i_dev(ni));
}
__device__ __forceinline__ unsigned f2ord(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(unsigned o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
// Kogge-Stone inclusive scan over the 32 lanes (lane l adds the value of lane l - o, o = 1, 2, 4, 8, 16).
__device__ __forceinline__ float lane_scan(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v = __fadd_rn(y, v);
  }
  return v;
}

}  // namespace fb
