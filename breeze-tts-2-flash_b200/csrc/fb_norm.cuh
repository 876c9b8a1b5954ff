// flashb: the eager Qwen3 RMSNorm and rotary embedding, as device helpers shared by every kernel of the library.
//
// Arithmetic contract (transformers Qwen3RMSNorm and apply_rotary_pos_emb, run eagerly on bf16 tensors):
//   norm:  r = 1 / sqrt(mean_fp32(x^2) + eps),  y = bf16(w * bf16(x * r))     (the fp32 product is cast back to the
//          input dtype before the weight multiply)
//   rope:  out = bf16(bf16(y * cos) + bf16(rotate_half(y) * sin)),  rotate_half(y) = [-y[D/2:], y[:D/2]]
// The sum of squares is an fp32 sum in an order of this file's choosing; the bf16 rounding points are the contract.
//
// Layouts are this library's own:
//   * rows of activations staged in shared memory are addressed through an offset functor off(m, u) -> byte offset
//     of 16-byte unit u (columns 8u .. 8u+7) of row m, so one routine serves plain pitched rows and the swizzled
//     tensor-core operand layouts;
//   * a head of 128 dims on one warp is held as rotary pairs: lane l owns dims {2l, 2l+1} and their rotation
//     partners {64+2l, 64+2l+1}, so rotate_half needs no data exchange between lanes.
#pragma once
#include "fb_common.cuh"

namespace fb {

// ------------------------------------------------------------------------------------------------ RMSNorm on rows
// Sum of squares of the 8 bf16 values in v, added to acc in element order.
__device__ __forceinline__ float sumsq8(const uint4& v, float acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = lo_f(w[i]), b = hi_f(w[i]);
    acc = fmaf(a, a, acc);
    acc = fmaf(b, b, acc);
  }
  return acc;
}

// One bf16 pair through the norm contract: bf16(w * bf16(x * r)) for both halves of a packed word.
__device__ __forceinline__ uint32_t rms_pair(uint32_t x2, uint32_t w2, float r) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo_f(x2) * r, hi_f(x2) * r);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 y = __floats2bfloat162_rn(lo_f(w2) * hf.x, hi_f(w2) * hf.y);
  return *reinterpret_cast<const uint32_t*>(&y);
}

// Eight values (one 16-byte unit) through the norm contract.
__device__ __forceinline__ uint4 rms_unit(const uint4& x, const uint4& w, float r) {
  return make_uint4(rms_pair(x.x, w.x, r), rms_pair(x.y, w.y, r), rms_pair(x.z, w.z, r), rms_pair(x.w, w.w, r));
}

__device__ __forceinline__ float rms_factor(float sumsq, int K, float eps) {
  return 1.0f / sqrtf(sumsq / (float)K + eps);
}

// Row factors rs[m] of M staged rows of K columns.  Warps [0, nwarps) of the caller's group take rows
// m = warp, warp + nwarps, ...; a lane sums its units u = lane, lane + 32, ... in order and the warp folds the lanes
// with a butterfly.  The caller synchronises before and after (every unit visible before, rs read after).
template <typename Off>
__device__ __forceinline__ void rms_row_factors(const unsigned char* xs, Off off, int M, int K, float eps, float* rs,
                                                int warp, int nwarps) {
  const int lane = threadIdx.x & 31, nu = K >> 3;
  for (int m = warp; m < M; m += nwarps) {
    float acc = 0.f;
#pragma unroll 4
    for (int u = lane; u < nu; u += 32) acc = sumsq8(*reinterpret_cast<const uint4*>(xs + off(m, u)), acc);
    acc = warp_sum(acc);
    if (lane == 0) rs[m] = rms_factor(acc, K, eps);
  }
}

// Apply the norm in place to M staged rows with factors rs and weight nw (global, K bf16): thread t of nthreads
// handles units i = t, t + nthreads, ... of the row-major unit order (row i / (K/8), unit i % (K/8)).
template <typename Off>
__device__ __forceinline__ void rms_rows_apply(unsigned char* xs, Off off, int M, int K, const bf16* nw,
                                               const float* rs, int t, int nthreads) {
  const int nu = K >> 3;
  if (nu <= nthreads && nthreads % nu == 0) {
    // each thread keeps one unit column: its weight unit is read once, the rows follow without divisions
    const int u = t % nu, dm = nthreads / nu;
    const uint4 w = *reinterpret_cast<const uint4*>(nw + (size_t)u * 8);
#pragma unroll 4
    for (int m = t / nu; m < M; m += dm) {
      uint4* p = reinterpret_cast<uint4*>(xs + off(m, u));
      *p = rms_unit(*p, w, rs[m]);
    }
    return;
  }
  for (int i = t; i < M * nu; i += nthreads) {
    const int m = i / nu, u = i - m * nu;
    uint4* p = reinterpret_cast<uint4*>(xs + off(m, u));
    *p = rms_unit(*p, *reinterpret_cast<const uint4*>(nw + (size_t)u * 8), rs[m]);
  }
}

// Offset functor of plain rows at a byte pitch.
struct PitchOff {
  int pitch;
  __device__ __forceinline__ uint32_t operator()(int m, int u) const { return (uint32_t)(m * pitch + u * 16); }
};

// ------------------------------------------------------------------------------------------------ one head, one warp
// Rotary-pair view of a 128-dim head held by one warp (lane l: dims 2l, 2l+1 in lo; 64+2l, 64+2l+1 in hi).
struct HeadPair {
  float lo[2], hi[2];
};

__device__ __forceinline__ HeadPair head_load(const bf16* p, int lane) {
  const uint32_t a = *reinterpret_cast<const uint32_t*>(p + 2 * lane);
  const uint32_t b = *reinterpret_cast<const uint32_t*>(p + 64 + 2 * lane);
  HeadPair h;
  h.lo[0] = lo_f(a);
  h.lo[1] = hi_f(a);
  h.hi[0] = lo_f(b);
  h.hi[1] = hi_f(b);
  return h;
}

// Write a head (values already on the bf16 grid, or rounded here) to 128 contiguous bf16.
__device__ __forceinline__ void head_store(bf16* p, const HeadPair& h, int lane) {
  *reinterpret_cast<__nv_bfloat162*>(p + 2 * lane) = __floats2bfloat162_rn(h.lo[0], h.lo[1]);
  *reinterpret_cast<__nv_bfloat162*>(p + 64 + 2 * lane) = __floats2bfloat162_rn(h.hi[0], h.hi[1]);
}

// q/k head norm (over its 128 dims) followed by RoPE, both with the eager rounding points; w, cs, sn are the norm
// weight and the position's cos / sin rows in the same rotary-pair view.  Result values lie on the bf16 grid.
__device__ __forceinline__ HeadPair head_norm_rope(const bf16* x, const HeadPair& w, const HeadPair& cs,
                                                   const HeadPair& sn, float eps, int lane) {
  const HeadPair v = head_load(x, lane);
  float acc = v.lo[0] * v.lo[0];
  acc = fmaf(v.lo[1], v.lo[1], acc);
  acc = fmaf(v.hi[0], v.hi[0], acc);
  acc = fmaf(v.hi[1], v.hi[1], acc);
  const float r = rms_factor(warp_sum(acc), 128, eps);
  HeadPair out;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float ylo = rbf(w.lo[e] * rbf(v.lo[e] * r));
    const float yhi = rbf(w.hi[e] * rbf(v.hi[e] * r));
    // rotate_half: the low half takes -y_hi, the high half takes +y_lo (negation is exact in bf16)
    out.lo[e] = rbf(rbf(ylo * cs.lo[e]) + rbf(-yhi * sn.lo[e]));
    out.hi[e] = rbf(rbf(yhi * cs.hi[e]) + rbf(ylo * sn.hi[e]));
  }
  return out;
}

}  // namespace fb
