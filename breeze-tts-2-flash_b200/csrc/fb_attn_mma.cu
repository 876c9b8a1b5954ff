// flashb: GQA decode attention on the tensor cores for many rows (the fused variant of fb_attn.cu: Qwen3 q_norm /
// k_norm + RoPE, the KV-cache write at cache_pos, attention over [0, cache_pos]), used when the batch alone fills
// the grid (one CTA per (row, KV head), no key split).
//
// Same semantics as fb_attn.cu, with one more rounding point: s = bf16(q . k), s = bf16(s * scaling), s = s + mask
// (bf16 add for a bf16 mask), p = exp(s - running max) in fp32 (the fast exponential intrinsic: a few fp32 ulps,
// below the bf16 rounding of p; the exact expf serialises on its special-case branches), o = sum bf16(p) v / sum p.
// The reference rounds the normalised probabilities to bf16 before p . v; here the unnormalised ones are rounded
// (both below the output's bf16 resolution).
//
// B200 design.  With 128 rows x 4 KV heads the scalar kernel is instruction-bound (each key costs ~130 instructions
// per head group: half-warp dot products, shuffles, one thread per head dimension for p . v).  Here each 64-key
// chunk is two small matrix products on mma.sync m16n8k16 (bf16 in, fp32 out):
//   S^T[64 keys x 8 heads] = K[64 x 128] . Q^T[128 x 8]   (warp w: keys 16 w .. 16 w + 15; the G <= 8 query heads
//                                                          of the group padded to 8 columns)
//   O^T[128 dims x 8 heads] += V^T[128 x 64] . P^T[64 x 8] (warp w: dims 32 w .. 32 w + 31)
// K and V chunks arrive by TMA tensor copies in the 128-byte-swizzle layout (two 64-dimension blocks of 64 rows),
// AM_STAGES chunks in flight on mbarriers, so that ldmatrix (plain for K, transposed for V) reads them without bank
// conflicts (one contiguous 1-D bulk copy per chunk, read by ldmatrix with 8-way conflicts, measured 73 vs 44 us
// at 128 rows).
// The online softmax runs on the S fragments: per-head chunk maxima and sums through warp shuffles and a 4-warp
// exchange in shared memory; P^T goes to shared memory as bf16 for the second product.  The mask values of a
// chunk are fetched by cp.async as far ahead as its K and V.  The first chunks are requested before
// griddepcontrol.wait (old cache rows are not written by the preceding kernel); the row written at cache_pos is
// patched into the staged chunk.  Every wait is bounded.
#include "fb_norm.cuh"

namespace fb {

namespace {

constexpr int AM_D = 128;
constexpr int AM_THREADS = 128;
constexpr int AM_CHUNK = 64;
constexpr int AM_TILE = AM_CHUNK * AM_D * 2;      // bytes of one staged K or V chunk (16 KB)
// chunks in flight per CTA: measured on B200 at 128 rows x 4 KV heads, two stages (three CTAs per SM) left every
// chunk waiting ~2 us for its copy; three stages (two CTAs per SM) cover that latency
#ifndef AM_STAGES
#define AM_STAGES 3
#endif


struct alignas(64) AttnMmaArgs {
  CUtensorMap tk, tv;      // the caches as [2 blocks of 64 dims][B * NKV * S rows][64], boxes of 64 rows x 2 blocks
  const bf16* qkv;
  long qkv_sb;
  const bf16* qn_w;
  const bf16* kn_w;
  float eps;
  const bf16* cos;
  const bf16* sin;
  long cs_sb;
  bf16* kc;
  bf16* vc;
  const void* mask;
  long m_sb;
  int mask_bf16;
  int mask_async;          // 1: mask rows 4-byte aligned, copied by cp.async; 0: plain loads
  const long long* cache_pos;
  float scaling;
  bf16* out;
  int S, NH, NKV;
  unsigned* err;
};

__device__ __forceinline__ void am_tma(void* dst, const CUtensorMap* map, int row, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(0), "r"(row), "r"(0), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_cta() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 4-byte asynchronous copy global -> shared of `bytes` (0, 2 or 4) source bytes, the rest zero-filled.
__device__ __forceinline__ void am_cp4(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void am_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void am_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void am_ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void am_ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void am_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Byte offset of 16-byte unit u (dims 8 u .. 8 u + 7) of row r in a staged chunk (two 8 KB blocks of 64 dims,
// 128-byte rows, unit j of a block at j ^ (r % 8)).
__device__ __forceinline__ uint32_t am_off(int r, int u) {
  return (uint32_t)(((u >> 3) << 13) + (r << 7) + ((((u & 7) ^ (r & 7))) << 4));
}

template <int G>
__global__ void __launch_bounds__(AM_THREADS) attn_mma_kernel(const __grid_constant__ AttnMmaArgs a) {
  extern __shared__ __align__(1024) unsigned char am_smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(am_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = sm;                       // [AM_STAGES][16 KB]
  unsigned char* sV = sm + AM_STAGES * AM_TILE; // [AM_STAGES][16 KB]
  __shared__ __align__(8) uint64_t full[AM_STAGES];
  __shared__ __align__(16) bf16 qs[8][AM_D];    // query heads of the group (rows >= G zero)
  __shared__ __align__(16) bf16 ps[8][AM_CHUNK + 8];   // P^T of the chunk: [head][key], bf16
  __shared__ float red_m[4][8], red_l[4][8];
  __shared__ __align__(16) unsigned char mring[AM_STAGES][AM_CHUNK * 4];   // the chunks' mask values (bf16 or fp32)
  __shared__ __align__(16) bf16 newk[AM_D];
  __shared__ __align__(16) bf16 newv[AM_D];

  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NH = a.NH, NKV = a.NKV, S = a.S;
  const long long pos = a.cache_pos[0];
  int len = (int)min((long long)S, pos + 1);
  if (len < 0) len = 0;
  const int nchunks = (len + AM_CHUNK - 1) / AM_CHUNK;
  const int row0 = (b * NKV + h) * S;           // first cache row of (b, h) in the tensor maps' row space

  if (tid == 0) {
    for (int i = 0; i < AM_STAGES; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&a.tv) : "memory");
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int s = c % AM_STAGES;
    mbar_arrive_expect_tx(&full[s], 2u * AM_TILE);
    am_tma(sK + s * AM_TILE, &a.tk, row0 + c * AM_CHUNK, &full[s]);
    am_tma(sV + s * AM_TILE, &a.tv, row0 + c * AM_CHUNK, &full[s]);
  };
  // mask values of chunk c into mring[c % AM_STAGES] by cp.async, one commit group per chunk (empty past the end),
  // requested as far ahead as the K / V copies
  const unsigned char* mrow_g = reinterpret_cast<const unsigned char*>(a.mask) +
                                (size_t)b * a.m_sb * (a.mask_bf16 ? 2 : 4);
  auto issue_mask = [&](int c) {
    const int s = c % AM_STAGES, p0 = c * AM_CHUNK;
    if (c < nchunks && !a.mask_async) {
      // rows not 4-byte aligned (odd stride of a bf16 mask): plain loads, this thread waits for its value
      if (tid < AM_CHUNK) {
        const int e = p0 + tid;
        if (a.mask_bf16)
          reinterpret_cast<bf16*>(mring[s])[tid] =
              e < len ? reinterpret_cast<const bf16*>(mrow_g)[e] : __float2bfloat16_rn(0.f);
        else
          reinterpret_cast<float*>(mring[s])[tid] = e < len ? reinterpret_cast<const float*>(mrow_g)[e] : 0.f;
      }
    } else if (c < nchunks) {
      if (a.mask_bf16) {
        if (tid < AM_CHUNK / 2) {
          const int e = p0 + 2 * tid;
          const int bytes = e < len ? (e + 1 < len ? 4 : 2) : 0;
          am_cp4(&mring[s][4 * tid], mrow_g + (size_t)(e < len ? e : 0) * 2, bytes);
        }
      } else if (tid < AM_CHUNK) {
        const int e = p0 + tid;
        am_cp4(&mring[s][4 * tid], mrow_g + (size_t)(e < len ? e : 0) * 4, e < len ? 4 : 0);
      }
    }
    am_cp_commit();
  };
  if (tid == 0)
    for (int c = 0; c < min(AM_STAGES, nchunks); ++c) issue(c);
  // the norm weights, this row's cos / sin and the mask are read before griddepcontrol.wait: in the decode step
  // they are written by the host or by launches at least two back (embed_rope, step_advance), complete before this
  // kernel can start; only q|k|v comes from the predecessor
  for (int c = 0; c < AM_STAGES; ++c) issue_mask(c);
  const HeadPair wq = head_load(a.qn_w, lane), wk = head_load(a.kn_w, lane);
  const HeadPair cs = head_load(a.cos + (size_t)b * a.cs_sb, lane), sn = head_load(a.sin + (size_t)b * a.cs_sb, lane);
  pdl_wait();
  pdl_trigger();

  // ---- queries of the group, and in every CTA the new key / value row (written to the cache by this CTA)
  for (int g = warp; g < 8; g += AM_THREADS / 32) {
    if (g < G) {
      const bf16* qr = a.qkv + (size_t)b * a.qkv_sb + (size_t)(h * G + g) * AM_D;
      head_store(qs[g], head_norm_rope(qr, wq, cs, sn, a.eps, lane), lane);
    } else {
      *reinterpret_cast<uint2*>(&qs[g][lane * 4]) = make_uint2(0u, 0u);
    }
  }
  const bool write = pos >= 0 && pos < S;
  if (write) {
    if (warp == 0) {
      const bf16* kr = a.qkv + (size_t)b * a.qkv_sb + (size_t)(NH + h) * AM_D;
      head_store(newk, head_norm_rope(kr, wk, cs, sn, a.eps, lane), lane);
    } else if (warp == 1) {
      const bf16* vp = a.qkv + (size_t)b * a.qkv_sb + (size_t)(NH + NKV + h) * AM_D;
      *reinterpret_cast<uint2*>(&newv[lane * 4]) = *reinterpret_cast<const uint2*>(vp + lane * 4);
    }
  }
  __syncthreads();
  if (write) {
    a.kc[((size_t)row0 + pos) * AM_D + tid] = newk[tid];
    a.vc[((size_t)row0 + pos) * AM_D + tid] = newv[tid];
  }
  // B fragments of Q^T for the 8 k-steps of S^T: b0 = Q[lane / 4][16 ks + 2 (lane % 4) ..], b1 = 8 dims further
  uint32_t qb[8][2];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qb[ks][0] = *reinterpret_cast<const uint32_t*>(&qs[lane >> 2][16 * ks + 2 * (lane & 3)]);
    qb[ks][1] = *reinterpret_cast<const uint32_t*>(&qs[lane >> 2][16 * ks + 8 + 2 * (lane & 3)]);
  }
  const int h0 = 2 * (lane & 3);                 // this thread's two head columns: h0, h0 + 1
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o[2][4];                                  // O^T tiles: dims 32 warp + 16 t + (lane / 4) (+ 8), heads h0, h0+1
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[t][i] = 0.f;

  bool ok = true;
  int cfail = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int s = c % AM_STAGES;
    const int p0 = c * AM_CHUNK;
    const int n = min(AM_CHUNK, len - p0);
    am_cp_wait<AM_STAGES - 1>();     // this thread's mask copies of chunk c have landed
    ok = __syncthreads_and(mbar_wait(&full[s], (c / AM_STAGES) & 1, a.err));
    if (!ok) {
      cfail = c;
      break;
    }
    unsigned char* ks_ = sK + s * AM_TILE;
    unsigned char* vs_ = sV + s * AM_TILE;
    // the row written this step (the copy may predate the write); V rows past the sequence zeroed (p = 0 there)
    if (write && pos >= p0 && pos < p0 + n && tid < 32) {
      const int r = (int)(pos - p0), u = tid & 15;
      const bf16* srcr = tid < 16 ? newk : newv;
      *reinterpret_cast<uint4*>((tid < 16 ? ks_ : vs_) + am_off(r, u)) = *reinterpret_cast<const uint4*>(srcr + u * 8);
    }
    for (int i = tid; i < (AM_CHUNK - n) * 16; i += AM_THREADS) {
      const int r = n + i / 16, u = i & 15;
      *reinterpret_cast<uint4*>(vs_ + am_off(r, u)) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();

    // ---- S^T = K . Q^T for keys 16 warp .. + 15
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const uint32_t kb = smem_u32(ks_);
      const int r = 16 * warp + ((lane >> 3) & 1) * 8 + (lane & 7);    // key row of this lane's ldmatrix address
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t af[4];
        am_ldsm_x4(kb + am_off(r, 2 * ks + (lane >> 4)), af);
        am_mma(sc, af, qb[ks][0], qb[ks][1]);
      }
    }
    // scores of keys k0 = 16 warp + lane / 4 (sc[0], sc[1]) and k0 + 8 (sc[2], sc[3]), heads h0, h0 + 1
    const int k0 = 16 * warp + (lane >> 2);
    float cm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = k0 + (i >> 1) * 8, hh = h0 + (i & 1);
      const float m = key >= n ? -INFINITY
                               : (a.mask_bf16 ? b2f(reinterpret_cast<const bf16*>(mring[s])[key])
                                              : reinterpret_cast<const float*>(mring[s])[key]);
      float v = -INFINITY;
      if (key < n && hh < G && m > -1e30f) {
        v = rbf(rbf(sc[i]) * a.scaling);
        v = a.mask_bf16 ? rbf(v + m) : v + m;
      }
      sc[i] = v;
      cm[i & 1] = fmaxf(cm[i & 1], v);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      cm[j] = fmaxf(cm[j], __shfl_xor_sync(FULL, cm[j], 4));
      cm[j] = fmaxf(cm[j], __shfl_xor_sync(FULL, cm[j], 8));
      cm[j] = fmaxf(cm[j], __shfl_xor_sync(FULL, cm[j], 16));
    }
    if (lane < 4) {
      red_m[warp][h0] = cm[0];
      red_m[warp][h0 + 1] = cm[1];
    }
    __syncthreads();
    float mnew[2], scale[2], ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float c4 = fmaxf(fmaxf(red_m[0][h0 + j], red_m[1][h0 + j]), fmaxf(red_m[2][h0 + j], red_m[3][h0 + j]));
      mnew[j] = fmaxf(m_run[j], c4);
      scale[j] = (m_run[j] > -INFINITY) ? __expf(m_run[j] - mnew[j]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = i & 1, key = k0 + (i >> 1) * 8;
      const float p = (sc[i] > -INFINITY) ? __expf(sc[i] - mnew[j]) : 0.f;
      ls[j] += p;
      ps[h0 + j][key] = __float2bfloat16_rn(p);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      ls[j] += __shfl_xor_sync(FULL, ls[j], 4);
      ls[j] += __shfl_xor_sync(FULL, ls[j], 8);
      ls[j] += __shfl_xor_sync(FULL, ls[j], 16);
    }
    if (lane < 4) {
      red_l[warp][h0] = ls[0];
      red_l[warp][h0 + 1] = ls[1];
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      o[t][0] *= scale[0];
      o[t][1] *= scale[1];
      o[t][2] *= scale[0];
      o[t][3] *= scale[1];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l_run[j] = l_run[j] * scale[j] + ((red_l[0][h0 + j] + red_l[1][h0 + j]) + (red_l[2][h0 + j] + red_l[3][h0 + j]));
      m_run[j] = mnew[j];
    }

    // ---- O^T += V^T . P^T for dims 32 warp .. + 31
    {
      const uint32_t vb = smem_u32(vs_);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        // P^T fragment: b0 = P[lane / 4][16 kk + 2 (lane % 4) ..], b1 = 8 keys further
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&ps[lane >> 2][16 * kk + 2 * (lane & 3)]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&ps[lane >> 2][16 * kk + 8 + 2 * (lane & 3)]);
        // V^T fragment via transposed ldmatrix: matrix q = lane / 8 covers dims + 8 (q % 2), keys + 8 (q / 2)
        const int key = 16 * kk + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int u = (32 * warp + 16 * t) / 8 + ((lane >> 3) & 1);
          uint32_t af[4];
          am_ldsm_x4_t(vb + am_off(key, u), af);
          am_mma(o[t], af, b0, b1);
        }
      }
    }
    __syncthreads();   // the stage, ps and red_* are reused
    if (tid == 0 && c + AM_STAGES < nchunks) {
      fence_proxy_async_cta();   // this stage's generic writes (patch, zeroed rows) before the copy overwrites it
      issue(c + AM_STAGES);
    }
    issue_mask(c + AM_STAGES);
  }
  if (!ok) {
    // a wait gave up: the error word is set; never leave with copies in flight into this CTA's shared memory
    am_cp_wait<0>();
    if (tid == 0)
      for (int c = cfail; c < min(cfail + AM_STAGES, nchunks); ++c)
        mbar_wait(&full[c % AM_STAGES], (c / AM_STAGES) & 1, a.err);
    return;
  }
  // ---- out[b, h G + head, dim] = O / l
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = i & 1, hh = h0 + j;
      const int d = 32 * warp + 16 * t + (lane >> 2) + (i >> 1) * 8;
      if (hh < G) {
        const float r = l_run[j] > 0.f ? o[t][i] / l_run[j] : 0.f;
        a.out[((size_t)b * NH + h * G + hh) * AM_D + d] = __float2bfloat16_rn(r);
      }
    }
}

}  // namespace

// Launches the tensor-core kernel for the fused decode attention when it applies (head_dim 128, GQA group <= 8,
// a contiguous cache [B][NKV][S][128], one CTA per (row, KV head) fills the grid); FB_ERR_UNSUPPORTED otherwise.
int attn_mma_fused(const bf16* qkv, long qkv_sb, const bf16* qn_w, const bf16* kn_w, float eps, const bf16* cos,
                   const bf16* sin, long cs_sb, bf16* kc, bf16* vc, long c_sb, long c_sh, int B, int NH, int NKV,
                   int S, const void* mask, int mask_bf16, long m_sb, const long long* cache_pos, float scaling,
                   bf16* out, cudaStream_t st) {
  const int G = NH / NKV;
  if (G > 8 || (G & (G - 1)) || c_sh != (long)S * AM_D || c_sb != c_sh * NKV) return FB_ERR_UNSUPPORTED;
  // the mask rows are copied 4 bytes at a time when 4-byte aligned
  const int mask_async = !((reinterpret_cast<uintptr_t>(mask) & 3) || (mask_bf16 && (m_sb & 1)));
  AttnMmaArgs a{};
  const long long rows = (long long)B * NKV * S;
  if (fbh::tmap_box(&a.tk, kc, rows, AM_D, 64, AM_CHUNK, 2, true) != FB_OK ||
      fbh::tmap_box(&a.tv, vc, rows, AM_D, 64, AM_CHUNK, 2, true) != FB_OK)
    return FB_ERR_UNSUPPORTED;
  a.qkv = qkv; a.qkv_sb = qkv_sb; a.qn_w = qn_w; a.kn_w = kn_w; a.eps = eps;
  a.cos = cos; a.sin = sin; a.cs_sb = cs_sb; a.kc = kc; a.vc = vc;
  a.mask = mask; a.m_sb = m_sb; a.mask_bf16 = mask_bf16; a.mask_async = mask_async;
  a.cache_pos = cache_pos; a.scaling = scaling;
  a.out = out; a.S = S; a.NH = NH; a.NKV = NKV;
  a.err = fbh::device_err_ptr();
  const size_t smem = 2 * AM_STAGES * (size_t)AM_TILE + 1024;
  const void* kern = nullptr;
  switch (G) {
    case 1: kern = (const void*)attn_mma_kernel<1>; break;
    case 2: kern = (const void*)attn_mma_kernel<2>; break;
    case 4: kern = (const void*)attn_mma_kernel<4>; break;
    default: kern = (const void*)attn_mma_kernel<8>; break;
  }
  static int attr_done[64][4] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int gi = G == 1 ? 0 : (G == 2 ? 1 : (G == 4 ? 2 : 3));
  if (dev < 64 && !attr_done[dev][gi]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("attn_mma: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev][gi] = 1;
  }
  void* args[] = {(void*)&a};
  return fbh::launch_pdl(kern, dim3(1, NKV, B), dim3(AM_THREADS), smem, st, args, true);
}

}  // namespace fb
