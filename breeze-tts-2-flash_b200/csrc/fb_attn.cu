// flashb: GQA split-KV flash-decoding attention for the backbone single-token decode step.
//
// Semantics (eager attention, transformers Qwen3 / UP/models/breeze.py:259-286, for q_len == 1):
//   s = bf16(q . k) ; s = bf16(s * scaling) ; s = s + mask (bf16 add for a bf16 mask, fp32 for an fp32 mask)
//   p = softmax_fp32(s) ; out = bf16(p . v)      (exponentials by the fast intrinsic: a few fp32 ulps)
// Keys whose additive mask is <= -1e30 are skipped; a row without any valid key gives 0.  Rounding points differ
// from eager in one place: the probabilities stay fp32 (eager rounds p to bf16 before p . v) because each split
// only knows its own running max; the effect is below bf16 resolution of the output.
// Fused variant (attn_decode_fused): Qwen3 q_norm / k_norm (RMSNorm over head_dim, eager double rounding) + RoPE
// (bf16(bf16(y*cos) + bf16(rotate_half(y)*sin))) and the KV-cache write at cache_pos, attending over
// [0, min(S, cache_pos + 1)): the official decode mask admits no key after the written slot
// (UP/models/cudagraph/backbone_graph.py:239-252), so the split range follows the real sequence length.
//
// B200 design: grid (nsplit, NKV, B) launched as thread-block clusters of nsplit CTAs (<= 16), one cluster per
// (b, kv-head).  Each CTA streams its key range in 64-position chunks (K and V rows are contiguous per (b, kv-head):
// one 16 KB bulk copy each, double-buffered in shared memory).  In the fused variant the first chunks are requested
// BEFORE griddepcontrol.wait (old cache slots are not written by the preceding kernel), so the KV stream overlaps the
// QKV GEMV's tail under PDL.  Per chunk, 256 threads run three short parallel steps: scores with a quad of threads
// per key (a 32-dim quarter each, 16-byte units read in a key-rotated order so the quads spread over the banks, two
// shuffles to combine), an online softmax with one warp per q head of the GQA group, and P.V with each thread
// owning two head dims over a quarter of the chunk's keys (the quarters added in order at the end).  The next
// chunk's mask values are loaded during the current chunk.  The split partials (m, l, o[128]) stay in each CTA's
// shared memory; after a cluster barrier, CTA g of the cluster merges head g by reading its peers' partials through
// distributed shared memory (in split order, so the result is deterministic) -- no global workspace, no atomics.
#include <cooperative_groups.h>

#include <cstdlib>

#include "fb_norm.cuh"

namespace cg = cooperative_groups;

namespace fb {

// fb_attn_mma.cu: the tensor-core kernel for the fused variant when the rows alone fill the grid
int attn_mma_fused(const bf16* qkv, long qkv_sb, const bf16* qn_w, const bf16* kn_w, float eps, const bf16* cos,
                   const bf16* sin, long cs_sb, bf16* kc, bf16* vc, long c_sb, long c_sh, int B, int NH, int NKV,
                   int S, const void* mask, int mask_bf16, long m_sb, const long long* cache_pos, float scaling,
                   bf16* out, cudaStream_t st);
thread_local int t_attn_path = -1;

constexpr int AT_D = 128;
constexpr int AT_THREADS = 256;
constexpr int AT_CHUNK = 64;
constexpr int AT_MAXCLUSTER = 16;   // splits per (b, kv-head) = CTAs per cluster (non-portable size 16)

struct AttnArgs {
  const bf16* q;
  long q_sb, q_sh;
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
  long c_sb, c_sh;
  const void* mask;
  long m_sb;
  int mask_bf16;
  const long long* cache_pos;
  float scaling;
  float* ws;
  int* counters;
  bf16* out;
  int S, NH, NKV, nsplit;
  unsigned* err;
};

// q of the group in shared memory as fp32, each 32-dim quarter padded to 36 floats (spreads the quarter reads of the
// score step over the banks)
__device__ __forceinline__ int at_qidx(int g, int d) { return g * 144 + (d >> 5) * 36 + (d & 31); }

template <int G, bool FUSED>
__global__ void __launch_bounds__(AT_THREADS) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sK = reinterpret_cast<bf16*>(smem);                       // [2][CHUNK][D]
  bf16* sV = sK + 2 * AT_CHUNK * AT_D;                            // [2][CHUNK][D]
  float* red = reinterpret_cast<float*>(sV + 2 * AT_CHUNK * AT_D); // [4 key quarters][G][D] P.V partial sums
  __shared__ __align__(8) uint64_t full[2];
  __shared__ __align__(16) float q_s[G * 144];
  __shared__ float s_s[G][AT_CHUNK];                              // scores, then unnormalised probabilities
  __shared__ float mrow[2][AT_CHUNK];                             // mask values of the chunk (by chunk parity)
  __shared__ float st_m[G], st_l[G], st_scale[G];
  __shared__ __align__(8) bf16 newk[AT_D];
  __shared__ __align__(8) bf16 newv[AT_D];
  __shared__ __align__(16) float part_o[G][AT_D];                 // this split's unnormalised o, read by peers

  cg::cluster_group cluster = cg::this_cluster();
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nsplit = a.nsplit;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NH = a.NH;

  long long pos = -1;
  int len = a.S;
  if (FUSED) {
    pos = a.cache_pos[0];
    len = (int)min((long long)a.S, pos + 1);
    if (len < 0) len = 0;
  }
  const int p_begin = (int)((long long)len * split / nsplit);
  const int p_end = (int)((long long)len * (split + 1) / nsplit);
  const int nchunks = (p_end - p_begin + AT_CHUNK - 1) / AT_CHUNK;
  const bf16* kbase = a.kc + (size_t)b * a.c_sb + (size_t)h * a.c_sh;
  const bf16* vbase = a.vc + (size_t)b * a.c_sb + (size_t)h * a.c_sh;

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    const int s = c & 1;
    const int p0 = p_begin + c * AT_CHUNK;
    const int n = min(AT_CHUNK, p_end - p0);
    const unsigned bytes = (unsigned)(n * AT_D * 2);
    mbar_arrive_expect_tx(&full[s], 2 * bytes);
    bulk_g2s(sK + (size_t)s * AT_CHUNK * AT_D, kbase + (size_t)p0 * AT_D, bytes, &full[s]);
    bulk_g2s(sV + (size_t)s * AT_CHUNK * AT_D, vbase + (size_t)p0 * AT_D, bytes, &full[s]);
  };
  // mask value of key tid of chunk c (threads < AT_CHUNK), -inf past the CTA's range
  auto mask_of = [&](int c) -> float {
    const int p = p_begin + c * AT_CHUNK + tid;
    if (tid >= AT_CHUNK || c >= nchunks || p >= p_end) return -INFINITY;
    const size_t mi = (size_t)b * a.m_sb + p;
    return a.mask_bf16 ? b2f(reinterpret_cast<const bf16*>(a.mask)[mi]) : reinterpret_cast<const float*>(a.mask)[mi];
  };
  if (FUSED && tid == 0) {
    for (int c = 0; c < min(2, nchunks); ++c) issue(c);
  }
  // Fused: the norm weights, this row's cos / sin and the first chunk's mask values are read before
  // griddepcontrol.wait.  In the decode step they are written by the host or by launches at least two back
  // (embed_rope, step_advance), which have completed before this kernel can start (its predecessor, the q|k|v GEMV,
  // lets it start only after its own griddepcontrol.wait); only q|k|v comes from the predecessor.
  HeadPair wq, wk, cs, sn;
  float mcur = -INFINITY;
  if (FUSED) {
    wq = head_load(a.qn_w, lane);
    wk = head_load(a.kn_w, lane);
    cs = head_load(a.cos + (size_t)b * a.cs_sb, lane);
    sn = head_load(a.sin + (size_t)b * a.cs_sb, lane);
    mcur = mask_of(0);
  }
  pdl_wait();
  pdl_trigger();
  if (!FUSED) {
    if (tid == 0)
      for (int c = 0; c < min(2, nchunks); ++c) issue(c);
    mcur = mask_of(0);
  }

  // ---- queries of this GQA group (and, in the owner CTA, the new key / value)
  for (int g = warp; g < G; g += AT_THREADS / 32) {
    const int hq = h * G + g;
    if (FUSED) {
      const bf16* qr = a.qkv + (size_t)b * a.qkv_sb + (size_t)hq * AT_D;
      const HeadPair qv = head_norm_rope(qr, wq, cs, sn, a.eps, lane);
      q_s[at_qidx(g, 2 * lane)] = qv.lo[0];
      q_s[at_qidx(g, 2 * lane + 1)] = qv.lo[1];
      q_s[at_qidx(g, 64 + 2 * lane)] = qv.hi[0];
      q_s[at_qidx(g, 64 + 2 * lane + 1)] = qv.hi[1];
    } else {
      const bf16* qp = a.q + (size_t)b * a.q_sb + (size_t)hq * a.q_sh;
#pragma unroll
      for (int j = 0; j < 4; ++j) q_s[at_qidx(g, lane * 4 + j)] = b2f(qp[lane * 4 + j]);
    }
  }
  const bool owner = FUSED && pos >= p_begin && pos < p_end;
  if (owner) {
    if (warp == 0) {
      const bf16* kr = a.qkv + (size_t)b * a.qkv_sb + (size_t)(NH + h) * AT_D;
      head_store(newk, head_norm_rope(kr, wk, cs, sn, a.eps, lane), lane);
    } else if (warp == 1) {
      const bf16* vp = a.qkv + (size_t)b * a.qkv_sb + (size_t)(NH + a.NKV + h) * AT_D;
      *reinterpret_cast<uint2*>(&newv[lane * 4]) = *reinterpret_cast<const uint2*>(vp + lane * 4);
    }
  }
  if (tid < G) {
    st_m[tid] = -INFINITY;
    st_l[tid] = 0.f;
  }
  __syncthreads();
  if (owner && tid < AT_D) {
    bf16* kd = a.kc + (size_t)b * a.c_sb + (size_t)h * a.c_sh + (size_t)pos * AT_D;
    bf16* vd = a.vc + (size_t)b * a.c_sb + (size_t)h * a.c_sh + (size_t)pos * AT_D;
    kd[tid] = newk[tid];
    vd[tid] = newv[tid];
  }

  // score step: thread = (key j of the chunk, 32-dim quarter e); P.V step: thread = (dims 2 dp, 2 dp + 1, keys
  // [16 kq, 16 kq + 16) of the chunk)
  const int sj = tid >> 2, se = tid & 3;
  const int dp = tid & 63, kq = tid >> 6;
  float o[G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g][0] = o[g][1] = 0.f;

  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    const int s = c & 1;
    const int p0 = p_begin + c * AT_CHUNK;
    const int n = min(AT_CHUNK, p_end - p0);
    if (tid < AT_CHUNK) {
      mrow[s][tid] = mcur;
      mcur = mask_of(c + 1);              // the next chunk's mask values, in flight during this chunk
    }
    ok = __syncthreads_and(mbar_wait(&full[s], (c >> 1) & 1, a.err));
    if (!ok) break;
    bf16* ks = sK + (size_t)s * AT_CHUNK * AT_D;
    bf16* vs = sV + (size_t)s * AT_CHUNK * AT_D;
    if (owner && pos >= p0 && pos < p0 + n) {   // the new key / value replace the slot's old contents
      if (tid < AT_D) {
        ks[(size_t)(pos - p0) * AT_D + tid] = newk[tid];
        vs[(size_t)(pos - p0) * AT_D + tid] = newv[tid];
      }
      __syncthreads();
    }
    // ---- scores: a quad of threads per key, each a quarter of the dims (16-byte units in a rotated order)
    {
      float d[G];
#pragma unroll
      for (int g = 0; g < G; ++g) d[g] = 0.f;
      if (sj < n) {
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)sj * AT_D + 32 * se);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ii = (i + sj) & 3;
          float kf[8];
          cvt8(kr[ii], kf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4* qp = reinterpret_cast<const float4*>(q_s + g * 144 + se * 36 + ii * 8);
            const float4 qa = qp[0], qb = qp[1];
            float acc = d[g];
            acc = fmaf(qa.x, kf[0], acc);
            acc = fmaf(qa.y, kf[1], acc);
            acc = fmaf(qa.z, kf[2], acc);
            acc = fmaf(qa.w, kf[3], acc);
            acc = fmaf(qb.x, kf[4], acc);
            acc = fmaf(qb.y, kf[5], acc);
            acc = fmaf(qb.z, kf[6], acc);
            acc = fmaf(qb.w, kf[7], acc);
            d[g] = acc;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        d[g] += __shfl_xor_sync(FULL, d[g], 1);
        d[g] += __shfl_xor_sync(FULL, d[g], 2);
      }
      const float m = mrow[s][sj];
      const bool valid = sj < n && m > -1e30f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if ((g & 3) == se) {
          float sc = rbf(rbf(d[g]) * a.scaling);
          sc = a.mask_bf16 ? rbf(sc + m) : sc + m;
          s_s[g][sj] = valid ? sc : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax statistics, one warp per head
    for (int g = warp; g < G; g += AT_THREADS / 32) {
      const float s0 = s_s[g][lane], s1 = s_s[g][lane + 32];
      const float cm = warp_max(fmaxf(s0, s1));
      const float mold = st_m[g];
      const float mnew = fmaxf(mold, cm);
      const bool any = mnew > -INFINITY;
      const float e0 = (any && s0 > -INFINITY) ? __expf(s0 - mnew) : 0.f;
      const float e1 = (any && s1 > -INFINITY) ? __expf(s1 - mnew) : 0.f;
      s_s[g][lane] = e0;
      s_s[g][lane + 32] = e1;
      const float es = warp_sum(e0 + e1);
      if (lane == 0) {
        const float scale = (mold > -INFINITY) ? __expf(mold - mnew) : 0.f;
        st_scale[g] = scale;
        st_l[g] = st_l[g] * scale + es;
        st_m[g] = mnew;
      }
    }
    __syncthreads();
    // ---- P . V: this thread's two dims over its quarter of the keys
#pragma unroll
    for (int g = 0; g < G; ++g) {
      o[g][0] *= st_scale[g];
      o[g][1] *= st_scale[g];
    }
    {
      const uint32_t* vr = reinterpret_cast<const uint32_t*>(vs) + dp;
      const int jb = kq * 16, je = min(jb + 16, n);
#pragma unroll 4
      for (int jj = jb; jj < je; ++jj) {
        const uint32_t v2 = vr[(size_t)jj * (AT_D / 2)];
        const float vx = lo_f(v2), vy = hi_f(v2);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pr = s_s[g][jj];
          o[g][0] = fmaf(pr, vx, o[g][0]);
          o[g][1] = fmaf(pr, vy, o[g][1]);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && c + 2 < nchunks) issue(c + 2);
  }
  if (!ok) {  // timed out: publish an empty partial so the cluster still completes its barriers
#pragma unroll
    for (int g = 0; g < G; ++g) o[g][0] = o[g][1] = 0.f;
    if (tid < G) {
      st_m[tid] = -INFINITY;
      st_l[tid] = 0.f;
    }
  }
  // the four key quarters' partial sums, added in quarter order
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<float2*>(red + ((size_t)kq * G + g) * AT_D + 2 * dp) = make_float2(o[g][0], o[g][1]);
  __syncthreads();
  for (int i = tid; i < G * AT_D; i += AT_THREADS) {
    const int g = i / AT_D, dd = i - g * AT_D;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) v += red[((size_t)q * G + g) * AT_D + dd];
    part_o[g][dd] = v;
  }

  // ---- merge across the cluster through distributed shared memory
  cluster.sync();
  if (tid < AT_D) {
    for (int g = split; g < G; g += nsplit) {
      float mv[AT_MAXCLUSTER], lv[AT_MAXCLUSTER], ov[AT_MAXCLUSTER];
#pragma unroll
      for (int sp = 0; sp < AT_MAXCLUSTER; ++sp) {  // all peer loads issued together
        if (sp < nsplit) {
          mv[sp] = *cluster.map_shared_rank(&st_m[g], sp);
          lv[sp] = *cluster.map_shared_rank(&st_l[g], sp);
          ov[sp] = *cluster.map_shared_rank(&part_o[g][tid], sp);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int sp = 0; sp < AT_MAXCLUSTER; ++sp)
        if (sp < nsplit) M = fmaxf(M, mv[sp]);
      float L = 0.f, O = 0.f;
      if (M > -INFINITY) {
#pragma unroll
        for (int sp = 0; sp < AT_MAXCLUSTER; ++sp) {
          if (sp < nsplit && mv[sp] > -INFINITY) {
            const float f = __expf(mv[sp] - M);
            L = fmaf(lv[sp], f, L);
            O = fmaf(ov[sp], f, O);
          }
        }
      }
      const float r = L > 0.f ? O / L : 0.f;
      a.out[((size_t)b * NH + h * G + g) * AT_D + tid] = __float2bfloat16_rn(r);
    }
  }
  cluster.sync();  // peers' shared memory must stay alive until every merge has read it
}

}  // namespace fb

namespace {
using namespace fb;

// K and V, two stages, then the P.V partial sums of the four key quarters
template <int G>
constexpr size_t at_smem() { return 4 * (size_t)AT_CHUNK * AT_D * 2 + 4 * (size_t)G * AT_D * 4; }

// Splits per (b, kv-head): about two CTAs per SM in all, at least 16 keys each, at most g_max_split (the cluster
// size; FLASHB_ATTN_SPLITS sets it, default AT_MAXCLUSTER).
int g_max_split = -1;
int g_mma = -1;   // the tensor-core kernel for the fused variant (FLASHB_ATTN_MMA=0 turns it off)

bool mma_enabled() {
  if (g_mma < 0) {
    const char* e = getenv("FLASHB_ATTN_MMA");
    g_mma = (e && e[0] == '0') ? 0 : 1;
  }
  return g_mma == 1;
}

int pick_nsplit(int B, int NKV, int S) {
  if (g_max_split < 0) {
    const char* e = getenv("FLASHB_ATTN_SPLITS");
    const int v = e ? atoi(e) : 0;
    g_max_split = (v >= 1 && v <= AT_MAXCLUSTER) ? v : AT_MAXCLUSTER;
  }
  const int target = 2 * fbh::grid_sms();
  int ns = (target + B * NKV - 1) / (B * NKV);
  const int cap_len = (S + 15) / 16;
  if (ns > cap_len) ns = cap_len;
  if (ns > g_max_split) ns = g_max_split;
  return ns < 1 ? 1 : ns;
}

template <int G, bool FUSED>
int launch_attn_t(AttnArgs& a, int B, cudaStream_t st) {
  auto kern = attn_decode_kernel<G, FUSED>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)at_smem<G>());
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      fbh::set_msg("attn: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = 1;
  }
  void* args[] = {(void*)&a};
  return fbh::launch_pdl((const void*)kern, dim3(a.nsplit, a.NKV, B), dim3(AT_THREADS), at_smem<G>(), st, args, true,
                         a.nsplit);
}

template <bool FUSED>
int dispatch_g(AttnArgs& a, int B, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch_attn_t<1, FUSED>(a, B, st);
    case 2: return launch_attn_t<2, FUSED>(a, B, st);
    case 4: return launch_attn_t<4, FUSED>(a, B, st);
    case 8: return launch_attn_t<8, FUSED>(a, B, st);
    default: fbh::set_msg("attn: GQA group %d not built (1, 2, 4, 8)", G); return FB_ERR_UNSUPPORTED;
  }
}

int fill_common(AttnArgs& a, const void* kc, const void* vc, int64_t c_sb, int64_t c_sh, int B, int NH, int NKV,
                int S, int D, const void* mask, int mask_is_bf16, int64_t m_sb, float scaling, float* ws,
                int64_t ws_floats, int32_t* counters, void* out) {
  (void)ws;
  (void)ws_floats;
  (void)counters;
  FB_CHECK_ARG(kc && vc && mask && out, "attn: null pointer argument");
  if (D != AT_D) {
    fbh::set_msg("attn: head_dim %d not built (128)", D);
    return FB_ERR_UNSUPPORTED;
  }
  FB_CHECK_ARG(B >= 1 && NKV >= 1 && NH >= NKV && NH % NKV == 0 && S >= 1, "attn: bad shape B=%d NH=%d NKV=%d S=%d",
               B, NH, NKV, S);
  FB_CHECK_ARG(((uintptr_t)kc & 15) == 0 && ((uintptr_t)vc & 15) == 0 && c_sb % 8 == 0 && c_sh % 8 == 0,
               "attn: KV cache must be 16-byte aligned with strides multiple of 8 elements");
  FB_CHECK_ARG(c_sh >= (int64_t)S * D && c_sb >= c_sh * NKV, "attn: KV strides overlap");
  FB_CHECK_ARG(B <= 65535 && NKV <= 65535, "attn: grid too large");
  a.kc = (bf16*)kc; a.vc = (bf16*)vc; a.c_sb = (long)c_sb; a.c_sh = (long)c_sh;
  a.mask = mask; a.mask_bf16 = mask_is_bf16 ? 1 : 0; a.m_sb = (long)m_sb;
  a.scaling = scaling; a.ws = nullptr; a.counters = nullptr; a.out = (bf16*)out;
  a.S = S; a.NH = NH; a.NKV = NKV;
  a.nsplit = pick_nsplit(B, NKV, S);
  a.err = fbh::device_err_ptr();
  return FB_OK;
}

}  // namespace

extern "C" int flashb_attn_last_path(void) { return fb::t_attn_path; }

extern "C" int64_t flashb_attn_ws_floats(int B, int NH, int NKV, int S, int D) {
  (void)B; (void)NH; (void)NKV; (void)S; (void)D;
  return 0;  // split partials are merged in distributed shared memory; no global workspace is needed
}

extern "C" int flashb_attn_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* kc, const void* vc,
                                  int64_t c_sb, int64_t c_sh, int B, int NH, int NKV, int S, int D, const void* mask,
                                  int mask_is_bf16, int64_t m_sb, float scaling, float* ws, int64_t ws_floats,
                                  int32_t* counters, void* out, void* stream) {
  AttnArgs a{};
  int rc = fill_common(a, kc, vc, c_sb, c_sh, B, NH, NKV, S, D, mask, mask_is_bf16, m_sb, scaling, ws, ws_floats,
                       counters, out);
  if (rc) return rc;
  FB_CHECK_ARG(q && ((uintptr_t)q & 7) == 0 && q_sh % 4 == 0 && q_sb % 4 == 0, "attn_decode: q misaligned");
  a.q = (const bf16*)q; a.q_sb = (long)q_sb; a.q_sh = (long)q_sh;
  return dispatch_g<false>(a, B, NH / NKV, (cudaStream_t)stream);
}

extern "C" int flashb_attn_decode_fused(const void* qkv, int64_t qkv_sb, const void* qn_w, const void* kn_w,
                                        float eps, const void* cos, const void* sin, int64_t cs_sb, void* kc,
                                        void* vc, int64_t c_sb, int64_t c_sh, int B, int NH, int NKV, int S, int D,
                                        const void* mask, int mask_is_bf16, int64_t m_sb, const int64_t* cache_pos,
                                        float scaling, float* ws, int64_t ws_floats, int32_t* counters, void* out,
                                        void* stream) {
  AttnArgs a{};
  int rc = fill_common(a, kc, vc, c_sb, c_sh, B, NH, NKV, S, D, mask, mask_is_bf16, m_sb, scaling, ws, ws_floats,
                       counters, out);
  if (rc) return rc;
  FB_CHECK_ARG(qkv && qn_w && kn_w && cos && sin && cache_pos, "attn_decode_fused: null pointer argument");
  FB_CHECK_ARG(((uintptr_t)qkv & 7) == 0 && qkv_sb % 4 == 0 && ((uintptr_t)cos & 7) == 0 && cs_sb % 4 == 0,
               "attn_decode_fused: qkv/cos misaligned");
  a.qkv = (const bf16*)qkv; a.qkv_sb = (long)qkv_sb;
  a.qn_w = (const bf16*)qn_w; a.kn_w = (const bf16*)kn_w; a.eps = eps;
  a.cos = (const bf16*)cos; a.sin = (const bf16*)sin; a.cs_sb = (long)cs_sb;
  a.cache_pos = (const long long*)cache_pos;
  if (a.nsplit == 1 && mma_enabled()) {
    // the rows alone fill the grid: the tensor-core kernel (one CTA per row and KV head)
    rc = attn_mma_fused(a.qkv, a.qkv_sb, a.qn_w, a.kn_w, eps, a.cos, a.sin, a.cs_sb, a.kc, a.vc, a.c_sb, a.c_sh, B,
                        NH, NKV, S, mask, a.mask_bf16, a.m_sb, a.cache_pos, scaling, a.out, (cudaStream_t)stream);
    if (rc != FB_ERR_UNSUPPORTED) {
      t_attn_path = 1;
      return rc;
    }
  }
  t_attn_path = 0;
  return dispatch_g<true>(a, B, NH / NKV, (cudaStream_t)stream);
}
