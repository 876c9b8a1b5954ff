// flashb: the whole backbone decode step as ONE persistent kernel (cooperative launch, one CTA per SM).
//
// The reference runs a step as 28 x 5 kernel launches plus eager ops inside a CUDA graph (flash/backbone.py:106-138);
// on B200 each of those launches costs a few microseconds of ramp-up and drain, comparable to the HBM time of its
// weights.  Here the step is one launch: a producer warp per CTA streams that CTA's slice of every weight matrix of
// every layer through the 64 KB-stage ring (fb_stream.cuh) without ever waiting for activations, and the consumer
// warps run the step's tasks separated by grid barriers (bounded, fb_persist.cuh):
//
//   prologue   [optional position advance] + embedding gather-sum (columns split over CTAs) + cos/sin rows
//   per layer  QKV GEMV (RMSNorm prologue) | GQA attention (q/k norm, RoPE, KV write; split-KV over CTAs, the last
//              CTA of each (b, kv-head) merges) | O GEMV + residual | gate/up GEMV (RMSNorm) + SiLU*up |
//              down GEMV + residual
//   epilogue   final RMSNorm + fp32 lm_head (rows split over all warps) + CFG
//
// Numerics are those of the separate kernels (fb_gemv.cu mma path, fb_attn.cu, fb_aux.cu): the GEMV sums are
// bitwise identical (same stage tiling and reduction order); the attention differs from fb_attn.cu only in its split
// boundaries.  Scratch (activations, split partials, merge tickets, barrier) lives in one caller-owned buffer that
// must be zeroed once; every step leaves its tickets and barrier count at zero.
#include "fb_persist.cuh"

namespace fb {

constexpr int BB_MAXB = 8;
constexpr int BB_MAXSPLIT = 32;
constexpr int BB_WSROW = 130;

struct BBLayer {
  const bf16 *ln1, *wq, *wk, *wv, *qn, *kn, *wo, *ln2, *wg, *wu, *wd;
  bf16 *kc, *vc;
};

struct BBArgs {
  int L, B, H, NH, NKV, F, V, C, vocab, S, max_pos, nsplit;
  float eps, qk_eps, scaling;
  long c_sb, c_sh;
  const BBLayer* layers;
  const bf16* embed;
  const bf16* norm_w;
  const float* lm_head;
  const bf16* cos_tab;
  const bf16* sin_tab;
  const long long* ids;
  long long* pos_ids;
  long long* cache_pos;
  void* mask;
  int mask_bf16;
  long m_sb;
  const float* gs;
  int advance;
  bf16* hidden_out;
  float* logits;
  float* cfg_out;
  bf16 *x, *qkv, *ao, *h1, *act, *cs;
  float* part;
  int* tickets;
  GridBar* bar;
  int nstages, xs_bytes;
  unsigned long long* trace;
  unsigned* err;
};

// Optional trace: thread 0 of each CTA stamps %globaltimer into its row of a.trace.
#define BB_STAMP(idx)                                                                        \
  do {                                                                                       \
    if (a.trace && threadIdx.x == 0)                                                         \
      a.trace[(size_t)blockIdx.x * (2 + 10 * a.L) + (idx)] = (unsigned long long)globaltimer(); \
  } while (0)

__device__ __forceinline__ void bb_norm_rope(const bf16* x, const bf16* w, float eps, const bf16* cs, const bf16* sn,
                                             int lane, float out[4]) {
  const int d0 = lane * 4;
  const uint2 xv = __ldcg(reinterpret_cast<const uint2*>(x + d0));
  const float v[4] = {lo_f(xv.x), hi_f(xv.x), lo_f(xv.y), hi_f(xv.y)};
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / 128.0f + eps);
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) y[j] = rbf(b2f(w[d0 + j]) * rbf(v[j] * r));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float partner = __shfl_xor_sync(FULL, y[j], 16);
    const float rot = lane < 16 ? -partner : partner;
    out[j] = rbf(rbf(y[j] * b2f(__ldcg(cs + d0 + j))) + rbf(rot * b2f(__ldcg(sn + d0 + j))));
  }
}

struct AttSmem {
  float q[8][128];
  float p[8][64];
  float st_m[8], st_l[8], st_scale[8];
  float mg_m[8][BB_MAXSPLIT], mg_l[8][BB_MAXSPLIT];
  __align__(16) bf16 newk[128];
  __align__(16) bf16 newv[128];
  int last;
};

// One split of one (b, kv-head): keys [p_begin, p_end) in chunks of 64.  Half-warp (w, hw) owns keys
// 16 * i + 2 * w + hw of a chunk and loads their K and V rows (16 bytes per lane) all at once, so a chunk costs one
// memory round trip.  Scores go to shared memory, an online softmax per q head keeps running (m, l), and each lane
// accumulates P.V for its 8 dimensions over its own keys; half-warps and then warps are summed in a fixed order
// (wp: 8 x G x 128 floats of scratch).  The partial (m, l, o) goes to a.part; the last split to finish its
// (b, kv-head) merges all splits in split order and resets the ticket.
template <int G>
__device__ void bb_attention(const BBArgs& a, const BBLayer& Lw, AttSmem& sm, float* wp, int item) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = a.nsplit;
  const int b = item / (a.NKV * ns);
  const int rem = item - b * a.NKV * ns;
  const int h = rem / ns, split = rem - h * ns;
  const int NH = a.NH;
  const long long pos = __ldcg(a.cache_pos);
  int len = (int)min((long long)a.S, pos + 1);
  if (len < 0) len = 0;
  const int p_begin = (int)((long long)len * split / ns), p_end = (int)((long long)len * (split + 1) / ns);
  const bf16* qkv = a.qkv + (size_t)b * (NH + 2 * a.NKV) * 128;
  const bf16* cs = a.cs + (size_t)b * 256;
  bf16* kbase = Lw.kc + (size_t)b * a.c_sb + (size_t)h * a.c_sh;
  bf16* vbase = Lw.vc + (size_t)b * a.c_sb + (size_t)h * a.c_sh;
  const bool owner = pos >= p_begin && pos < p_end;

  for (int g = warp; g < G; g += ST_CWARPS) {
    float qv[4];
    bb_norm_rope(qkv + (size_t)(h * G + g) * 128, Lw.qn, a.qk_eps, cs, cs + 128, lane, qv);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.q[g][lane * 4 + j] = qv[j];
  }
  if (owner) {
    if (warp == ST_CWARPS - 1) {
      float kv[4];
      bb_norm_rope(qkv + (size_t)(NH + h) * 128, Lw.kn, a.qk_eps, cs, cs + 128, lane, kv);
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.newk[lane * 4 + j] = __float2bfloat16_rn(kv[j]);
    } else if (warp == ST_CWARPS - 2) {
      *reinterpret_cast<uint2*>(&sm.newv[lane * 4]) =
          __ldcg(reinterpret_cast<const uint2*>(qkv + (size_t)(NH + a.NKV + h) * 128) + lane);
    }
  }
  if (tid < G) {
    sm.st_m[tid] = -INFINITY;
    sm.st_l[tid] = 0.f;
  }
  named_sync(1, PK_CONSUMERS);
  if (owner && tid < 128) {
    kbase[(size_t)pos * 128 + tid] = sm.newk[tid];
    vbase[(size_t)pos * 128 + tid] = sm.newv[tid];
  }
  const int l16 = lane & 15, hw = lane >> 4;
  float qf[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) qf[g][j] = sm.q[g][l16 * 8 + j];
  float o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) o[g][j] = 0.f;

  for (int p0 = p_begin; p0 < p_end; p0 += 64) {
    const int n = min(64, p_end - p0);
    uint4 kr[4], vr[4];
    float mk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // all loads of this chunk in flight at once
      const int j = 16 * i + 2 * warp + hw;
      const int pj = p0 + j;
      if (j < n && pj != pos) {
        kr[i] = __ldcg(reinterpret_cast<const uint4*>(kbase + (size_t)pj * 128) + l16);
        vr[i] = __ldcg(reinterpret_cast<const uint4*>(vbase + (size_t)pj * 128) + l16);
      } else {
        kr[i] = make_uint4(0, 0, 0, 0);
        vr[i] = make_uint4(0, 0, 0, 0);
      }
      mk[i] = -INFINITY;
      if (j < n) {
        const size_t mi = (size_t)b * a.m_sb + pj;
        mk[i] = a.mask_bf16 ? b2f(__ldcg(reinterpret_cast<const bf16*>(a.mask) + mi))
                            : __ldcg(reinterpret_cast<const float*>(a.mask) + mi);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = 16 * i + 2 * warp + hw;
      if (owner && p0 + j == pos) {
        kr[i] = *reinterpret_cast<const uint4*>(&sm.newk[l16 * 8]);
        vr[i] = *reinterpret_cast<const uint4*>(&sm.newv[l16 * 8]);
      }
      float kf[8];
      cvt8(kr[i], kf);
      float d[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float acc = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = fmaf(qf[g][u], kf[u], acc);
        d[g] = acc;
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) d[g] += __shfl_xor_sync(FULL, d[g], off);
      if (l16 == 0 && j < n) {
        const bool valid = mk[i] > -1e30f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float sc = rbf(rbf(d[g]) * a.scaling);
          sc = a.mask_bf16 ? rbf(sc + mk[i]) : sc + mk[i];
          sm.p[g][j] = valid ? sc : -INFINITY;
        }
      }
    }
    named_sync(1, PK_CONSUMERS);
    for (int g = warp; g < G; g += ST_CWARPS) {
      const float s0 = lane < n ? sm.p[g][lane] : -INFINITY;
      const float s1 = lane + 32 < n ? sm.p[g][lane + 32] : -INFINITY;
      const float cm = warp_max(fmaxf(s0, s1));
      const float mold = sm.st_m[g];
      const float mnew = fmaxf(mold, cm);
      const bool any = mnew > -INFINITY;
      const float e0 = (any && s0 > -INFINITY) ? expf(s0 - mnew) : 0.f;
      const float e1 = (any && s1 > -INFINITY) ? expf(s1 - mnew) : 0.f;
      if (lane < n) sm.p[g][lane] = e0;
      if (lane + 32 < n) sm.p[g][lane + 32] = e1;
      const float es = warp_sum(e0 + e1);
      if (lane == 0) {
        const float scale = (mold > -INFINITY) ? expf(mold - mnew) : 0.f;
        sm.st_scale[g] = scale;
        sm.st_l[g] = sm.st_l[g] * scale + es;
        sm.st_m[g] = mnew;
      }
    }
    named_sync(1, PK_CONSUMERS);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sc = sm.st_scale[g];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[g][u] *= sc;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = 16 * i + 2 * warp + hw;
      if (j < n) {
        float vf[8];
        cvt8(vr[i], vf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pj = sm.p[g][j];
#pragma unroll
          for (int u = 0; u < 8; ++u) o[g][u] = fmaf(pj, vf[u], o[g][u]);
        }
      }
    }
    named_sync(1, PK_CONSUMERS);  // p consumed before the next chunk overwrites it
  }
  // half-warps, then warps, in a fixed order
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int u = 0; u < 8; ++u) o[g][u] += __shfl_xor_sync(FULL, o[g][u], 16);
  if (hw == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int u = 0; u < 8; ++u) wp[((size_t)warp * G + g) * 128 + l16 * 8 + u] = o[g][u];
  }
  named_sync(1, PK_CONSUMERS);
  const int rowbase = b * NH + h * G;
  for (int i = tid; i < G * 128; i += PK_CONSUMERS) {
    const int g = i >> 7, d = i & 127;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < ST_CWARPS; ++w) s += wp[((size_t)w * G + g) * 128 + d];
    float* wr = a.part + ((size_t)(rowbase + g) * ns + split) * BB_WSROW;
    wr[d] = s;
    if (d == 0) {
      wr[128] = sm.st_m[g];
      wr[129] = sm.st_l[g];
    }
  }
  __threadfence();
  named_sync(1, PK_CONSUMERS);
  if (tid == 0) sm.last = atomicAdd(&a.tickets[b * a.NKV + h], 1) == ns - 1;
  named_sync(1, PK_CONSUMERS);
  if (!sm.last) return;
  __threadfence();
  for (int i = tid; i < G * ns; i += PK_CONSUMERS) {
    const int g = i / ns, sp = i - g * ns;
    const float* w = a.part + ((size_t)(rowbase + g) * ns + sp) * BB_WSROW;
    sm.mg_m[g][sp] = __ldcg(w + 128);
    sm.mg_l[g][sp] = __ldcg(w + 129);
  }
  named_sync(1, PK_CONSUMERS);
  for (int i = tid; i < G * 128; i += PK_CONSUMERS) {
    const int g = i >> 7, d = i & 127;
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, sm.mg_m[g][sp]);
    float vals[BB_MAXSPLIT];
#pragma unroll
    for (int sp = 0; sp < BB_MAXSPLIT; ++sp)
      vals[sp] = (sp < ns) ? __ldcg(a.part + ((size_t)(rowbase + g) * ns + sp) * BB_WSROW + d) : 0.f;
    float L = 0.f, O = 0.f;
    if (M > -INFINITY) {
#pragma unroll
      for (int sp = 0; sp < BB_MAXSPLIT; ++sp) {
        if (sp < ns && sm.mg_m[g][sp] > -INFINITY) {
          const float f = expf(sm.mg_m[g][sp] - M);
          L = fmaf(sm.mg_l[g][sp], f, L);
          O = fmaf(vals[sp], f, O);
        }
      }
    }
    a.ao[(size_t)b * NH * 128 + (size_t)(h * G + g) * 128 + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
  }
  if (tid == 0) a.tickets[b * a.NKV + h] = 0;
}

template <int G>
__global__ void __launch_bounds__(PK_THREADS, 1) bb_step_kernel(const BBArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int B = a.B, H = a.H, NH = a.NH, NKV = a.NKV, F = a.F, NST = a.nstages;
  unsigned char* xs = smem;
  unsigned char* zero16 = smem + a.xs_bytes;
  unsigned char* ringb = zero16 + 128;
  float* red = reinterpret_cast<float*>(ringb + (size_t)NST * ST_BYTES);
  float* sums = red + ST_CWARPS * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(sums + 128);
  uint64_t* empty = full + PK_MAX_STAGES;
  __shared__ __align__(16) AttSmem att;
  __shared__ float nred[ST_CWARPS * 16];   // load_x keeps up to 16 rows of norm partials
  __shared__ int s_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ST_CWARPS);
    }
    fence_mbar_init();
  }
  if (tid < 32) reinterpret_cast<uint32_t*>(zero16)[tid] = 0u;
  __syncthreads();
  Ring rg{ringb, full, empty, NST};
  const int QKVN = (NH + 2 * NKV) * 128;

  if (warp == ST_CWARPS) {
    // ------------------------------------------------------------------ producer
    int t = 0;
    bool ok = true;
    auto qkv_row = [&](const BBLayer& W) {
      return [&W, NH, NKV, H](int n, int) -> const bf16* {
        return n < NH * 128 ? W.wq + (size_t)n * H
                            : (n < (NH + NKV) * 128 ? W.wk + (size_t)(n - NH * 128) * H
                                                    : W.wv + (size_t)(n - (NH + NKV) * 128) * H);
      };
    };
    BBLayer Lw = a.layers[0];
    for (int l = 0; l < a.L && ok; ++l) {
      const BBLayer Ln = a.layers[l + 1 < a.L ? l + 1 : l];
      auto o_row = [&](int n, int) { return Lw.wo + (size_t)n * NH * 128; };
      auto gu_row = [&](int n, int mat) { return (mat ? Lw.wu : Lw.wg) + (size_t)n * H; };
      auto d_row = [&](int n, int) { return Lw.wd + (size_t)n * F; };
      ok = ok && produce_task<1>(rg, t, QKVN, H, qkv_row(Lw), a.err);
      ok = ok && produce_task<1>(rg, t, H, NH * 128, o_row, a.err);
      ok = ok && produce_task<2>(rg, t, F, H, gu_row, a.err);
      ok = ok && produce_task<1>(rg, t, H, F, d_row, a.err);
      Lw = Ln;
    }
    for (int u = max(0, t - NST); u < t; ++u)
      if (!mbar_wait_warp(&full[u % NST], (u / NST) & 1, a.err)) break;
    return;
  }

  // ------------------------------------------------------------------ consumers
  unsigned epoch = 0;
  BB_STAMP(0);
  // prologue: position advance (CTA 0), embedding columns of this CTA, cos/sin rows (CTA 0)
  if (blockIdx.x == 0) {
    if (a.advance && tid == 0) {
      const long long p = a.cache_pos[0] + 1;
      a.cache_pos[0] = p;
      for (int b = 0; b < B; ++b) {
        a.pos_ids[b] += 1;
        if (p >= 0 && p < a.S) {
          if (a.mask_bf16) reinterpret_cast<bf16*>(a.mask)[(size_t)b * a.m_sb + p] = __float2bfloat16_rn(0.f);
          else reinterpret_cast<float*>(a.mask)[(size_t)b * a.m_sb + p] = 0.f;
        }
      }
    }
    named_sync(1, PK_CONSUMERS);
    for (int i = tid; i < B * 32; i += PK_CONSUMERS) {  // 128 dims = 16 vectors of cos + 16 of sin per row
      const int b = i >> 5, j = i & 31;
      long long p = a.pos_ids[b];
      p = p < 0 ? 0 : (p >= a.max_pos ? a.max_pos - 1 : p);
      const bf16* src = (j < 16 ? a.cos_tab : a.sin_tab) + p * 128 + (j & 15) * 8;
      *reinterpret_cast<uint4*>(a.cs + (size_t)b * 256 + (j >> 4) * 128 + (j & 15) * 8) =
          *reinterpret_cast<const uint4*>(src);
    }
  }
  {
    const int chunks = H >> 3;
    const int c0 = (int)((long long)chunks * blockIdx.x / gridDim.x);
    const int c1 = (int)((long long)chunks * (blockIdx.x + 1) / gridDim.x);
    const long long rows = (long long)a.C * a.vocab;
    for (int i = tid; i < B * (c1 - c0); i += PK_CONSUMERS) {
      const int b = i / (c1 - c0), j = c0 + (i - b * (c1 - c0));
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int c0 = 0; c0 < a.C; c0 += 16) {  // 16 independent row loads in flight, summed in codebook order
        uint4 v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int c = c0 + q;
          if (c < a.C) {
            long long r = a.ids[(size_t)b * a.C + c] + (long long)c * a.vocab;
            r = r < 0 ? 0 : (r >= rows ? rows - 1 : r);
            v[q] = ld_nc_v4(a.embed + (size_t)r * H + (size_t)j * 8);
          }
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (c0 + q < a.C) {
            float f[8];
            cvt8(v[q], f);
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[u] += f[u];
          }
        }
      }
      uint4 o;
      o.x = pack2(acc[0], acc[1]);
      o.y = pack2(acc[2], acc[3]);
      o.z = pack2(acc[4], acc[5]);
      o.w = pack2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(a.x + (size_t)b * H + (size_t)j * 8) = o;
    }
  }
  if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
  BB_STAMP(1);

  int t = 0;
  const int xp_h = H * 2 + 16, xp_o = NH * 128 * 2 + 16, xp_f = F * 2 + 16;
  const int nitems = B * NKV * a.nsplit;
  for (int l = 0; l < a.L; ++l) {
    const BBLayer Lw = a.layers[l];
    // QKV
    load_x(xs, xp_h, a.x, H, B, H, Lw.ln1, a.eps, nred);
    if (!consume_task<1>(rg, t, QKVN, H, xs, xp_h, B, zero16, red, sums,
                         [&](int n0, int nu, const float* sm) {
                           if (tid < nu * B) {
                             const int i = tid / B, m = tid - i * B;
                             a.qkv[(size_t)m * QKVN + n0 + i] = __float2bfloat16_rn(sm[i * 8 + m]);
                           }
                         }, a.err)) return;
    BB_STAMP(2 + 10 * l + 0);
    if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
    BB_STAMP(2 + 10 * l + 1);
    // attention
    if ((int)blockIdx.x < nitems) bb_attention<G>(a, Lw, att, reinterpret_cast<float*>(xs), blockIdx.x);
    BB_STAMP(2 + 10 * l + 2);
    if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
    BB_STAMP(2 + 10 * l + 3);
    // O projection + residual: h1 = x + o
    load_x(xs, xp_o, a.ao, NH * 128, B, NH * 128, nullptr, 0.f, nred);
    if (!consume_task<1>(rg, t, H, NH * 128, xs, xp_o, B, zero16, red, sums,
                         [&](int n0, int nu, const float* sm) {
                           if (tid < nu * B) {
                             const int i = tid / B, m = tid - i * B, n = n0 + i;
                             const float r = b2f(__ldcg(a.x + (size_t)m * H + n));
                             a.h1[(size_t)m * H + n] = __float2bfloat16_rn(r + rbf(sm[i * 8 + m]));
                           }
                         }, a.err)) return;
    BB_STAMP(2 + 10 * l + 4);
    if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
    BB_STAMP(2 + 10 * l + 5);
    // gate/up + SiLU*up
    load_x(xs, xp_h, a.h1, H, B, H, Lw.ln2, a.eps, nred);
    if (!consume_task<2>(rg, t, F, H, xs, xp_h, B, zero16, red, sums,
                         [&](int n0, int nu, const float* sm) {
                           if (tid < nu * B) {
                             const int i = tid / B, m = tid - i * B;
                             const float g = rbf(sm[i * 8 + m]);
                             const float u = rbf(sm[(i + 8) * 8 + m]);
                             a.act[(size_t)m * F + n0 + i] = __float2bfloat16_rn(rbf(g / (1.0f + expf(-g))) * u);
                           }
                         }, a.err)) return;
    BB_STAMP(2 + 10 * l + 6);
    if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
    BB_STAMP(2 + 10 * l + 7);
    // down + residual: x = h1 + d
    load_x(xs, xp_f, a.act, F, B, F, nullptr, 0.f, nred);
    if (!consume_task<1>(rg, t, H, F, xs, xp_f, B, zero16, red, sums,
                         [&](int n0, int nu, const float* sm) {
                           if (tid < nu * B) {
                             const int i = tid / B, m = tid - i * B, n = n0 + i;
                             const float r = b2f(__ldcg(a.h1 + (size_t)m * H + n));
                             a.x[(size_t)m * H + n] = __float2bfloat16_rn(r + rbf(sm[i * 8 + m]));
                           }
                         }, a.err)) return;
    BB_STAMP(2 + 10 * l + 8);
    if (!grid_sync(a.bar, epoch, a.err, &s_flag)) return;
    BB_STAMP(2 + 10 * l + 9);
  }

  grid_exit(a.bar);
  // final RMSNorm (redundant per CTA, fp32 copy in the now idle ring) + fp32 lm_head + CFG
  float* hs = reinterpret_cast<float*>(ringb);
  {
    float ss[BB_MAXB];
#pragma unroll
    for (int m = 0; m < BB_MAXB; ++m) ss[m] = 0.f;
    for (int i = tid; i < B * (H >> 3); i += PK_CONSUMERS) {
      const int m = i / (H >> 3), j = i - m * (H >> 3);
      float f[8];
      cvt8(__ldcg(reinterpret_cast<const uint4*>(a.x + (size_t)m * H) + j), f);
      float q = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) q = fmaf(f[u], f[u], q);
#pragma unroll
      for (int mm = 0; mm < BB_MAXB; ++mm)
        if (mm == m) ss[mm] += q;
    }
#pragma unroll
    for (int m = 0; m < BB_MAXB; ++m) {
      const float q = warp_sum(ss[m]);
      if (lane == 0) nred[warp * 8 + m] = q;
    }
    named_sync(1, PK_CONSUMERS);
    for (int i = tid; i < B * (H >> 3); i += PK_CONSUMERS) {
      const int m = i / (H >> 3), j = i - m * (H >> 3);
      float q = 0.f;
#pragma unroll
      for (int w = 0; w < ST_CWARPS; ++w) q += nred[w * 8 + m];
      const float r = 1.0f / sqrtf(q / (float)H + a.eps);
      float f[8], w8[8], y[8];
      cvt8(__ldcg(reinterpret_cast<const uint4*>(a.x + (size_t)m * H) + j), f);
      cvt8(*reinterpret_cast<const uint4*>(a.norm_w + (size_t)j * 8), w8);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        y[u] = rbf(w8[u] * rbf(f[u] * r));
        hs[(size_t)m * H + j * 8 + u] = y[u];
      }
      if (blockIdx.x == 0) {
        uint4 o;
        o.x = pack2(y[0], y[1]);
        o.y = pack2(y[2], y[3]);
        o.z = pack2(y[4], y[5]);
        o.w = pack2(y[6], y[7]);
        *reinterpret_cast<uint4*>(a.hidden_out + (size_t)m * H + j * 8) = o;
      }
    }
    named_sync(1, PK_CONSUMERS);
  }
  const int half = B >= 2 ? B / 2 : 1;
  const float gsv = a.gs ? a.gs[0] : 1.0f;
  const int gw = gridDim.x * ST_CWARPS;
  for (int v = blockIdx.x * ST_CWARPS + warp; v < a.V; v += gw) {
    const float* wr = a.lm_head + (size_t)v * H;
    float acc[BB_MAXB];
#pragma unroll
    for (int m = 0; m < BB_MAXB; ++m) acc[m] = 0.f;
    for (int j = lane * 4; j < H; j += 512) {
      uint4 u4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (j + i * 128 < H) u4[i] = ld_nc_v4(wr + j + i * 128);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (j + i * 128 >= H) break;
        const float w4[4] = {__uint_as_float(u4[i].x), __uint_as_float(u4[i].y), __uint_as_float(u4[i].z),
                             __uint_as_float(u4[i].w)};
#pragma unroll
        for (int m = 0; m < BB_MAXB; ++m) {
          if (m < B) {
            const float4 h4 = *reinterpret_cast<const float4*>(hs + (size_t)m * H + j + i * 128);
            acc[m] = fmaf(w4[0], h4.x, acc[m]);
            acc[m] = fmaf(w4[1], h4.y, acc[m]);
            acc[m] = fmaf(w4[2], h4.z, acc[m]);
            acc[m] = fmaf(w4[3], h4.w, acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < BB_MAXB; ++m)
      if (m < B) acc[m] = warp_sum(acc[m]);
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < BB_MAXB; ++m)
        if (m < B) a.logits[(size_t)m * a.V + v] = acc[m];
      if (B >= 2) {
#pragma unroll
        for (int hh = 0; hh < BB_MAXB / 2; ++hh) {
          if (hh < half) {
            float c = 0.f, u = 0.f;
#pragma unroll
            for (int m = 0; m < BB_MAXB; ++m) {
              if (m == hh) c = acc[m];
              if (m == hh + half) u = acc[m];
            }
            a.cfg_out[(size_t)hh * a.V + v] = __fadd_rn(u, __fmul_rn(gsv, __fsub_rn(c, u)));
          }
        }
      } else {
        a.cfg_out[v] = acc[0];
      }
    }
  }
}

}  // namespace fb

// ------------------------------------------------------------------------------------------------ host API
namespace {
using namespace fb;

struct ScratchLayout {
  size_t x, qkv, ao, h1, act, cs, part, tickets, bar, total;
  int nsplit;
};

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

ScratchLayout bb_layout(const fb_bb_config* c, int nsms) {
  ScratchLayout s{};
  const int B = c->batch, H = c->hidden, NH = c->heads, NKV = c->kv_heads, F = c->ffn;
  int ns = nsms / (B * NKV);
  if (ns > BB_MAXSPLIT) ns = BB_MAXSPLIT;
  if (ns < 1) ns = 1;
  s.nsplit = ns;
  size_t o = 0;
  s.x = o; o = al256(o + (size_t)B * H * 2);
  s.qkv = o; o = al256(o + (size_t)B * (NH + 2 * NKV) * 128 * 2);
  s.ao = o; o = al256(o + (size_t)B * NH * 128 * 2);
  s.h1 = o; o = al256(o + (size_t)B * H * 2);
  s.act = o; o = al256(o + (size_t)B * F * 2);
  s.cs = o; o = al256(o + (size_t)B * 256 * 2);
  s.part = o; o = al256(o + (size_t)B * NH * ns * BB_WSROW * 4);
  s.tickets = o; o = al256(o + (size_t)B * NKV * 4);
  s.bar = o; o = al256(o + sizeof(GridBar));
  s.total = o;
  return s;
}

template <int G>
int launch_bb(BBArgs& a, size_t smem, cudaStream_t st) {
  auto kern = bb_step_kernel<G>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_done[dev] < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("bb_step: cudaFuncSetAttribute(%zu): %s", smem, cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = (int)smem;
  }
  int nb = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, PK_THREADS, smem);
  if (e != cudaSuccess || nb < 1) {
    fbh::set_msg("bb_step: kernel not resident (occupancy %d): %s", nb, cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(fbh::num_sms());
  cfg.blockDim = dim3(PK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&a};
  e = cudaLaunchKernelExC(&cfg, (const void*)kern, args);
  if (e != cudaSuccess) {
    fbh::set_msg("bb_step launch: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

}  // namespace

extern "C" int64_t flashb_bb_scratch_bytes(const fb_bb_config* cfg) {
  if (!cfg) return -1;
  return (int64_t)bb_layout(cfg, fbh::num_sms()).total;
}

extern "C" int64_t flashb_bb_layer_bytes(void) { return (int64_t)sizeof(fb_bb_layer); }

extern "C" int flashb_bb_step(const fb_bb_config* c, const void* layers_dev, void* scratch, const int64_t* ids,
                              int64_t* position_ids, int64_t* cache_pos, void* mask, int mask_is_bf16, int64_t m_sb,
                              const float* gs, int advance, void* hidden_out, float* logits, float* cfg_out,
                              void* stream) {
  static_assert(sizeof(fb_bb_layer) == sizeof(BBLayer), "fb_bb_layer layout");
  FB_CHECK_ARG(c && layers_dev && scratch && ids && position_ids && cache_pos && mask && hidden_out && logits &&
                   cfg_out, "bb_step: null pointer argument");
  FB_CHECK_ARG(c->head_dim == 128, "bb_step: head_dim must be 128");
  FB_CHECK_ARG(c->batch >= 1 && c->batch <= BB_MAXB && c->layers >= 1, "bb_step: batch must be 1..8");
  FB_CHECK_ARG(c->hidden % 16 == 0 && c->ffn % 16 == 0 && c->heads % c->kv_heads == 0, "bb_step: bad dims");
  FB_CHECK_ARG(c->batch == 1 || gs, "bb_step: guidance scale required for batch >= 2");
  FB_CHECK_ARG(((uintptr_t)scratch & 255) == 0, "bb_step: scratch must be 256-byte aligned");
  const int nsms = fbh::num_sms();
  FB_CHECK_ARG(c->batch * c->kv_heads <= nsms, "bb_step: batch * kv_heads exceeds the SM count");
  const ScratchLayout L = bb_layout(c, nsms);
  BBArgs a{};
  a.L = c->layers; a.B = c->batch; a.H = c->hidden; a.NH = c->heads; a.NKV = c->kv_heads; a.F = c->ffn;
  a.V = c->lm_rows; a.C = c->codebooks; a.vocab = c->vocab; a.S = c->cache_len; a.max_pos = c->max_pos;
  a.nsplit = L.nsplit; a.eps = c->eps; a.qk_eps = c->qk_eps; a.scaling = c->scaling;
  a.c_sb = (long)c->cache_stride_b; a.c_sh = (long)c->cache_stride_h;
  a.layers = (const BBLayer*)layers_dev;
  a.embed = (const bf16*)c->embed; a.norm_w = (const bf16*)c->norm_w; a.lm_head = c->lm_head32;
  a.cos_tab = (const bf16*)c->cos_tab; a.sin_tab = (const bf16*)c->sin_tab;
  a.ids = (const long long*)ids; a.pos_ids = (long long*)position_ids; a.cache_pos = (long long*)cache_pos;
  a.mask = mask; a.mask_bf16 = mask_is_bf16 ? 1 : 0; a.m_sb = (long)m_sb; a.gs = gs; a.advance = advance;
  a.hidden_out = (bf16*)hidden_out; a.logits = logits; a.cfg_out = cfg_out;
  unsigned char* sc = (unsigned char*)scratch;
  a.x = (bf16*)(sc + L.x); a.qkv = (bf16*)(sc + L.qkv); a.ao = (bf16*)(sc + L.ao); a.h1 = (bf16*)(sc + L.h1);
  a.act = (bf16*)(sc + L.act); a.cs = (bf16*)(sc + L.cs); a.part = (float*)(sc + L.part);
  a.tickets = (int*)(sc + L.tickets); a.bar = (GridBar*)(sc + L.bar);
  a.trace = (unsigned long long*)c->trace;
  a.err = fbh::device_err_ptr();
  // shared memory: activations (widest K), zero block, ring, reduction scratch, mbarriers
  const int kmax = c->ffn > c->hidden ? (c->ffn > c->heads * 128 ? c->ffn : c->heads * 128)
                                      : (c->hidden > c->heads * 128 ? c->hidden : c->heads * 128);
  const int group = c->heads / c->kv_heads;
  a.xs_bytes = (int)al256((size_t)c->batch * (kmax * 2 + 16));
  if ((size_t)a.xs_bytes < (size_t)ST_CWARPS * group * 128 * 4) a.xs_bytes = ST_CWARPS * group * 128 * 4;
  const size_t fixed = (size_t)a.xs_bytes + 128 + ST_CWARPS * 128 * 4 + 128 * 4 + 2 * PK_MAX_STAGES * 8;
  const size_t budget = 227 * 1024 - sizeof(AttSmem) - ST_CWARPS * 8 * 4 - 64;
  int nst = (int)((budget - fixed) / ST_BYTES);
  if (nst > PK_MAX_STAGES) nst = PK_MAX_STAGES;
  if (nst < 2) {
    fbh::set_msg("bb_step: batch * widest K = %d does not leave room for two ring stages", c->batch * kmax);
    return FB_ERR_UNSUPPORTED;
  }
  a.nstages = nst;
  const size_t smem = fixed + (size_t)nst * ST_BYTES;
  FB_CHECK_ARG((size_t)c->batch * c->hidden * 4 <= (size_t)nst * ST_BYTES, "bb_step: hidden too large");
  cudaStream_t st = (cudaStream_t)stream;
  switch (c->heads / c->kv_heads) {
    case 1: return launch_bb<1>(a, smem, st);
    case 2: return launch_bb<2>(a, smem, st);
    case 4: return launch_bb<4>(a, smem, st);
    case 8: return launch_bb<8>(a, smem, st);
    default: fbh::set_msg("bb_step: GQA group %d not built", c->heads / c->kv_heads); return FB_ERR_UNSUPPORTED;
  }
}
