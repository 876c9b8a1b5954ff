// flashb: one depth-decoder frame (every codebook of the frame, CFG sampling included) as ONE persistent launch.
//
// Follows the official graph loop DepthDecoderGraph._full_loop (UP/models/cudagraph/depth_decoder_graph.py:558-654,
// UP = third_party/breeze-tts) with the eager rounding points of BreezeDecoderLayer (UP/models/breeze.py:378-425), and
// replaces the reference's depth megakernel (flash/csrc/depth_frame.cu:656-853) with a B200 design: one CTA per SM,
// a producer warp streaming every weight slice of the frame (projector, 4 x {q|k|v, o, gate|up, down}, codebook
// head) through the 64 KB-stage ring (fb_stream.cuh, tensor-core GEMV), consumer warps running the tasks between
// bounded grid barriers (fb_persist.cuh):
//
//   per codebook step s (T = 2 tokens at s = 0, else 1; M = B * T rows):
//     E   embeddings (s = 0: [backbone hidden, embed(first_cb)]; s > 0: embed(clamp(tok + s*V))) @ projector^T
//     per layer  S1 RMSNorm + q|k|v GEMV, each unit = the rotary pair of rows (d, d+64) so RoPE is applied in the
//                   epilogue; k, v written to the frame's KV cache at the token's position
//                S2 attention over positions 0..pos (<= n_decode + 1 keys, every CTA computes all rows; no merge)
//                   + o GEMV
//                S3 RMSNorm(bf16(x + o)) + gate|up GEMV + SiLU*up
//                S4 down GEMV + residual
//     S5  final RMSNorm + codebook-head GEMV -> fp32 logits
//     sampler  CTA h samples half-row h: CFG, codec-id mask, temperature, top-k, top-p, softmax, argmax(p / q),
//              with its own exp routine and fixed summation order, bit-identical to the C oracle (oracle/sampler.c)
//
// Scratch (residual stream, q, o, act, logits, KV cache, barrier) is one caller-owned buffer, zeroed once.
#include "fb_persist.cuh"

namespace fb {

constexpr int DD_MAXB = 4;      // batch rows (two CFG pairs)
constexpr int DD_MAXV = 4096;   // sampler vocabulary bound (composite key packs 12 index bits)

struct DDLayer {
  const bf16 *ln1, *wq, *wk, *wv, *wo, *ln2, *wg, *wu, *wd;
};

struct DDArgs {
  int L, B, H, AE, NH, NKV, F, V, CB, NCB, P;
  float eps, scaling;
  const DDLayer* layers;
  const bf16 *embed, *proj, *normf, *head_t, *cos_tab, *sin_tab;
  const long long* first_cb;
  const bf16* bh;
  long long* tokbuf;
  long long* outtok;
  const float* temp;
  const long long* topk;
  const float* topp;
  const long long* dosample;
  const float* gs;
  const float* q;
  float* dbg;
  const long long* forced;
  bf16 *xres, *qb, *ob, *act, *kc, *vc;
  float* logits;
  GridBar* bar;
  int nstages, xs_bytes;
  unsigned* err;
};

// ------------------------------------------------------------------------------------------------ sampler math
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

// Sampler for half-row h (all 256 consumer threads of the CTA).  `arr` is shared scratch for DD_MAXV 64-bit keys.
__device__ void dd_sample(const DDArgs& a, int step, int h, unsigned long long* arr, int* s_int) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = a.B >= 2 ? a.B / 2 : 1;
  const int V = a.V;
  const float* lc = a.logits + (size_t)h * V;
  const float* lu = a.B >= 2 ? a.logits + (size_t)(h + half) * V : nullptr;
  const float gs = a.gs[h], temp = a.temp[h], topp = a.topp[h];
  const long long tk = a.topk[h];
  int V2 = 1;
  while (V2 < V) V2 <<= 1;
  // 1) CFG, codec mask, temperature -> composite keys (key desc, index asc); greedy argmax(cfg)
  float gbest = -INFINITY;
  int gidx = 0x7fffffff;
  for (int i = tid; i < V2; i += PK_CONSUMERS) {
    unsigned long long comp = 0ull;
    if (i < V) {
      float cfg = __ldcg(lc + i);
      if (lu) {
        const float u = __ldcg(lu + i);
        cfg = __fadd_rn(u, __fmul_rn(gs, __fsub_rn(cfg, u)));
      }
      if (i >= a.CB) cfg = -INFINITY;
      if (cfg > gbest || (cfg == gbest && i < gidx)) {
        gbest = cfg;
        gidx = i;
      }
      const float key = __fdiv_rn(cfg, temp);
      comp = ((unsigned long long)f2ord(key) << 12) | (unsigned long long)(4095 - i);
    }
    arr[i] = comp;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, gbest, o);
    const int oi = __shfl_xor_sync(FULL, gidx, o);
    if (ov > gbest || (ov == gbest && oi < gidx)) {
      gbest = ov;
      gidx = oi;
    }
  }
  float* gv = reinterpret_cast<float*>(s_int + 4);
  if (lane == 0) {
    gv[warp] = gbest;
    s_int[16 + warp] = gidx;
  }
  named_sync(1, PK_CONSUMERS);
  if (tid == 0) {
    float bv = gv[0];
    int bi = s_int[16];
    for (int w = 1; w < ST_CWARPS; ++w)
      if (gv[w] > bv || (gv[w] == bv && s_int[16 + w] < bi)) {
        bv = gv[w];
        bi = s_int[16 + w];
      }
    s_int[0] = bi;
  }
  // 2) bitonic sort, descending
  for (int k = 2; k <= V2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < (V2 >> 1); i += PK_CONSUMERS) {
        const int lo = 2 * i - (i & (j - 1));
        const int hi = lo + j;
        const unsigned long long x = arr[lo], y = arr[hi];
        const bool desc = (lo & k) == 0;
        if (desc ? (x < y) : (x > y)) {
          arr[lo] = y;
          arr[hi] = x;
        }
      }
      named_sync(1, PK_CONSUMERS);
    }
  }
  // 3) warp 0: top-k / top-p / softmax / argmax(p / q) with the canonical sums (lane l owns ranks l*C .. l*C+C-1)
  if (warp == 0) {
    const int maxk = V < 1024 ? V : 1024;
    const int kk = tk > 0 ? (tk < maxk ? (int)tk : maxk) : maxk;
    const int C = (kk + 31) / 32;
    const float key0 = ord2f((unsigned)(arr[0] >> 12));
    auto e_of = [&](int r) { return fb_exp_dev(__fsub_rn(ord2f((unsigned)(arr[r] >> 12)), key0)); };
    float b = 0.f;
    for (int j = 0; j < C; ++j) {
      const int r = lane * C + j;
      if (r < kk) b = __fadd_rn(b, e_of(r));
    }
    const float S = __shfl_sync(FULL, lane_scan(b), 31);
    float bp = 0.f;
    for (int j = 0; j < C; ++j) {
      const int r = lane * C + j;
      if (r < kk) bp = __fadd_rn(bp, __fdiv_rn(e_of(r), S));
    }
    const float inclp = lane_scan(bp);
    const float exclp = __shfl_up_sync(FULL, inclp, 1);
    float run = lane ? exclp : 0.f;
    float s2 = 0.f;
    unsigned keepmask = 0u;
    for (int j = 0; j < C; ++j) {
      const int r = lane * C + j;
      if (r >= kk) break;
      const float e = e_of(r);
      const bool keep = (r == 0) || !(run > topp);
      run = __fadd_rn(run, __fdiv_rn(e, S));
      if (keep) {
        s2 = __fadd_rn(s2, e);
        keepmask |= 1u << j;
      }
    }
    const float S2 = __shfl_sync(FULL, lane_scan(s2), 31);
    const float* qrow = a.q + ((size_t)step * half + h) * V;
    float best = -1.f;
    int bidx = 0x7fffffff;
    for (int j = 0; j < C; ++j) {
      if (!((keepmask >> j) & 1u)) continue;
      const int r = lane * C + j;
      const int id = 4095 - (int)(arr[r] & 4095ull);
      const float sc = __fdiv_rn(__fdiv_rn(e_of(r), S2), __ldg(qrow + id));
      if (sc > best || (sc == best && id < bidx)) {
        best = sc;
        bidx = id;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, best, o);
      const int oi = __shfl_xor_sync(FULL, bidx, o);
      if (ov > best || (ov == best && oi < bidx)) {
        best = ov;
        bidx = oi;
      }
    }
    if (lane == 0) {
      int tokv = a.dosample[h] ? bidx : s_int[0];
      tokv = tokv < 0 ? 0 : (tokv > V - 1 ? V - 1 : tokv);
      a.outtok[(size_t)h * a.NCB + step] = tokv;
      if (a.B >= 2) a.outtok[(size_t)(h + half) * a.NCB + step] = tokv;
      if (a.forced) {
        const long long fc = a.forced[(size_t)step * a.B + h];
        tokv = (int)(fc < 0 ? 0 : (fc > V - 1 ? V - 1 : fc));
      }
      a.tokbuf[h] = tokv;
      if (a.B >= 2) {
        long long tu = tokv;
        if (a.forced) {
          const long long fc = a.forced[(size_t)step * a.B + h + half];
          tu = fc < 0 ? 0 : (fc > V - 1 ? V - 1 : fc);
        }
        a.tokbuf[h + half] = tu;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ attention (S2)
// All M x NH query rows over the layer's cached keys 0..pos(m); one warp per row, lane = 4 head dimensions; every key
// of the row loaded at once.  Eager rounding: s = bf16(bf16(q.k) * scaling), p = bf16(softmax_fp32(s)),
// out = bf16(sum p v).  Output rows go to xs (the o-projection input).
template <int G>
__device__ void dd_attention(const DDArgs& a, int l, int step, int T, unsigned char* xs, int x_pitch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.B * T;
  const int QD = a.NH * 128;
  constexpr int KB = 16;        // keys per load batch (all loads of a batch in flight together)
  constexpr int MAXK = 32;      // positions 0..n_decode, n_decode <= 31
  for (int row = warp; row < M * a.NH; row += ST_CWARPS) {
    const int m = row / a.NH, qh = row - m * a.NH;
    const int b = m / T, t = m - b * T;
    const int pos = step == 0 ? t : step + 1;
    const int kvh = qh / G;
    const uint2 q2 = __ldcg(reinterpret_cast<const uint2*>(a.qb + (size_t)m * QD + qh * 128) + lane);
    const float qf[4] = {lo_f(q2.x), hi_f(q2.x), lo_f(q2.y), hi_f(q2.y)};
    const size_t base = ((((size_t)l * a.B + b) * a.NKV + kvh) * a.P) * 128;
    float s[MAXK];
    float mx = -INFINITY;
#pragma unroll
    for (int j0 = 0; j0 < MAXK; j0 += KB) {
      if (j0 > pos) break;
      uint2 kr[KB];
#pragma unroll
      for (int j = 0; j < KB; ++j)
        if (j0 + j <= pos) kr[j] = __ldcg(reinterpret_cast<const uint2*>(a.kc + base + (size_t)(j0 + j) * 128) + lane);
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        if (j0 + j <= pos) {
          float d = qf[0] * lo_f(kr[j].x);
          d = fmaf(qf[1], hi_f(kr[j].x), d);
          d = fmaf(qf[2], lo_f(kr[j].y), d);
          d = fmaf(qf[3], hi_f(kr[j].y), d);
          d = warp_sum(d);
          s[j0 + j] = rbf(rbf(d) * a.scaling);
          mx = fmaxf(mx, s[j0 + j]);
        }
      }
    }
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < MAXK; ++j) {
      if (j <= pos) {
        s[j] = expf(s[j] - mx);
        den += s[j];
      }
    }
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j0 = 0; j0 < MAXK; j0 += KB) {
      if (j0 > pos) break;
      uint2 vr[KB];
#pragma unroll
      for (int j = 0; j < KB; ++j)
        if (j0 + j <= pos) vr[j] = __ldcg(reinterpret_cast<const uint2*>(a.vc + base + (size_t)(j0 + j) * 128) + lane);
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        if (j0 + j <= pos) {
          const float p = rbf(s[j0 + j] / den);
          o[0] = fmaf(p, lo_f(vr[j].x), o[0]);
          o[1] = fmaf(p, hi_f(vr[j].x), o[1]);
          o[2] = fmaf(p, lo_f(vr[j].y), o[2]);
          o[3] = fmaf(p, hi_f(vr[j].y), o[3]);
        }
      }
    }
    uint2 ov;
    ov.x = pack2(o[0], o[1]);
    ov.y = pack2(o[2], o[3]);
    *reinterpret_cast<uint2*>(xs + (size_t)m * x_pitch + (size_t)(qh * 128 + lane * 4) * 2) = ov;
  }
  named_sync(1, PK_CONSUMERS);
}

// x_mid = bf16(xres + ob) then RMSNorm (S3 input), all M rows.
__device__ void dd_load_mid(unsigned char* xs, int x_pitch, const DDArgs& a, int M, const bf16* nw, float* nred) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, kv = H >> 3;
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) ss[m] = 0.f;
  for (int i = tid; i < M * kv; i += PK_CONSUMERS) {
    const int m = i / kv, j = i - m * kv;
    float x[8], o[8];
    cvt8(__ldcg(reinterpret_cast<const uint4*>(a.xres + (size_t)m * H) + j), x);
    cvt8(__ldcg(reinterpret_cast<const uint4*>(a.ob + (size_t)m * H) + j), o);
    float v[8];
    float q = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      v[u] = rbf(x[u] + o[u]);
      q = fmaf(v[u], v[u], q);
    }
    uint4 pk;
    pk.x = pack2(v[0], v[1]);
    pk.y = pack2(v[2], v[3]);
    pk.z = pack2(v[4], v[5]);
    pk.w = pack2(v[6], v[7]);
    *reinterpret_cast<uint4*>(xs + (size_t)m * x_pitch + j * 16) = pk;
#pragma unroll
    for (int mm = 0; mm < 8; ++mm)
      if (mm == m) ss[mm] += q;
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const float q = warp_sum(ss[m]);
    if (lane == 0) nred[warp * 8 + m] = q;
  }
  named_sync(1, PK_CONSUMERS);
  float rs[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float q = 0.f;
#pragma unroll
    for (int w = 0; w < ST_CWARPS; ++w) q += nred[w * 8 + m];
    rs[m] = 1.0f / sqrtf(q / (float)H + a.eps);
  }
  for (int i = tid; i < M * kv; i += PK_CONSUMERS) {
    const int m = i / kv, j = i - m * kv;
    uint4* px = reinterpret_cast<uint4*>(xs + (size_t)m * x_pitch + j * 16);
    float f[8], w[8];
    cvt8(*px, f);
    cvt8(*reinterpret_cast<const uint4*>(nw + (size_t)j * 8), w);
    float r = 0.f;
#pragma unroll
    for (int mm = 0; mm < 8; ++mm)
      if (mm == m) r = rs[mm];
    uint4 o;
    o.x = pack2(w[0] * rbf(f[0] * r), w[1] * rbf(f[1] * r));
    o.y = pack2(w[2] * rbf(f[2] * r), w[3] * rbf(f[3] * r));
    o.z = pack2(w[4] * rbf(f[4] * r), w[5] * rbf(f[5] * r));
    o.w = pack2(w[6] * rbf(f[6] * r), w[7] * rbf(f[7] * r));
    *px = o;
  }
  named_sync(1, PK_CONSUMERS);
}

template <int G>
__global__ void __launch_bounds__(PK_THREADS, 1) dd_frame_kernel(const DDArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H, AE = a.AE, NH = a.NH, NKV = a.NKV, F = a.F, V = a.V, NST = a.nstages;
  unsigned char* xs = smem;
  unsigned char* zero16 = smem + a.xs_bytes;
  unsigned char* ringb = zero16 + 128;
  float* red = reinterpret_cast<float*>(ringb + (size_t)NST * ST_BYTES);
  float* sums = red + ST_CWARPS * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(sums + 128);
  uint64_t* empty = full + PK_MAX_STAGES;
  __shared__ float nred[ST_CWARPS * 8];
  __shared__ int s_int[32];

  const int tid = threadIdx.x, warp = tid >> 5;
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
  const int QKVU = (NH + 2 * NKV) * 64;  // rotary pair units
  auto qkv_row = [&](const DDLayer& W) {
    return [&W, NH, NKV, H](int u, int mat) -> const bf16* {
      const int hh = u >> 6, d = (u & 63) + mat * 64;
      if (hh < NH) return W.wq + (size_t)(hh * 128 + d) * H;
      if (hh < NH + NKV) return W.wk + (size_t)((hh - NH) * 128 + d) * H;
      return W.wv + (size_t)((hh - NH - NKV) * 128 + d) * H;
    };
  };

  if (warp == ST_CWARPS) {
    // ------------------------------------------------------------------ producer
    int t = 0;
    bool ok = true;
    for (int s = 0; s < a.NCB && ok; ++s) {
      ok = ok && produce_task<1>(rg, t, H, AE, [&](int n, int) { return a.proj + (size_t)n * AE; }, a.err);
      for (int l = 0; l < a.L && ok; ++l) {
        const DDLayer W = a.layers[l];
        ok = ok && produce_task<2>(rg, t, QKVU, H, qkv_row(W), a.err);
        ok = ok && produce_task<1>(rg, t, H, NH * 128, [&](int n, int) { return W.wo + (size_t)n * NH * 128; },
                                   a.err);
        ok = ok && produce_task<2>(rg, t, F, H, [&](int n, int mat) { return (mat ? W.wu : W.wg) + (size_t)n * H; },
                                   a.err);
        ok = ok && produce_task<1>(rg, t, H, F, [&](int n, int) { return W.wd + (size_t)n * F; }, a.err);
      }
      ok = ok && produce_task<1>(rg, t, V, H, [&](int n, int) { return a.head_t + ((size_t)s * V + n) * H; },
                                 a.err);
    }
    for (int u = max(0, t - NST); u < t; ++u)
      if (!mbar_wait_warp(&full[u % NST], (u / NST) & 1, a.err)) break;
    return;
  }

  // ------------------------------------------------------------------ consumers
  unsigned epoch = 0;
  int t = 0;
  const int half = a.B >= 2 ? a.B / 2 : 1;
  const int QD = NH * 128;
  const int xp_ae = AE * 2 + 16, xp_h = H * 2 + 16, xp_q = QD * 2 + 16, xp_f = F * 2 + 16;
  for (int s = 0; s < a.NCB; ++s) {
    const int T = s == 0 ? 2 : 1;
    const int M = a.B * T;
    // E: gather embeddings into xs, projector GEMV -> xres
    {
      const int kv = AE >> 3;
      const long long rows = (long long)(a.NCB + 1) * V;
      for (int i = tid; i < M * kv; i += PK_CONSUMERS) {
        const int m = i / kv, j = i - m * kv;
        const int b = m / T, tt = m - b * T;
        const uint4* src;
        if (s == 0 && tt == 0) {
          src = reinterpret_cast<const uint4*>(a.bh + (size_t)b * AE);
        } else {
          long long id = (s == 0) ? __ldcg(a.first_cb + b) : __ldcg(a.tokbuf + b) + (long long)s * V;
          id = id < 0 ? 0 : (id >= rows ? rows - 1 : id);
          src = reinterpret_cast<const uint4*>(a.embed + (size_t)id * AE);
        }
        *reinterpret_cast<uint4*>(xs + (size_t)m * xp_ae + j * 16) = __ldcg(src + j);
      }
      named_sync(1, PK_CONSUMERS);
      if (!consume_task<1>(rg, t, H, AE, xs, xp_ae, M, zero16, red, sums,
                           [&](int n0, int nu, const float* sm) {
                             if (tid < nu * M) {
                               const int i = tid / M, m = tid - i * M;
                               a.xres[(size_t)m * H + n0 + i] = __float2bfloat16_rn(sm[i * 8 + m]);
                             }
                           }, a.err)) return;
      if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
    }
    for (int l = 0; l < a.L; ++l) {
      const DDLayer W = a.layers[l];
      // S1: RMSNorm + q|k|v (rotary pairs) + RoPE + KV write
      load_x(xs, xp_h, a.xres, H, M, H, W.ln1, a.eps, nred);
      if (!consume_task<2>(rg, t, QKVU, H, xs, xp_h, M, zero16, red, sums,
                           [&](int n0, int nu, const float* sm) {
                             if (tid < nu * M) {
                               const int i = tid / M, m = tid - i * M;
                               const int u = n0 + i, hh = u >> 6, d = u & 63;
                               const int b = m / T, tt = m - b * T;
                               const int pos = s == 0 ? tt : s + 1;
                               float y0 = rbf(sm[i * 8 + m]), y1 = rbf(sm[(i + 8) * 8 + m]);
                               if (hh < NH + NKV) {
                                 const float c0 = b2f(a.cos_tab[pos * 128 + d]), s0 = b2f(a.sin_tab[pos * 128 + d]);
                                 const float c1 = b2f(a.cos_tab[pos * 128 + d + 64]);
                                 const float s1 = b2f(a.sin_tab[pos * 128 + d + 64]);
                                 const float o0 = rbf(rbf(y0 * c0) + rbf(-y1 * s0));
                                 const float o1 = rbf(rbf(y1 * c1) + rbf(y0 * s1));
                                 y0 = o0;
                                 y1 = o1;
                               }
                               if (hh < NH) {
                                 a.qb[(size_t)m * QD + hh * 128 + d] = __float2bfloat16_rn(y0);
                                 a.qb[(size_t)m * QD + hh * 128 + d + 64] = __float2bfloat16_rn(y1);
                               } else {
                                 const int kvh = hh < NH + NKV ? hh - NH : hh - NH - NKV;
                                 bf16* cache = hh < NH + NKV ? a.kc : a.vc;
                                 bf16* dst = cache + ((((size_t)l * a.B + b) * NKV + kvh) * a.P + pos) * 128;
                                 dst[d] = __float2bfloat16_rn(y0);
                                 dst[d + 64] = __float2bfloat16_rn(y1);
                               }
                             }
                           }, a.err)) return;
      if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
      // S2: attention (every CTA, all rows) + o GEMV
      dd_attention<G>(a, l, s, T, xs, xp_q);
      if (!consume_task<1>(rg, t, H, QD, xs, xp_q, M, zero16, red, sums,
                           [&](int n0, int nu, const float* sm) {
                             if (tid < nu * M) {
                               const int i = tid / M, m = tid - i * M;
                               a.ob[(size_t)m * H + n0 + i] = __float2bfloat16_rn(sm[i * 8 + m]);
                             }
                           }, a.err)) return;
      if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
      // S3: RMSNorm(bf16(x + o)) + gate|up + SiLU*up
      dd_load_mid(xs, xp_h, a, M, W.ln2, nred);
      if (!consume_task<2>(rg, t, F, H, xs, xp_h, M, zero16, red, sums,
                           [&](int n0, int nu, const float* sm) {
                             if (tid < nu * M) {
                               const int i = tid / M, m = tid - i * M;
                               const float g = rbf(sm[i * 8 + m]);
                               const float u = rbf(sm[(i + 8) * 8 + m]);
                               a.act[(size_t)m * F + n0 + i] = __float2bfloat16_rn(rbf(g / (1.0f + expf(-g))) * u);
                             }
                           }, a.err)) return;
      if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
      // S4: down + residual: xres = bf16(bf16(xres + o) + bf16(d))
      load_x(xs, xp_f, a.act, F, M, F, nullptr, 0.f, nred);
      if (!consume_task<1>(rg, t, H, F, xs, xp_f, M, zero16, red, sums,
                           [&](int n0, int nu, const float* sm) {
                             if (tid < nu * M) {
                               const int i = tid / M, m = tid - i * M, n = n0 + i;
                               const float xm = rbf(b2f(__ldcg(a.xres + (size_t)m * H + n)) +
                                                    b2f(__ldcg(a.ob + (size_t)m * H + n)));
                               a.xres[(size_t)m * H + n] = __float2bfloat16_rn(xm + rbf(sm[i * 8 + m]));
                             }
                           }, a.err)) return;
      if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
    }
    // S5: final RMSNorm of each row's last token + codebook head -> fp32 logits
    load_x(xs, xp_h, a.xres + (size_t)(T - 1) * H, (long)T * H, a.B, H, a.normf, a.eps, nred);
    if (!consume_task<1>(rg, t, V, H, xs, xp_h, a.B, zero16, red, sums,
                         [&](int n0, int nu, const float* sm) {
                           if (tid < nu * a.B) {
                             const int i = tid / a.B, b = tid - i * a.B;
                             const float v = sm[i * 8 + b];
                             a.logits[(size_t)b * V + n0 + i] = v;
                             if (a.dbg) a.dbg[((size_t)s * a.B + b) * V + n0 + i] = v;
                           }
                         }, a.err)) return;
    if (!grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
    if ((int)blockIdx.x < half) dd_sample(a, s, blockIdx.x, reinterpret_cast<unsigned long long*>(xs), s_int);
    if (s + 1 < a.NCB && !grid_sync(a.bar, epoch, a.err, &s_int[31])) return;
  }
  grid_exit(a.bar);
}

}  // namespace fb

// ------------------------------------------------------------------------------------------------ host API
namespace {
using namespace fb;

struct DDLayout {
  size_t xres, qb, ob, act, kc, vc, logits, bar, total;
};
size_t al256d(size_t v) { return (v + 255) / 256 * 256; }

DDLayout dd_layout(const fb_dd_config* c) {
  DDLayout s{};
  const size_t M = (size_t)c->batch * 2;
  const size_t P = (size_t)c->n_decode + 1;
  size_t o = 0;
  s.xres = o; o = al256d(o + M * c->hidden * 2);
  s.qb = o; o = al256d(o + M * c->heads * 128 * 2);
  s.ob = o; o = al256d(o + M * c->hidden * 2);
  s.act = o; o = al256d(o + M * c->ffn * 2);
  s.kc = o; o = al256d(o + (size_t)c->layers * c->batch * c->kv_heads * P * 128 * 2);
  s.vc = o; o = al256d(o + (size_t)c->layers * c->batch * c->kv_heads * P * 128 * 2);
  s.logits = o; o = al256d(o + (size_t)c->batch * c->vocab * 4);
  s.bar = o; o = al256d(o + sizeof(GridBar));
  s.total = o;
  return s;
}

template <int G>
int launch_dd(DDArgs& a, size_t smem, cudaStream_t st) {
  auto kern = dd_frame_kernel<G>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_done[dev] < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("dd_frame: cudaFuncSetAttribute(%zu): %s", smem, cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = (int)smem;
  }
  int nb = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, PK_THREADS, smem);
  if (e != cudaSuccess || nb < 1) {
    fbh::set_msg("dd_frame: kernel not resident (occupancy %d): %s", nb, cudaGetErrorString(e));
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
    fbh::set_msg("dd_frame launch: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return FB_OK;
}

}  // namespace

extern "C" int64_t flashb_dd_scratch_bytes(const fb_dd_config* cfg) {
  if (!cfg) return -1;
  return (int64_t)dd_layout(cfg).total;
}

extern "C" int64_t flashb_dd_layer_bytes(void) { return (int64_t)sizeof(fb_dd_layer); }

extern "C" int flashb_dd_frame(const fb_dd_config* c, const void* layers_dev, void* scratch, const int64_t* first_cb,
                               const void* bh, int64_t* tokbuf, int64_t* outtok, const float* temp,
                               const int64_t* topk, const float* topp, const int64_t* dosample, const float* gs,
                               const float* q, float* dbg, const int64_t* forced, void* stream) {
  static_assert(sizeof(fb_dd_layer) == sizeof(DDLayer), "fb_dd_layer layout");
  FB_CHECK_ARG(c && layers_dev && scratch && first_cb && bh && tokbuf && outtok && temp && topk && topp && dosample &&
                   gs && q, "dd_frame: null pointer argument");
  FB_CHECK_ARG(c->head_dim == 128 && c->batch >= 1 && c->batch <= DD_MAXB && (c->batch == 1 || c->batch % 2 == 0),
               "dd_frame: head_dim must be 128, batch 1, 2 or 4");
  FB_CHECK_ARG(c->vocab >= 1 && c->vocab <= DD_MAXV && c->codebook_size >= 1 && c->codebook_size <= c->vocab,
               "dd_frame: vocab must be <= %d and codebook_size <= vocab", DD_MAXV);
  FB_CHECK_ARG(c->n_decode >= 1 && c->n_decode <= 31, "dd_frame: n_decode must be 1..31");
  FB_CHECK_ARG(c->hidden % 16 == 0 && c->embed_dim % 16 == 0 && c->ffn % 16 == 0 && c->heads % c->kv_heads == 0,
               "dd_frame: bad dims");
  FB_CHECK_ARG(((uintptr_t)scratch & 255) == 0, "dd_frame: scratch must be 256-byte aligned");
  const DDLayout Lo = dd_layout(c);
  DDArgs a{};
  a.L = c->layers; a.B = c->batch; a.H = c->hidden; a.AE = c->embed_dim; a.NH = c->heads; a.NKV = c->kv_heads;
  a.F = c->ffn; a.V = c->vocab; a.CB = c->codebook_size; a.NCB = c->n_decode; a.P = c->n_decode + 1;
  a.eps = c->eps; a.scaling = c->scaling;
  a.layers = (const DDLayer*)layers_dev;
  a.embed = (const bf16*)c->embed; a.proj = (const bf16*)c->proj; a.normf = (const bf16*)c->normf;
  a.head_t = (const bf16*)c->head_t; a.cos_tab = (const bf16*)c->cos_tab; a.sin_tab = (const bf16*)c->sin_tab;
  a.first_cb = (const long long*)first_cb; a.bh = (const bf16*)bh; a.tokbuf = (long long*)tokbuf;
  a.outtok = (long long*)outtok; a.temp = temp; a.topk = (const long long*)topk; a.topp = topp;
  a.dosample = (const long long*)dosample; a.gs = gs; a.q = q; a.dbg = dbg; a.forced = (const long long*)forced;
  unsigned char* sc = (unsigned char*)scratch;
  a.xres = (bf16*)(sc + Lo.xres); a.qb = (bf16*)(sc + Lo.qb); a.ob = (bf16*)(sc + Lo.ob);
  a.act = (bf16*)(sc + Lo.act); a.kc = (bf16*)(sc + Lo.kc); a.vc = (bf16*)(sc + Lo.vc);
  a.logits = (float*)(sc + Lo.logits); a.bar = (GridBar*)(sc + Lo.bar);
  a.err = fbh::device_err_ptr();
  int kmax = c->embed_dim;
  if (c->ffn > kmax) kmax = c->ffn;
  if (c->heads * 128 > kmax) kmax = c->heads * 128;
  if (c->hidden > kmax) kmax = c->hidden;
  const size_t M = (size_t)c->batch * 2;
  size_t xs = al256d(M * (kmax * 2 + 16));
  if (xs < (size_t)DD_MAXV * 8) xs = (size_t)DD_MAXV * 8;  // sampler keys reuse the activation buffer
  a.xs_bytes = (int)xs;
  const size_t fixed = xs + 128 + ST_CWARPS * 128 * 4 + 128 * 4 + 2 * PK_MAX_STAGES * 8;
  const size_t budget = 227 * 1024 - ST_CWARPS * 8 * 4 - 32 * 4 - 256;
  int nst = (int)((budget - fixed) / ST_BYTES);
  if (nst > PK_MAX_STAGES) nst = PK_MAX_STAGES;
  if (nst < 2) {
    fbh::set_msg("dd_frame: activations too large for two ring stages");
    return FB_ERR_UNSUPPORTED;
  }
  a.nstages = nst;
  const size_t smem = fixed + (size_t)nst * ST_BYTES;
  cudaStream_t st = (cudaStream_t)stream;
  switch (c->heads / c->kv_heads) {
    case 1: return launch_dd<1>(a, smem, st);
    case 2: return launch_dd<2>(a, smem, st);
    case 4: return launch_dd<4>(a, smem, st);
    case 8: return launch_dd<8>(a, smem, st);
    default: fbh::set_msg("dd_frame: GQA group %d not built", c->heads / c->kv_heads); return FB_ERR_UNSUPPORTED;
  }
}
