// flashb: one depth-decoder frame (every codebook of the frame, CFG sampling included) as ONE persistent launch.
//
// Follows the official graph loop DepthDecoderGraph._full_loop (UP/models/cudagraph/depth_decoder_graph.py:558-654,
// UP = third_party/breeze-tts) with the eager rounding points of BreezeDecoderLayer (UP/models/breeze.py:378-425), and
// replaces the reference's depth megakernel (flash/csrc/depth_frame.cu:656-853) with a B200 design: one CTA per SM,
// a producer warp streaming every weight slice of the frame (projector, 4 x {q|k|v, o, gate|up, down}, codebook
// head) through the stage ring (fb_stream.cuh, tensor-core GEMV), consumer warps running the tasks between
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
//     sampler  every CTA samples every half-row (redundantly, so no barrier follows): CFG, codec-id mask,
//              temperature, top-k (radix select of the k-th largest key, then a sort of the k survivors), top-p,
//              softmax, argmax(p / q), with its own exp routine and fixed summation order, bit-identical to the C
//              oracle (oracle/sampler.c); CTA 0 writes the tokens out, every CTA feeds its copy to the next step
//
// Stages are 32 KB (16 x 1024 columns in the mma.sync build; 64 or 128 weight rows x 256 or 128 columns in the
// tcgen05 build of lane-sized grids, whose GEMVs run on tcgen05.mma with the 16 activation rows as N); the ring
// holds as many as fit beside the activations (three or four at the full-size model) and the producer runs ahead
// across tasks.  Global -> shared staging of activations (cross-CTA data) uses cp.async.cg with every chunk in
// flight at once: one L2 round trip per phase.  The large phases are not inlined so that a step's code stays
// resident in the instruction cache.
//
// Scratch (residual stream, q, o, act, logits, KV cache, barrier, split-task partials and tags) is one caller-owned
// buffer, zeroed once.
#define FB_ST_KC 1024
#define FB_ST_TMA 1
#define FB_PK_MAX_STAGES 8
#include <cstring>
#include <mutex>

#include "fb_persist.cuh"
#include "fb_sample.cuh"
#include "fb_tc.cuh"

namespace fb {

constexpr int DD_MAXB = 16;     // batch rows (eight CFG pairs)
constexpr int DD_MAXV = 4096;   // sampler vocabulary bound (composite key packs 12 index bits)
constexpr int DD_MAXL = 8;      // layers (their tensor maps travel in the argument block)
constexpr int DD_TC_KX = 2048;  // tcgen05 build: activation columns staged at once (larger K runs in passes)
constexpr int DD_TC_SUMS = 2048;  // tcgen05 build: floats of the accumulator dump (8 groups x 16 rows x 16)
#ifndef DD_TC_MAX_GRID
#define DD_TC_MAX_GRID 32         // tcgen05 build on grids of at most this many CTAs
#endif
enum { DD_WQ, DD_WK, DD_WV, DD_WO, DD_WG, DD_WU, DD_WD, DD_NMAPS };

struct DDLayer {
  const bf16 *ln1, *wq, *wk, *wv, *wo, *ln2, *wg, *wu, *wd;
};

// LN12 streaming (tcgen05 build): a depth matrix in the lossless 12-bit format -- its data bytes behind a tensor map
// (fbh::tmap_ln12), the 16-byte row records (header, three inline patches), the overflow patches and their count,
// the 8-entry exponent table as two words.
constexpr int DD_MAXH = 31;           // codebook heads (n_decode <= 31)
struct LNMat {
  const uint4* meta;
  const unsigned* ovf;
  long long novf;
  unsigned lo, hi;
};

struct alignas(64) DDArgs {
  CUtensorMap tm_proj, tm_head;           // projector [H, AE]; codebook heads [n_decode * V, H]
  CUtensorMap tm[DD_MAXL][DD_NMAPS];      // per layer: wq, wk, wv, wo, wg, wu, wd
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
  int nstages, xs_bytes, att_off, keep_off, att_bc, att_split, d_xchunk;
  int keep_cols;                          // tcgen05 build: x_mid kept only for the CTA's S4 columns (0 = all)
  // tcgen05 bf16 build: 128-row tasks with split K (0 = the 64-row task) for the projector, o, down, the heads; the
  // fp32 partial sums of split parts and their per-block publication tags (zeroed at every frame start)
  int s3_proj, s3_o, s3_down, s3_head;
  float* part;
  unsigned* flags;
  int nflags;
  unsigned long long wait_ns;             // grid-barrier wait limit
  const bf16 *ptab, *ttab;                // optional per-token step table (codebook steps >= 1), or null
  int l2_keep;                            // 1: weight copies carry the L2 evict_last hint
  unsigned* err;
  unsigned long long* trace;
  int ln12;                               // 1: tm / tm_proj / tm_hd map LN12 data (tcgen05 build)
  LNMat ln[DD_MAXL][DD_NMAPS], ln_proj, ln_hd[DD_MAXH];
  CUtensorMap tm_hd[DD_MAXH];             // LN12: one map per codebook head [V, H]
};
static_assert(sizeof(DDArgs) <= 32764, "the depth frame's argument block exceeds the kernel parameter limit");

// Optional trace: thread 0 of each CTA stamps %globaltimer at the end of every task and barrier of step s
// (row layout [grid][n_decode][11 + 9 * layers]: start, E, barrier, 9 per layer, head, barrier, 6 sampler phases).
#define DD_TRACE_SLOTS(L) (11 + 9 * (L))
// tcgen05 build: after the phase rows, a detail row of 8 stamps for each of the first DD_DETAIL_CALLS GEMV tasks of
// each CTA ([grid][DD_DETAIL_CALLS][8]: task entry, first stage in, last MMA issued, MMAs complete, accumulators
// dumped, epilogues done, task end; blocks of the task)
#define DD_DETAIL_CALLS 64
#define DD_STAMP(s, idx)                                                                                   \
  do {                                                                                                     \
    if (a.trace && threadIdx.x == 0)                                                                       \
      a.trace[((size_t)blockIdx.x * a.NCB + (s)) * DD_TRACE_SLOTS(a.L) + (idx)] =                          \
          (unsigned long long)globaltimer();                                                               \
  } while (0)

// Shared-memory layout of the sampler inside the activation buffer: V composite keys, up to 1024 sorted survivors,
// two 256-bin histograms, the two logit rows.
__host__ __device__ constexpr size_t dd_sampler_bytes(int V) {
  return (size_t)V * 8 + 1024 * 8 + 2 * 256 * 4 + 2 * (size_t)V * 4;
}

// Sampler for half-row h (all 256 consumer threads of the CTA); returns the sampled token (before forcing).
// Composite key = (order-preserving bits of cfg / temperature) << 12 | (4095 - index): descending key order is the
// official order (value descending, ties by lower index).  The kk largest keys are found by radix selection on 8-bit
// digits (histograms in shared memory, early exit once the boundary bin is taken whole), gathered, and sorted
// descending by a bitonic network (one warp up to 64 survivors).  Warp 0 then runs the canonical sums of
// oracle/sampler.c on the sorted survivors.
__device__ __noinline__ int dd_sample(const DDArgs& a, int step, int h, unsigned char* buf, int* s_int) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = a.B >= 2 ? a.B / 2 : 1;
  const int V = a.V;
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(buf);
  unsigned long long* top = keys + V;
  unsigned* hist = reinterpret_cast<unsigned*>(top + 1024);
  float* lg = reinterpret_cast<float*>(hist + 512);
  {
    // both logit rows to shared memory in one round trip (cp.async.cg: written by other CTAs, L2 only)
    const float* g0 = a.logits + (size_t)h * V;
    const float* g1 = a.B >= 2 ? a.logits + (size_t)(h + half) * V : nullptr;
    if ((V & 3) == 0) {
      const int nch = V >> 2;
      for (int i = tid; i < (g1 ? 2 : 1) * nch; i += PK_CONSUMERS)
        cp_async16(lg + (size_t)i * 4, (i < nch ? g0 + (size_t)i * 4 : g1 + (size_t)(i - nch) * 4));
      cp_async_commit();
      cp_async_wait<0>();
    } else {
      for (int i = tid; i < V; i += PK_CONSUMERS) {
        lg[i] = __ldcg(g0 + i);
        if (g1) lg[V + i] = __ldcg(g1 + i);
      }
    }
    named_sync(1, PK_CONSUMERS);
  }
  const float* lc = lg;
  const float* lu = a.B >= 2 ? lg + V : nullptr;
  const float gs = a.gs[h], temp = a.temp[h], topp = a.topp[h];
  const long long tk = a.topk[h];
  const bool dosample = a.dosample[h] != 0;
  // 1) CFG, codec mask, temperature -> composite keys; greedy argmax(cfg)
  float gbest = -INFINITY;
  int gidx = 0x7fffffff;
  for (int i = tid; i < V; i += PK_CONSUMERS) {
    float cfg = lc[i];
    if (lu) {
      const float u = lu[i];
      cfg = __fadd_rn(u, __fmul_rn(gs, __fsub_rn(cfg, u)));
    }
    if (i >= a.CB) cfg = -INFINITY;
    if (cfg > gbest || (cfg == gbest && i < gidx)) {
      gbest = cfg;
      gidx = i;
    }
    const float key = __fdiv_rn(cfg, temp);
    keys[i] = ((unsigned long long)f2ord(key) << 12) | (unsigned long long)(4095 - i);
  }
  hist[tid] = 0u;
  hist[256 + tid] = 0u;
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
  if (tid == 0) s_int[12] = 0;   // survivor counter
  named_sync(1, PK_CONSUMERS);
  DD_STAMP(step, 3 + 9 * a.L + 2);
  if (!dosample) {
    float bv = gv[0];
    int bi = s_int[16];
    for (int w = 1; w < ST_CWARPS; ++w)
      if (gv[w] > bv || (gv[w] == bv && s_int[16 + w] < bi)) {
        bv = gv[w];
        bi = s_int[16 + w];
      }
    named_sync(1, PK_CONSUMERS);
    return bi;
  }
  const int maxk = V < 1024 ? V : 1024;
  const int kk = tk > 0 ? (tk < maxk ? (int)tk : maxk) : maxk;
  // 2) radix select of the kk-th largest key (keys are unique: the low 12 bits hold the index)
  unsigned long long prefix = 0ull, pmask = 0ull;
  int r = kk;
  const int shifts[6] = {36, 28, 20, 12, 4, 0};
  for (int p = 0; p < 6; ++p) {
    const int sh = shifts[p];
    unsigned* hc = hist + (p & 1) * 256;
    for (int i = tid; i < V; i += PK_CONSUMERS) {
      const unsigned long long k = keys[i];
      if ((k & pmask) == prefix) atomicAdd(&hc[(unsigned)(k >> sh) & 255u], 1u);
    }
    named_sync(1, PK_CONSUMERS);
    if (warp == 0) {
      unsigned c[8];
      unsigned tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hc[255 - 8 * lane - j];
        tot += c[j];
      }
      unsigned incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned excl = incl - tot;
      const unsigned hit = __ballot_sync(FULL, excl < (unsigned)r && (unsigned)r <= incl);
      if (lane == __ffs(hit) - 1) {
        int rr = r - (int)excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (rr > 0 && rr <= (int)c[j]) {
            s_int[1] = 255 - 8 * lane - j;
            s_int[2] = rr;
            s_int[3] = (int)c[j] == rr;
            rr = 0;
          } else if (rr > 0) {
            rr -= (int)c[j];
          }
        }
      }
    }
    hist[((p + 1) & 1) * 256 + tid] = 0u;   // clear the other histogram for the next pass
    named_sync(1, PK_CONSUMERS);
    prefix |= (unsigned long long)s_int[1] << sh;
    pmask |= 255ull << sh;
    r = s_int[2];
    if (s_int[3]) break;
  }
  DD_STAMP(step, 3 + 9 * a.L + 3);
  // 3) gather the kk survivors (key >= threshold; exactly kk of them), pad to a power of two, sort descending
  int n2 = 1;
  while (n2 < kk) n2 <<= 1;
  if (n2 < 64) n2 = 64;                      // up to 64 survivors: one register sort in warp 0
  for (int i = tid; i < V; i += PK_CONSUMERS) {
    const unsigned long long k = keys[i];
    if (k >= prefix) top[atomicAdd(&s_int[12], 1)] = k;
  }
  for (int i = kk + tid; i < n2; i += PK_CONSUMERS) top[i] = 0ull;
  named_sync(1, PK_CONSUMERS);
  if (n2 == 64) {
    if (warp == 0) {
      // bitonic network over elements i = lane (e0) and i = lane + 32 (e1), partners exchanged by shuffles; the
      // position with bit j clear keeps the larger key in a descending block (bit k clear), the smaller otherwise
      unsigned long long e0 = top[lane], e1 = top[lane + 32];
#pragma unroll
      for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
          if (j == 32) {
            if (e0 < e1) {                   // k = 64: one descending block; position lane is the lower one
              const unsigned long long x = e0;
              e0 = e1;
              e1 = x;
            }
          } else {
            const unsigned long long o0 = __shfl_xor_sync(FULL, e0, j), o1 = __shfl_xor_sync(FULL, e1, j);
            const bool lo = (lane & j) == 0;
            const bool d0 = (lane & k) == 0, d1 = ((lane + 32) & k) == 0;
            e0 = (d0 == lo) ? (e0 > o0 ? e0 : o0) : (e0 < o0 ? e0 : o0);
            e1 = (d1 == lo) ? (e1 > o1 ? e1 : o1) : (e1 < o1 ? e1 : o1);
          }
        }
      }
      top[lane] = e0;
      top[lane + 32] = e1;
      __syncwarp();
    }
  } else {
    for (int k = 2; k <= n2; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < (n2 >> 1); i += PK_CONSUMERS) {
          const int lo = 2 * i - (i & (j - 1)), hi = lo + j;
          const unsigned long long x = top[lo], y = top[hi];
          if (((lo & k) == 0) ? (x < y) : (x > y)) {
            top[lo] = y;
            top[hi] = x;
          }
        }
        named_sync(1, PK_CONSUMERS);
      }
  }
  DD_STAMP(step, 3 + 9 * a.L + 4);
  // 4) warp 0: top-p / softmax / argmax(p / q) with the canonical sums (lane l owns ranks l*C .. l*C+C-1)
  if (warp == 0) {
    const int C = (kk + 31) / 32;
    const float key0 = ord2f((unsigned)(top[0] >> 12));
    auto e_of = [&](int rk) { return fb_exp_dev(__fsub_rn(ord2f((unsigned)(top[rk] >> 12)), key0)); };
    float bsum = 0.f;
    for (int j = 0; j < C; ++j) {
      const int rk = lane * C + j;
      if (rk < kk) bsum = __fadd_rn(bsum, e_of(rk));
    }
    const float S = __shfl_sync(FULL, lane_scan(bsum), 31);
    DD_STAMP(step, 3 + 9 * a.L + 5);
    float bp = 0.f;
    for (int j = 0; j < C; ++j) {
      const int rk = lane * C + j;
      if (rk < kk) bp = __fadd_rn(bp, __fdiv_rn(e_of(rk), S));
    }
    const float inclp = lane_scan(bp);
    const float exclp = __shfl_up_sync(FULL, inclp, 1);
    float run = lane ? exclp : 0.f;
    float s2 = 0.f;
    unsigned keepmask = 0u;
    for (int j = 0; j < C; ++j) {
      const int rk = lane * C + j;
      if (rk >= kk) break;
      const float e = e_of(rk);
      const bool keep = (rk == 0) || !(run > topp);
      run = __fadd_rn(run, __fdiv_rn(e, S));
      if (keep) {
        s2 = __fadd_rn(s2, e);
        keepmask |= 1u << j;
      }
    }
    const float S2 = __shfl_sync(FULL, lane_scan(s2), 31);
    DD_STAMP(step, 3 + 9 * a.L + 6);
    const float* qrow = a.q + ((size_t)step * half + h) * V;
    float best = -1.f;
    int bidx = 0x7fffffff;
    for (int j = 0; j < C; ++j) {
      if (!((keepmask >> j) & 1u)) continue;
      const int rk = lane * C + j;
      const int id = 4095 - (int)(top[rk] & 4095ull);
      const float sc = __fdiv_rn(__fdiv_rn(e_of(rk), S2), __ldg(qrow + id));
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
    if (lane == 0) s_int[0] = bidx;
  }
  named_sync(1, PK_CONSUMERS);
  return s_int[0];
}

// ------------------------------------------------------------------------------------------------ attention (S2)
// Shared-memory bytes of the attention staging area for a chunk of `bc` batch rows (their q rows, the layer's K and
// V of every position for their KV heads, scores).
__host__ __device__ constexpr size_t dd_attn_bytes(int bc, int NH, int NKV, int P) {
  return (size_t)bc * NH * 256 + 2 * (size_t)bc * NKV * P * 256 + (size_t)bc * NH * 32 * 4;
}

// The step's token at position `pos` of every batch row, all NH query heads, over the layer's cached positions
// 0..pos, computed by every CTA (the o-projection that follows needs every row).  Batch rows go in chunks of
// a.att_bc; per chunk one round trip stages q, K and V in shared memory with cp.async, then scores (one thread per
// (row, key)), softmax (a warp per row) and p.V (one thread per (row, 8 dims)).  Eager rounding:
// s = bf16(bf16(q.k) * scaling), p = bf16(softmax_fp32(s)), out = bf16(sum p v).  Output rows go to xs (the
// o-projection input); `att` is the staging area.
template <int G>
__device__ __noinline__ void dd_attention(const DDArgs& a, int l, int pos, unsigned char* xs, int x_pitch,
                                          unsigned char* att) {
  const int tid = threadIdx.x;
  const int NH = a.NH, NKV = a.NKV, QD = NH * 128;
  const int np = pos + 1;
  for (int b0 = 0; b0 < a.B; b0 += a.att_bc) {
    const int nb = min(a.att_bc, a.B - b0);
    const int nrow = nb * NH;
    bf16* qs = reinterpret_cast<bf16*>(att);
    bf16* ks = qs + (size_t)nrow * 128;
    bf16* vs = ks + (size_t)nb * NKV * np * 128;
    float* ps = reinterpret_cast<float*>(vs + (size_t)nb * NKV * np * 128);
    const int qch = nrow * 16, kch = nb * NKV * np * 16;
    for (int i = tid; i < qch + 2 * kch; i += PK_CONSUMERS) {
      const bf16* src;
      bf16* dst;
      if (i < qch) {
        const int row = i >> 4, c = i & 15, bb = row / NH, qh = row - bb * NH;
        src = a.qb + (size_t)(b0 + bb) * QD + qh * 128 + c * 8;
        dst = qs + (size_t)row * 128 + c * 8;
      } else {
        int j = i - qch;
        const bool isv = j >= kch;
        if (isv) j -= kch;
        const int row = j >> 4, c = j & 15, bk = row / np, p = row - bk * np;
        const int bb = bk / NKV, kvh = bk - bb * NKV;
        src = (isv ? a.vc : a.kc) + ((((size_t)l * a.B + b0 + bb) * NKV + kvh) * a.P + p) * 128 + c * 8;
        dst = (isv ? vs : ks) + (size_t)row * 128 + c * 8;
      }
      cp_async16(dst, src);
    }
    cp_async_commit();
    cp_async_wait<0>();
    named_sync(1, PK_CONSUMERS);
    for (int i = tid; i < nrow * np; i += PK_CONSUMERS) {
      const int row = i / np, j = i - row * np;
      const int bb = row / NH, qh = row - bb * NH;
      const uint4* qr = reinterpret_cast<const uint4*>(qs + (size_t)row * 128);
      const uint4* kr = reinterpret_cast<const uint4*>(ks + ((size_t)(bb * NKV + qh / G) * np + j) * 128);
      float d = 0.f;
#pragma unroll 4
      for (int cc = 0; cc < 16; ++cc) {
        const int c = (cc + j) & 15;               // rotate the chunk order by key: fewer bank conflicts
        float qf[8], kf[8];
        cvt8(qr[c], qf);
        cvt8(kr[c], kf);
#pragma unroll
        for (int u = 0; u < 8; ++u) d = fmaf(qf[u], kf[u], d);
      }
      ps[row * 32 + j] = rbf(rbf(d) * a.scaling);
    }
    named_sync(1, PK_CONSUMERS);
    // softmax per row: a warp per row, a lane per key (np <= 32)
    for (int row = tid >> 5; row < nrow; row += PK_CONSUMERS / 32) {
      float* pr = ps + row * 32;
      const int lane = tid & 31;
      const float v = lane < np ? pr[lane] : -INFINITY;
      const float mx = warp_max(v);
      const float e = lane < np ? __expf(v - mx) : 0.f;
      const float den = warp_sum(e);
      if (lane < np) pr[lane] = rbf(e / den);
    }
    named_sync(1, PK_CONSUMERS);
    for (int i = tid; i < nrow * 16; i += PK_CONSUMERS) {
      const int row = i >> 4, c = i & 15;
      const int bb = row / NH, qh = row - bb * NH;
      const float* pr = ps + row * 32;
      const bf16* vb = vs + (size_t)(bb * NKV + qh / G) * np * 128 + c * 8;
      float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < np; ++j) {
        float vf[8];
        cvt8(*reinterpret_cast<const uint4*>(vb + (size_t)j * 128), vf);
        const float p = pr[j];
#pragma unroll
        for (int u = 0; u < 8; ++u) o[u] = fmaf(p, vf[u], o[u]);
      }
      uint4 ov;
      ov.x = pack2(o[0], o[1]);
      ov.y = pack2(o[2], o[3]);
      ov.z = pack2(o[4], o[5]);
      ov.w = pack2(o[6], o[7]);
      *reinterpret_cast<uint4*>(xs + xs_off(b0 + bb, qh * 16 + c, x_pitch)) = ov;
    }
    named_sync(1, PK_CONSUMERS);
  }
}

// Shared-memory bytes of one (batch row, KV head) pair in the distributed attention mode: its G q rows, the layer's
// K and V of positions 0..P-1, G x 32 scores.
__host__ __device__ constexpr size_t dd_pair_bytes(int G, int P) {
  return (size_t)G * 256 + 2 * (size_t)P * 256 + (size_t)G * 32 * 4;
}

// Distributed attention: this CTA's (batch row, KV head) pairs [p0, p1) (pair i = row i / NKV, KV head i % NKV),
// all staged in one cp.async round trip.  The same arithmetic and rounding points as dd_attention; the output goes
// over each pair's q slice in a.qb (no other CTA reads that slice before the barrier that follows).
template <int G>
__device__ __noinline__ void dd_attention_pairs(const DDArgs& a, int l, int pos, int p0, int p1, unsigned char* att) {
  const int tid = threadIdx.x;
  const int QD = a.NH * 128, NKV = a.NKV;
  const int np = pos + 1, npair = p1 - p0;
  if (npair <= 0) return;
  const size_t pb = dd_pair_bytes(G, np);
  auto qs_of = [&](int k) { return reinterpret_cast<bf16*>(att + (size_t)k * pb); };
  auto ks_of = [&](int k) { return qs_of(k) + G * 128; };
  auto vs_of = [&](int k) { return ks_of(k) + (size_t)np * 128; };
  auto ps_of = [&](int k) { return reinterpret_cast<float*>(vs_of(k) + (size_t)np * 128); };
  auto qg_of = [&](int k) {
    const int pi = p0 + k, b = pi / NKV, kvh = pi - b * NKV;
    return a.qb + (size_t)b * QD + (size_t)kvh * G * 128;
  };
  const int qch = G * 16, kch = np * 16, per = qch + 2 * kch;
  for (int i = tid; i < npair * per; i += PK_CONSUMERS) {
    const int k = i / per;
    int j = i - k * per;
    if (j < qch) {
      cp_async16(qs_of(k) + (size_t)j * 8, qg_of(k) + (size_t)j * 8);
    } else {
      j -= qch;
      const bool isv = j >= kch;
      if (isv) j -= kch;
      const int pi = p0 + k, b = pi / NKV, kvh = pi - b * NKV;
      const size_t kvoff = ((((size_t)l * a.B + b) * NKV + kvh) * a.P) * 128;
      cp_async16((isv ? vs_of(k) : ks_of(k)) + (size_t)j * 8, (isv ? a.vc : a.kc) + kvoff + (size_t)j * 8);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  named_sync(1, PK_CONSUMERS);
  const float scaling = a.scaling;
  for (int i = tid; i < npair * G * np; i += PK_CONSUMERS) {
    const int k = i / (G * np);
    const int r = i - k * G * np;
    const int hq = r / np, j = r - hq * np;
    const uint4* qr = reinterpret_cast<const uint4*>(qs_of(k) + (size_t)hq * 128);
    const uint4* kr = reinterpret_cast<const uint4*>(ks_of(k) + (size_t)j * 128);
    float d = 0.f;
#pragma unroll 4
    for (int cc = 0; cc < 16; ++cc) {
      const int c = (cc + j) & 15;
      float qf[8], kf[8];
      cvt8(qr[c], qf);
      cvt8(kr[c], kf);
#pragma unroll
      for (int u = 0; u < 8; ++u) d = fmaf(qf[u], kf[u], d);
    }
    ps_of(k)[hq * 32 + j] = rbf(rbf(d) * scaling);
  }
  named_sync(1, PK_CONSUMERS);
  // softmax per (pair, q head) row: a warp per row, a lane per key (np <= 32)
  for (int row = tid >> 5; row < npair * G; row += PK_CONSUMERS / 32) {
    const int k = row / G, hq = row - k * G;
    float* pr = ps_of(k) + hq * 32;
    const int lane = tid & 31;
    const float v = lane < np ? pr[lane] : -INFINITY;
    const float mx = warp_max(v);
    const float e = lane < np ? __expf(v - mx) : 0.f;
    const float den = warp_sum(e);
    if (lane < np) pr[lane] = rbf(e / den);
  }
  named_sync(1, PK_CONSUMERS);
  for (int i = tid; i < npair * G * 16; i += PK_CONSUMERS) {
    const int k = i / (G * 16);
    const int r = i - k * G * 16;
    const int hq = r >> 4, c = r & 15;
    const float* pr = ps_of(k) + hq * 32;
    const bf16* vs = vs_of(k);
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < np; ++j) {
      float vf[8];
      cvt8(*reinterpret_cast<const uint4*>(vs + (size_t)j * 128 + c * 8), vf);
      const float p = pr[j];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = fmaf(p, vf[u], o[u]);
    }
    uint4 ov;
    ov.x = pack2(o[0], o[1]);
    ov.y = pack2(o[2], o[3]);
    ov.z = pack2(o[4], o[5]);
    ov.w = pack2(o[6], o[7]);
    *reinterpret_cast<uint4*>(qg_of(k) + (size_t)hq * 128 + c * 8) = ov;
  }
  named_sync(1, PK_CONSUMERS);
}

// x_mid = bf16(xres + ob) then RMSNorm (S3 input), all M rows.  xres and ob arrive with cp.async (one round trip);
// the un-normalised x_mid rows are also kept in `keep` ([M][H] bf16) for the down projection's residual.
// keep_c0 / a.keep_cols > 0 (tcgen05 build): ob is staged at xs + 16 H * 2 (past the 16 staged rows, free in S3) and
// only x_mid columns [keep_c0, keep_c0 + keep_cols) -- this CTA's S4 output columns -- are kept, [M][keep_cols].
__device__ __noinline__ void dd_load_mid(unsigned char* xs, int x_pitch, const DDArgs& a, int M, const bf16* nw,
                                         float* nred, bf16* keep, int keep_c0) {
  const int tid = threadIdx.x;
  const int H = a.H, kv = H >> 3, kc = a.keep_cols;
  bf16* const ost = kc ? reinterpret_cast<bf16*>(xs + (size_t)16 * H * 2) : keep;   // ob staging, [M][H]
  // (row m, unit j) items: one unit column per thread when the threads cover whole rows (no divisions per item)
  const bool cols = kv <= PK_CONSUMERS && PK_CONSUMERS % kv == 0;
  const int dm = cols ? PK_CONSUMERS / kv : 0, jc = cols ? tid % kv : 0, mc = cols ? tid / kv : 0;
  const int nit = cols ? (M - mc + dm - 1) / dm : (M * kv - tid + PK_CONSUMERS - 1) / PK_CONSUMERS;
#pragma unroll 4
  for (int k = 0; k < nit; ++k) {
    int m, j;
    if (cols) {
      m = mc + k * dm;
      j = jc;
    } else {
      const int i = tid + k * PK_CONSUMERS;
      m = i / kv;
      j = i - m * kv;
    }
    cp_async16(xs + xs_off(m, j, x_pitch), a.xres + (size_t)m * H + (size_t)j * 8);
    cp_async16(ost + (size_t)m * H + (size_t)j * 8, a.ob + (size_t)m * H + (size_t)j * 8);
  }
  cp_async_commit();
  cp_async_wait<0>();
#pragma unroll 4
  for (int k = 0; k < nit; ++k) {
    int m, j;
    if (cols) {
      m = mc + k * dm;
      j = jc;
    } else {
      const int i = tid + k * PK_CONSUMERS;
      m = i / kv;
      j = i - m * kv;
    }
    uint4* px = reinterpret_cast<uint4*>(xs + xs_off(m, j, x_pitch));
    uint4* pk = reinterpret_cast<uint4*>(ost + (size_t)m * H + (size_t)j * 8);
    float x[8], o[8];
    cvt8(*px, x);
    cvt8(*pk, o);
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = rbf(x[u] + o[u]);
    uint4 w;
    w.x = pack2(v[0], v[1]);
    w.y = pack2(v[2], v[3]);
    w.z = pack2(v[4], v[5]);
    w.w = pack2(v[6], v[7]);
    *px = w;
    if (!kc) {
      *pk = w;
    } else {
      const int col = j * 8 - keep_c0;
      if (col >= 0 && col < kc) *reinterpret_cast<uint4*>(keep + (size_t)m * kc + col) = w;
    }
  }
  named_sync(1, PK_CONSUMERS);
  row_rms(xs, x_pitch, M, H, a.eps, nred);
  apply_rms(xs, x_pitch, M, H, nw, nred);
  named_sync(1, PK_CONSUMERS);
}

// ------------------------------------------------------------------------------------------------ frame kernel
// The kernel body only sequences the phases below; every phase is a separate (non-inlined) function with its own
// register budget: 9 warps per CTA cap a thread at 168 registers, and spilled values would reload from L2 (the L1
// left beside 220 KB of shared memory is small).  Per-CTA state the phases share lives in file-scope shared memory.
__shared__ float g_dd_nred[ST_CWARPS * 16];
__shared__ int g_dd_int[32];
__shared__ int g_dd_call;                          // trace builds: GEMV tasks this CTA has run (detail timeline)
__shared__ int g_dd_l2keep;                        // the producer's L2 policy for weight copies (DDArgs::l2_keep)
__shared__ long long g_dd_tok[DD_MAXB];            // tokens fed to the next step (this CTA's copy)
__shared__ __align__(16) bf16 g_dd_cs[2][128];     // [cos|sin][dim] of the sub-step's position
__shared__ uint32_t g_dd_tmem;                     // tcgen05 build: TMEM base of the accumulators
__shared__ __align__(8) uint64_t g_dd_mbar;        // tcgen05 build: "the MMAs issued so far are complete"
// LN12 streaming: per ring slot, the decoded stage is ready (one arrival per decoder warp), and what the producer
// tells the decoders about the slot's copy (published by its arrive on the slot's full barrier)
struct LNSlot {
  unsigned lo, hi;
  const unsigned* ovf;
  long long novf;
  int g, q;
};
__shared__ __align__(8) uint64_t g_dd_dfull[FB_PK_MAX_STAGES];
__shared__ LNSlot g_dd_lnslot[FB_PK_MAX_STAGES];
constexpr int LN_ROWS = 64;                        // rows per LN12 stage (the MMA's M)
constexpr int LN_META_OFF = 7168;                  // the rows' 16-byte records, inside the slot
constexpr int LN_DATA_OFF = 8192;                  // the rows' data: [64 rows][3 slots][128 B]
constexpr int LN_DATA_BYTES = LN_ROWS * 384;
constexpr int LN_DEC_WARPS = 7;                    // consumer warps 1-7 decode while warp 0 issues the MMAs
constexpr int LN_DEC_BAR = 7;                      // their named barrier

struct DDSm {
  unsigned char* xs;
  unsigned char* zero16;
  float* red;
  float* sums;
  Ring rg;
};
// NT = 1 or 2: mma.sync build with NT activation tiles of 8 rows; NT = 0: the tcgen05 build (activations staged in
// the B-operand layout, 1024-aligned; the reduction area becomes the accumulator dump).
template <int NT>
__device__ __forceinline__ DDSm dd_smem(const DDArgs& a) {
  extern __shared__ __align__(128) unsigned char smem[];
  DDSm m;
  m.xs = (NT > 0) ? smem
            : reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
  m.zero16 = m.xs + a.xs_bytes;
  unsigned char* ringb = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(m.zero16 + 128) + (ST_ALIGN - 1)) & ~uintptr_t(ST_ALIGN - 1));
  m.red = reinterpret_cast<float*>(ringb + (size_t)a.nstages * ST_BYTES);
  m.sums = m.red + ((NT > 0) ? ST_CWARPS * 128 * NT : DD_TC_SUMS);
  uint64_t* full = reinterpret_cast<uint64_t*>(m.sums + 128 * (NT > 0 ? NT : 0));
  m.rg = Ring{ringb, full, full + PK_MAX_STAGES, a.nstages, &g_dd_int[28]};
  return m;
}

// Consumer cursor: ring stage counter, grid-barrier epoch, ok (0 once a bounded wait gave up), tcgen05 build: phase
// of g_dd_mbar.
struct DDCur {
  int t;
  unsigned epoch;
  int ok;
  unsigned tph;
};

// ------------------------------------------------------------------------------------------------ tcgen05 build
// A GEMV task on the tensor cores: blocks of weight rows (the MMA's M) against the 16 staged activation rows
// (N = 16), fp32 sums in TMEM.  KIND 0: 64 consecutive output units per block (M = 64, stages of 64 rows x 256
// columns); KIND 1: 128 units of gate rows and the same units of up rows (two M = 128 accumulators, stages of
// 2 x 128 rows x 64 columns); KIND 2: one q / k / v head per block (M = 128, stages of 128 rows x 128 columns: 64
// rotary pair units, rows d and d + 64 of the head).  64-row blocks spread the 1024-row matrices of the depth
// model over 16 CTAs instead of 8; the 4096-row gate|up task keeps 128-unit blocks (fewer per-block epilogues).  A stage is 32 KB of weights in the canonical K-major 128-byte-swizzle layout, streamed by
// the producer warp with one (KIND 1: two) TMA tensor copies; CTA c owns blocks [nb c / G, nb (c + 1) / G).
//
// LN12 streaming (DDArgs::ln12): every stage is 64 rows of one matrix x one lane octet q of one 1024-column group g,
// i.e. columns 1024 g + 256 c + 64 q + (0..63) of the four chunks c: the producer copies the 24 KB of LN12 data
// ([64 rows][3 slots][128 B], one tensor copy) and the rows' 1 KB of records into the slot's upper part, consumer
// warps 1-7 decode them into the slot as four 64-column strips [64 rows][128 B] (128-byte swizzle), and warp 0
// runs M = 64 MMAs over the strips.  Blocks are 64 units for every kind; KIND 1 alternates gate / up stages and
// KIND 2 the head's rows 0-63 / 64-127 per K slice, into two accumulators.
template <int KIND>
constexpr int tc_cols() { return KIND == 0 ? 256 : (KIND == 1 ? 64 : 128); }   // columns per stage
template <int KIND>
__device__ __forceinline__ int tc_units(bool ln) { return (KIND == 1 && !ln) ? 128 : 64; }   // units per block
template <int KIND>
__device__ __forceinline__ void tc_task_blocks(int units, int& b0, int& b1, bool ln) {
  const int UB = tc_units<KIND>(ln);
  const int nb = (units + UB - 1) / UB;
  b0 = (int)((long long)nb * blockIdx.x / gridDim.x);
  b1 = (int)((long long)nb * (blockIdx.x + 1) / gridDim.x);
}

// Producer half.  src(n0, mat) gives the tensor map and first row of the block starting at unit n0 (mat 1: the up
// rows of KIND 1).
// Weight copies carry an L2 evict_last hint: the lanes of the GPU stream the same depth weights at about the same
// time, and a codebook step's weights (123 MB with the step table) nearly fit the 126 MB L2, so keeping them ahead of
// the activations and KV traffic lets the later lanes read them from L2.
__device__ __forceinline__ void tma_load_3d_l2(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_l2(void* dst, const void* tmap, int c0, int c1, int c2, int c3,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Source of a block's rows: the tensor map, the first row, and (LN12 streaming) the matrix's records.
struct DDSrc {
  const void* map;
  int row;
  const LNMat* ln;
};

template <int KIND, bool ln, typename SrcFn>
__device__ __forceinline__ bool produce_task_tc(Ring& rg, int& t, int units, int K, SrcFn src, unsigned* err) {
  constexpr int C = tc_cols<KIND>();
  const int UB = tc_units<KIND>(ln);
  const int lane = threadIdx.x & 31;
  const uint64_t pol = g_dd_l2keep ? policy_evict_last() : policy_evict_normal();
  int b0, b1;
  tc_task_blocks<KIND>(units, b0, b1, ln);
  if constexpr (ln) {
    // per K slice (g, q): one stage per matrix of the block (KIND 1: gate, up; KIND 2: the head's two row halves)
    constexpr int NM = KIND == 0 ? 1 : 2;
    const int nks = K >> 8;
    for (int bi = b0; bi < b1; ++bi) {
      for (int kc = 0; kc < nks; ++kc) {
        for (int mm = 0; mm < NM; ++mm, ++t) {
          const int s = t % rg.nst;
          if (t >= rg.nst && !ring_wait_empty(rg, s, ((t / rg.nst) - 1) & 1, err)) return false;
          if (lane == 0) {
            const DDSrc w = src(bi * UB, KIND == 1 ? mm : 0);
            const int row = w.row + (KIND == 2 ? LN_ROWS * mm : 0);
            LNSlot& inf = g_dd_lnslot[s];
            inf.lo = w.ln->lo;
            inf.hi = w.ln->hi;
            inf.ovf = w.ln->ovf;
            inf.novf = w.ln->novf;
            inf.g = kc >> 2;
            inf.q = kc & 3;
            unsigned char* st = rg.base + (size_t)s * ST_BYTES;
            mbar_arrive_expect_tx(&rg.full[s], (unsigned)(LN_DATA_BYTES + LN_ROWS * 16));
            tma_load_4d_l2(st + LN_DATA_OFF, w.map, (kc & 3) * 128, 0, kc >> 2, row, &rg.full[s], pol);
            bulk_g2s(st + LN_META_OFF, w.ln->meta + row, LN_ROWS * 16, &rg.full[s]);
          }
          __syncwarp();
        }
      }
    }
    return true;
  }
  const int nkc = (K + C - 1) / C;
  int s = t % rg.nst;                                          // ring slot of stage t, advanced without divisions
  unsigned par = (unsigned)((t / rg.nst) + 1) & 1u;            // parity of the slot's previous use
  for (int bi = b0; bi < b1; ++bi) {
    const DDSrc w0 = src(bi * UB, 0);
    const DDSrc w1 = KIND == 1 ? src(bi * UB, 1) : DDSrc{nullptr, 0, nullptr};
    for (int kc = 0; kc < nkc; ++kc, ++t) {
      if (t >= rg.nst && !ring_wait_empty(rg, s, par, err)) return false;
      if (lane == 0) {
        unsigned char* st = rg.base + (size_t)s * ST_BYTES;
        mbar_arrive_expect_tx(&rg.full[s], (unsigned)ST_BYTES);
        if (KIND == 1) {
          tma_load_3d_l2(st, w0.map, 0, w0.row, kc, &rg.full[s], pol);             // [128 rows][128 B]
          tma_load_3d_l2(st + ST_BYTES / 2, w1.map, 0, w1.row, kc, &rg.full[s], pol);
        } else if (KIND == 0) {
          tma_load_3d_l2(st, w0.map, 0, w0.row, kc * 4, &rg.full[s], pol);         // [4][64 rows][128 B]
        } else {
          tma_load_3d_l2(st, w0.map, 0, w0.row, kc * 2, &rg.full[s], pol);         // [2][128 rows][128 B]
        }
      }
      __syncwarp();
      if (++s == rg.nst) {
        s = 0;
        par ^= 1u;
      }
    }
  }
  return true;
}

// LN12 decode of stages t0 .. t0 + nk - 1 by consumer warps 1-7 (224 threads): wait for the slot's copy, read its
// 64 rows x 8 lanes items (16 bytes of each of the three slots, the row record) into registers, meet (the decoded
// strips overwrite the copied bytes), rebuild each bf16 -- high byte = the row's shifted table entry of the 3-bit
// index (a byte permute over the two table words) with the sign, low byte as stored; then the row's patches that fall
// in the item's 32 columns -- and store 16 bytes per chunk into the strips; then publish to the async proxy and
// arrive on the slot's decoded barrier.  A failed wait still decodes (shared memory only; overflow patch reads are
// bounded by the matrix's count) and arrives, so nobody waits in vain, and raises the abort flag.
__device__ __noinline__ void ln12_decode_stages(const Ring& rg, int t0, int nk, unsigned* err, int* abort_flag) {
  const int dt = threadIdx.x - 32;
  const int lane = threadIdx.x & 31;
  for (int i = 0; i < nk; ++i) {
    const int t = t0 + i, s = t % rg.nst;
    if (!mbar_wait(&rg.full[s], (t / rg.nst) & 1, err)) *abort_flag = 1;
    unsigned char* st = rg.base + (size_t)s * ST_BYTES;
    const LNSlot inf = g_dd_lnslot[s];
    uint4 r0[3], r1[3], rw[3], mt[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int it = dt + 32 * LN_DEC_WARPS * k;
      if (it < LN_ROWS * 8) {
        const int r = it >> 3, l = it & 7;
        const unsigned char* rp = st + LN_DATA_OFF + r * 384 + l * 16;
        r0[k] = *reinterpret_cast<const uint4*>(rp);
        r1[k] = *reinterpret_cast<const uint4*>(rp + 128);
        rw[k] = *reinterpret_cast<const uint4*>(rp + 256);
        mt[k] = *reinterpret_cast<const uint4*>(st + LN_META_OFF + r * 16);
      }
    }
    named_sync(LN_DEC_BAR, 32 * LN_DEC_WARPS);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int it = dt + 32 * LN_DEC_WARPS * k;
      if (it < LN_ROWS * 8) {
        const int r = it >> 3, l = it & 7;
        const unsigned hdr = mt[k].x;
        const unsigned sb = (((hdr >> 10) & 7u) ^ 4u) - 4u;        // the row's table shift, -4 .. 3
        const unsigned add = (sb & 0xFFu) * 0x01010101u;
        const unsigned lo = __vadd4(inf.lo, add), hi = __vadd4(inf.hi, add);
        const unsigned w[4] = {rw[k].x, rw[k].y, rw[k].z, rw[k].w};
        unsigned H[4][2];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          H[c][0] = __byte_perm(lo, hi, w[c] & 0x7777u) | (w[c] & 0x80808080u);
          H[c][1] = __byte_perm(lo, hi, (w[c] >> 16) & 0x7777u) | ((w[c] << 4) & 0x80808080u);
        }
        const unsigned a0[4] = {r0[k].x, r0[k].z, r1[k].x, r1[k].z};   // low bytes of elements 0-3 per chunk
        const unsigned a1[4] = {r0[k].y, r0[k].w, r1[k].y, r1[k].w};   // elements 4-7
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 o;
          o.x = __byte_perm(a0[c], H[c][0], 0x5140);
          o.y = __byte_perm(a0[c], H[c][0], 0x7362);
          o.z = __byte_perm(a1[c], H[c][1], 0x5140);
          o.w = __byte_perm(a1[c], H[c][1], 0x7362);
          *reinterpret_cast<uint4*>(st + c * 8192 + r * 128 + ((l ^ (r & 7)) << 4)) = o;
        }
        // the row's patches in this item's columns: the exact high byte, over what this thread just stored
        const unsigned cnt = hdr & 1023u;
        if (cnt) {
          const long long ooff = (long long)(hdr >> 13);
          const unsigned lane_g = (unsigned)(inf.q * 8 + l);
          for (unsigned pi = 0; pi < cnt; ++pi) {
            unsigned v;
            if (pi < 3) {
              v = pi == 0 ? mt[k].y : (pi == 1 ? mt[k].z : mt[k].w);
            } else {
              const long long o = ooff + (long long)pi - 3;
              if (o >= inf.novf) break;
              v = __ldg(inf.ovf + o);
            }
            const unsigned col = v >> 8;
            if ((int)(col >> 10) == inf.g && ((col >> 3) & 31u) == lane_g)
              st[((col >> 8) & 3u) * 8192 + r * 128 + ((l ^ (r & 7)) << 4) + 2 * (col & 7u) + 1] = (unsigned char)v;
          }
        }
      }
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(&g_dd_dfull[s]);
  }
}

// Consumer half (all 256 consumer threads).  The activations of the first K pass are staged at xs (B-operand
// layout) by the caller; stage_x(p) restages pass p (K > DD_TC_KX, or a further block).  Consumer warp 0 waits for
// the stages and its lane 0 issues the MMAs (four independent accumulator chains per matrix, summed in a fixed
// order) and commits them to the ring's empty barriers and to g_dd_mbar.  Warps 0-3 then copy the accumulators out
// of TMEM into `dump` as groups of 16 rows x 16 activation rows in the order the mma.sync epilogues read them
// (KIND 0: 16 units; KIND 1 and 2: rows 0-7 the 8 units' matrix-0 rows, 8-15 their matrix-1 rows), and the
// threads run epi(n0, nu, group, local thread) per group, as many groups at once as the threads allow.  A failed
// wait in warp 0 still commits (so nobody else waits in vain) and is reported to every thread through shared
// memory after the next barrier.
template <int KIND, bool ln, typename EpiFn, typename StageFn>
__device__ __forceinline__ bool consume_task_tc(Ring& rg, DDCur& c, int units, int K, const unsigned char* xs,
                                                float* dump, EpiFn epi, StageFn stage_x, unsigned* err,
                                                unsigned long long* det, int bM) {
  constexpr int C = tc_cols<KIND>();
  constexpr int GU = KIND == 0 ? 16 : 8;                       // units per group
  constexpr int NM = KIND == 0 ? 1 : 2;                        // LN12: stages per K slice
  const int UB = tc_units<KIND>(ln);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b0, b1;
  tc_task_blocks<KIND>(units, b0, b1, ln);
  const int KX = K < DD_TC_KX ? K : DD_TC_KX;
  const int npass = (K + KX - 1) / KX;
  const int ncp = KX / C;                                      // stages per pass
  const uint32_t tmem = g_dd_tmem, xsa = smem_u32(xs);
  int* abort_flag = &g_dd_int[29];
  if (threadIdx.x == 0) *abort_flag = 0;
  fence_proxy_async();                 // the caller's staging writes -> visible to the tensor core
  named_sync(1, PK_CONSUMERS);
  if (det && threadIdx.x == 0) {
    det[0] = globaltimer();
    det[7] = (unsigned long long)(b1 - b0);
  }
  for (int bi = b0; bi < b1; ++bi) {
    for (int p = 0; p < npass; ++p) {
      if (p > 0 || (bi > b0 && npass > 1)) {
        stage_x(p);
        fence_proxy_async();
        named_sync(1, PK_CONSUMERS);
      }
      const int nk = ln ? (min(KX, K - p * KX) >> 8) * NM : min(ncp, (K - p * KX + C - 1) / C);
      if (warp == 0) {
        tc_after();
        if (lane == 0) {
          // Lane 0 alone waits and issues; the ring position advances without divisions
          int s = c.t % rg.nst;
          unsigned par = (unsigned)(c.t / rg.nst) & 1u;
          const uint32_t ring0 = smem_u32(rg.base);
          for (int kcp = 0; kcp < nk; ++kcp) {
            const bool ok = mbar_wait(ln ? &g_dd_dfull[s] : &rg.full[s], par, err);
            if (det && bi == b0 && p == 0 && kcp == 0) det[1] = globaltimer();
            if (!ok) *abort_flag = 1;
            const uint32_t wa = ring0 + (uint32_t)s * ST_BYTES;
            if (ok && ln) {
              // LN12 stage: K slice ks of the pass (1024 (ks / 4) + 256 c + 64 (ks % 4) + 0..63 for strips c = 0..3),
              // matrix mm; M = 64 MMAs, chain jj = the 16-column step within the strip
              const int ks = kcp / NM, mm = kcp - ks * NM;
              const uint32_t dcol = tmem + (uint32_t)(mm * 64);
              const uint32_t xs0 = xsa + (uint32_t)((((ks >> 2) << 4) + (ks & 3)) << 11);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int cs = j >> 2, jj = j & 3;
                const uint32_t acc = (p > 0 || ks > 0 || cs > 0) ? 1u : 0u;
                tc_mma16_m64(dcol + (uint32_t)(jj * 16), tc_desc_sw128(wa + (uint32_t)(cs * 8192 + jj * 32)),
                             tc_desc_sw128(xs0 + (uint32_t)(cs * 8192 + jj * 32)), acc);
              }
            } else if (ok) {
              // activations: 64-column blocks of 16 rows x 128 B (2 KB) from block kcp C / 64 of the pass
              const uint32_t xs0 = xsa + (uint32_t)(kcp * (C / 64)) * 2048u;
#pragma unroll
              for (int j = 0; j < C / 16; ++j) {
                const uint64_t bd =
                    tc_desc_sw128(xs0 + (uint32_t)(((16 * j) >> 6) * 2048 + (((16 * j) & 63) >> 4) * 32));
                if (KIND == 1) {
                  // gate: [128 rows][128 B] at 0, up at 16 KB; two chains each
                  const uint32_t acc = (p > 0 || kcp > 0 || j >= 2) ? 1u : 0u;
                  const uint32_t ch = (uint32_t)((j & 1) * 16);
                  tc_mma16(tmem + ch, tc_desc_sw128(wa + (uint32_t)((j & 3) * 32)), bd, acc);
                  tc_mma16(tmem + 32 + ch, tc_desc_sw128(wa + (uint32_t)(ST_BYTES / 2 + (j & 3) * 32)), bd, acc);
                } else if (KIND == 0) {
                  const uint32_t acc = (p > 0 || kcp > 0 || j >= 4) ? 1u : 0u;
                  const uint64_t ad = tc_desc_sw128(wa + (uint32_t)((j >> 2) * 8192 + (j & 3) * 32));
                  tc_mma16_m64(tmem + (uint32_t)((j & 3) * 16), ad, bd, acc);
                } else {
                  const uint32_t acc = (p > 0 || kcp > 0 || j >= 4) ? 1u : 0u;
                  const uint64_t ad = tc_desc_sw128(wa + (uint32_t)((j >> 2) * 16384 + (j & 3) * 32));
                  tc_mma16(tmem + (uint32_t)((j & 3) * 16), ad, bd, acc);
                }
              }
            }
            tc_commit(&rg.empty[s]);
            if (++s == rg.nst) {
              s = 0;
              par ^= 1u;
            }
          }
          if (det && bi == b0) det[2] = globaltimer();
          tc_commit(&g_dd_mbar);
        }
        __syncwarp();
      } else if constexpr (ln) {
        ln12_decode_stages(rg, c.t, nk, err, abort_flag);
      }
      c.t += nk;
      // the pass's MMAs are complete: the staged activations may be replaced, the accumulators read
      if (!mbar_wait(&g_dd_mbar, c.tph & 1, err)) *abort_flag = 1;
      ++c.tph;
      tc_after();
      if (det && threadIdx.x == 0 && bi == b0) det[3] = globaltimer();
    }
    // accumulators -> dump (warps 0-3, TMEM lane quarter = warp) -> epilogues.  KIND 0 (M = 64): block row r sits
    // in lane (r % 16) of quarter r / 16, so warp q's lanes 0-15 hold rows 16 q ..; KIND 1 and 2 (M = 128): row =
    // lane of the 128.  KIND 1 goes in two rounds of 64 units (8 groups each) through the 8-group dump.
    float kg1[16], ku1[16];                                    // KIND 1, warps 2-3: their units for round 2
    if constexpr (ln && KIND != 0) {
      // LN12, two M = 64 accumulators (matrix 0 at column 0, matrix 1 at 64): unit d = 16 warp + lane (lanes 0-15)
      if (warp < 4) {
        const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
        const int d = warp * 16 + (lane & 15);
        float* g = dump + (d >> 3) * 256 + (d & 7) * 16;
        for (int mm = 0; mm < 2; ++mm) {
          float c0[16], c1[16], v[16];
          tc_ld16(tq + mm * 64, c0);
          tc_ld16(tq + mm * 64 + 16, c1);
#pragma unroll
          for (int m = 0; m < 16; ++m) v[m] = c0[m] + c1[m];
          tc_ld16(tq + mm * 64 + 32, c0);
          tc_ld16(tq + mm * 64 + 48, c1);
          if (lane < 16) {
#pragma unroll
            for (int m = 0; m < 16; ++m) g[mm * 128 + m] = (v[m] + c0[m]) + c1[m];
          }
        }
      }
    } else if (warp < 4) {
      const int L = warp * 32 + lane;
      const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
      float c0[16], c1[16], v[16];
      tc_ld16(tq, c0);
      tc_ld16(tq + 16, c1);
#pragma unroll
      for (int m = 0; m < 16; ++m) v[m] = c0[m] + c1[m];
      tc_ld16(tq + 32, c0);
      tc_ld16(tq + 48, c1);
      if (KIND == 2) {
        float* d = dump + ((L & 63) >> 3) * 256 + ((L >> 6) * 8 + (L & 7)) * 16;
#pragma unroll
        for (int m = 0; m < 16; ++m) d[m] = (v[m] + c0[m]) + c1[m];
      } else if (KIND == 0 && lane < 16) {
        const int r = warp * 16 + lane;                          // block row (unit)
        float* d = dump + (r >> 4) * 256 + (r & 15) * 16;
#pragma unroll
        for (int m = 0; m < 16; ++m) d[m] = (v[m] + c0[m]) + c1[m];
      }
      if (KIND == 1) {
        // units 0..63 now (warps 0-1), units 64..127 after the first round's epilogues (warps 2-3)
#pragma unroll
        for (int m = 0; m < 16; ++m) c0[m] = c0[m] + c1[m];     // up
        if (warp < 2) {
          float* g = dump + (L >> 3) * 256 + (L & 7) * 16;
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            g[m] = v[m];
            g[128 + m] = c0[m];
          }
        }
#pragma unroll
        for (int m = 0; m < 16; ++m) c1[m] = v[m];                // keep gate for round 2
        if (warp >= 2) {
#pragma unroll
          for (int m = 0; m < 16; ++m) kg1[m] = c1[m], ku1[m] = c0[m];
        }
      }
    }
    tc_before();
    named_sync(1, PK_CONSUMERS);
    if (det && threadIdx.x == 0 && bi == b0) det[4] = globaltimer();
    if (*abort_flag) return false;
    // groups side by side: a group's epilogue uses GU x M threads, so 256 / (GU M) groups run at once (thread t
    // takes group slot t / (GU M) as local thread t % (GU M))
    const int gw = GU * bM;
    const int gq = gw >= PK_CONSUMERS ? 1 : PK_CONSUMERS / gw;
    const int gs = (int)threadIdx.x / gw, lt = (int)threadIdx.x - gs * gw;
    if (KIND == 1 && !ln) {
      for (int g = gs; g < 8 && gs < gq; g += gq) {
        const int n0 = bi * UB + g * GU;
        const int nu = min(GU, units - n0);
        if (nu > 0) epi(n0, nu, dump + g * 256, lt);
      }
      named_sync(1, PK_CONSUMERS);
      if (warp >= 2 && warp < 4) {
        const int Lr = (warp - 2) * 32 + lane;
        float* g = dump + (Lr >> 3) * 256 + (Lr & 7) * 16;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          g[m] = kg1[m];
          g[128 + m] = ku1[m];
        }
      }
      named_sync(1, PK_CONSUMERS);
      for (int g = gs; g < 8 && gs < gq; g += gq) {
        const int n0 = bi * UB + 64 + g * GU;
        const int nu = min(GU, units - n0);
        if (nu > 0) epi(n0, nu, dump + g * 256, lt);
      }
    } else
    {
      // KIND 0: 4 groups of 16 units; KIND 1 and 2: 8 groups of 8 units
      constexpr int NGR = KIND == 0 ? 4 : 8;
      for (int g = gs; g < NGR && gs < gq; g += gq) {
        const int n0 = bi * UB + g * GU;
        const int nu = min(GU, units - n0);
        if (nu > 0) epi(n0, nu, dump + g * 256, lt);
      }
    }
    if (det && threadIdx.x == 0 && bi == b0) det[5] = globaltimer();
    named_sync(1, PK_CONSUMERS);       // the dump and the accumulators are reused by the next block
  }
  if (det && threadIdx.x == 0) det[6] = globaltimer();
  return true;
}

// ------------------------------------------------------------------------------------------------ 128-row tasks
// A plain GEMV task (o, down, projector, heads) in blocks of 128 output units split over S parts of K: item i =
// (block i / S, part i % S), CTA c owns items [items c / G, items (c + 1) / G).  A stage is 128 rows x 128 columns
// ([2][128 rows][128 B], the q|k|v stage layout), consumed by 8 M = 128 MMAs -- twice the bytes per MMA of the
// 64-row task, whose M = 64 MMAs cost the same issue time.  Parts 0 .. S - 2 publish their fp32 sums (release tag
// in a.flags); the CTA holding part S - 1 waits for them (bounded), adds them in part order before its own, and
// runs the epilogue.  Items are assigned in order, so a waiter only waits for items of earlier CTAs or its own.
__device__ __forceinline__ void tc3_items(int units, int S, int& i0, int& i1) {
  const int items = (units >> 7) * S;
  i0 = (int)((long long)items * blockIdx.x / gridDim.x);
  i1 = (int)((long long)items * (blockIdx.x + 1) / gridDim.x);
}

template <typename SrcFn>
__device__ __forceinline__ bool produce_task_tc3(Ring& rg, int& t, int units, int K, int S, SrcFn src,
                                                 unsigned* err) {
  const int lane = threadIdx.x & 31;
  const uint64_t pol = g_dd_l2keep ? policy_evict_last() : policy_evict_normal();
  const int nks = (K / S) >> 7;
  int i0, i1;
  tc3_items(units, S, i0, i1);
  int s = t % rg.nst;
  unsigned par = (unsigned)((t / rg.nst) + 1) & 1u;
  for (int it = i0; it < i1; ++it) {
    const int blk = it / S, part = it - blk * S;
    const DDSrc w = src(blk * 128, 0);
    for (int kc = 0; kc < nks; ++kc, ++t) {
      if (t >= rg.nst && !ring_wait_empty(rg, s, par, err)) return false;
      if (lane == 0) {
        unsigned char* st = rg.base + (size_t)s * ST_BYTES;
        mbar_arrive_expect_tx(&rg.full[s], (unsigned)ST_BYTES);
        tma_load_3d_l2(st, w.map, 0, w.row, (part * nks + kc) * 2, &rg.full[s], pol);   // [2][128 rows][128 B]
      }
      __syncwarp();
      if (++s == rg.nst) {
        s = 0;
        par ^= 1u;
      }
    }
  }
  return true;
}

template <typename EpiFn, typename StageFn>
__device__ __forceinline__ bool consume_task_tc3(const DDArgs& a, Ring& rg, DDCur& c, int units, int K, int S,
                                                 const unsigned char* xs, float* dump, EpiFn epi, StageFn stage_x,
                                                 unsigned long long* det) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Kp = K / S, nks = Kp >> 7;
  const int KX = K < DD_TC_KX ? K : DD_TC_KX;
  int i0, i1;
  tc3_items(units, S, i0, i1);
  const uint32_t tmem = g_dd_tmem, xsa = smem_u32(xs);
  unsigned* const err = a.err;
  int* abort_flag = &g_dd_int[29];
  if (tid == 0) *abort_flag = 0;
  fence_proxy_async();                 // the caller's staging (pass 0) -> visible to the tensor core
  named_sync(1, PK_CONSUMERS);
  if (det && tid == 0) {
    det[0] = globaltimer();
    det[7] = (unsigned long long)(i1 - i0);
  }
  const unsigned tag = c.epoch + 1u;   // unique per phase within the frame (flags are zeroed at frame start)
  int staged = 0;
  for (int it = i0; it < i1; ++it) {
    const int blk = it / S, part = it - blk * S;
    const int k0 = part * Kp, pass = k0 / KX, kin = k0 - pass * KX;
    if (pass != staged) {
      stage_x(pass);
      fence_proxy_async();
      named_sync(1, PK_CONSUMERS);
      staged = pass;
    }
    if (warp == 0) {
      tc_after();
      if (lane == 0) {
        int s = c.t % rg.nst;
        unsigned par = (unsigned)(c.t / rg.nst) & 1u;
        const uint32_t ring0 = smem_u32(rg.base);
        for (int kcp = 0; kcp < nks; ++kcp) {
          const bool ok = mbar_wait(&rg.full[s], par, err);
          if (det && it == i0 && kcp == 0) det[1] = globaltimer();
          if (!ok) *abort_flag = 1;
          if (ok) {
            const uint32_t wa = ring0 + (uint32_t)s * ST_BYTES;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int col = kin + kcp * 128 + 16 * j;            // column within the staged pass
              const uint64_t bd =
                  tc_desc_sw128(xsa + (uint32_t)((col >> 6) << 11) + (uint32_t)(((col & 63) >> 4) << 5));
              const uint64_t ad = tc_desc_sw128(wa + (uint32_t)((j >> 2) * 16384 + (j & 3) * 32));
              tc_mma16(tmem + (uint32_t)((j & 3) * 16), ad, bd, (kcp > 0 || j >= 4) ? 1u : 0u);
            }
          }
          tc_commit(&rg.empty[s]);
          if (++s == rg.nst) {
            s = 0;
            par ^= 1u;
          }
        }
        if (det && it == i0) det[2] = globaltimer();
        tc_commit(&g_dd_mbar);
      }
      __syncwarp();
    }
    c.t += nks;
    if (!mbar_wait(&g_dd_mbar, c.tph & 1, err)) *abort_flag = 1;
    ++c.tph;
    tc_after();
    if (det && tid == 0 && it == i0) det[3] = globaltimer();
    if (warp < 4) {
      // unit L = TMEM lane; its 16 activation rows are the columns of the four chains
      const int L = warp * 32 + lane;
      const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
      float c0[16], c1[16], v[16];
      tc_ld16(tq, c0);
      tc_ld16(tq + 16, c1);
#pragma unroll
      for (int m = 0; m < 16; ++m) v[m] = c0[m] + c1[m];
      tc_ld16(tq + 32, c0);
      tc_ld16(tq + 48, c1);
      float* d = dump + (L >> 4) * 256 + (L & 15) * 16;
#pragma unroll
      for (int m = 0; m < 16; ++m) d[m] = (v[m] + c0[m]) + c1[m];
    }
    tc_before();
    named_sync(1, PK_CONSUMERS);
    if (det && tid == 0 && it == i0) det[4] = globaltimer();
    if (*abort_flag) return false;
    float* const pb = a.part + (size_t)blk * (S - 1) * 2048;
    if (part < S - 1) {
      for (int i = tid; i < 2048; i += PK_CONSUMERS) __stcg(pb + (size_t)part * 2048 + i, dump[i]);
      __threadfence();
      named_sync(1, PK_CONSUMERS);
      if (tid == 0) st_release_u32(&a.flags[blk * (S - 1) + part], tag);
    } else {
      if (S > 1) {
        if (tid == 0) {
          int ok = 1;
          const uint64_t t0 = globaltimer();
          for (int q = 0; q < S - 1 && ok; ++q) {
            int spins = 0;
            while (ld_acquire_u32(&a.flags[blk * (S - 1) + q]) != tag) {
              if (++spins == 256) {
                spins = 0;
                if (ld_acquire_u32(&a.bar->abort)) {
                  set_error(err, FB_ERR_ABORTED);
                  ok = 0;
                  break;
                }
                if (globaltimer() - t0 > a.wait_ns) {
                  set_error(err, FB_ERR_TIMEOUT);
                  atomicExch(&a.bar->abort, 1u);
                  ok = 0;
                  break;
                }
              }
            }
          }
          *abort_flag = ok ? 0 : 1;
        }
        named_sync(1, PK_CONSUMERS);
        if (*abort_flag) return false;
        for (int i = tid; i < 2048; i += PK_CONSUMERS) {
          float v = __ldcg(pb + i);
          for (int q = 1; q < S - 1; ++q) v += __ldcg(pb + (size_t)q * 2048 + i);
          dump[i] = v + dump[i];
        }
        named_sync(1, PK_CONSUMERS);
      }
      // 8 groups of 16 units, as many side by side as the threads allow (a group uses 16 M threads)
      const int gw = 16 * a.B;
      const int gq = gw >= PK_CONSUMERS ? 1 : PK_CONSUMERS / gw;
      const int gs = tid / gw, lt = tid - gs * gw;
      for (int g = gs; g < 8 && gs < gq; g += gq) {
        const int n0 = blk * 128 + g * 16;
        const int nu = min(16, units - n0);
        if (nu > 0) epi(n0, nu, dump + g * 256, lt);
      }
    }
    if (det && tid == 0 && it == i0) det[5] = globaltimer();
    named_sync(1, PK_CONSUMERS);       // the dump and the accumulators are reused by the next item
  }
  if (det && tid == 0) det[6] = globaltimer();
  return true;
}

// One GEMV task of a phase: the mma.sync stream (NT > 0; KIND 1 / 2 -> two matrices per unit) or the tcgen05 path
// (NT = 0).  x_pitch: the staged activations' row pitch (mma.sync builds).  xg / ldx: activations too large to stage
// whole (mma.sync, column chunks).  stage_x: restaging of further K passes (tcgen05 build).
template <int NT, int KIND, typename EpiFn, typename StageFn>
__device__ __forceinline__ bool dd_gemv(const DDArgs& a, DDSm& m, DDCur& c, int units, int K, int x_pitch, EpiFn epi,
                                        StageFn stage_x, const bf16* xg = nullptr, long ldx = 0, int s3 = 0) {
  if constexpr (NT <= 0) {
    // trace builds: the first DD_DETAIL_CALLS tasks of each CTA record a detail timeline after the phase trace
    unsigned long long* det = nullptr;
    const int call = g_dd_call;
    if (a.trace && call < DD_DETAIL_CALLS)
      det = a.trace + (size_t)gridDim.x * a.NCB * DD_TRACE_SLOTS(a.L) + ((size_t)blockIdx.x * DD_DETAIL_CALLS + call) * 8;
    bool ok;
    if (NT == 0 && KIND == 0 && s3 > 0)
      ok = consume_task_tc3(a, m.rg, c, units, K, s3, m.xs, m.red, epi, stage_x, det);
    else
      ok = consume_task_tc<KIND, (NT < 0)>(m.rg, c, units, K, m.xs, m.red, epi, stage_x, a.err, det, a.B);
    if (threadIdx.x == 0) g_dd_call = call + 1;
    return ok;
  } else {
    return consume_task<KIND == 0 ? 1 : 2, NT>(m.rg, c.t, units, K, m.xs, x_pitch, a.B, m.zero16, m.red, m.sums, epi,
                                                a.err, xg, ldx);
  }
}

// Producer warp: every weight slice of the frame, in the consumers' order, through the ring (two 8-row TMA tensor
// copies per stage; the maps travel in the argument block).
template <int NT>
__device__ __noinline__ void dd_producer(const DDArgs& a) {
  DDSm m = dd_smem<NT>(a);
  const int H = a.H, AE = a.AE, NH = a.NH, NKV = a.NKV, F = a.F, V = a.V;
  const int QKVU = (NH + 2 * NKV) * 64;  // rotary pair units
  const int L = a.L, NCB = a.NCB;
  unsigned* const err = a.err;
  {
    // every tensor map of the frame into the descriptor cache first (a miss would stall the first copy of a phase)
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 2 + DD_NMAPS * L; i += 32)
      tma_prefetch_map(i == 0 ? &a.tm_proj : (i == 1 ? &a.tm_head : &a.tm[(i - 2) / DD_NMAPS][(i - 2) % DD_NMAPS]));
    if (a.ln12)
      for (int i = lane; i < NCB; i += 32) tma_prefetch_map(&a.tm_hd[i]);
  }
  constexpr bool ln = NT < 0;
  int t = 0;
  bool ok = true;
  for (int s = 0; s < NCB && ok; ++s) {
    const bool tab = a.ptab && s >= 1;     // stage E and layer 0's q|k|v come from the step table
    for (int sub = 0; sub < (s == 0 ? 2 : 1) && ok; ++sub) {
      if constexpr (NT <= 0) {
        auto src = [&](int n, int) { return DDSrc{&a.tm_proj, n, &a.ln_proj}; };
        if (!tab)
          ok = ok && (a.s3_proj && !ln ? produce_task_tc3(m.rg, t, H, AE, a.s3_proj, src, err)
                                       : produce_task_tc<0, ln>(m.rg, t, H, AE, src, err));
      } else {
        if (!tab)
          ok = ok && produce_task_tma<1>(m.rg, t, H, AE, [&](int n, int) { return TmaRows{&a.tm_proj, n}; }, err);
      }
      for (int l = 0; l < L && ok; ++l) {
        const CUtensorMap* W = a.tm[l];
        const bool skip_qkv = tab && l == 0;
        if constexpr (NT <= 0) {
          // one head per block: rows hh * 128 .. + 127 of wq / wk / wv
          const LNMat* LW = a.ln[l];
          if (!skip_qkv) ok = ok && produce_task_tc<2, ln>(m.rg, t, QKVU, H, [&](int u, int) {
            const int hh = u >> 6;
            if (hh < NH) return DDSrc{&W[DD_WQ], hh * 128, &LW[DD_WQ]};
            if (hh < NH + NKV) return DDSrc{&W[DD_WK], (hh - NH) * 128, &LW[DD_WK]};
            return DDSrc{&W[DD_WV], (hh - NH - NKV) * 128, &LW[DD_WV]};
          }, err);
          auto src_o = [&](int n, int) { return DDSrc{&W[DD_WO], n, &LW[DD_WO]}; };
          ok = ok && (a.s3_o && !ln ? produce_task_tc3(m.rg, t, H, NH * 128, a.s3_o, src_o, err)
                                    : produce_task_tc<0, ln>(m.rg, t, H, NH * 128, src_o, err));
          ok = ok && produce_task_tc<1, ln>(m.rg, t, F, H, [&](int n, int mat) {
            return DDSrc{&W[mat ? DD_WU : DD_WG], n, &LW[mat ? DD_WU : DD_WG]};
          }, err);
          auto src_d = [&](int n, int) { return DDSrc{&W[DD_WD], n, &LW[DD_WD]}; };
          ok = ok && (a.s3_down && !ln ? produce_task_tc3(m.rg, t, H, F, a.s3_down, src_d, err)
                                       : produce_task_tc<0, ln>(m.rg, t, H, F, src_d, err));
        } else {
          // unit u = (head hh, rotary pair d): matrix 0 carries row hh * 128 + d, matrix 1 row hh * 128 + 64 + d
          if (!skip_qkv) ok = ok && produce_task_tma<2>(m.rg, t, QKVU, H, [&](int u, int mat) {
            const int hh = u >> 6, d = (u & 63) + mat * 64;
            if (hh < NH) return TmaRows{&W[DD_WQ], hh * 128 + d};
            if (hh < NH + NKV) return TmaRows{&W[DD_WK], (hh - NH) * 128 + d};
            return TmaRows{&W[DD_WV], (hh - NH - NKV) * 128 + d};
          }, err);
          ok = ok && produce_task_tma<1>(m.rg, t, H, NH * 128, [&](int n, int) { return TmaRows{&W[DD_WO], n}; }, err);
          ok = ok && produce_task_tma<2>(m.rg, t, F, H,
                                         [&](int n, int mat) { return TmaRows{&W[mat ? DD_WU : DD_WG], n}; }, err);
          ok = ok && produce_task_tma<1>(m.rg, t, H, F, [&](int n, int) { return TmaRows{&W[DD_WD], n}; }, err);
        }
      }
    }
    if constexpr (NT <= 0) {
      auto src_h = [&](int n, int) {
        return ln ? DDSrc{&a.tm_hd[s], n, &a.ln_hd[s]} : DDSrc{&a.tm_head, s * V + n, nullptr};
      };
      ok = ok && (a.s3_head && !ln ? produce_task_tc3(m.rg, t, V, H, a.s3_head, src_h, err)
                                   : produce_task_tc<0, ln>(m.rg, t, V, H, src_h, err));
    } else {
      ok = ok && produce_task_tma<1>(m.rg, t, V, H, [&](int n, int) { return TmaRows{&a.tm_head, s * V + n}; }, err);
    }
  }
  // never leave with copies in flight into this CTA's shared memory
  for (int u = max(0, t - m.rg.nst); u < t; ++u)
    if (!mbar_wait_warp(&m.rg.full[u % m.rg.nst], (u / m.rg.nst) & 1, err)) break;
}

// First output column of this CTA's S4 (down) work in the tcgen05 build: its first 64-unit block, or with the
// 128-row split task the block of its first item (x_mid is kept from there for a.keep_cols columns).
template <int NT>
__device__ __forceinline__ int dd_s4_col0(const DDArgs& a) {
  if constexpr (NT > 0) {
    return 0;
  } else {
    if (NT == 0 && a.s3_down) {
      int i0, i1;
      tc3_items(a.H, a.s3_down, i0, i1);
      return (i0 / a.s3_down) * 128;
    }
    int b0, b1;
    tc_task_blocks<0>(a.H, b0, b1, false);
    return b0 * 64;
  }
}

// E: gather the token embeddings (cp.async, one round trip, with the position's rotary rows) -> projector -> xres
template <int NT>
__device__ __noinline__ DDCur dd_phase_e(const DDArgs& a, DDCur c, int s, int sub, int pos) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, AE = a.AE, H = a.H, V = a.V;
  const int xp_ae = (NT > 0) ? AE * 2 + 16 : 0;
  bf16* const xres = a.xres;   // locals: stores through them cannot alias the argument block
  DD_STAMP(s, 0);
  const int kv = AE >> 3;
  const long long rows = (long long)(a.NCB + 1) * V;
#pragma unroll 4
  for (int i = tid; i < M * kv; i += PK_CONSUMERS) {
    const int b = i / kv, j = i - b * kv;
    const bf16* src;
    if (s == 0 && sub == 0) {
      src = a.bh + (size_t)b * AE;
    } else {
      long long id = (s == 0) ? __ldcg(a.first_cb + b) : g_dd_tok[b] + (long long)s * V;
      id = id < 0 ? 0 : (id >= rows ? rows - 1 : id);
      src = a.embed + (size_t)id * AE;
    }
    cp_async16(m.xs + xs_off(b, j, xp_ae), src + (size_t)j * 8);
  }
  if (tid < 32) {    // cos / sin rows of the position, 16 chunks of 16 bytes each
    const int tab = tid >> 4, cc = tid & 15;
    cp_async16(&g_dd_cs[tab][cc * 8], (tab ? a.sin_tab : a.cos_tab) + (size_t)pos * 128 + cc * 8);
  }
  cp_async_commit();
  cp_async_wait<0>();
  named_sync(1, PK_CONSUMERS);
  if (!dd_gemv<NT, 0>(a, m, c, H, AE, xp_ae,
                      [&](int n0, int nu, const float* sm, int lt) {
                        if (lt < nu * M) {
                          const int i = lt / M, r = lt - i * M;
                          xres[(size_t)r * H + n0 + i] = __float2bfloat16_rn(sm[i * MS + r]);
                        }
                      }, [](int) {}, nullptr, 0, a.s3_proj)) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, 1);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, 2);
  return c;
}

// Codebook step >= 1 with the per-token step table (flashb_dd_tab_build): stage E and layer 0's q|k|v become table
// reads.  Every CTA copies its share of the batch rows' ptab rows into the residual stream and takes its share of
// the (row, head, rotary pair) units of their ttab rows: RoPE at `pos`, then q / the layer-0 KV cache written as the
// S1 epilogue writes them (same rounding points: the table holds the bf16 GEMV outputs).  One barrier follows, in
// place of the two of E and layer-0 S1.
__device__ __noinline__ DDCur dd_phase_tab(const DDArgs& a, DDCur c, int s, int pos) {
  const int tid = threadIdx.x, M = a.B, H = a.H, NH = a.NH, NKV = a.NKV, QD = NH * 128, V = a.V;
  const int QKV = (NH + 2 * NKV) * 128, P = a.P;
  bf16 *const xres = a.xres, *const qb = a.qb, *const kcache = a.kc, *const vcache = a.vc;
  DD_STAMP(s, 0);
  if (tid < 32) {    // cos / sin rows of the position for the later layers' S1 epilogues
    const int tab = tid >> 4, cc = tid & 15;
    cp_async16(&g_dd_cs[tab][cc * 8], (tab ? a.sin_tab : a.cos_tab) + (size_t)pos * 128 + cc * 8);
  }
  cp_async_commit();
  const long long trows = (long long)(a.NCB - 1) * V, erows = (long long)(a.NCB + 1) * V;
  auto trow = [&](int b) -> long long {      // the embedding gather's clamp, then the table's range
    long long id = g_dd_tok[b] + (long long)s * V;
    id = id < 0 ? 0 : (id >= erows ? erows - 1 : id);
    const long long t = id - V;
    return t < 0 ? 0 : (t >= trows ? trows - 1 : t);
  };
  const int gt = (int)blockIdx.x * PK_CONSUMERS + tid, gs = (int)gridDim.x * PK_CONSUMERS;
  const int hu = H >> 3;
  for (int i = gt; i < M * hu; i += gs) {
    const int b = i / hu, u = i - b * hu;
    reinterpret_cast<uint4*>(xres + (size_t)b * H)[u] =
        __ldcg(reinterpret_cast<const uint4*>(a.ptab + (size_t)trow(b) * H) + u);
  }
  cp_async_wait<0>();
  named_sync(1, PK_CONSUMERS);
  const int npair = (NH + 2 * NKV) * 64;
  for (int i = gt; i < M * npair; i += gs) {
    const int b = i / npair, u = i - b * npair, hh = u >> 6, d = u & 63;
    const bf16* src = a.ttab + (size_t)trow(b) * QKV + (size_t)hh * 128;
    float y0 = b2f(src[d]), y1 = b2f(src[d + 64]);
    if (hh < NH + NKV) {
      const float c0 = b2f(g_dd_cs[0][d]), s0 = b2f(g_dd_cs[1][d]);
      const float c1 = b2f(g_dd_cs[0][d + 64]), s1 = b2f(g_dd_cs[1][d + 64]);
      const float o0 = rbf(rbf(y0 * c0) + rbf(-y1 * s0));
      const float o1 = rbf(rbf(y1 * c1) + rbf(y0 * s1));
      y0 = o0;
      y1 = o1;
    }
    if (hh < NH) {
      qb[(size_t)b * QD + hh * 128 + d] = __float2bfloat16_rn(y0);
      qb[(size_t)b * QD + hh * 128 + d + 64] = __float2bfloat16_rn(y1);
    } else {
      const int kvh = hh < NH + NKV ? hh - NH : hh - NH - NKV;
      bf16* cache = hh < NH + NKV ? kcache : vcache;
      bf16* dst = cache + ((((size_t)0 * M + b) * NKV + kvh) * P + pos) * 128;
      dst[d] = __float2bfloat16_rn(y0);
      dst[d + 64] = __float2bfloat16_rn(y1);
    }
  }
  DD_STAMP(s, 1);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, 2);
  return c;
}

// S1: RMSNorm + q|k|v (rotary pairs) + RoPE + KV write at `pos`
template <int NT>
__device__ __noinline__ DDCur dd_phase_s1(const DDArgs& a, DDCur c, int s, int pos, int l) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, H = a.H, NH = a.NH, NKV = a.NKV, QD = NH * 128;
  const int tb = 3 + 9 * l;
  const int P = a.P;
  bf16 *const qb = a.qb, *const kcache = a.kc, *const vcache = a.vc;
  const int xp = (NT > 0) ? H * 2 + 16 : 0;
  load_x(m.xs, xp, a.xres, H, M, H, a.layers[l].ln1, a.eps, g_dd_nred);
  if (!dd_gemv<NT, 2>(a, m, c, (NH + 2 * NKV) * 64, H, xp,
                           [&](int n0, int nu, const float* sm, int lt) {
                             if (lt < nu * M) {
                               const int i = lt / M, b = lt - i * M;
                               const int u = n0 + i, hh = u >> 6, d = u & 63;
                               float y0 = rbf(sm[i * MS + b]), y1 = rbf(sm[(i + 8) * MS + b]);
                               if (hh < NH + NKV) {
                                 const float c0 = b2f(g_dd_cs[0][d]), s0 = b2f(g_dd_cs[1][d]);
                                 const float c1 = b2f(g_dd_cs[0][d + 64]), s1 = b2f(g_dd_cs[1][d + 64]);
                                 const float o0 = rbf(rbf(y0 * c0) + rbf(-y1 * s0));
                                 const float o1 = rbf(rbf(y1 * c1) + rbf(y0 * s1));
                                 y0 = o0;
                                 y1 = o1;
                               }
                               if (hh < NH) {
                                 qb[(size_t)b * QD + hh * 128 + d] = __float2bfloat16_rn(y0);
                                 qb[(size_t)b * QD + hh * 128 + d + 64] = __float2bfloat16_rn(y1);
                               } else {
                                 const int kvh = hh < NH + NKV ? hh - NH : hh - NH - NKV;
                                 bf16* cache = hh < NH + NKV ? kcache : vcache;
                                 bf16* dst = cache + ((((size_t)l * M + b) * NKV + kvh) * P + pos) * 128;
                                 dst[d] = __float2bfloat16_rn(y0);
                                 dst[d + 64] = __float2bfloat16_rn(y1);
                               }
                             }
                           }, [](int) {})) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, tb + 0);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, tb + 1);
  return c;
}

// S2: attention + o GEMV.  Small batches: every CTA computes every row (no barrier).  Otherwise CTA i takes
// (batch row, KV head) pair i, writes it over its q slice, and a barrier precedes the o-projection.
template <int G, int NT>
__device__ __noinline__ DDCur dd_phase_s2(const DDArgs& a, DDCur c, int s, int pos, int l) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, H = a.H, NKV = a.NKV, QD = a.NH * 128;
  const int xp_q = (NT > 0) ? QD * 2 + 16 : 0;
  const int tb = 3 + 9 * l;
  bf16* const ob = a.ob;
  if (a.att_split) {
    const int npairs = a.B * NKV;
    const int p0 = (int)((long long)npairs * blockIdx.x / gridDim.x);
    const int p1 = (int)((long long)npairs * (blockIdx.x + 1) / gridDim.x);
    dd_attention_pairs<G>(a, l, pos, p0, p1, m.xs + a.att_off);
    if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) {
      c.ok = 0;
      return c;
    }
    load_x(m.xs, xp_q, a.qb, QD, M, QD, nullptr, 0.f, g_dd_nred);
  } else {
    dd_attention<G>(a, l, pos, m.xs, xp_q, m.xs + a.att_off);
  }
  DD_STAMP(s, tb + 2);
  if (!dd_gemv<NT, 0>(a, m, c, H, QD, xp_q,
                      [&](int n0, int nu, const float* sm, int lt) {
                        if (lt < nu * M) {
                          const int i = lt / M, r = lt - i * M;
                          ob[(size_t)r * H + n0 + i] = __float2bfloat16_rn(sm[i * MS + r]);
                        }
                      }, [](int) {}, nullptr, 0, a.s3_o)) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, tb + 3);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, tb + 4);
  return c;
}

// S3: RMSNorm(bf16(x + o)) + gate|up + SiLU*up; the un-normalised x_mid rows stay in shared memory for S4
template <int NT>
__device__ __noinline__ DDCur dd_phase_s3(const DDArgs& a, DDCur c, int s, int l) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, H = a.H, F = a.F;
  const int tb = 3 + 9 * l;
  bf16* xkeep = reinterpret_cast<bf16*>(m.xs + a.keep_off);
  bf16* const act = a.act;
  const int xp = (NT > 0) ? H * 2 + 16 : 0;
  dd_load_mid(m.xs, xp, a, M, a.layers[l].ln2, g_dd_nred, xkeep, dd_s4_col0<NT>(a));
  if (!dd_gemv<NT, 1>(a, m, c, F, H, xp,
                      [&](int n0, int nu, const float* sm, int lt) {
                        if (lt < nu * M) {
                          const int i = lt / M, r = lt - i * M;
                          const float g = rbf(sm[i * MS + r]);
                          const float u = rbf(sm[(i + 8) * MS + r]);
                          act[(size_t)r * F + n0 + i] = __float2bfloat16_rn(silu_rbf(g) * u);
                        }
                      }, [](int) {})) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, tb + 5);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, tb + 6);
  return c;
}

// S4: down + residual: xres = bf16(x_mid + bf16(d)); act rows too large to stage whole go in column chunks
template <int NT>
__device__ __noinline__ DDCur dd_phase_s4(const DDArgs& a, DDCur c, int s, int l) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, H = a.H, F = a.F;
  const int tb = 3 + 9 * l;
  const bf16* xkeep = reinterpret_cast<const bf16*>(m.xs + a.keep_off);
  bf16* const xres = a.xres;
  const int kc = a.keep_cols;
  const int kc0 = dd_s4_col0<NT>(a);
  // tcgen05 build: act in passes of DD_TC_KX columns; mma.sync: whole, or in column chunks (d_xchunk)
  auto stage = [&](int p) {
    const int k0 = p * DD_TC_KX;
    load_x(m.xs, 0, a.act + k0, F, M, min(DD_TC_KX, F - k0), nullptr, 0.f, g_dd_nred);
  };
  if (NT <= 0) stage(0);
  else if (!a.d_xchunk) load_x(m.xs, F * 2 + 16, a.act, F, M, F, nullptr, 0.f, g_dd_nred);
  if (!dd_gemv<NT, 0>(a, m, c, H, F, a.d_xchunk ? ST_KC * 2 + 16 : F * 2 + 16,
                      [&](int n0, int nu, const float* sm, int lt) {
                        if (lt < nu * M) {
                          const int i = lt / M, r = lt - i * M, n = n0 + i;
                          const float xm = b2f(kc ? xkeep[(size_t)r * kc + (n - kc0)] : xkeep[(size_t)r * H + n]);
                          xres[(size_t)r * H + n] = __float2bfloat16_rn(xm + rbf(sm[i * MS + r]));
                        }
                      }, stage, a.d_xchunk ? a.act : nullptr, F, a.s3_down)) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, tb + 7);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, tb + 8);
  return c;
}

// S5: final RMSNorm + codebook head -> fp32 logits
template <int NT>
__device__ __noinline__ DDCur dd_phase_s5(const DDArgs& a, DDCur c, int s) {
  constexpr int MS = (NT > 0) ? 8 * NT : 16;
  DDSm m = dd_smem<NT>(a);
  const int tid = threadIdx.x, M = a.B, H = a.H, V = a.V;
  const int te = 3 + 9 * a.L;
  float *const logits = a.logits, *const dbg = a.dbg;
  const int xp = (NT > 0) ? H * 2 + 16 : 0;
  load_x(m.xs, xp, a.xres, H, M, H, a.normf, a.eps, g_dd_nred);
  if (!dd_gemv<NT, 0>(a, m, c, V, H, xp,
                      [&](int n0, int nu, const float* sm, int lt) {
                        if (lt < nu * M) {
                          const int i = lt / M, b = lt - i * M;
                          const float v = sm[i * MS + b];
                          logits[(size_t)b * V + n0 + i] = v;
                          if (dbg) dbg[((size_t)s * M + b) * V + n0 + i] = v;
                        }
                      }, [](int) {}, nullptr, 0, a.s3_head)) {
    c.ok = 0;
    return c;
  }
  DD_STAMP(s, te + 0);
  if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) c.ok = 0;
  DD_STAMP(s, te + 1);
  return c;
}

// Sampling.  One CFG pair: every CTA samples it (no barrier follows), CTA 0 publishes.  Several pairs: CTA h samples
// pair h and publishes it, then one barrier hands every CTA the fed-forward tokens (one barrier instead of `half`
// samplers in series on every CTA).
__device__ __noinline__ DDCur dd_phase_sample(const DDArgs& a, DDCur c, int s) {
  const int tid = threadIdx.x, V = a.V;
  const int half = a.B >= 2 ? a.B / 2 : 1;
  const int te = 3 + 9 * a.L;
  extern __shared__ __align__(128) unsigned char smem[];
  const bool redundant = half == 1;
  const int h_begin = redundant ? 0 : (int)blockIdx.x;
  const int h_end = redundant ? 1 : ((int)blockIdx.x < half ? (int)blockIdx.x + 1 : 0);
  for (int h = h_begin; h < h_end; ++h) {
    int tokv = dd_sample(a, s, h, smem, g_dd_int);
    tokv = tokv < 0 ? 0 : (tokv > V - 1 ? V - 1 : tokv);
    if (tid == 0) {
      for (int r = 0; r < (a.B >= 2 ? 2 : 1); ++r) {
        const int b = h + r * half;
        long long fed = tokv;
        if (a.forced) {
          const long long fc = a.forced[(size_t)s * a.B + b];
          fed = fc < 0 ? 0 : (fc > V - 1 ? V - 1 : fc);
        }
        g_dd_tok[b] = fed;
        if (blockIdx.x == 0 || !redundant) {
          a.outtok[(size_t)b * a.NCB + s] = tokv;
          a.tokbuf[b] = fed;
        }
      }
    }
  }
  if (!redundant && s + 1 < a.NCB) {
    if (!grid_sync(a.bar, c.epoch, a.err, &g_dd_int[31], a.wait_ns)) {
      c.ok = 0;
      return c;
    }
    if (tid < a.B) g_dd_tok[tid] = __ldcg(a.tokbuf + tid);
  }
  named_sync(1, PK_CONSUMERS);
  DD_STAMP(s, te + 7);
  return c;
}

template <int G, int NT>
__global__ void __launch_bounds__(PK_THREADS, 1) dd_frame_kernel(const __grid_constant__ DDArgs a) {
  const int tid = threadIdx.x, warp = tid >> 5;
  {
    DDSm m = dd_smem<NT>(a);
    if (tid == 0) {
      for (int s = 0; s < m.rg.nst; ++s) {
        mbar_init(&m.rg.full[s], 1);
        mbar_init(&m.rg.empty[s], (NT > 0) ? ST_CWARPS : 1);   // tcgen05 build: released by one tcgen05.commit
        if (NT < 0) mbar_init(&g_dd_dfull[s], LN_DEC_WARPS);
      }
      if (NT <= 0) mbar_init(&g_dd_mbar, 1);
      fence_mbar_init();
    }
    if (tid < 32) reinterpret_cast<uint32_t*>(m.zero16)[tid] = 0u;
    if (tid == 0) g_dd_int[28] = 0;                         // the consumers' "stopped early" flag
    if (tid == 0) g_dd_call = 0;
    if (tid == 0) g_dd_l2keep = a.l2_keep;
    if (NT <= 0 && warp == 0) tc_alloc(&g_dd_tmem, NT < 0 ? 128 : 64);  // 4 chains x 16 columns (LN12: x 2)
  }
  // the split tasks' publication tags start every frame at zero (ordered before their first use by a grid barrier)
  if (NT == 0 && a.flags && blockIdx.x == 0 && tid < a.nflags) a.flags[tid] = 0u;
  if (NT <= 0) tc_before();
  __syncthreads();
  if (NT <= 0) tc_after();
  if (warp == ST_CWARPS) {
    dd_producer<NT>(a);
    return;
  }
  // Codebook step 0 feeds two tokens (positions 0 and 1); they run as two sub-steps of one token each, which gives
  // the same values (GEMV rows are independent, position 0 does not attend to position 1) with M = B rows always.
  // A phase that gave up on a bounded wait returns ok = 0 on every consumer thread alike; the loop then ends.
  DDCur c{0, 0u, 1, 0u};
  for (int s = 0; s < a.NCB && c.ok; ++s) {
    for (int sub = 0; sub < (s == 0 ? 2 : 1) && c.ok; ++sub) {
      const int pos = s == 0 ? sub : s + 1;
      const bool tab = a.ptab && s >= 1;
      c = tab ? dd_phase_tab(a, c, s, pos) : dd_phase_e<NT>(a, c, s, sub, pos);
      for (int l = 0; l < a.L && c.ok; ++l) {
        if (!(tab && l == 0)) c = dd_phase_s1<NT>(a, c, s, pos, l);
        if (c.ok) c = dd_phase_s2<G, NT>(a, c, s, pos, l);
        if (c.ok) c = dd_phase_s3<NT>(a, c, s, l);
        if (c.ok) c = dd_phase_s4<NT>(a, c, s, l);
      }
    }
    if (c.ok) c = dd_phase_s5<NT>(a, c, s);
    if (c.ok) c = dd_phase_sample(a, c, s);
  }
  if (!c.ok && tid == 0) {
    // stopped early: the producer must not wait for ring slots nobody will release
    *reinterpret_cast<volatile int*>(&g_dd_int[28]) = 1;
    __threadfence_block();
  }
  if (NT <= 0) {
    // every MMA of this CTA has completed (each task waits for its last commit); free the accumulators
    tc_before();
    named_sync(1, PK_CONSUMERS);
    tc_after();
    if (warp == 0) tc_dealloc(g_dd_tmem, NT < 0 ? 128 : 64);
  }
  if (c.ok) grid_exit(a.bar);
}

}  // namespace fb

// ------------------------------------------------------------------------------------------------ host API
namespace {
using namespace fb;

struct DDLayout {
  size_t xres, qb, ob, act, kc, vc, logits, bar, part, flags, total;
};
// Blocks of 128 output units a split task may cover (the hidden size or the codebook vocabulary).
int dd_split_blocks(const fb_dd_config* c) { return ((c->hidden > c->vocab ? c->hidden : c->vocab) + 127) / 128; }
size_t al256d(size_t v) { return (v + 255) / 256 * 256; }

DDLayout dd_layout(const fb_dd_config* c) {
  DDLayout s{};
  const size_t M = (size_t)c->batch;       // one token per row per sub-step
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
  s.part = o; o = al256d(o + (size_t)dd_split_blocks(c) * 2048 * 4);     // one fp32 partial (S = 2) per block
  s.flags = o; o = al256d(o + (size_t)dd_split_blocks(c) * 4);
  s.total = o;
  return s;
}

// Checks of the configuration's fields, made before anything is sized or enqueued from them.
int dd_validate(const fb_dd_config* c) {
  FB_CHECK_ARG(c->head_dim == 128 && c->batch >= 1 && c->batch <= DD_MAXB && (c->batch == 1 || c->batch % 2 == 0),
               "dd_frame: head_dim must be 128, batch 1 or an even number up to %d", DD_MAXB);
  FB_CHECK_ARG(c->vocab >= 1 && c->vocab <= DD_MAXV && c->codebook_size >= 1 && c->codebook_size <= c->vocab,
               "dd_frame: vocab must be <= %d and codebook_size <= vocab", DD_MAXV);
  FB_CHECK_ARG(c->n_decode >= 1 && c->n_decode <= 31, "dd_frame: n_decode must be 1..31");
  FB_CHECK_ARG(c->heads >= 1 && c->kv_heads >= 1 && c->heads <= 64 && c->heads % c->kv_heads == 0,
               "dd_frame: heads must be 1..64 and a multiple of kv_heads >= 1");
  FB_CHECK_ARG(c->hidden >= 64 && c->embed_dim >= 64 && c->ffn >= 64 && c->hidden <= 65536 &&
                   c->embed_dim <= 65536 && c->ffn <= 65536 && c->hidden % 64 == 0 && c->embed_dim % 64 == 0 &&
                   c->ffn % 64 == 0,
               "dd_frame: hidden, embed_dim and ffn must be positive multiples of 64 up to 65536");
  FB_CHECK_ARG(c->layers >= 1 && c->layers <= DD_MAXL && c->layers_host,
               "dd_frame: 1..%d layers, with the host copy of the layer table (layers_host)", DD_MAXL);
  return FB_OK;
}

template <int G, int NT>
int launch_dd(DDArgs& a, size_t smem, int grid, cudaStream_t st) {
  auto kern = dd_frame_kernel<G, NT>;
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
  cfg.gridDim = dim3(grid);
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

extern "C" int flashb_dd_tab_build(const fb_dd_config* c, void* ptab, void* ttab, void* work, void* stream) {
  FB_CHECK_ARG(c && ptab && ttab && work && c->layers_host && c->embed && c->proj, "dd_tab_build: null argument");
  if (int rc = dd_validate(c)) return rc;
  FB_CHECK_ARG(c->n_decode >= 2, "dd_tab_build: the table covers codebook steps 1 .. n_decode - 1");
  const fb_dd_layer* L0 = (const fb_dd_layer*)c->layers_host;
  const int V = c->vocab, H = c->hidden, AE = c->embed_dim, QD = c->heads * 128, KD = c->kv_heads * 128;
  const int rows = (c->n_decode - 1) * V;
  const bf16* emb = (const bf16*)c->embed + (size_t)V * AE;    // embedding rows vocab .. n_decode vocab - 1
  // ptab = embed rows . proj^T (the frame's stage E), then ttab = RMSNorm(ptab; ln1) . [wq; wk; wv]^T (layer 0's S1)
  int rc = flashb_gemv_seg(emb, AE, rows, AE, nullptr, 0.f, c->proj, H, nullptr, 0, nullptr, 0, ptab, H, stream);
  if (rc) return rc;
  rc = flashb_rmsnorm(ptab, H, rows, H, L0->ln1, c->eps, work, H, stream);
  if (rc) return rc;
  return flashb_gemv_seg(work, H, rows, H, nullptr, 0.f, L0->wq, QD, L0->wk, KD, L0->wv, KD, ttab, QD + 2 * KD,
                         stream);
}

extern "C" int64_t flashb_dd_scratch_bytes(const fb_dd_config* cfg) {
  if (!cfg) return -1;
  return (int64_t)dd_layout(cfg).total;
}

extern "C" int64_t flashb_dd_layer_bytes(void) { return (int64_t)sizeof(fb_dd_layer); }

extern "C" int64_t flashb_dd_barrier_offset(const fb_dd_config* cfg) {
  if (!cfg) return -1;
  return (int64_t)dd_layout(cfg).bar;
}

extern "C" int flashb_dd_frame(const fb_dd_config* c, const void* layers_dev, void* scratch, const int64_t* first_cb,
                               const void* bh, int64_t* tokbuf, int64_t* outtok, const float* temp,
                               const int64_t* topk, const float* topp, const int64_t* dosample, const float* gs,
                               const float* q, float* dbg, const int64_t* forced, void* stream) {
  static_assert(sizeof(fb_dd_layer) == sizeof(DDLayer), "fb_dd_layer layout");
  FB_CHECK_ARG(c && layers_dev && scratch && first_cb && bh && tokbuf && outtok && temp && topk && topp && dosample &&
                   gs && q, "dd_frame: null pointer argument");
  if (int rc = dd_validate(c)) return rc;
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
  a.part = (float*)(sc + Lo.part); a.flags = (unsigned*)(sc + Lo.flags); a.nflags = dd_split_blocks(c);
  a.err = fbh::device_err_ptr();
  a.wait_ns = c->wait_ns > 0 ? (unsigned long long)c->wait_ns : WAIT_LIMIT_NS;
  a.trace = (unsigned long long*)c->trace;
  FB_CHECK_ARG(!c->ptab == !c->ttab, "dd_frame: step table needs both ptab and ttab");
  a.ptab = (const bf16*)c->ptab;
  a.ttab = (const bf16*)c->ttab;
  {
    const char* e = getenv("FLASHB_DD_L2_KEEP");      // L2 policy of the weight copies (tuning): 1 evict_last
    a.l2_keep = (e && e[0] == '1') ? 1 : 0;
  }
  const size_t M = (size_t)c->batch;
  const int grid = c->grid > 0 ? c->grid : fbh::grid_sms();
  if (grid > fbh::num_sms() || grid < (c->batch >= 2 ? c->batch / 2 : 1)) {
    fbh::set_msg("dd_frame: grid %d outside [%d, %d] (one CTA per SM, one per CFG pair at least)", grid,
                 c->batch >= 2 ? c->batch / 2 : 1, fbh::num_sms());
    return FB_ERR_ARG;
  }
  // Build: on a small grid (a lane of the GPU) the tcgen05 GEMVs (NT = 0): a CTA streams several 128-row blocks
  // and the per-CTA rate decides; on a large grid the mma.sync stream with 16-row groups spreads each matrix over
  // every SM (NT = 1 or 2 activation tiles of 8 rows).
  const int QD = c->heads * 128, KD = c->kv_heads * 128;
  const bool tc = grid <= DD_TC_MAX_GRID && c->hidden % 256 == 0 && c->embed_dim % 256 == 0 && c->ffn % 256 == 0 &&
                  QD % 256 == 0;
  // NT = -1: the tcgen05 build streaming LN12 (fb_dd_config.ln12; set up below)
  const int NT = tc ? (c->ln12 ? -1 : 0) : (c->batch > 8 ? 2 : 1);
  {
    // tensor maps of every streamed matrix, built from the host copy of the layer table (cached per matrix):
    // mma.sync build: 8-row boxes of ST_KC columns.  tcgen05 build: the stage of the task's kind, 64 rows x 256
    // columns (plain), 128 x 64 (gate, up), 128 x 128 (q, k, v heads)
    const DDLayer* hl = (const DDLayer*)c->layers_host;
    auto map = [&](CUtensorMap* out, const void* base, long long rows, int K, int kind) {
      if (!tc) return fbh::tmap_rows(out, base, rows, K, ST_KC);
      return fbh::tmap_box(out, base, rows, K, 64, kind == 0 ? 64 : 128, kind == 0 ? 4 : (kind == 1 ? 1 : 2), true);
    };
    // tcgen05 bf16 build: the plain matrices as 128-row tasks (maps of 128-row boxes), split in 2 parts of K when
    // that still leaves no more items than CTAs and each part stays inside one staged pass of activations
    auto fits = [&](int K, int S) {          // every part of K inside one staged pass of activations
      const int KX = K < DD_TC_KX ? K : DD_TC_KX, Kp = K / S;
      for (int p = 0; p < S; ++p)
        if ((p * Kp) % KX + Kp > KX) return false;
      return true;
    };
    auto split_of = [&](long long rows, int K) {
      if (!tc || c->ln12 || rows % 128) return 0;
      if (2 * (rows / 128) <= grid && K % 256 == 0 && fits(K, 2)) return 2;
      return (K % 128 == 0 && fits(K, 1)) ? 1 : 0;
    };
    // Which tasks take the 128-row form (tuning: FLASHB_DD_TASK128 = four digits for projector, o, down, heads;
    // default 0011).  Measured at the bench's lane (B = 16, grid 18, a frame alone): 6.613 ms with none, 6.575 with
    // the heads, 6.535 with the heads and the split down, 6.754 adding the split o: its parts' exchange through L2
    // (about 3 us) outweighs the shorter MMA stream of a 1024-column task.
    const char* t128 = getenv("FLASHB_DD_TASK128");
    const bool use128[4] = {t128 && strlen(t128) == 4 ? t128[0] == '1' : false,
                            t128 && strlen(t128) == 4 ? t128[1] == '1' : false,
                            t128 && strlen(t128) == 4 ? t128[2] == '1' : true,
                            t128 && strlen(t128) == 4 ? t128[3] == '1' : true};
    a.s3_proj = use128[0] ? split_of(c->hidden, c->embed_dim) : 0;
    a.s3_o = use128[1] ? split_of(c->hidden, QD) : 0;
    a.s3_down = use128[2] ? split_of(c->hidden, c->ffn) : 0;
    a.s3_head = use128[3] ? split_of(c->vocab, c->hidden) : 0;
    int rc = map(&a.tm_proj, c->proj, c->hidden, c->embed_dim, a.s3_proj ? 2 : 0);
    if (!rc) rc = map(&a.tm_head, c->head_t, (long long)c->n_decode * c->vocab, c->hidden, a.s3_head ? 2 : 0);
    for (int l = 0; l < c->layers && !rc; ++l) {
      const DDLayer& W = hl[l];
      rc = map(&a.tm[l][DD_WQ], W.wq, QD, c->hidden, 2);
      if (!rc) rc = map(&a.tm[l][DD_WK], W.wk, KD, c->hidden, 2);
      if (!rc) rc = map(&a.tm[l][DD_WV], W.wv, KD, c->hidden, 2);
      if (!rc) rc = map(&a.tm[l][DD_WO], W.wo, c->hidden, QD, a.s3_o ? 2 : 0);
      if (!rc) rc = map(&a.tm[l][DD_WG], W.wg, c->ffn, c->hidden, 1);
      if (!rc) rc = map(&a.tm[l][DD_WU], W.wu, c->ffn, c->hidden, 1);
      if (!rc) rc = map(&a.tm[l][DD_WD], W.wd, c->hidden, c->ffn, a.s3_down ? 2 : 0);
    }
    if (rc) return rc;
  }
  if (tc && c->ln12) {
    // LN12 streaming: the data maps replace the bf16 ones (64-row boxes); records, patches and tables per matrix
    FB_CHECK_ARG(c->hidden % 1024 == 0 && c->embed_dim % 1024 == 0 && c->ffn % 1024 == 0 && QD % 1024 == 0 &&
                     c->vocab % 64 == 0 && KD % 64 == 0,
                 "dd_frame: LN12 streaming needs hidden, embed_dim, ffn, heads x 128 multiples of 1024 and vocab, "
                 "kv_heads x 128 multiples of 64");
    auto lnm = [&](int i, CUtensorMap* tm, LNMat* out, long long N, int K) {
      const fb_ln12_mat& e = c->ln12[i];
      if (!e.data || !e.meta || (reinterpret_cast<uintptr_t>(e.meta) & 15) || (!e.ovf && e.n_ovf > 0) || e.n_ovf < 0) {
        fbh::set_msg("dd_frame: LN12 matrix %d: null or misaligned pointers", i);
        return (int)FB_ERR_ARG;
      }
      *out = LNMat{(const uint4*)e.meta, (const unsigned*)e.ovf, (long long)e.n_ovf, e.lut_lo, e.lut_hi};
      return fbh::tmap_ln12(tm, e.data, N, K, LN_ROWS);
    };
    int rc = 0;
    for (int l = 0; l < c->layers && !rc; ++l) {
      const int i0 = l * DD_NMAPS;
      rc = lnm(i0 + DD_WQ, &a.tm[l][DD_WQ], &a.ln[l][DD_WQ], QD, c->hidden);
      if (!rc) rc = lnm(i0 + DD_WK, &a.tm[l][DD_WK], &a.ln[l][DD_WK], KD, c->hidden);
      if (!rc) rc = lnm(i0 + DD_WV, &a.tm[l][DD_WV], &a.ln[l][DD_WV], KD, c->hidden);
      if (!rc) rc = lnm(i0 + DD_WO, &a.tm[l][DD_WO], &a.ln[l][DD_WO], c->hidden, QD);
      if (!rc) rc = lnm(i0 + DD_WG, &a.tm[l][DD_WG], &a.ln[l][DD_WG], c->ffn, c->hidden);
      if (!rc) rc = lnm(i0 + DD_WU, &a.tm[l][DD_WU], &a.ln[l][DD_WU], c->ffn, c->hidden);
      if (!rc) rc = lnm(i0 + DD_WD, &a.tm[l][DD_WD], &a.ln[l][DD_WD], c->hidden, c->ffn);
    }
    const int ip = c->layers * DD_NMAPS;
    if (!rc) rc = lnm(ip, &a.tm_proj, &a.ln_proj, c->hidden, c->embed_dim);
    for (int h = 0; h < c->n_decode && !rc; ++h) rc = lnm(ip + 1 + h, &a.tm_hd[h], &a.ln_hd[h], c->vocab, c->hidden);
    if (rc) return rc;
    a.ln12 = 1;
  }
  // One buffer, several uses, sized for the largest:
  //   GEMV input rows of every phase (E: embed_dim, S1 / S3 / S5: hidden, S2: heads x 128; S4: ffn, whole or as
  //   two column-chunk buffers when whole rows would leave fewer than 3 ring stages; the tcgen05 build stages 16
  //   rows of at most DD_TC_KX columns in the B-operand layout);
  //   x_mid rows kept from S3 to S4 (keep_off, past the S4 input region); attention output rows + staging (att_off);
  //   the sampler's keys.
  const size_t xp_kc = ST_KC * 2 + 16;
  const size_t KXe = (size_t)(c->embed_dim < DD_TC_KX ? c->embed_dim : DD_TC_KX);
  const size_t KXf = (size_t)(c->ffn < DD_TC_KX ? c->ffn : DD_TC_KX);
  size_t rows, att_off;
  if (tc) {
    rows = 16 * 2 * KXe;
    if (16 * 2 * (size_t)c->hidden > rows) rows = 16 * 2 * (size_t)c->hidden;
    if (16 * 2 * (size_t)QD > rows) rows = 16 * 2 * (size_t)QD;
    att_off = al256d(16 * 2 * (size_t)QD);
  } else {
    rows = M * (c->embed_dim * 2 + 16);
    if (M * (c->hidden * 2 + 16) > rows) rows = M * (c->hidden * 2 + 16);
    if (M * (QD * 2 + 16) > rows) rows = M * (QD * 2 + 16);
    att_off = al256d(M * (QD * 2 + 16));
  }
  const size_t xs_smp = al256d(dd_sampler_bytes(c->vocab));
  const size_t budget = 227 * 1024 - ST_CWARPS * 16 * 4 - 32 * 4 - DD_MAXB * 8 - 2 * 128 * 2 - 256 - 16;
  const size_t red_bytes = tc ? DD_TC_SUMS * 4 + 1024 : ST_CWARPS * 128 * 4 * NT + 128 * 4 * NT;
  const size_t slot = ST_BYTES;
  auto stages_for = [&](size_t xsb) {
    const size_t fixed = xsb + 128 + ST_ALIGN + red_bytes + 2 * PK_MAX_STAGES * 8;
    int n = fixed < budget ? (int)((budget - fixed) / slot) : 0;
    return n > PK_MAX_STAGES ? PK_MAX_STAGES : n;
  };
  // x_mid kept from S3 to S4 (its rows also stage ob in S3).  tcgen05 build with room for ob beside the 16 staged
  // rows: only the CTA's S4 columns (its blocks of 64 output units), ob staged in the free half of the rows region
  int keep_cols = 0;
  if (a.s3_down) {
    // the blocks of 128 columns a CTA's split items touch
    const int S = a.s3_down, items = c->hidden / 128 * S;
    for (int g = 0; g < grid; ++g) {
      const int i0 = (int)((long long)items * g / grid), i1 = (int)((long long)items * (g + 1) / grid);
      if (i1 > i0 && ((i1 - 1) / S + 1 - i0 / S) * 128 > keep_cols) keep_cols = ((i1 - 1) / S + 1 - i0 / S) * 128;
    }
  } else {
    const int s4_blocks = (c->hidden + 63) / 64;
    keep_cols = (s4_blocks + grid - 1) / grid * 64;
  }
  a.keep_cols = (tc && (size_t)2 * 16 * c->hidden * 2 <= (size_t)16 * 2 * KXf && keep_cols < c->hidden) ? keep_cols : 0;
  const size_t keep_rows = a.keep_cols ? (size_t)a.keep_cols : (size_t)c->hidden;
  auto layout = [&](int d_chunk, size_t& keep_off, size_t& base) {
    const size_t d_region = tc ? 16 * 2 * KXf : (d_chunk ? 2 * M * xp_kc : M * (c->ffn * 2 + 16));
    keep_off = al256d(d_region > rows ? d_region : rows);
    base = al256d(keep_off + M * keep_rows * 2);
    if (al256d(rows) > base) base = al256d(rows);
    if (xs_smp > base) base = xs_smp;
  };
  size_t keep_off = 0, base = 0;
  a.d_xchunk = 0;
  layout(0, keep_off, base);
  if (!tc && stages_for(base) < 3) {
    a.d_xchunk = 1;
    layout(1, keep_off, base);
  }
  // attention: the whole batch in one staging round when that still leaves 4 ring stages; otherwise the
  // (batch row, KV head) pairs spread over the CTAs (distributed mode: one extra grid barrier per layer, small
  // staging); if even a CTA's share of pairs leaves fewer than 3 stages, the batch in chunks of rows on every CTA
  const int G = c->heads / c->kv_heads;
  size_t xs = al256d(att_off + dd_attn_bytes(c->batch, c->heads, c->kv_heads, c->n_decode + 1));
  if (xs < base) xs = base;
  int nst = stages_for(xs);
  a.att_bc = c->batch;
  a.att_split = 0;
  // ring depth wanted / acceptable, in slots (tcgen05 slots are half as large)
  const int want = 4, accept = 3, least = 2;
  if (nst < want) {
    const int per_cta = (c->batch * c->kv_heads + grid - 1) / grid;
    size_t xs_split = al256d(att_off + per_cta * dd_pair_bytes(G, c->n_decode + 1));
    if (xs_split < base) xs_split = base;
    if (stages_for(xs_split) >= accept) {
      xs = xs_split;
      nst = stages_for(xs);
      a.att_split = 1;
    }
  }
  while (nst < want && !a.att_split && a.att_bc > 1) {
    a.att_bc = (a.att_bc + 1) / 2;
    xs = al256d(att_off + dd_attn_bytes(a.att_bc, c->heads, c->kv_heads, c->n_decode + 1));
    if (xs < base) xs = base;
    nst = stages_for(xs);
  }
  if (nst < least) {
    fbh::set_msg("dd_frame: activations too large for %d ring slots", least);
    return FB_ERR_UNSUPPORTED;
  }
  a.xs_bytes = (int)xs;
  a.att_off = (int)att_off;
  a.keep_off = (int)keep_off;
  const size_t fixed = xs + 128 + ST_ALIGN + red_bytes + 2 * PK_MAX_STAGES * 8;
  a.nstages = nst;
  const size_t smem = fixed + (size_t)nst * slot;
  cudaStream_t st = (cudaStream_t)stream;
  if (NT < 0) {
    switch (G) {
      case 1: return launch_dd<1, -1>(a, smem, grid, st);
      case 2: return launch_dd<2, -1>(a, smem, grid, st);
      case 4: return launch_dd<4, -1>(a, smem, grid, st);
      case 8: return launch_dd<8, -1>(a, smem, grid, st);
      default: fbh::set_msg("dd_frame: GQA group %d not built", G); return FB_ERR_UNSUPPORTED;
    }
  }
  const int key = G * 10 + NT;
  switch (key) {
    case 10: return launch_dd<1, 0>(a, smem, grid, st);
    case 11: return launch_dd<1, 1>(a, smem, grid, st);
    case 12: return launch_dd<1, 2>(a, smem, grid, st);
    case 20: return launch_dd<2, 0>(a, smem, grid, st);
    case 21: return launch_dd<2, 1>(a, smem, grid, st);
    case 22: return launch_dd<2, 2>(a, smem, grid, st);
    case 40: return launch_dd<4, 0>(a, smem, grid, st);
    case 41: return launch_dd<4, 1>(a, smem, grid, st);
    case 42: return launch_dd<4, 2>(a, smem, grid, st);
    case 80: return launch_dd<8, 0>(a, smem, grid, st);
    case 81: return launch_dd<8, 1>(a, smem, grid, st);
    case 82: return launch_dd<8, 2>(a, smem, grid, st);
    default: fbh::set_msg("dd_frame: GQA group %d not built", G); return FB_ERR_UNSUPPORTED;
  }
}

// ------------------------------------------------------------------------------------------------ no-allocation variant
// Scratch of flashb_dd_frame_noalloc: a fixed 1 MiB area in device memory, reserved on every GPU that loads this
// library until the process exits.  In host code this name is only a stand-in for the symbol, never a device
// address; the host fetches the real address per device with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_dd_static_scratch[FB_DD_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_dd_static_mu;
void* g_dd_static_ptr[64] = {nullptr};
}  // namespace

extern "C" int flashb_dd_frame_noalloc(const fb_dd_config* c, const void* layers_dev, const int64_t* first_cb,
                                       const void* bh, int64_t* tokbuf, int64_t* outtok, const float* temp,
                                       const int64_t* topk, const float* topp, const int64_t* dosample,
                                       const float* gs, const float* q, float* dbg, const int64_t* forced,
                                       void* stream) {
  FB_CHECK_ARG(c, "dd_frame_noalloc: null config");
  // every field is checked before the layout is computed from it, so no size below can wrap
  if (int rc = dd_validate(c)) return rc;
  const DDLayout Lo = dd_layout(c);
  FB_CHECK_ARG(Lo.total <= (size_t)FB_DD_NOALLOC_SCRATCH_BYTES && Lo.bar + sizeof(GridBar) <= Lo.total,
               "dd_frame_noalloc: this configuration needs %zu bytes of scratch; the built-in area holds %u "
               "(use flashb_dd_frame with a caller-owned buffer)", Lo.total, (unsigned)FB_DD_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fbh::set_msg("dd_frame_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  FB_CHECK_ARG(dev >= 0 && dev < 64, "dd_frame_noalloc: device ordinal %d out of range", dev);
  void* base = nullptr;
  {
    // one-time set-up per device, with that device current: the device address of the static area
    std::lock_guard<std::mutex> lk(g_dd_static_mu);
    if (!g_dd_static_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_dd_static_scratch);
      if (e != cudaSuccess || !p) {
        fbh::set_msg("dd_frame_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        return FB_ERR_CUDA;
      }
      g_dd_static_ptr[dev] = p;
    }
    base = g_dd_static_ptr[dev];
  }
  // The area keeps whatever the previous call left.  Only the grid-barrier words must start at zero (a frame cut
  // short by a timeout leaves its abort flag set); everything else a frame reads it first writes itself.
  e = cudaMemsetAsync((unsigned char*)base + Lo.bar, 0, sizeof(GridBar), (cudaStream_t)stream);
  if (e != cudaSuccess) {
    fbh::set_msg("dd_frame_noalloc: clearing the barrier words: %s", cudaGetErrorString(e));
    return FB_ERR_CUDA;
  }
  return flashb_dd_frame(c, layers_dev, base, first_cb, bh, tokbuf, outtok, temp, topk, topp, dosample, gs, q, dbg,
                         forced, stream);
}
