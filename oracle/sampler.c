/* CPU oracle: the depth-decoder CFG sampler, bit-exact restatement (TEST INFRASTRUCTURE ONLY).
 *
 * Follows the official graph-safe sampler DepthDecoderGraph._cfg_sample
 * (UP/models/cudagraph/depth_decoder_graph.py:485-556, UP = third_party/breeze-tts) and the flash kernel's fused
 * version (flash/csrc/depth_frame.cu:381-654):
 *   cfg = u + gs * (c - u)            three separately rounded fp32 ops (no FMA)        (:494-499)
 *   ids >= codebook_size -> -inf      mask_invalid_codec_token_logits (UP/models/logits_process.py:7-25)
 *   key = cfg / temperature           IEEE division                                     (:508)
 *   top-k, k = top_k > 0 ? min(top_k, maxk) : maxk, maxk = min(1024, V)                (:510-522)
 *   top-p on the softmax of the sorted kept keys, shift-right removal, rank 0 kept      (:524-536)
 *   p = softmax(kept), token = argmax(p / q) with q ~ Exp(1)                            (:539-551)
 *     (torch.multinomial(p, 1) == argmax(p / Exp(1)) is the identity the reference relies on,
 *      flash/csrc/depth_frame.cu:6-8 and flash/depth.py:160-169)
 *   greedy = argmax(cfg) (first index on ties); token = do_sample ? sampled : greedy; clamp to [0, V-1].
 *
 * Rank order is (key descending, index ascending).  The exponential and the three sums are defined exactly as the
 * CUDA sampler evaluates them, so the CPU and GPU tokens are bitwise equal given identical logits:
 *   fb_exp(x): Cody-Waite range reduction x = n ln2 + r (ln2 split into a 15-bit head and a tail, W. J. Cody and
 *              W. Waite, "Software Manual for the Elementary Functions", 1980), exp(r) by the degree-7 Taylor
 *              polynomial sum r^i/i! evaluated by Horner's rule with fused multiply-adds, scaled by 2^n through the
 *              exponent bits.  Inputs <= -103 give 0 (so -inf gives 0).
 *   sums:      32 lanes; lane l owns ranks [l*C, l*C + C), C = ceil(k / 32); each lane adds its ranks in order from
 *              0.0f; lane sums are combined by a Kogge-Stone inclusive scan with offsets 1, 2, 4, 8, 16 (lane l adds
 *              the value of lane l - o); the total is lane 31's value and lane l's exclusive prefix is lane l-1's.
 *   top-p:     p_r = e_r / S; the lane sums of p are scanned the same way; cum_{r-1} = the lane's exclusive prefix
 *              (lane l-1's inclusive value, 0 for lane 0) plus the lane's earlier p_r added in rank order;
 *              rank r is kept iff r == 0 or !(cum_{r-1} > top_p).  S2 = the same sum over the kept e_r.
 * Build with -ffp-contract=off so the compiler adds no FMA of its own. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float exp2i(int n) { /* 2^n for n in [-126, 127] */
  uint32_t b = (uint32_t)(n + 127) << 23;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

float fb_exp(float x) {
  if (!(x > -103.0f)) return 0.0f;
  if (x > 88.0f) return INFINITY;
  const float n = rintf(x * 0x1.715476p+0f);
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
  if (ni < -125) return (p * exp2i(ni + 100)) * exp2i(-100);
  return p * exp2i(ni);
}

typedef struct {
  float key;
  int idx;
} kv_t;

static int rank_cmp(const void* a, const void* b) {
  const kv_t* x = (const kv_t*)a;
  const kv_t* y = (const kv_t*)b;
  if (x->key > y->key) return -1;
  if (x->key < y->key) return 1;
  return (x->idx < y->idx) ? -1 : (x->idx > y->idx);
}

static void lane_scan(const float* in, float* incl) {
  float s[32], t[32];
  memcpy(s, in, sizeof(s));
  for (int o = 1; o < 32; o <<= 1) {
    for (int l = 0; l < 32; ++l) t[l] = (l >= o) ? s[l - o] + s[l] : s[l];
    memcpy(s, t, sizeof(s));
  }
  memcpy(incl, s, sizeof(s));
}

/* One half-row.  lu == NULL means no CFG pair (batch 1).  Returns the token; *greedy_out gets argmax(cfg). */
int fb_sample_row(const float* lc, const float* lu, int V, int codebook_size, float gs, float temp, long long topk,
                  float topp, long long dosample, const float* q, int* greedy_out) {
  kv_t* kv = (kv_t*)malloc(sizeof(kv_t) * (size_t)V);
  float best_g = -INFINITY;
  int gidx = 0;
  int have_g = 0;
  for (int i = 0; i < V; ++i) {
    float cfg = lc[i];
    if (lu) {
      const float u = lu[i];
      const float d = cfg - u;
      const float m = gs * d;
      cfg = u + m;
    }
    if (i >= codebook_size) cfg = -INFINITY;
    if (!have_g || cfg > best_g) {
      best_g = cfg;
      gidx = i;
      have_g = 1;
    }
    kv[i].key = cfg / temp;
    kv[i].idx = i;
  }
  const int maxk = V < 1024 ? V : 1024;
  const int k = topk > 0 ? (topk < maxk ? (int)topk : maxk) : maxk;
  qsort(kv, (size_t)V, sizeof(kv_t), rank_cmp);
  const int C = (k + 31) / 32;
  float e[1024];
  for (int r = 0; r < k; ++r) e[r] = fb_exp(kv[r].key - kv[0].key);
  float b[32], incl[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int j = 0; j < C; ++j) {
      const int r = l * C + j;
      if (r < k) s = s + e[r];
    }
    b[l] = s;
  }
  lane_scan(b, incl);
  const float S = incl[31];
  float pr[1024], bp[32], inclp[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int j = 0; j < C; ++j) {
      const int r = l * C + j;
      if (r < k) {
        pr[r] = e[r] / S;
        s = s + pr[r];
      }
    }
    bp[l] = s;
  }
  lane_scan(bp, inclp);
  unsigned char keep[1024];
  float b2[32], incl2[32];
  for (int l = 0; l < 32; ++l) {
    float run = l ? inclp[l - 1] : 0.0f;
    float s2 = 0.0f;
    for (int j = 0; j < C; ++j) {
      const int r = l * C + j;
      if (r >= k) break;
      keep[r] = (r == 0) || !(run > topp);
      run = run + pr[r];
      if (keep[r]) s2 = s2 + e[r];
    }
    b2[l] = s2;
  }
  lane_scan(b2, incl2);
  const float S2 = incl2[31];
  float best = -1.0f;
  int bidx = 0x7fffffff;
  for (int r = 0; r < k; ++r) {
    if (!keep[r]) continue;
    const int id = kv[r].idx;
    const float sc = (e[r] / S2) / q[id];
    if (sc > best || (sc == best && id < bidx)) {
      best = sc;
      bidx = id;
    }
  }
  free(kv);
  if (greedy_out) *greedy_out = gidx;
  int tok = dosample ? bidx : gidx;
  if (tok < 0) tok = 0;
  if (tok > V - 1) tok = V - 1;
  return tok;
}

/* Vectorised helper for tests: fb_exp over n floats. */
void fb_exp_n(const float* x, float* y, int n) {
  for (int i = 0; i < n; ++i) y[i] = fb_exp(x[i]);
}

/* ---------------------------------------------------------------------------------------------------------------
 * The backbone (codebook-0) sampler: bit-exact restatement of the host-sync-free sample_logits of the reference
 * (flash/sampling.py:56-97, itself bitwise equal to the official models/cudagraph/sampling.py sample_logits) for one
 * row of CFG logits, in the official op order:
 *   repetition penalty on the ids marked present: x > 0 ? x / p : x * p           (flash/sampling.py:44-47, 81-82)
 *   suppressed ids -> -inf                                                         (:83-84)
 *   do_sample == 0: token = argmax(x), first index among equal maxima, a NaN counts as the maximum (torch.argmax)
 *   key = x / temperature                                                          (:89)
 *   top-k (top_k > 0): threshold = the k-th largest key (k = min(top_k, V), duplicates counted, torch.topk), keys
 *     below it -> -inf: every key equal to the threshold stays                      (:90-93)
 *   top-p (top_p < 1): over the keys in rank order, cumulative softmax, shift-right removal, rank 0 kept (:94-100)
 *   probs = softmax(keys); ok = the multinomial validity predicate: every prob finite, none negative, sum != 0 (so
 *     a NaN key, a +inf key or nothing finite left all give ok = 0)
 *   token = argmax(probs / q), q ~ Exp(1) (torch.multinomial(probs, 1) == argmax(probs / Exp(1)), the identity the
 *     reference's depth kernel relies on); with !ok the multinomial weights are all 1.0 (flash/sampling.py:50-53),
 *     so token = argmax(1 / q).  Ties of the score go to the lower index.
 * Rank order is (key descending, index ascending); ranks past the kept prefix have probability 0.  The exponential
 * and the sums are those of fb_sample_row (32 lanes own contiguous rank ranges of C = ceil(n / 32), in-lane sums in
 * rank order from 0.0f, Kogge-Stone scan), over the n = V ranks. */
static int bb_rank_cmp(const void* a, const void* b) { return rank_cmp(a, b); }

int fb_bb_sample_row(const float* logits, int V, const unsigned char* present, float penalty,
                     const long long* suppress, int n_suppress, float temp, long long topk, float topp,
                     long long dosample, const float* q, int* ok_out) {
  float* x = (float*)malloc(sizeof(float) * (size_t)V);
  for (int i = 0; i < V; ++i) {
    float v = logits[i];
    if (present && present[i] && penalty != 1.0f) v = v > 0.0f ? v / penalty : v * penalty;
    x[i] = v;
  }
  for (int j = 0; j < n_suppress; ++j)
    if (suppress[j] >= 0 && suppress[j] < V) x[suppress[j]] = -INFINITY;
  if (!dosample) {
    int g = 0;
    for (int i = 0; i < V; ++i) {
      if (isnan(x[g])) break;
      if (isnan(x[i]) || x[i] > x[g]) g = i;
    }
    free(x);
    if (ok_out) *ok_out = 1;
    return g;
  }
  kv_t* kv = (kv_t*)malloc(sizeof(kv_t) * (size_t)V);
  int any_nan = 0;
  for (int i = 0; i < V; ++i) {
    float k = x[i] / temp;
    if (isnan(k)) { /* torch ranks a NaN first, keeps it through top-k, and the softmax turns every prob to NaN */
      any_nan = 1;
      k = -INFINITY;
    }
    kv[i].key = k;
    kv[i].idx = i;
  }
  free(x);
  qsort(kv, (size_t)V, sizeof(kv_t), bb_rank_cmp);
  /* top-k: ranks whose key is below the k-th key leave (a prefix stays: keys equal to the threshold included) */
  int nk = V;
  if (topk > 0) {
    const int k = topk < V ? (int)topk : V;
    const float thr = kv[k - 1].key;
    nk = k;
    while (nk < V && !(kv[nk].key < thr)) ++nk;
  }
  const int C = (V + 31) / 32;
  float* e = (float*)malloc(sizeof(float) * (size_t)V);
  float* pr = (float*)malloc(sizeof(float) * (size_t)V);
  unsigned char* keep = (unsigned char*)malloc((size_t)V);
  for (int r = 0; r < V; ++r) e[r] = r < nk ? fb_exp(kv[r].key - kv[0].key) : 0.0f;
  float b[32], incl[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int j = 0; j < C; ++j) {
      const int r = l * C + j;
      if (r < V) s = s + e[r];
    }
    b[l] = s;
  }
  lane_scan(b, incl);
  const float S = incl[31];
  for (int r = 0; r < V; ++r) keep[r] = r < nk;
  if (topp < 1.0f) {
    float bp[32], inclp[32];
    for (int l = 0; l < 32; ++l) {
      float s = 0.0f;
      for (int j = 0; j < C; ++j) {
        const int r = l * C + j;
        if (r < V) {
          pr[r] = e[r] / S;
          s = s + pr[r];
        }
      }
      bp[l] = s;
    }
    lane_scan(bp, inclp);
    for (int l = 0; l < 32; ++l) {
      float run = l ? inclp[l - 1] : 0.0f;
      for (int j = 0; j < C; ++j) {
        const int r = l * C + j;
        if (r >= V) break;
        if (keep[r]) keep[r] = (r == 0) || !(run > topp);
        run = run + pr[r];
      }
    }
  }
  float b2[32], incl2[32];
  for (int l = 0; l < 32; ++l) {
    float s2 = 0.0f;
    for (int j = 0; j < C; ++j) {
      const int r = l * C + j;
      if (r < V && keep[r]) s2 = s2 + e[r];
    }
    b2[l] = s2;
  }
  lane_scan(b2, incl2);
  const float S2 = incl2[31];
  const int ok = !any_nan && isfinite(kv[0].key) && S2 > 0.0f && isfinite(S2);
  float best = -1.0f;
  int bidx = 0x7fffffff;
  for (int r = 0; r < V; ++r) {
    const int id = kv[r].idx;
    float sc;
    if (ok) {
      if (!keep[r]) continue;
      sc = (e[r] / S2) / q[id];
    } else {
      sc = 1.0f / q[id];
    }
    if (sc > best || (sc == best && id < bidx)) {
      best = sc;
      bidx = id;
    }
  }
  free(kv);
  free(e);
  free(pr);
  free(keep);
  if (ok_out) *ok_out = ok;
  return bidx;
}
