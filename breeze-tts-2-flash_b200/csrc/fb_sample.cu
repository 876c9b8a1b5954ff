// flashb: the backbone (codebook-0) sampler on the device, one CTA per row of CFG logits.
//
// Replaces the reference's host-sync-free torch sampler (flash/sampling.py:56-97 sample_logits, bitwise equal to the
// official models/cudagraph/sampling.py) that runs after every backbone step, with the same op order:
//   repetition penalty on the ids marked present (x > 0 ? x / p : x * p), suppressed ids -> -inf;
//   greedy: argmax (first index among equal maxima, a NaN counts as the maximum);
//   sampling: key = x / T; top-k keeps every key >= the k-th largest (duplicates counted); top-p over the keys in
//   rank order (cumulative softmax, shift-right removal, rank 0 kept); probs = softmax; the validity flag of the
//   official multinomial (every prob finite and >= 0, sum != 0); token = argmax(probs / q) with q ~ Exp(1) supplied
//   by the caller (torch.multinomial(p, 1) == argmax(p / Exp(1))), or argmax(1 / q) for an invalid row (the
//   reference then draws from all-ones weights).
// Rank order is (key descending, index ascending): a bitonic sort of 64-bit composite keys (order-preserving key bits
// above the complemented index) over the next power of two >= V in shared memory.  The exponential, the sums (32
// lanes over contiguous rank ranges, in-lane in rank order, Kogge-Stone scan) and the divisions are exactly those of
// oracle/sampler.c fb_bb_sample_row, so given the same logits and q the tokens and flags are bitwise equal.
#include "fb_sample.cuh"

namespace fb {

constexpr int BS_THREADS = 256;
constexpr int BS_MAXV = 4096;

struct BsArgs {
  const float* logits;
  long ld;
  int rows, V;
  unsigned char* present;     // [rows, V] or null
  long ldp;
  float penalty;
  const long long* suppress;
  int n_suppress;
  const float* temp;
  const long long* topk;
  const float* topp;
  const long long* dosample;
  const float* q;
  long ldq;
  long long* tokens;
  int pair_half;              // > 0: row r's token goes to both rows of its CFG pair (blocks of 2 pair_half rows)
  long long* ok;
  int mark_present;
};

// (value, index) of the better candidate: NaN first, then the larger value, then the lower index
__device__ __forceinline__ void greedy_pick(float& v, int& i, float v2, int i2) {
  const bool n1 = v != v, n2 = v2 != v2;
  const bool take = (n2 && !n1) || (n1 == n2 && (n1 ? i2 < i : (v2 > v || (v2 == v && i2 < i))));
  if (take) {
    v = v2;
    i = i2;
  }
}
// (score, index): the larger score, then the lower index
__device__ __forceinline__ void score_pick(float& s, int& i, float s2, int i2) {
  if (s2 > s || (s2 == s && i2 < i)) {
    s = s2;
    i = i2;
  }
}

__global__ void __launch_bounds__(BS_THREADS) cb0_sample_kernel(const BsArgs a) {
  extern __shared__ __align__(16) unsigned char bs_smem[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(bs_smem);   // [BS_MAXV] composite rank keys
  float* xs = reinterpret_cast<float*>(keys + BS_MAXV);   // [BS_MAXV] penalised logits, later the e_r of the ranks
  __shared__ float red_v[BS_THREADS / 32];
  __shared__ int red_i[BS_THREADS / 32];
  __shared__ int s_nan, s_nk;
  __shared__ float s_tot[3];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.V;
  const float* lg = a.logits + (size_t)r * a.ld;
  const unsigned char* pres = a.present ? a.present + (size_t)r * a.ldp : nullptr;
  for (int i = tid; i < V; i += BS_THREADS) {
    float x = lg[i];
    if (pres && pres[i] && a.penalty != 1.0f) x = x > 0.0f ? __fdiv_rn(x, a.penalty) : __fmul_rn(x, a.penalty);
    xs[i] = x;
  }
  if (tid == 0) s_nan = 0;
  __syncthreads();
  for (int j = tid; j < a.n_suppress; j += BS_THREADS) {
    const long long id = a.suppress[j];
    if (id >= 0 && id < V) xs[id] = -INFINITY;
  }
  __syncthreads();

  auto block_pick = [&](float v, int i, bool greedy) {
    // warp, then block reduction of (value, index) candidates; every thread gets the winner's index
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(FULL, v, o);
      const int i2 = __shfl_xor_sync(FULL, i, o);
      if (greedy) greedy_pick(v, i, v2, i2); else score_pick(v, i, v2, i2);
    }
    if (lane == 0) {
      red_v[warp] = v;
      red_i[warp] = i;
    }
    __syncthreads();
    float bv = red_v[0];
    int bi = red_i[0];
    for (int w = 1; w < BS_THREADS / 32; ++w) {
      if (greedy) greedy_pick(bv, bi, red_v[w], red_i[w]); else score_pick(bv, bi, red_v[w], red_i[w]);
    }
    __syncthreads();
    return bi;
  };

  const bool sample = a.dosample[r] != 0;
  int tok;
  int ok = 1;
  if (!sample) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int j = tid; j < V; j += BS_THREADS) greedy_pick(v, i, xs[j], j);
    tok = block_pick(v, i, true);
  } else {
    // ---- keys and their rank order
    const float T = a.temp[r];
    int N = 1;
    while (N < V) N <<= 1;
    for (int i = tid; i < N; i += BS_THREADS) {
      unsigned long long k = 0ull;
      if (i < V) {
        float key = __fdiv_rn(xs[i], T);
        if (key != key) {                  // torch ranks a NaN first and the softmax turns every prob to NaN
          s_nan = 1;
          key = -INFINITY;
        }
        k = ((unsigned long long)f2ord(key) << 32) | (unsigned long long)(0xffffffffu - (unsigned)i);
      }
      keys[i] = k;
    }
    __syncthreads();
    for (int size = 2; size <= N; size <<= 1) {           // bitonic sort, descending
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < N / 2; i += BS_THREADS) {
          const int lo = 2 * i - (i & (stride - 1));
          const int hi = lo + stride;
          const bool desc = (lo & size) == 0;
          const unsigned long long x = keys[lo], y = keys[hi];
          if ((x < y) == desc) {
            keys[lo] = y;
            keys[hi] = x;
          }
        }
        __syncthreads();
      }
    }
    auto key_at = [&](int rank) { return ord2f((unsigned)(keys[rank] >> 32)); };
    auto idx_at = [&](int rank) { return (int)(0xffffffffu - (unsigned)(keys[rank] & 0xffffffffull)); };
    // ---- top-k: the ranks with a key >= the k-th key (a prefix of the rank order)
    const long long tk = a.topk[r];
    if (tid == 0) s_nk = V;
    __syncthreads();
    if (tk > 0) {
      const int k = tk < V ? (int)tk : V;
      const float thr = key_at(k - 1);
      // first rank >= k whose key is below the threshold
      for (int i = k + tid; i < V; i += BS_THREADS)
        if (key_at(i) < thr && (i == k || !(key_at(i - 1) < thr))) s_nk = i;
      __syncthreads();
    }
    const int nk = s_nk;
    const float k0 = key_at(0);
    for (int i = tid; i < V; i += BS_THREADS) xs[i] = i < nk ? fb_exp_dev(__fsub_rn(key_at(i), k0)) : 0.0f;
    __syncthreads();
    // ---- the canonical sums (warp 0): lane l owns ranks [l C, l C + C)
    const float tp = a.topp[r];
    const int C = (V + 31) / 32;
    if (warp == 0) {
      float s = 0.0f;
      for (int j = 0; j < C; ++j) {
        const int rk = lane * C + j;
        if (rk < V) s = __fadd_rn(s, xs[rk]);
      }
      const float S = __shfl_sync(FULL, lane_scan(s), 31);
      unsigned rm[4] = {0u, 0u, 0u, 0u};      // bit j: rank lane C + j removed by top-p (C <= 128)
      if (tp < 1.0f) {
        float sp = 0.0f;
        for (int j = 0; j < C; ++j) {
          const int rk = lane * C + j;
          if (rk < V) sp = __fadd_rn(sp, __fdiv_rn(xs[rk], S));
        }
        const float incl = lane_scan(sp);
        const float prev = __shfl_up_sync(FULL, incl, 1);
        float run = lane ? prev : 0.0f;
        for (int j = 0; j < C; ++j) {
          const int rk = lane * C + j;
          if (rk >= V) break;
          if (rk < nk && !(rk == 0 || !(run > tp))) rm[j >> 5] |= 1u << (j & 31);
          run = __fadd_rn(run, __fdiv_rn(xs[rk], S));
        }
      }
      float s2 = 0.0f;
      for (int j = 0; j < C; ++j) {
        const int rk = lane * C + j;
        if (rk < nk && !((rm[j >> 5] >> (j & 31)) & 1u)) s2 = __fadd_rn(s2, xs[rk]);
      }
      const float S2 = __shfl_sync(FULL, lane_scan(s2), 31);
      // removed ranks: e_r -> 0 for the final scores (they cannot win: every kept score is > 0 when ok)
      for (int j = 0; j < C; ++j) {
        const int rk = lane * C + j;
        if (rk < V && ((rm[j >> 5] >> (j & 31)) & 1u)) xs[rk] = 0.0f;
      }
      if (lane == 0) {
        s_tot[0] = S;
        s_tot[1] = S2;
      }
    }
    __syncthreads();
    const float S2 = s_tot[1];
    ok = !s_nan && isfinite(k0) && S2 > 0.0f && isfinite(S2);
    float best = -1.0f;
    int bi = 0x7fffffff;
    const float* qr = a.q + (size_t)r * a.ldq;
    if (ok) {
      for (int rk = tid; rk < nk; rk += BS_THREADS) {
        if (xs[rk] == 0.0f && rk != 0) continue;          // removed by top-p (a kept e_r is > 0)
        const int id = idx_at(rk);
        score_pick(best, bi, __fdiv_rn(__fdiv_rn(xs[rk], S2), qr[id]), id);
      }
    } else {
      for (int i = tid; i < V; i += BS_THREADS) score_pick(best, bi, __fdiv_rn(1.0f, qr[i]), i);
    }
    tok = block_pick(best, bi, false);
  }
  if (tid == 0) {
    if (a.pair_half > 0) {
      const int h = a.pair_half, o = (r / h) * 2 * h + r % h;
      a.tokens[o] = tok;
      a.tokens[o + h] = tok;
    } else {
      a.tokens[r] = tok;
    }
    if (a.ok) a.ok[r] = ok;
    if (a.mark_present && a.present && tok >= 0 && tok < V) a.present[(size_t)r * a.ldp + tok] = 1;
  }
}

}  // namespace fb

extern "C" int flashb_cb0_sample(const float* logits, int64_t ld, int rows, int V, unsigned char* present,
                                 int64_t ldp, float repetition_penalty, const int64_t* suppress, int n_suppress,
                                 const float* temp, const int64_t* topk, const float* topp, const int64_t* dosample,
                                 const float* q, int64_t ldq, int64_t* tokens, int pair_half, int64_t* ok,
                                 int mark_present, void* stream) {
  using namespace fb;
  FB_CHECK_ARG(logits && temp && topk && topp && dosample && q && tokens, "cb0_sample: null pointer argument");
  FB_CHECK_ARG(rows >= 1 && rows <= 65535 && V >= 1 && V <= BS_MAXV && ld >= V && ldq >= V,
               "cb0_sample: rows %d, V %d (<= %d) or strides out of range", rows, V, BS_MAXV);
  FB_CHECK_ARG(!present || ldp >= V, "cb0_sample: presence-mask stride below V");
  FB_CHECK_ARG(n_suppress >= 0 && (n_suppress == 0 || suppress), "cb0_sample: suppress list");
  FB_CHECK_ARG(repetition_penalty > 0.0f, "cb0_sample: repetition penalty must be positive");
  FB_CHECK_ARG(pair_half >= 0 && (pair_half == 0 || rows % pair_half == 0),
               "cb0_sample: pair_half %d must divide rows %d", pair_half, rows);
  BsArgs a{};
  a.logits = logits; a.ld = (long)ld; a.rows = rows; a.V = V;
  a.present = present; a.ldp = (long)ldp; a.penalty = repetition_penalty;
  a.suppress = (const long long*)suppress; a.n_suppress = n_suppress;
  a.temp = temp; a.topk = (const long long*)topk; a.topp = topp; a.dosample = (const long long*)dosample;
  a.q = q; a.ldq = (long)ldq; a.tokens = (long long*)tokens; a.pair_half = pair_half;
  a.ok = (long long*)ok; a.mark_present = mark_present;
  void* args[] = {(void*)&a};
  const size_t smem = (size_t)BS_MAXV * (8 + 4);
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(cb0_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("cb0_sample: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = 1;
  }
  return fbh::launch_pdl((const void*)cb0_sample_kernel, dim3(rows), dim3(BS_THREADS), smem, (cudaStream_t)stream,
                         args, true);
}
