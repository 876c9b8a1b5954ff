// flashb: the two ends of the backbone decode step that the reference leaves to eager torch ops
// (flash/backbone.py:114-116 and :127-138; official UP/models/cudagraph/backbone_graph.py:254-285).
//
//   embed_rope   x[b] = bf16(sum_c table[ids[b, c] + c * vocab])  (BreezeBackboneModelEmbeddings,
//                UP/models/breeze.py:798-803: gather per codebook, fp32 accumulation in codebook order, one rounding)
//                + the cos/sin rows of position_ids[b] gathered from host-precomputed bf16 tables (the rotary module's
//                own fp32 cos/sin cast to bf16, UP/models/breeze.py:159-186).
//   lm_head_cfg  hidden = Qwen3RMSNorm(x) (bf16); logits = float(hidden) @ W32^T (fp32 lm_head); CFG combine
//                u + gs * (c - u) with three separately rounded fp32 ops.
// Both are small HBM streams (the lm_head reads V*H*4 bytes, 16.8 MB at the synthetic config): one warp per output
// row, 16-byte non-allocating loads with four in flight per lane.
#include "fb_common.cuh"

namespace fb {

__global__ void __launch_bounds__(256) embed_rope_kernel(const long long* __restrict__ ids, int C, int vocab,
                                                         const bf16* __restrict__ table, int H,
                                                         const long long* __restrict__ pos_ids,
                                                         const bf16* __restrict__ cos_tab,
                                                         const bf16* __restrict__ sin_tab, int D, int max_pos,
                                                         bf16* __restrict__ x_out, bf16* __restrict__ cos_out,
                                                         bf16* __restrict__ sin_out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const long long rows = (long long)C * vocab;
  for (int j = threadIdx.x * 8; j < H; j += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < C; ++c) {
      long long r = ids[(size_t)b * C + c] + (long long)c * vocab;
      r = r < 0 ? 0 : (r >= rows ? rows - 1 : r);
      float f[8];
      cvt8(ld_nc_v4(table + (size_t)r * H + j), f);
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] += f[t];
    }
    uint4 o;
    o.x = pack2(acc[0], acc[1]);
    o.y = pack2(acc[2], acc[3]);
    o.z = pack2(acc[4], acc[5]);
    o.w = pack2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(x_out + (size_t)b * H + j) = o;
  }
  long long p = pos_ids[b];
  p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
  for (int j = threadIdx.x * 8; j < D; j += blockDim.x * 8) {
    *reinterpret_cast<uint4*>(cos_out + (size_t)b * D + j) = *reinterpret_cast<const uint4*>(cos_tab + p * D + j);
    *reinterpret_cast<uint4*>(sin_out + (size_t)b * D + j) = *reinterpret_cast<const uint4*>(sin_tab + p * D + j);
  }
}

constexpr int LM_MAXB = 16;
constexpr int LM_THREADS = 256;

// grid = #SMs; each CTA normalises x (redundantly) into shared memory as fp32, then one warp per vocab row.
__global__ void __launch_bounds__(LM_THREADS) lm_head_cfg_kernel(const bf16* __restrict__ x, int B, int H,
                                                                 const bf16* __restrict__ nw, float eps,
                                                                 const float* __restrict__ W, int V,
                                                                 const float* __restrict__ gs,
                                                                 bf16* __restrict__ hidden_out,
                                                                 float* __restrict__ logits, float* __restrict__ cfg) {
  extern __shared__ __align__(16) float hs[];  // [B][H] fp32 values of the bf16 hidden state
  __shared__ float red[LM_THREADS / 32][LM_MAXB];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int b = 0; b < B; ++b) {
    float s = 0.f;
    for (int j = tid * 8; j < H; j += LM_THREADS * 8) {
      float f[8];
      cvt8(*reinterpret_cast<const uint4*>(x + (size_t)b * H + j), f);
#pragma unroll
      for (int t = 0; t < 8; ++t) s = fmaf(f[t], f[t], s);
    }
    s = warp_sum(s);
    if (lane == 0) red[warp][b] = s;
  }
  __syncthreads();
  for (int b = 0; b < B; ++b) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < LM_THREADS / 32; ++w) tot += red[w][b];
    const float r = 1.0f / sqrtf(tot / (float)H + eps);
    for (int j = tid * 8; j < H; j += LM_THREADS * 8) {
      float f[8], w8[8];
      cvt8(*reinterpret_cast<const uint4*>(x + (size_t)b * H + j), f);
      cvt8(*reinterpret_cast<const uint4*>(nw + j), w8);
      float y[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) y[t] = rbf(w8[t] * rbf(f[t] * r));
#pragma unroll
      for (int t = 0; t < 8; ++t) hs[(size_t)b * H + j + t] = y[t];
      if (blockIdx.x == 0) {
        uint4 o;
        o.x = pack2(y[0], y[1]);
        o.y = pack2(y[2], y[3]);
        o.z = pack2(y[4], y[5]);
        o.w = pack2(y[6], y[7]);
        *reinterpret_cast<uint4*>(hidden_out + (size_t)b * H + j) = o;
      }
    }
  }
  __syncthreads();
  const int half = B >= 2 ? B / 2 : 1;
  const float g = gs ? gs[0] : 1.0f;
  const int nw_total = gridDim.x * (LM_THREADS / 32);
  for (int v = blockIdx.x * (LM_THREADS / 32) + warp; v < V; v += nw_total) {
    const float* wr = W + (size_t)v * H;
    float acc[LM_MAXB];
#pragma unroll
    for (int b = 0; b < LM_MAXB; ++b) acc[b] = 0.f;
    for (int j = lane * 4; j < H; j += 128 * 4) {
      uint4 u[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (j + i * 128 < H) u[i] = ld_nc_v4(wr + j + i * 128);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (j + i * 128 >= H) break;
        const float w4[4] = {__uint_as_float(u[i].x), __uint_as_float(u[i].y), __uint_as_float(u[i].z),
                             __uint_as_float(u[i].w)};
#pragma unroll
        for (int b = 0; b < LM_MAXB; ++b) {
          if (b < B) {
            const float4 h4 = *reinterpret_cast<const float4*>(hs + (size_t)b * H + j + i * 128);
            acc[b] = fmaf(w4[0], h4.x, acc[b]);
            acc[b] = fmaf(w4[1], h4.y, acc[b]);
            acc[b] = fmaf(w4[2], h4.z, acc[b]);
            acc[b] = fmaf(w4[3], h4.w, acc[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < LM_MAXB; ++b)
      if (b < B) acc[b] = warp_sum(acc[b]);
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < LM_MAXB; ++b)
        if (b < B) logits[(size_t)b * V + v] = acc[b];
      if (B >= 2) {
#pragma unroll
        for (int hh = 0; hh < LM_MAXB / 2; ++hh) {
          if (hh < half) {
            const float c = acc[hh], u = acc[hh + half];
            const float d = __fsub_rn(c, u);
            cfg[(size_t)hh * V + v] = __fadd_rn(u, __fmul_rn(g, d));
          }
        }
      } else {
        cfg[v] = acc[0];
      }
    }
  }
}

// Per-step position update of the streaming loop, on device so a captured frame needs no host work: cache_pos += 1,
// position_ids[b] += 1 and the new slot of every mask row becomes valid (0).  This is what the reference's loop does
// on the host before each backbone replay (flash/main_loop.py:123-140; UP/models/cudagraph/backbone_graph.py:
// 239-252, 392-395).
__global__ void step_advance_kernel(long long* cache_pos, long long* position_ids, int B, void* mask, int mask_bf16,
                                    long m_sb, int S) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    const long long p = cache_pos[0] + 1;
    cache_pos[0] = p;
    for (int b = 0; b < B; ++b) {
      position_ids[b] += 1;
      if (p >= 0 && p < S) {
        if (mask_bf16) reinterpret_cast<bf16*>(mask)[(size_t)b * m_sb + p] = __float2bfloat16_rn(0.f);
        else reinterpret_cast<float*>(mask)[(size_t)b * m_sb + p] = 0.f;
      }
    }
  }
}

// Greedy branch of the backbone sampler (sample_logits with do_sample=False is torch.argmax,
// flash/sampling.py:56-97; UP/models/cudagraph/sampling.py): token = argmax(cfg[h, 0:n_valid]) with torch's
// semantics (first maximal index; a NaN counts as the maximum), ids >= n_valid suppressed as the reference suppresses
// the EOS / reserved ids with -inf.  Written to first_cb[h] and, for CFG pairs, first_cb[h + half].
__global__ void __launch_bounds__(256) cb0_greedy_kernel(const float* __restrict__ cfg, long ld, int half, int n_valid,
                                                         int B, long long* __restrict__ first_cb) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[8];
  __shared__ int si[8];
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = cfg + (size_t)h * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto better = [](float v, int i, float w, int j) {
    if (isnan(w)) return isnan(v) && i < j;
    if (isnan(v)) return true;
    return v > w || (v == w && i < j);
  };
  for (int i = tid; i < n_valid; i += blockDim.x) {
    const float v = row[i];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(FULL, bv, o);
    const int i = __shfl_xor_sync(FULL, bi, o);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    if (bi == 0x7fffffff) bi = 0;
    first_cb[h] = bi;
    if (B >= 2) first_cb[h + half] = bi;
  }
}

// Frame assembly of the streaming loop (flash/main_loop.py:268, 310-312: frame = [token, depth_tokens[0]], repeated
// for both CFG rows): ids[b, 0] = first_cb[b]; ids[b, c] = depth_tok[b, c - 1] for c = 1 .. C - 1.
__global__ void frame_ids_kernel(const long long* __restrict__ first_cb, const long long* __restrict__ depth_tok,
                                 int n_decode, int B, int C, long long* __restrict__ ids) {
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < B * C; i += blockDim.x) {
    const int b = i / C, c = i - b * C;
    ids[i] = c == 0 ? first_cb[b] : depth_tok[(size_t)b * n_decode + c - 1];
  }
}

}  // namespace fb

using namespace fb;

extern "C" int flashb_cb0_greedy(const float* cfg_logits, int64_t ld, int half, int n_valid, int B,
                                 int64_t* first_cb, void* stream) {
  FB_CHECK_ARG(cfg_logits && first_cb && half >= 1 && n_valid >= 1 && n_valid <= ld && (B == half || B == 2 * half),
               "cb0_greedy: bad argument (half=%d n_valid=%d ld=%lld B=%d)", half, n_valid, (long long)ld, B);
  long l = (long)ld;
  long long* fc = (long long*)first_cb;
  void* args[] = {(void*)&cfg_logits, (void*)&l, (void*)&half, (void*)&n_valid, (void*)&B, (void*)&fc};
  return fbh::launch_pdl((const void*)cb0_greedy_kernel, dim3(half), dim3(256), 0, (cudaStream_t)stream, args, true);
}

extern "C" int flashb_frame_ids(const int64_t* first_cb, const int64_t* depth_tok, int n_decode, int B, int C,
                                int64_t* ids, void* stream) {
  FB_CHECK_ARG(first_cb && depth_tok && ids && B >= 1 && C >= 1 && C - 1 <= n_decode,
               "frame_ids: bad argument (B=%d C=%d n_decode=%d)", B, C, n_decode);
  const long long* fc = (const long long*)first_cb;
  const long long* dt = (const long long*)depth_tok;
  long long* io = (long long*)ids;
  void* args[] = {(void*)&fc, (void*)&dt, (void*)&n_decode, (void*)&B, (void*)&C, (void*)&io};
  return fbh::launch_pdl((const void*)frame_ids_kernel, dim3(1), dim3(128), 0, (cudaStream_t)stream, args, true);
}

extern "C" int flashb_step_advance(int64_t* cache_pos, int64_t* position_ids, int B, void* mask, int mask_is_bf16,
                                   int64_t m_sb, int S, void* stream) {
  FB_CHECK_ARG(cache_pos && position_ids && mask && B >= 1 && S >= 1, "step_advance: bad argument");
  long long* cp = (long long*)cache_pos;
  long long* pp = (long long*)position_ids;
  long msb = (long)m_sb;
  void* args[] = {(void*)&cp, (void*)&pp, (void*)&B, (void*)&mask, (void*)&mask_is_bf16, (void*)&msb, (void*)&S};
  return fbh::launch_pdl((const void*)step_advance_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, args, true);
}

extern "C" int flashb_embed_rope(const int64_t* ids, int B, int C, int vocab, const void* table, int H,
                                 const int64_t* position_ids, const void* cos_tab, const void* sin_tab, int D,
                                 int max_pos, void* x_out, void* cos_out, void* sin_out, void* stream) {
  FB_CHECK_ARG(ids && table && position_ids && cos_tab && sin_tab && x_out && cos_out && sin_out,
               "embed_rope: null pointer argument");
  FB_CHECK_ARG(B >= 1 && C >= 1 && vocab >= 1 && H % 8 == 0 && D % 8 == 0 && max_pos >= 1,
               "embed_rope: bad shape B=%d C=%d vocab=%d H=%d D=%d", B, C, vocab, H, D);
  const long long* ip = (const long long*)ids;
  const bf16* tp = (const bf16*)table;
  const long long* pp = (const long long*)position_ids;
  const bf16* ct = (const bf16*)cos_tab;
  const bf16* stt = (const bf16*)sin_tab;
  bf16* xo = (bf16*)x_out;
  bf16* co = (bf16*)cos_out;
  bf16* so = (bf16*)sin_out;
  void* args[] = {(void*)&ip, (void*)&C, (void*)&vocab, (void*)&tp, (void*)&H, (void*)&pp, (void*)&ct,
                  (void*)&stt, (void*)&D, (void*)&max_pos, (void*)&xo, (void*)&co, (void*)&so};
  return fbh::launch_pdl((const void*)embed_rope_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, args, true);
}

// ------------------------------------------------------------------------------------------------ many-row lm_head
// logits[B, V] = float(hidden[B, H]) @ W32[V, H]^T for up to LMR_MAXB rows in one pass over the fp32 lm_head, and the
// CFG combine of every block of `block` rows laid out [cond_0 .. cond_{h-1}, uncond_0 .. uncond_{h-1}] (h = block / 2):
// cfg[blk * h + k] = u + gs * (c - u), three separately rounded fp32 ops.  hidden is the final-norm output (bf16).
// Tiled fp32 FMA on the CUDA cores (the lm_head is fp32, like the reference's): CTA = LMR_VT vocab rows x all B rows,
// K in chunks of LMR_KC columns double-buffered in shared memory by cp.async; thread = 2 vocab rows x 4 batch rows,
// 4 columns per shared-memory read.  Every output is one thread's fp32 sum in column order (deterministic).
constexpr int LMR_MAXB = 128;
constexpr int LMR_VT = 16;
constexpr int LMR_KC = 128;
constexpr int LMR_THREADS = 256;
constexpr int LMR_WP = LMR_KC + 4;         // fp32 row pitch of a W chunk (2-way bank spread of the 8 row pairs)
constexpr int LMR_HP = LMR_KC + 8;         // bf16 row pitch of a hidden chunk

__global__ void __launch_bounds__(LMR_THREADS) lm_head_rows_kernel(const bf16* __restrict__ hid, long ldh, int B,
                                                                   int H, const float* __restrict__ W, int V,
                                                                   const float* __restrict__ gs, int block,
                                                                   float* __restrict__ logits,
                                                                   float* __restrict__ cfg) {
  extern __shared__ __align__(16) unsigned char lmr_smem[];
  auto ws = reinterpret_cast<float(*)[LMR_VT][LMR_WP]>(lmr_smem);                          // [2][VT][WP]
  auto hs = reinterpret_cast<bf16(*)[LMR_MAXB][LMR_HP]>(lmr_smem + 2 * sizeof(float) * LMR_VT * LMR_WP);
  auto outs = reinterpret_cast<float(*)[LMR_VT + 1]>(ws);    // after the K loop: [B][VT + 1] over the W chunks
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  const int v0 = blockIdx.x * LMR_VT;
  const int vb = tid & 7, bb = tid >> 3;        // vocab rows v0 + 2 vb (+1), batch rows 4 bb .. 4 bb + 3
  const int nk = (H + LMR_KC - 1) / LMR_KC;
  auto stage = [&](int kc, int buf) {
    const int k0 = kc * LMR_KC;
    // W: LMR_VT rows x LMR_KC fp32 = 512 16-byte units; hidden: B rows x LMR_KC bf16 = B x 16 units
    for (int i = tid; i < LMR_VT * (LMR_KC / 4); i += LMR_THREADS) {
      const int r = i / (LMR_KC / 4), u = i - r * (LMR_KC / 4);
      const int v = min(v0 + r, V - 1), k = k0 + 4 * u;
      if (k < H) cp_async16(&ws[buf][r][4 * u], W + (size_t)v * H + k);
    }
    for (int i = tid; i < B * (LMR_KC / 8); i += LMR_THREADS) {
      const int r = i / (LMR_KC / 8), u = i - r * (LMR_KC / 8);
      const int k = k0 + 8 * u;
      if (k < H) cp_async16(&hs[buf][r][8 * u], hid + (size_t)r * ldh + k);
    }
    cp_async_commit();
  };
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  stage(0, 0);
  for (int kc = 0; kc < nk; ++kc) {
    if (kc + 1 < nk) {
      stage(kc + 1, (kc + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int buf = kc & 1, kw = min(LMR_KC, H - kc * LMR_KC);
    for (int k = 0; k < kw; k += 4) {
      const float4 w0 = *reinterpret_cast<const float4*>(&ws[buf][2 * vb][k]);
      const float4 w1 = *reinterpret_cast<const float4*>(&ws[buf][2 * vb + 1][k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int b = 4 * bb + j;
        const uint2 hv = *reinterpret_cast<const uint2*>(&hs[buf][b < B ? b : 0][k]);
        const float h0 = lo_f(hv.x), h1 = hi_f(hv.x), h2 = lo_f(hv.y), h3 = hi_f(hv.y);
        float s0 = acc[0][j], s1 = acc[1][j];
        s0 = fmaf(w0.x, h0, s0); s0 = fmaf(w0.y, h1, s0); s0 = fmaf(w0.z, h2, s0); s0 = fmaf(w0.w, h3, s0);
        s1 = fmaf(w1.x, h0, s1); s1 = fmaf(w1.y, h1, s1); s1 = fmaf(w1.z, h2, s1); s1 = fmaf(w1.w, h3, s1);
        acc[0][j] = s0;
        acc[1][j] = s1;
      }
    }
    __syncthreads();
  }
  static_assert(LMR_MAXB * (LMR_VT + 1) <= 2 * LMR_VT * LMR_WP, "outs must fit over the W chunks");
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = 4 * bb + j, v = v0 + 2 * vb + i;
      if (b < B) {
        outs[b][2 * vb + i] = acc[i][j];
        if (v < V) logits[(size_t)b * V + v] = acc[i][j];
      }
    }
  __syncthreads();
  if (!cfg) return;
  // CFG of every block: one thread per (pair, vocab row of the tile)
  const float g = gs ? gs[0] : 1.0f;
  const int h = block >= 2 ? block / 2 : 1;
  const int npair = block >= 2 ? (B / block) * h : B;
  for (int i = tid; i < npair * LMR_VT; i += LMR_THREADS) {
    const int pr = i / LMR_VT, vv = i - pr * LMR_VT, v = v0 + vv;
    if (v >= V) continue;
    float r;
    if (block >= 2) {
      const int blk = pr / h, k = pr - blk * h;
      const float c = outs[blk * block + k][vv], u = outs[blk * block + h + k][vv];
      r = __fadd_rn(u, __fmul_rn(g, __fsub_rn(c, u)));
    } else {
      r = outs[pr][vv];
    }
    cfg[(size_t)pr * V + v] = r;
  }
}

extern "C" int flashb_lm_head_cfg(const void* x, int B, int H, const void* norm_w, float eps, const float* W32,
                                  int V, const float* gs, void* hidden_out, float* logits, float* cfg_out,
                                  void* stream) {
  FB_CHECK_ARG(x && norm_w && W32 && hidden_out && logits && cfg_out, "lm_head_cfg: null pointer argument");
  FB_CHECK_ARG(B >= 1 && B <= LM_MAXB && H % 8 == 0 && V >= 1, "lm_head_cfg: bad shape B=%d H=%d V=%d", B, H, V);
  FB_CHECK_ARG(B == 1 || gs, "lm_head_cfg: guidance scale pointer required for B >= 2");
  const size_t smem = (size_t)B * H * 4;
  FB_CHECK_ARG(smem <= 200 * 1024, "lm_head_cfg: B*H too large");
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_done[dev] < (int)smem) {
    cudaError_t e = cudaFuncSetAttribute(lm_head_cfg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("lm_head_cfg: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = (int)smem;
  }
  const bf16* xp = (const bf16*)x;
  const bf16* np = (const bf16*)norm_w;
  bf16* ho = (bf16*)hidden_out;
  void* args[] = {(void*)&xp, (void*)&B, (void*)&H, (void*)&np, (void*)&eps, (void*)&W32, (void*)&V,
                  (void*)&gs, (void*)&ho, (void*)&logits, (void*)&cfg_out};
  return fbh::launch_pdl((const void*)lm_head_cfg_kernel, dim3(fbh::grid_sms()), dim3(LM_THREADS), smem,
                         (cudaStream_t)stream, args, true);
}

namespace {
int lm_head_rows_launch(const bf16* hp, long ldh, int B, int H, const float* W32, int V, const float* gs, int block,
                        float* logits, float* cfg_out, cudaStream_t st) {
  void* args[] = {(void*)&hp, (void*)&ldh, (void*)&B, (void*)&H, (void*)&W32, (void*)&V, (void*)&gs, (void*)&block,
                  (void*)&logits, (void*)&cfg_out};
  const size_t smem = 2 * sizeof(float) * LMR_VT * LMR_WP + 2 * sizeof(bf16) * LMR_MAXB * LMR_HP;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(lm_head_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      fbh::set_msg("lm_head_rows: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return FB_ERR_CUDA;
    }
    attr_done[dev] = 1;
  }
  return fbh::launch_pdl((const void*)lm_head_rows_kernel, dim3((V + LMR_VT - 1) / LMR_VT), dim3(LMR_THREADS), smem, st,
                         args, true);
}
}  // namespace

// Final norm + lm_head + CFG for B rows in blocks of `block` rows (each laid out [cond.., uncond..]): the norm as the
// standalone RMSNorm (hidden_out), then one pass of lm_head_rows_kernel over the fp32 lm_head for every row.
extern "C" int flashb_lm_head_cfg_blocks(const void* x, int B, int H, const void* norm_w, float eps, const float* W32,
                                         int V, const float* gs, int block, void* hidden_out, float* logits,
                                         float* cfg_out, void* stream) {
  FB_CHECK_ARG(x && norm_w && W32 && hidden_out && logits && cfg_out, "lm_head_cfg_blocks: null pointer argument");
  FB_CHECK_ARG(B >= 1 && B <= LMR_MAXB && H % 8 == 0 && V >= 1, "lm_head_cfg_blocks: bad shape B=%d H=%d V=%d", B, H,
               V);
  FB_CHECK_ARG(block >= 1 && B % block == 0 && (block == 1 || block % 2 == 0),
               "lm_head_cfg_blocks: block %d must divide B = %d and be 1 or even", block, B);
  FB_CHECK_ARG(block == 1 || gs, "lm_head_cfg_blocks: guidance scale pointer required for CFG blocks");
  FB_CHECK_ARG(((uintptr_t)W32 & 15) == 0 && ((uintptr_t)hidden_out & 15) == 0 && H % 4 == 0,
               "lm_head_cfg_blocks: 16-byte aligned lm_head and hidden rows required");
  int rc = flashb_rmsnorm(x, H, B, H, norm_w, eps, hidden_out, H, stream);
  if (rc) return rc;
  return lm_head_rows_launch((const bf16*)hidden_out, H, B, H, W32, V, gs, block, logits, cfg_out,
                             (cudaStream_t)stream);
}

// Plain fp32 lm_head of B already normalised rows at row stride ldh (the prefill's last tokens).
extern "C" int flashb_lm_head_rows(const void* hidden, int64_t ldh, int B, int H, const float* W32, int V,
                                   float* logits, void* stream) {
  FB_CHECK_ARG(hidden && W32 && logits, "lm_head_rows: null pointer argument");
  FB_CHECK_ARG(B >= 1 && B <= LMR_MAXB && H % 8 == 0 && V >= 1 && ldh >= H && ldh % 8 == 0,
               "lm_head_rows: bad shape B=%d H=%d V=%d ldh=%lld", B, H, V, (long long)ldh);
  FB_CHECK_ARG(((uintptr_t)W32 & 15) == 0 && ((uintptr_t)hidden & 15) == 0 && H % 4 == 0,
               "lm_head_rows: 16-byte aligned lm_head and hidden rows required");
  return lm_head_rows_launch((const bf16*)hidden, (long)ldh, B, H, W32, V, nullptr, 1, logits, nullptr,
                             (cudaStream_t)stream);
}

// ------------------------------------------------------------------------------------------------ LN12 decode
// LN12 (the reference's lossless 12-bit weight storage, flash/ln12_format.py; layout in include/flashb.h) to bf16,
// HBM to HBM.  One warp per (row n, 1024-column group g): lane l reads its three 16-byte units of the group (low
// bytes of chunks 0-3 and their nibble words, 512-byte coalesced rows), forms the high byte of each of its 32
// values from the row's shifted 8-entry table and the sign bit, and writes 8 consecutive bf16 of each chunk
// (k = 1024 g + 256 c + 8 l + j).  Then, after a warp barrier, the row's patches in this group overwrite the high
// byte of their value exactly (the first three from the row record, the rest from the overflow list).
namespace {
__global__ void __launch_bounds__(256) ln12_decode_kernel(const unsigned char* __restrict__ data,
                                                          const uint4* __restrict__ meta,
                                                          const uint32_t* __restrict__ ovf, uint32_t lut_lo,
                                                          uint32_t lut_hi, int N, int K, bf16* __restrict__ out,
                                                          long ldo) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int G = K >> 10;
  const long w = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (long)N * G) return;
  const int n = (int)(w / G), g = (int)(w - (long)n * G);
  const unsigned char* grp = data + ((size_t)n * G + g) * 1536;
  const uint4 s0 = __ldcs(reinterpret_cast<const uint4*>(grp) + lane);
  const uint4 s1 = __ldcs(reinterpret_cast<const uint4*>(grp + 512) + lane);
  const uint4 s2 = __ldcs(reinterpret_cast<const uint4*>(grp + 1024) + lane);
  const uint4 rec = meta[n];
  const uint32_t hdr = rec.x;
  const int cnt = (int)(hdr & 1023u), ooff = (int)(hdr >> 13);
  const int sh = (int)((hdr >> 10) & 7u) - (((hdr >> 10) & 4u) ? 8 : 0);
  // the row's table: every entry + sh (the encoder keeps shifted entries inside 0..127, so no byte carries)
  const uint32_t add = (uint32_t)sh * 0x01010101u;
  const uint32_t t_lo = lut_lo + add, t_hi = lut_hi + add;
  const uint32_t lows[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};   // chunk c: words 2c, 2c + 1
  const uint32_t words[4] = {s2.x, s2.y, s2.z, s2.w};
  bf16* row = out + (size_t)n * ldo + (size_t)g * 1024 + lane * 8;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t wd = words[c];
    uint32_t o[4];
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      uint32_t pair = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * jp + h;
        const uint32_t ix = (wd >> (4 * j)) & 7u;
        const uint32_t sign = (wd >> (j < 4 ? 8 * j + 7 : 8 * (j - 4) + 3)) & 1u;
        const uint32_t e = ((ix < 4 ? t_lo >> (8 * ix) : t_hi >> (8 * (ix - 4))) & 0x7Fu) | (sign << 7);
        const uint32_t lo = (lows[2 * c + (j >> 2)] >> (8 * (j & 3))) & 0xFFu;
        pair |= ((e << 8) | lo) << (16 * h);
      }
      o[jp] = pair;
    }
    *reinterpret_cast<uint4*>(row + c * 256) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (cnt == 0) return;
  __syncwarp();                     // the warp's decoded values are written before a patch overwrites one
  for (int p = lane; p < cnt; p += 32) {
    const uint32_t v = p == 0 ? rec.y : (p == 1 ? rec.z : (p == 2 ? rec.w : ovf[ooff + p - 3]));
    const int k = (int)(v >> 8);
    if ((k >> 10) != g) continue;
    const int kk = k & 1023, c = kk >> 8, l = (kk >> 3) & 31, j = kk & 7;
    const unsigned char lo = grp[(c >> 1) * 512 + l * 16 + (c & 1) * 8 + j];
    reinterpret_cast<unsigned short*>(out + (size_t)n * ldo)[k] = (unsigned short)(((v & 0xFFu) << 8) | lo);
  }
}
}  // namespace

extern "C" int flashb_ln12_decode(const void* data, const void* meta, const void* ovf, uint32_t lut_lo,
                                  uint32_t lut_hi, int N, int K, void* out, int64_t ldo, void* stream) {
  FB_CHECK_ARG(data && meta && out && N >= 1 && K >= 1024 && K % 1024 == 0 && ldo >= K && ldo % 8 == 0,
               "ln12_decode: bad arguments (N=%d K=%d ldo=%lld)", N, K, (long long)ldo);
  FB_CHECK_ARG(((uintptr_t)data & 15) == 0 && ((uintptr_t)meta & 15) == 0 && ((uintptr_t)out & 15) == 0,
               "ln12_decode: data, meta and out must be 16-byte aligned");
  const unsigned char* dp = (const unsigned char*)data;
  const uint4* mp = (const uint4*)meta;
  const uint32_t* op = (const uint32_t*)ovf;
  bf16* outp = (bf16*)out;
  long l = (long)ldo;
  const long warps = (long)N * (K / 1024);
  void* args[] = {(void*)&dp, (void*)&mp, (void*)&op, (void*)&lut_lo, (void*)&lut_hi, (void*)&N, (void*)&K,
                  (void*)&outp, (void*)&l};
  return fbh::launch_pdl((const void*)ln12_decode_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0,
                         (cudaStream_t)stream, args, true);
}
