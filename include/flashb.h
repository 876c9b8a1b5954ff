/* flashb: C ABI of the B200 (sm_100a) kernels for the Breeze-TTS-2 streaming-decode hot path.
 *
 * Every entry point takes raw device pointers, element strides and sizes, launches on the given CUDA stream
 * (a cudaStream_t passed as void*; NULL = legacy default stream) and returns FB_OK or an FB_ERR_* code; the message
 * of the last failure on the calling thread is flashb_last_error().  No entry point allocates device memory or
 * synchronises the stream (flashb_device_error excepted), so all of them can be captured in a CUDA graph.  bf16
 * arguments are IEEE bfloat16 bit patterns (uint16); fp32 arguments are float.
 *
 * The reference binds the same operations as pybind11 functions of JIT-built torch extensions; each declaration
 * cites the reference function it replaces (paths relative to the reference project root).
 */
#ifndef FLASHB_H
#define FLASHB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FB_OK = 0,
  FB_ERR_ARG = 1,         /* invalid pointer, shape, stride or alignment */
  FB_ERR_CUDA = 2,        /* a CUDA runtime call failed (launch, attribute, occupancy) */
  FB_ERR_UNSUPPORTED = 3, /* valid but not built: head_dim != 128, group size not in {1,2,4,8}, M > 8 ... */
  FB_ERR_STATE = 4,       /* object not initialised / used on another device */
  FB_ERR_TIMEOUT = 5,     /* a device-side wait ran out of time (reported through flashb_device_error) */
  FB_ERR_DEVICE = 6,      /* the device reported an error */
  FB_ERR_ABORTED = 7      /* a persistent kernel stopped at a barrier because its abort flag was set: by another
                           * CTA whose bounded wait expired, or by the host (reported through flashb_device_error) */
};

/* ---------------------------------------------------------------------------------------------- library */
const char* flashb_last_error(void);
const char* flashb_version(void);
/* Reads (and with clear != 0 resets) the device error word of the current device: 0 or an FB_ERR_* code set by a
 * kernel whose bounded wait expired.  Synchronises the device.  No reference counterpart (the reference's spin
 * barriers are unbounded, flash/csrc/depth_common.cuh:52-65). */
int flashb_device_error(int clear);
/* Which kernel the calling thread's last GEMV call launched: 0 = the scalar-FMA fallback (K % 64 != 0),
 * 1 = the mma.sync weight stream, 2 = the tcgen05 kernel (enough 128-row blocks for the grid); -1 before any.
 * For tests and profiling; no reference counterpart. */
int flashb_gemv_last_path(void);
/* Which kernel the calling thread's last fused decode attention launched: 0 = the split-KV scalar kernel, 1 = the
 * tensor-core kernel (one CTA per row and KV head, when the rows alone fill the grid); -1 before any.  For tests;
 * no reference counterpart. */
int flashb_attn_last_path(void);
/* CTAs per 128-row block of the calling thread's last tcgen05 GEMV launch: 1, or S >= 2 when the block's K range
 * was split over a thread-block cluster of S CTAs (too few blocks for the grid).  For tests; no reference
 * counterpart. */
int flashb_gemv_last_split(void);
/* Split K over a cluster also for M <= 16 rows (1) or not (0, the default: the mma.sync kernel is faster there on
 * a whole B200).  Process-wide; no reference counterpart. */
void flashb_set_gemv_split(int enable);
/* Activation rows per row group of the tcgen05 GEMV when M > 16: 16, 32, 64 (the default) or 128.  The groups
 * run side by side, each on an equal share of the SMs, and read the same weight tiles at about the same time, so
 * that L2 serves all but the first read; wider groups read each tile for more rows (the MMA's N).  Process-wide;
 * no reference counterpart. */
int flashb_set_gemv_group_rows(int rows);
/* Timeline of the tcgen05 GEMV launches issued after this call (null: off, the default): CTA c of a launch writes 8
 * uint64 at buf[8 c] -- %globaltimer ns at entry, producer past the dependent-launch wait, first stage in, last MMA
 * committed, epilogue done, split-K reduction done, exit -- and its SM id.  buf must hold 8 x the launch's CTAs;
 * each launch overwrites it.  Process-wide diagnostic; no reference counterpart. */
void flashb_set_gemv_trace(void* buf);
/* The many-rows tcgen05 GEMV (17..128 rows, no norm: activation rows as the MMA's M side, split K over a cluster)
 * on (1, the default) or off (0: those calls take the row-group kernel).  Process-wide; no reference counterpart. */
void flashb_set_gemv_rows_path(int enable);
/* Programmatic dependent launch on (1, default) / off (0) for all later launches of this process. */
void flashb_set_pdl(int enable);
/* SM budget of the calling host thread (0, the default: every SM).  Launches issued later by this thread -- directly
 * or while it captures a CUDA graph -- size their grids for at most `sms` SMs (persistent GEMV and LM-head grids,
 * decode-attention split counts, depth-frame grids when fb_dd_config.grid is 0), so that work on two streams, each
 * sized for part of the GPU, runs side by side instead of queueing for SMs.  The kernels are latency-bound at these
 * sizes, which makes two half-GPU lanes faster in aggregate than one whole-GPU lane.  No reference counterpart
 * (the reference decodes one request at a time). */
void flashb_set_sm_budget(int sms);
/* The grid size (SMs) the calling thread's launches use now. */
int flashb_sm_budget(void);

/* ---------------------------------------------------------------------------------------------- decode attention
 * Replaces attn_decode (flash/csrc/bb_attn.cu:416-429): GQA single-token attention of q [B, NH, 1, D] over the
 * static KV cache kc/vc [B, NKV, S, D] (position stride D, element strides c_sb/c_sh for batch/head) with the
 * additive mask [B|1, 1, 1, >=S] (bf16 if mask_is_bf16 else fp32; m_sb = 0 broadcasts one row).  Keys whose mask is
 * <= -1e30 contribute nothing; a row with no valid key gives 0.  out [B, 1, NH, D] bf16 contiguous.
 * ws / ws_floats / counters: the reference's workspace arguments, kept in the signature and unused (may be NULL):
 * the split-KV partials are merged inside each thread-block cluster through distributed shared memory, so
 * flashb_attn_ws_floats() returns 0.  D must be 128; NH / NKV in {1, 2, 4, 8}. */
int64_t flashb_attn_ws_floats(int B, int NH, int NKV, int S, int D);
int flashb_attn_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* kc, const void* vc, int64_t c_sb,
                       int64_t c_sh, int B, int NH, int NKV, int S, int D, const void* mask, int mask_is_bf16,
                       int64_t m_sb, float scaling, float* ws, int64_t ws_floats, int32_t* counters, void* out,
                       void* stream);

/* Replaces attn_decode_fused (flash/csrc/bb_attn.cu:433-460): qkv [B, (NH + 2 NKV) * D] raw q|k|v projections
 * (row stride qkv_sb); Qwen3 q_norm/k_norm (weights qn_w/kn_w [D], eps) + RoPE with cos/sin [B, 1, D] bf16 (row
 * stride cs_sb); writes the new k (normed, roped) and v at slot cache_pos[0] (device int64) of kc/vc, then attends
 * over slots [0, min(S, cache_pos + 1)) under the mask.  Launched with programmatic dependent launch, the kernel
 * reads cache_pos, the norm weights, cos/sin and the mask before the previous kernel in the stream has finished;
 * only qkv may come from that previous kernel.  The others must be written at least two launches earlier (as
 * embed_rope and step_advance are in the decode step), on the host, or by a kernel that does not allow dependent
 * launch (flashb_set_pdl(0) turns dependent launch off). */
int flashb_attn_decode_fused(const void* qkv, int64_t qkv_sb, const void* qn_w, const void* kn_w, float eps,
                             const void* cos, const void* sin, int64_t cs_sb, void* kc, void* vc, int64_t c_sb,
                             int64_t c_sh, int B, int NH, int NKV, int S, int D, const void* mask, int mask_is_bf16,
                             int64_t m_sb, const int64_t* cache_pos, float scaling, float* ws, int64_t ws_floats,
                             int32_t* counters, void* out, void* stream);

/* ---------------------------------------------------------------------------------------------- fused GEMVs
 * y[m, n] = sum_k xin[m, k] * W[n, k], nn.Linear layout (W [N, K] bf16 row-major contiguous), fp32 accumulation,
 * M = 1..2^20 rows (the reference: 1..8; more than 128 rows -- the prefill's dense GEMMs -- run in tiles of 128; x row stride ldx, y row stride ldy, both multiples of 8 elements),
 * K % 8 == 0.  All pointers 16-byte aligned.  More than 16 rows run on the tcgen05 kernel (K % 64 == 0), which then
 * streams the weights once for all rows; otherwise in row blocks (16 rows, or 8 / 4 / 2 / 1 when K % 64 != 0). */
/* Replaces gemv_seg (flash/csrc/bb_fused.cu:293-316): y[:, 0:N0+N1+N2] = norm?(x) @ [W0; W1; W2]^T, where norm is
 * the eager Qwen3 RMSNorm with weight nw [K] when nw != NULL.  W1/W2 may be NULL with N1/N2 = 0. */
int flashb_gemv_seg(const void* x, int64_t ldx, int M, int K, const void* nw, float eps, const void* W0, int N0,
                    const void* W1, int N1, const void* W2, int N2, void* y, int64_t ldy, void* stream);
/* Replaces gemv_resid (flash/csrc/bb_fused.cu:319-335): y = bf16(res + bf16(x @ W^T)); res row stride ldr. */
int flashb_gemv_resid(const void* x, int64_t ldx, int M, int K, const void* W, int N, const void* res, int64_t ldr,
                      void* y, int64_t ldy, void* stream);
/* Replaces gemv_gateup (flash/csrc/bb_fused.cu:338-356): act = bf16(bf16(silu(bf16(n @ Wg^T))) * bf16(n @ Wu^T)),
 * n = RMSNorm(x; nw, eps), or n = x when nw == NULL (rows normalised beforehand); Wg, Wu [N, K]. */
int flashb_gemv_gateup(const void* x, int64_t ldx, int M, int K, const void* nw, float eps, const void* Wg,
                       const void* Wu, int N, void* y, int64_t ldy, void* stream);
/* Replaces rmsnorm (flash/csrc/bb_fused.cu:358-368): y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))). */
int flashb_rmsnorm(const void* x, int64_t ldx, int M, int K, const void* w, float eps, void* y, int64_t ldy,
                   void* stream);

/* ---------------------------------------------------------------------------------------------- backbone step ends
 * Replaces the eager embedding and rotary ops of the decode step (flash/backbone.py:114-116; official
 * UP/models/cudagraph/backbone_graph.py:257-268, UP = third_party/breeze-tts): x[b] = bf16(sum_c table[ids[b, c] +
 * c * vocab]) over C codebooks (table [C * vocab, H] bf16, ids [B, C] int64 contiguous), and cos/sin rows [B, D]
 * gathered from the precomputed bf16 tables [max_pos, D] at position_ids[b] (int64, clamped to [0, max_pos)). */
int flashb_embed_rope(const int64_t* ids, int B, int C, int vocab, const void* table, int H,
                      const int64_t* position_ids, const void* cos_tab, const void* sin_tab, int D, int max_pos,
                      void* x_out, void* cos_out, void* sin_out, void* stream);
/* Replaces the final norm, the fp32 lm_head and CFG (flash/backbone.py:127-138): hidden = RMSNorm(x; norm_w, eps)
 * [B, H] bf16; logits[b] = float(hidden[b]) @ W32^T (W32 [V, H] fp32); for B >= 2, cfg[h] = u + gs * (c - u) with
 * c = logits[h], u = logits[h + B/2] (three separately rounded fp32 ops), else cfg = logits[0].  gs: device fp32
 * scalar. */
int flashb_lm_head_cfg(const void* x, int B, int H, const void* norm_w, float eps, const float* W32, int V,
                       const float* gs, void* hidden_out, float* logits, float* cfg_out, void* stream);
/* flashb_lm_head_cfg for B <= 128 rows in CFG blocks of `block` rows (1, or an even divisor of B), each block laid
 * out [cond_0 .. cond_{h-1}, uncond_0 .. uncond_{h-1}] (h = block / 2): the final RMSNorm of every row
 * (hidden_out [B, H] bf16, contiguous), logits [B, V] fp32 in one pass over the fp32 lm_head, and
 * cfg_out[blk * h + k] = u + gs (c - u) for every block (block 1: cfg_out = logits).  No reference counterpart as a
 * kernel: the reference runs one CFG pair per graph (flash/backbone.py:127-138); this serves many streams' pairs
 * decoded as one batch. */
int flashb_lm_head_cfg_blocks(const void* x, int B, int H, const void* norm_w, float eps, const float* W32, int V,
                              const float* gs, int block, void* hidden_out, float* logits, float* cfg_out,
                              void* stream);

/* Device-side per-frame position update of the streaming loop (the host-side cache_position / position_ids /
 * _set_attention_mask updates of flash/main_loop.py:123-140 and UP/models/cudagraph/backbone_graph.py:239-252,
 * 392-395): cache_pos[0] += 1; position_ids[b] += 1; mask[b * m_sb + cache_pos[0]] = 0 for every row b. */
int flashb_step_advance(int64_t* cache_pos, int64_t* position_ids, int B, void* mask, int mask_is_bf16, int64_t m_sb,
                        int S, void* stream);

/* Greedy backbone sampler: the do_sample=False branch of the reference's host-sync-free sample_logits
 * (flash/sampling.py:56-97, bitwise the official UP/models/cudagraph/sampling.py), i.e. torch.argmax of the CFG logits,
 * with every id >= n_valid suppressed (the reference's suppress_idx / EOS handling, flash/main_loop.py:98-108).
 * cfg_logits [half, ld] fp32; the token goes to first_cb[h] and, when B == 2 * half, first_cb[h + half]. */
int flashb_cb0_greedy(const float* cfg_logits, int64_t ld, int half, int n_valid, int B, int64_t* first_cb,
                      void* stream);

/* The backbone sampler (codebook 0): replaces the reference's host-sync-free sample_logits (flash/sampling.py:56-97,
 * bitwise the official models/cudagraph/sampling.py) with one CTA per row of logits [rows, ld] fp32 (V <= 4096):
 * repetition penalty on the ids marked in present [rows, ldp] (uint8, or NULL; x > 0 ? x / p : x * p), the
 * `suppress` ids -> -inf, then per row: dosample == 0 -> argmax (first index, NaN first); else key = x / temp,
 * top-k (topk > 0: keys below the k-th largest -> -inf, ties kept), top-p (topp < 1), softmax, token =
 * argmax(probs / q) with q [rows, ldq] fp32 Exp(1) draws (torch.multinomial(probs, 1) == argmax(probs / Exp(1))).
 * ok[row] (or NULL) = the official multinomial's validity predicate (every prob finite and >= 0, sum != 0); an invalid
 * row samples from all-ones weights, argmax(1 / q), as the reference's sanitised multinomial does.  Per-row
 * parameters temp/topp fp32 and topk/dosample int64 [rows].  pair_half == 0: tokens [rows] int64; pair_half = h > 0:
 * the rows are CFG pairs of blocks laid out [cond_0 .. cond_{h-1}, uncond_0 .. uncond_{h-1}] (the backbone's input
 * ids), and row r's token goes to tokens[(r / h) 2h + r % h] and tokens[(r / h) 2h + h + r % h].  mark_present != 0
 * then marks each token in `present` (the token history of the next frame).  Graph-capturable; no host sync. */
int flashb_cb0_sample(const float* logits, int64_t ld, int rows, int V, unsigned char* present, int64_t ldp,
                      float repetition_penalty, const int64_t* suppress, int n_suppress, const float* temp,
                      const int64_t* topk, const float* topp, const int64_t* dosample, const float* q, int64_t ldq,
                      int64_t* tokens, int pair_half, int64_t* ok, int mark_present, void* stream);

/* Frame assembly of the streaming loop (flash/main_loop.py:268 and :310-312): the backbone input of the next step is
 * ids[b] = [first_cb[b], depth_tok[b, 0 .. C-2]] (ids [B, C] int64, depth_tok [B, n_decode] int64, C - 1 <= n_decode),
 * built on the device instead of by torch.cat / repeat. */
int flashb_frame_ids(const int64_t* first_cb, const int64_t* depth_tok, int n_decode, int B, int C, int64_t* ids,
                     void* stream);

/* Replaces the backbone prefill attention (flash/prefill_attn.py:15-46 bz_prefill_attention -> the eager
 * transformers attention, UP/models/breeze.py:259-286) with a tcgen05 kernel: causal GQA attention of
 * q [B, NH, L, 128] over k/v [B, NKV, S, 128] (bf16; strides per batch / head / position in elements, multiples of
 * 8, position strides at least 128, 16-byte aligned base; q, k and v are read by TMA tensor copies through maps
 * encoded per call and cached per base and shape) with the eager rounding points s = bf16(bf16(q k^T) * scaling), s = bf16(s + mask),
 * p = bf16(softmax_fp32(s)), out = bf16(p v).  mask: additive [B | 1, 1, L, S] (bf16 if mask_is_bf16, else fp32;
 * m_sb = 0 broadcasts one mask), or NULL.  causal != 0 promises that every key j > i is masked for query i (the
 * reference's prefill mask), so key tiles above the diagonal are skipped (they carry probability exactly 0).
 * Computes q heads [h0, h1) only (a head-group shard); out [B, L, NH, 128] bf16 with strides o_sb, o_sl, o_sh.
 * Rows whose every key is masked are written as 0. */
int flashb_prefill_attn(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sl, const void* k, int64_t k_sb,
                        int64_t k_sh, int64_t k_sl, const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl,
                        const void* mask, int mask_is_bf16, int64_t m_sb, int64_t m_sl, int B, int NH, int NKV, int L,
                        int S, int D, float scaling, int causal, int h0, int h1, void* out, int64_t o_sb,
                        int64_t o_sl, int64_t o_sh, void* stream);

/* flashb_prefill_attn for the query tiles [tile0, tile1) only (query rows [128 tile0, min(L, 128 tile1))): a
 * query-row shard of a multi-GPU prefill; the output rows of the other tiles are not written.  No reference
 * counterpart (the reference runs the prefill attention on one GPU). */
int flashb_prefill_attn_tiles(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_sl, const void* k, int64_t k_sb,
                              int64_t k_sh, int64_t k_sl, const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl,
                              const void* mask, int mask_is_bf16, int64_t m_sb, int64_t m_sl, int B, int NH, int NKV,
                              int L, int S, int D, float scaling, int causal, int h0, int h1, int tile0, int tile1,
                              void* out, int64_t o_sb, int64_t o_sl, int64_t o_sh, void* stream);
/* The prefill's q|k|v tail for every prompt token (replaces, with flashb_prefill_attn and the GEMV entry points, the
 * eager layers of BackbonePrefillGraphCache._forward, UP/models/cudagraph/backbone_prefill_graph.py:95-112):
 * qkv [B L, (NH + 2 NKV) 128] bf16 raw projections (row stride ldq; token t = b L + l): q heads rewritten in place
 * as RoPE(q_norm(q)), k heads as RoPE(k_norm(k)) written to kc[b, j, cache_position[l], :], v heads copied to
 * vc[b, j, cache_position[l], :] (kc / vc [B, NKV, S, 128] bf16, batch / head strides c_sb / c_sh elements).  RoPE
 * rows cos_tab / sin_tab [P, 128] bf16 at position_ids[b, l] (int64 [B, L]); cache_position int64 [L].  Tokens
 * whose position or slot is out of range are skipped. */
int flashb_prefill_qkv(void* qkv, int64_t ldq, int B, int L, int NH, int NKV, const void* qn_w, const void* kn_w,
                       float eps, const void* cos_tab, const void* sin_tab, int P, const int64_t* position_ids,
                       const int64_t* cache_position, void* kc, void* vc, int64_t c_sb, int64_t c_sh, int S,
                       void* stream);
/* The prefill's logits (backbone_prefill_graph.py:111): logits [B, V] fp32 = W32 [V, H] fp32 . hidden[b] for B <= 128
 * already normalised bf16 rows at row stride ldh (the last token of each prompt). */
int flashb_lm_head_rows(const void* hidden, int64_t ldh, int B, int H, const float* W32, int V, float* logits,
                        void* stream);

/* LN12 -> bf16 on the device (the reference's lossless 12-bit weight storage, flash/ln12_format.py, read by its depth
 * kernels through dd2_init_ln12, flash/csrc/depth_frame.cu:800-823): a matrix W[N, K] (K % 1024 == 0) stored as
 * data [N][K / 1024][3][32][16 B] (slot 0: low bytes of the chunks 0, 1 of lane l's elements k = 1024 g + 256 c +
 * 8 l + j; slot 1: chunks 2, 3; slot 2: four nibble words -- 3-bit table index of element j at bits 4j.., its sign at
 * bit 8j + 7 (j < 4) or 8 (j - 4) + 3), meta [N][4] uint32 row records {hdr = (overflow offset << 13) | ((shift & 7)
 * << 10) | patch count, patch 0, 1, 2}, ovf uint32 (patches 3.. of each row, (k << 8) | exact high byte) and the
 * 8-entry table of high-byte exponent values as two little-endian words (lut_lo, lut_hi), each row's entries
 * offset by its shift.  Writes bf16 out[N, K] (row stride ldo elements): bit-exact the encoded matrix. */
int flashb_ln12_decode(const void* data, const void* meta, const void* ovf, uint32_t lut_lo, uint32_t lut_hi, int N,
                       int K, void* out, int64_t ldo, void* stream);

/* ---------------------------------------------------------------------------------------------- depth frame
 * Replaces the reference's depth frame megakernel dd2_init / dd2_frame (flash/csrc/depth_frame.cu:758-853, 923-934),
 * itself the kernel form of the official DepthDecoderGraph._full_loop (UP/models/cudagraph/depth_decoder_graph.py:
 * 558-654): ONE cooperative launch decodes all n_decode codebooks of a frame for `batch` rows (1, or up to 4 CFG
 * pairs cond[0..half) | uncond[half..2 half), e.g. several streams served together), sampling each codebook on the device (CFG u + gs (c - u), ids >= codebook_size
 * masked, / temperature, top-k (0 -> min(1024, vocab)), top-p, softmax, token = argmax(p / q)).
 * Layer descriptors (fb_dd_layer[layers]) in device memory; `scratch`: flashb_dd_scratch_bytes() bytes, 256-byte
 * aligned, zeroed once (and after a reported device error).  first_cb [batch] int64; bh [batch, embed_dim] bf16;
 * tokbuf [batch] int64 (receives the last token fed forward); outtok [batch, n_decode] int64 (sampled tokens);
 * temp/topp/gs [half] fp32, topk/dosample [half] int64; q [n_decode, half, vocab] fp32 Exp(1) draws;
 * dbg (optional) [n_decode, batch, vocab] fp32 logits; forced (optional) [n_decode, batch] int64 tokens fed to the
 * next codebook instead of the sampled ones (teacher forcing, for verification). */
typedef struct {
  const void *ln1, *wq, *wk, *wv, *wo, *ln2, *wg, *wu, *wd; /* bf16 */
} fb_dd_layer;
/* One depth matrix in the LN12 format (flash/ln12_format.py; flashb_ln12_decode): data [N][K / 1024][3][32][16 B],
 * meta [N][4] uint32 (16-byte aligned), ovf [n_ovf] uint32 overflow patches (reads past n_ovf are skipped), the
 * 8-entry table as two little-endian words. */
typedef struct {
  const void* data;
  const void* meta;
  const void* ovf;
  int64_t n_ovf;
  uint32_t lut_lo, lut_hi;
} fb_ln12_mat;
typedef struct {
  int layers, batch, hidden, embed_dim, heads, kv_heads, head_dim, ffn;
  int vocab, codebook_size, n_decode;
  float eps, scaling;
  const void* embed;   /* [(n_decode + 1) * vocab, embed_dim] bf16 */
  const void* proj;    /* [hidden, embed_dim] bf16 (inputs_embeds_projector) */
  const void* normf;   /* [hidden] bf16 */
  const void* head_t;  /* [n_decode, vocab, hidden] bf16 (codebook heads, transposed) */
  const void* cos_tab; /* [n_decode + 2, 128] bf16 */
  const void* sin_tab;
  uint64_t* trace;     /* optional: [grid][n_decode][11 + 9 * layers] %globaltimer stamps per CTA (task ends, barriers),
                          then (tcgen05 build, grids <= 32) [grid][64][8] per GEMV task of a CTA's first 64: entry,
                          first stage in, last MMA issued, MMAs complete, accumulators dumped, epilogues done, end,
                          blocks of the task */
  int grid;            /* CTAs of the launch, one per SM: 0 = every SM; fewer leave SMs to work on other streams */
  const void* layers_host; /* fb_dd_layer[layers] in host memory, the same pointers as layers_dev: the weight matrices'
                            * TMA tensor maps are built from it on the host (cached per matrix) */
  int64_t wait_ns;         /* limit of each grid-barrier wait in ns; 0 = 2 s.  On expiry the CTA records
                            * FB_ERR_TIMEOUT, sets the barrier's abort flag and the frame winds down */
  const void* ptab;        /* optional per-token step table (flashb_dd_tab_build; both null = none): ptab
                            * [(n_decode - 1) vocab, hidden] bf16 = projector output of embedding row vocab + t, */
  const void* ttab;        /* ttab [(n_decode - 1) vocab, (heads + 2 kv_heads) 128] bf16 = layer 0's pre-RoPE q|k|v of
                            * RMSNorm(ptab row t).  Codebook steps >= 1 then read their stage E and layer-0 q|k|v
                            * there instead of running the projector and layer-0 q|k|v GEMVs */
  const fb_ln12_mat* ln12; /* optional host array (null = none) of every streamed depth matrix in LN12, in the
                            * reference's order (dd2_init_ln12, flash/csrc/depth_frame.cu:800-823): per layer wq, wk,
                            * wv, wo, wg, wu, wd, then the projector, then the n_decode codebook heads [vocab, hidden].
                            * The tcgen05 build (grids <= 32) then streams the 12-bit bytes and decodes them in shared
                            * memory before the MMAs (about 25% fewer weight bytes, the same bf16 values); other builds
                            * read the bf16 matrices.  Needs hidden, ffn, heads x 128, embed_dim multiples of 1024 and
                            * vocab, kv_heads x 128 multiples of 64 */
} fb_dd_config;
int64_t flashb_dd_scratch_bytes(const fb_dd_config* cfg);
/* Builds the per-token step table of the reference's dd2_tab_build (flash/csrc/depth_frame.cu:714-754, 894-913): for
 * every table row t < (n_decode - 1) vocab (embedding row vocab + t, the ids codebook steps 1 .. n_decode - 1 can
 * feed), ptab[t] = bf16(proj . embed[vocab + t]) and ttab[t] = bf16([wq; wk; wv] of layer 0 . RMSNorm(ptab[t]; ln1)),
 * with the library's GEMV kernels (the same arithmetic contract as the frame's stage E and layer-0 q|k|v).  work:
 * [(n_decode - 1) vocab, hidden] bf16 scratch.  Enqueued on `stream`; the buffers are the caller's. */
int flashb_dd_tab_build(const fb_dd_config* cfg, void* ptab, void* ttab, void* work, void* stream);
int64_t flashb_dd_layer_bytes(void);
/* Byte offset, within the scratch buffer, of the frame's grid-barrier state: four uint32 words (arrival count, exit
 * count, abort flag, padding), zero between frames.  A non-zero abort word (set by the host, e.g. with
 * cudaMemsetAsync on the frame's stream or another stream) makes a frame stop at its next barrier wait, record
 * FB_ERR_ABORTED in the device error word and return; the scratch must then be zeroed again before the next frame.
 * No reference counterpart (the reference's barriers cannot be cancelled, flash/csrc/depth_common.cuh:52-65). */
int64_t flashb_dd_barrier_offset(const fb_dd_config* cfg);
int flashb_dd_frame(const fb_dd_config* cfg, const void* layers_dev, void* scratch, const int64_t* first_cb,
                    const void* bh, int64_t* tokbuf, int64_t* outtok, const float* temp, const int64_t* topk,
                    const float* topp, const int64_t* dosample, const float* gs, const float* q, float* dbg,
                    const int64_t* forced, void* stream);

/* No counterpart in the reference.  flashb_dd_frame without a scratch argument, for callers that may not allocate
 * device memory themselves: a host that reaches this library over a plain C FFI with no allocator of its own, or a
 * serving loop that forbids cudaMalloc after start-up (it can block on the device and it can fail).  The scratch is
 * instead a fixed area of FB_DD_NOALLOC_SCRATCH_BYTES (1 MiB) inside the library, reserved on every GPU that loads
 * it until the process exits; configurations whose flashb_dd_scratch_bytes() exceeds it are rejected with
 * FB_ERR_ARG.  Everything else is as for flashb_dd_frame; nothing is allocated and no allocating routine is called.
 * The first call on a device looks up the area's device address (with that device current) and keeps it until the
 * process exits; make that first call before any stream capture, and make no call on a device after resetting it
 * (cudaDeviceReset gives the area a new address, and the kept one would be stale).  The configuration is checked
 * field by field before anything is sized or enqueued from it.  Each call clears the area's barrier words on `stream` first; the rest of the area
 * keeps the previous call's contents and needs no clearing.  All calls on a device share the one area: calls that
 * can overlap on the GPU (different streams, no ordering between them) race and corrupt each other. */
#define FB_DD_NOALLOC_SCRATCH_BYTES (1u << 20)
int flashb_dd_frame_noalloc(const fb_dd_config* cfg, const void* layers_dev, const int64_t* first_cb, const void* bh,
                            int64_t* tokbuf, int64_t* outtok, const float* temp, const int64_t* topk,
                            const float* topp, const int64_t* dosample, const float* gs, const float* q, float* dbg,
                            const int64_t* forced, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASHB_H */
