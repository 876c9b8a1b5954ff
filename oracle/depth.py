"""Depth-decoder frame oracle (test infrastructure; see ``oracle/__init__.py``).

Restates ``DepthDecoderGraph._full_loop`` (``UP/models/cudagraph/depth_decoder_graph.py:558-654``) in numpy with the
eager (non-compiled) rounding points of ``BreezeDecoderLayer`` (``UP/models/breeze.py:378-425``):

  step 0: ids = [0, first_cb] embedded without offset, row 0 replaced by the backbone hidden state (:562-577),
          projected by ``inputs_embeds_projector`` (:578), positions [0, 1], causal mask (:581-593);
          logits = fp32 head[0] applied to the normed hidden of position 1 (:595-603).
  step s: id = clamp(tok + s * V, 0, num_codebooks * V - 1) (:616-621), projected, position s + 1 (:624-637),
          logits = fp32 head[s] (:645-650).
  every step: CFG sampler (:485-556) -> token clamped to [0, V-1] and written to both CFG halves (:611-613, 652-654).

``num_codebooks`` in the reference config counts the backbone's codebook too: a frame decodes ``num_codebooks - 1``
depth codebooks (``depth_decoder_graph.py:134-135``); the embedding table has ``num_codebooks * V`` rows
(``UP/models/breeze.py:479-481``) and the head ``num_codebooks - 1`` matrices [H, V] (``breeze.py:607-611``).
"""
import numpy as np

from . import decode as dec
from . import sampler as smp
from .bf16 import round_bf16

F32 = np.float32
BF16_MIN = F32(-3.3895313892515355e38)   # torch.finfo(torch.bfloat16).min, the eager causal-mask fill value


class DepthWeights:
    """Depth-decoder weights as float32 arrays holding bf16 values (head in fp32, bf16-exact)."""

    def __init__(self, layers, embed, proj, normf, head32, vocab, codebook_size, n_decode, eps, theta, nh, nkv,
                 head_dim=128):
        self.layers = layers          # dicts: ln1 wq wk wv wo ln2 wg wu wd
        self.embed = embed            # [(n_decode + 1) * vocab, AE]
        self.proj = proj              # [H, AE]
        self.normf = normf            # [H]
        self.head32 = head32          # [n_decode, H, vocab] fp32
        self.vocab = vocab
        self.codebook_size = codebook_size
        self.n_decode = n_decode
        self.eps = eps
        self.theta = theta
        self.nh = nh
        self.nkv = nkv
        self.head_dim = head_dim


def depth_layer(x, L, kc, vc, positions, cos_t, sin_t, eps, scaling, nh, nkv, D):
    """One ``BreezeDecoderLayer`` (``UP/models/breeze.py:400-425``) for T new tokens at ``positions``; kc/vc
    [B, NKV, max_seq, D] are the layer's StaticCache tensors, updated in place."""
    B, T, _ = x.shape
    h = dec.rmsnorm(x, L['ln1'], eps)
    q = dec.linear(h, L['wq']).reshape(B, T, nh, D).transpose(0, 2, 1, 3)
    k = dec.linear(h, L['wk']).reshape(B, T, nkv, D).transpose(0, 2, 1, 3)
    v = dec.linear(h, L['wv']).reshape(B, T, nkv, D).transpose(0, 2, 1, 3)
    c = cos_t[positions][None, None]
    s = sin_t[positions][None, None]
    q = dec.rope(q, c, s)
    k = dec.rope(k, c, s)
    kc[:, :, positions] = k
    vc[:, :, positions] = v
    Smax = kc.shape[2]
    key = np.arange(Smax)[None, :]
    allowed = key <= np.asarray(positions)[:, None]                 # [T, Smax] causal over the static cache
    mask = np.where(allowed, F32(0.0), BF16_MIN).astype(F32)[None, None]
    a = dec.attention_eager(q, kc, vc, mask, scaling, mask_bf16=True)   # [B, T, NH, D]
    o = dec.linear(a.reshape(B, T, nh * D), L['wo'])
    x = round_bf16(x + o)
    h = dec.rmsnorm(x, L['ln2'], eps)
    m = dec.linear(dec.silu_mul(dec.linear(h, L['wg']), dec.linear(h, L['wu'])), L['wd'])
    return round_bf16(x + m)


def depth_frame(W, bh, first_cb, q, temp, topk, topp, dosample, gs, forced=None, sampler='c'):
    """One frame.  bh [B, AE] backbone hidden (bf16 values), first_cb [B] int, q [n_decode, half, V] fp32,
    per-half sampling parameters (sequences of length half).  ``forced`` [n_decode, B] teacher-forces the token fed
    to the next step (the verification tap of ``flash/csrc/depth_frame.cu:38-40, 645``).

    Returns (tokens [B, n_decode] int64, logits [n_decode, B, V] fp32, sampled [B, n_decode] int64); ``tokens``
    are the tokens fed forward (the forced ones when ``forced`` is given, as the flash kernel writes them),
    ``sampled`` what the sampler chose from each step's logits."""
    bh = np.asarray(bh, F32)
    B = bh.shape[0]
    half = B // 2 if B >= 2 else 1
    V, n = W.vocab, W.n_decode
    D, nh, nkv = W.head_dim, W.nh, W.nkv
    Smax = 2 + n
    nL = len(W.layers)
    kc = np.zeros((nL, B, nkv, Smax, D), F32)
    vc = np.zeros_like(kc)
    cos_t, sin_t = dec.rope_tables(W.theta, D, np.arange(Smax))
    scaling = D ** -0.5
    tokens = np.zeros((B, n), np.int64)
    sampled = np.zeros((B, n), np.int64)
    all_logits = np.zeros((n, B, V), F32)
    tok = None
    for step in range(n):
        if step == 0:
            ids = np.stack([np.zeros(B, np.int64), np.asarray(first_cb, np.int64)], axis=1)
            emb = np.asarray(W.embed, F32)[ids]                      # [B, 2, AE]
            emb[:, 0] = bh
            positions = [0, 1]
        else:
            ids = np.clip(tok + step * V, 0, (n + 1) * V - 1)
            emb = np.asarray(W.embed, F32)[ids][:, None]             # [B, 1, AE]
            positions = [step + 1]
        x = dec.linear(emb, W.proj)
        for li, L in enumerate(W.layers):
            x = depth_layer(x, L, kc[li], vc[li], positions, cos_t, sin_t, W.eps, scaling, nh, nkv, D)
        h = dec.rmsnorm(x, W.normf, W.eps)[:, -1]
        logits = np.matmul(h, W.head32[step]).astype(F32)           # [B, V] fp32
        all_logits[step] = logits
        th = np.zeros(half, np.int64)
        for hh in range(half):
            lu = logits[hh + half] if B >= 2 else None
            if sampler == 'c':
                t, _ = smp.sample_row(logits[hh], lu, W.codebook_size, gs[hh], temp[hh], topk[hh], topp[hh],
                                      dosample[hh], q[step, hh])
            else:
                t, _ = smp.sample_row_torch(logits[hh], lu, V, W.codebook_size, gs[hh], temp[hh], topk[hh],
                                            topp[hh], dosample[hh], q[step, hh])
            th[hh] = t
        tok = np.clip(np.concatenate([th, th]) if B >= 2 else th, 0, V - 1)
        sampled[:, step] = tok
        if forced is not None:
            tok = np.clip(np.asarray(forced[step], np.int64), 0, V - 1)
        tokens[:, step] = tok
    return tokens, all_logits, sampled
