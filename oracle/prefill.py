"""Prefill-attention oracle (test infrastructure; see ``oracle/__init__.py``).

``bz_prefill_attention`` (``flash/prefill_attn.py:15-24``): when the keys outnumber the queries and the mask is a
4-D tensor over every key, K/V/mask are trimmed to the first L slots (slots >= L are masked with finfo.min, whose
exp underflows to exactly 0, so the trim changes no value), then the eager attention runs
(``UP/models/breeze.py:259-286``; ``oracle.decode.attention_eager``).  Output [B, L, NH, D].
"""
import numpy as np

from . import decode as dec


def trim(q, k, v, mask):
    """The reference's trimming rule: keys sliced to [:L] when L > 1, S > L and the mask covers every key."""
    L = q.shape[2]
    S = k.shape[2]
    if L > 1 and S > L and mask is not None and mask.ndim == 4 and mask.shape[-1] == S:
        return k[:, :, :L], v[:, :, :L], mask[..., :L]
    return k, v, mask


def prefill_attention(q, k, v, mask, scaling, mask_bf16=True):
    """q [B, NH, L, D], k/v [B, NKV, S, D], additive mask [B | 1, 1, L, S] or None -> out [B, L, NH, D]."""
    k, v, mask = trim(q, k, v, mask)
    return dec.attention_eager(np.asarray(q, np.float32), np.asarray(k, np.float32), np.asarray(v, np.float32),
                               mask, scaling, mask_bf16=mask_bf16)


def prefill_qkv(qkv, B, L, NH, NKV, qn_w, kn_w, eps, cos, sin, kc, vc, cache_pos, head_dim=128):
    """The attention's projection tail for every prompt token (transformers ``Qwen3Attention.forward`` up to the cache
    update, as the reference prefill runs it through ``BackbonePrefillGraphCache._forward``,
    ``UP/models/cudagraph/backbone_prefill_graph.py:95-112``): q = RoPE(q_norm(q)), k = RoPE(k_norm(k)), the
    StaticCache update ``keys[:, :, cache_position] = k`` (and v).  qkv [B L, (NH + 2 NKV) D] raw projections;
    cos/sin [B, L, D] rows of the token positions; kc/vc [B, NKV, S, D] (modified).  Returns q [B, NH, L, D]."""
    D = head_dim
    qkv = np.asarray(qkv, np.float32).reshape(B, L, -1)
    q = qkv[..., : NH * D].reshape(B, L, NH, D)
    k = qkv[..., NH * D: (NH + NKV) * D].reshape(B, L, NKV, D)
    v = qkv[..., (NH + NKV) * D:].reshape(B, L, NKV, D)
    c = np.asarray(cos, np.float32).reshape(B, L, 1, D)
    s = np.asarray(sin, np.float32).reshape(B, L, 1, D)
    q = dec.rope(dec.rmsnorm(q, qn_w, eps), c, s)
    k = dec.rope(dec.rmsnorm(k, kn_w, eps), c, s)
    pos = np.asarray(cache_pos).reshape(-1)
    kc[:, :, pos, :] = k.transpose(0, 2, 1, 3)
    vc[:, :, pos, :] = v.transpose(0, 2, 1, 3)
    return q.transpose(0, 2, 1, 3)


def prefill_forward(W, emb, mask, position_ids, cache_pos, kcs, vcs, head_dim=128, layers=None):
    """``BackbonePrefillGraphCache._forward`` (``UP/models/cudagraph/backbone_prefill_graph.py:95-112``): the Qwen3
    backbone over the prompt embeddings emb [B, L, H] (eager bf16 semantics, every layer: RMSNorm -> q|k|v ->
    ``prefill_qkv`` -> causal attention over the trimmed cache (``prefill_attention``) -> o + residual -> RMSNorm ->
    SwiGLU -> down + residual), writing each layer's StaticCache (kcs/vcs modified in place), then the final norm.
    mask [B, 1, L, S] additive (bf16 values); position_ids [B, L].  Returns (hidden [B, L, H] bf16 values,
    logits [B, V] fp32 = lm_head(hidden[:, -1].float()))."""
    emb = np.asarray(emb, np.float32)
    B, L, H = emb.shape
    x = emb.reshape(B * L, H)
    cos, sin = dec.rope_tables(W.theta, head_dim, np.asarray(position_ids).reshape(-1))
    cos, sin = cos.reshape(B, L, head_dim), sin.reshape(B, L, head_dim)
    scaling = head_dim ** -0.5
    for li, Lw in enumerate(W.layers if layers is None else W.layers[:layers]):
        NH, NKV = Lw['wq'].shape[0] // head_dim, Lw['wk'].shape[0] // head_dim
        qkv = dec.gemv_seg(x, Lw['ln1'], W.eps, [Lw['wq'], Lw['wk'], Lw['wv']])
        q = prefill_qkv(qkv, B, L, NH, NKV, Lw['qn'], Lw['kn'], W.eps, cos, sin, kcs[li], vcs[li], cache_pos,
                        head_dim)
        ao = prefill_attention(q, kcs[li], vcs[li], mask, scaling)
        h1 = dec.gemv_resid(ao.reshape(B * L, -1), Lw['wo'], x)
        act = dec.gemv_gateup(h1, Lw['ln2'], W.eps, Lw['wg'], Lw['wu'])
        x = dec.gemv_resid(act, Lw['wd'], h1)
    h = dec.rmsnorm(x, W.norm, W.eps).reshape(B, L, H)
    return h, dec.lm_head_fp32(h[:, -1], W.lm_head32)
