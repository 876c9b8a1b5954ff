"""Backbone decode-step oracle (test infrastructure; see ``oracle/__init__.py``).

numpy restatement of the reference's eager PyTorch arithmetic for one single-token decode step of the Qwen3-style
backbone, with every bf16 rounding point of the eager graph.  All arrays are float32 holding bf16 values unless a
docstring says fp32.  Matmul accumulation is fp32 (numpy sgemm), like cuBLAS; its summation order differs from any
GPU kernel, which is why parity against this oracle is a tolerance, not bit equality.

Reference call stack for one step (``UP/models/cudagraph/backbone_graph.py:254-285`` ``BackboneGraph._decode_step``):
embed-sum (``UP/models/breeze.py:798-803``) -> Qwen3DecoderLayer x L (transformers ``modeling_qwen3``, pinned
4.57.3 by ``UP/requirements.txt:4``; called via ``UP/models/breeze_backbone_factory.py:163-181``) -> final
Qwen3RMSNorm -> fp32 lm_head -> CFG.  The flash hook restates the same step with kernels at
``flash/backbone.py:106-138``.
"""
import numpy as np

from .bf16 import round_bf16

F32 = np.float32


def rmsnorm(x, w, eps):
    """Eager RMSNorm: ``w * bf16(x * rsqrt(mean(x^2) + eps))`` rounded to bf16.

    ``UP/models/breeze.py:129-134`` (BreezeRMSNorm); transformers Qwen3RMSNorm is the same code.  The variance is
    an fp32 mean, the normalised value is cast back to bf16 (``.to(input_dtype)``) and the bf16 weight product is
    rounded again: two rounding points.
    """
    x = np.asarray(x, F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    h = round_bf16(x * (F32(1.0) / np.sqrt(var + F32(eps))))
    return round_bf16(np.asarray(w, F32) * h)


def linear(x, W):
    """``nn.Linear`` without bias in bf16: ``bf16(x @ W^T)`` with fp32 accumulation.  W is [N, K]."""
    return round_bf16(np.matmul(np.asarray(x, F32), np.asarray(W, F32).T))


def rotate_half(x):
    """``UP/models/breeze.py:211-215``: cat(-x2, x1) over the last dimension."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def rope(x, cos, sin):
    """``apply_rotary_pos_emb`` (``UP/models/breeze.py:218-242``) in bf16: ``bf16(bf16(x*cos) + bf16(rot(x)*sin))``.

    x [..., D]; cos/sin broadcastable to x (bf16 values)."""
    return round_bf16(round_bf16(x * cos) + round_bf16(rotate_half(x) * sin))


def rope_tables(theta, head_dim, positions):
    """cos/sin rows for integer ``positions`` as the default rotary embedding computes them.

    ``UP/models/breeze.py:159-186`` / transformers Qwen3RotaryEmbedding with the default rope init:
    inv_freq = 1 / theta ** (arange(0, D, 2) / D) in fp32; freqs = inv_freq * pos (fp32); emb = cat(freqs, freqs);
    cos/sin in fp32 then cast to bf16.  Computed with torch on the CPU so the values are those of the reference."""
    import torch
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.float32).reshape(-1)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    from .bf16 import from_torch
    return from_torch(emb.cos().to(torch.bfloat16)), from_torch(emb.sin().to(torch.bfloat16))


def attention_eager(q, k, v, mask, scaling, mask_bf16=True):
    """Eager GQA attention for queries q [B, NH, T, D] over keys/values [B, NKV, S, D].

    ``UP/models/breeze.py:259-286`` (identical to transformers Qwen3 ``eager_attention_forward``):
    s = bf16(q @ k^T) ; s = bf16(s * scaling) ; s = s + mask (bf16 add when the mask is bf16) ;
    p = bf16(softmax_fp32(s)) ; out = bf16(p @ v), returned as [B, T, NH, D] (the ``transpose(1, 2)``).
    ``mask`` is additive, broadcastable to [B, 1, T, S] (finfo.min or -inf for masked keys), or None.

    Rows whose keys are all masked (``mask <= -1e30`` everywhere) return 0, like the reference flash kernel
    (``flash/csrc/bb_attn.cu:183-186``: such rows have no active chunk and the combine sums nothing); the official
    decode graph never produces such a row because the current slot is always valid."""
    q = np.asarray(q, F32)
    B, NH, T, D = q.shape
    NKV = k.shape[1]
    G = NH // NKV
    kr = np.repeat(np.asarray(k, F32), G, axis=1)
    vr = np.repeat(np.asarray(v, F32), G, axis=1)
    s = round_bf16(np.matmul(q, kr.transpose(0, 1, 3, 2)))
    s = round_bf16(s * F32(scaling))
    dead = None
    if mask is not None:
        m = np.asarray(mask, F32)
        s = s + m
        if mask_bf16:
            s = round_bf16(s)
        dead = np.all(np.broadcast_to(m <= F32(-1e30), s.shape), axis=-1)
    mx = s.max(axis=-1, keepdims=True)
    e = np.exp(s - mx, dtype=F32)
    p = round_bf16(e / e.sum(axis=-1, keepdims=True, dtype=F32))
    out = round_bf16(np.matmul(p, vr))
    if dead is not None and dead.any():
        out = np.where(dead[..., None], F32(0.0), out)
    return out.transpose(0, 2, 1, 3)


def attn_decode(query, kc, vc, mask, scaling, mask_bf16=True):
    """Single-token decode attention: query [B, NH, 1, D] over the cache [B, NKV, S, D]; mask [B|1, 1, 1, S].

    Restates ``flash/csrc/bb_attn.cu:416-429`` ``attn_decode``; semantics are the eager ones above.
    Returns [B, 1, NH, D]."""
    S = kc.shape[2]
    m = None if mask is None else np.asarray(mask, F32)[..., :S]
    return attention_eager(query, kc, vc, m, scaling, mask_bf16)


def attn_decode_fused(qkv, qn_w, kn_w, eps, cos, sin, kc, vc, mask, cache_pos, scaling, mask_bf16=True):
    """q/k RMSNorm + RoPE + KV-cache write at ``cache_pos`` + decode attention, in place on kc/vc.

    Restates ``flash/csrc/bb_attn.cu:433-460`` ``attn_decode_fused``, whose semantics are transformers
    ``Qwen3Attention.forward`` for one token: q = q_norm(q_proj(x)), k = k_norm(k_proj(x)), RoPE on both, the
    StaticCache update at ``cache_position``, then eager attention.  qkv [B, (NH + 2 NKV) * D] raw projections;
    cos/sin [B, 1, D]; kc/vc [B, NKV, S, D] (modified).  Returns [B, 1, NH, D]."""
    qkv = np.asarray(qkv, F32)
    B = qkv.shape[0]
    NKV, S, D = kc.shape[1], kc.shape[2], kc.shape[3]
    NH = qkv.shape[1] // D - 2 * NKV
    q = qkv[:, : NH * D].reshape(B, NH, D)
    k = qkv[:, NH * D: (NH + NKV) * D].reshape(B, NKV, D)
    v = qkv[:, (NH + NKV) * D:].reshape(B, NKV, D)
    c = np.asarray(cos, F32).reshape(B, 1, D)
    s = np.asarray(sin, F32).reshape(B, 1, D)
    q = rope(rmsnorm(q, qn_w, eps), c, s)
    k = rope(rmsnorm(k, kn_w, eps), c, s)
    pos = int(np.asarray(cache_pos).reshape(-1)[0])
    kc[:, :, pos, :] = k
    vc[:, :, pos, :] = v
    return attn_decode(q[:, :, None, :], kc, vc, mask, scaling, mask_bf16)


def gemv_seg(x, nw, eps, Ws):
    """``y = norm?(x) @ [W0; W1; W2]^T`` rounded to bf16 (``flash/csrc/bb_fused.cu:293-316``).

    With a norm weight the prologue is the eager RMSNorm above (``bb_fused.cu:95-137``)."""
    h = rmsnorm(x, nw, eps) if nw is not None else np.asarray(x, F32)
    return np.concatenate([linear(h, W) for W in Ws if W is not None and np.asarray(W).size], axis=-1)


def gemv_resid(x, W, res):
    """``y = bf16(res + bf16(x @ W^T))`` (``flash/csrc/bb_fused.cu:319-335``; the eager residual add of
    ``Qwen3DecoderLayer.forward`` after o_proj / down_proj)."""
    return round_bf16(np.asarray(res, F32) + linear(x, W))


def silu_mul(g, u):
    """Qwen3MLP / BreezeMLP activation in bf16: ``bf16(bf16(silu(g)) * u)`` (``UP/models/breeze.py:206-208``)."""
    g = np.asarray(g, F32)
    a = round_bf16(g / (F32(1.0) + np.exp(-g, dtype=F32)))
    return round_bf16(a * np.asarray(u, F32))


def gemv_gateup(x, nw, eps, Wg, Wu):
    """``act = bf16(bf16(silu(bf16(n @ Wg^T))) * bf16(n @ Wu^T))``, n = RMSNorm(x) (``flash/csrc/bb_fused.cu:338-356``)."""
    h = rmsnorm(x, nw, eps)
    return silu_mul(linear(h, Wg), linear(h, Wu))


def embed_sum(table, ids, vocab):
    """``BreezeBackboneModelEmbeddings.forward`` (``UP/models/breeze.py:798-803``): gather row ``ids[b, c] + c*vocab``
    of the [num_codebooks * vocab, H] bf16 table for every codebook c and sum over codebooks with fp32 accumulation
    and one bf16 rounding (torch's bf16 ``sum``).  ids [B, C] int -> [B, H]."""
    ids = np.asarray(ids, np.int64)
    C = ids.shape[1]
    rows = ids + np.arange(C, dtype=np.int64)[None, :] * vocab
    g = np.asarray(table, F32)[rows]          # [B, C, H]
    return round_bf16(g.sum(axis=1, dtype=F32))


def lm_head_fp32(h, W32):
    """fp32 lm_head on the bf16 hidden state (``UP/models/cudagraph/backbone_graph.py:276-277``)."""
    return np.matmul(np.asarray(h, F32), np.asarray(W32, F32).T).astype(F32)


def cfg_combine(logits, half, gs):
    """``u + gs * (c - u)`` with three separately rounded fp32 ops (``backbone_graph.py:280-285``).
    logits [2*half, V] -> [half, V]."""
    c, u = logits[:half], logits[half:2 * half]
    return (u + (F32(gs) * (c - u)).astype(F32)).astype(F32)


class BackboneWeights:
    """Per-layer weight arrays of a Qwen3-style backbone (float32 holding bf16 values)."""

    def __init__(self, layers, norm, embed, lm_head32, vocab, eps, theta):
        self.layers = layers        # list of dicts: ln1 wq wk wv qn kn wo ln2 wg wu wd
        self.norm = norm
        self.embed = embed
        self.lm_head32 = lm_head32  # fp32 [V, H]
        self.vocab = vocab
        self.eps = eps
        self.theta = theta


def backbone_layer(x, L, kc, vc, mask, cache_pos, cos, sin, eps, scaling):
    """One Qwen3DecoderLayer for a single token, expressed with the five kernels of ``flash/backbone.py:120-126``:
    gemv_seg(RMSNorm + q|k|v) -> attn_decode_fused -> gemv_resid(o) -> gemv_gateup -> gemv_resid(down)."""
    B = x.shape[0]
    qkv = gemv_seg(x, L['ln1'], eps, [L['wq'], L['wk'], L['wv']])
    ao = attn_decode_fused(qkv, L['qn'], L['kn'], eps, cos, sin, kc, vc, mask, cache_pos, scaling)
    h1 = gemv_resid(ao.reshape(B, -1), L['wo'], x)
    act = gemv_gateup(h1, L['ln2'], eps, L['wg'], L['wu'])
    return gemv_resid(act, L['wd'], h1)


def backbone_step(W, ids, kcs, vcs, mask, cache_pos, position_ids, gs, head_dim=128, hidden_out=None):
    """One decode step: ids [B, C] codebook ids; kcs/vcs per-layer caches (modified in place);
    mask [B, 1, 1, S]; position_ids [B] (RoPE positions); returns (hidden [B, H] bf16, logits [B, V] fp32,
    cfg [half, V] fp32)."""
    B = ids.shape[0]
    x = embed_sum(W.embed, ids, W.vocab)
    cos, sin = rope_tables(W.theta, head_dim, np.asarray(position_ids).reshape(-1))
    cos, sin = cos.reshape(B, 1, head_dim), sin.reshape(B, 1, head_dim)
    scaling = head_dim ** -0.5
    for li, L in enumerate(W.layers):
        x = backbone_layer(x, L, kcs[li], vcs[li], mask, cache_pos, cos, sin, W.eps, scaling)
    h = rmsnorm(x, W.norm, W.eps)
    logits = lm_head_fp32(h, W.lm_head32)
    half = B // 2 if B >= 2 else 1
    cfg = cfg_combine(logits, half, gs) if B >= 2 else logits[:1]
    return h, logits, cfg
