"""The backbone prefill on flashb kernels, with the reference's surface
(``UP/models/cudagraph/backbone_prefill_graph.py:95-112``, ``BackbonePrefillGraphCache._forward``).

``prefill_forward(st, inputs_embeds, causal_mask, position_ids, cache_position, kv_layers)`` runs the Qwen3 backbone
over the prompt embeddings [B, L, H] and writes every layer's StaticCache slots at ``cache_position``, as the
reference's eager ``self.model(...)`` call does, then the final norm and the fp32 lm_head of the last token:

    per layer   rmsnorm (B L rows)                                        flashb_rmsnorm
                q|k|v GEMM (tcgen05, tiles of 128 rows)                   flashb_gemv_seg
                q/k head norm + RoPE, K/V written to the cache            flashb_prefill_qkv
                causal GQA attention over the cache's first L slots       flashb_prefill_attn
                o GEMM + residual                                         flashb_gemv_resid
                rmsnorm, gate|up GEMM + SiLU*up, down GEMM + residual     flashb_rmsnorm, _gemv_gateup, _gemv_resid
    end         final rmsnorm (hidden states), lm_head on the last token  flashb_rmsnorm, flashb_lm_head_rows

Returns ``(hidden [B, L, H] bf16, logits [B, V] fp32)`` like the reference.  Every launch is graph-capturable (the
reference captures ``_forward`` per length bucket); the per-length activation buffers are allocated on the first call
of a length (inside a capture they come from the graph's pool, as the reference's own outputs do).

``install()`` makes ``BackbonePrefillGraphCache._forward`` take this path when the graph qualifies (CUDA, bf16,
head_dim 128, the decode hook's weight layout) and keeps the official (attention-hooked) forward otherwise.
"""
import torch

from . import backbone as bb
from . import kernels
from .prefill_attn import _trim, prefill_attention

ORIG = {}


def _bufs(st, T):
    key = ('prefill_bufs', T)
    b = st.get(key)
    if b is None:
        L0 = st['layers'][0]
        H = L0.wq.shape[1]
        qkv_n = L0.wq.shape[0] + L0.wk.shape[0] + L0.wv.shape[0]
        dev, bf = L0.wq.device, torch.bfloat16
        b = dict(xn=torch.empty(T, H, dtype=bf, device=dev), qkv=torch.empty(T, qkv_n, dtype=bf, device=dev),
                 ao=torch.empty(T, L0.wq.shape[0], dtype=bf, device=dev), h1=torch.empty(T, H, dtype=bf, device=dev),
                 act=torch.empty(T, L0.wg.shape[0], dtype=bf, device=dev),
                 xa=torch.empty(T, H, dtype=bf, device=dev), xb=torch.empty(T, H, dtype=bf, device=dev))
        st[key] = b
    return b


def prefill_forward(st, inputs_embeds, causal_mask, position_ids, cache_position, kv_layers, hidden_out=None,
                    logits_out=None):
    """See the module docstring.  ``st``: the backbone state of ``flashb.backbone`` (weights, rotary tables, fp32
    lm_head); kv_layers: [(keys, values)] per layer, [B, NKV, S, 128] bf16, written in place."""
    fx = kernels.fused()
    B, L, H = inputs_embeds.shape
    T = B * L
    b = _bufs(st, T)
    x = inputs_embeds.reshape(T, H)
    if not x.is_contiguous():
        x = x.contiguous()
    pos = position_ids.reshape(B, L)
    pos = pos if pos.dtype == torch.int64 and pos.is_contiguous() else pos.to(torch.int64).contiguous()
    cp = cache_position.reshape(-1)
    cp = cp if cp.dtype == torch.int64 and cp.is_contiguous() else cp.to(torch.int64).contiguous()
    xn, qkv, ao, h1, act = b['xn'], b['qkv'], b['ao'], b['h1'], b['act']
    outs = (b['xa'], b['xb'])
    for li, Lw in enumerate(st['layers']):
        kc, vc = kv_layers[li]
        NH, NKV = Lw.wq.shape[0] // 128, Lw.wk.shape[0] // 128
        fx.rmsnorm(x, Lw.ln1_w, Lw.ln1_eps, xn)
        fx.gemv_seg(xn, None, Lw.ln1_eps, Lw.wq, Lw.wk, Lw.wv, qkv)
        fx.prefill_qkv(qkv, B, L, NH, NKV, Lw.qn_w, Lw.kn_w, Lw.qk_eps, st['cos_tab'], st['sin_tab'], pos, cp, kc, vc)
        q = qkv.as_strided((B, NH, L, 128), (L * qkv.stride(0), 128, qkv.stride(0), 1))
        k, v, m = _trim(q, kc, vc, causal_mask)
        prefill_attention(q, k, v, m, Lw.scaling, causal=True, out=ao.view(B, L, NH, 128))
        fx.gemv_resid(ao, Lw.wo, x, h1)
        fx.rmsnorm(h1, Lw.ln2_w, Lw.ln2_eps, xn)
        fx.gemv_gateup(xn, None, Lw.ln2_eps, Lw.wg, Lw.wu, act)
        y = outs[li & 1]
        fx.gemv_resid(act, Lw.wd, h1, y)
        x = y
    hidden = hidden_out if hidden_out is not None else torch.empty(B, L, H, dtype=torch.bfloat16, device=x.device)
    fx.rmsnorm(x, st['norm_w'], st['norm_eps'], hidden.view(T, H))
    W32 = st['lm_head32']
    logits = logits_out if logits_out is not None else torch.empty(B, W32.shape[0], dtype=torch.float32,
                                                                   device=x.device)
    fx.lm_head_rows(hidden[:, -1], W32, logits)
    return hidden, logits


def _eligible(st, inputs_embeds, attention_mask, position_ids, cache_position, graph):
    if st is None or not inputs_embeds.is_cuda or inputs_embeds.dtype != torch.bfloat16 or inputs_embeds.dim() != 3:
        return False
    B, L, H = inputs_embeds.shape
    if B != graph.batch_size or L > graph.max_seq_len or H != st['layers'][0].wq.shape[1]:
        return False
    m = attention_mask
    if m is None or m.dim() != 4 or m.shape[2] != L or m.dtype not in (torch.bfloat16, torch.float32):
        return False
    if position_ids is None or position_ids.numel() != B * L or cache_position is None or cache_position.numel() != L:
        return False
    return all(L_.wq.shape[0] % 128 == 0 for L_ in st['layers'])


def fused_prefill_forward(self, inputs_embeds, attention_mask, position_ids, cache_position):
    """Drop-in for ``BackbonePrefillGraphCache._forward``: flashb's prefill when the graph qualifies, else the
    official forward (with the prefill attention hook when that is installed)."""
    graph = self.backbone_graph
    st = bb._prep(graph)
    if not _eligible(st, inputs_embeds, attention_mask, position_ids, cache_position, graph):
        return ORIG['_forward'](self, inputs_embeds, attention_mask, position_ids, cache_position)
    kv = [(L.keys, L.values) for L in graph.static_cache.layers]
    return prefill_forward(st, inputs_embeds, attention_mask, position_ids, cache_position, kv)


def install(api=None):
    from models.cudagraph.backbone_prefill_graph import BackbonePrefillGraphCache
    if '_forward' in ORIG:
        return
    ORIG['_forward'] = BackbonePrefillGraphCache._forward
    BackbonePrefillGraphCache._forward = fused_prefill_forward
    print('[flashb] backbone prefill on flashb kernels (tcgen05 GEMMs and attention, cache writes)', flush=True)
