"""Backbone decode step on the flashb kernels, with the reference hook's surface (``flash/backbone.py:1-148``).

``install()`` replaces ``BackboneGraph._decode_step`` (``UP/models/cudagraph/backbone_graph.py:254-285``) with
``fused_decode_step``, which the official graph captures in its CUDA graph.  Per step:

    embed_rope                         gather-sum of the codebook embeddings + cos/sin rows      (1 launch)
    per layer: gemv_seg (RMSNorm + q|k|v) -> attn_decode_fused (q/k norm, RoPE, KV write, GQA)
               -> gemv_resid (o_proj + residual) -> gemv_gateup (RMSNorm + SwiGLU) -> gemv_resid (down + residual)
    lm_head_cfg                        final RMSNorm + fp32 lm_head + CFG                       (1 launch)

Unlike the reference, the embedding, rotary gather, lm_head and CFG also run as library kernels.  The step is the
2 + 5 x layers launches above, chained with programmatic dependent launch and captured by the caller's CUDA graph.
Unsupported graphs (head_dim != 128, GQA group outside {1, 2, 4, 8}, biases, non-SiLU MLP, more
than 8 batch rows, an audio-embedding projector) route to the original method, as the reference does
(``flash/backbone.py:49-103``).
"""
import torch

from . import _native, kernels
from ._native import check

# The reference's per-GPU launch-shape table (R rows/warp, U unroll, warps), kept for import compatibility; the
# B200 kernels choose their launch shape themselves.
GEMV_CFG = {
    1: dict(qkv=(2, 1, 8), o=(1, 1, 8), gateup=(1, 1, 8), down=(1, 1, 8)),
    2: dict(qkv=(2, 1, 8), o=(1, 1, 8), gateup=(1, 1, 8), down=(1, 1, 8)),
    4: dict(qkv=(2, 1, 8), o=(1, 1, 8), gateup=(1, 1, 8), down=(1, 1, 8)),
    8: dict(qkv=(2, 1, 8), o=(1, 1, 8), gateup=(1, 1, 8), down=(1, 1, 8)),
}
_WS = {}
ORIG = {}
# rows above which the RMSNorms run apart from the GEMVs (the many-rows GEMV kernel takes 17..128 rows)
ROWS_NORM_APART = 16


def workspace(device, B, NH, NKV, S, D=128):
    """The reference's attention workspace arguments (flash/backbone.py:27-37); flashb's attention needs none, so
    these are one-element placeholders kept for the call signature."""
    key = (str(device), B, NH, NKV, S)
    w = _WS.get(key)
    if w is None:
        one = torch.empty(1, device=device, dtype=torch.float32)
        w = dict(scores=one, cmax=one, part=one, counters=torch.zeros(1, device=device, dtype=torch.int32))
        _WS[key] = w
    return w


class Layer:
    __slots__ = ('ln1_w', 'ln1_eps', 'wq', 'wk', 'wv', 'qn_w', 'kn_w', 'qk_eps', 'scaling', 'wo', 'ln2_w', 'ln2_eps',
                 'wg', 'wu', 'wd')


def _bf16_2d(t):
    return t is not None and t.dtype == torch.bfloat16 and t.is_contiguous()


def make_state(B, layers, norm_w, norm_eps, embed_table, vocab, lm_head32, cos_tab, sin_tab, max_seq_len, device):
    """Buffers and weight handles for one graph: ``layers`` is a list of ``Layer``."""
    H = layers[0].wq.shape[1]
    nq, nk = layers[0].wq.shape[0], layers[0].wk.shape[0]
    I = layers[0].wg.shape[0]
    bf = dict(dtype=torch.bfloat16, device=device)
    return dict(B=B, layers=layers, norm_w=norm_w, norm_eps=float(norm_eps), embed=embed_table, vocab=int(vocab),
                lm_head32=lm_head32, cos_tab=cos_tab, sin_tab=sin_tab,
                x0=torch.empty(B, H, **bf), cos=torch.empty(B, 1, 128, **bf), sin=torch.empty(B, 1, 128, **bf),
                qkv=torch.empty(B, nq + 2 * nk, **bf), ao=torch.empty(B, 1, nq // 128, 128, **bf),
                h1=torch.empty(B, H, **bf), act=torch.empty(B, I, **bf), x=torch.empty(B, H, **bf),
                xn=torch.empty(B, H, **bf) if B > ROWS_NORM_APART else None,
                ws=workspace(device, B, nq // 128, nk // 128, max_seq_len))


def weights_of(graph):
    """The official graph's weights as ``Layer`` records plus (norm, embedding table, lm_head): attribute reads and
    the checks of what the kernels cover, on any device.  None when the graph is outside it (``flash/backbone.py:
    49-103``: the reference's hook makes the same checks)."""
    model = graph.model
    if graph.batch_size not in GEMV_CFG or len(model.layers) == 0:
        return None
    Ls = []
    for layer in model.layers:
        at, mlp = layer.self_attn, layer.mlp
        L = Layer()
        L.ln1_w, L.ln1_eps = layer.input_layernorm.weight, float(layer.input_layernorm.variance_epsilon)
        L.ln2_w, L.ln2_eps = layer.post_attention_layernorm.weight, float(
            layer.post_attention_layernorm.variance_epsilon)
        L.wq, L.wk, L.wv, L.wo = at.q_proj.weight, at.k_proj.weight, at.v_proj.weight, at.o_proj.weight
        L.qn_w, L.kn_w = at.q_norm.weight, at.k_norm.weight
        L.qk_eps = float(at.q_norm.variance_epsilon)
        if float(at.k_norm.variance_epsilon) != L.qk_eps:
            return None
        L.scaling = float(at.scaling)
        L.wg, L.wu, L.wd = mlp.gate_proj.weight, mlp.up_proj.weight, mlp.down_proj.weight
        for m in (at.q_proj, at.k_proj, at.v_proj, at.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            if getattr(m, 'bias', None) is not None:
                return None
        if not all(_bf16_2d(t) for t in (L.ln1_w, L.ln2_w, L.wq, L.wk, L.wv, L.wo, L.qn_w, L.kn_w, L.wg, L.wu, L.wd)):
            return None
        if getattr(mlp, 'act_fn', None).__class__.__name__ not in ('SiLU', 'SiLUActivation'):
            return None
        if at.head_dim != 128 or at.num_key_value_groups not in (1, 2, 4, 8) or getattr(at, 'sliding_window', None):
            return None
        Ls.append(L)
    emb = graph.embed_tokens
    if getattr(emb, 'audio_embeds_projector', None) is not None or not _bf16_2d(emb.embed_audio_tokens.weight):
        return None
    lm = graph.lm_head
    if getattr(lm, 'bias', None) is not None or lm.weight.dtype != torch.float32 or not _bf16_2d(model.norm.weight):
        return None
    return Ls, model.norm, emb.embed_audio_tokens.weight, lm.weight


def _prep(graph):
    """Weight handles + buffers for an official BackboneGraph on a GPU; None -> unsupported, use the original step."""
    st = getattr(graph, '_bb_state', None)
    if st is not None and st['B'] == graph.batch_size:
        return st
    try:
        if not torch.device(graph.device).type == 'cuda':
            return None
        got = weights_of(graph)
        if got is None:
            return None
        Ls, norm, table, lm_w = got
        if not all(t.is_cuda for L in Ls for t in (L.wq, L.wk, L.wv, L.wo, L.wg, L.wu, L.wd)):
            return None
        model, B = graph.model, graph.batch_size
        dev = graph.device
        S = graph.max_seq_len
        with torch.no_grad():
            pos = torch.arange(S + 1, device=dev)[None]
            dummy = torch.zeros(1, S + 1, 128, dtype=torch.bfloat16, device=dev)
            cos, sin = model.rotary_emb(dummy, pos)
        st = make_state(B, Ls, norm.weight, norm.variance_epsilon, table, table.shape[0] // graph.num_codebooks,
                        lm_w.contiguous(), cos[0].contiguous().to(torch.bfloat16),
                        sin[0].contiguous().to(torch.bfloat16), S, dev)
        kernels.attn()
        kernels.fused()
        graph._bb_state = st
        print(f'[flashb] fused backbone decode step enabled (B={B}, layers={len(Ls)})', flush=True)
        return st
    except Exception as e:  # pragma: no cover - the official path stays available
        print(f'[flashb] fused backbone path unavailable ({e!r}); using the original decode step', flush=True)
        return None


def run_layers(st, x, kv_layers, mask, cache_position):
    """The 28 x 5 kernel body; ``x`` is the embedded input [B, H]; returns the final residual stream [B, H].

    With more than ROWS_NORM_APART rows (the shared step of many streams) each RMSNorm runs as its own launch into
    ``xn`` and the q|k|v and gate|up GEMVs take the normalised rows: the many-rows GEMV kernel has no norm prologue
    (it would re-read every row for the sums of squares on every CTA).  The values are the same: the norm is the
    same eager Qwen3 RMSNorm either way."""
    fx, ax = kernels.fused(), kernels.attn()
    B = st['B']
    ws = st['ws']
    qkv, ao, h1, act, xb, xn = st['qkv'], st['ao'], st['h1'], st['act'], st['x'], st.get('xn')
    for li, L in enumerate(st['layers']):
        kc, vc = kv_layers[li]
        if xn is not None:
            fx.rmsnorm(x, L.ln1_w, L.ln1_eps, xn)
            fx.gemv_seg(xn, None, L.ln1_eps, L.wq, L.wk, L.wv, qkv)
        else:
            fx.gemv_seg(x, L.ln1_w, L.ln1_eps, L.wq, L.wk, L.wv, qkv)
        ax.attn_decode_fused(qkv, L.qn_w, L.kn_w, L.qk_eps, st['cos'], st['sin'], kc, vc, mask, cache_position,
                             L.scaling, ws['scores'], ws['cmax'], ws['part'], ws['counters'], ao)
        fx.gemv_resid(ao.view(B, -1), L.wo, x, h1)
        if xn is not None:
            fx.rmsnorm(h1, L.ln2_w, L.ln2_eps, xn)
            fx.gemv_gateup(xn, None, L.ln2_eps, L.wg, L.wu, act)
        else:
            fx.gemv_gateup(h1, L.ln2_w, L.ln2_eps, L.wg, L.wu, act)
        fx.gemv_resid(act, L.wd, h1, xb)
        x = xb
    return x


def fused_decode_step(graph, advance=False):
    """One backbone decode step on the official graph's buffers (``BackboneGraph._decode_step``).  ``advance``
    (flashb extension, off for the official graph) first moves cache_position / position_ids / mask by one slot on
    the device, as the streaming loop does on the host between steps."""
    st = _prep(graph)
    if st is None:
        return ORIG['_decode_step'](graph)
    B = graph.batch_size
    fx = kernels.fused()
    if advance:
        check(_native.lib().flashb_step_advance(graph.cache_position.data_ptr(), graph.position_ids.data_ptr(), B,
                                                graph.attn_mask.data_ptr(), int(graph.attn_mask.dtype ==
                                                                                torch.bfloat16),
                                                graph.attn_mask.stride(0), graph.max_seq_len,
                                                torch.cuda.current_stream(graph.hidden_buf.device).cuda_stream))
    fx.embed_rope(graph.input_ids_buf.view(B, -1), st['vocab'], st['embed'], graph.position_ids.view(-1),
                  st['cos_tab'], st['sin_tab'], st['x0'], st['cos'], st['sin'])
    layers = graph.static_cache.layers
    x = run_layers(st, st['x0'], [(L.keys, L.values) for L in layers], graph.attn_mask, graph.cache_position)
    # flashb extension: ``graph.cfg_block`` rows per CFG block (several independent groups of streams in one graph,
    # each laid out [cond..., uncond...]); the official graph is one block
    blk = getattr(graph, 'cfg_block', B)
    hb = graph.hidden_buf.view(B, -1)
    if blk == B and B <= 16:
        fx.lm_head_cfg(x, st['norm_w'], st['norm_eps'], st['lm_head32'], graph.guidance_scale, hb, graph.logits_buf,
                       graph.cfg_logits_buf)
    else:
        # every CFG block in one pass over the fp32 lm_head
        fx.lm_head_cfg_blocks(x, st['norm_w'], st['norm_eps'], st['lm_head32'], graph.guidance_scale, blk, hb,
                              graph.logits_buf, graph.cfg_logits_buf)


def install(api=None):
    from models.cudagraph.backbone_graph import BackboneGraph
    if '_decode_step' in ORIG:
        return
    kernels.attn()
    kernels.fused()
    ORIG['_decode_step'] = BackboneGraph._decode_step
    BackboneGraph._decode_step = fused_decode_step
    print('[flashb] installed: fused backbone decode step', flush=True)
