"""Generate the golden fixtures in tests/golden/ from the reference's OWN PyTorch implementation.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py [--ref <reference root>]

It imports the reference's official modules (``third_party/breeze-tts``: ``models.breeze``,
``models.cudagraph.backbone_graph``, ``models.cudagraph.depth_decoder_graph``) and transformers' Qwen3 layers (the
backbone arithmetic the reference calls through ``UP/models/breeze_backbone_factory.py:163-181``), runs them on the
CPU on the seeded inputs of ``tests/golden/synth.py`` and writes their outputs as ``*.npz``.  The reference does not
exist on the GPU box; the committed fixtures travel instead.

Version shims (the reference pins transformers 4.57.3, this image has 5.5): the default rope init function is
registered for ``BreezeRotaryEmbedding`` (``UP/models/breeze.py:156``), and ``StaticLayer.lazy_initialization``
accepts the one-argument call of ``backbone_graph.py:199`` / ``depth_decoder_graph.py:462``.  In 5.5 the static
cache writes at its running length instead of ``cache_position``; both flows below write exactly the slots the 4.57.3
cache would (prefill fills [0, P) and decode appends), which the script asserts.  5.5's ``create_causal_mask`` also
ignores ``cache_position`` for the depth graph's decode masks (every decode mask would admit slot 0 only), so the
depth masks are rebuilt with the 4.57.3 rule: 0 where key <= cache_position, finfo(bf16).min elsewhere.
``module.to(torch.bfloat16)`` would also round the rotary ``inv_freq`` buffer to bf16; it is restored to the fp32
values the rotary modules compute at construction, as a checkpoint loaded in bf16 keeps them.

Sampling: ``torch.multinomial(probs, 1)`` inside the official sampler is replaced by ``argmax(probs / q)`` with q a
fixed Exp(1) draw, the identity the reference's own kernel relies on (``flash/csrc/depth_frame.cu:6-8``), so the
fixtures are deterministic.
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import synth  # noqa: E402


REF_ROOT = []


def ref_env(ref_root):
    REF_ROOT[:] = [ref_root]
    up = os.path.join(ref_root, 'third_party', 'breeze-tts')
    sys.path.insert(0, up)
    import transformers.cache_utils as cu
    import models.breeze as mb

    def default_rope(config=None, device=None, seq_len=None, **kw):
        base = getattr(config, 'rope_theta', None)
        if base is None:
            base = config.rope_parameters['rope_theta']
        dim = getattr(config, 'head_dim', None) or config.hidden_size // config.num_attention_heads
        inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).to(device=device, dtype=torch.float) / dim))
        return inv, 1.0

    mb.ROPE_INIT_FUNCTIONS['default'] = default_rope
    mb.BreezeRotaryEmbedding.compute_default_rope_parameters = staticmethod(default_rope)
    orig = cu.StaticLayer.lazy_initialization

    def lazy(self, k, v=None):
        return orig(self, k, k if v is None else v)

    cu.StaticLayer.lazy_initialization = lazy
    return up


class _Mod:
    """Stands in for the attention module argument of eager_attention_forward."""

    def __init__(self, groups):
        self.num_key_value_groups = groups
        self.training = False


def gold_attention(out):
    from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward
    c = synth.ATTN
    q, k, v, mask = synth.attn_inputs()
    o, _ = eager_attention_forward(_Mod(c['NH'] // c['NKV']), q, k, v, mask, scaling=c['D'] ** -0.5)
    out['attn'] = dict(out=synth.np_bits(o), digest=synth.digest(q, k, v, mask))
    # fp32-upcast variant (the CPU baseline form of config 1)
    o32, _ = eager_attention_forward(_Mod(c['NH'] // c['NKV']), q.float(), k.float(), v.float(), mask.float(),
                                     scaling=c['D'] ** -0.5)
    out['attn']['out_fp32'] = o32.numpy()


def gold_attention1(out):
    """Config 1 at its exact shapes: the bf16 eager attention and its fp32-upcast form, no mask (every key valid)."""
    from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward
    c = synth.ATTN1
    q, k, v = synth.attn1_inputs()
    mod = _Mod(c['NH'] // c['NKV'])
    o, _ = eager_attention_forward(mod, q, k, v, None, scaling=c['D'] ** -0.5)
    o32, _ = eager_attention_forward(mod, q.float(), k.float(), v.float(), None, scaling=c['D'] ** -0.5)
    out['attn1'] = dict(out=synth.np_bits(o), out_fp32=o32.numpy(), digest=synth.digest(q, k, v))


def _swiglu_ref(c, x, gamma, wg, wu, wd):
    import models.breeze as mb
    norm = mb.BreezeRMSNorm(c['K'], eps=c['eps']).to(torch.bfloat16)
    norm.weight.data.copy_(gamma)
    with torch.no_grad():
        h = norm(x)
        act = torch.nn.functional.silu(torch.nn.functional.linear(h, wg)) * torch.nn.functional.linear(h, wu)
        y = x + torch.nn.functional.linear(act, wd)
    return h, act, y


def gold_gemv2(out):
    """Config 2 at its exact shapes through BreezeRMSNorm, F.linear and silu (UP/models/breeze.py:120-208)."""
    c = synth.GEMV2
    x, gamma, wg, wu, wd = synth.gemv2_inputs()
    h, act, y = _swiglu_ref(c, x, gamma, wg, wu, wd)
    out['gemv2'] = dict(norm=synth.np_bits(h), act=synth.np_bits(act), y=synth.np_bits(y),
                        digest=synth.digest(x, gamma, wg, wu, wd))


def gold_gemv(out):
    c = synth.GEMV
    x, gamma, wg, wu, wd = synth.gemv_inputs()
    h, act, y = _swiglu_ref(c, x, gamma, wg, wu, wd)
    out['gemv'] = dict(norm=synth.np_bits(h), act=synth.np_bits(act), y=synth.np_bits(y),
                       digest=synth.digest(x, gamma, wg, wu, wd))


def _qwen3_config(c):
    from transformers import Qwen3Config
    cfg = Qwen3Config(hidden_size=c['H'], intermediate_size=c['F'], num_hidden_layers=c['L'],
                      num_attention_heads=c['NH'], num_key_value_heads=c['NKV'], head_dim=c['D'],
                      rms_norm_eps=c['eps'], rope_theta=c['theta'], vocab_size=c['vocab'],
                      max_position_embeddings=4096, attention_bias=False)
    cfg._attn_implementation = 'eager'
    cfg.num_codebooks = c['ncb']
    cfg.audio_embed_size = c['H']
    return cfg


def _official_backbone(c, w, dtype):
    """The official BackboneGraph over transformers Qwen3 layers (the reference's backbone), weights from w, run in
    ``dtype``, with the prefill KV of w written into its StaticCache and the generation state set."""
    from models.breeze_backbone_factory import BreezeBackboneAdapter
    from models.cudagraph.backbone_graph import BackboneGraph
    cfg = _qwen3_config(c)
    layers, norm, rot = BreezeBackboneAdapter._create_qwen3_layers(cfg)
    model = BreezeBackboneAdapter(cfg, layers, norm, rot)
    inv = model.rotary_emb.inv_freq.clone()
    model = model.to(dtype)
    model.rotary_emb.inv_freq = inv
    with torch.no_grad():
        for L, lw in zip(model.layers, w['layers']):
            a, m = L.self_attn, L.mlp
            L.input_layernorm.weight.copy_(lw['ln1'])
            a.q_proj.weight.copy_(lw['wq'])
            a.k_proj.weight.copy_(lw['wk'])
            a.v_proj.weight.copy_(lw['wv'])
            a.q_norm.weight.copy_(lw['qn'])
            a.k_norm.weight.copy_(lw['kn'])
            a.o_proj.weight.copy_(lw['wo'])
            L.post_attention_layernorm.weight.copy_(lw['ln2'])
            m.gate_proj.weight.copy_(lw['wg'])
            m.up_proj.weight.copy_(lw['wu'])
            m.down_proj.weight.copy_(lw['wd'])
        model.norm.weight.copy_(w['norm'])
        model.embed_tokens.embed_audio_tokens.weight.copy_(w['embed'])
    lm_head = torch.nn.Linear(c['H'], c['vocab'], bias=False)
    with torch.no_grad():
        lm_head.weight.copy_(w['lm_head'])
    g = BackboneGraph(model, lm_head, model.embed_tokens, cfg, device='cpu', dtype=dtype,
                      max_seq_len=c['S'], guidance_scale=c['gs'], batch_size=c['B'])
    g.prepare_eager()
    P = c['prefill']
    with torch.inference_mode():
        for li, (k, v) in enumerate(w['kv']):
            g.static_cache.layers[li].update(k.to(dtype), v.to(dtype))
    am = torch.ones(c['B'], P, dtype=torch.long)
    for b, p in enumerate(c['pad']):
        am[b, :p] = 0
    g.set_generation_state(am)
    g._prefill_len = P
    return g


def gold_backbone(out):
    c = synth.BACKBONE
    w = synth.backbone_weights()
    g = _official_backbone(c, w, torch.bfloat16)
    P = c['prefill']
    hidden, cfg_logits = g.run(w['ids'], 0)
    kv_new = []
    for li in range(c['L']):
        K = g.static_cache.layers[li].keys
        V = g.static_cache.layers[li].values
        assert torch.equal(K[:, :, :P], w['kv'][li][0]), 'prefill slots moved'
        kv_new.append((K[:, :, P].clone(), V[:, :, P].clone()))
        assert float(K[:, :, P + 1:].abs().sum()) == 0.0, 'decode wrote past cache_position'
    out['backbone'] = dict(hidden=synth.np_bits(hidden), logits=g.logits_buf.numpy().copy(),
                           cfg=cfg_logits.numpy().copy(), mask=g.attn_mask.float().numpy().copy(),
                           position_ids=g.position_ids.numpy().copy(), cache_position=g.cache_position.numpy().copy(),
                           k_new=np.stack([synth.np_bits(k) for k, _ in kv_new]),
                           v_new=np.stack([synth.np_bits(v) for _, v in kv_new]),
                           digest=synth.digest(w['embed'], w['lm_head'], *[t for kv in w['kv'] for t in kv]))


def gold_drift(out):
    """End-to-end drift of the 28-layer config 3 step (KV 1023 + the new token), from the reference's own modules:

    * ``bf16``: the official eager step in bf16 (the reference's arithmetic);
    * ``fp32``: the same modules and weights run in fp32 (the exact model the bf16 run approximates);
    * ``oracle``: the numpy restatement (tests' oracle): the bf16 eager rounding points of the official step, with
      numpy's fp32 summation order instead of torch's.
    The oracle is bit-exact to the official modules at reduced shapes; over 28 chained layers a different summation
    order alone makes rare 1-ulp bf16 rounding flips that compound.  ``oracle_vs_bf16`` measures that compounding
    between two implementations of the reference's own arithmetic, ``bf16_vs_fp32`` the reference's own error."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import decode as dec
    from oracle.bf16 import from_torch as ft
    c = synth.BACKBONE28
    w = synth.backbone_weights(c)
    g = _official_backbone(c, w, torch.bfloat16)
    g.run(w['ids'], 0)
    lg16 = g.logits_buf.numpy().copy()
    pids, mask = g.position_ids.numpy().copy(), g.attn_mask.float().numpy().copy()
    del g
    g = _official_backbone(c, w, torch.float32)
    g.run(w['ids'], 0)
    lg32 = g.logits_buf.numpy().copy()
    del g
    layers = [{k: ft(v) for k, v in L.items()} for L in w['layers']]
    W = dec.BackboneWeights(layers, ft(w['norm']), ft(w['embed']), w['lm_head'].numpy(), c['vocab'], c['eps'],
                            c['theta'])
    P = c['prefill']
    kcs = [np.zeros((c['B'], c['NKV'], c['S'], c['D']), np.float32) for _ in range(c['L'])]
    vcs = [np.zeros_like(x) for x in kcs]
    for li, (k, v) in enumerate(w['kv']):
        kcs[li][:, :, :P] = ft(k)
        vcs[li][:, :, :P] = ft(v)
    _, lgo, _ = dec.backbone_step(W, w['ids'].numpy()[:, 0, :], kcs, vcs, mask, P, pids.reshape(-1), c['gs'])

    def rel(a, b):
        return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))

    d = dict(logits_bf16=lg16, logits_fp32=lg32, logits_oracle=lgo, bf16_vs_fp32=rel(lg16, lg32),
             oracle_vs_bf16=rel(lgo, lg16), oracle_vs_fp32=rel(lgo, lg32),
             argmax_bf16_fp32=float(np.mean(lg16.argmax(-1) == lg32.argmax(-1))),
             digest=synth.digest(w['embed'], w['lm_head'], w['ids']))
    print('drift:', {k: v for k, v in d.items() if not k.startswith('logits')}, flush=True)
    out['drift'] = d


def _patched_multinomial(qsrc):
    """torch.multinomial(probs, 1) -> argmax(probs / q[step]) for the official sampler (one q row set per call)."""
    state = {'i': 0}

    def mult(probs, n, *a, **kw):
        q = qsrc[state['i']]
        state['i'] += 1
        return torch.argmax(probs / q.to(probs.dtype), dim=-1, keepdim=True)

    return mult, state


def _official_depth(c, w, dtype):
    """The official DepthDecoderGraph (eager, on the CPU) in ``dtype`` with the weights of w."""
    import models.breeze as mb
    import models.breeze_base_config as bc
    import models.cudagraph.depth_decoder_graph as ddg
    cfg = bc.BreezeDepthDecoderConfig(num_codebooks=c['ncb'], backbone_hidden_size=c['AE'], vocab_size=c['vocab'],
                                      hidden_size=c['H'], intermediate_size=c['F'], num_hidden_layers=c['L'],
                                      num_attention_heads=c['NH'], num_key_value_heads=c['NKV'], head_dim=c['D'],
                                      max_position_embeddings=64, rms_norm_eps=c['eps'], rope_theta=c['theta'])
    cfg._attn_implementation = 'eager'
    model = mb.BreezeDepthDecoderForCausalLM(cfg)
    inv = model.model.rotary_emb.inv_freq.clone()
    model = model.to(dtype)
    model.model.rotary_emb.inv_freq = inv
    dm = model.model
    assert dm.backbone_hidden_state_projector is None
    with torch.no_grad():
        for L, lw in zip(dm.layers, w['layers']):
            a, m = L.self_attn, L.mlp
            L.input_layernorm.weight.copy_(lw['ln1'])
            a.q_proj.weight.copy_(lw['wq'])
            a.k_proj.weight.copy_(lw['wk'])
            a.v_proj.weight.copy_(lw['wv'])
            a.o_proj.weight.copy_(lw['wo'])
            L.post_attention_layernorm.weight.copy_(lw['ln2'])
            m.gate_proj.weight.copy_(lw['wg'])
            m.up_proj.weight.copy_(lw['wu'])
            m.down_proj.weight.copy_(lw['wd'])
        dm.embed_tokens.weight.copy_(w['embed'])
        dm.inputs_embeds_projector.weight.copy_(w['proj'])
        dm.norm.weight.copy_(w['normf'])
        model.codebooks_head.weight.data = w['head'].clone().to(dtype)
    g = ddg.DepthDecoderGraph(model, cfg, device='cpu', dtype=dtype, do_sample=True, top_k=c['topk'],
                              top_p=c['topp'], temperature=c['temp'], guidance_scale=c['gs'],
                              codec_codebook_size=c['codebook_size'], fast=False, debug=True, batch_size=c['B'])
    g.prepare_eager()
    _fix_depth_masks(g)
    return g, ddg


def gold_depth(out):
    c = synth.DEPTH
    w = synth.depth_weights()
    g, ddg = _official_depth(c, w, torch.bfloat16)
    mult, st = _patched_multinomial([w['q'][s] for s in range(c['ncb'] - 1)])
    orig = ddg.torch.multinomial
    ddg.torch.multinomial = mult
    try:
        toks = g.run(w['bh'], w['first'])
    finally:
        ddg.torch.multinomial = orig
    assert st['i'] == c['ncb'] - 1
    out['depth'] = dict(tokens=g.output_tokens.numpy().copy(), logits=g.debug_logits.numpy().copy(),
                        ret=toks.numpy().copy(), digest=synth.digest(w['embed'], w['proj'], w['head'], w['bh'], w['q']))


def gold_depth_drift(out):
    """Argmax agreement of the full config 4 depth logits (8 CFG pairs, 16 codebooks, teacher-forced on fixed random
    tokens so every implementation sees the same inputs at every step), from the reference's own modules:
    the official eager step in bf16, the same in fp32, and the oracle (the bf16 rounding points with numpy's
    summation order).  Random-weight logits over 2048 ids have top-2 gaps down to ~1e-4 of their scale, so two
    implementations of the same bf16 arithmetic that differ only in fp32 summation order disagree on a few rows."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import depth as odepth
    from oracle.bf16 import from_torch as ft
    c = synth.DEPTH4
    w = synth.depth_weights(c)
    nd, B = c['ncb'] - 1, c['B']
    forced = torch.randint(0, c['codebook_size'], (nd, B // 2), generator=torch.Generator().manual_seed(77))
    logits = {}
    for name, dt in (('bf16', torch.bfloat16), ('fp32', torch.float32)):
        g, ddg = _official_depth(c, w, dt)
        state = {'i': 0}

        def mult(probs, n, *a, **kw):
            t = forced[state['i']].view(-1, 1)
            state['i'] += 1
            return t

        orig = ddg.torch.multinomial
        ddg.torch.multinomial = mult
        try:
            g.run(w['bh'].to(dt), w['first'])
        finally:
            ddg.torch.multinomial = orig
        assert state['i'] == nd
        logits[name] = g.debug_logits.float().numpy().copy()
        del g
    layers = [{k: ft(v) for k, v in L.items()} for L in w['layers']]
    W = odepth.DepthWeights(layers, ft(w['embed']), ft(w['proj']), ft(w['normf']), w['head'].numpy(), c['vocab'],
                            c['codebook_size'], nd, c['eps'], c['theta'], c['NH'], c['NKV'])
    half = B // 2
    par = (np.full(half, c['temp'], np.float32), np.full(half, c['topk']), np.full(half, c['topp'], np.float32),
           np.ones(half, np.int64), np.full(half, c['gs'], np.float32))
    fo = np.concatenate([forced.numpy(), forced.numpy()], 1)
    _, lgo, _ = odepth.depth_frame(W, ft(w['bh']), w['first'].numpy(), w['q'].numpy(), *par, forced=fo)
    lg16, lg32 = logits['bf16'], logits['fp32']
    lgo = np.asarray(lgo, np.float32).reshape(lg16.shape)

    def agree(a, b):
        return float(np.mean(a.argmax(-1) == b.argmax(-1)))

    def rel(a, b):
        return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))

    d = dict(logits_bf16=lg16, logits_fp32=lg32, logits_oracle=lgo, forced=forced.numpy(),
             argmax_bf16_fp32=agree(lg16, lg32), argmax_oracle_bf16=agree(lgo, lg16), rel_bf16_fp32=rel(lg16, lg32),
             rel_oracle_bf16=rel(lgo, lg16), rows=int(np.prod(lg16.shape[:-1])),
             digest=synth.digest(w['embed'], w['proj'], w['head'], w['bh'], w['q']))
    print('depth drift:', {k: v for k, v in d.items() if not k.startswith(('logits', 'forced'))}, flush=True)
    out['depth_drift'] = d


def _fix_depth_masks(g):
    mn = torch.finfo(torch.bfloat16).min
    S = g.max_seq
    key = torch.arange(S)
    pm = torch.where(key[None, :] <= torch.arange(2)[:, None], 0.0, mn).to(torch.bfloat16)
    g.prefill_attn = pm[None, None].expand(g.batch_size, 1, 2, S).contiguous()
    g.decode_attn = [torch.where(key <= int(p[0]), 0.0, mn).to(torch.bfloat16).view(1, 1, 1, S)
                     .expand(g.batch_size, 1, 1, S).contiguous() for p in g.decode_cache_positions]


def gold_sampler(out):
    import models.cudagraph.depth_decoder_graph as ddg
    c = synth.SAMPLER
    lc, lu, q, params = synth.sampler_cases()
    V = c['vocab']
    toks = []
    for r, (gs, temp, topk, topp, ds) in enumerate(params):
        # the official sampler, bound to a minimal object with the buffers it reads (B = 2, half = 1)
        o = type('S', (), {})()
        o.batch_size, o.half, o.vocab_size, o.codec_codebook_size = 2, 1, V, c['codebook_size']
        o.guidance_scale = torch.tensor([[gs]])
        o.temperature_buf = torch.tensor([[temp]])
        o.top_k_buf = torch.tensor([[topk]])
        o.top_p_buf = torch.tensor([[topp]])
        o.do_sample_buf = torch.tensor([ds])
        o._max_k = min(1024, V)
        o._topk_ranks = torch.arange(o._max_k)
        o._debug_probs_slot = None
        o._tok_buf = torch.zeros(2, dtype=torch.long)
        logits = torch.stack([lc[r], lu[r]])[:, None, :].clone()
        mult, _ = _patched_multinomial([q[r][None]])
        orig = ddg.torch.multinomial
        ddg.torch.multinomial = mult
        try:
            ddg.DepthDecoderGraph._cfg_sample(o, logits)
        finally:
            ddg.torch.multinomial = orig
        toks.append(int(o._tok_buf[0].clamp(0, V - 1)))
    out['sampler'] = dict(tokens=np.asarray(toks, np.int64), digest=synth.digest(lc, lu, q))


def gold_bb_sampler(out):
    """The reference's backbone sampler flash/sampling.py sample_logits (host-sync-free, bitwise equal to the
    official one), loaded from its file, with torch.multinomial(probs, 1) -> argmax(probs / q)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location('ref_flash_sampling', os.path.join(REF_ROOT[0], 'flash',
                                                                                      'sampling.py'))
    fs = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fs)
    c = synth.BB_SAMPLER
    x, present, q, params = synth.bb_sampler_cases()
    sup = torch.tensor(c['suppress'], dtype=torch.long)
    toks, oks = [], []
    for r, (pen, temp, topk, topp, ds, use_sup) in enumerate(params):
        qr = q[r][None]

        def mult(probs, n, *a, **kw):
            return torch.argmax(probs / qr.to(probs.dtype), dim=-1, keepdim=True)

        orig = fs.torch.multinomial
        fs.torch.multinomial = mult
        try:
            tok, ok = fs.sample_logits(x[r][None].clone(), temperature=temp, top_k=topk, top_p=topp, do_sample=bool(ds),
                                       present=present[r][None], repetition_penalty=pen,
                                       suppress_idx=sup if use_sup else None)
        finally:
            fs.torch.multinomial = orig
        toks.append(int(tok.reshape(-1)[0]))
        oks.append(int(bool(ok)))
    out['bb_sampler'] = dict(tokens=np.asarray(toks, np.int64), ok=np.asarray(oks, np.int64),
                             digest=synth.digest(x, present.to(torch.uint8), q))


def gold_prefill(out):
    from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward
    c = synth.PREFILL
    q, k, v, mask = synth.prefill_inputs()
    o, _ = eager_attention_forward(_Mod(c['NH'] // c['NKV']), q, k, v, mask, scaling=c['D'] ** -0.5)
    out['prefill'] = dict(out=synth.np_bits(o), digest=synth.digest(q, k, v, mask))


def gold_ln12(out):
    """The reference's LN12 encoder (``flash/ln12_format.py``: choose_lut, encode, to_inline) on a matrix with the
    format's special cases (shifted row tables, patches, overflow patches)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location('ref_ln12', os.path.join(REF_ROOT[0], 'flash', 'ln12_format.py'))
    fmt = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fmt)
    w = synth.ln12_matrix()
    u = w.contiguous().view(torch.int16).numpy().view(np.uint16)
    lut = fmt.choose_lut(u)
    packed, hdr, pat = fmt.encode(u, lut)
    meta, ovf = fmt.to_inline(hdr, pat)
    assert np.array_equal(fmt.decode(packed, hdr, pat, lut, *u.shape), u), 'reference LN12 round trip'
    out['ln12'] = dict(data=packed, meta=meta, ovf=ovf, lut=np.asarray(lut, np.uint8), hdr=hdr, patches=pat,
                       digest=synth.digest(w))


def gold_prefill_forward(out):
    """The reference's own prefill forward (``BackbonePrefillGraphCache._forward``, official modules in bf16 on the
    CPU) on the BACKBONE weights: hidden states, last-token logits and the cache slots it wrote."""
    from models.cudagraph.backbone_prefill_graph import BackbonePrefillGraphCache
    c = synth.BACKBONE
    w = synth.backbone_weights()
    g = _official_backbone(c, w, torch.bfloat16)
    pf = object.__new__(BackbonePrefillGraphCache)       # the constructor asks for a CUDA graph pool
    pf.backbone_graph, pf.model, pf.lm_head = g, g.model, g.lm_head
    emb, mask, pos, cp = synth.prefill_forward_inputs()
    # the reference's own mask builder gives the same mask
    am = (pos >= 0) & torch.ones_like(pos, dtype=torch.bool)
    for b, pad in enumerate(synth.PREFILL_FWD['pads']):
        am[b, :pad] = False
    chk = torch.empty_like(mask)
    BackbonePrefillGraphCache._update_causal_mask(am.long(), chk)
    assert torch.equal(chk, mask), 'the test mask differs from the reference prefill mask'
    L = emb.shape[1]
    with torch.inference_mode():
        for layer in g.static_cache.layers:
            layer.keys.zero_()
            layer.values.zero_()
            # transformers 5.x StaticLayer.update writes at its own running length instead of the cache_position
            # argument (4.57.3, which the reference pins, writes at cache_position = arange(L)): start it at 0
            if hasattr(layer, 'cumulative_length'):
                layer.cumulative_length.zero_()
        h, lg = pf._forward(emb, mask, pos, cp)
        ks = np.stack([synth.np_bits(layer.keys[:, :, :L]) for layer in g.static_cache.layers])
        vs = np.stack([synth.np_bits(layer.values[:, :, :L]) for layer in g.static_cache.layers])
        past = sum(float(layer.keys[:, :, L:].abs().sum()) for layer in g.static_cache.layers)
    assert past == 0.0, 'the prefill wrote past its slots'
    out['prefill_fwd'] = dict(hidden=synth.np_bits(h), logits=lg.numpy().copy(), keys=ks, values=vs,
                              digest=synth.digest(emb, mask, pos, w['embed'], w['lm_head']))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('BREEZE_REF'),
                    help='root of the reference checkout (or set BREEZE_REF)')
    ap.add_argument('--only', default='', help='comma-separated fixture names to regenerate (default: all)')
    args = ap.parse_args()
    if not args.ref:
        ap.error('the reference checkout is required: pass --ref or set BREEZE_REF')
    ref_env(args.ref)
    torch.manual_seed(0)
    out = {}
    only = set(args.only.split(',')) if args.only else None
    for fn in (gold_attention, gold_attention1, gold_gemv, gold_gemv2, gold_backbone, gold_depth, gold_sampler,
               gold_prefill, gold_drift, gold_depth_drift, gold_bb_sampler, gold_prefill_forward, gold_ln12):
        if only and fn.__name__[len('gold_'):] not in only:
            continue
        fn(out)
        print('ok', fn.__name__, flush=True)
    for name, d in out.items():
        np.savez_compressed(os.path.join(HERE, f'{name}.npz'), **{k: np.asarray(v) for k, v in d.items()})
    print('wrote', sorted(out))


if __name__ == '__main__':
    main()
