"""The drop-in boundary against the reference's OWN official classes, on the CPU.

flashb's hooks patch ``BackboneGraph``, ``DepthDecoderGraph`` and ``BackbonePrefillGraphCache`` of the reference's
vendored runtime, as the reference's hook package does (``flash/__init__.py``, ``flash/backbone.py``,
``flash/depth.py``, ``flash/prefill_attn.py``).  These tests import the official classes from a reference checkout,
build small official objects on the CPU (the shapes of tests/golden/synth.py), install flashb's hooks and check:

* the methods are swapped and the originals kept;
* every attribute the hooks read exists on the official objects and resolves to the official weights (the backbone
  state of ``_prep``, the depth kernel's weight list built through ``_DepthShim`` / ``DepthMegakernel``, the
  buffers ``_full_loop_mk`` passes to the kernel);
* the prefill hook is reached through the official ``_forward`` (on CPU tensors it hands the work to the eager
  attention, so the official output is reproduced exactly).

No kernel runs (there is no GPU here).  The reference checkout is found through ``BREEZE_REF`` or, failing that, a
directory named ``reference`` beside this repository; without one the tests are skipped.
"""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _ref_root():
    r = os.environ.get('BREEZE_REF') or os.path.join(os.path.dirname(REPO), 'reference')
    return r if os.path.isdir(os.path.join(r, 'third_party', 'breeze-tts', 'models')) else None


ROOT = _ref_root()
pytestmark = pytest.mark.skipif(ROOT is None, reason='no reference checkout (set BREEZE_REF)')


@pytest.fixture(scope='module')
def mg():
    sys.path.insert(0, os.path.join(HERE, 'golden'))
    import make_golden
    make_golden.ref_env(ROOT)
    return make_golden


def test_backbone_hook_on_the_official_graph(mg):
    import synth
    from models.cudagraph.backbone_graph import BackboneGraph
    from flashb import backbone as bb
    c = synth.BACKBONE
    w = synth.backbone_weights()
    g = mg._official_backbone(c, w, torch.bfloat16)
    orig = BackboneGraph._decode_step
    bb.install()
    try:
        assert BackboneGraph._decode_step is bb.fused_decode_step
        assert bb.ORIG['_decode_step'] is orig
        # on the CPU the hook hands the step back to the official method, as for any graph it does not cover
        assert bb._prep(g) is None
        got = bb.weights_of(g)
        assert got is not None, 'the official graph must be eligible for the fused step'
        Ls, norm, table, lm_w = got
        model = g.model
        assert g.batch_size == c['B'] and len(Ls) == len(model.layers) == c['L']
        for L, layer in zip(Ls, model.layers):
            at, mlp = layer.self_attn, layer.mlp
            assert L.wq is at.q_proj.weight and L.wk is at.k_proj.weight and L.wv is at.v_proj.weight
            assert L.wo is at.o_proj.weight and L.qn_w is at.q_norm.weight and L.kn_w is at.k_norm.weight
            assert L.wg is mlp.gate_proj.weight and L.wu is mlp.up_proj.weight and L.wd is mlp.down_proj.weight
            assert L.ln1_w is layer.input_layernorm.weight and L.ln2_w is layer.post_attention_layernorm.weight
            assert L.ln1_eps == c['eps'] and L.scaling == pytest.approx(c['D'] ** -0.5)
        assert table is g.embed_tokens.embed_audio_tokens.weight
        assert table.shape[0] // g.num_codebooks == c['vocab']
        assert lm_w is g.lm_head.weight and lm_w.dtype == torch.float32
        assert norm is model.norm and float(norm.variance_epsilon) == c['eps']
        # the rotary module the hook evaluates once per position of the static cache
        cos, sin = model.rotary_emb(torch.zeros(1, 5, 128, dtype=torch.bfloat16), torch.arange(5)[None])
        assert cos.shape[-1] == 128 and sin.shape[-1] == 128
        # the buffers fused_decode_step reads and writes on the official graph
        for name in ('input_ids_buf', 'position_ids', 'cache_position', 'attn_mask', 'hidden_buf', 'logits_buf',
                     'cfg_logits_buf', 'guidance_scale', 'static_cache', 'max_seq_len', 'num_codebooks'):
            assert hasattr(g, name), name
        assert all(hasattr(L, 'keys') and hasattr(L, 'values') for L in g.static_cache.layers)
        assert g.static_cache.layers[0].keys.shape == (c['B'], c['NKV'], c['S'], c['D'])
    finally:
        BackboneGraph._decode_step = orig
        bb.ORIG.pop('_decode_step', None)


def test_depth_hook_on_the_official_graph(mg):
    import synth
    from models.cudagraph import depth_decoder_graph as ddg
    from flashb import depth as fd
    cls = ddg.DepthDecoderGraph
    saved = {k: cls.__dict__[k] for k in ('capture', 'prepare_eager', 'set_top_k', '_full_loop')}
    c = synth.DEPTH
    w = synth.depth_weights()
    g, _ = mg._official_depth(c, w, torch.bfloat16)
    fd.install()
    try:
        assert cls._full_loop is not saved['_full_loop'] and cls.prepare_eager is not saved['prepare_eager']
        g.prepare_eager()                     # the wrapped official method attaches the frame kernel
        mk = g._mega2
        assert mk is not None, 'the official graph must be eligible for the frame kernel'
        layers, embed, proj, normf, head_t, cos, sin, eps, scaling, cb = mk.ops.args
        dm = g.depth_model
        assert len(layers) == len(dm.layers) == c['L']
        for L, layer in zip(layers, dm.layers):
            at, mlp = layer.self_attn, layer.mlp
            assert torch.equal(L['wq'], at.q_proj.weight) and torch.equal(L['wo'], at.o_proj.weight)
            assert torch.equal(L['wg'], mlp.gate_proj.weight) and torch.equal(L['wd'], mlp.down_proj.weight)
            assert torch.equal(L['ln1'], layer.input_layernorm.weight)
        assert torch.equal(embed, dm.embed_tokens.weight) and torch.equal(proj, dm.inputs_embeds_projector.weight)
        assert torch.equal(normf, dm.norm.weight)
        # heads transposed once to [n_decode, vocab, hidden], bf16-exact
        assert torch.equal(head_t.float(), w['head'].permute(0, 2, 1))
        assert head_t.shape == (c['ncb'] - 1, c['vocab'], c['H'])
        assert cb == c['codebook_size'] and eps == pytest.approx(c['eps'])
        # the official buffers _full_loop_mk hands to the kernel
        for name in ('first_cb_token_buf', 'backbone_hidden_buf', '_tok_buf', 'output_tokens', 'temperature_buf',
                     'top_k_buf', 'top_p_buf', 'do_sample_buf', 'guidance_scale', 'num_decode_codebooks',
                     'batch_size', 'vocab_size'):
            assert hasattr(g, name), name
        assert g._mk2_q[c['B']].shape == (g.num_decode_codebooks, c['B'] // 2, g.vocab_size)
        assert g.output_tokens.shape[-1] == g.num_decode_codebooks == c['ncb'] - 1
        with pytest.raises(ValueError):
            g.set_top_k(2000)                 # beyond the frame sampler's top-k range
    finally:
        for k, v in saved.items():
            setattr(cls, k, v)
        if '_flash_depth' in cls.__dict__:
            delattr(cls, '_flash_depth')


def test_prefill_hook_through_the_official_forward(mg, monkeypatch):
    import synth
    from transformers import AttentionInterface
    from models.cudagraph.backbone_prefill_graph import BackbonePrefillGraphCache
    from flashb import prefill_attn as pa
    c = synth.BACKBONE
    w = synth.backbone_weights()
    g = mg._official_backbone(c, w, torch.bfloat16)
    # the cache's constructor asks for a CUDA graph pool; _forward only needs model, lm_head and the graph
    pf = object.__new__(BackbonePrefillGraphCache)
    pf.backbone_graph, pf.model, pf.lm_head = g, g.model, g.lm_head
    B, L, S = c['B'], 8, c['S']
    gen = torch.Generator().manual_seed(5)
    emb = torch.randn(B, L, c['H'], generator=gen).to(torch.bfloat16)
    am = torch.ones(B, L, dtype=torch.long)
    causal = torch.empty(B, 1, L, S, dtype=torch.bfloat16)
    BackbonePrefillGraphCache._update_causal_mask(am, causal)
    pos = torch.arange(L)[None].repeat(B, 1)
    cp = torch.arange(L)

    def run():
        with torch.inference_mode():
            for layer in g.static_cache.layers:
                layer.keys.zero_()
                layer.values.zero_()
            return pf._forward(emb, causal, pos, cp)

    h_ref, lg_ref = run()
    saved = BackbonePrefillGraphCache.__dict__['_forward']
    calls = []
    trim = pa._trim
    monkeypatch.setattr(pa, '_trim', lambda *a: calls.append(1) or trim(*a))
    pa.install()
    try:
        assert AttentionInterface._global_mapping[pa.NAME] is pa.bz_prefill_attention
        h, lg = run()
        assert len(calls) == c['L'], 'the hook must serve every layer of the official prefill'
        # CPU tensors go to the eager attention after the reference's key trimming: the same output
        assert torch.equal(h, h_ref) and np.array_equal(lg.numpy(), lg_ref.numpy())
        assert g.model.layers[0].self_attn.config._attn_implementation != pa.NAME   # restored after the call
    finally:
        BackbonePrefillGraphCache._forward = saved
        if '_pf_installed' in BackbonePrefillGraphCache.__dict__:
            delattr(BackbonePrefillGraphCache, '_pf_installed')


def test_whole_prefill_hook_on_the_official_cache(mg):
    """flashb.prefill replaces ``BackbonePrefillGraphCache._forward``; on CPU tensors it hands the call to the
    official forward (the flashb path needs the GPU), whose output is unchanged."""
    import synth
    from models.cudagraph.backbone_prefill_graph import BackbonePrefillGraphCache
    from flashb import prefill as fpf
    c = synth.BACKBONE
    w = synth.backbone_weights()
    g = mg._official_backbone(c, w, torch.bfloat16)
    pf = object.__new__(BackbonePrefillGraphCache)
    pf.backbone_graph, pf.model, pf.lm_head = g, g.model, g.lm_head
    emb, mask, pos, cp = synth.prefill_forward_inputs()

    def run():
        with torch.inference_mode():
            for layer in g.static_cache.layers:
                layer.keys.zero_()
                layer.values.zero_()
                if hasattr(layer, 'cumulative_length'):
                    layer.cumulative_length.zero_()
            return pf._forward(emb, mask, pos, cp)

    h_ref, lg_ref = run()
    saved = BackbonePrefillGraphCache.__dict__['_forward']
    fpf.install()
    try:
        assert BackbonePrefillGraphCache._forward is fpf.fused_prefill_forward
        assert fpf.ORIG['_forward'] is saved
        # the state the flashb path would use resolves to the official weights (the decode hook's reading)
        from flashb import backbone as bb
        Ls, norm, _, lm_w = bb.weights_of(g)
        assert Ls[0].wq is g.model.layers[0].self_attn.q_proj.weight and lm_w is g.lm_head.weight
        h, lg = run()
        assert torch.equal(h, h_ref) and torch.equal(lg, lg_ref)
    finally:
        BackbonePrefillGraphCache._forward = saved
        fpf.ORIG.pop('_forward', None)
