"""GPU parity of the tcgen05 causal GQA prefill attention (``flashb_prefill_attn``) against the reference's eager
outputs (golden fixture) and the oracle: config 5 shapes, ragged lengths, left padding, fp32 and bf16 masks,
strided q, the reference's key trimming, head-range shards, and run-to-run determinism.  Bar: max |gpu - ref| <=
1e-2 * max |ref| on rows with a live key (fully masked rows are 0 on both sides)."""
import numpy as np
import pytest
import torch

import synth
from gpu_util import E2E_TOL, TOL, assert_argmax_agree, assert_close, np32
from oracle import prefill as opf
from oracle.bf16 import bits_to_f32

pytestmark = pytest.mark.gpu


def _pf():
    from flashb import prefill_attn
    return prefill_attn


def _mask(B, L, S, pads, dtype=torch.bfloat16, causal=True):
    qi = torch.arange(L).view(L, 1)
    ki = torch.arange(S).view(1, S)
    m = torch.full((B, 1, L, S), torch.finfo(torch.bfloat16).min, dtype=torch.float32)
    for b, p in enumerate(pads):
        allowed = (ki >= p) & ((ki <= qi) if causal else torch.ones_like(ki, dtype=torch.bool))
        m[b, 0].masked_fill_(allowed, 0.0)
    return m.to(dtype)


def _live(B, L, pads):
    live = np.ones((B, L), bool)
    for b, p in enumerate(pads):
        live[b, :p] = False
    return live


def _inputs(B, NH, NKV, L, S, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, NH, L, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, NKV, S, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, NKV, S, 128, generator=g).to(torch.bfloat16)
    return q, k, v


def test_prefill_matches_reference_golden():
    z = np.load(synth.__file__.replace('synth.py', 'prefill.npz'))
    q, k, v, m = synth.prefill_inputs()
    c = synth.PREFILL
    out = _pf().prefill_attention(q.cuda(), k.cuda(), v.cuda(), m.cuda(), c['D'] ** -0.5)
    torch.cuda.synchronize()
    got = np32(out)
    ref = bits_to_f32(z['out'])
    live = _live(c['B'], c['L'], c['pad'])
    assert_close(got[live], ref[live], what='prefill vs reference eager')
    assert np.all(got[~live] == 0)


@pytest.mark.parametrize('L,pads', [(512, (0, 37)), (300, (5, 0)), (129, (0, 0)), (1, (0, 0))])
def test_prefill_matches_oracle(L, pads):
    B, NH, NKV = 2, 16, 4
    q, k, v = _inputs(B, NH, NKV, L, L, seed=L)
    m = _mask(B, L, L, pads)
    out = _pf().prefill_attention(q.cuda(), k.cuda(), v.cuda(), m.cuda(), 128 ** -0.5)
    torch.cuda.synchronize()
    ref = opf.prefill_attention(np32(q), np32(k), np32(v), np32(m), 128 ** -0.5)
    live = _live(B, L, pads)
    assert_close(np32(out)[live], ref[live], what=f'L={L}')
    assert_argmax_agree(np32(out)[live], ref[live], what=f'L={L}')


@pytest.mark.parametrize('L,pads,masked', [(700, (0, 45), True), (640, (0, 0), False)])
def test_prefill_kept_and_recomputed_tiles(L, pads, masked):
    """More key tiles than pass 1 keeps in TMEM (four): pass 2 reads the first four tiles' scores back and
    recomputes S for the rest, and pass 1 alternates its two S / K buffers over an odd and an even tile count.  A
    bf16 causal mask with left padding, and no mask at all (non-causal, every key of every row)."""
    B, NH, NKV = 2, 8, 2
    q, k, v = _inputs(B, NH, NKV, L, L, seed=L + 1)
    if masked:
        m = _mask(B, L, L, pads)
        out = _pf().prefill_attention(q.cuda(), k.cuda(), v.cuda(), m.cuda(), 128 ** -0.5)
        ref = opf.prefill_attention(np32(q), np32(k), np32(v), np32(m), 128 ** -0.5)
    else:
        out = _pf().prefill_attention(q.cuda(), k.cuda(), v.cuda(), None, 128 ** -0.5, causal=False)
        ref = opf.prefill_attention(np32(q), np32(k), np32(v), None, 128 ** -0.5)
    torch.cuda.synchronize()
    live = _live(B, L, pads)
    assert_close(np32(out)[live], ref[live], what=f'L={L}')
    assert_argmax_agree(np32(out)[live], ref[live], what=f'L={L}')


def test_prefill_fp32_mask_noncausal_and_no_mask():
    B, NH, NKV, L = 2, 8, 2, 200
    q, k, v = _inputs(B, NH, NKV, L, L, seed=7)
    pf = _pf()
    m32 = _mask(B, L, L, (3, 0), dtype=torch.float32, causal=False)
    out = pf.prefill_attention(q.cuda(), k.cuda(), v.cuda(), m32.cuda(), 128 ** -0.5, causal=False)
    ref = opf.prefill_attention(np32(q), np32(k), np32(v), m32.numpy(), 128 ** -0.5, mask_bf16=False)
    live = _live(B, L, (3, 0))
    torch.cuda.synchronize()
    assert_close(np32(out)[live], ref[live], what='fp32 mask, non-causal')
    out2 = pf.prefill_attention(q.cuda(), k.cuda(), v.cuda(), None, 128 ** -0.5, causal=True)
    ref2 = opf.prefill_attention(np32(q), np32(k), np32(v), np32(_mask(B, L, L, (0, 0))), 128 ** -0.5)
    torch.cuda.synchronize()
    assert_close(np32(out2), ref2, what='no mask, causal flag')


def test_bz_prefill_trims_keys_and_takes_strided_q():
    """The hook: q as the transposed view the layer produces, K/V of a longer static cache with a mask over every
    slot -> trimmed to L exactly as the reference does."""
    B, NH, NKV, L, S = 2, 16, 4, 160, 384
    g = torch.Generator().manual_seed(11)
    q_lin = torch.randn(B, L, NH * 128, generator=g).to(torch.bfloat16).cuda()
    q = q_lin.view(B, L, NH, 128).transpose(1, 2)
    k = torch.randn(B, NKV, S, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, NKV, S, 128, generator=g).to(torch.bfloat16).cuda()
    m = _mask(B, L, S, (0, 9)).cuda()
    out, w = _pf().bz_prefill_attention(None, q, k, v, m, scaling=128 ** -0.5)
    torch.cuda.synchronize()
    assert w is None and out.shape == (B, L, NH, 128)
    ref = opf.prefill_attention(np32(q), np32(k), np32(v), np32(m), 128 ** -0.5)
    live = _live(B, L, (0, 9))
    assert_close(np32(out)[live], ref[live], what='trimmed hook')


def test_prefill_head_shard_and_determinism():
    B, NH, NKV, L = 2, 16, 4, 256
    q, k, v = _inputs(B, NH, NKV, L, L, seed=5)
    m = _mask(B, L, L, (0, 0)).cuda()
    pf = _pf()
    full = pf.prefill_attention(q.cuda(), k.cuda(), v.cuda(), m, 128 ** -0.5)
    again = pf.prefill_attention(q.cuda(), k.cuda(), v.cuda(), m, 128 ** -0.5)
    h0, h1 = pf.shard_heads(NH, NKV, 4, 2)
    part = torch.zeros(B, L, h1 - h0, 128, dtype=torch.bfloat16, device='cuda')
    pf.prefill_attention(q.cuda(), k.cuda(), v.cuda(), m, 128 ** -0.5, heads=(h0, h1), out=part)
    torch.cuda.synchronize()
    assert torch.equal(full, again)
    assert torch.equal(part, full[:, :, h0:h1])


# ------------------------------------------------------------------------------------------------ the whole prefill
def _prefill_case(hidden, heads, kv_heads, ffn, layers, B, L, S, pads, seed):
    """A synthetic backbone (flashb.engine) with its decode state, prompt embeddings, the reference prefill's
    left-padding positions and causal mask (``BackbonePrefillGraphCache._copy_inputs`` / ``_update_causal_mask``)."""
    from flashb.engine import BackboneConfig, SyntheticBackboneGraph
    cfg = BackboneConfig(hidden=hidden, layers=layers, heads=heads, kv_heads=kv_heads, ffn=ffn)
    g = SyntheticBackboneGraph(cfg, batch_size=B, max_seq_len=S, seed=seed)
    for Lc in g.static_cache.layers:
        Lc.keys.zero_()
        Lc.values.zero_()
    gen = torch.Generator().manual_seed(seed + 7)
    emb = torch.randn(B, L, hidden, generator=gen).to(torch.bfloat16)
    am = torch.ones(B, L, dtype=torch.long)
    for b, p in enumerate(pads):
        am[b, :p] = 0
        emb[b, :p] = 0
    pos = am.cumsum(-1) - 1
    pos.masked_fill_(am == 0, 1)
    qi, ki = torch.arange(L).view(1, L, 1), torch.arange(S).view(1, 1, S)
    valid = torch.zeros(B, S, dtype=torch.bool)
    valid[:, :L] = am.bool()
    allowed = (ki <= qi) & valid[:, None, :]
    mask = torch.full((B, 1, L, S), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    mask[:, 0].masked_fill_(allowed, 0.0)
    return g, emb, mask, pos, torch.arange(L)


def _run_prefill(g, emb, mask, pos, cp):
    from flashb import prefill as fpf
    st = g._bb_state
    kv = [(Lc.keys, Lc.values) for Lc in g.static_cache.layers]
    h, lg = fpf.prefill_forward(st, emb.cuda(), mask.cuda(), pos.cuda(), cp.cuda(), kv)
    torch.cuda.synchronize()
    return h, lg, kv


def _oracle_prefill(g, emb, mask, pos, cp):
    from oracle import decode as dec
    st = g._bb_state
    layers = [dict(ln1=np32(L.ln1_w), wq=np32(L.wq), wk=np32(L.wk), wv=np32(L.wv), qn=np32(L.qn_w), kn=np32(L.kn_w),
                   wo=np32(L.wo), ln2=np32(L.ln2_w), wg=np32(L.wg), wu=np32(L.wu), wd=np32(L.wd))
              for L in st['layers']]
    W = dec.BackboneWeights(layers, np32(g.norm_w), np32(g.embed), g.lm_head32.cpu().numpy(), g.cfg.vocab, g.cfg.eps,
                            g.cfg.theta)
    kcs = [np32(Lc.keys).copy() for Lc in g.static_cache.layers]
    vcs = [np32(Lc.values).copy() for Lc in g.static_cache.layers]
    h, lg = opf.prefill_forward(W, np32(emb), np32(mask), pos.numpy(), cp.numpy(), kcs, vcs)
    return h, lg, kcs, vcs


@pytest.mark.parametrize('hidden,heads,kv_heads,ffn,L,S,pads', [
    (512, 4, 2, 1024, 40, 96, [0, 7]),            # small: ragged tiles, left padding
    (2048, 16, 4, 6144, 512, 1024, [0, 37]),      # config 5's shapes (B 2, L 512, 16 q / 4 KV heads), 2 layers
])
def test_prefill_forward_matches_oracle(hidden, heads, kv_heads, ffn, L, S, pads):
    """The whole prefill (``BackbonePrefillGraphCache._forward``) on flashb kernels: hidden states of every live
    token, the last-token logits and every layer's cache slots [0, L) against the oracle's eager restatement.
    Layer 0's cache (one GEMM and the q|k|v tail) holds the kernel bar; the values after more layers hold the
    end-to-end bar of the decode tests (rare 1-ulp bf16 flips from another summation order compound through the
    layers, as the drift study of tests/golden/make_golden.py shows for the reference itself)."""
    g, emb, mask, pos, cp = _prefill_case(hidden, heads, kv_heads, ffn, 2, 2, L, S, pads, seed=11)
    h_ref, lg_ref, kcs, vcs = _oracle_prefill(g, emb, mask, pos, cp)
    h, lg, kv = _run_prefill(g, emb, mask, pos, cp)
    live = _live(2, L, pads)
    assert_close(np32(h)[live], h_ref[live], tol=E2E_TOL, what='prefill hidden (live tokens)')
    assert_close(lg.cpu().numpy(), lg_ref, what='prefill last-token logits')
    assert_argmax_agree(lg.cpu().numpy(), lg_ref, what='prefill logits')
    for li, (kc, vc) in enumerate(kv):
        kk, vv = np32(kc)[:, :, :L], np32(vc)[:, :, :L]
        for b, p in enumerate(pads):
            tol = TOL if li == 0 else E2E_TOL
            assert_close(kk[b, :, p:], kcs[li][b, :, p:L], tol=tol, what=f'layer {li} keys row {b}')
            assert_close(vv[b, :, p:], vcs[li][b, :, p:L], tol=tol, what=f'layer {li} values row {b}')
        assert float(kc[:, :, L:].abs().sum()) == 0.0, 'the prefill wrote past its slots'
    from flashb._native import device_error
    assert device_error() == 0


def test_prefill_forward_graph_capture_and_determinism():
    """Captured in a CUDA graph (as the reference captures ``_forward`` per length bucket) and replayed: the same
    bits as an eager call."""
    g, emb, mask, pos, cp = _prefill_case(512, 4, 2, 1024, 2, 2, 64, 128, [0, 3], seed=12)
    h0, lg0, _ = _run_prefill(g, emb, mask, pos, cp)
    h0, lg0 = h0.clone(), lg0.clone()
    from flashb import prefill as fpf
    st = g._bb_state
    kv = [(Lc.keys, Lc.values) for Lc in g.static_cache.layers]
    e, m, p, c = emb.cuda(), mask.cuda(), pos.cuda(), cp.cuda()
    hid = torch.empty_like(h0)
    lgo = torch.empty_like(lg0)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fpf.prefill_forward(st, e, m, p, c, kv, hidden_out=hid, logits_out=lgo)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            fpf.prefill_forward(st, e, m, p, c, kv, hidden_out=hid, logits_out=lgo)
    torch.cuda.current_stream().wait_stream(s)
    hid.zero_()
    lgo.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(hid, h0) and torch.equal(lgo, lg0)
    del graph


def test_prefill_query_tile_ranges_assemble_the_full_output():
    """The query-row split of a multi-GPU prefill (``row_shards`` ranges computed with ``tiles=``), run on one GPU
    range by range: every range writes exactly its rows, each equal to the whole call's, and the ranges of 8 ranks
    over L = 1000 cover every row."""
    pf = _pf()
    B, NH, NKV, L = 2, 8, 2, 1000
    q, k, v = _inputs(B, NH, NKV, L, L, seed=21)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    m = _mask(B, L, L, [0, 9]).cuda()
    full = pf.prefill_attention(q, k, v, m, 128 ** -0.5)
    ranges = pf.row_shards(L, 8)
    out = torch.full_like(full, float('nan'))
    for t0, t1 in ranges:
        if t1 > t0:
            rows = min(L, t1 * 128) - t0 * 128
            part = torch.full((B, rows, NH, 128), float('nan'), dtype=torch.bfloat16, device='cuda')
            pf.prefill_attention(q, k, v, m, 128 ** -0.5, out=part, tiles=(t0, t1))
            out[:, t0 * 128:t0 * 128 + rows] = part
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any()
    assert torch.equal(out, full)
