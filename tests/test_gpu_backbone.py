"""GPU parity of the whole backbone decode step (``flashb.backbone.fused_decode_step``) against the oracle, its
CUDA-graph capture, the device-side position advance, and run-to-run determinism."""
import numpy as np
import pytest
import torch

from gpu_util import E2E_TOL, assert_argmax_agree, assert_close, np32
from oracle import decode as dec

pytestmark = pytest.mark.gpu


def _graph(layers=2, S=1024, valid=300, seed=2, B=2):
    from flashb.engine import BackboneConfig, SyntheticBackboneGraph
    cfg = BackboneConfig(layers=layers)
    g = SyntheticBackboneGraph(cfg, batch_size=B, max_seq_len=S, seed=seed)
    g.fill_kv(valid)
    ids = torch.randint(0, cfg.vocab, (B, 1, cfg.codebooks), generator=torch.Generator().manual_seed(seed + 1))
    g.input_ids_buf.copy_(ids.cuda())
    return g


def _oracle(g):
    st = g._bb_state
    layers = []
    for L in st['layers']:
        layers.append(dict(ln1=np32(L.ln1_w), wq=np32(L.wq), wk=np32(L.wk), wv=np32(L.wv), qn=np32(L.qn_w),
                           kn=np32(L.kn_w), wo=np32(L.wo), ln2=np32(L.ln2_w), wg=np32(L.wg), wu=np32(L.wu),
                           wd=np32(L.wd)))
    W = dec.BackboneWeights(layers, np32(g.norm_w), np32(g.embed), g.lm_head32.cpu().numpy(), g.cfg.vocab,
                            g.cfg.eps, g.cfg.theta)
    kcs = [np32(L.keys).copy() for L in g.static_cache.layers]
    vcs = [np32(L.values).copy() for L in g.static_cache.layers]
    return W, kcs, vcs


def test_backbone_step_matches_oracle():
    g = _graph(layers=2)
    W, kcs, vcs = _oracle(g)
    pos = int(g.cache_position.item())
    h_ref, lg_ref, cfg_ref = dec.backbone_step(W, g.input_ids_buf.view(2, -1).cpu().numpy(), kcs, vcs,
                                               np32(g.attn_mask), pos, g.position_ids.view(-1).cpu().numpy(),
                                               float(g.guidance_scale.item()))
    g.decode_step()
    torch.cuda.synchronize()
    assert_close(np32(g.hidden_buf).reshape(2, -1), h_ref, what='hidden')
    assert_close(g.logits_buf.cpu().numpy(), lg_ref, what='logits')
    assert_close(g.cfg_logits_buf.cpu().numpy(), cfg_ref, what='cfg logits')
    for li in range(2):
        assert_close(np32(g.static_cache.layers[li].keys)[:, :, pos], kcs[li][:, :, pos], what='k write')
    assert_argmax_agree(g.logits_buf.cpu().numpy(), lg_ref, what='logits')


def test_backbone_graph_capture_and_advance_match_eager():
    """Three captured steps (advance + step) replayed equal three eager steps, bit for bit."""
    ga = _graph(layers=3, S=512, valid=100, seed=5)
    gb = _graph(layers=3, S=512, valid=100, seed=5)
    for _ in range(3):
        ga.decode_step(advance=True)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gb.decode_step(advance=True)   # warm-up (first step) outside the graph
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            gb.decode_step(advance=True)
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert int(ga.cache_position.item()) == int(gb.cache_position.item()) == 103
    assert torch.equal(ga.cfg_logits_buf, gb.cfg_logits_buf)
    assert torch.equal(ga.hidden_buf, gb.hidden_buf)
    for la, lb in zip(ga.static_cache.layers, gb.static_cache.layers):
        assert torch.equal(la.keys, lb.keys) and torch.equal(la.values, lb.values)


@pytest.mark.parametrize('S', [256, 1024, 4096])
def test_backbone_full_depth_per_layer_parity(S):
    """28 layers at the config 3 KV sweep (cache length S, position S - 1): every layer of the GPU step, fed the
    GPU's own input for that layer, matches the oracle layer within the bf16 bar; so does the final norm + fp32
    lm_head + CFG on the GPU's final residual.
    (Comparing only the end of 28 chained layers measures the compounding of 1-ulp bf16 rounding flips, not the
    parity of any kernel; that end-to-end drift is bounded separately below.)"""
    from flashb import backbone as bbm
    from flashb import kernels
    g = _graph(layers=28, S=S, valid=S - 1)
    W, kcs, vcs = _oracle(g)
    st = g._bb_state
    B, pos = 2, S - 1
    fx = kernels.fused()
    fx.embed_rope(g.input_ids_buf.view(B, -1), st['vocab'], st['embed'], g.position_ids.view(-1), st['cos_tab'],
                  st['sin_tab'], st['x0'], st['cos'], st['sin'])
    pids = g.position_ids.view(-1).cpu().numpy()
    cos, sin = dec.rope_tables(W.theta, 128, pids)
    cos, sin = cos.reshape(B, 1, 128), sin.reshape(B, 1, 128)
    mask = np32(g.attn_mask)
    x = st['x0'].clone()
    torch.cuda.synchronize()
    assert_close(np32(x), dec.embed_sum(W.embed, g.input_ids_buf.view(B, -1).cpu().numpy(), W.vocab), what='embed')
    for li, (L, KV) in enumerate(zip(st['layers'], g.static_cache.layers)):
        sub = dict(st)
        sub['layers'] = [L]
        xin = x.clone()
        x = bbm.run_layers(sub, xin, [(KV.keys, KV.values)], g.attn_mask, g.cache_position).clone()
        torch.cuda.synchronize()
        ref = dec.backbone_layer(np32(xin), W.layers[li], kcs[li], vcs[li], mask, pos, cos, sin, W.eps, 128 ** -0.5)
        assert_close(np32(x), ref, what=f'layer {li}')
    fx.lm_head_cfg(x, st['norm_w'], st['norm_eps'], st['lm_head32'], g.guidance_scale, g.hidden_buf.view(B, -1),
                   g.logits_buf, g.cfg_logits_buf)
    torch.cuda.synchronize()
    h = dec.rmsnorm(np32(x), W.norm, W.eps)
    lg = dec.lm_head_fp32(h, W.lm_head32)
    assert_close(g.logits_buf.cpu().numpy(), lg, what='lm_head')
    assert_close(g.cfg_logits_buf.cpu().numpy(), dec.cfg_combine(lg, 1, float(g.guidance_scale.item())), what='cfg')


@pytest.mark.parametrize('S', [256, 1024, 4096])
def test_backbone_step_full_depth_argmax_and_determinism(S):
    """28 chained layers end to end at the config 3 KV sweep: the logits' argmax agrees with the oracle's on every
    row, the compounded drift stays within E2E_TOL of max |logit| (each layer alone is held to 1e-2 above), and two
    runs are bitwise equal."""
    g = _graph(layers=28, S=S, valid=S - 1)
    W, kcs, vcs = _oracle(g)
    pos = S - 1
    h_ref, lg_ref, cfg_ref = dec.backbone_step(W, g.input_ids_buf.view(2, -1).cpu().numpy(), kcs, vcs,
                                               np32(g.attn_mask), pos, g.position_ids.view(-1).cpu().numpy(),
                                               float(g.guidance_scale.item()))
    k0 = [L.keys.clone() for L in g.static_cache.layers]
    g.decode_step()
    torch.cuda.synchronize()
    first = g.cfg_logits_buf.clone()
    assert_close(g.logits_buf.cpu().numpy(), lg_ref, tol=E2E_TOL, what='28-layer logits (compounded)')
    assert_close(g.cfg_logits_buf.cpu().numpy(), cfg_ref, tol=E2E_TOL, what='28-layer cfg logits (compounded)')
    assert_argmax_agree(g.logits_buf.cpu().numpy(), lg_ref, what='28-layer logits')
    for L, k in zip(g.static_cache.layers, k0):
        L.keys.copy_(k)
    g.decode_step()
    torch.cuda.synchronize()
    assert torch.equal(first, g.cfg_logits_buf)
