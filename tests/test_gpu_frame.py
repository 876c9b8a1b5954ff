"""GPU tests of the streaming-frame pieces: the greedy codebook-0 kernel (torch.argmax semantics), the frame-ids
assembly, and ``FrameEngine`` (graph-captured frames) against the oracle's backbone step, the C sampler oracle
(codebook 0 sampled with the reference runtime's parameters on the engine's own Exp(1) draws and token history) and
the standalone depth frame."""
import numpy as np
import pytest
import torch

from gpu_util import E2E_TOL, assert_close, np32
from oracle import decode as dec
from oracle import frame as ofr

pytestmark = pytest.mark.gpu


def _lib():
    from flashb._native import lib
    return lib()


def _greedy(cfg, half, n_valid, B):
    out = torch.full((B,), -1, dtype=torch.long, device='cuda')
    from flashb._native import check
    check(_lib().flashb_cb0_greedy(cfg.data_ptr(), cfg.stride(0), half, n_valid, B, out.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize('half,B', [(1, 2), (1, 1), (2, 4)])
def test_cb0_greedy_matches_torch_argmax(half, B):
    g = torch.Generator().manual_seed(half * 10 + B)
    cfg = torch.randn(half, 2049, generator=g)
    cfg[0, 2048] = 1e9                 # suppressed id (>= n_valid) must not win
    cfg[0, 700] = cfg[0, 300] = 50.0   # tie -> lower index
    if half > 1:
        cfg[1, 1500] = float('nan')    # NaN counts as the maximum (torch.argmax)
    got = _greedy(cfg.cuda(), half, 2048, B)
    for h in range(half):
        ref = int(torch.argmax(cfg[h, :2048]).item())
        assert ref == ofr.greedy_cb0(cfg[h].numpy(), 2048)
        assert got[h] == ref
        if B == 2 * half:
            assert got[h + half] == ref
    assert got[0] == 300
    if half > 1:
        assert got[1] == 1500


def test_frame_ids_assembly():
    from flashb._native import check
    B, C, n = 2, 17, 16
    fc = torch.tensor([5, 9], dtype=torch.long, device='cuda')
    dt = torch.arange(B * n, dtype=torch.long, device='cuda').view(B, n)
    ids = torch.full((B, C), -1, dtype=torch.long, device='cuda')
    check(_lib().flashb_frame_ids(fc.data_ptr(), dt.data_ptr(), n, B, C, ids.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = torch.cat([fc.view(B, 1), dt[:, :C - 1]], 1)
    assert torch.equal(ids, ref)


def _small_engine(streams=2, prompt=40, frames=4, group=1, lanes=1):
    from flashb.engine import BackboneConfig, DepthConfig, FrameEngine
    bcfg = BackboneConfig(hidden=512, layers=2, heads=8, kv_heads=2, ffn=1024, vocab=65, codebooks=7)
    dcfg = DepthConfig(hidden=256, embed_dim=512, layers=2, heads=2, kv_heads=1, ffn=512, vocab=64,
                       codebook_size=60, n_decode=6)
    eng = FrameEngine(bcfg, dcfg, streams, prompt, frames, seed=4, group=group, lanes=lanes)
    return eng


def _cb0_expected(eng, cfg_rows, c0, present_before):
    """Codebook 0 of sampler rows c0.. from their CFG logits: the C oracle of the backbone sampler with the engine's
    parameters, the draws it used (left in cb0_q) and the token history before the step."""
    from oracle import sampler as osmp
    p = eng.CB0_PARAMS
    q = eng.cb0_q.cpu().numpy()
    sup = list(range(eng.n_valid, eng.bcfg.vocab))
    out = []
    for k in range(cfg_rows.shape[0]):
        t, ok = osmp.bb_sample_row(cfg_rows[k], present_before[c0 + k], p['repetition_penalty'], sup,
                                   p['temperature'], p['top_k'], p['top_p'], p['do_sample'], q[c0 + k])
        assert ok == 1
        out.append(t)
    return out


def _oracle_backbone(bb):
    st = bb._bb_state
    layers = [dict(ln1=np32(L.ln1_w), wq=np32(L.wq), wk=np32(L.wk), wv=np32(L.wv), qn=np32(L.qn_w), kn=np32(L.kn_w),
                   wo=np32(L.wo), ln2=np32(L.ln2_w), wg=np32(L.wg), wu=np32(L.wu), wd=np32(L.wd))
              for L in st['layers']]
    return dec.BackboneWeights(layers, np32(bb.norm_w), np32(bb.embed), bb.lm_head32.cpu().numpy(), bb.cfg.vocab,
                               bb.cfg.eps, bb.cfg.theta)


@pytest.mark.parametrize('group,lanes', [(1, 1), (2, 1), (4, 1), (8, 1), (1, 2), (2, 3), (2, 6)])
def test_frame_engine_matches_oracle_and_standalone_depth(group, lanes):
    """group 2: two streams share one slot (rows [c0, c1, u0, u1]); every row must still match the oracle.
    lanes > 1: the slots' frames run on several CUDA streams side by side, each lane sized for part of the SMs."""
    n_slots = max(1, lanes) * (2 if lanes > 1 else 1)
    eng = _small_engine(streams=max(2, group) * n_slots if lanes > 1 else max(2, group), group=group, lanes=lanes)
    eng.capture()
    R = 2 * group
    W = _oracle_backbone(eng.streams[0].bb)
    C = eng.bcfg.codebooks
    state = []
    for st in eng.streams:
        bb = st.bb
        state.append(dict(mask=np32(bb.attn_mask).copy(), pos=int(bb.cache_position.item()),
                          pids=bb.position_ids.view(-1).cpu().numpy().copy()))
    for f in range(3):
        # each frame is checked from the device's own state (its KV cache so far), so the comparison is per frame and
        # does not compound earlier frames' rounding differences
        before = []
        present = eng.cb0_present.cpu().numpy().copy()
        for st in eng.streams:
            bb = st.bb
            before.append(dict(kcs=[np32(L.keys).copy() for L in bb.static_cache.layers],
                               vcs=[np32(L.values).copy() for L in bb.static_cache.layers],
                               ids=np.concatenate([st.first_cb.cpu().numpy()[:, None],
                                                   st.outtok.cpu().numpy()[:, :C - 1]], 1)))
        eng.step()
        torch.cuda.synchronize()
        for i, st in enumerate(eng.streams):
            bb, sv, bf = st.bb, state[i], before[i]
            np.testing.assert_array_equal(bb.input_ids_buf.view(R, -1).cpu().numpy(), bf['ids'])
            sv['pos'] += 1
            sv['pids'] += 1
            sv['mask'][..., sv['pos']] = 0.0
            gs = float(bb.guidance_scale.item())
            h, lg, _ = dec.backbone_step(W, bf['ids'], bf['kcs'], bf['vcs'], sv['mask'], sv['pos'], sv['pids'], gs)
            assert int(bb.cache_position.item()) == sv['pos']
            # the hidden state leaves a stack of layers, each held to 1e-2 alone (test_gpu_backbone); through the
            # stack 1-ulp bf16 flips of the residual adds compound, so it gets the stack's bound
            assert_close(np32(bb.hidden_buf).reshape(R, -1), h, tol=E2E_TOL, what=f'slot {i} frame {f} hidden')
            g_lg = bb.logits_buf.cpu().numpy()
            assert_close(g_lg, lg, what=f'slot {i} frame {f} logits')
            # CFG u + gs (c - u) amplifies logit rounding differences ~(2 gs - 1)x by construction; the combine
            # itself (three separately rounded fp32 ops) is checked exactly on the kernel's own logits
            g_cfg = bb.cfg_logits_buf.cpu().numpy()
            np.testing.assert_array_equal(g_cfg, dec.cfg_combine(g_lg, group, gs))
            cb0 = _cb0_expected(eng, g_cfg, st.c0, present)
            np.testing.assert_array_equal(st.first_cb.cpu().numpy(), cb0 + cb0)
            # the engine's depth launch consumed this frame's hidden state and cb0: a standalone launch agrees
            d = eng.depth
            out = torch.zeros_like(st.outtok)
            tb = torch.zeros_like(st.tokbuf)
            st.desc.frame(st.first_cb, bb.hidden_buf.view(R, -1), tb, out, d.temperature[:group], d.top_k[:group],
                          d.top_p[:group], d.do_sample[:group], d.guidance_scale[:group], st.q)
            torch.cuda.synchronize()
            assert torch.equal(out, st.outtok)
    from flashb._native import device_error
    assert device_error() == 0


@pytest.mark.parametrize('group,slots,lanes', [(2, 3, 3), (1, 2, 1), (4, 2, 2), (8, 2, 2), (8, 8, 8)])
def test_frame_engine_shared_backbone_matches_oracle(group, slots, lanes):
    """One backbone graph for every slot's rows (slot i = rows [2 g i, 2 g (i + 1)), its own CFG block), the depth
    frames per slot on the lanes: every slot's block matches the oracle's step on that block, and the depth launch
    consumed the block's hidden state and codebook 0.  32 and 128 rows take the many-rows GEMV kernel with the
    RMSNorms apart."""
    from flashb.engine import BackboneConfig, DepthConfig, FrameEngine
    bcfg = BackboneConfig(hidden=512, layers=2, heads=8, kv_heads=2, ffn=1024, vocab=65, codebooks=7)
    dcfg = DepthConfig(hidden=256, embed_dim=512, layers=2, heads=2, kv_heads=1, ffn=512, vocab=64,
                       codebook_size=60, n_decode=6)
    eng = FrameEngine(bcfg, dcfg, group * slots, 40, 4, seed=4, group=group, lanes=lanes, shared_backbone=True)
    eng.capture()
    bb = eng.bb
    R, G2 = bb.batch_size, 2 * group
    assert R == G2 * slots
    W = _oracle_backbone(bb)
    C = bcfg.codebooks
    mask = np32(bb.attn_mask).copy()
    pos = int(bb.cache_position.item())
    pids = bb.position_ids.view(-1).cpu().numpy().copy()
    for f in range(3):
        kcs = [np32(L.keys).copy() for L in bb.static_cache.layers]
        vcs = [np32(L.values).copy() for L in bb.static_cache.layers]
        ids = np.concatenate([eng.first_cb.cpu().numpy()[:, None], eng.outtok.cpu().numpy()[:, :C - 1]], 1)
        present = eng.cb0_present.cpu().numpy().copy()
        eng.step()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bb.input_ids_buf.view(R, -1).cpu().numpy(), ids)
        pos += 1
        pids += 1
        mask[..., pos] = 0.0
        assert int(bb.cache_position.item()) == pos
        gs = float(bb.guidance_scale.item())
        g_h = np32(bb.hidden_buf).reshape(R, -1)
        g_lg = bb.logits_buf.cpu().numpy()
        g_cfg = bb.cfg_logits_buf.cpu().numpy()
        for i, st in enumerate(eng.streams):
            r = slice(st.r0, st.r0 + G2)
            h, lg, _ = dec.backbone_step(W, ids[r], [k[r] for k in kcs], [v[r] for v in vcs], mask[r], pos, pids[r],
                                         gs)
            assert_close(g_h[r], h, tol=E2E_TOL, what=f'slot {i} frame {f} hidden')
            assert_close(g_lg[r], lg, what=f'slot {i} frame {f} logits')
            cfg_blk = g_cfg[st.r0 // 2:st.r0 // 2 + group]
            np.testing.assert_array_equal(cfg_blk, dec.cfg_combine(g_lg[r], group, gs))
            cb0 = _cb0_expected(eng, cfg_blk, st.c0, present)
            np.testing.assert_array_equal(st.first_cb.cpu().numpy(), cb0 + cb0)
            # the sampled tokens joined the streams' histories (the next frame's repetition penalty)
            assert all(eng.cb0_present[st.c0 + k, cb0[k]].item() == 1 for k in range(group))
            d = eng.depth
            out = torch.zeros_like(st.outtok)
            tb = torch.zeros_like(st.tokbuf)
            st.desc.frame(st.first_cb, st.bh, tb, out, d.temperature[:group], d.top_k[:group], d.top_p[:group],
                          d.do_sample[:group], d.guidance_scale[:group], st.q)
            torch.cuda.synchronize()
            assert torch.equal(out, st.outtok)
    from flashb._native import device_error
    assert device_error() == 0


def test_frame_engine_free_running_lanes_equal_joined_steps():
    """Steps issued with the lanes joined only after the last one give the same tokens as steps joined one by one:
    each slot's frames stay in order on its lane stream, and no lane reads another's buffers."""
    ea = _small_engine(streams=8, group=2, lanes=2)
    eb = _small_engine(streams=8, group=2, lanes=2)
    ea.capture()
    eb.capture()
    for t in range(4):
        ea.step()
        eb.step(fork=(t == 0), join=(t == 3))
    torch.cuda.synchronize()
    for sa, sb in zip(ea.streams, eb.streams):
        assert torch.equal(sa.outtok, sb.outtok) and torch.equal(sa.first_cb, sb.first_cb)
        assert torch.equal(sa.bb.cfg_logits_buf, sb.bb.cfg_logits_buf)


def test_frame_engine_greedy_cb0():
    """cb0='greedy' keeps the greedy branch: codebook 0 is the argmax of the stream's CFG logits."""
    from flashb.engine import BackboneConfig, DepthConfig, FrameEngine
    bcfg = BackboneConfig(hidden=512, layers=2, heads=8, kv_heads=2, ffn=1024, vocab=65, codebooks=7)
    dcfg = DepthConfig(hidden=256, embed_dim=512, layers=2, heads=2, kv_heads=1, ffn=512, vocab=64,
                       codebook_size=60, n_decode=6)
    eng = FrameEngine(bcfg, dcfg, 4, 40, 4, seed=4, group=2, shared_backbone=True, cb0='greedy')
    eng.capture()
    eng.step()
    torch.cuda.synchronize()
    g_cfg = eng.bb.cfg_logits_buf.cpu().numpy()
    for st in eng.streams:
        cb0 = [ofr.greedy_cb0(g_cfg[st.r0 // 2 + k], eng.n_valid) for k in range(2)]
        np.testing.assert_array_equal(st.first_cb.cpu().numpy(), cb0 + cb0)


def test_frame_engine_graph_equals_eager():
    ea = _small_engine(streams=1)
    eb = _small_engine(streams=1)
    eb.capture()
    # capture() ran one eager frame on stream 0 and rewound its position: do the same on the eager engine
    ea.backbone_part(0)
    ea.depth_part(0)
    torch.cuda.synchronize()
    ea.streams[0].bb.set_position(ea.prompt_len - 1)
    for _ in range(3):
        ea.frame(0)
        eb.frame(0)
    torch.cuda.synchronize()
    sa, sb = ea.streams[0], eb.streams[0]
    assert torch.equal(sa.outtok, sb.outtok) and torch.equal(sa.first_cb, sb.first_cb)
    assert torch.equal(sa.bb.cfg_logits_buf, sb.bb.cfg_logits_buf)
