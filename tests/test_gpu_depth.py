"""GPU parity of the depth-decoder frame kernel (``flashb_dd_frame``) against the oracle.

* teacher-forced logits of every codebook step vs ``oracle.depth.depth_frame`` (bf16 bar, argmax agreement);
* the sampled tokens bit-exact: the C sampler oracle run on the kernel's own logits (debug tap) must pick exactly the
  tokens the kernel wrote, for sampling, greedy, top-p and codebook-masked configurations;
* a free-running frame equals the teacher-forced oracle driven by the kernel's own tokens;
* run-to-run determinism and CUDA-graph replay.
"""
import json

import numpy as np
import pytest
import torch

from gpu_util import DEPTH_ARGMAX_MIN, assert_argmax_agree, assert_close, np32
from oracle import depth as odepth
from oracle import sampler as osmp

pytestmark = pytest.mark.gpu


def _model(small=True, B=2, seed=3, **kw):
    from flashb.engine import DepthConfig, SyntheticDepth
    if small:
        cfg = DepthConfig(hidden=256, embed_dim=384, layers=2, heads=2, kv_heads=1, ffn=512, vocab=64,
                          codebook_size=60, n_decode=6)
    else:
        cfg = DepthConfig()
    for k, v in kw.items():
        setattr(cfg, k, v)
    m = SyntheticDepth(cfg, batch=B, seed=seed)
    g = torch.Generator(device='cpu').manual_seed(seed + 10)
    m.backbone_hidden_buf.copy_(torch.randn(B, cfg.embed_dim, generator=g).to(torch.bfloat16))
    m.first_cb_token_buf.copy_(torch.randint(0, cfg.codebook_size, (B,), generator=g))
    m.q.copy_(torch.empty(m.q.shape).exponential_(1, generator=g))
    return m


def _weights(m):
    c = m.cfg
    layers = [{k: np32(v) for k, v in L.items()} for L in m.layers]
    head32 = m.head_t.float().permute(0, 2, 1).contiguous().cpu().numpy()
    return odepth.DepthWeights(layers, np32(m.embed), np32(m.proj), np32(m.normf), head32, c.vocab, c.codebook_size,
                               c.n_decode, c.eps, c.theta, c.heads, c.kv_heads)


def _params(m):
    return (m.temperature.cpu().numpy(), m.top_k.cpu().numpy(), m.top_p.cpu().numpy(), m.do_sample.cpu().numpy(),
            m.guidance_scale.cpu().numpy())


def _run(m, forced=None):
    c = m.cfg
    dbg = torch.zeros(c.n_decode, m.batch, c.vocab, dtype=torch.float32, device='cuda')
    f = None if forced is None else torch.as_tensor(forced, dtype=torch.long, device='cuda').contiguous()
    m.frame(dbg=dbg, forced=f)
    torch.cuda.synchronize()
    return m.output_tokens.cpu().numpy().copy(), dbg.cpu().numpy(), m.tok_buf.cpu().numpy().copy()


def _check_sampler(m, logits, outtok):
    """Every step's kernel token == the C sampler oracle on the kernel's own logits of that step."""
    c = m.cfg
    temp, topk, topp, ds, gs = _params(m)
    q = m.q.cpu().numpy()
    half = m.half
    for s in range(c.n_decode):
        for h in range(half):
            lu = logits[s, h + half] if m.batch >= 2 else None
            t, _ = osmp.sample_row(logits[s, h], lu, c.codebook_size, gs[h], temp[h], topk[h], topp[h], ds[h],
                                   q[s, h])
            t = min(max(int(t), 0), c.vocab - 1)
            assert outtok[h, s] == t, f'step {s} row {h}: kernel {outtok[h, s]} oracle {t}'
            if m.batch >= 2:
                assert outtok[h + half, s] == t


SAMPLING = {
    'sample': dict(temp=0.9, topk=50, topp=1.0, ds=1, gs=4.0),
    'greedy': dict(temp=1.0, topk=0, topp=1.0, ds=0, gs=3.0),
    'top_p': dict(temp=1.3, topk=0, topp=0.8, ds=1, gs=2.0),
    'top_k1': dict(temp=0.7, topk=1, topp=0.9, ds=1, gs=1.0),
}


def _set(m, p):
    m.temperature.fill_(p['temp'])
    m.top_k.fill_(p['topk'])
    m.top_p.fill_(p['topp'])
    m.do_sample.fill_(p['ds'])
    m.guidance_scale.fill_(p['gs'])


@pytest.mark.parametrize('B,grid', [(1, 0), (2, 0), (4, 0), (8, 0), (16, 0), (1, 4), (2, 8), (16, 12), (16, 32)])
def test_depth_forced_logits_match_oracle(B, grid):
    """grid 0: every SM, the mma.sync build; a grid of at most 32 CTAs (a lane of the GPU) runs the tcgen05 build."""
    m = _model(B=B)
    m.desc.cfg.grid = grid
    c = m.cfg
    forced = np.random.default_rng(B).integers(0, c.vocab, (c.n_decode, B))
    outtok, logits, _ = _run(m, forced)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    tok_ref, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                            m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits')
    assert_argmax_agree(logits, lg_ref, min_frac=DEPTH_ARGMAX_MIN, what='depth logits')
    np.testing.assert_array_equal(m.tok_buf.cpu().numpy(), np.clip(forced[-1], 0, c.vocab - 1))
    _check_sampler(m, logits, outtok)


@pytest.mark.parametrize('mode', sorted(SAMPLING))
def test_depth_sampler_bit_exact(mode):
    m = _model(B=2, seed=7)
    _set(m, SAMPLING[mode])
    outtok, logits, _ = _run(m)
    _check_sampler(m, logits, outtok)


def test_depth_free_running_equals_forced_oracle():
    """Without forcing, the kernel feeds its own tokens forward: the oracle teacher-forced by those tokens reproduces
    every step's logits."""
    m = _model(B=2, seed=11)
    c = m.cfg
    outtok, logits, tok = _run(m)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=outtok.T.copy())
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits')
    np.testing.assert_array_equal(tok, outtok[:, -1])


@pytest.mark.parametrize('B,grid', [(2, 0), (8, 0), (16, 0), (16, 74), (16, 18), (16, 8), (2, 18)])
def test_depth_full_size_forced_and_sampler(B, grid):
    """The synthetic full-size depth decoder (4 layers, hidden 1024, 16 codebooks of 2048).  B = 8 (four CFG pairs)
    runs the distributed attention mode ((row, KV head) pairs spread over the CTAs) and one sampler CTA per pair.  A
    grid of fewer CTAs than SMs (a lane of the GPU) spreads the same tasks over fewer CTAs; with fewer CTAs than
    pairs (18 or 8 < 16 x 2) a CTA takes several pairs, staged together."""
    m = _model(small=False, B=B, seed=5)
    m.desc.cfg.grid = grid
    c = m.cfg
    forced = np.random.default_rng(5).integers(0, c.vocab, (c.n_decode, B))
    outtok, logits, _ = _run(m, forced)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits')
    assert_argmax_agree(logits, lg_ref, min_frac=DEPTH_ARGMAX_MIN, what='depth logits')
    _check_sampler(m, logits, outtok)


def test_depth_determinism_and_graph_replay():
    m = _model(small=False, B=2, seed=6)
    m.frame()
    torch.cuda.synchronize()
    first = m.output_tokens.clone()
    m.frame()
    torch.cuda.synchronize()
    assert torch.equal(first, m.output_tokens)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            m.frame()
    torch.cuda.current_stream().wait_stream(s)
    m.output_tokens.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(first, m.output_tokens)
    g = torch.Generator(device='cpu').manual_seed(99)
    m.q.copy_(torch.empty(m.q.shape).exponential_(1, generator=g))
    graph.replay()
    torch.cuda.synchronize()
    _, logits, _ = _run(m)
    _check_sampler(m, logits, m.output_tokens.cpu().numpy())


# ------------------------------------------------------------------------------------------------ failure detection
def _barrier_words(m):
    """The frame's grid-barrier state in the scratch buffer: [count, exitc, abort, pad] as int32."""
    import ctypes
    from flashb import _native
    off = int(_native.lib().flashb_dd_barrier_offset(ctypes.byref(m.desc.cfg)))
    assert off >= 0 and off % 256 == 0
    return m.desc.scratch[off:off + 16].view(torch.int32)


def _fresh_frame_ok(m, ref):
    """After a failed frame the host zeroes the scratch; the next frame must match an undisturbed one."""
    from flashb import _native
    m.desc.scratch.zero_()
    out, logits, _ = _run(m)
    _native.check_device()
    np.testing.assert_array_equal(out, ref)


def test_depth_host_abort_winds_down():
    """The host sets the barrier's abort word before a frame: the frame stops at its first barrier wait, records
    FB_ERR_ABORTED, every CTA (producer warps included) returns promptly, and Python raises FlashbError.  Nothing
    faults or hangs: the injected state is a flag the kernel polls while it waits."""
    import time
    from flashb import _native
    m = _model(B=2, seed=31)
    m.desc.cfg.grid = 8
    ref, _, _ = _run(m)
    _native.check_device()
    _barrier_words(m)[2].fill_(1)
    t0 = time.perf_counter()
    m.frame()
    with pytest.raises(_native.FlashbError) as ei:
        _native.check_device()
    assert ei.value.rc == 7 and time.perf_counter() - t0 < 1.0
    _fresh_frame_ok(m, ref)


def test_depth_barrier_wait_expires():
    """A grid-barrier wait runs out: with a 10 ms wait limit (fb_dd_config.wait_ns) and the arrival counter set on
    the host so that the first barrier can never complete (it wraps past the target after half the grid has
    arrived), the late CTAs time out, record FB_ERR_TIMEOUT and raise the abort flag, the others stop at their next
    wait, and Python raises FlashbError with the timeout code.  Nothing faults or hangs: every wait is bounded."""
    import time
    from flashb import _native
    m = _model(B=2, seed=32)
    m.desc.cfg.grid = 8
    ref, _, _ = _run(m)
    _native.check_device()
    m.desc.cfg.wait_ns = 10_000_000
    _barrier_words(m)[0].fill_(-(8 // 2))
    t0 = time.perf_counter()
    m.frame()
    with pytest.raises(_native.FlashbError) as ei:
        _native.check_device()
    assert ei.value.rc == 5 and time.perf_counter() - t0 < 1.0
    m.desc.cfg.wait_ns = 0
    _fresh_frame_ok(m, ref)


@pytest.mark.parametrize('small,B,grid', [(True, 2, 0), (False, 16, 18), (False, 2, 0), (False, 16, 0)])
def test_depth_step_table(small, B, grid):
    """The per-token step table (the reference's dd2_tab_build / dd2_tab_set): codebook steps >= 1 read stage E and
    layer 0's q|k|v from the table.  The table itself equals the oracle's projector and layer-0 q|k|v of every
    embedding row it covers; frames with it match the oracle (teacher-forced logits) on both builds (tcgen05 on a
    lane-sized grid, mma.sync on the whole GPU); the sampler stays bit-exact on the kernel's logits."""
    from flashb import depth as fdep
    from oracle import decode as dec
    m = _model(small=small, B=B, seed=7)
    m.desc.cfg.grid = grid
    c = m.cfg
    pt, tt = fdep.tab_build(m.desc)
    # the table against the oracle on a sample of its rows (every step's first and last token, a few between)
    W = _weights(m)
    rows = np.unique(np.concatenate([np.arange(0, pt.shape[0], max(1, pt.shape[0] // 37)), [pt.shape[0] - 1]]))
    emb = np32(m.embed)[c.vocab + rows]
    p_ref = dec.linear(emb, W.proj)
    assert_close(np32(pt)[rows], p_ref, what='ptab')
    L0 = W.layers[0]
    t_ref = dec.gemv_seg(np32(pt)[rows], L0['ln1'], c.eps, [L0['wq'], L0['wk'], L0['wv']])
    assert_close(np32(tt)[rows], t_ref, what='ttab')
    fdep.tab_set(m.desc, pt, tt)
    forced = np.random.default_rng(7).integers(0, c.vocab, (c.n_decode, B))
    outtok, logits, _ = _run(m, forced)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits (step table)')
    _check_sampler(m, logits, outtok)
    # without the table again: the same frame as before the table was set
    fdep.tab_set(m.desc, None, None)
    outtok2, logits2, _ = _run(m, forced)
    for s in range(c.n_decode):
        assert_close(logits2[s], lg_ref[s], what=f'step {s} logits (no table)')
    from flashb._native import device_error
    assert device_error() == 0


def test_ln12_device_decode_is_bit_exact():
    """flashb_ln12_decode on the reference-encoded fixture matrix (shifted rows, inline and overflow patches) and on
    a full-size depth matrix gives back every bit of the bf16 weights."""
    import synth
    from flashb import ln12
    z = np.load(synth.__file__.replace('synth.py', 'ln12.npz'))
    w = synth.ln12_matrix()
    N, K = w.shape
    d, m, o, lut = ln12.to_device(z['data'], z['meta'], z['ovf'], z['lut'], 'cuda')
    out = torch.full((N, K), float('nan'), dtype=torch.bfloat16, device='cuda')
    ln12.decode_device(d, m, o, lut, out)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu().view(torch.int16), w.view(torch.int16))
    g = torch.Generator().manual_seed(8)
    w2 = (torch.randn(4096, 1024, generator=g) * 0.02).to(torch.bfloat16)
    enc = ln12.encode(w2)
    out2 = torch.empty(4096, 1024, dtype=torch.bfloat16, device='cuda')
    ln12.decode_device(*ln12.to_device(*enc, 'cuda'), out2)
    torch.cuda.synchronize()
    assert torch.equal(out2.cpu().view(torch.int16), w2.view(torch.int16))


def test_dd2_init_ln12_frames_equal_the_bf16_frames():
    """The reference's dd2_init_ln12 surface: the depth matrices handed over in LN12 are decoded on the device and
    the frames are bit-identical to the frames on the bf16 weights."""
    from flashb import depth as fdep
    from flashb import ln12
    m = _model(small=False, B=2, seed=9, layers=1, ffn=1024, embed_dim=1024, vocab=128, codebook_size=120,
               n_decode=4)
    ops = fdep.DepthOps()
    L = m.layers
    w = []
    for layer in L:
        w += [layer[k] for k in ('ln1', 'wq', 'wk', 'wv', 'wo', 'ln2', 'wg', 'wu', 'wd')]
    w += [m.embed, m.proj, m.normf, m.head_t, m.cos_tab, m.sin_tab]
    ops.dd2_init(w, eps=m.cfg.eps, codebook_size=m.cfg.codebook_size)
    args = (m.first_cb_token_buf, m.backbone_hidden_buf, m.tok_buf, m.output_tokens, m.temperature, m.top_k,
            m.top_p, m.do_sample, m.guidance_scale, m.q)
    ops.dd2_frame(*args)
    torch.cuda.synchronize()
    ref = m.output_tokens.clone()
    enc = [ln12.encode(x) for x in ops.ln12_mats()]
    dev = [ln12.to_device(*e, 'cuda') for e in enc]
    luts = torch.tensor([list(x[3]) for x in dev], dtype=torch.int64)
    ops.dd2_init_ln12([x[0] for x in dev], [x[1] for x in dev], [x[2] for x in dev], luts)
    for a, b in zip(ops.ln12_mats(), [x for layer in L for x in (layer['wq'], layer['wk'], layer['wv'], layer['wo'],
                                                                 layer['wg'], layer['wu'], layer['wd'])] +
                    [m.proj] + [m.head_t[s] for s in range(m.head_t.shape[0])]):
        assert torch.equal(a, b)
    m.output_tokens.zero_()
    ops.dd2_frame(*args)
    torch.cuda.synchronize()
    assert torch.equal(m.output_tokens, ref)
    assert json.loads(ops.dd2_info())['ln12'] == 1


@pytest.mark.parametrize('B,grid,kw', [
    (16, 18, {}),                                                     # the bench's lane: full-size model, B = 16
    (2, 8, dict(layers=1, n_decode=4, vocab=128, codebook_size=120)),
    (8, 12, dict(layers=2, n_decode=5, vocab=256, codebook_size=250, ffn=2048)),
])
def test_depth_ln12_streaming(B, grid, kw):
    """LN12 streamed by the frame (the reference's depth path on 12-bit weights): on a lane-sized grid the tcgen05
    build copies the LN12 bytes, decodes them in shared memory and runs its MMAs on the decoded strips.  The
    teacher-forced logits match the oracle on the bf16 weights (the decoded values are the same bits) and the frame
    on bf16 weights; the sampler stays bit-exact on the kernel's logits; switching back gives the bf16 frame."""
    m = _model(small=False, B=B, seed=11, **kw)
    m.desc.cfg.grid = grid
    c = m.cfg
    forced = np.random.default_rng(11).integers(0, c.vocab, (c.n_decode, B))
    _, lg_bf16, _ = _run(m, forced)
    m.use_ln12(True)
    outtok, logits, _ = _run(m, forced)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits (LN12 streamed)')
        assert_close(logits[s], lg_bf16[s], what=f'step {s} logits (LN12 vs bf16 frame)')
    assert_argmax_agree(logits, lg_ref, min_frac=DEPTH_ARGMAX_MIN, what='depth logits (LN12)')
    _check_sampler(m, logits, outtok)
    m.use_ln12(False)
    _, lg_back, _ = _run(m, forced)
    np.testing.assert_array_equal(lg_back, lg_bf16)
    from flashb._native import device_error
    assert device_error() == 0


def test_depth_ln12_streaming_with_step_table_and_patches():
    """LN12 streaming with the step table, on weights whose rows need every kind of record: shifted tables, inline
    patches and overflow patches (a few rows scaled far from the rest and a few wide outliers per row)."""
    from flashb import depth as fdep
    from flashb import ln12
    m = _model(small=False, B=16, seed=12, layers=1, n_decode=4, vocab=128, codebook_size=120)
    m.desc.cfg.grid = 18
    g = torch.Generator(device='cpu').manual_seed(12)
    for w in m.mats():
        wc = w.float().cpu()
        rows = torch.randint(0, wc.shape[0], (8,), generator=g)
        wc[rows] *= 16.0                                              # rows whose exponents sit higher: a shift
        r2 = torch.randint(0, wc.shape[0], (wc.shape[0] // 8,), generator=g)
        c2 = torch.randint(0, wc.shape[1], (wc.shape[0] // 8, 6), generator=g)
        wc[r2[:, None], c2] *= 2.0 ** 10                              # outliers: patches, > 3 in some rows
        w.copy_(wc.to(torch.bfloat16))
    counts = [(ln12.encode(w)[1][:, 0] & 1023) for w in m.mats()]
    assert max(int(x.max()) for x in counts) > 3                      # overflow patches are exercised
    pt, tt = fdep.tab_build(m.desc)
    fdep.tab_set(m.desc, pt, tt)
    m.use_ln12(True)
    c = m.cfg
    forced = np.random.default_rng(12).integers(0, c.vocab, (c.n_decode, 16))
    outtok, logits, _ = _run(m, forced)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits (LN12 + table, patched weights)')
    _check_sampler(m, logits, outtok)


def test_depth_ln12_streaming_refuses_unsupported_shapes():
    """LN12 streaming needs 64-row multiples (a stage's rows); a lane-sized frame of a 96-entry codebook is refused
    before anything runs."""
    from flashb._native import FlashbError
    m = _model(small=False, B=2, layers=1, n_decode=3, vocab=96, codebook_size=90)
    m.desc.cfg.grid = 4
    with pytest.raises(FlashbError):
        m.use_ln12(True)
        _run(m)


@pytest.mark.parametrize('mask,grid', [('0000', 18), ('1111', 18), ('1111', 32), ('0011', 8)])
def test_depth_task_forms(mask, grid, monkeypatch):
    """The plain GEMV tasks in their 64-row form and in the 128-row form, split over two CTAs in K where the grid
    allows (FLASHB_DD_TASK128: projector, o, down, heads): the same frame against the oracle, and the sampler
    bit-exact on the kernel's logits.  Grid 32 splits the heads too; grid 8 keeps every part whole."""
    monkeypatch.setenv('FLASHB_DD_TASK128', mask)
    m = _model(small=False, B=16, seed=13)
    m.desc.cfg.grid = grid
    c = m.cfg
    forced = np.random.default_rng(13).integers(0, c.vocab, (c.n_decode, 16))
    outtok, logits, _ = _run(m, forced)
    W = _weights(m)
    temp, topk, topp, ds, gs = _params(m)
    _, lg_ref, _ = odepth.depth_frame(W, np32(m.backbone_hidden_buf), m.first_cb_token_buf.cpu().numpy(),
                                      m.q.cpu().numpy(), temp, topk, topp, ds, gs, forced=forced)
    for s in range(c.n_decode):
        assert_close(logits[s], lg_ref[s], what=f'step {s} logits (task forms {mask}, grid {grid})')
    _check_sampler(m, logits, outtok)
    # a second frame on the same scratch: the split parts' tags start again from zero
    outtok2, logits2, _ = _run(m, forced)
    np.testing.assert_array_equal(logits2, logits)
    from flashb._native import device_error
    assert device_error() == 0


def test_dd2_init_ln12_streaming_surface():
    """The reference surface with LN12 streaming switched on (DepthOps.ln12_stream before the first frame, a lane-
    sized grid): the frame streams the 12-bit bytes and its teacher-forced logits match the frame on the decoded
    bf16 matrices."""
    from flashb import depth as fdep
    from flashb import ln12
    m = _model(small=False, B=2, seed=14, layers=1, ffn=1024, embed_dim=1024, vocab=128, codebook_size=120,
               n_decode=4)
    w = []
    for layer in m.layers:
        w += [layer[k] for k in ('ln1', 'wq', 'wk', 'wv', 'wo', 'ln2', 'wg', 'wu', 'wd')]
    w += [m.embed, m.proj, m.normf, m.head_t, m.cos_tab, m.sin_tab]
    forced = torch.as_tensor(np.random.default_rng(14).integers(0, m.cfg.vocab, (m.cfg.n_decode, 2)),
                             dtype=torch.long, device='cuda').contiguous()
    args = (m.first_cb_token_buf, m.backbone_hidden_buf, m.tok_buf, m.output_tokens, m.temperature, m.top_k,
            m.top_p, m.do_sample, m.guidance_scale, m.q)
    out = []
    for stream in (False, True):
        ops = fdep.DepthOps()
        ops.dd2_init(w, eps=m.cfg.eps, codebook_size=m.cfg.codebook_size)
        enc = [ln12.to_device(*ln12.encode(x), 'cuda') for x in ops.ln12_mats()]
        luts = torch.tensor([list(x[3]) for x in enc], dtype=torch.int64)
        ops.dd2_init_ln12([x[0] for x in enc], [x[1] for x in enc], [x[2] for x in enc], luts)
        ops.ln12_stream = stream
        saved = dict(fdep.GRIDS)
        try:
            fdep.GRIDS[2] = 8
            dbg = torch.zeros(m.cfg.n_decode, 2, m.cfg.vocab, dtype=torch.float32, device='cuda')
            ops.dd2_frame(*args, dbg=dbg, forced=forced)
            torch.cuda.synchronize()
        finally:
            fdep.GRIDS.clear()
            fdep.GRIDS.update(saved)
        assert (ops.desc[2].cfg.ln12 is not None) == stream
        out.append(dbg.cpu().numpy())
    for s in range(m.cfg.n_decode):
        assert_close(out[1][s], out[0][s], what=f'step {s} logits (LN12 streamed vs decoded)')
