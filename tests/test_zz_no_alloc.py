"""The allocation-free depth-frame entry point, ``flashb_dd_frame_noalloc``, called through the C ABI.

Some callers cannot allocate device memory themselves: a host that reaches the library over a plain C FFI without
an allocator of its own, or a serving loop that forbids cudaMalloc once it runs.  For them the depth frame can run
on a fixed scratch area built into the library instead of a caller-owned buffer.  These tests check that such a
call gives the same results as the regular entry point (``flashb_dd_frame``) run on the same inputs, over calls in a
row whose inputs and batch change from call to call (the area keeps the previous call's contents, so a read of stale
scratch would show), and that configurations too large for the area or malformed are refused before any work is
enqueued.

This file is named to be collected last, so a stop-at-first-failure run has run every other test before it; it
also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_close

pytestmark = pytest.mark.gpu

FB_ERR_ARG = 1


def _depth(seed, batch):
    from flashb.engine import DepthConfig, SyntheticDepth
    m = SyntheticDepth(DepthConfig(), batch=batch, seed=seed)
    g = torch.Generator().manual_seed(seed + 10)
    m.backbone_hidden_buf.copy_(torch.randn(batch, m.cfg.embed_dim, generator=g).to(torch.bfloat16))
    m.first_cb_token_buf.copy_(torch.randint(0, m.cfg.codebook_size, (batch,), generator=g))
    m.q.copy_(torch.empty(m.q.shape).exponential_(1, generator=g))
    return m


def _noalloc(m, outtok, tokbuf, dbg, forced=None, cfg=None):
    """One call of the allocation-free entry point on the model's inputs and the given output buffers."""
    from flashb._native import lib
    d = m.desc
    _p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    return lib().flashb_dd_frame_noalloc(
        ctypes.byref(cfg if cfg is not None else d.cfg), d.table.data_ptr(), m.first_cb_token_buf.data_ptr(),
        m.backbone_hidden_buf.data_ptr(), tokbuf.data_ptr(), outtok.data_ptr(), m.temperature.data_ptr(),
        m.top_k.data_ptr(), m.top_p.data_ptr(), m.do_sample.data_ptr(), m.guidance_scale.data_ptr(), m.q.data_ptr(),
        _p(dbg), _p(forced), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize('teacher_forced', [True, False])
def test_noalloc_matches_regular_entry_point_over_changing_calls(teacher_forced):
    from flashb._native import check, device_error
    # call 0: 4 rows (two CFG pairs), call 1: 2 rows with other weights and inputs (the area's layout shifts over
    # what call 0 left), call 2: the first model again
    models = [_depth(seed=21, batch=4), _depth(seed=37, batch=2)]
    order = [0, 1, 0]
    refs = []
    for i, m in enumerate(models):
        c = m.cfg
        forced = None
        if teacher_forced:
            forced = torch.as_tensor(np.random.default_rng(3 + i).integers(0, c.vocab, (c.n_decode, m.batch)),
                                     dtype=torch.long, device='cuda')
        # the regular entry point, with its caller-owned scratch, on this model's own inputs
        dbg = torch.zeros(c.n_decode, m.batch, c.vocab, dtype=torch.float32, device='cuda')
        m.frame(dbg=dbg, forced=forced)
        torch.cuda.synchronize()
        refs.append((dbg, m.output_tokens.clone(), m.tok_buf.clone(), forced))
    for call, i in enumerate(order):
        m, (dbg_ref, out_ref, tok_ref, forced) = models[i], refs[i]
        outtok = torch.full_like(out_ref, -1)
        tokbuf = torch.full_like(tok_ref, -1)
        dbg = torch.zeros_like(dbg_ref)
        check(_noalloc(m, outtok, tokbuf, dbg, forced))
        torch.cuda.synchronize()
        for s in range(m.cfg.n_decode):
            assert_close(dbg[s].cpu().numpy(), dbg_ref[s].cpu().numpy(), what=f'call {call} step {s} logits')
        assert torch.equal(outtok, out_ref), f'call {call}: sampled tokens differ'
        assert torch.equal(tokbuf, tok_ref), f'call {call}: fed-forward tokens differ'
    assert device_error() == 0


def test_noalloc_refuses_a_configuration_larger_than_its_area():
    from flashb import _native
    m = _depth(seed=22, batch=2)
    big = _native.FbDDConfig.from_buffer_copy(bytes(m.desc.cfg))
    big.batch, big.ffn = 16, 65536          # valid fields whose scratch is far beyond the 1 MiB area
    need = _native.lib().flashb_dd_scratch_bytes(ctypes.byref(big))
    assert need > (1 << 20)
    out = torch.zeros(16, m.cfg.n_decode, dtype=torch.long, device='cuda')
    tok = torch.zeros(16, dtype=torch.long, device='cuda')
    rc = _noalloc(m, out, tok, None, cfg=big)
    assert rc == FB_ERR_ARG
    assert b'built-in area' in _native.lib().flashb_last_error()


@pytest.mark.parametrize('field,value', [('kv_heads', 0), ('ffn', -64), ('hidden', 1 << 30), ('batch', 3)])
def test_noalloc_refuses_malformed_fields_before_sizing(field, value):
    from flashb import _native
    m = _depth(seed=23, batch=2)
    bad = _native.FbDDConfig.from_buffer_copy(bytes(m.desc.cfg))
    setattr(bad, field, value)
    out = torch.zeros_like(m.output_tokens)
    tok = torch.zeros_like(m.tok_buf)
    rc = _noalloc(m, out, tok, None, cfg=bad)
    assert rc == FB_ERR_ARG
    assert b'built-in area' not in _native.lib().flashb_last_error()
    torch.cuda.synchronize()
    assert _native.device_error() == 0
