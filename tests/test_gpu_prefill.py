"""GPU parity of the tcgen05 causal GQA prefill attention (``flashb_prefill_attn``) against the reference's eager
outputs (golden fixture) and the oracle: config 5 shapes, ragged lengths, left padding, fp32 and bf16 masks,
strided q, the reference's key trimming, head-range shards, and run-to-run determinism.  Bar: max |gpu - ref| <=
1e-2 * max |ref| on rows with a live key (fully masked rows are 0 on both sides)."""
import numpy as np
import pytest
import torch

import synth
from gpu_util import TOL, assert_argmax_agree, assert_close, np32
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
