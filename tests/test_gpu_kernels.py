"""GPU parity of the individual kernels against the CPU oracle on identical seeded bf16 inputs.

Tolerance: max |gpu - oracle| <= 1e-2 * max |oracle| for bf16 / fp32 outputs; the oracle is
itself bit-exact against the reference's eager modules (tests/test_oracle_golden.py)."""
import numpy as np
import pytest
import torch

from gpu_util import TOL, assert_close, bf16_min, np32, randn
from oracle import decode as dec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def ops():
    from flashb import kernels
    return kernels.fused(), kernels.attn()


# ------------------------------------------------------------------------------------------------ GEMVs
@pytest.mark.parametrize('M', [1, 2, 4, 8, 12, 16])
def test_gemv_seg_norm_qkv(ops, M):
    fx, _ = ops
    K = 2048
    x = randn((M, K), 1)
    nw = randn((K,), 2, 0.1, 1.0)
    Wq, Wk, Wv = randn((2048, K), 3, 0.02), randn((512, K), 4, 0.02), randn((512, K), 5, 0.02)
    y = torch.empty(M, 3072, dtype=torch.bfloat16, device='cuda')
    fx.gemv_seg(x, nw, 1e-6, Wq, Wk, Wv, y)
    ref = dec.gemv_seg(np32(x), np32(nw), 1e-6, [np32(Wq), np32(Wk), np32(Wv)])
    assert_close(np32(y), ref, what=f'gemv_seg M={M}')


def test_gemv_seg_plain_odd_shapes(ops):
    fx, _ = ops
    M, K = 2, 1000   # K % 8 == 0 but not a multiple of the stage width
    x = randn((M, K), 11)
    W0, W1 = randn((77, K), 12, 0.05), randn((13, K), 13, 0.05)
    y = torch.empty(M, 90, dtype=torch.bfloat16, device='cuda')
    fx.gemv_seg(x, None, 0.0, W0, W1, None, y)
    ref = dec.gemv_seg(np32(x), None, 0.0, [np32(W0), np32(W1)])
    assert_close(np32(y), ref, what='gemv_seg odd')


@pytest.mark.parametrize('M,K,N', [(2, 2048, 2048), (2, 3072, 2048), (2, 6144, 2048), (4, 4096, 1024), (1, 2048, 5),
                                   (8, 6144, 2048), (8, 6144, 37),    # M x K too large for 64 KB stages: 32 KB build
                                   (16, 2048, 2048), (16, 6144, 2048), (12, 6144, 300)])  # two row tiles; x chunked
def test_gemv_resid(ops, M, K, N):
    fx, _ = ops
    x = randn((M, K), 21)
    W = randn((N, K), 22, 0.02)
    res = randn((M, N), 23)
    y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    fx.gemv_resid(x, W, res, y)
    ref = dec.gemv_resid(np32(x), np32(W), np32(res))
    assert_close(np32(y), ref, what='gemv_resid')


@pytest.mark.parametrize('M', [1, 2, 4, 8, 16])
def test_config2_gateup_then_down(ops, M):
    """RMSNorm + [6144 x 2048] gate|up GEMV + SiLU*up, then the [2048 x 3072] down GEMV."""
    fx, _ = ops
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(M, 2048, generator=g)).to(torch.bfloat16).cuda()
    gamma = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16).cuda()
    W1 = (0.02 * torch.randn(6144, 2048, generator=g)).to(torch.bfloat16).cuda()
    W2 = (0.02 * torch.randn(2048, 3072, generator=g)).to(torch.bfloat16).cuda()
    act = torch.empty(M, 3072, dtype=torch.bfloat16, device='cuda')
    y = torch.empty(M, 2048, dtype=torch.bfloat16, device='cuda')
    fx.gemv_gateup(x, gamma, 1e-6, W1[:3072], W1[3072:], act)
    fx.gemv_resid(act, W2, x, y)
    ref_act = dec.gemv_gateup(np32(x), np32(gamma), 1e-6, np32(W1[:3072]), np32(W1[3072:]))
    assert_close(np32(act), ref_act, what='gateup')
    ref_y = dec.gemv_resid(np32(act), np32(W2), np32(x))
    assert_close(np32(y), ref_y, what='down')
    # exactness rate: identical rounding points, only the fp32 summation order differs
    assert np.mean(np32(act) == ref_act) > 0.9


def test_config2_against_reference_golden(ops):
    """BASELINE config 2 exactly (seed 1, M 2), checked directly against the reference's own BreezeRMSNorm /
    F.linear / silu output (tests/golden/gemv2.npz)."""
    import synth
    from oracle.bf16 import bits_to_f32
    fx, _ = ops
    z = np.load(synth.__file__.rsplit('/', 1)[0] + '/gemv2.npz')
    x, gamma, wg, wu, wd = [t.cuda() for t in synth.gemv2_inputs()]
    M, F, K = x.shape[0], wg.shape[0], x.shape[1]
    act = torch.empty(M, F, dtype=torch.bfloat16, device='cuda')
    y = torch.empty(M, K, dtype=torch.bfloat16, device='cuda')
    fx.gemv_gateup(x, gamma, synth.GEMV2['eps'], wg, wu, act)
    fx.gemv_resid(act, wd, x, y)
    torch.cuda.synchronize()
    assert_close(np32(act), bits_to_f32(z['act']), what='config 2 act vs reference')
    assert_close(np32(y), bits_to_f32(z['y']), what='config 2 y vs reference')


def test_rmsnorm(ops):
    fx, _ = ops
    x = randn((4, 2048), 31, 3.0)
    w = randn((2048,), 32, 0.1, 1.0)
    y = torch.empty_like(x)
    fx.rmsnorm(x, w, 1e-6, y)
    ref = dec.rmsnorm(np32(x), np32(w), 1e-6)
    assert_close(np32(y), ref, what='rmsnorm')
    assert np.mean(np32(y) == ref) > 0.99


def test_gemv_rejects_bad_tensors(ops):
    fx, _ = ops
    x = randn((2, 2048), 1)
    W = randn((64, 1024), 2)
    y = torch.empty(2, 64, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(RuntimeError):
        fx.gemv_resid(x, W, y, y)          # K mismatch
    with pytest.raises(RuntimeError):
        fx.gemv_seg(x.float(), None, 0.0, W, None, None, y)


# ------------------------------------------------------------------------------------------------ attention
def _attn_ws(B, NH, NKV, S):
    from flashb import kernels
    n = kernels.attn_ws_floats(B, NH, NKV, S)
    return (torch.empty(1, device='cuda'), torch.empty(1, device='cuda'), torch.empty(n, device='cuda'),
            torch.zeros(B * NKV, dtype=torch.int32, device='cuda'))


def _mask(B, S, valid, dtype=torch.bfloat16):
    m = torch.full((B, 1, 1, S), bf16_min() if dtype == torch.bfloat16 else -3.4e38, dtype=torch.float32)
    for b, (lo, hi) in enumerate(valid):
        m[b, 0, 0, lo:hi] = 0
    return m.to(dtype).cuda()


@pytest.mark.parametrize('NH,NKV,S,valid', [
    (16, 4, 1024, ((0, 1024), (0, 1024))),
    (16, 4, 1000, ((0, 700), (13, 1000))),       # ragged S, left padding
    (16, 8, 2048, ((0, 1500), (300, 1700))),     # real model GQA group 2
    (16, 4, 4096, ((0, 4096), (0, 4096))),       # the 4096 sweep point, above the reference's 2048 cap
    (8, 1, 70, ((0, 1), (69, 70))),              # single valid key
    (16, 2, 64, ((0, 64), (0, 64))),             # group 8
])
def test_attn_decode(ops, NH, NKV, S, valid):
    _, ax = ops
    B = 2
    q = randn((B, NH, 1, 128), 40)
    k = randn((B, NKV, S, 128), 41)
    v = randn((B, NKV, S, 128), 42)
    mask = _mask(B, S, valid)
    out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    ax.attn_decode(q, k, v, mask, 128 ** -0.5, sc, cm, part, cnt, out)
    ref = dec.attn_decode(np32(q), np32(k), np32(v), np32(mask), 128 ** -0.5)
    assert_close(np32(out), ref, what=f'attn S={S}')



def test_attn_decode_config1_against_reference_golden(ops):
    """BASELINE config 1 exactly (seed 0, B 2, 16 q / 4 KV, KV 1024, every key valid), checked directly against the
    reference's own eager attention output (tests/golden/attn1.npz), bf16 and fp32-upcast forms."""
    import synth
    from oracle.bf16 import bits_to_f32
    _, ax = ops
    z = np.load(synth.__file__.rsplit('/', 1)[0] + '/attn1.npz')
    q, k, v = synth.attn1_inputs()
    c = synth.ATTN1
    B, NH, NKV, S = c['B'], c['NH'], c['NKV'], c['S']
    mask = torch.zeros(B, 1, 1, S, dtype=torch.bfloat16, device='cuda')
    out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    ax.attn_decode(q.cuda(), k.cuda(), v.cuda(), mask, 128 ** -0.5, sc, cm, part, cnt, out)
    torch.cuda.synchronize()
    assert_close(np32(out), bits_to_f32(z['out']), what='config 1 vs reference bf16')
    assert_close(np32(out), z['out_fp32'], what='config 1 vs reference fp32 upcast')


def test_attn_decode_fp32_mask_and_dead_row(ops):
    _, ax = ops
    B, NH, NKV, S = 2, 16, 4, 300
    q, k, v = randn((B, NH, 1, 128), 50), randn((B, NKV, S, 128), 51), randn((B, NKV, S, 128), 52)
    m = torch.zeros(B, 1, 1, S)
    m[0, 0, 0, 100:] = float('-inf')
    m[1] = float('-inf')                       # batch 1: every key masked -> zero output
    m[0, 0, 0, :50] = torch.linspace(-3, 0, 50)  # a non-trivial additive fp32 mask
    mask = m.cuda()
    out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    ax.attn_decode(q, k, v, mask, 128 ** -0.5, sc, cm, part, cnt, out)
    ref = dec.attn_decode(np32(q), np32(k), np32(v), np32(mask), 128 ** -0.5, mask_bf16=False)
    assert_close(np32(out)[0], ref[0], what='fp32 mask')
    assert float(out[1].abs().max()) == 0.0


@pytest.mark.parametrize('NKV,S,pos', [(4, 1024, 1023), (4, 2048, 700), (8, 512, 64), (4, 4096, 4000)])
def test_attn_decode_fused(ops, NKV, S, pos):
    _, ax = ops
    B, NH = 2, 16
    qkv = randn((B, (NH + 2 * NKV) * 128), 60, 2.0)
    qn, kn = randn((128,), 61, 0.1, 1.0), randn((128,), 62, 0.1, 1.0)
    kc, vc = randn((B, NKV, S, 128), 63), randn((B, NKV, S, 128), 64)
    kc[:, :, pos:] = 0
    vc[:, :, pos:] = 0
    from flashb.engine import rope_table
    cos_t, sin_t = rope_table(1e6, 128, S, 'cuda')
    pids = torch.tensor([pos, pos - 3])
    cos, sin = cos_t[pids].view(B, 1, 128).contiguous(), sin_t[pids].view(B, 1, 128).contiguous()
    mask = _mask(B, S, ((0, pos + 1), (3, pos + 1)))
    cp = torch.tensor([pos], dtype=torch.long, device='cuda')
    out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    kc_ref, vc_ref = np32(kc).copy(), np32(vc).copy()
    ax.attn_decode_fused(qkv, qn, kn, 1e-6, cos, sin, kc, vc, mask, cp, 128 ** -0.5, sc, cm, part, cnt, out)
    ref = dec.attn_decode_fused(np32(qkv), np32(qn), np32(kn), 1e-6, np32(cos), np32(sin), kc_ref, vc_ref,
                                np32(mask), pos, 128 ** -0.5)
    assert_close(np32(out), ref, what='fused attn')
    # the cache write itself: v bit-exact, k (norm + RoPE) within one bf16 ulp
    assert np.array_equal(np32(vc), vc_ref)
    assert_close(np32(kc)[:, :, pos], kc_ref[:, :, pos], tol=1e-2, what='k write')
    assert np.mean(np32(kc)[:, :, pos] == kc_ref[:, :, pos]) > 0.95


@pytest.mark.parametrize('B,NKV,S,pos,budget', [(16, 4, 600, 515, 18), (128, 4, 576, 515, 0), (40, 8, 300, 63, 0),
                                                 (128, 4, 4096, 4095, 0),     # config 3's longest cache, 128 rows
                                                 (24, 2, 200, 64, 8), (64, 4, 130, 0, 64), (128, 16, 96, 95, 0),
                                                 (32, 4, 301, 150, 16)])
def test_attn_decode_fused_tensor_cores(ops, B, NKV, S, pos, budget):
    """Many rows: one CTA per (row, KV head) with the two products of each 64-key chunk on mma.sync (the
    tensor-core kernel) -- ragged last chunks, chunk-aligned positions, GQA groups 4, 2 and 1, left padding, and an
    odd mask row stride (S = 301: mask rows not 4-byte aligned, read with plain loads)."""
    _, ax = ops
    NH = 16
    qkv = randn((B, (NH + 2 * NKV) * 128), 80, 2.0)
    qn, kn = randn((128,), 81, 0.1, 1.0), randn((128,), 82, 0.1, 1.0)
    kc, vc = randn((B, NKV, S, 128), 83), randn((B, NKV, S, 128), 84)
    kc[:, :, pos:] = 0
    vc[:, :, pos:] = 0
    from flashb.engine import rope_table
    cos_t, sin_t = rope_table(1e6, 128, S, 'cuda')
    pids = torch.tensor([max(0, pos - (b % 5)) for b in range(B)])
    cos, sin = cos_t[pids].view(B, 1, 128).contiguous(), sin_t[pids].view(B, 1, 128).contiguous()
    mask = _mask(B, S, tuple((min(b % 5, pos), pos + 1) for b in range(B)))
    cp = torch.tensor([pos], dtype=torch.long, device='cuda')
    out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    kc_ref, vc_ref = np32(kc).copy(), np32(vc).copy()
    from flashb._native import lib
    try:
        _budget(budget)
        ax.attn_decode_fused(qkv, qn, kn, 1e-6, cos, sin, kc, vc, mask, cp, 128 ** -0.5, sc, cm, part, cnt, out)
        torch.cuda.synchronize()
        path = lib().flashb_attn_last_path()
    finally:
        _budget(0)
    assert path == 1, f'expected the tensor-core kernel, got path {path}'
    ref = dec.attn_decode_fused(np32(qkv), np32(qn), np32(kn), 1e-6, np32(cos), np32(sin), kc_ref, vc_ref,
                                np32(mask), pos, 128 ** -0.5)
    assert_close(np32(out), ref, what=f'tensor-core fused attn B={B}')
    assert np.array_equal(np32(vc), vc_ref)
    assert_close(np32(kc)[:, :, pos], kc_ref[:, :, pos], tol=1e-2, what='k write')
    from flashb._native import device_error
    assert device_error() == 0


def test_attn_determinism(ops):
    _, ax = ops
    B, NH, NKV, S = 2, 16, 4, 2048
    q, k, v = randn((B, NH, 1, 128), 70), randn((B, NKV, S, 128), 71), randn((B, NKV, S, 128), 72)
    mask = _mask(B, S, ((0, S), (0, S)))
    sc, cm, part, cnt = _attn_ws(B, NH, NKV, S)
    outs = []
    for _ in range(3):
        out = torch.empty(B, 1, NH, 128, dtype=torch.bfloat16, device='cuda')
        ax.attn_decode(q, k, v, mask, 128 ** -0.5, sc, cm, part, cnt, out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


# ------------------------------------------------------------------------------------------------ step ends
def test_embed_rope(ops):
    fx, _ = ops
    B, C, V, H = 2, 16, 2049, 2048
    table = randn((C * V, H), 80)
    ids = torch.randint(0, V, (B, C), generator=torch.Generator().manual_seed(81)).cuda()
    from flashb.engine import rope_table
    cos_t, sin_t = rope_table(1e6, 128, 600, 'cuda')
    pos = torch.tensor([517, 3], dtype=torch.long, device='cuda')
    x = torch.empty(B, H, dtype=torch.bfloat16, device='cuda')
    cos = torch.empty(B, 1, 128, dtype=torch.bfloat16, device='cuda')
    sin = torch.empty_like(cos)
    fx.embed_rope(ids, V, table, pos, cos_t, sin_t, x, cos, sin)
    ref = dec.embed_sum(np32(table), ids.cpu().numpy(), V)
    assert_close(np32(x), ref, what='embed')
    assert np.mean(np32(x) == ref) > 0.99
    assert torch.equal(cos.view(B, 128), cos_t[pos.cpu()].cuda()) and torch.equal(sin.view(B, 128), sin_t[pos.cpu()])


@pytest.mark.parametrize('B', [1, 2, 4])
def test_lm_head_cfg(ops, B):
    fx, _ = ops
    H, V = 2048, 2049
    x = randn((B, H), 90, 2.0)
    nw = randn((H,), 91, 0.1, 1.0)
    W = randn((V, H), 92, 0.02).float()
    gs = torch.tensor([4.0], device='cuda')
    hid = torch.empty(B, H, dtype=torch.bfloat16, device='cuda')
    logits = torch.empty(B, V, device='cuda')
    half = B // 2 if B >= 2 else 1
    cfg = torch.empty(half, V, device='cuda')
    fx.lm_head_cfg(x, nw, 1e-6, W, gs, hid, logits, cfg)
    h_ref = dec.rmsnorm(np32(x), np32(nw), 1e-6)
    assert_close(np32(hid), h_ref, what='final norm')
    lg_ref = dec.lm_head_fp32(np32(hid), W.cpu().numpy())   # same bf16 hidden -> only summation order differs
    assert_close(logits.cpu().numpy(), lg_ref, tol=1e-5, what='lm_head')
    cfg_ref = dec.cfg_combine(logits.cpu().numpy(), half, 4.0) if B >= 2 else logits.cpu().numpy()[:1]
    assert np.array_equal(cfg.cpu().numpy(), cfg_ref), 'CFG combine is elementwise: bit-exact given the logits'


@pytest.mark.parametrize('B,block,V', [(128, 16, 2049), (32, 8, 2049), (16, 16, 100), (6, 1, 37), (128, 128, 2049)])
def test_lm_head_cfg_blocks(ops, B, block, V):
    """Final norm + fp32 lm_head + CFG for many rows in CFG blocks, one pass over the lm_head: logits within fp32
    summation-order error of the oracle on the kernel's own normed hidden, every block's CFG rows bit-exact given the
    logits."""
    fx, _ = ops
    H = 2048
    x = randn((B, H), 93, 2.0)
    nw = randn((H,), 94, 0.1, 1.0)
    W = randn((V, H), 95, 0.02).float()
    gs = torch.tensor([4.0], device='cuda')
    hid = torch.empty(B, H, dtype=torch.bfloat16, device='cuda')
    logits = torch.empty(B, V, device='cuda')
    npair = B // 2 if block >= 2 else B
    cfg = torch.empty(npair, V, device='cuda')
    fx.lm_head_cfg_blocks(x, nw, 1e-6, W, gs, block, hid, logits, cfg)
    torch.cuda.synchronize()
    assert_close(np32(hid), dec.rmsnorm(np32(x), np32(nw), 1e-6), what='final norm')
    lg = logits.cpu().numpy()
    assert_close(lg, dec.lm_head_fp32(np32(hid), W.cpu().numpy()), tol=1e-5, what='lm_head')
    if block >= 2:
        h = block // 2
        ref = np.concatenate([dec.cfg_combine(lg[b0:b0 + block], h, 4.0) for b0 in range(0, B, block)])
    else:
        ref = lg
    assert np.array_equal(cfg.cpu().numpy(), ref), 'CFG combine is elementwise: bit-exact given the logits'


# ------------------------------------------------------------------------------------------------ tcgen05 GEMV
def _budget(n):
    from flashb._native import lib
    lib().flashb_set_sm_budget(n)


def _path():
    from flashb._native import lib
    return lib().flashb_gemv_last_path()


@pytest.mark.parametrize('kind,M,budget', [('gateup', 16, 18), ('gateup', 2, 18), ('gateup', 5, 64),
                                           ('qkv', 16, 18), ('qkv', 1, 8), ('o', 16, 18), ('o', 7, 4),
                                           ('down', 16, 18), ('down', 2, 18), ('odd', 3, 2)])
def test_gemv_tcgen05_matches_oracle(ops, kind, M, budget):
    """The tcgen05 kernel (weights as the MMA's 128-row M side, fp32 sums in TMEM) runs when the grid has enough
    128-row blocks; a small SM budget (a lane of the GPU) selects it for the backbone's shapes."""
    fx, _ = ops
    K = {'down': 6144, 'odd': 1024}.get(kind, 2048)
    x = randn((M, K), 41)
    nw = randn((K,), 42, 0.1, 1.0)
    try:
        _budget(budget)
        if kind == 'gateup':
            Wg, Wu = randn((6144, K), 43, 0.02), randn((6144, K), 44, 0.02)
            y = torch.empty(M, 6144, dtype=torch.bfloat16, device='cuda')
            fx.gemv_gateup(x, nw, 1e-6, Wg, Wu, y)
            ref = dec.gemv_gateup(np32(x), np32(nw), 1e-6, np32(Wg), np32(Wu))
        elif kind == 'qkv':
            Wq, Wk, Wv = randn((2048, K), 45, 0.02), randn((512, K), 46, 0.02), randn((512, K), 47, 0.02)
            y = torch.empty(M, 3072, dtype=torch.bfloat16, device='cuda')
            fx.gemv_seg(x, nw, 1e-6, Wq, Wk, Wv, y)
            ref = dec.gemv_seg(np32(x), np32(nw), 1e-6, [np32(Wq), np32(Wk), np32(Wv)])
        else:
            N = 300 if kind == 'odd' else 2048
            W = randn((N, K), 48, 0.02)
            res = randn((M, N), 49)
            y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
            fx.gemv_resid(x, W, res, y)
            ref = dec.gemv_resid(np32(x), np32(W), np32(res))
        torch.cuda.synchronize()
        path = _path()
    finally:
        _budget(0)
    assert path == 2, f'expected the tcgen05 kernel, got path {path}'
    assert_close(np32(y), ref, what=f'tcgen05 {kind} M={M}')
    from flashb._native import device_error
    assert device_error() == 0


def test_gemv_more_rows_without_tensor_cores(ops):
    """More than 16 rows with K % 64 != 0 (no tcgen05 kernel): row blocks of 16 through the M <= 16 paths."""
    fx, _ = ops
    M, K, N = 40, 1000, 300
    x = randn((M, K), 71)
    W = randn((N, K), 72, 0.02)
    res = randn((M, N), 73)
    y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    fx.gemv_resid(x, W, res, y)
    assert_close(np32(y), dec.gemv_resid(np32(x), np32(W), np32(res)), what='gemv_resid M=40 K=1000')
    nw = randn((K,), 74, 0.1, 1.0)
    y2 = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
    fx.gemv_seg(x, nw, 1e-6, W, None, None, y2)
    assert_close(np32(y2), dec.gemv_seg(np32(x), np32(nw), 1e-6, [np32(W)]), what='gemv_seg M=40 K=1000')


def _split():
    from flashb._native import lib
    return lib().flashb_gemv_last_split()


@pytest.mark.parametrize('kind,M,budget,rows,split', [
    # row groups of 16 side by side (blockIdx.y), each on its share of the SMs
    ('gateup', 128, 18, 16, 1), ('gateup', 40, 32, 16, 1), ('qkv', 128, 8, 16, 1), ('qkv', 17, 8, 16, 1),
    ('o', 64, 4, 16, 1), ('down', 100, 4, 16, 1), ('qkv', 128, 0, 16, 1), ('gateup', 128, 0, 16, 1),
    ('o', 128, 0, 16, 1), ('down', 128, 0, 16, 1), ('down', 33, 0, 16, 3),
    # wide tiles (MMA N = 32, 64, 128), whole blocks per CTA
    ('gateup', 40, 32, 32, 1), ('down', 100, 8, 128, 1), ('qkv', 60, 8, 64, 1),
    # too few 128-row blocks for the grid: each block's K range split over a cluster
    ('qkv', 128, 0, 128, 6), ('o', 128, 0, 128, 8), ('down', 128, 0, 128, 8), ('gateup', 128, 0, 128, 3),
    ('o', 2, 0, 16, 8), ('qkv', 16, 0, 16, 6), ('down', 33, 0, 64, 8), ('gateup', 2, 0, 16, 3),
    ('odd', 70, 0, 128, 8), ('o', 128, 64, 128, 4),
    # the default: two groups of 64 rows on 74 SMs each (the shared backbone's 128 rows)
    ('qkv', 128, 0, 64, 3), ('o', 128, 0, 64, 4), ('down', 128, 0, 64, 4), ('gateup', 128, 0, 64, 1)])
def test_gemv_tcgen05_wide_and_split_k(ops, kind, M, budget, rows, split):
    """More than 16 activation rows on the tcgen05 kernel: row groups of 16 side by side (the default) or wide MMA
    tiles of 32 / 64 / 128 rows, and split K over a thread-block cluster with the partial sums reduced through
    distributed shared memory (budget 0 = all SMs, e.g. 148 on B200: 16 blocks of a 2048-row matrix become 16
    clusters of 8; for groups of at most 16 rows only when switched on)."""
    fx, _ = ops
    K = {'down': 6144, 'odd': 1024}.get(kind, 2048)
    x = randn((M, K), 51)
    nw = randn((K,), 52, 0.1, 1.0)
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    if budget == 0 and nsm < 148:
        pytest.skip('split counts are for a 148-SM B200')
    from flashb._native import lib
    try:
        _budget(budget)
        lib().flashb_set_gemv_rows_path(0)     # the many-rows kernel would take the calls without norm
        lib().flashb_set_gemv_split(1 if rows == 16 and split > 1 else 0)
        assert lib().flashb_set_gemv_group_rows(rows) == 0
        if kind == 'gateup':
            Wg, Wu = randn((6144, K), 53, 0.02), randn((6144, K), 54, 0.02)
            y = torch.empty(M, 6144, dtype=torch.bfloat16, device='cuda')
            fx.gemv_gateup(x, nw, 1e-6, Wg, Wu, y)
            ref = dec.gemv_gateup(np32(x), np32(nw), 1e-6, np32(Wg), np32(Wu))
        elif kind == 'qkv':
            Wq, Wk, Wv = randn((2048, K), 55, 0.02), randn((512, K), 56, 0.02), randn((512, K), 57, 0.02)
            y = torch.empty(M, 3072, dtype=torch.bfloat16, device='cuda')
            fx.gemv_seg(x, nw, 1e-6, Wq, Wk, Wv, y)
            ref = dec.gemv_seg(np32(x), np32(nw), 1e-6, [np32(Wq), np32(Wk), np32(Wv)])
        else:
            N = 300 if kind == 'odd' else 2048
            W = randn((N, K), 58, 0.02)
            res = randn((M, N), 59)
            y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
            fx.gemv_resid(x, W, res, y)
            ref = dec.gemv_resid(np32(x), np32(W), np32(res))
        torch.cuda.synchronize()
        path, got_split = _path(), _split()
        # the same call again gives the same bits (the split's reduction order is fixed)
        y2 = torch.empty_like(y)
        if kind == 'gateup':
            fx.gemv_gateup(x, nw, 1e-6, Wg, Wu, y2)
        elif kind == 'qkv':
            fx.gemv_seg(x, nw, 1e-6, Wq, Wk, Wv, y2)
        else:
            fx.gemv_resid(x, W, res, y2)
        torch.cuda.synchronize()
    finally:
        _budget(0)
        lib().flashb_set_gemv_rows_path(1)
        lib().flashb_set_gemv_split(0)
        lib().flashb_set_gemv_group_rows(64)   # the library's default
    assert path == 2, f'expected the tcgen05 kernel, got path {path}'
    assert got_split == split, f'expected split {split}, got {got_split}'
    assert_close(np32(y), ref, what=f'tcgen05 {kind} M={M} rows={rows} split={split}')
    assert torch.equal(y, y2)
    from flashb._native import device_error
    assert device_error() == 0


@pytest.mark.parametrize('kind,M,budget', [
    ('qkv', 128, 0), ('o', 128, 0), ('gateup', 128, 0), ('down', 128, 0),
    ('qkv', 17, 0), ('o', 64, 0), ('gateup', 100, 0), ('down', 33, 0),
    ('qkv', 128, 64), ('gateup', 128, 40), ('down', 128, 18), ('odd', 70, 0), ('o', 128, 16)])
def test_gemv_many_rows_matches_oracle(ops, kind, M, budget):
    """17..128 activation rows without norm: the many-rows tcgen05 kernel (rows as the MMA's M side, 128-unit tiles,
    K split over a cluster chosen from the occupancy API, partial sums pushed through distributed shared memory).
    Checked against the oracle at the backbone's shapes and at SM budgets that force other splits, and for identical
    bits on a second call."""
    fx, _ = ops
    from flashb._native import lib
    K = {'down': 6144, 'odd': 1024}.get(kind, 2048)
    x = randn((M, K), 61)
    try:
        _budget(budget)
        if kind == 'gateup':
            Wg, Wu = randn((6144, K), 63, 0.02), randn((6144, K), 64, 0.02)
            y = torch.empty(M, 6144, dtype=torch.bfloat16, device='cuda')
            call = lambda out: fx.gemv_gateup(x, None, 1e-6, Wg, Wu, out)
            ref = dec.silu_mul(dec.linear(np32(x), np32(Wg)), dec.linear(np32(x), np32(Wu)))
        elif kind == 'qkv':
            Wq, Wk, Wv = randn((2048, K), 65, 0.02), randn((512, K), 66, 0.02), randn((512, K), 67, 0.02)
            y = torch.empty(M, 3072, dtype=torch.bfloat16, device='cuda')
            call = lambda out: fx.gemv_seg(x, None, 1e-6, Wq, Wk, Wv, out)
            ref = dec.gemv_seg(np32(x), None, 1e-6, [np32(Wq), np32(Wk), np32(Wv)])
        else:
            N = 304 if kind == 'odd' else 2048
            W = randn((N, K), 68, 0.02)
            res = randn((M, N), 69)
            y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
            call = lambda out: fx.gemv_resid(x, W, res, out)
            ref = dec.gemv_resid(np32(x), np32(W), np32(res))
        call(y)
        torch.cuda.synchronize()
        path, split = _path(), _split()
        y2 = torch.full_like(y, float('nan'))
        call(y2)
        torch.cuda.synchronize()
    finally:
        _budget(0)
    assert path == 3, f'expected the many-rows kernel, got path {path}'
    assert 1 <= split <= 8
    assert_close(np32(y), ref, what=f'many-rows {kind} M={M} budget={budget} split={split}')
    assert torch.equal(y, y2), 'a second call must give the same bits'
    from flashb._native import device_error
    assert device_error() == 0
