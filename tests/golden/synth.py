"""Seeded synthetic inputs shared by the golden-fixture generator and the tests (test infrastructure).

Every tensor comes from ``torch.randn`` on a CPU ``torch.Generator`` seeded per fixture, scaled, then cast to bf16,
so the generator script (run once in the build container, next to the reference) and the tests (run anywhere with
the same torch build) see identical values.  ``digest`` fingerprints the inputs so a fixture is never compared
against drifted inputs.
"""
import hashlib

import numpy as np
import torch


def gen(seed):
    return torch.Generator().manual_seed(int(seed))


def randn_bf16(g, shape, std=1.0, mean=0.0):
    return (torch.randn(shape, generator=g) * std + mean).to(torch.bfloat16)


def digest(*tensors):
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()[:16]


# ---------------------------------------------------------------- decode attention (small S)
ATTN = dict(seed=100, B=2, NH=16, NKV=4, D=128, S=80, valid=((0, 70), (5, 70)))


def attn_inputs(c=ATTN):
    g = gen(c['seed'])
    q = randn_bf16(g, (c['B'], c['NH'], 1, c['D']))
    k = randn_bf16(g, (c['B'], c['NKV'], c['S'], c['D']))
    v = randn_bf16(g, (c['B'], c['NKV'], c['S'], c['D']))
    mask = torch.full((c['B'], 1, 1, c['S']), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    for b, (lo, hi) in enumerate(c['valid']):
        mask[b, 0, 0, lo:hi + 1] = 0
    return q, k, v, mask


# ---------------------------------------------------------------- decode attention at config 1's exact shapes
# B 2 (CFG pair), 16 q / 4 KV heads, head_dim 128, KV length 1024, every key valid, q/k/v ~ N(0, 1), seed 0
ATTN1 = dict(seed=0, B=2, NH=16, NKV=4, D=128, S=1024)


def attn1_inputs(c=ATTN1):
    g = gen(c['seed'])
    q = randn_bf16(g, (c['B'], c['NH'], 1, c['D']))
    k = randn_bf16(g, (c['B'], c['NKV'], c['S'], c['D']))
    v = randn_bf16(g, (c['B'], c['NKV'], c['S'], c['D']))
    return q, k, v


# ---------------------------------------------------------------- RMSNorm + gate/up + SiLU + down (config 2, small)
GEMV = dict(seed=101, M=2, K=512, F=384, eps=1e-6)


def gemv_inputs(c=GEMV):
    g = gen(c['seed'])
    x = randn_bf16(g, (c['M'], c['K']))
    gamma = randn_bf16(g, (c['K'],), std=0.1, mean=1.0)
    wg = randn_bf16(g, (c['F'], c['K']), std=0.02)
    wu = randn_bf16(g, (c['F'], c['K']), std=0.02)
    wd = randn_bf16(g, (c['K'], c['F']), std=0.02)
    return x, gamma, wg, wu, wd


# ---------------------------------------------------------------- config 2 at its exact shapes
# x [2, 2048] ~ N(0, 1), gamma = 1 + 0.1 N(0, 1), eps 1e-6, W1 [6144, 2048] ~ N(0, 0.02) (rows 0..3071 gate,
# 3072..6143 up), then the SwiGLU down projection W2 [2048, 3072] ~ N(0, 0.02) with the residual x; seed 1
GEMV2 = dict(seed=1, M=2, K=2048, F=3072, eps=1e-6)


def gemv2_inputs(c=GEMV2):
    g = gen(c['seed'])
    x = randn_bf16(g, (c['M'], c['K']))
    gamma = randn_bf16(g, (c['K'],), std=0.1, mean=1.0)
    w1 = randn_bf16(g, (2 * c['F'], c['K']), std=0.02)
    w2 = randn_bf16(g, (c['K'], c['F']), std=0.02)
    return x, gamma, w1[:c['F']], w1[c['F']:], w2


# ---------------------------------------------------------------- backbone decode step (config 3, reduced)
BACKBONE = dict(seed=102, B=2, H=512, NH=8, NKV=2, D=128, F=1024, L=2, vocab=65, ncb=16, theta=1e6, eps=1e-6,
                S=96, prefill=60, pad=(0, 3), gs=4.0)


# the full config 3 model (28 layers, hidden 2048, FFN 6144, 16 q / 4 KV heads), KV length 1023 + the new token: the
# end-to-end drift study of make_golden.py (bf16 eager vs fp32, and the oracle's summation order vs torch's)
BACKBONE28 = dict(seed=106, B=2, H=2048, NH=16, NKV=4, D=128, F=6144, L=28, vocab=2049, ncb=16, theta=1e6, eps=1e-6,
                  S=1024, prefill=1023, pad=(0, 3), gs=4.0)


# LN12: a bf16 matrix like a depth weight (normal, std 0.02) with what makes the format's special cases: a row at
# 2^-5 scale and one at 2^6 (their exponents leave the table: a shifted row table), a few huge and tiny values
# (patches), a row with more than three patches (the overflow list), and exact zeros
LN12 = dict(seed=108, N=48, K=2048)


def ln12_matrix(c=LN12):
    g = gen(c['seed'])
    w = torch.randn(c['N'], c['K'], generator=g) * 0.02
    w[5] *= 2.0 ** -5
    w[9] *= 2.0 ** 6
    w[13, [3, 700, 1500, 2047, 1024]] = torch.tensor([300.0, -1e-9, 7e4, -2e-7, 1e-3])
    w[20, 17] = -65000.0
    w[31, :64] = 0.0
    return w.to(torch.bfloat16)


# the whole prefill forward (BackbonePrefillGraphCache._forward) on the BACKBONE weights: 24 prompt tokens, row 1
# left-padded by 5 (positions and causal mask as the reference prefill forms them)
PREFILL_FWD = dict(seed=107, L=24, pads=(0, 5))


def prefill_forward_inputs(c=BACKBONE, p=PREFILL_FWD):
    """emb [B, L, H] bf16 (pad tokens zero), causal mask [B, 1, L, S] bf16 (finfo.min / 0), position_ids [B, L],
    cache_position [L], as ``_copy_inputs`` / ``_update_causal_mask`` of the reference prefill build them."""
    g = gen(p['seed'])
    B, L, S, H = c['B'], p['L'], c['S'], c['H']
    emb = randn_bf16(g, (B, L, H))
    am = torch.ones(B, L, dtype=torch.long)
    for b, pad in enumerate(p['pads']):
        am[b, :pad] = 0
        emb[b, :pad] = 0
    pos = am.cumsum(-1) - 1
    pos.masked_fill_(am == 0, 1)
    qi, ki = torch.arange(L).view(1, L, 1), torch.arange(S).view(1, 1, S)
    valid = torch.zeros(B, S, dtype=torch.bool)
    valid[:, :L] = am.bool()
    mask = torch.full((B, 1, L, S), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    mask[:, 0].masked_fill_((ki <= qi) & valid[:, None, :], 0.0)
    return emb, mask, pos, torch.arange(L)


def backbone_weights(c=BACKBONE):
    """Returns a dict of bf16 tensors (lm_head fp32, bf16-exact)."""
    g = gen(c['seed'])
    H, NH, NKV, D, F = c['H'], c['NH'], c['NKV'], c['D'], c['F']
    layers = []
    for _ in range(c['L']):
        layers.append(dict(
            ln1=randn_bf16(g, (H,), 0.1, 1.0), wq=randn_bf16(g, (NH * D, H), 0.02), wk=randn_bf16(g, (NKV * D, H), 0.02),
            wv=randn_bf16(g, (NKV * D, H), 0.02), qn=randn_bf16(g, (D,), 0.1, 1.0), kn=randn_bf16(g, (D,), 0.1, 1.0),
            wo=randn_bf16(g, (H, NH * D), 0.02), ln2=randn_bf16(g, (H,), 0.1, 1.0), wg=randn_bf16(g, (F, H), 0.02),
            wu=randn_bf16(g, (F, H), 0.02), wd=randn_bf16(g, (H, F), 0.02)))
    norm = randn_bf16(g, (H,), 0.1, 1.0)
    embed = randn_bf16(g, (c['ncb'] * c['vocab'], H), 1.0)
    lm_head = randn_bf16(g, (c['vocab'], H), 0.02).float()
    kv = [(randn_bf16(g, (c['B'], NKV, c['prefill'], D)), randn_bf16(g, (c['B'], NKV, c['prefill'], D)))
          for _ in range(c['L'])]
    ids = torch.randint(0, c['vocab'], (c['B'], 1, c['ncb']), generator=g)
    return dict(layers=layers, norm=norm, embed=embed, lm_head=lm_head, kv=kv, ids=ids)


# ---------------------------------------------------------------- depth frame (config 4, reduced)
DEPTH = dict(seed=103, B=2, H=256, AE=384, NH=2, NKV=1, D=128, F=512, L=2, vocab=64, codebook_size=60, ncb=6,
             theta=500000.0, eps=1e-5, gs=4.0, temp=0.9, topk=50, topp=1.0, q_seed=42)


# the full config 4 depth decoder with 8 CFG pairs (16 rows): the argmax-agreement study of make_golden.py
DEPTH4 = dict(seed=107, B=16, H=1024, AE=2048, NH=8, NKV=2, D=128, F=4096, L=4, vocab=2048, codebook_size=2048,
              ncb=17, theta=500000.0, eps=1e-5, gs=4.0, temp=0.9, topk=50, topp=1.0, q_seed=42)


def depth_weights(c=DEPTH):
    g = gen(c['seed'])
    H, AE, NH, NKV, D, F = c['H'], c['AE'], c['NH'], c['NKV'], c['D'], c['F']
    layers = []
    for _ in range(c['L']):
        layers.append(dict(
            ln1=randn_bf16(g, (H,), 0.1, 1.0), wq=randn_bf16(g, (NH * D, H), 0.02), wk=randn_bf16(g, (NKV * D, H), 0.02),
            wv=randn_bf16(g, (NKV * D, H), 0.02), wo=randn_bf16(g, (H, NH * D), 0.02), ln2=randn_bf16(g, (H,), 0.1, 1.0),
            wg=randn_bf16(g, (F, H), 0.02), wu=randn_bf16(g, (F, H), 0.02), wd=randn_bf16(g, (H, F), 0.02)))
    embed = randn_bf16(g, (c['ncb'] * c['vocab'], AE), 1.0)
    proj = randn_bf16(g, (H, AE), 0.02)
    normf = randn_bf16(g, (H,), 0.1, 1.0)
    head = randn_bf16(g, (c['ncb'] - 1, H, c['vocab']), 0.02).float()
    bh = randn_bf16(g, (c['B'], AE), 1.0)
    first = torch.randint(0, c['codebook_size'], (c['B'] // 2,), generator=g).repeat(2)
    gq = gen(c['q_seed'])
    q = torch.empty(c['ncb'] - 1, c['B'] // 2, c['vocab']).exponential_(1.0, generator=gq)
    return dict(layers=layers, embed=embed, proj=proj, normf=normf, head=head, bh=bh, first=first, q=q)


# ---------------------------------------------------------------- sampler rows (real vocab 2051, codebook 2048)
SAMPLER = dict(seed=104, rows=48, vocab=2051, codebook_size=2048)


def sampler_cases(c=SAMPLER):
    """Per row: cond/uncond logits, q, and parameters (gs, temp, topk, topp, dosample) covering the edge cases."""
    g = gen(c['seed'])
    V = c['vocab']
    params = []
    ks = [50, 1, 0, 1024, 64, 65, 7, 300]
    ps = [1.0, 0.9, 0.5, 0.0, 1.0, 0.95]
    for r in range(c['rows']):
        params.append((float([1.0, 4.0, 0.0, 2.5][r % 4]), float([0.9, 1.0, 0.5, 1.3][(r // 4) % 4]),
                       int(ks[r % len(ks)]), float(ps[(r // 3) % len(ps)]), int(r % 11 != 5)))
    lc = torch.randn((c['rows'], V), generator=g) * 3.0
    lu = lc + torch.randn((c['rows'], V), generator=g) * 0.5
    # exact ties in a few rows: duplicate the best logit at a higher index
    for r in range(0, c['rows'], 6):
        j = int(torch.argmax(lc[r]))
        lc[r, (j + 17) % 2048] = lc[r, j]
        lu[r, (j + 17) % 2048] = lu[r, j]
    q = torch.empty((c['rows'], V)).exponential_(1.0, generator=g)
    return lc, lu, q, params


# ---------------------------------------------------------------- backbone (codebook-0) sampler rows
# the CFG logits row of the backbone: vocab + 1 ids; the runtime's parameters are do_sample, T 0.9, top-k 50,
# top-p 1.0, repetition penalty 1.1 over the ids generated so far, the reserved codec ids suppressed
BB_SAMPLER = dict(seed=108, rows=60, vocab=2049, n_present=300, suppress=(2048, 2047))


def bb_sampler_cases(c=BB_SAMPLER):
    """Per row: logits, presence mask, q, and (penalty, temp, topk, topp, dosample, suppress?) covering the runtime
    defaults, greedy, top-k ties at the threshold, top-p, no top-k, and invalid rows (a NaN; everything
    suppressed)."""
    g = gen(c['seed'])
    V, R = c['vocab'], c['rows']
    x = torch.randn((R, V), generator=g) * 3.0
    present = torch.zeros((R, V), dtype=torch.bool)
    for r in range(R):
        present[r, torch.randperm(V, generator=g)[:c['n_present']]] = True
    q = torch.empty((R, V)).exponential_(1.0, generator=g)
    params = []
    ks = [50, 0, 1, 7, 2049, 50, 64]
    ps = [1.0, 0.9, 0.5, 1.0, 0.95]
    for r in range(R):
        params.append((float([1.1, 1.0, 1.3][r % 3]), float([0.9, 1.0, 0.5, 1.4][(r // 3) % 4]), int(ks[r % len(ks)]),
                       float(ps[(r // 2) % len(ps)]), int(r % 9 != 4), int(r % 5 != 2)))
    # exact ties at the top-k threshold: copy the 7th-largest value onto other ids
    for r in range(0, R, 4):
        v = torch.sort(x[r], descending=True).values[6]
        for j in (11, 500, 1500):
            x[r, j] = v
    x[7, 123] = float('nan')                       # invalid: a NaN in the logits
    x[13] = float('-inf')                          # greedy over nothing finite: index 0
    x[14] = float('-inf')                          # invalid once suppressed: only the suppressed ids are finite
    x[14, 2047], x[14, 2048] = 5.0, 3.0
    return x, present, q, params


# ---------------------------------------------------------------- causal prefill attention (config 5, small L)
PREFILL = dict(seed=105, B=2, NH=16, NKV=4, D=128, L=40, pad=(0, 6))


def prefill_inputs(c=PREFILL):
    g = gen(c['seed'])
    q = randn_bf16(g, (c['B'], c['NH'], c['L'], c['D']))
    k = randn_bf16(g, (c['B'], c['NKV'], c['L'], c['D']))
    v = randn_bf16(g, (c['B'], c['NKV'], c['L'], c['D']))
    L = c['L']
    qi = torch.arange(L).view(L, 1)
    ki = torch.arange(L).view(1, L)
    mask = torch.full((c['B'], 1, L, L), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    for b, p in enumerate(c['pad']):
        allowed = (ki <= qi) & (ki >= p)
        mask[b, 0].masked_fill_(allowed, 0.0)
    return q, k, v, mask


def np_bits(t):
    """bf16 tensor -> uint16 numpy array of its bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
