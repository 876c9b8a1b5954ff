"""GPU parity of the backbone sampler (``flashb_cb0_sample``, ``flashb.sampling``): tokens and validity flags
bitwise equal to the C oracle (oracle/sampler.c fb_bb_sample_row, itself pinned to the reference's own
flash/sampling.py sample_logits by tests/golden/bb_sampler.npz) on the same logits and Exp(1) draws."""
import numpy as np
import pytest
import torch

from oracle import sampler as osmp

pytestmark = pytest.mark.gpu


def _oracle(x, present, pen, sup, temp, topk, topp, ds, q):
    out = [osmp.bb_sample_row(x[r], None if present is None else present[r], pen, sup, temp[r], topk[r], topp[r], ds[r],
                              q[r]) for r in range(x.shape[0])]
    return np.array([t for t, _ in out]), np.array([o for _, o in out])


def test_backbone_sampler_golden_rows():
    """The reference's golden rows: repetition penalty, suppression, greedy, top-k ties, top-p, invalid rows."""
    import synth
    from flashb.sampling import sample_rows
    c = synth.BB_SAMPLER
    x, present, q, params = synth.bb_sampler_cases()
    z = np.load(synth.__file__.rsplit('/', 1)[0] + '/bb_sampler.npz')
    sup = torch.tensor(c['suppress'], dtype=torch.long, device='cuda')
    for r, (pen, temp, topk, topp, ds, use_sup) in enumerate(params):
        tok, ok = sample_rows(x[r:r + 1].cuda(), temp, topk, topp, ds, present[r:r + 1].to(torch.uint8).cuda(), pen,
                              sup if use_sup else None, q=q[r:r + 1].cuda())
        torch.cuda.synchronize()
        assert (int(tok[0]), int(ok[0])) == (int(z['tokens'][r]), int(z['ok'][r])), f'row {r} {params[r]}'


@pytest.mark.parametrize('V,topk,topp,ds', [(2049, 50, 1.0, 1), (2049, 0, 0.9, 1), (2049, 50, 0.8, 1),
                                            (4096, 1024, 0.95, 1), (100, 7, 1.0, 1), (2049, 50, 1.0, 0),
                                            (1, 0, 1.0, 1), (3000, 2999, 0.5, 1)])
def test_backbone_sampler_many_rows(V, topk, topp, ds):
    """64 rows at once (one per stream of a slot set), per-row temperatures, a presence mask with penalty 1.1 and
    the reserved ids suppressed; the tokens are also written as CFG-pair ids (blocks of 8 pairs) and marked in the
    presence mask."""
    from flashb.sampling import sample_rows
    R = 64
    g = torch.Generator().manual_seed(V + topk)
    x = torch.randn(R, V, generator=g) * 3.0
    x[::5, :V // 3] = torch.round(x[::5, :V // 3])          # many exact ties
    present = (torch.rand(R, V, generator=g) < 0.1).to(torch.uint8)
    q = torch.empty(R, V).exponential_(1.0, generator=g)
    temp = 0.5 + torch.rand(R, generator=g)
    sup = torch.tensor([V - 1] if V > 1 else [], dtype=torch.long)
    xc, pc, qc = x.cuda(), present.cuda(), q.cuda()
    ids = torch.full((2 * R,), -1, dtype=torch.long, device='cuda')
    tok, ok = sample_rows(xc, temp.cuda(), topk, topp, ds, pc.clone(), 1.1, sup.cuda(), q=qc)
    _, _ = sample_rows(xc, temp.cuda(), topk, topp, ds, pc, 1.1, sup.cuda(), q=qc, tokens=ids, pair_half=8,
                       mark_present=True)
    torch.cuda.synchronize()
    ref_t, ref_ok = _oracle(x.numpy(), present.numpy(), 1.1, sup.tolist(), temp.numpy(), [topk] * R, [topp] * R,
                            [ds] * R, q.numpy())
    np.testing.assert_array_equal(tok.cpu().numpy(), ref_t)
    np.testing.assert_array_equal(ok.cpu().numpy(), ref_ok)
    blocks = ids.view(R // 8, 2, 8)
    assert torch.equal(blocks[:, 0].reshape(-1), tok) and torch.equal(blocks[:, 1].reshape(-1), tok)
    marked = pc.cpu().numpy()[np.arange(R), ref_t]
    assert (marked == 1).all()


def test_sample_logits_surface():
    """The reference's call signature (one row, 0-dim ok) on the device."""
    from flashb.sampling import sample_logits
    V = 2049
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(1, V, generator=g) * 3).cuda()
    q = torch.empty(1, V).exponential_(1.0, generator=g).cuda()
    present = torch.zeros(1, V, dtype=torch.bool, device='cuda')
    present[0, :100] = True
    tok, ok = sample_logits(x, temperature=0.9, top_k=50, top_p=1.0, do_sample=True, present=present,
                            repetition_penalty=1.1, suppress_idx=torch.tensor([2048], device='cuda'), q=q)
    t_ref, ok_ref = osmp.bb_sample_row(x[0].cpu().numpy(), present[0].cpu().numpy(), 1.1, [2048], 0.9, 50, 1.0, 1,
                                       q[0].cpu().numpy())
    assert tok.shape == (1,) and ok.dim() == 0 and bool(ok) == bool(ok_ref) and int(tok[0]) == t_ref
