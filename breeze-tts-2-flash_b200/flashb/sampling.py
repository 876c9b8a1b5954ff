"""The backbone sampler on the device, with the reference's Python surface (``flash/sampling.py``).

``sample_logits(logits, *, temperature, top_k, top_p, do_sample, present, repetition_penalty, suppress_idx, ok_true)``
returns ``(token, ok)`` like the reference's host-sync-free sampler (``flash/sampling.py:56-97``): the official op
order (repetition penalty on the ids in ``present``, suppression, greedy argmax or temperature / top-k / top-p /
softmax / multinomial) and the multinomial's validity predicate as a device flag instead of a device-side assert.
Here it is one ``flashb_cb0_sample`` launch (one CTA per row) instead of ~10 torch ops.  The multinomial draw is
``argmax(probs / q)`` with ``q`` Exp(1) draws (the identity ``torch.multinomial(p, 1) == argmax(p / Exp(1))``): pass
``q`` to control the randomness, else it is drawn on the device from torch's generator.
"""
import torch

from . import _native
from ._native import check

_INF = float('inf')


class InvalidDistribution(RuntimeError):
    """The backbone sampling distribution is invalid (nan / inf / negative / all-zero probabilities); raised for the
    current request only (the reference's name, ``flash/sampling.py:25-29``)."""


def _rows(t, rows, dtype, device):
    t = torch.as_tensor(t, device=device).to(dtype)
    return (t.reshape(1).expand(rows) if t.numel() == 1 else t.reshape(rows)).contiguous()


def sample_rows(logits, temperature, top_k, top_p, do_sample, present=None, repetition_penalty=1.0,
                suppress_idx=None, q=None, tokens=None, pair_half=0, ok=None, mark_present=False):
    """Every row of ``logits`` [rows, V] fp32 at once (per-row parameters: scalars or [rows] tensors).  Returns
    (tokens, ok [rows] int64 0/1): tokens [rows], or with ``pair_half`` = h > 0 the [2 rows] backbone ids of CFG
    blocks [cond_0 .. cond_{h-1}, uncond_0 .. uncond_{h-1}] (row r's token in both rows of its pair).  ``present``
    [rows, V] uint8/bool presence masks (updated in place with the sampled tokens when ``mark_present``)."""
    def _ensure(cond, msg):
        if not cond:
            raise _native.FlashbError(_native.FB_ERR_ARG, msg)

    _ensure(logits.dtype == torch.float32 and logits.is_cuda and logits.dim() == 2 and logits.stride(1) == 1,
            'logits: [rows, V] fp32 CUDA with unit stride')
    rows, V = logits.shape
    dev = logits.device
    temp = _rows(temperature, rows, torch.float32, dev)
    topk = _rows(top_k, rows, torch.int64, dev)
    topp = _rows(top_p, rows, torch.float32, dev)
    ds = _rows(do_sample, rows, torch.int64, dev)
    if q is None:
        q = torch.empty(rows, V, dtype=torch.float32, device=dev).exponential_(1.0)
    _ensure(q.dtype == torch.float32 and q.shape == (rows, V) and q.stride(1) == 1, 'q: [rows, V] fp32')
    if present is not None:
        _ensure(present.dtype in (torch.uint8, torch.bool) and present.shape[-1] == V and present.stride(-1) == 1,
                'present: [rows, V] uint8/bool')
        present = present.view(torch.uint8) if present.dtype == torch.bool else present
        ldp = present.stride(0) if present.dim() == 2 and present.shape[0] == rows else 0
        _ensure(ldp >= V, 'present: one row per logits row')
    sup = None
    if suppress_idx is not None and suppress_idx.numel() > 0:
        sup = suppress_idx.to(device=dev, dtype=torch.int64).contiguous()
    if tokens is None:
        tokens = torch.empty(2 * rows if pair_half else rows, dtype=torch.int64, device=dev)
    _ensure(tokens.dtype == torch.int64 and tokens.is_contiguous() and tokens.numel() >= (2 if pair_half else 1) * rows,
            'tokens: int64, contiguous, one per row (two with pair_half)')
    ok = torch.empty(rows, dtype=torch.int64, device=dev) if ok is None else ok
    _p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    check(_native.lib().flashb_cb0_sample(
        logits.data_ptr(), logits.stride(0), rows, V, _p(present), ldp if present is not None else 0,
        float(repetition_penalty), _p(sup), 0 if sup is None else sup.numel(), temp.data_ptr(), topk.data_ptr(),
        topp.data_ptr(), ds.data_ptr(), q.data_ptr(), q.stride(0), tokens.data_ptr(), int(pair_half), ok.data_ptr(),
        int(bool(mark_present)), torch.cuda.current_stream(dev).cuda_stream))
    return tokens, ok


def sample_logits(logits, *, temperature, top_k, top_p, do_sample, present=None, repetition_penalty=1.0,
                  suppress_idx=None, ok_true=None, q=None):
    """Drop-in for the reference's ``sample_logits``: logits [..., V] (one row), returns (token of shape
    logits.shape[:-1], 0-dim bool ok) on the device, no host sync."""
    shape = logits.shape[:-1]
    x = logits.reshape(-1, logits.shape[-1]).float().contiguous()
    pres = None
    if present is not None:
        pres = present.reshape(-1, present.shape[-1]).to(torch.uint8)
        if pres.shape[0] == 1 and x.shape[0] > 1:
            pres = pres.expand(x.shape[0], -1).contiguous()
    tok, ok = sample_rows(x, temperature, top_k, top_p, do_sample, pres, repetition_penalty, suppress_idx,
                          q=None if q is None else q.reshape(x.shape).float().contiguous())
    return tok.view(shape), ok.bool().all()
