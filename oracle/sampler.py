"""ctypes wrapper of ``oracle/sampler.c`` (test infrastructure; see ``oracle/__init__.py``).

``sample_row`` is the bit-exact CPU restatement of the depth sampler (``UP/models/cudagraph/depth_decoder_graph.py:
485-556``; ``flash/csrc/depth_frame.cu:381-654``).  ``sample_row_torch`` restates the same rule with the official
torch ops (topk / sort / softmax / cumsum), with ``torch.multinomial(probs, 1)`` replaced by ``argmax(probs / q)``
(``flash/csrc/depth_frame.cu:6-8``); it is the tolerance-level check of the C version against the official
arithmetic.
"""
import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_LOCK = threading.Lock()


def build():
    """Compile ``oracle/_build/liboracle.so`` (gcc via the Makefile) if missing or stale."""
    so = os.path.join(_HERE, '_build', 'liboracle.so')
    src = os.path.join(_HERE, 'sampler.c')
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(['make', '-s', '-C', _HERE], check=True)
    return so


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            L = ctypes.CDLL(build())
            fp = ctypes.POINTER(ctypes.c_float)
            L.fb_exp.restype = ctypes.c_float
            L.fb_exp.argtypes = [ctypes.c_float]
            L.fb_exp_n.restype = None
            L.fb_exp_n.argtypes = [fp, fp, ctypes.c_int]
            L.fb_sample_row.restype = ctypes.c_int
            L.fb_sample_row.argtypes = [fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_longlong, ctypes.c_float, ctypes.c_longlong, fp,
                                        ctypes.POINTER(ctypes.c_int)]
            L.fb_bb_sample_row.restype = ctypes.c_int
            L.fb_bb_sample_row.argtypes = [fp, ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
                                           ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_float,
                                           ctypes.c_longlong, fp, ctypes.POINTER(ctypes.c_int)]
            _LIB = L
    return _LIB


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def fb_exp(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().fb_exp_n(_fp(x), _fp(y), x.size)
    return y


def sample_row(lc, lu, codebook_size, gs, temp, topk, topp, dosample, q):
    """Returns (token, greedy).  lc/lu: [V] fp32 cond/uncond logits (lu None = no CFG pair); q: [V] fp32."""
    lc = np.ascontiguousarray(lc, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    lu_p = None
    if lu is not None:
        lu = np.ascontiguousarray(lu, np.float32)
        lu_p = _fp(lu)
    g = ctypes.c_int(0)
    t = lib().fb_sample_row(_fp(lc), lu_p, lc.size, int(codebook_size), float(gs), float(temp), int(topk),
                            float(topp), int(dosample), _fp(q), ctypes.byref(g))
    return int(t), int(g.value)


def bb_sample_row(logits, present, penalty, suppress, temp, topk, topp, dosample, q):
    """The backbone sampler (fb_bb_sample_row): returns (token, ok).  logits/q: [V] fp32; present: [V] bool or
    None; suppress: int ids or None."""
    x = np.ascontiguousarray(logits, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    pres = None if present is None else np.ascontiguousarray(present, np.uint8)
    sup = None if suppress is None or len(suppress) == 0 else np.ascontiguousarray(suppress, np.int64)
    ok = ctypes.c_int(0)
    t = lib().fb_bb_sample_row(_fp(x), x.size, None if pres is None else pres.ctypes.data, float(penalty),
                               None if sup is None else sup.ctypes.data, 0 if sup is None else sup.size, float(temp),
                               int(topk), float(topp), int(dosample), _fp(q), ctypes.byref(ok))
    return int(t), int(ok.value)


def sample_rows(logits, half, codebook_size, gs, temp, topk, topp, dosample, q):
    """All half-rows of one step: logits [B, V] (cond rows first, then uncond), q [half, V]; per-half parameters
    given as sequences.  Returns tokens [half]."""
    B = logits.shape[0]
    out = []
    for h in range(half):
        lu = logits[h + half] if B >= 2 else None
        t, _ = sample_row(logits[h], lu, codebook_size, gs[h], temp[h], topk[h], topp[h], dosample[h], q[h])
        out.append(t)
    return np.asarray(out, np.int64)


def sample_row_torch(lc, lu, vocab, codebook_size, gs, temp, topk, topp, dosample, q):
    """The official ``_cfg_sample`` op sequence for one half-row with torch CPU ops (multinomial -> argmax(p/q))."""
    import torch
    import torch.nn.functional as F
    c = torch.as_tensor(np.asarray(lc, np.float32))[None]
    if lu is not None:
        u = torch.as_tensor(np.asarray(lu, np.float32))[None]
        cfg = u + torch.tensor([[gs]], dtype=torch.float32) * (c - u)
    else:
        cfg = c.clone()
    if codebook_size < vocab:
        cfg[..., codebook_size:vocab] = float('-inf')
    scaled = cfg / torch.tensor([[temp]], dtype=torch.float32)
    max_k = min(1024, vocab)
    eff = topk if topk > 0 else max_k
    tv, ti = torch.topk(scaled, max_k)
    tv = torch.where(torch.arange(max_k) < eff, tv, torch.full_like(tv, float('-inf')))
    scaled = torch.full_like(scaled, float('-inf')).scatter_(1, ti, tv)
    sl, si = torch.sort(scaled, descending=True)
    cp = torch.cumsum(F.softmax(sl, dim=-1), dim=-1)
    rm = cp > torch.tensor([[topp]], dtype=torch.float32)
    rm = F.pad(rm[..., :-1], (1, 0), value=False)
    sl = torch.where(rm, torch.full_like(sl, float('-inf')), sl)
    scaled = torch.full_like(scaled, float('-inf')).scatter_(1, si, sl)
    probs = F.softmax(scaled, dim=-1)
    greedy = int(torch.argmax(cfg, dim=-1)[0])
    sampled = int(torch.argmax(probs / torch.as_tensor(np.asarray(q, np.float32))[None], dim=-1)[0])
    tok = sampled if dosample else greedy
    return min(max(tok, 0), vocab - 1), greedy
