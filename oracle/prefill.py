"""Prefill-attention oracle (test infrastructure; see ``oracle/__init__.py``).

``bz_prefill_attention`` (``flash/prefill_attn.py:15-24``): when the keys outnumber the queries and the mask is a
4-D tensor over every key, K/V/mask are trimmed to the first L slots (slots >= L are masked with finfo.min, whose
exp underflows to exactly 0, so the trim changes no value), then the eager attention runs
(``UP/models/breeze.py:259-286``; ``oracle.decode.attention_eager``).  Output [B, L, NH, D].
"""
import numpy as np

from . import decode as dec


def trim(q, k, v, mask):
    """The reference's trimming rule: keys sliced to [:L] when L > 1, S > L and the mask covers every key."""
    L = q.shape[2]
    S = k.shape[2]
    if L > 1 and S > L and mask is not None and mask.ndim == 4 and mask.shape[-1] == S:
        return k[:, :, :L], v[:, :, :L], mask[..., :L]
    return k, v, mask


def prefill_attention(q, k, v, mask, scaling, mask_bf16=True):
    """q [B, NH, L, D], k/v [B, NKV, S, D], additive mask [B | 1, 1, L, S] or None -> out [B, L, NH, D]."""
    k, v, mask = trim(q, k, v, mask)
    return dec.attention_eager(np.asarray(q, np.float32), np.asarray(k, np.float32), np.asarray(v, np.float32),
                               mask, scaling, mask_bf16=mask_bf16)
