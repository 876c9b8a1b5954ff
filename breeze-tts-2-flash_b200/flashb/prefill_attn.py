"""Backbone prefill attention on the flashb tcgen05 kernel, with the reference hook's surface
(``flash/prefill_attn.py:1-46``).

``bz_prefill_attention(module, query, key, value, attention_mask, scaling, dropout, **kw)`` follows the reference:
the keys are trimmed to the prefill length L under the same condition, then the attention runs, here as one
``flashb_prefill_attn`` launch (tcgen05 MMAs, fp32 accumulators in TMEM) instead of the eager
``eager_attention_forward``.  It returns ``(out [B, L, NH, D], None)``: the eager probabilities are not materialised
(the prefill graph does not use them).  Shapes the kernel does not cover (head_dim != 128, dropout, non-bf16
tensors) go to the official eager function, as the reference's own checks do.

``install()`` registers it under the reference's name and switches ``BackbonePrefillGraphCache._forward`` to it.

``prefill_attention_sharded`` splits a long prefill over the ranks of a process group and gathers the full output
with one NCCL all-gather into one buffer (``all_gather_into_tensor``): by KV-head group when the ranks divide the KV
heads (each rank reads only its group's K/V), else by query rows in contiguous tile ranges balanced for the causal
work (the N = 8 split of 4 KV heads).
"""
import torch

from . import _native
from ._native import check

NAME = 'bz_prefill'


def _ok(t):
    return t.is_cuda and t.dtype == torch.bfloat16 and t.stride(-1) == 1 and t.shape[-1] == 128


def _trim(query, key, value, attention_mask):
    L = query.shape[2]
    if (L > 1 and key.shape[2] > L and attention_mask is not None and attention_mask.dim() == 4
            and attention_mask.shape[-1] == key.shape[2]):
        return key[:, :, :L], value[:, :, :L], attention_mask[..., :L]
    return key, value, attention_mask


def prefill_attention(query, key, value, attention_mask, scaling, causal=True, heads=None, out=None, tiles=None):
    """q [B, NH, L, 128], k/v [B, NKV, S, 128] bf16 (any strides with unit last stride), additive mask
    [B | 1, 1, L, S] or None -> out [B, L, NH, 128] bf16.  ``heads`` = (h0, h1) computes those q heads only; then
    ``out`` may instead be [B, L, h1 - h0, 128] (head h goes to out[:, :, h - h0]).  ``tiles`` = (t0, t1) computes
    the query rows of 128-row tiles [t0, t1) only; then ``out`` may instead hold just those rows ([B, >= rows, NH,
    128], row 128 t0 first)."""
    B, NH, L, D = query.shape
    NKV, S = key.shape[1], key.shape[2]
    h0, h1 = heads if heads is not None else (0, NH)
    ntile = (L + 127) // 128
    t0, t1 = tiles if tiles is not None else (0, ntile)
    if out is None:
        out = torch.empty(B, L, NH, D, dtype=torch.bfloat16, device=query.device)
    base = out.data_ptr()
    if out.shape[2] == h1 - h0 and h0:
        base -= h0 * out.stride(2) * out.element_size()     # the kernel indexes heads absolutely
    if tiles is not None and out.shape[1] < L and t0:
        base -= t0 * 128 * out.stride(1) * out.element_size()   # ... and query rows too
    m = attention_mask
    if m is not None:
        if m.dtype not in (torch.bfloat16, torch.float32) or m.stride(-1) != 1:
            m = m.to(torch.float32 if m.dtype != torch.bfloat16 else m.dtype).contiguous()
        m_sb = 0 if m.shape[0] == 1 else m.stride(0)
        m_sl = m.stride(2) if m.shape[2] > 1 else 0
    check(_native.lib().flashb_prefill_attn_tiles(
        query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
        key.data_ptr(), key.stride(0), key.stride(1), key.stride(2),
        value.data_ptr(), value.stride(0), value.stride(1), value.stride(2),
        None if m is None else m.data_ptr(), int(m is not None and m.dtype == torch.bfloat16),
        0 if m is None else m_sb, 0 if m is None else m_sl, B, NH, NKV, L, S, D, float(scaling), int(bool(causal)),
        h0, h1, t0, t1, base, out.stride(0), out.stride(1), out.stride(2),
        torch.cuda.current_stream(query.device).cuda_stream))
    return out


def bz_prefill_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """Drop-in for the reference's ``bz_prefill_attention`` (``flash/prefill_attn.py:15-24``)."""
    key, value, attention_mask = _trim(query, key, value, attention_mask)
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    if (dropout and module is not None and getattr(module, 'training', False)) or not all(
            _ok(t) for t in (query, key, value)):
        from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward
        return eager_attention_forward(module, query, key, value, attention_mask, scaling=scaling, dropout=dropout,
                                       **kwargs)
    causal = bool(getattr(module, 'is_causal', True)) if module is not None else True
    return prefill_attention(query, key, value, attention_mask, scaling, causal=causal), None


def shard_heads(NH, NKV, n, r):
    """q-head range [h0, h1) of rank r of n: the q heads of KV groups [r * NKV / n, (r + 1) * NKV / n)."""
    if NKV % n:
        raise ValueError(f'{NKV} KV heads do not split over {n} ranks')
    G, hk = NH // NKV, NKV // n
    return r * hk * G, (r + 1) * hk * G


def row_shards(L, n, causal=True):
    """Contiguous 128-row query-tile ranges [(t0, t1)] of n ranks that minimise the largest rank's work (tile t
    attends to t + 1 key tiles when causal, else every tile costs the same): the smallest capacity whose greedy
    packing needs at most n ranges (binary search), the last ranges possibly empty when there are fewer tiles
    than ranks."""
    T = (L + 127) // 128
    w = [(t + 1) if causal else 1 for t in range(T)]

    def pack(cap):
        bounds, acc = [0], 0
        for t, x in enumerate(w):
            if acc + x > cap and acc > 0:
                bounds.append(t)
                acc = 0
            acc += x
        return bounds

    lo, hi = max(w), sum(w)
    while lo < hi:
        mid = (lo + hi) // 2
        if len(pack(mid)) <= n:
            hi = mid
        else:
            lo = mid + 1
    bounds = pack(lo)
    bounds += [T] * (n + 1 - len(bounds))
    return [(bounds[r], bounds[r + 1]) for r in range(n)]


def gather_head_shards(part, group=None):
    """All-gather every rank's [B, L, NH / n, D] head shard into [B, L, NH, D] (heads in rank order): one NCCL
    all_gather_into_tensor into a rank-major buffer, then one strided copy."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    buf = torch.empty((n * part.shape[0],) + tuple(part.shape[1:]), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(buf, part.contiguous(), group=group)
    B, L, hn, D = part.shape
    return buf.view(n, B, L, hn, D).permute(1, 2, 0, 3, 4).reshape(B, L, n * hn, D)


def gather_row_shards(part, ranges, L, group=None, out=None):
    """All-gather every rank's query-row shard (part [B, R, NH, D], R = the largest range's rows, this rank's rows
    first) into out [B, L, NH, D]: one NCCL all_gather_into_tensor, then each rank's rows copied into place."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    buf = torch.empty((n * part.shape[0],) + tuple(part.shape[1:]), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(buf, part.contiguous(), group=group)
    B, _, NH, D = part.shape
    buf = buf.view((n,) + tuple(part.shape))
    if out is None:
        out = torch.empty(B, L, NH, D, dtype=part.dtype, device=part.device)
    for j, (t0, t1) in enumerate(ranges):
        r0, r1 = t0 * 128, min(L, t1 * 128)
        if r1 > r0:
            out[:, r0:r1].copy_(buf[j, :, :r1 - r0])
    return out


# Shortest prompt 'auto' splits over ranks: measured on 2 x B200, L 512 ran 63 us on one GPU and 101 us split (the
# all-gather dominates), L 4096 1.81 ms on one GPU and 1.14 ms split.
SPLIT_MIN_LEN = 2048


def prefill_attention_sharded(query, key, value, attention_mask, scaling, group=None, causal=True, split='auto'):
    """Multi-GPU prefill attention, every rank of ``group`` returning out [B, L, NH, 128].  split 'heads': each rank
    computes the q heads of its KV-head group (reading only that group's K/V; NKV % world_size == 0); 'rows': each
    rank computes a contiguous range of 128-row query tiles balanced for the causal work (any world size); 'none':
    every rank computes the whole call; 'auto': none below SPLIT_MIN_LEN query rows, else heads when the ranks divide
    the KV heads, else rows."""
    import torch.distributed as dist
    B, NH, L, D = query.shape
    n, r = dist.get_world_size(group), dist.get_rank(group)
    NKV = key.shape[1]
    if split == 'auto':
        split = 'none' if (L < SPLIT_MIN_LEN or n == 1) else ('heads' if NKV % n == 0 else 'rows')
    if split == 'none':
        return prefill_attention(query, key, value, attention_mask, scaling, causal=causal)
    if split == 'heads':
        h0, h1 = shard_heads(NH, NKV, n, r)
        part = torch.empty(B, L, h1 - h0, D, dtype=torch.bfloat16, device=query.device)
        prefill_attention(query, key, value, attention_mask, scaling, causal=causal, heads=(h0, h1), out=part)
        return gather_head_shards(part, group)
    ranges = row_shards(L, n, causal)
    rows = max(min(L, t1 * 128) - t0 * 128 for t0, t1 in ranges)
    part = torch.zeros(B, max(rows, 1), NH, D, dtype=torch.bfloat16, device=query.device)
    t0, t1 = ranges[r]
    if t1 > t0:
        prefill_attention(query, key, value, attention_mask, scaling, causal=causal, out=part, tiles=(t0, t1))
    return gather_row_shards(part, ranges, L, group)


def install(api=None):
    from transformers import AttentionInterface
    from models.cudagraph.backbone_prefill_graph import BackbonePrefillGraphCache
    if getattr(BackbonePrefillGraphCache, '_pf_installed', False):
        return
    _native.lib()
    AttentionInterface.register(NAME, bz_prefill_attention)
    orig = BackbonePrefillGraphCache._forward

    def _forward(self, *a, **k):
        cfg = self.model.layers[0].self_attn.config
        prev = cfg._attn_implementation
        cfg._attn_implementation = NAME
        try:
            return orig(self, *a, **k)
        finally:
            cfg._attn_implementation = prev

    BackbonePrefillGraphCache._forward = _forward
    BackbonePrefillGraphCache._pf_installed = True
    print('[flashb] backbone prefill attention on the tcgen05 kernel', flush=True)
