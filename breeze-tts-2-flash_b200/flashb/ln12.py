"""LN12: the reference's lossless 12-bit storage of bf16 depth-decoder weights (``flash/ln12_format.py``), written
anew from the format's definition so that flashb reads and writes the same bytes.

A bf16 value is its high byte H (sign + the 7 high exponent bits e1) and its low byte (exponent LSB + 7 mantissa
bits).  The low byte is stored raw; H becomes a nibble: the sign and a 3-bit index into an 8-entry table of e1 values
chosen per matrix (the 8 most frequent), optionally shifted by -4..3 for a row whose exponents sit elsewhere.
Values whose e1 is not in the row's table are "patches": stored exactly as (column << 8) | H.  That is 12 bits a
weight plus a 16-byte record per row (LN12i, the inline layout the reference's kernels read) and the rare overflow
patches.

Byte layout of a matrix W[N, K] (K % 1024 == 0), fixed by the reference's GEMV lane mapping (lane l of a warp owns
elements k = 1024 g + 256 c + 8 l + j of chunk c = 0..3, j = 0..7 of each 1024-column group g):

    data[n][g][slot][lane][16 B]   slot 0: low bytes of chunks 0, 1 (8 + 8); slot 1: chunks 2, 3; slot 2: four
                                   32-bit nibble words (chunks 0..3) -- word bits 4j..4j+2 = index of element j, the
                                   sign of element j < 4 at bit 8j + 7, of element j >= 4 at bit 8 (j - 4) + 3
    meta[n] = {hdr, p0, p1, p2}    hdr = (overflow offset << 13) | ((shift & 7) << 10) | patch count; the first three
                                   patches inline (unused slots 0xFFFFFFFF), the rest at ovf[offset ..]
    lut                            the 8 table entries (ascending), as two little-endian uint32 (lo, hi)

``encode`` returns (data uint8, meta uint32 [N, 4], ovf uint32, lut uint8[8]); ``decode`` inverts it exactly (numpy,
the CPU reference of ``flashb_ln12_decode``).
"""
import numpy as np

NLUT = 8
SHIFTS = (0, 1, -1, 2, -2, 3, -3, -4)      # per-row table shifts, in order of preference (ties keep the earlier)


def _e1(u):
    return ((u >> 8) & 0x7F).astype(np.uint8)


def table(u):
    """The matrix's 8 most frequent e1 values (ties: the smaller value first), ascending."""
    counts = np.bincount(_e1(u).ravel(), minlength=128)
    order = sorted(range(128), key=lambda v: (-counts[v], v))
    return np.array(sorted(order[:NLUT]), np.uint8)


def _row_shifts(e1, lut):
    """Per row, the shift of the table that covers the most of its values (ties: earlier in SHIFTS)."""
    N = e1.shape[0]
    key = (np.arange(N, dtype=np.int64)[:, None] << 7) | e1
    hist = np.bincount(key.ravel(), minlength=N * 128).reshape(N, 128)
    best = np.full(N, -2, np.int64)
    shift = np.zeros(N, np.int64)
    for sh in SHIFTS:
        vals = lut.astype(np.int64) + sh
        if vals.min() < 0 or vals.max() > 127:
            cover = np.full(N, -1, np.int64)
        else:
            cover = hist[:, vals].sum(axis=1)
        better = cover > best
        best[better] = cover[better]
        shift[better] = sh
    return shift


def encode_hdr(u, lut):
    """LN12 with the row header / patch list of the non-inline layout: (data, hdr uint32 [N], patches uint32)."""
    u = np.asarray(u, np.uint16)
    N, K = u.shape
    if K % 1024:
        raise ValueError('LN12 needs K % 1024 == 0')
    G = K // 1024
    e1 = _e1(u)
    shift = _row_shifts(e1, lut)
    # index of each value's e1 in its row's shifted table (the later entry when two are equal, never the case for a
    # table of distinct values); 8 = not in the table (a patch).  inv maps e1 - shift + 8 (0 .. 139) to the index.
    inv = np.full(144, NLUT, np.uint8)
    for i in range(NLUT):
        inv[int(lut[i]) + 8] = i
    idx = inv[(e1.astype(np.int16) - shift.astype(np.int16)[:, None] + 8)]
    esc = idx == NLUT
    idx = np.where(esc, np.uint8(0), idx)
    pr, pc = np.nonzero(esc)                                                # row-major order
    patches = (pc.astype(np.uint32) << 8) | (u[pr, pc] >> 8).astype(np.uint32)
    count = np.bincount(pr, minlength=N).astype(np.int64)
    offset = np.concatenate([[0], np.cumsum(count)[:-1]]).astype(np.int64)
    if N and (count.max() >= 1024 or offset[-1] + count[-1] >= (1 << 19)):
        raise ValueError('LN12 patch header overflow')
    hdr = ((offset << 13) | ((shift & 7) << 10) | count).astype(np.uint32)
    # nibble words: 8 elements per word
    sign = (u >> 15).astype(np.uint8).reshape(N, K // 8, 8)
    ix = idx.reshape(N, K // 8, 8)
    words = np.zeros((N, K // 8), np.uint32)
    for j in range(8):
        words |= ix[..., j].astype(np.uint32) << np.uint32(4 * j)
        words |= sign[..., j].astype(np.uint32) << np.uint32(8 * j + 7 if j < 4 else 8 * (j - 4) + 3)
    low = (u & 0xFF).astype(np.uint8).reshape(N, G, 4, 32, 8)                # [n, g, chunk, lane, j]
    data = np.empty((N, G, 3, 32, 16), np.uint8)
    data[:, :, 0, :, :8], data[:, :, 0, :, 8:] = low[:, :, 0], low[:, :, 1]
    data[:, :, 1, :, :8], data[:, :, 1, :, 8:] = low[:, :, 2], low[:, :, 3]
    w4 = np.ascontiguousarray(words.reshape(N, G, 4, 32).transpose(0, 1, 3, 2))   # [n, g, lane, chunk]
    data[:, :, 2] = w4.view(np.uint8).reshape(N, G, 32, 16)
    return data.reshape(-1), hdr, patches.astype(np.uint32)


def inline(hdr, patches):
    """The inline row records (LN12i): meta [N, 4] uint32 and the overflow patches."""
    N = hdr.size
    count = (hdr & np.uint32(1023)).astype(np.int64)
    start = (hdr >> np.uint32(13)).astype(np.int64)
    shift_bits = (hdr >> np.uint32(10)) & np.uint32(7)
    meta = np.full((N, 4), 0xFFFFFFFF, np.uint32)
    for s in range(3):
        has = count > s
        meta[has, 1 + s] = patches[start[has] + s]
    extra = np.maximum(count - 3, 0)
    ooff = np.concatenate([[0], np.cumsum(extra)[:-1]]).astype(np.int64)
    if N and ooff[-1] + extra[-1] >= (1 << 19):
        raise ValueError('LN12 overflow offset too large')
    ovf = [patches[start[n] + 3:start[n] + count[n]] for n in range(N) if count[n] > 3]
    ovf = np.concatenate(ovf).astype(np.uint32) if ovf else np.zeros(0, np.uint32)
    meta[:, 0] = (ooff.astype(np.uint32) << np.uint32(13)) | (shift_bits << np.uint32(10)) | count.astype(np.uint32)
    return meta, ovf


def encode(w):
    """bf16 matrix (uint16 bits, or a torch bf16 tensor) -> (data, meta, ovf, lut) of the LN12i layout."""
    u = _bits(w)
    lut = table(u)
    data, hdr, patches = encode_hdr(u, lut)
    meta, ovf = inline(hdr, patches)
    return data, meta, ovf, lut


def decode(data, meta, ovf, lut, N, K):
    """The bf16 bits [N, K] (uint16) of an LN12i matrix."""
    G = K // 1024
    d = np.asarray(data, np.uint8).reshape(N, G, 3, 32, 16)
    meta = np.asarray(meta, np.uint32).reshape(N, 4)
    hdr = meta[:, 0]
    count = (hdr & np.uint32(1023)).astype(np.int64)
    ooff = (hdr >> np.uint32(13)).astype(np.int64)
    sh = ((hdr >> np.uint32(10)) & np.uint32(7)).astype(np.int64)
    sh = np.where(sh >= 4, sh - 8, sh)
    rows_lut = (np.asarray(lut, np.int64)[None, :] + sh[:, None]) & 0xFF        # [N, 8]
    low = np.empty((N, G, 4, 32, 8), np.uint8)
    low[:, :, 0], low[:, :, 1] = d[:, :, 0, :, :8], d[:, :, 0, :, 8:]
    low[:, :, 2], low[:, :, 3] = d[:, :, 1, :, :8], d[:, :, 1, :, 8:]
    words = np.ascontiguousarray(d[:, :, 2]).view(np.uint32).reshape(N, G, 32, 4).transpose(0, 1, 3, 2)
    words = words.reshape(N, K // 8)
    high = np.empty((N, K // 8, 8), np.uint32)
    for j in range(8):
        ix = ((words >> np.uint32(4 * j)) & np.uint32(7)).astype(np.int64)
        s = (words >> np.uint32(8 * j + 7 if j < 4 else 8 * (j - 4) + 3)) & np.uint32(1)
        high[..., j] = np.take_along_axis(rows_lut, ix, axis=1).astype(np.uint32) | (s << np.uint32(7))
    high = high.reshape(N, K)
    for n in np.nonzero(count)[0]:
        for p in range(count[n]):
            v = int(meta[n, 1 + p]) if p < 3 else int(ovf[ooff[n] + p - 3])
            high[n, v >> 8] = v & 0xFF
    return ((high.astype(np.uint16) << np.uint16(8)) | low.reshape(N, K).astype(np.uint16)).astype(np.uint16)


def lut_words(lut):
    """The table as the (lo, hi) little-endian uint32 pair."""
    l8 = np.ascontiguousarray(np.asarray(lut, np.uint8))
    return int(l8[:4].view(np.uint32)[0]), int(l8[4:].view(np.uint32)[0])


def _bits(w):
    if isinstance(w, np.ndarray):
        return w.astype(np.uint16)
    import torch
    return w.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def to_device(data, meta, ovf, lut, device):
    """An encoded matrix as the device tensors the kernels read: (data uint8, meta int32 [N, 4], ovf int32, (lo, hi))."""
    import torch
    d = torch.from_numpy(np.ascontiguousarray(data, np.uint8)).to(device)
    m = torch.from_numpy(np.ascontiguousarray(meta, np.uint32).view(np.int32)).to(device)
    o = np.ascontiguousarray(ovf, np.uint32).view(np.int32)
    o = torch.from_numpy(o if o.size else np.zeros(1, np.int32)).to(device)
    return d, m, o, lut_words(lut)


def decode_device(data, meta, ovf, lut, out):
    """``flashb_ln12_decode``: device LN12 tensors (``to_device``; lut as (lo, hi) or 8 table bytes) -> out [N, K]
    bf16 (written in place), on the current stream."""
    import torch
    from . import _native
    from ._native import check
    lo, hi = lut if isinstance(lut, tuple) else lut_words(lut)
    N, K = out.shape
    if out.dtype != torch.bfloat16 or out.stride(1) != 1 or data.numel() != N * K * 3 // 2 or meta.numel() != N * 4:
        raise ValueError('ln12: tensors do not match out [N, K] bf16')
    check(_native.lib().flashb_ln12_decode(data.data_ptr(), meta.data_ptr(), ovf.data_ptr(), int(lo) & 0xFFFFFFFF,
                                           int(hi) & 0xFFFFFFFF, N, K, out.data_ptr(), out.stride(0),
                                           torch.cuda.current_stream(out.device).cuda_stream))
    return out
