"""LN12, the reference's lossless 12-bit weight storage (flash/ln12_format.py), on the CPU: flashb's encoder writes
the same bytes as the reference's own encoder (tests/golden/ln12.npz, made by it on a matrix with the format's special
cases), and decoding gives back every bit."""
import numpy as np
import torch

import synth
from flashb import ln12


def _bits(w):
    return w.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_encoder_writes_the_reference_bytes():
    z = np.load(synth.__file__.replace('synth.py', 'ln12.npz'))
    w = synth.ln12_matrix()
    assert str(z['digest']) == synth.digest(w)
    data, meta, ovf, lut = ln12.encode(w)
    assert np.array_equal(lut, z['lut'])
    assert np.array_equal(data, z['data'])
    assert np.array_equal(meta, z['meta'])
    assert np.array_equal(ovf, z['ovf'])
    # the fixture exercises shifted row tables, inline and overflow patches
    hdr = z['meta'][:, 0]
    assert len(set(((hdr >> 10) & 7).tolist())) > 2 and int((hdr & 1023).max()) > 3 and z['ovf'].size > 0


def test_decode_is_lossless():
    z = np.load(synth.__file__.replace('synth.py', 'ln12.npz'))
    u = _bits(synth.ln12_matrix())
    assert np.array_equal(ln12.decode(z['data'], z['meta'], z['ovf'], z['lut'], *u.shape), u)


def test_round_trip_of_weight_like_matrices():
    g = torch.Generator().manual_seed(3)
    for N, K, std in ((64, 1024, 0.02), (16, 4096, 0.5), (8, 2048, 1e-3)):
        w = (torch.randn(N, K, generator=g) * std).to(torch.bfloat16)
        u = _bits(w)
        data, meta, ovf, lut = ln12.encode(u)
        assert data.size == N * K * 3 // 2 and meta.shape == (N, 4)
        assert np.array_equal(ln12.decode(data, meta, ovf, lut, N, K), u)
        # 12 bits a weight plus the row records and the rare patches
        total = data.size + meta.size * 4 + ovf.size * 4 + 8
        assert total < 0.8 * N * K * 2
