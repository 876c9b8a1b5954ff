"""Streaming-frame oracle (test infrastructure; see ``oracle/__init__.py``).

One frame of the reference's streaming loop (``flash/main_loop.py:252-312``) on the oracle's backbone step
(``oracle.decode.backbone_step``) and depth frame (``oracle.depth.depth_frame``):

    ids      = [cb0, depth tokens[0 : C-1]] of the previous frame, both CFG rows     (main_loop.py:268, 310-312)
    backbone = one decode step at the next cache slot (position advanced first)    (main_loop.py:123-140)
    cb0      = argmax of the CFG logits over ids < n_valid: the greedy branch of sample_logits (flash/sampling.py),
               EOS / reserved ids suppressed
    depth    = every depth codebook with the CFG top-k sampler, Exp(1) draws q supplied        (main_loop.py:260)

Also the seeded synthetic weights that the CPU baseline times (numpy RNG; the same shapes as the GPU bench's
synthetic models, not the same values).
"""
import numpy as np

from . import decode as dec
from . import depth as odepth
from .bf16 import round_bf16

F32 = np.float32
BF16_MIN = F32(-3.3895313892515355e38)


class _Pools:
    """Seeded bf16 value pools, one per (std, mean); a weight is a rotated slice of its pool (a fresh copy, so every
    matrix has its own memory).  Drawing 1.4 G values one by one takes minutes in numpy; the CPU baseline only needs
    weights of the right shapes and magnitudes, so this keeps its setup to seconds."""

    def __init__(self, rng, n=1 << 24):
        self.rng, self.n, self.pools = rng, n, {}

    def __call__(self, shape, std=1.0, mean=0.0):
        key = (float(std), float(mean))
        p = self.pools.get(key)
        if p is None:
            p = self.rng.standard_normal(self.n, dtype=F32)
            p = round_bf16(p * F32(std) + F32(mean))
            self.pools[key] = p
        count = int(np.prod(shape))
        out = np.empty(count, F32)
        off = int(self.rng.integers(0, self.n))
        done = 0
        while done < count:
            k = min(count - done, self.n - off)
            out[done:done + k] = p[off:off + k]
            done += k
            off = 0
        return out.reshape(shape)


def synthetic_backbone(rng, layers, hidden, heads, kv_heads, ffn, vocab, codebooks, eps=1e-6, theta=1e6, D=128):
    _bf = _Pools(rng)
    Ls = []
    for _ in range(layers):
        Ls.append(dict(ln1=_bf((hidden,), 0.1, 1.0), wq=_bf((heads * D, hidden), 0.02),
                       wk=_bf((kv_heads * D, hidden), 0.02), wv=_bf((kv_heads * D, hidden), 0.02),
                       qn=_bf((D,), 0.1, 1.0), kn=_bf((D,), 0.1, 1.0),
                       wo=_bf((hidden, heads * D), 0.02), ln2=_bf((hidden,), 0.1, 1.0),
                       wg=_bf((ffn, hidden), 0.02), wu=_bf((ffn, hidden), 0.02),
                       wd=_bf((hidden, ffn), 0.02)))
    return dec.BackboneWeights(Ls, _bf((hidden,), 0.1, 1.0), _bf((codebooks * vocab, hidden)),
                               _bf((vocab, hidden), 0.02), vocab, eps, theta)


def synthetic_depth(rng, layers, hidden, embed_dim, heads, kv_heads, ffn, vocab, codebook_size, n_decode, eps=1e-5,
                    theta=5e5, D=128):
    _bf = _Pools(rng)
    Ls = []
    for _ in range(layers):
        Ls.append(dict(ln1=_bf((hidden,), 0.1, 1.0), wq=_bf((heads * D, hidden), 0.02),
                       wk=_bf((kv_heads * D, hidden), 0.02), wv=_bf((kv_heads * D, hidden), 0.02),
                       wo=_bf((hidden, heads * D), 0.02), ln2=_bf((hidden,), 0.1, 1.0),
                       wg=_bf((ffn, hidden), 0.02), wu=_bf((ffn, hidden), 0.02),
                       wd=_bf((hidden, ffn), 0.02)))
    head32 = _bf((n_decode, hidden, vocab), 0.02)
    return odepth.DepthWeights(Ls, _bf(((n_decode + 1) * vocab, embed_dim)), _bf((hidden, embed_dim), 0.02),
                               _bf((hidden,), 0.1, 1.0), head32, vocab, codebook_size, n_decode, eps, theta,
                               heads, kv_heads, D)


def greedy_cb0(cfg_row, n_valid):
    """torch.argmax semantics on cfg_row[:n_valid]: first maximal index, a NaN counts as the maximum."""
    r = np.asarray(cfg_row[:n_valid], F32)
    nan = np.isnan(r)
    if nan.any():
        return int(np.argmax(nan))
    return int(np.argmax(r))


class FrameStream:
    """One stream's state: per-layer KV caches (float32 holding bf16), mask, positions, last frame's tokens."""

    def __init__(self, BW, n_decode, prompt_len, max_seq_len, rng, n_valid, batch=2, D=128):
        nkv = BW.layers[0]['wk'].shape[0] // D
        S = max_seq_len
        _bf = _Pools(rng, 1 << 22)
        self.kcs, self.vcs = [], []
        for _ in BW.layers:
            k = np.zeros((batch, nkv, S, D), F32)
            v = np.zeros((batch, nkv, S, D), F32)
            k[:, :, :prompt_len] = _bf((batch, nkv, prompt_len, D))
            v[:, :, :prompt_len] = _bf((batch, nkv, prompt_len, D))
            self.kcs.append(k)
            self.vcs.append(v)
        self.mask = np.full((batch, 1, 1, S), BF16_MIN, F32)
        self.mask[..., :prompt_len] = 0.0
        self.pos = prompt_len - 1                      # the next frame writes slot prompt_len
        self.position_ids = np.full(batch, prompt_len - 1, np.int64)
        self.first_cb = np.full(batch, int(rng.integers(0, n_valid)), np.int64)
        self.outtok = np.repeat(rng.integers(0, n_valid, (1, n_decode)), batch, axis=0).astype(np.int64)
        self.batch = batch


def frame(BW, DW, st, n_valid, gs_bb, depth_params, q):
    """Advance ``st`` by one frame; returns (frame tokens [1 + n_decode], backbone cfg logits, depth logits)."""
    C = BW.embed.shape[0] // BW.vocab
    ids = np.concatenate([st.first_cb[:, None], st.outtok[:, :C - 1]], axis=1)
    st.pos += 1
    st.position_ids += 1
    st.mask[..., st.pos] = 0.0
    h, _, cfg = dec.backbone_step(BW, ids, st.kcs, st.vcs, st.mask, st.pos, st.position_ids, gs_bb)
    cb0 = greedy_cb0(cfg[0], n_valid)
    st.first_cb[:] = cb0
    temp, topk, topp, ds, gs = depth_params
    _, dlog, sampled = odepth.depth_frame(DW, h, st.first_cb, q, temp, topk, topp, ds, gs)
    st.outtok = sampled
    return np.concatenate([[cb0], sampled[0]]), cfg, dlog
