"""Kernel modules with the reference's call surface (``flash/kernels.py:1-99``), backed by ``libflashb.so``.

The reference JIT-builds four torch extensions and returns their pybind modules; here ``load(name)`` returns a small
Python object per former extension whose methods keep the reference names, argument order and error behaviour
(``RuntimeError`` on a bad tensor) and call the C ABI of ``include/flashb.h`` on the current CUDA stream, so they are
captured by CUDA graphs exactly like the reference's launches.

  flash_bb_attn   attn_decode, attn_decode_fused                   (flash/csrc/bb_attn.cu:462-470)
  flash_bb_fused  gemv_seg, gemv_resid, gemv_gateup, rmsnorm       (flash/csrc/bb_fused.cu:370-378)
                  + embed_rope, lm_head_cfg (the step's eager ends, flash/backbone.py:114-138)
  flash_dd_full / flash_dd_kv   the depth frame (flashb.depth)      (flash/csrc/depth_frame.cu:923-934)
"""
import threading
import time

import torch

from . import _native
from ._native import check

SPECS = {
    'flash_bb_attn': ('fb_attn.cu', 'GQA split-KV decode attention (+ q/k norm, RoPE, KV write)'),
    'flash_bb_fused': ('fb_gemv.cu fb_aux.cu', 'RMSNorm+GEMV, residual GEMV, SwiGLU GEMV, RMSNorm, embed, lm_head'),
    'flash_dd_full': ('fb_depth.cu', 'depth frame kernel'),
    'flash_dd_kv': ('fb_depth.cu', 'depth frame kernel (same build; kept for the reference name)'),
}
_LOCK = threading.Lock()
_MODS = {}
_INFO = {}


def _req(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _bf16(t, name):
    _req(t.is_cuda and t.dtype == torch.bfloat16, f'{name} must be a CUDA bf16 tensor')


class AttnOps:
    """flash_bb_attn: ``attn_decode`` / ``attn_decode_fused`` (flash/csrc/bb_attn.cu:416-460).

    The reference's workspace arguments (``scores``, ``cmax``, ``part``, ``counters``) are accepted for call
    compatibility and unused: the split-KV partials are merged inside each thread-block cluster through distributed
    shared memory.  The optional ``dbg`` probability tap of the reference is not provided."""

    @staticmethod
    def _common(kc, vc, mask, part, counters, out, B, NH):
        _req(kc.dim() == 4 and vc.dim() == 4 and kc.shape == vc.shape and kc.stride() == vc.stride(), 'kc/vc shape')
        _bf16(kc, 'kc')
        _bf16(vc, 'vc')
        _req(kc.shape[0] == B and kc.shape[3] == 128 and kc.stride(3) == 1 and kc.stride(2) == 128, 'kc layout')
        NKV, S = kc.shape[1], kc.shape[2]
        _req(NH % NKV == 0, 'NH must be a multiple of NKV')
        _req(mask.dim() == 4 and mask.shape[-1] >= S and mask.stride(-1) == 1 and mask.shape[2] == 1, 'mask layout')
        _req(mask.shape[0] in (B, 1), 'mask batch')
        _req(mask.dtype in (torch.bfloat16, torch.float32), 'mask dtype')
        _req(out.dtype == torch.bfloat16 and out.is_contiguous() and out.numel() == B * NH * 128, 'out')
        m_sb = 0 if mask.shape[0] == 1 else mask.stride(0)
        return NKV, S, m_sb

    def attn_decode(self, query, kc, vc, mask, scaling, scores, cmax, part, counters, out, dbg=None):
        _req(dbg is None, 'attn_decode: the dbg probability tap is not provided by flashb')
        _bf16(query, 'query')
        _req(query.dim() == 4 and query.shape[2] == 1 and query.shape[3] == 128 and query.stride(3) == 1, 'query')
        B, NH = query.shape[0], query.shape[1]
        NKV, S, m_sb = self._common(kc, vc, mask, part, counters, out, B, NH)
        check(_native.lib().flashb_attn_decode(
            _p(query), query.stride(0), query.stride(1), _p(kc), _p(vc), kc.stride(0), kc.stride(1), B, NH, NKV, S,
            128, _p(mask), int(mask.dtype == torch.bfloat16), m_sb, float(scaling), None, 0, None, _p(out),
            _stream(query)))

    def attn_decode_fused(self, qkv, qn_w, kn_w, eps, cos, sin, kc, vc, mask, cache_pos, scaling, scores, cmax, part,
                          counters, out, dbg=None):
        _req(dbg is None, 'attn_decode_fused: the dbg probability tap is not provided by flashb')
        _bf16(qkv, 'qkv')
        _req(qkv.dim() == 2 and qkv.stride(1) == 1, 'qkv must be [B, (NH+2NKV)*D] with unit inner stride')
        B = qkv.shape[0]
        NKV = kc.shape[1]
        NH = qkv.shape[1] // 128 - 2 * NKV
        _req(NH >= NKV and qkv.shape[1] == (NH + 2 * NKV) * 128, 'qkv width')
        _req(qn_w.numel() == 128 and kn_w.numel() == 128 and qn_w.is_contiguous() and kn_w.is_contiguous(), 'norms')
        _req(cos.dtype == torch.bfloat16 and sin.dtype == torch.bfloat16 and cos.is_contiguous() and
             sin.is_contiguous() and cos.numel() == B * 128 and sin.numel() == B * 128, 'cos/sin must be [B,1,128]')
        _req(cache_pos.dtype == torch.int64 and cache_pos.is_cuda and cache_pos.numel() >= 1, 'cache_pos')
        NKV, S, m_sb = self._common(kc, vc, mask, part, counters, out, B, NH)
        check(_native.lib().flashb_attn_decode_fused(
            _p(qkv), qkv.stride(0), _p(qn_w), _p(kn_w), float(eps), _p(cos), _p(sin), 128, _p(kc), _p(vc),
            kc.stride(0), kc.stride(1), B, NH, NKV, S, 128, _p(mask), int(mask.dtype == torch.bfloat16), m_sb,
            _p(cache_pos), float(scaling), None, 0, None, _p(out), _stream(qkv)))


def attn_ws_floats(B, NH, NKV, S):
    """fp32 global workspace the decode attention needs (0: partials are merged in distributed shared memory)."""
    return int(_native.lib().flashb_attn_ws_floats(B, NH, NKV, S, 128))


class FusedOps:
    """flash_bb_fused: the skinny GEMVs (flash/csrc/bb_fused.cu:293-368).  ``R``, ``U`` and ``warps`` are the
    reference's per-GPU launch-shape knobs; they are accepted for call compatibility and ignored (the B200 kernels
    size their grid from the SM count and stream weights through a bulk-copy ring)."""

    @staticmethod
    def _x(x):
        _bf16(x, 'x')
        _req(x.dim() == 2 and x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.shape[1] % 8 == 0, 'x layout')
        return x.shape[0], x.shape[1]

    @staticmethod
    def _w(W, K):
        _bf16(W, 'W')
        _req(W.is_contiguous() and W.dim() == 2 and W.shape[1] == K, 'W must be contiguous [N, K]')

    def gemv_seg(self, x, nw, eps, W0, W1, W2, y, R=2, U=1, warps=8):
        M, K = self._x(x)
        self._w(W0, K)
        N0 = W0.shape[0]
        N1 = W1.shape[0] if W1 is not None and W1.numel() else 0
        N2 = W2.shape[0] if W2 is not None and W2.numel() else 0
        if N1:
            self._w(W1, K)
        if N2:
            self._w(W2, K)
        _req(y.dtype == torch.bfloat16 and y.shape[0] == M and y.shape[1] == N0 + N1 + N2 and y.stride(1) == 1, 'y')
        if nw is not None:
            _req(nw.dtype == torch.bfloat16 and nw.is_contiguous() and nw.numel() == K, 'nw')
        check(_native.lib().flashb_gemv_seg(_p(x), x.stride(0), M, K, _p(nw), float(eps), _p(W0), N0,
                                            _p(W1) if N1 else None, N1, _p(W2) if N2 else None, N2, _p(y),
                                            y.stride(0), _stream(x)))

    def gemv_resid(self, x, W, res, y, R=2, U=1, warps=8):
        M, K = self._x(x)
        self._w(W, K)
        N = W.shape[0]
        _req(res.dtype == torch.bfloat16 and res.shape[0] == M and res.shape[1] == N and res.stride(1) == 1, 'res')
        _req(y.dtype == torch.bfloat16 and y.shape[0] == M and y.shape[1] == N and y.stride(1) == 1, 'y')
        check(_native.lib().flashb_gemv_resid(_p(x), x.stride(0), M, K, _p(W), N, _p(res), res.stride(0), _p(y),
                                              y.stride(0), _stream(x)))

    def gemv_gateup(self, x, nw, eps, Wg, Wu, y, R=1, U=1, warps=8):
        M, K = self._x(x)
        self._w(Wg, K)
        self._w(Wu, K)
        _req(Wg.shape[0] == Wu.shape[0], 'Wg/Wu rows')
        N = Wg.shape[0]
        _req(y.dtype == torch.bfloat16 and y.shape[0] == M and y.shape[1] == N and y.stride(1) == 1, 'y')
        if nw is not None:
            _req(nw.dtype == torch.bfloat16 and nw.is_contiguous() and nw.numel() == K, 'nw')
        check(_native.lib().flashb_gemv_gateup(_p(x), x.stride(0), M, K, _p(nw), float(eps), _p(Wg), _p(Wu), N,
                                               _p(y), y.stride(0), _stream(x)))

    def rmsnorm(self, x, w, eps, y):
        M, K = self._x(x)
        _req(w.dtype == torch.bfloat16 and w.is_contiguous() and w.numel() == K, 'w')
        _req(y.dtype == torch.bfloat16 and y.shape[0] == M and y.shape[1] == K and y.stride(1) == 1 and
             y.stride(0) % 8 == 0, 'y')
        check(_native.lib().flashb_rmsnorm(_p(x), x.stride(0), M, K, _p(w), float(eps), _p(y), y.stride(0),
                                           _stream(x)))

    def embed_rope(self, ids, vocab, table, position_ids, cos_tab, sin_tab, x_out, cos_out, sin_out):
        """x_out[b] = bf16(sum_c table[ids[b, c] + c*vocab]); cos/sin rows of position_ids gathered from the tables."""
        _req(ids.dtype == torch.int64 and ids.is_contiguous(), 'ids must be contiguous int64 [B, C]')
        B, C = ids.shape[0], ids.shape[-1]
        _bf16(table, 'table')
        H = table.shape[1]
        D = cos_tab.shape[1]
        _req(position_ids.dtype == torch.int64 and position_ids.is_contiguous() and position_ids.numel() == B, 'pos')
        check(_native.lib().flashb_embed_rope(_p(ids), B, C, int(vocab), _p(table), H, _p(position_ids),
                                              _p(cos_tab), _p(sin_tab), D, cos_tab.shape[0], _p(x_out), _p(cos_out),
                                              _p(sin_out), _stream(ids)))

    def lm_head_cfg(self, x, norm_w, eps, W32, gs, hidden_out, logits, cfg_out):
        """hidden = RMSNorm(x); logits = float(hidden) @ W32^T; cfg = u + gs * (c - u)."""
        _bf16(x, 'x')
        B, H = x.shape[0], x.shape[-1]
        _req(W32.dtype == torch.float32 and W32.is_contiguous() and W32.shape[1] == H, 'W32')
        V = W32.shape[0]
        _req(logits.dtype == torch.float32 and logits.is_contiguous() and logits.numel() >= B * V, 'logits')
        check(_native.lib().flashb_lm_head_cfg(_p(x), B, H, _p(norm_w), float(eps), _p(W32), V, _p(gs),
                                               _p(hidden_out), _p(logits), _p(cfg_out), _stream(x)))

    def lm_head_rows(self, hidden, W32, logits):
        """logits [B, V] fp32 = W32 [V, H] . hidden[b] for normalised bf16 rows (any row stride, unit inner stride):
        the prefill's last-token logits (``UP/models/cudagraph/backbone_prefill_graph.py:111``)."""
        _bf16(hidden, 'hidden')
        B, H = hidden.shape
        _req(hidden.stride(1) == 1 and hidden.stride(0) % 8 == 0, 'hidden layout')
        _req(W32.dtype == torch.float32 and W32.is_contiguous() and W32.shape[1] == H, 'W32 [V, H] fp32')
        V = W32.shape[0]
        _req(logits.dtype == torch.float32 and logits.is_contiguous() and tuple(logits.shape) == (B, V), 'logits')
        check(_native.lib().flashb_lm_head_rows(_p(hidden), hidden.stride(0), B, H, _p(W32), V, _p(logits),
                                                _stream(hidden)))

    def prefill_qkv(self, qkv, B, L, NH, NKV, qn_w, kn_w, eps, cos_tab, sin_tab, position_ids, cache_position, kc,
                    vc):
        """The prefill's q|k|v tail in place (``flashb_prefill_qkv``): qkv [B L, (NH + 2 NKV) 128] bf16; q heads
        rewritten, k / v heads written to the caches kc / vc [B, NKV, S, 128] at cache_position."""
        _bf16(qkv, 'qkv')
        _req(qkv.dim() == 2 and qkv.shape[0] == B * L and qkv.shape[1] >= (NH + 2 * NKV) * 128 and qkv.stride(1) == 1,
             'qkv [B L, (NH + 2 NKV) 128]')
        for t, n in ((kc, 'kc'), (vc, 'vc')):
            _bf16(t, n)
            _req(t.dim() == 4 and t.shape[0] == B and t.shape[1] == NKV and t.shape[3] == 128 and t.stride(3) == 1
                 and t.stride(2) == 128, f'{n} [B, NKV, S, 128] with rows of 128')
        _req(kc.stride() == vc.stride() and kc.shape == vc.shape, 'kc / vc layouts differ')
        _req(position_ids.dtype == torch.int64 and position_ids.is_contiguous() and position_ids.numel() == B * L,
             'position_ids int64 [B, L]')
        _req(cache_position.dtype == torch.int64 and cache_position.is_contiguous() and cache_position.numel() == L,
             'cache_position int64 [L]')
        _req(cos_tab.shape == sin_tab.shape and cos_tab.shape[-1] == 128 and cos_tab.is_contiguous(), 'rope tables')
        check(_native.lib().flashb_prefill_qkv(_p(qkv), qkv.stride(0), B, L, NH, NKV, _p(qn_w), _p(kn_w), float(eps),
                                               _p(cos_tab), _p(sin_tab), cos_tab.shape[0], _p(position_ids),
                                               _p(cache_position), _p(kc), _p(vc), kc.stride(0), kc.stride(1),
                                               kc.shape[2], _stream(qkv)))

    def lm_head_cfg_blocks(self, x, norm_w, eps, W32, gs, block, hidden_out, logits, cfg_out):
        """lm_head_cfg for B rows in CFG blocks of ``block`` rows (each [cond..., uncond...]), one pass over the
        fp32 lm_head for every row; cfg_out rows: block b's pairs at [b * block / 2, (b + 1) * block / 2)."""
        _bf16(x, 'x')
        B, H = x.shape[0], x.shape[-1]
        _req(x.is_contiguous() and hidden_out.is_contiguous(), 'x / hidden_out contiguous')
        _req(W32.dtype == torch.float32 and W32.is_contiguous() and W32.shape[1] == H, 'W32')
        V = W32.shape[0]
        _req(logits.dtype == torch.float32 and logits.is_contiguous() and logits.numel() >= B * V, 'logits')
        check(_native.lib().flashb_lm_head_cfg_blocks(_p(x), B, H, _p(norm_w), float(eps), _p(W32), V, _p(gs),
                                                      int(block), _p(hidden_out), _p(logits), _p(cfg_out),
                                                      _stream(x)))


def load(name, verbose=False):
    """Load the library (built ahead of time by ``flashb.build``) and return the ops object for ``name``."""
    with _LOCK:
        if name in _MODS:
            return _MODS[name]
        _req(name in SPECS, f'unknown kernel module {name}')
        t = time.perf_counter()
        _native.lib()
        if name == 'flash_bb_attn':
            mod = AttnOps()
        elif name == 'flash_bb_fused':
            mod = FusedOps()
        else:
            from . import depth as _depth
            mod = _depth.DepthOps()
        _MODS[name] = mod
        _INFO[name] = dict(file=_native.lib_path(), seconds=round(time.perf_counter() - t, 3))
        return mod


def load_all(verbose=False):
    return {n: load(n, verbose) for n in SPECS}


def attn():
    return load('flash_bb_attn')


def fused():
    return load('flash_bb_fused')


def depth(variant):
    return load(f'flash_dd_{variant}')


def info():
    d = dict(_INFO)
    d['version'] = _native.lib().flashb_version().decode()
    return d
