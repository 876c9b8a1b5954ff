"""Synthetic-weight streams for the benchmark and the GPU tests.

There is no checkpoint in this environment, so the benchmark and the tests build models with the BASELINE
architecture and seeded random bf16 weights directly in HBM.  ``SyntheticBackboneGraph`` carries the attributes of
the official ``BackboneGraph`` that ``flashb.backbone.fused_decode_step`` reads (``input_ids_buf``,
``position_ids``, ``cache_position``, ``attn_mask``, ``static_cache.layers[i].keys/values``, ``hidden_buf``,
``logits_buf``, ``cfg_logits_buf``, ``guidance_scale``), so the same step function runs here and inside the
official runtime.  Weights of a layer live in one contiguous allocation (the reference packs its decode weights the
same way, ``flash/weight_pack.py:45-64``), q|k|v rows adjacent.
"""
from dataclasses import dataclass

import torch

from . import backbone as bb
from . import kernels
from ._native import check, lib


@dataclass
class BackboneConfig:
    hidden: int = 2048
    layers: int = 28
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 2049          # lm_head rows = per-codebook vocabulary of the backbone embedding
    codebooks: int = 16
    theta: float = 1e6
    eps: float = 1e-6

    def weight_bytes_per_layer(self):
        """bf16 bytes of the layer's seven matrices (96,468,992 at the BASELINE config; the four norm vectors,
        8.7 KB, are not counted)."""
        H, D = self.hidden, self.head_dim
        mats = (self.heads * D + 2 * self.kv_heads * D) * H + H * self.heads * D + 3 * self.ffn * H
        return 2 * mats


def _randn(shape, gen, device, std=1.0, mean=0.0):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(torch.bfloat16)


def rope_table(theta, head_dim, n, device):
    """cos/sin [n, D] bf16 for positions 0..n-1, computed as the default rotary embedding does (fp32, then bf16)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(n, dtype=torch.float32)
    f = pos[:, None] * inv[None, :]
    e = torch.cat((f, f), dim=-1)
    return e.cos().to(torch.bfloat16).to(device), e.sin().to(torch.bfloat16).to(device)


class _KV:
    __slots__ = ('keys', 'values')

    def __init__(self, k, v):
        self.keys, self.values = k, v


class _Cache:
    def __init__(self, layers):
        self.layers = layers


class SyntheticBackboneGraph:
    """A backbone decode graph with synthetic weights: B rows (B/2 CFG pairs), static KV cache of ``max_seq_len``."""

    def __init__(self, cfg: BackboneConfig, batch_size=2, max_seq_len=2048, device='cuda', seed=2, gs=4.0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.batch_size = B = batch_size
        self.half = B // 2 if B >= 2 else 1
        self.max_seq_len = S = max_seq_len
        self.num_codebooks = cfg.codebooks
        H, D, NH, NKV, F = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.ffn
        dev = self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        layers = []
        self._packs = []
        for _ in range(cfg.layers):
            L = bb.Layer()
            sizes = [(NH * D + 2 * NKV * D) * H, H * NH * D, F * H, F * H, H * F]
            pack = torch.empty(sum(sizes), dtype=torch.bfloat16, device=dev)
            self._packs.append(pack)
            o = 0
            views = []
            for s in sizes:
                views.append(pack[o:o + s])
                o += s
            qkv = views[0].view(NH * D + 2 * NKV * D, H)
            qkv.copy_(_randn(qkv.shape, g, dev, 0.02))
            L.wq, L.wk, L.wv = qkv[:NH * D], qkv[NH * D:NH * D + NKV * D], qkv[NH * D + NKV * D:]
            L.wo = views[1].view(H, NH * D)
            L.wo.copy_(_randn(L.wo.shape, g, dev, 0.02))
            L.wg = views[2].view(F, H)
            L.wg.copy_(_randn(L.wg.shape, g, dev, 0.02))
            L.wu = views[3].view(F, H)
            L.wu.copy_(_randn(L.wu.shape, g, dev, 0.02))
            L.wd = views[4].view(H, F)
            L.wd.copy_(_randn(L.wd.shape, g, dev, 0.02))
            L.ln1_w = _randn((H,), g, dev, 0.1, 1.0)
            L.ln2_w = _randn((H,), g, dev, 0.1, 1.0)
            L.qn_w = _randn((D,), g, dev, 0.1, 1.0)
            L.kn_w = _randn((D,), g, dev, 0.1, 1.0)
            L.ln1_eps = L.ln2_eps = L.qk_eps = cfg.eps
            L.scaling = D ** -0.5
            layers.append(L)
        self.norm_w = _randn((H,), g, dev, 0.1, 1.0)
        self.embed = _randn((cfg.codebooks * cfg.vocab, H), g, dev, 1.0)
        self.lm_head32 = _randn((cfg.vocab, H), g, dev, 0.02).float()
        cos_tab, sin_tab = rope_table(cfg.theta, D, S + 1, dev)
        self.static_cache = _Cache([_KV(torch.zeros(B, NKV, S, D, dtype=torch.bfloat16, device=dev),
                                        torch.zeros(B, NKV, S, D, dtype=torch.bfloat16, device=dev))
                                    for _ in range(cfg.layers)])
        self.input_ids_buf = torch.zeros(B, 1, cfg.codebooks, dtype=torch.long, device=dev)
        self.position_ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.cache_position = torch.zeros(1, dtype=torch.long, device=dev)
        self.attn_mask = torch.full((B, 1, 1, S), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16, device=dev)
        self.hidden_buf = torch.zeros(B, 1, H, dtype=torch.bfloat16, device=dev)
        self.logits_buf = torch.zeros(B, cfg.vocab, dtype=torch.float32, device=dev)
        self.cfg_logits_buf = torch.zeros(self.half, cfg.vocab, dtype=torch.float32, device=dev)
        self.guidance_scale = torch.tensor([gs], dtype=torch.float32, device=dev)
        self._bb_state = bb.make_state(B, layers, self.norm_w, cfg.eps, self.embed, cfg.vocab, self.lm_head32,
                                       cos_tab, sin_tab, S, dev)
        self._gen = g

    # ------------------------------------------------------------------------------------------ state helpers
    def fill_kv(self, valid_len, seed=7, std=1.0):
        """Random N(0, std) keys/values in slots [0, valid_len) of every layer; positions set so that the next
        step writes slot ``valid_len``."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for L in self.static_cache.layers:
            L.keys.zero_()
            L.values.zero_()
            L.keys[:, :, :valid_len].copy_(_randn(L.keys[:, :, :valid_len].shape, g, self.device, std))
            L.values[:, :, :valid_len].copy_(_randn(L.values[:, :, :valid_len].shape, g, self.device, std))
        self.set_position(valid_len)

    def set_position(self, pos, pad_lens=None):
        """Next step writes slot ``pos``; RoPE positions pos - pad_len; keys [pad_len, pos] valid."""
        B, S = self.batch_size, self.max_seq_len
        pad = torch.zeros(B, dtype=torch.long) if pad_lens is None else torch.as_tensor(pad_lens, dtype=torch.long)
        self.cache_position.fill_(pos)
        self.position_ids.copy_((pos - pad).view(B, 1).to(self.device))
        kv = torch.arange(S)
        valid = (kv[None, :] >= pad[:, None]) & (kv[None, :] <= pos)
        m = torch.full((B, S), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
        m[valid] = 0
        self.attn_mask.copy_(m.view(B, 1, 1, S).to(self.device))

    def advance(self):
        """On-device: next position (cache_position += 1, position_ids += 1, unmask the new slot)."""
        B, S = self.batch_size, self.max_seq_len
        check(lib().flashb_step_advance(self.cache_position.data_ptr(), self.position_ids.data_ptr(), B,
                                        self.attn_mask.data_ptr(), 1, self.attn_mask.stride(0), S,
                                        torch.cuda.current_stream(self.device).cuda_stream))

    def decode_step(self, advance=False):
        bb.fused_decode_step(self, advance=advance)

    def layer_weight_bytes(self):
        return self.cfg.weight_bytes_per_layer()


@dataclass
class DepthConfig:
    hidden: int = 1024
    embed_dim: int = 2048
    layers: int = 4
    heads: int = 8
    kv_heads: int = 2
    ffn: int = 4096
    vocab: int = 2048
    codebook_size: int = 2048
    n_decode: int = 16
    theta: float = 500000.0
    eps: float = 1e-5

    def step_weight_bytes(self):
        """bf16 bytes streamed per codebook step: the layers, the projector and one codebook head."""
        H, D = self.hidden, 128
        layer = (self.heads * D + 2 * self.kv_heads * D) * H + H * self.heads * D + 3 * self.ffn * H
        return 2 * (self.layers * layer + H * self.embed_dim + self.vocab * H)


class SyntheticDepth:
    """A depth decoder with synthetic bf16 weights (heads stored transposed [n_decode, vocab, hidden]) and the
    official graph's I/O buffers for ``batch`` rows."""

    def __init__(self, cfg: DepthConfig, batch=2, device='cuda', seed=3):
        from .depth import DepthModelDesc
        self.cfg = cfg
        self.device = dev = torch.device(device)
        self.batch = B = batch
        self.half = B // 2 if B >= 2 else 1
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, AE, D, NH, NKV, F = cfg.hidden, cfg.embed_dim, 128, cfg.heads, cfg.kv_heads, cfg.ffn
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                ln1=_randn((H,), g, dev, 0.1, 1.0), wq=_randn((NH * D, H), g, dev, 0.02),
                wk=_randn((NKV * D, H), g, dev, 0.02), wv=_randn((NKV * D, H), g, dev, 0.02),
                wo=_randn((H, NH * D), g, dev, 0.02), ln2=_randn((H,), g, dev, 0.1, 1.0),
                wg=_randn((F, H), g, dev, 0.02), wu=_randn((F, H), g, dev, 0.02), wd=_randn((H, F), g, dev, 0.02)))
        self.embed = _randn(((cfg.n_decode + 1) * cfg.vocab, AE), g, dev, 1.0)
        self.proj = _randn((H, AE), g, dev, 0.02)
        self.normf = _randn((H,), g, dev, 0.1, 1.0)
        self.head_t = _randn((cfg.n_decode, cfg.vocab, H), g, dev, 0.02)
        self.cos_tab, self.sin_tab = rope_table(cfg.theta, D, cfg.n_decode + 2, dev)
        self.desc = DepthModelDesc(self.layers, self.embed, self.proj, self.normf, self.head_t, self.cos_tab,
                                   self.sin_tab, cfg.eps, D ** -0.5, cfg.codebook_size, B, dev)
        hb = self.half
        self.backbone_hidden_buf = torch.zeros(B, AE, dtype=torch.bfloat16, device=dev)
        self.first_cb_token_buf = torch.zeros(B, dtype=torch.long, device=dev)
        self.output_tokens = torch.zeros(B, cfg.n_decode, dtype=torch.long, device=dev)
        self.tok_buf = torch.zeros(B, dtype=torch.long, device=dev)
        self.temperature = torch.full((hb,), 0.9, dtype=torch.float32, device=dev)
        self.top_k = torch.full((hb,), 50, dtype=torch.long, device=dev)
        self.top_p = torch.full((hb,), 1.0, dtype=torch.float32, device=dev)
        self.do_sample = torch.ones(hb, dtype=torch.long, device=dev)
        self.guidance_scale = torch.full((hb,), 4.0, dtype=torch.float32, device=dev)
        self.q = torch.ones(cfg.n_decode, hb, cfg.vocab, dtype=torch.float32, device=dev)

    def frame(self, dbg=None, forced=None):
        self.desc.frame(self.first_cb_token_buf, self.backbone_hidden_buf, self.tok_buf, self.output_tokens,
                        self.temperature, self.top_k, self.top_p, self.do_sample, self.guidance_scale, self.q, dbg,
                        forced)


def backbone_step_bytes(cfg: BackboneConfig, batch, kv_len, include_lm_head=True):
    """Algorithmic HBM bytes of one decode step: every weight once, the valid KV once, the fp32 lm_head once."""
    w = cfg.layers * cfg.weight_bytes_per_layer()
    kv = cfg.layers * batch * cfg.kv_heads * kv_len * cfg.head_dim * 2 * 2
    lm = cfg.vocab * cfg.hidden * 4 if include_lm_head else 0
    return w + kv + lm


def launches_per_backbone_step(cfg: BackboneConfig):
    return 2 + 5 * cfg.layers


__all__ = ['BackboneConfig', 'SyntheticBackboneGraph', 'DepthConfig', 'SyntheticDepth', 'backbone_step_bytes',
           'rope_table', 'kernels']
