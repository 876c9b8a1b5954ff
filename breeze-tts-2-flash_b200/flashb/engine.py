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

    def __init__(self, cfg: BackboneConfig, batch_size=2, max_seq_len=2048, device='cuda', seed=2, gs=4.0,
                 weights_from=None):
        """``weights_from``: another SyntheticBackboneGraph whose weights this one shares (a second stream of the same
        replica: own KV cache and buffers, same weights)."""
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
        if weights_from is not None:
            src = weights_from
            if src.cfg != cfg or src.max_seq_len < S:
                raise ValueError('weights_from: different config or shorter rotary table')
            layers = src._bb_state['layers']
            self._packs, self.norm_w, self.embed, self.lm_head32 = src._packs, src.norm_w, src.embed, src.lm_head32
            cos_tab, sin_tab = src._bb_state['cos_tab'], src._bb_state['sin_tab']
        else:
            layers = self._make_weights(cfg, g, dev)
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

    def _make_weights(self, cfg, g, dev):
        H, D, NH, NKV, F = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.ffn
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
        return layers

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

    def frame_weight_bytes(self, step_table=False, rows=2, ln12=False):
        """Algorithmic bytes of one frame: n_decode codebook steps of weights; with the step table, steps >= 1 read
        ``rows`` table rows (hidden + layer-0 q|k|v, bf16) instead of the projector and layer 0's q|k|v matrices.
        ln12: the streamed matrices as LN12 (1.5 bytes a weight + a 16-byte record per row; overflow patches, a few
        per matrix, left out)."""
        H, D, AE, V, F = self.hidden, 128, self.embed_dim, self.vocab, self.ffn
        qkv = (self.heads + 2 * self.kv_heads) * D

        def mat(n, k):
            return n * k * 1.5 + n * 16 if ln12 else n * k * 2

        layer = mat(qkv, H) + mat(H, self.heads * D) + 2 * mat(F, H) + mat(H, F)
        step = self.layers * layer + mat(H, AE) + mat(V, H)
        full = self.n_decode * step
        if not step_table:
            return int(full)
        saved = mat(H, AE) + mat(qkv, H) - 2 * rows * (H + qkv)
        return int(full - (self.n_decode - 1) * saved)


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

    def mats(self):
        """The streamed matrices in the LN12 descriptor order: per layer q, k, v, o, gate, up, down; the projector;
        the codebook heads."""
        out = []
        for L in self.layers:
            out += [L['wq'], L['wk'], L['wv'], L['wo'], L['wg'], L['wu'], L['wd']]
        return out + [self.proj] + [self.head_t[s] for s in range(self.head_t.shape[0])]

    def ln12(self):
        """The matrices encoded in LN12 (``flashb.ln12.encode`` on the host, once) as device tensors for
        ``flashb.depth.ln12_set``."""
        if getattr(self, '_ln12', None) is None:
            from . import ln12 as L12
            enc = []
            for w in self.mats():
                d, m, o, lut = L12.encode(w)
                enc.append(L12.to_device(d, m, o, lut, self.device))
            self._ln12 = enc
        return self._ln12

    def use_ln12(self, on=True):
        from . import depth as fdep
        fdep.ln12_set(self.desc, self.ln12() if on else None)


class _Slot:
    """``g`` streams decoded together: one backbone graph and one depth launch over 2 g rows laid out
    [cond_0 .. cond_{g-1}, uncond_0 .. uncond_{g-1}] (the CFG pair of stream k is rows k and k + g), which is the row
    order every kernel on the path already uses for B = 2 g."""
    __slots__ = ('g', 'bb', 'bh', 'first_cb', 'outtok', 'tokbuf', 'q', 'graph', 'desc', 'lane', 'r0', 'c0')


class sm_budget:
    """Context manager: launches issued by this host thread inside it (directly or into a CUDA graph being captured)
    size their grids for at most ``sms`` SMs (``flashb_set_sm_budget``); 0 = every SM."""

    def __init__(self, sms):
        self.sms = int(sms)

    def __enter__(self):
        lib().flashb_set_sm_budget(self.sms)
        return self

    def __exit__(self, *exc):
        lib().flashb_set_sm_budget(0)
        return False


class FrameEngine:
    """One replica on one GPU for the streaming decode: a synthetic backbone and depth decoder whose weights are
    shared by ``n_streams`` independent streams (own KV cache, positions and I/O buffers each).

    Streams are served in slots of ``group`` streams (1, 2, 4 or 8): a slot's streams share every weight read of the
    backbone step (GEMV rows M = 2 g) and of the depth frame (B = 2 g), and advance in lockstep (same cache
    position; the bench's streams all start after the same prompt length).  ``frame(i)`` runs one frame of every
    stream of slot i on the current CUDA stream, the body of the reference's streaming loop
    (``flash/main_loop.py:252-312``) without host synchronisation:

        frame_ids    next backbone input = [cb0, depth tokens] of the previous frame            (1 launch)
        backbone     step on those ids, position advanced on the device                         (2 + 1 + 5 x layers)
        cb0          codebook-0 token from the CFG logits: the backbone sampler (cb0='sample': the reference
                     runtime's repetition penalty 1.1 over the stream's earlier codebook-0 tokens, reserved ids
                     suppressed, T 0.9, top-k 50, top-p 1.0, multinomial on fresh Exp(1) draws, validity flag)
                     or its greedy branch (cb0='greedy')                                          (1 launch)
        depth frame  every depth codebook, CFG top-k sampled on the device (with draw_q, its Exp(1) draws made
                     fresh on the device before the launch, as the reference's _full_loop does) (1 launch)

    The first three are captured into one CUDA graph per slot (``capture()``); the depth frame is a single launch.
    Each stream starts after a ``prompt_len``-token prompt whose KV cache is random (the prefill stand-in).
    ``single_slot`` adds one extra single-stream slot on the same weights (``self.single``), for frame latency.

    ``lanes`` > 1 splits the GPU: slot i belongs to lane i % lanes, every lane has its own CUDA stream, depth scratch
    and an SM budget of num_sms // lanes (grids of its persistent kernels, split counts of its attention), and
    ``step()`` runs the lanes side by side.  Every kernel here is latency-bound at decode sizes, so two half-GPU
    lanes finish two slots sooner than one whole-GPU lane finishes them one after the other.

    ``shared_backbone``: one backbone graph for the rows of every slot (slot i = rows [2 g i, 2 g (i + 1)), each
    laid out [cond, uncond] with its own CFG block), captured on the whole GPU: its GEMVs run as row groups of 64 rows
    side by side in one launch each, which read every weight tile at about the same time (L2 serves all but the
    first read), and its attention covers every row in one launch.  The depth launches stay per slot, on the
    lanes.  ``step()`` then replays the one backbone graph and forks the lanes for the depth frames."""

    # the reference runtime's backbone sampling parameters (UP/breeze_infer/runtime.py, api.py REPETITION_PENALTY)
    CB0_PARAMS = dict(temperature=0.9, top_k=50, top_p=1.0, do_sample=1, repetition_penalty=1.1)

    def __init__(self, bcfg: BackboneConfig, dcfg: DepthConfig, n_streams, prompt_len, max_frames, device='cuda',
                 seed=0, depth_only=False, group=1, single_slot=False, lanes=1, shared_backbone=False, cb0='sample'):
        """``depth_only``: no backbone (a random hidden state per stream feeds the depth frame) -- for timing or
        profiling the depth frame alone on a small device footprint."""
        if bcfg.codebooks - 1 > dcfg.n_decode or dcfg.embed_dim != bcfg.hidden:
            raise ValueError('backbone codebooks must be <= 1 + depth codebooks and depth embed_dim == backbone hidden')
        if group not in (1, 2, 4, 8) or n_streams % group:
            raise ValueError('group must be 1, 2, 4 or 8 and divide the number of streams')
        if lanes < 1:
            raise ValueError('lanes must be at least 1 (more lanes than slots leave some lanes idle)')
        self.bcfg, self.dcfg, self.group = bcfg, dcfg, group
        self.device = dev = torch.device(device)
        self.lanes = lanes
        nsm = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == 'cuda' else 0
        self.lane_sms = 0 if lanes == 1 else nsm // lanes
        self.prompt_len = prompt_len
        # a multiple of 8 positions: the mask rows (bf16, one per position) start 16-byte aligned
        self.max_seq_len = (prompt_len + max_frames + 2 + 7) // 8 * 8
        self.n_valid = min(dcfg.codebook_size, bcfg.vocab)
        self.depth_only = depth_only
        self.depth = SyntheticDepth(dcfg, batch=2 * group, device=dev, seed=seed + 3)
        self.lane_desc = [self.depth.desc]
        self.lane_stream = [None]
        if lanes > 1:
            from .depth import DepthModelDesc
            d = self.depth
            self.lane_desc = [DepthModelDesc(d.layers, d.embed, d.proj, d.normf, d.head_t, d.cos_tab, d.sin_tab,
                                             dcfg.eps, 128 ** -0.5, dcfg.codebook_size, 2 * group, dev)
                              for _ in range(lanes)]
            for ld in self.lane_desc:
                ld.cfg.grid = self.lane_sms
            self.lane_stream = [torch.cuda.Stream(dev) for _ in range(lanes)]
        self._gen = torch.Generator(device='cpu').manual_seed(seed + 17)
        self._first_bb = None
        self._seed = seed
        self.shared = bool(shared_backbone) and not depth_only
        self.bb = None
        self.bb_graph = None
        n_slots = n_streams // group
        if cb0 not in ('sample', 'greedy'):
            raise ValueError("cb0 must be 'sample' or 'greedy'")
        self.cb0 = cb0
        self.draw_q = True          # depth Exp(1) draws made on the device before each depth launch
        # the engine's own generator for every Exp(1) draw it makes (reproducible whatever else draws)
        self.rng = torch.Generator(device=dev)
        self.rng.manual_seed(seed + 29)
        V = bcfg.vocab
        # per stream (rows in slot order; the single-stream slot last): token history, Exp(1) draws, validity flag
        ns = n_streams + (1 if single_slot else 0)
        p = self.CB0_PARAMS
        self.cb0_present = torch.zeros(ns, V, dtype=torch.uint8, device=dev)
        self.cb0_q = torch.ones(ns, V, dtype=torch.float32, device=dev)
        self.cb0_ok = torch.ones(ns, dtype=torch.int64, device=dev)
        self.cb0_temp = torch.full((ns,), p['temperature'], dtype=torch.float32, device=dev)
        self.cb0_topk = torch.full((ns,), p['top_k'], dtype=torch.int64, device=dev)
        self.cb0_topp = torch.full((ns,), p['top_p'], dtype=torch.float32, device=dev)
        self.cb0_ds = torch.full((ns,), p['do_sample'], dtype=torch.int64, device=dev)
        self.cb0_suppress = torch.arange(self.n_valid, V, dtype=torch.int64, device=dev)
        if self.shared:
            R = 2 * group * n_slots
            if R > 128:
                raise ValueError('shared_backbone: at most 128 backbone rows (64 streams) per graph')
            self.bb = SyntheticBackboneGraph(bcfg, R, self.max_seq_len, dev, seed=seed + 2)
            self.bb.cfg_block = 2 * group
            self._first_bb = self.bb
            self.bb.fill_kv(prompt_len, seed=1000 + seed)
            self.bb.set_position(prompt_len - 1)
            gen = self._gen
            self.first_cb = torch.cat([torch.randint(0, self.n_valid, (group,), generator=gen).repeat(2)
                                       for _ in range(n_slots)]).to(dev)
            self.outtok = torch.cat([torch.randint(0, dcfg.codebook_size, (group, dcfg.n_decode),
                                                   generator=gen).repeat(2, 1) for _ in range(n_slots)]).to(dev)
        self.streams = [self._slot(group, 1000 + seed + i, row0=2 * group * i if self.shared else None)
                        for i in range(n_slots)]
        for i, st in enumerate(self.streams):
            st.lane = i % lanes
            st.desc = self.lane_desc[st.lane]
            st.c0 = i * group                  # its streams' rows of the codebook-0 sampler state
        self.single = None
        if single_slot:
            from .depth import DepthModelDesc
            d = self.depth
            self.single = self._slot(1, 999 + seed)
            self.single.lane = None
            self.single.c0 = n_streams
            self.single.desc = d.desc if group == 1 else DepthModelDesc(
                d.layers, d.embed, d.proj, d.normf, d.head_t, d.cos_tab, d.sin_tab, dcfg.eps, 128 ** -0.5,
                dcfg.codebook_size, 2, dev)
        self.step_table = None
        self.ln12 = False

    def use_ln12(self, on=True):
        """Frames of every slot stream the depth weights in LN12 (12-bit, lossless; decoded in shared memory by the
        tcgen05 build) instead of bf16."""
        from . import depth as fdep
        mats = self.depth.ln12() if on else None
        descs = {id(x): x for x in [self.depth.desc] + list(self.lane_desc) +
                 ([self.single.desc] if self.single is not None else [])}
        for dd in descs.values():
            fdep.ln12_set(dd, mats)
        self.ln12 = on

    def use_step_table(self, on=True):
        """Frames of every slot read the per-token step table (built once from the shared depth weights,
        ``flashb.depth.tab_build``) for stage E and layer 0's q|k|v of codebook steps >= 1; off: computed."""
        from . import depth as fdep
        if on and self.step_table is None:
            self.step_table = fdep.tab_build(self.depth.desc)
        descs = {id(x): x for x in [self.depth.desc] + list(self.lane_desc) +
                 ([self.single.desc] if self.single is not None else [])}
        for dd in descs.values():
            fdep.tab_set(dd, *(self.step_table if on else (None, None)))

    def _slot(self, g, kv_seed, row0=None):
        """A slot of g streams; row0: its first row in the shared backbone graph (None: a backbone of its own)."""
        dcfg, dev, gen = self.dcfg, self.device, self._gen
        st = _Slot()
        st.g = g
        st.r0 = row0
        if row0 is not None:
            st.bb = self.bb
            st.bh = self.bb.hidden_buf.view(self.bb.batch_size, -1)[row0:row0 + 2 * g]
            st.first_cb = self.first_cb[row0:row0 + 2 * g]
            st.outtok = self.outtok[row0:row0 + 2 * g]
            st.tokbuf = torch.zeros(2 * g, dtype=torch.long, device=dev)
            st.q = torch.empty(dcfg.n_decode, g, dcfg.vocab).exponential_(1, generator=gen).to(dev)
            st.graph = None
            st.desc = self.depth.desc
            st.lane = 0
            return st
        if self.depth_only:
            st.bb = None
            st.bh = torch.randn(2 * g, dcfg.embed_dim, generator=gen).to(torch.bfloat16).to(dev)
        else:
            st.bb = SyntheticBackboneGraph(self.bcfg, 2 * g, self.max_seq_len, dev, seed=self._seed + 2,
                                           weights_from=self._first_bb)
            self._first_bb = self._first_bb or st.bb
            st.bb.fill_kv(self.prompt_len, seed=kv_seed)
            st.bb.set_position(self.prompt_len - 1)
            st.bh = st.bb.hidden_buf.view(2 * g, -1)
        st.first_cb = torch.randint(0, self.n_valid, (g,), generator=gen).repeat(2).to(dev)
        st.outtok = torch.randint(0, dcfg.codebook_size, (g, dcfg.n_decode), generator=gen).repeat(2, 1).to(dev)
        st.tokbuf = torch.zeros(2 * g, dtype=torch.long, device=dev)
        st.q = torch.empty(dcfg.n_decode, g, dcfg.vocab).exponential_(1, generator=gen).to(dev)
        st.graph = None
        st.desc = self.depth.desc
        st.lane = 0
        return st

    def _get(self, i):
        return self.single if i == 'single' else self.streams[i]

    def _cb0(self, cfg_logits, c0, rows, g, first_cb, stream):
        """Codebook 0 of `rows` streams (sampler state rows [c0, c0 + rows)) from their CFG logits rows, into the
        CFG-pair ids first_cb (blocks of 2 g rows)."""
        if self.cb0 == 'greedy':
            for b in range(rows // g):
                check(lib().flashb_cb0_greedy(cfg_logits[b * g:].data_ptr(), cfg_logits.stride(0), g, self.n_valid,
                                              2 * g, first_cb[2 * g * b:].data_ptr(), stream))
            return
        V = self.bcfg.vocab
        q = self.cb0_q[c0:c0 + rows]           # this frame's Exp(1) draws (draw_cb0, before the graph replays)
        r = slice(c0, c0 + rows)
        check(lib().flashb_cb0_sample(
            cfg_logits.data_ptr(), cfg_logits.stride(0), rows, V, self.cb0_present[r].data_ptr(), V,
            float(self.CB0_PARAMS['repetition_penalty']), self.cb0_suppress.data_ptr(), self.cb0_suppress.numel(),
            self.cb0_temp[r].data_ptr(), self.cb0_topk[r].data_ptr(), self.cb0_topp[r].data_ptr(),
            self.cb0_ds[r].data_ptr(), q.data_ptr(), V, first_cb.data_ptr(), g, self.cb0_ok[r].data_ptr(), 1,
            stream))

    def draw_cb0(self, c0, rows):
        """Fresh Exp(1) draws of the codebook-0 multinomial of sampler rows [c0, c0 + rows), on the current stream
        (eager, outside the captured graphs, from the engine's generator)."""
        if self.cb0 == 'sample':
            self.cb0_q[c0:c0 + rows].exponential_(1.0, generator=self.rng)

    def shared_backbone_part(self):
        """The shared backbone graph's body: frame ids of every row, one backbone step, codebook 0 of every
        stream."""
        bb, g = self.bb, self.group
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().flashb_frame_ids(self.first_cb.data_ptr(), self.outtok.data_ptr(), self.dcfg.n_decode,
                                     bb.batch_size, self.bcfg.codebooks, bb.input_ids_buf.data_ptr(), stream))
        bb.decode_step(advance=True)
        self._cb0(bb.cfg_logits_buf, 0, len(self.streams) * g, g, self.first_cb, stream)

    # one frame, split into its backbone part (graph-capturable) and the depth launch
    def backbone_part(self, i):
        st = self._get(i)
        if st.r0 is not None:
            raise ValueError('slots of a shared backbone have no backbone part of their own (shared_backbone_part)')
        g = st.g
        stream = torch.cuda.current_stream(self.device).cuda_stream
        C = self.bcfg.codebooks
        check(lib().flashb_frame_ids(st.first_cb.data_ptr(), st.outtok.data_ptr(), self.dcfg.n_decode, 2 * g, C,
                                     st.bb.input_ids_buf.data_ptr(), stream))
        st.bb.decode_step(advance=True)
        self._cb0(st.bb.cfg_logits_buf, st.c0, g, g, st.first_cb, stream)

    def depth_part(self, i):
        st, d = self._get(i), self.depth
        g = st.g
        if self.draw_q:
            # the frame's Exp(1) draws (the reference: one exponential_ per codebook)
            st.q.exponential_(1.0, generator=self.rng)
        st.desc.frame(st.first_cb, st.bh, st.tokbuf, st.outtok, d.temperature[:g], d.top_k[:g], d.top_p[:g],
                      d.do_sample[:g], d.guidance_scale[:g], st.q)

    def _slots(self):
        return list(enumerate(self.streams)) + ([('single', self.single)] if self.single is not None else [])

    def capture(self):
        """One CUDA graph per slot for its backbone part.  Every slot first runs one eager frame (kernel attributes
        are set on first use, per batch size), then its position is put back.  Nothing to capture without a
        backbone."""
        if self.depth_only:
            for i, _ in self._slots():
                self.depth_part(i)
            torch.cuda.synchronize(self.device)
            return
        if self.shared:
            self.shared_backbone_part()
            for i in range(len(self.streams)):
                with sm_budget(self.lane_sms):
                    self.depth_part(i)
            torch.cuda.synchronize(self.device)
            self.bb.set_position(self.prompt_len - 1)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    self.shared_backbone_part()
                self.bb_graph = graph
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
        for i, st in ([] if self.shared else self._slots()[:1]) + (
                [self._slots()[-1]] if self.single is not None else []):
            with sm_budget(self._budget(st)):
                self.backbone_part(i)
                self.depth_part(i)
            torch.cuda.synchronize(self.device)
            st.bb.set_position(self.prompt_len - 1)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for i, st in self._slots():
                if st.r0 is not None:
                    continue
                graph = torch.cuda.CUDAGraph()
                with sm_budget(self._budget(st)), torch.cuda.graph(graph, stream=side):
                    self.backbone_part(i)
                st.graph = graph
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)

    def _budget(self, st):
        return 0 if st.lane is None else self.lane_sms

    def step(self, before_part=None, after_part=None, fork=True, join=True):
        """One frame of every slot (not the single-stream slot), lanes side by side.  fork: the lanes first wait for
        the work already on the current stream; join: the current stream waits for every lane at the end.  Steps in
        a row need the fork only on the first and the join only on the last, so that a lane never waits for the
        others between steps.  ``before_part(kind, i, stream)``, if given, is called before each part ('bb' or
        'dd') of slot i with the CUDA stream it is issued on, and with ('end', None, stream) once per lane stream
        after its last part; ``after_part('dd', i, stream)`` after the depth part of slot i."""
        cur = torch.cuda.current_stream(self.device)
        if self.shared:
            # the backbone of every slot (one graph on the whole GPU), then the depth frames on the lanes
            if before_part is not None:
                before_part('bb', -1, cur)
            self.draw_cb0(0, len(self.streams) * self.group)
            if self.bb_graph is not None:
                self.bb_graph.replay()
            else:
                self.shared_backbone_part()
            if before_part is not None:
                before_part('bbend', -1, cur)
            lanes = self.lane_stream if self.lanes > 1 else [cur]
            if self.lanes > 1 and fork:
                for ls in lanes:
                    ls.wait_stream(cur)
            for i, st in enumerate(self.streams):
                s = lanes[st.lane]
                with torch.cuda.stream(s):
                    if before_part is not None:
                        before_part('dd', i, s)
                    self.depth_part(i)
                    if after_part is not None:
                        after_part('dd', i, s)
            for ls in lanes:
                if before_part is not None:
                    before_part('end', None, ls)
                if self.lanes > 1 and join:
                    cur.wait_stream(ls)
            return
        if self.lanes == 1:
            for i in range(len(self.streams)):
                self.frame(i, before_part, after_part)
            if before_part is not None:
                before_part('end', None, cur)
            return
        if fork:
            for ls in self.lane_stream:
                ls.wait_stream(cur)
        for i, st in enumerate(self.streams):
            with torch.cuda.stream(self.lane_stream[st.lane]):
                self.frame(i, before_part, after_part)
        for ls in self.lane_stream:
            if before_part is not None:
                before_part('end', None, ls)
            if join:
                cur.wait_stream(ls)

    def frame(self, i, before_part=None, after_part=None):
        st = self._get(i)
        if st.r0 is not None:
            raise ValueError('slots of a shared backbone run their frames through step()')
        stream = torch.cuda.current_stream(self.device)
        if before_part is not None and st.bb is not None:
            before_part('bb', i, stream)
        if st.bb is None:
            pass
        elif st.graph is not None:
            self.draw_cb0(st.c0, st.g)
            st.graph.replay()
        else:
            self.draw_cb0(st.c0, st.g)
            self.backbone_part(i)
        if before_part is not None:
            before_part('dd', i, stream)
        self.depth_part(i)
        if after_part is not None:
            after_part('dd', i, stream)

    def launches_per_frame(self):
        """flashb kernel launches per slot frame (the Exp(1) draws are torch's own kernels and not counted).  A
        backbone graph: frame ids, position advance, embedding, 5 per layer (7 when the rows exceed
        backbone.ROWS_NORM_APART: the two RMSNorms run apart), the LM head (one launch for one CFG block, else a final
        norm and one pass for every block) and codebook 0 (one sampler launch, or a greedy pick per slot); with a
        shared backbone its launches are shared out over the slots.  Plus one depth launch."""
        from . import backbone as bb
        L = self.bcfg.layers
        if self.shared:
            n = len(self.streams)
            cb0 = 1 if self.cb0 == 'sample' else n
            lm = 1 if n == 1 and 2 * self.group <= 16 else 2
            per_layer = 7 if 2 * self.group * n > bb.ROWS_NORM_APART else 5
            return (3 + per_layer * L + lm + cb0) / n + 1
        return 3 + 5 * L + 1 + 1 + 1

    def frame_bytes(self):
        """Algorithmic HBM bytes of one slot frame at the current KV length: backbone step + 16 depth steps."""
        if self.depth_only:
            return self.dcfg.frame_weight_bytes(self.step_table is not None, 2 * self.group, self.ln12)
        kv = int(self.streams[0].bb.cache_position.item()) + 1
        if self.shared:
            n = len(self.streams)
            return backbone_step_bytes(self.bcfg, 2 * self.group * n, kv) / n + \
                self.dcfg.frame_weight_bytes(self.step_table is not None, 2 * self.group, self.ln12)
        return backbone_step_bytes(self.bcfg, 2 * self.group, kv) + \
            self.dcfg.frame_weight_bytes(self.step_table is not None, 2 * self.group, self.ln12)


def backbone_step_bytes(cfg: BackboneConfig, batch, kv_len, include_lm_head=True):
    """Algorithmic HBM bytes of one decode step: every weight once, the valid KV once, the fp32 lm_head once."""
    w = cfg.layers * cfg.weight_bytes_per_layer()
    kv = cfg.layers * batch * cfg.kv_heads * kv_len * cfg.head_dim * 2 * 2
    lm = cfg.vocab * cfg.hidden * 4 if include_lm_head else 0
    return w + kv + lm


def launches_per_backbone_step(cfg: BackboneConfig):
    return 2 + 5 * cfg.layers


__all__ = ['BackboneConfig', 'SyntheticBackboneGraph', 'DepthConfig', 'SyntheticDepth', 'FrameEngine',
           'backbone_step_bytes', 'rope_table', 'kernels']
