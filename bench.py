#!/usr/bin/env python
"""Streaming-decode throughput of the flashb hot path on 1..8 B200s (one replica per GPU, no collective).

Workload (BASELINE config 5 with configs 3 and 4): 64 independent streams per GPU (64 N for the job: weak scaling,
streams assigned round-robin, one replica per GPU), each after a 512-token prompt (random KV, the prefill stand-in).
One backbone graph decodes every stream's rows on the whole GPU (--backbone shared: 128 rows, GEMVs in row groups
of 64); the depth frames run 8 streams per launch (--group) on 8 lanes side by side (--lanes), each lane on its own
CUDA stream with its kernels sized for 1/8 of the SMs.  A STEP is one frame of every stream on this rank:

    frame = next backbone ids from the previous frame -> 28-layer backbone decode step (B = 2 CFG rows, KV length
            512 + t, hidden 2048, 16 q / 4 kv heads, FFN 6144, fp32 lm_head + CFG) -> codebook-0 token (the
            reference runtime's backbone sampler on the device: repetition penalty 1.1, T 0.9, top-k 50) -> depth
            frame (4 layers, hidden 1024, 16 codebooks of 2048, CFG scale 4, top-k 50, T 0.9, sampled on the device)

Every frame's random draws are fresh: the Exp(1) draws of both multinomials are made on the device each step.
Outputs one JSON line (rank 0): ``value`` = frames/s of the whole job with every input resident in HBM (max over
ranks of the device time), ``e2e`` = the same through the engine API with the depth frame's Exp(1) draws copied
from pinned host memory before each frame and the frame's tokens and codebook-0 validity flags read back to the host
after it, every step (as the reference's loop reads its token and flag), ``roofline`` for the dominant kernel (the depth frame kernel) and
``roofline_backbone`` for the backbone step's attention + GEMV kernels, ``cpu_baseline`` = the CPU oracle port of
the same frame on this host's cores.

``--impl reference`` times that CPU port alone (rank 0; other ranks exit 0), one frame per step.
``--case depth`` / ``--case backbone`` time one part alone (profiling entry points; same JSON shape, no baselines).
"""
import argparse
import json
import os
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(HERE, 'breeze-tts-2-flash_b200')]

N_STREAMS = 64
PROMPT = 512
PEAKS_FALLBACK = dict(hbm_gbs=6650.0, bf16_tflops=1590.0)
# dram__bytes_read.sum + dram__bytes_write.sum of one dd_frame_kernel launch at the bench's default shape (8 streams
# per launch, B = 16 rows, one lane's grid of 18 CTAs: the tcgen05 build), from ncu --set full captures of the
# full-size depth model, keyed by (step table, LN12 weights): with the table 2,041,333,000 B read + 8,110,592 B
# written (bf16) and 1,042,911,000 + 8,060,672 (LN12); without it 2,174,940,416 + 7,735,296 (bf16).
DD_TRAFFIC_BYTES = {(1, 0): 2049443592, (1, 1): 1050971672, (0, 0): 2182675712}
PREFILL_CFG = dict(B=2, NH=16, NKV=4, L=512, D=128, pads=(0, 37))


def args_():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=30)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='flashb', choices=['flashb', 'reference'])
    p.add_argument('--streams', type=int, default=N_STREAMS,
                   help='streams per GPU (the job serves streams x N: weak scaling, one replica per GPU)')
    p.add_argument('--prompt', type=int, default=PROMPT)
    p.add_argument('--case', default='frame', choices=['frame', 'depth', 'backbone', 'prefill', 'config1', 'config2',
                                                      'config3', 'config5'])
    p.add_argument('--group', type=int, default=8, choices=[1, 2, 4, 8],
                   help='streams decoded together per launch (their GEMV rows share every weight read)')
    p.add_argument('--lanes', type=int, default=8,
                   help='GPU lanes: slots run on this many CUDA streams side by side, each sized for 1/lanes of the '
                        'SMs')
    p.add_argument('--backbone', default='shared', choices=['shared', 'lanes'],
                   help='shared: one backbone graph for every slot on the whole GPU (row groups of 64 per GEMV '
                        'launch); lanes: a backbone graph per slot on its lane')
    p.add_argument('--cpu-seconds', type=float, default=10.0, help='CPU baseline sample length')
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--no-per-config', action='store_true', help='skip the per-config kernel figures (configs 1-3)')
    p.add_argument('--step-table', type=int, default=1, choices=[0, 1],
                   help='depth frames read the per-token step table for stage E and layer 0 q|k|v of steps >= 1')
    p.add_argument('--ln12', type=int, default=0, choices=[0, 1],
                   help='depth frames stream their weights in LN12 (12-bit lossless, decoded in shared memory)')
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(HERE, 'MEASURED_PEAKS.json')) as f:
            d = json.load(f)
        return dict(hbm_gbs=float(d['hbm_gbs']), bf16_tflops=float(d['bf16_tflops']), source='measured')
    except Exception:
        return dict(PEAKS_FALLBACK, source='fallback')


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampled every 100 ms while the timed region runs: started ahead (it takes a few hundred ms to print
    its first sample), and only the samples after mark() -- the start of the timed region -- are kept."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_ids):
        self.proc, self.path = None, None
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix='.csv')
            os.close(fd)
            self.out = open(self.path, 'w')
            self.proc = subprocess.Popen(['nvidia-smi', '-i', ','.join(str(i) for i in gpu_ids),
                                          f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '100'], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        self.skip = 0

    def _lines(self):
        try:
            with open(self.path) as f:
                return sum(1 for _ in f)
        except Exception:
            return 0

    def wait_started(self, timeout=3.0):
        """Returns once nvidia-smi has printed a sample (or after `timeout` seconds)."""
        t0 = time.time()
        while self.proc is not None and self._lines() == 0 and time.time() - t0 < timeout:
            time.sleep(0.02)

    def mark(self):
        """The timed region starts now: earlier samples are dropped."""
        if self.proc is not None:
            self.out.flush()
            self.skip = self._lines()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(',')]
                if len(c) >= 9:
                    rows.append(c)
        os.unlink(self.path)
        if not rows:
            return None
        rows = rows[self.skip:] or rows[-1:]   # samples from the timed region (else the last one)
        sm = sorted(float(r[1]) for r in rows if r[1].replace('.', '').isdigit())
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == 'active'})
        return dict(sm_mhz=sm[len(sm) // 2] if sm else None,
                    sm_max_mhz=float(rows[0][2]) if rows[0][2].replace('.', '').isdigit() else None,
                    reasons=reasons, samples=len(rows))


# ------------------------------------------------------------------------------------------------ CPU port
# Slots of the CPU port's KV cache: the capacity of the reference server's StaticCache (max_seq_len 2048 in
# UP/breeze_infer/api.py).  The eager attention of the reference attends over every slot of its static cache (the
# invalid ones masked), so the port does the same whatever the prompt length.
CPU_CACHE_LEN = 2048


def cpu_threads():
    """Host cores this process may run on (its CPU affinity), the BLAS thread count of both CPU legs."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_frames(seconds=None, frames=None, warmup=1, prompt=PROMPT, seed=0, cache_len=CPU_CACHE_LEN, layers=28):
    """The oracle port of one stream's frame (oracle/frame.py: 28-layer backbone step + greedy codebook 0 + 16-codebook
    depth frame, numpy + the C sampler) on this host, its BLAS set to cpu_threads() threads whatever OMP_NUM_THREADS
    a launcher exported.  Times `frames` frames, or frames until `seconds` have passed (at least 2), after `warmup`
    untimed ones.  Returns dict(value frames/s, frames, seconds, threads, cache_len)."""
    import numpy as np
    from threadpoolctl import threadpool_limits
    from oracle import frame as ofr
    threads = cpu_threads()
    with threadpool_limits(limits=threads):
        rng = np.random.default_rng(seed)
        BW = ofr.synthetic_backbone(rng, layers, 2048, 16, 4, 6144, 2049, 17)
        DW = ofr.synthetic_depth(rng, 4, 1024, 2048, 8, 2, 4096, 2048, 2048, 16)
        st = ofr.FrameStream(BW, 16, prompt, cache_len, rng, 2048)
        q = rng.exponential(size=(16, 1, 2048)).astype(np.float32)
        params = (np.array([0.9], np.float32), np.array([50]), np.array([1.0], np.float32), np.array([1]),
                  np.array([4.0], np.float32))
        room = cache_len - prompt - 1               # frames the cache can still take
        for _ in range(min(warmup, room)):
            ofr.frame(BW, DW, st, 2048, 4.0, params, q)
        n = 0
        t0 = time.perf_counter()
        while n < room - warmup:
            ofr.frame(BW, DW, st, 2048, 4.0, params, q)
            n += 1
            el = time.perf_counter() - t0
            if (frames and n >= frames) or (not frames and el >= seconds and n >= 2):
                break
    return dict(value=n / el, frames=n, seconds=el, threads=threads, cache_len=cache_len)


def cpu_sample(r, prompt):
    return (f"{r['frames']} frames of one stream ({r['seconds']:.1f} s after 1 warm-up frame): numpy/C oracle port of "
            f"the 28-layer backbone step (KV cache of {r['cache_len']} slots, {prompt} prompt slots valid + one per "
            f"frame) + greedy codebook 0 + 16-codebook depth frame, {r['threads']} BLAS threads")


def reference_config(a, threads):
    """The `config` of the --impl reference line: what that arm runs (one stream on the host CPU)."""
    return dict(workload='one stream\'s streaming frame on the host CPU: the oracle port of the reference path '
                         '(numpy + C sampler): 28-layer backbone decode step, greedy codebook 0, 16-codebook depth '
                         'frame with CFG top-k sampling', streams=1, prompt_len=a.prompt, cache_len=CPU_CACHE_LEN,
                threads=threads, device='cpu', step='one frame of the stream')


def frame_config(a, world, my_streams, lanes, shared, lane_sms, kv_len, case='frame'):
    """The `config` of the flashb arm's bench line."""
    wl = {'frame': f'streaming frames: 28-layer backbone decode step (2 CFG rows per stream, KV 512+t) + '
                   f'codebook 0 sampled on the device (repetition penalty 1.1, T 0.9, top-k 50) + 16-codebook depth '
                   f'frame (4 layers, V 2048, CFG 4, top-k 50, T 0.9; fresh Exp(1) draws every frame); '
                   f'{a.group} stream(s) per depth launch share the weight reads; {lanes} lane(s) of the GPU side '
                   f'by side; ' + (f'one backbone graph for all {my_streams} streams ({2 * my_streams} rows, GEMVs '
                                   f'as row groups of 64)' if shared else
                                   f'a backbone graph per {a.group} streams on its lane'),
          'depth': 'depth frame only (4 layers, hidden 1024, 16 codebooks of 2048, CFG + top-k 50 sampling)',
          'backbone': 'backbone decode step only (28 layers, hidden 2048, B=2, KV 512+t) + frame link'}[case]
    return dict(workload=wl, streams=my_streams * world, streams_per_gpu=my_streams,
                step='one frame of every stream on the rank', streams_per_launch=a.group, prompt_len=a.prompt,
                kv_len=kv_len, parallelism=f'replica x{world}', lanes=lanes, backbone='shared' if shared else 'lanes',
                lane_sms=lane_sms,
                l2='inputs larger than L2: 2.70 GB backbone weights per step, 130 MB depth weights per codebook '
                   'step; no flush',
                cb0='sampled on the device: the reference runtime\'s backbone sampler (repetition penalty 1.1 over '
                    'the stream\'s earlier codebook-0 tokens, reserved ids suppressed, T 0.9, top-k 50, top-p 1.0, '
                    'multinomial on fresh Exp(1) draws, validity flag)',
                prefill='not timed (random prompt KV)',
                depth_step_table=bool(a.step_table), depth_weights='LN12 (12-bit, decoded in shared memory)' if a.ln12
                else 'bf16')


def run_reference(a):
    """--impl reference: the CPU oracle port of one stream's frame, one frame per step (rank 0 only; other ranks exit
    0 without work), the same function and cache capacity as the flashb arm's cpu_baseline."""
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    r = cpu_frames(frames=a.steps, warmup=a.warmup, prompt=a.prompt)
    v = r['value']
    print(json.dumps(dict(
        impl='reference', metric='frames/s', value=round(v, 4), unit='frames/s', n_gpus=a.gpus, steps=r['frames'],
        warmup=a.warmup, ms_per_step=round(r['seconds'] / r['frames'] * 1e3, 3), higher_is_better=True,
        scaling='weak', vs_baseline=None, dtype='bf16', data='synthetic', config=reference_config(a, r['threads']),
        cpu_baseline=dict(value=round(v, 4), unit='frames/s', cores=r['threads'], kind='port',
                          sample=cpu_sample(r, a.prompt)),
        e2e=dict(value=round(v, 4), unit='frames/s', h2d_bytes_per_step=0, d2h_bytes_per_step=0))), flush=True)


# ------------------------------------------------------------------------------------------------ prefill
def prefill_flops(B, NH, L, D):
    """Algorithmic FLOPs of causal attention: q k^T and p v over the L (L + 1) / 2 admitted (query, key) pairs."""
    return 4 * B * NH * D * L * (L + 1) // 2


def _prefill_inputs(dev, B, NH, NKV, L, D, pads, seed=4):
    import torch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, NH, L, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, NKV, L, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, NKV, L, D, generator=g).to(torch.bfloat16).to(dev)
    qi, ki = torch.arange(L).view(L, 1), torch.arange(L).view(1, L)
    m = torch.full((B, 1, L, L), torch.finfo(torch.bfloat16).min)
    for b, p in enumerate(pads):
        m[b, 0].masked_fill_((ki <= qi) & (ki >= p), 0.0)
    return q, k, v, m.to(torch.bfloat16).to(dev)


def _time_prefill(call, dev, iters, warmup):
    import torch
    from flashb import replicas
    for _ in range(warmup):
        call()
    replicas.barrier(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(iters):
        call()
    e1.record(st)
    replicas.barrier(dev)
    return replicas.max_over_ranks(e0.elapsed_time(e1) / iters, dev)


def measure_prefill(dev, world, rank, iters=50, warmup=5, long_len=4096, long_iters=10):
    """Config 5's causal GQA prefill attention on the tcgen05 kernel, inputs resident.  With 2 or more ranks a
    prompt of at least ``prefill_attn.SPLIT_MIN_LEN`` rows is split (``prefill_attention_sharded``: by KV-head group
    when the ranks divide the 4 KV heads, else by causal-balanced query-row tiles, as for 8 ranks) and one NCCL
    all_gather_into_tensor assembles the output; a shorter one (config 5) runs whole on every rank.  A long prompt
    (L = long_len) is timed on one GPU and, for N > 1, split over the ranks.
    Returns the bench line's ``prefill`` object (rank 0) with TFLOP/s of the whole call."""
    from flashb import prefill_attn
    c = PREFILL_CFG
    B, NH, NKV, L, D = c['B'], c['NH'], c['NKV'], c['L'], c['D']
    q, k, v, m = _prefill_inputs(dev, B, NH, NKV, L, D, c['pads'])
    sharded = world > 1 and L >= prefill_attn.SPLIT_MIN_LEN          # config 5 is too short to gain from a split
    split = ('heads' if NKV % world == 0 else 'rows') if world > 1 else None

    def call():
        if sharded:
            return prefill_attn.prefill_attention_sharded(q, k, v, m, D ** -0.5)
        return prefill_attn.prefill_attention(q, k, v, m, D ** -0.5)

    ms = _time_prefill(call, dev, iters, warmup)
    fl = prefill_flops(B, NH, L, D)
    peak = peaks()['bf16_tflops']
    ach = fl / (ms / 1e3) / 1e12
    # the long prompt: one GPU alone and (N > 1) split over the ranks
    ql, kl, vl, ml = _prefill_inputs(dev, B, NH, NKV, long_len, D, c['pads'], seed=5)
    ms1 = _time_prefill(lambda: prefill_attn.prefill_attention(ql, kl, vl, ml, D ** -0.5), dev, long_iters, 2)
    fll = prefill_flops(B, NH, long_len, D)
    long = dict(L=long_len, ms_one_gpu=round(ms1, 4), tflops_one_gpu=round(fll / (ms1 / 1e3) / 1e12, 2))
    if world > 1:
        msn = _time_prefill(lambda: prefill_attn.prefill_attention_sharded(ql, kl, vl, ml, D ** -0.5), dev,
                            long_iters, 2)
        long.update(ms_sharded=round(msn, 4), split=split, speedup=round(ms1 / msn, 3),
                    tflops_sharded=round(fll / (msn / 1e3) / 1e12, 2))
    del ql, kl, vl, ml
    split_txt = {'heads': 'KV-head groups', 'rows': 'causal-balanced query-row tiles'}.get(split)
    return dict(kernel='prefill_attn_kernel (tcgen05)', config=f'B={B} L={L} NH={NH} NKV={NKV} D={D} causal, pads '
                f'{list(c["pads"])}', parallel=(split_txt + ' + NCCL all_gather_into_tensor') if sharded else
                'whole call per rank', ms=round(ms, 4), algorithmic_flops=fl, achieved=round(ach, 2),
                unit='TFLOP/s', bound='tensor', peak=peak, frac=round(ach / peak, 4),
                launches_per_call=1 + (1 if sharded else 0), long_prompt=long)


# ------------------------------------------------------------------------------------------------ per-config kernels
L2_BYTES = 126 * 1024 * 1024


def _time_calls(fn, n, dev, warmup=5):
    """Average device time (ms) of fn(i) over n calls, i = 0..n-1, CUDA events on the current stream."""
    import torch
    for i in range(warmup):
        fn(i)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for i in range(n):
        fn(i)
    e1.record(st)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / n


def _time_graph(fn, n, dev, reps=5):
    """Average device time (ms) per call of fn(i), i = 0..n-1, captured back to back in one CUDA graph (as the decode
    step runs them: no host work between calls, consecutive launches chained by programmatic dependent launch) and
    replayed ``reps`` times after one untimed replay."""
    import torch
    for i in range(3):
        fn(i)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    g.replay()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize(dev)
    del g
    return e0.elapsed_time(e1) / (reps * n)


def _roof(nbytes, ms, pk, **kw):
    ach = nbytes / (ms / 1e3) / 1e9
    return dict(us=round(ms * 1e3, 2), algorithmic_bytes=int(nbytes), achieved=round(ach, 1), unit='GB/s',
                peak=pk['hbm_gbs'], frac=round(ach / pk['hbm_gbs'], 4), **kw)


def _rn(dev, seed):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def rn(shape, std=1.0, mean=0.0):
        return (torch.randn(shape, generator=g, device=dev) * std + mean).to(torch.bfloat16)
    return rn


def measure_config1(dev, iters=128):
    """Config 1: attn_decode at B 2, 16 q / 4 KV heads, head_dim 128, KV 1024, every key valid.  Distinct q/K/V sets
    are rotated (their total above L2), so every call reads its K/V from HBM."""
    import torch
    from flashb import kernels
    pk, ax, rn = peaks(), kernels.attn(), _rn(dev, 0)
    B, NH, NKV, S, D = 2, 16, 4, 1024, 128
    kvb = 2 * B * NKV * S * D * 2
    nset = 2 * L2_BYTES // kvb + 1
    qs = [rn((B, NH, 1, D)) for _ in range(nset)]
    ks = [rn((B, NKV, S, D)) for _ in range(nset)]
    vs = [rn((B, NKV, S, D)) for _ in range(nset)]
    mask = torch.zeros(B, 1, 1, S, dtype=torch.bfloat16, device=dev)
    o = torch.empty(B, 1, NH, D, dtype=torch.bfloat16, device=dev)
    nws = kernels.attn_ws_floats(B, NH, NKV, S)
    ws = (torch.empty(1, device=dev), torch.empty(1, device=dev), torch.empty(max(1, nws), device=dev),
          torch.zeros(B * NKV, dtype=torch.int32, device=dev))
    def call(i):
        j = i % nset
        ax.attn_decode(qs[j], ks[j], vs[j], mask, D ** -0.5, *ws, o)

    ms = _time_graph(call, iters, dev)
    ms_warm = _time_graph(lambda i: ax.attn_decode(qs[0], ks[0], vs[0], mask, D ** -0.5, *ws, o), iters, dev)
    ms_one = _time_calls(call, iters, dev)
    nbytes = kvb + 2 * B * NH * D * 2
    return _roof(nbytes, ms, pk, shape='B 2, 16 q / 4 KV heads, head_dim 128, KV 1024',
                 timing=f'{iters} calls back to back in a CUDA graph', us_l2_resident=round(ms_warm * 1e3, 2),
                 us_eager_calls=round(ms_one * 1e3, 2),
                 rotation=f'{nset} buffer sets ({nset * kvb / 2 ** 20:.0f} MiB)')


def measure_config2(dev, iters=64):
    """Config 2: gemv_gateup [6144 x 2048] (RMSNorm + SiLU*up) then gemv_resid [2048 x 3072], M = 2; weight sets
    rotated above L2."""
    import torch
    from flashb import kernels
    pk, fx, rn = peaks(), kernels.fused(), _rn(dev, 1)
    M, K, F = 2, 2048, 3072
    wbytes = (2 * F * K + K * F) * 2
    nset = 2 * L2_BYTES // wbytes + 1
    w1 = [rn((2 * F, K), 0.02) for _ in range(nset)]
    w2 = [rn((K, F), 0.02) for _ in range(nset)]
    x, gamma = rn((M, K)), rn((K,), 0.1, 1.0)
    act = torch.empty(M, F, dtype=torch.bfloat16, device=dev)
    y = torch.empty(M, K, dtype=torch.bfloat16, device=dev)

    def pair(i):
        W = w1[i % nset]
        fx.gemv_gateup(x, gamma, 1e-6, W[:F], W[F:], act)
        fx.gemv_resid(act, w2[i % nset], x, y)

    ms = _time_graph(pair, iters, dev)
    ms_gu = _time_graph(lambda i: fx.gemv_gateup(x, gamma, 1e-6, w1[i % nset][:F], w1[i % nset][F:], act), iters,
                        dev)
    ms_dn = _time_graph(lambda i: fx.gemv_resid(act, w2[i % nset], x, y), iters, dev)
    ms_one = _time_calls(pair, iters, dev)
    io = (M * K * 2 + K * 2 + M * F * 2) + (M * F * 2 + 2 * M * K * 2)
    return _roof(wbytes + io, ms, pk, shape='RMSNorm + gate|up [6144 x 2048] + SiLU*up, then down [2048 x 3072] + '
                 'residual, M 2', timing=f'{iters} call pairs back to back in a CUDA graph',
                 us_eager_calls=round(ms_one * 1e3, 2), rotation=f'{nset} weight sets',
                 gateup=_roof(2 * F * K * 2 + M * K * 2 + M * F * 2, ms_gu, pk),
                 down=_roof(K * F * 2 + M * F * 2 + 2 * M * K * 2, ms_dn, pk))


def measure_config3(dev, iters=20, kvs=(256, 1024, 4096)):
    """Config 3: the whole 28-layer backbone decode step (B 2, one CUDA graph of its 142 launches) at each KV length
    (weights 2.70 GB, above L2 on their own)."""
    import torch
    from flashb.engine import BackboneConfig, SyntheticBackboneGraph, backbone_step_bytes
    pk = peaks()
    bcfg = BackboneConfig()
    Smax = max(kvs)
    bb = SyntheticBackboneGraph(bcfg, batch_size=2, max_seq_len=Smax, device=dev, seed=2)
    bb.fill_kv(Smax - 1)
    bb.input_ids_buf.copy_(torch.randint(0, bcfg.vocab, (2, 1, bcfg.codebooks), generator=torch.Generator()
                                         .manual_seed(3)).to(dev))
    sweep = {}
    graph = None
    for L in kvs:
        bb.set_position(L - 1)
        if graph is None:
            for _ in range(3):
                bb.decode_step()
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                bb.decode_step()
        ms = _time_calls(lambda i: graph.replay(), iters, dev, warmup=3)
        sweep[f'kv{L}'] = _roof(backbone_step_bytes(bcfg, 2, L), ms, pk)
    del graph, bb
    torch.cuda.empty_cache()
    return dict(shape='28 layers, hidden 2048, 16 q / 4 KV heads, FFN 6144, B 2; weights + valid KV + fp32 lm_head '
                'per step', launches=2 + 5 * bcfg.layers, **sweep)


def prefill_forward_flops(bcfg, B, L, pads):
    """Algorithmic FLOPs of one prefill forward: the seven GEMMs of every layer over B L tokens, the causal
    attention over each row's live keys (QK^T and PV), the last-token fp32 lm_head."""
    H, D, NH = bcfg.hidden, bcfg.head_dim, bcfg.heads
    params = (NH * D + 2 * bcfg.kv_heads * D) * H + H * NH * D + 3 * bcfg.ffn * H
    gemm = 2 * B * L * params
    attn = 0
    for p in pads:
        n = L - p
        attn += 2 * 2 * NH * D * (n * (n + 1) // 2)
    return bcfg.layers * (gemm + attn) + 2 * B * bcfg.vocab * H


def measure_prefill_forward(dev, iters=5, L=512, pads=(0, 37)):
    """Config 5's prefill (``BackbonePrefillGraphCache._forward``: B 2, L 512, the 28-layer backbone writing its
    StaticCache, last-token logits) on flashb's kernels, captured in one CUDA graph as the reference captures it."""
    import torch
    from flashb import prefill as fpf
    from flashb.engine import BackboneConfig, SyntheticBackboneGraph
    pk = peaks()
    bcfg = BackboneConfig()
    B, S = 2, 1024
    bb = SyntheticBackboneGraph(bcfg, batch_size=B, max_seq_len=S, device=dev, seed=2)
    gen = torch.Generator().manual_seed(9)
    emb = (torch.randn(B, L, bcfg.hidden, generator=gen)).to(torch.bfloat16)
    am = torch.ones(B, L, dtype=torch.long)
    for b, p in enumerate(pads):
        am[b, :p] = 0
        emb[b, :p] = 0
    pos = am.cumsum(-1) - 1
    pos.masked_fill_(am == 0, 1)
    qi, ki = torch.arange(L).view(1, L, 1), torch.arange(S).view(1, 1, S)
    valid = torch.zeros(B, S, dtype=torch.bool)
    valid[:, :L] = am.bool()
    mask = torch.full((B, 1, L, S), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
    mask[:, 0].masked_fill_((ki <= qi) & valid[:, None, :], 0.0)
    e, m, p_, c = emb.to(dev), mask.to(dev), pos.to(dev), torch.arange(L, device=dev)
    st = bb._bb_state
    kv = [(Lc.keys, Lc.values) for Lc in bb.static_cache.layers]
    hid = torch.empty(B, L, bcfg.hidden, dtype=torch.bfloat16, device=dev)
    lg = torch.empty(B, st['lm_head32'].shape[0], dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(2):
            fpf.prefill_forward(st, e, m, p_, c, kv, hidden_out=hid, logits_out=lg)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            fpf.prefill_forward(st, e, m, p_, c, kv, hidden_out=hid, logits_out=lg)
    torch.cuda.current_stream(dev).wait_stream(s)
    ms = _time_calls(lambda i: graph.replay(), iters, dev, warmup=2)
    flops = prefill_forward_flops(bcfg, B, L, pads)
    ach = flops / (ms / 1e3) / 1e12
    peak = pk.get('bf16_tflops', 1590.0)
    del graph, bb, st, kv
    torch.cuda.empty_cache()
    return dict(shape=f'B {B}, L {L} (pads {list(pads)}), 28 layers, hidden 2048, 16 q / 4 KV heads, FFN 6144, '
                f'cache {S}', ms=round(ms, 4), algorithmic_flops=int(flops), achieved=round(ach, 2), unit='TFLOP/s',
                bound='tensor', peak=peak, frac=round(ach / peak, 4),
                launches=2 + 9 * bcfg.layers, timing='one CUDA graph of the whole forward, replayed')


def measure_per_config(dev):
    """BASELINE configs 1-3 at their own shapes, each on the kernels behind its reference entry point, inputs
    resident and larger than L2 between calls, and config 5's whole prefill forward.  Returns the bench line's
    ``per_config`` object."""
    return dict(config1_attn_decode=measure_config1(dev), config2_gemv_pair=measure_config2(dev),
                config3_backbone_step=measure_config3(dev), config5_prefill_forward=measure_prefill_forward(dev))


# ------------------------------------------------------------------------------------------------ GPU
def main():
    a = args_()
    if a.impl == 'reference':
        run_reference(a)
        return
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)
    from flashb import replicas
    from flashb.engine import BackboneConfig, DepthConfig, FrameEngine, backbone_step_bytes
    if a.case in ('config1', 'config2', 'config3'):
        # one BASELINE config alone (a profiling entry point): a.steps calls after a.warmup
        fn = dict(config1=measure_config1, config2=measure_config2, config3=measure_config3)[a.case]
        r = fn(dev, iters=a.steps)
        head = r if a.case != 'config3' else r['kv1024']
        if rank == 0:
            print(json.dumps(dict(metric='HBM GB/s', value=head['achieved'], unit='GB/s', n_gpus=world,
                                  steps=a.steps, warmup=a.warmup, ms_per_step=head['us'] / 1e3, higher_is_better=True,
                                  scaling='weak', vs_baseline=None, dtype='bf16', data='synthetic',
                                  config=dict(workload=a.case), roofline=dict(bound='hbm', **head), detail=r)),
                  flush=True)
        return
    if a.case == 'config5':
        # config 5's whole prefill forward alone (a profiling entry point)
        r = measure_prefill_forward(dev, iters=a.steps)
        if rank == 0:
            print(json.dumps(dict(metric='prefill TFLOP/s', value=r['achieved'], unit='TFLOP/s', n_gpus=world,
                                  steps=a.steps, warmup=a.warmup, ms_per_step=r['ms'], higher_is_better=True,
                                  scaling='weak', vs_baseline=None, dtype='bf16', data='synthetic',
                                  config=dict(workload='config5 prefill forward'),
                                  roofline=dict(bound='tensor', achieved=r['achieved'], peak=r['peak'],
                                                unit='TFLOP/s', frac=r['frac'], traffic=None),
                                  gpu_launches=a.steps * r['launches'], detail=r)), flush=True)
        return
    if a.case == 'prefill':
        pf = measure_prefill(dev, world, rank, iters=a.steps, warmup=max(3, a.warmup))
        if rank == 0:
            print(json.dumps(dict(metric='prefill TFLOP/s', value=pf['achieved'], unit='TFLOP/s', n_gpus=world,
                                  steps=a.steps, warmup=a.warmup, ms_per_step=pf['ms'], higher_is_better=True,
                                  scaling='strong', vs_baseline=None, dtype='bf16', data='synthetic',
                                  config=dict(workload='causal GQA prefill attention, ' + pf['config']),
                                  roofline=dict(bound='tensor', achieved=pf['achieved'], peak=pf['peak'],
                                                unit='TFLOP/s', frac=pf['frac'], traffic=None),
                                  gpu_launches=a.steps * pf['launches_per_call'], detail=pf)), flush=True)
        if world > 1:
            replicas.barrier(dev)
            dist.destroy_process_group()
        return
    bcfg = BackboneConfig(codebooks=17)
    dcfg = DepthConfig()
    total_streams = a.streams * world
    my_streams = len(replicas.streams_for_rank(total_streams, rank, world))
    total_steps = a.warmup + a.steps
    n_runs = 1 if a.no_e2e else 2
    if my_streams % a.group:
        raise SystemExit(f'{my_streams} streams per rank do not split into groups of {a.group}')
    LAT_FRAMES = 20
    # frame: at most one lane per slot; the one-part cases keep the requested lanes, so that a single slot can be
    # timed or profiled at a lane's grid size
    lanes = max(1, min(a.lanes, my_streams // a.group)) if a.case == 'frame' else max(1, a.lanes)
    # one shared backbone graph holds at most 128 rows (64 streams); more streams per GPU run per-lane graphs
    shared = a.backbone == 'shared' and a.case in ('frame', 'backbone') and 2 * my_streams <= 128
    eng = FrameEngine(bcfg, dcfg, my_streams, a.prompt, n_runs * total_steps + LAT_FRAMES + 8, device=dev, seed=0,
                      depth_only=(a.case == 'depth'), group=a.group, single_slot=(a.case == 'frame'),
                      lanes=lanes, shared_backbone=shared)
    if a.step_table:
        eng.use_step_table(True)
    if a.ln12:
        eng.use_ln12(True)
    eng.capture()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        replicas.barrier(dev)

    def maxred(x):
        return replicas.max_over_ranks(x, dev)

    def sumred(x):
        return replicas.sum_over_ranks(x, dev)

    case = a.case
    S = len(eng.streams)          # slots of a.group streams each

    def one_step(ev):
        """One frame of every slot; with ev (a list) an event is recorded before each part on the stream the part
        runs on, and once per lane stream at the end: ev gets (lane stream, kind, event) in issue order."""
        def mark(kind, i, s):
            if ev is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record(s)
                ev.append((s, kind, e))
        if case != 'backbone':
            eng.step(mark)       # the frame, or the depth part alone (an engine without backbone)
            return
        # the backbone part alone, on the current stream (graphs captured with the lane's SM budget, or the shared
        # graph of every slot)
        if eng.shared:
            mark('bb', -1, stream)
            eng.bb_graph.replay()
        else:
            for i in range(S):
                mark('bb', i, stream)
                eng.streams[i].graph.replay()
        mark('end', None, stream)

    # ---- device-resident run
    for _ in range(a.warmup):
        one_step(None)
    kv0 = int(eng.streams[0].bb.cache_position.item()) + 1 if eng.streams[0].bb is not None else 0
    gpu_ids = [int(x) for x in os.environ['CUDA_VISIBLE_DEVICES'].split(',')] \
        if os.environ.get('CUDA_VISIBLE_DEVICES', '').replace(',', '').isdigit() else list(range(world))
    clocks = Clocks(gpu_ids[:world]) if rank == 0 else None
    if clocks:
        clocks.wait_started()
    evs = []
    barrier()
    if clocks:
        clocks.mark()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for t in range(a.steps):
        one_step(evs)   # the lanes join at the end of every step (measured faster than lanes running free)
    t_end.record(stream)
    barrier()
    clk = clocks.stop() if clocks else None
    ms = t_start.elapsed_time(t_end)
    ms_max = maxred(ms)
    frames = sumred(S * a.group * a.steps)
    value = frames / (ms_max / 1e3)
    # per-part durations: each part runs from its event to the next event recorded on the same (lane) stream
    bb_ms, dd_ms = [], []
    last = {}
    for s_, kind, e in evs:
        prev = last.get(s_.cuda_stream)
        if prev is not None:
            (bb_ms if prev[0] == 'bb' else dd_ms).append(prev[1].elapsed_time(e))
        last[s_.cuda_stream] = None if kind in ('end', 'bbend') else (kind, e)
    kv1 = int(eng.streams[0].bb.cache_position.item()) + 1 if eng.streams[0].bb is not None else 0
    pk = peaks()
    dd_bytes = dcfg.frame_weight_bytes(eng.step_table is not None, 2 * a.group, bool(a.ln12))
    bb_rows = 2 * a.group * (S if eng.shared else 1)      # rows of one backbone graph
    bb_bytes = backbone_step_bytes(bcfg, bb_rows, (kv0 + kv1) // 2)
    roof = None
    if dd_ms:
        dd_avg = sum(dd_ms) / len(dd_ms)
        ach = dd_bytes / (dd_avg / 1e3) / 1e9
        roof = dict(kernel='dd_frame_kernel', bound='hbm', achieved=round(ach, 1), peak=pk['hbm_gbs'], unit='GB/s',
                    frac=round(ach / pk['hbm_gbs'], 4), traffic=DD_TRAFFIC_BYTES.get((int(a.step_table), int(a.ln12))),
                    algorithmic_bytes=dd_bytes, launch_ms=round(dd_avg, 4), peak_source=pk['source'],
                    grid=eng.lane_sms or torch.cuda.get_device_properties(dev).multi_processor_count,
                    concurrent_launches=lanes, achieved_all_lanes=round(ach * lanes, 1),
                    frac_all_lanes=round(ach * lanes / pk['hbm_gbs'], 4))
    roof_bb = None
    if bb_ms:
        bb_avg = sum(bb_ms) / len(bb_ms)
        ach = bb_bytes / (bb_avg / 1e3) / 1e9
        nconc = 1 if eng.shared else lanes
        roof_bb = dict(kernels=('backbone step of every slot (GQA decode attention + fused GEMVs + ends, one graph, '
                                f'{bb_rows} rows)' if eng.shared else
                                'backbone step (GQA decode attention + fused GEMVs + ends, 146 launches as a graph)'),
                       bound='hbm', achieved=round(ach, 1), peak=pk['hbm_gbs'], unit='GB/s',
                       frac=round(ach / pk['hbm_gbs'], 4), algorithmic_bytes=bb_bytes, step_ms=round(bb_avg, 4),
                       peak_source=pk['source'], concurrent_steps=nconc, achieved_all_lanes=round(ach * nconc, 1),
                       frac_all_lanes=round(ach * nconc / pk['hbm_gbs'], 4))

    # ---- end-to-end run through the engine API with host buffers
    e2e = None
    if not a.no_e2e and case == 'frame':
        R = 8
        G = a.group
        qh = torch.empty(R, dcfg.n_decode, G, dcfg.vocab).exponential_(1, generator=torch.Generator().manual_seed(5))
        qh = qh.pin_memory()
        toks_h = torch.zeros(2, S, 2 * G + 2 * G * dcfg.n_decode + G, dtype=torch.long).pin_memory()
        h2d = S * qh[0].numel() * 4
        d2h = S * toks_h[0, 0].numel() * 8
        got = [[None] * S, [None] * S]   # per token buffer and slot: the event after that frame's token copies

        copy_stream = torch.cuda.Stream(dev)
        q_in = [None]                    # event: this step's draws are on the device

        def e2e_step(t):
            # every slot: its Exp(1) draws go in from pinned host memory before its frame; after the frame its
            # tokens and validity flags come out into half t % 2 of a double-buffered pinned array.  Before step t
            # reuses a half, the host waits for the tokens step t - 2 copied there (and so holds them), which keeps
            # one step of work queued on the GPU while the host reads the previous one; the lanes still join on
            # the device at the end of every step, so a frame's draws are not replaced while it runs.  The draws go
            # in on a copy stream that starts after that join, so the copy runs beside the backbone step (which
            # does not read them) and each depth frame waits for it.
            def h2d_q(kind, i, s):
                if kind == 'bb':    # i = -1: the shared backbone of every slot
                    for j in (range(S) if i < 0 else (i,)):
                        if got[t & 1][j] is not None:
                            got[t & 1][j].synchronize()
                    copy_stream.wait_stream(s)
                    with torch.cuda.stream(copy_stream):
                        for j in (range(S) if i < 0 else (i,)):
                            eng.streams[j].q.copy_(qh[(j + t) % R], non_blocking=True)
                    q_in[0] = torch.cuda.Event()
                    q_in[0].record(copy_stream)
                elif kind == 'dd' and q_in[0] is not None:
                    s.wait_event(q_in[0])

            def d2h_tokens(kind, i, s):
                st = eng.streams[i]
                toks_h[t & 1, i, :2 * G].copy_(st.first_cb, non_blocking=True)
                toks_h[t & 1, i, 2 * G:-G].copy_(st.outtok.view(-1), non_blocking=True)
                toks_h[t & 1, i, -G:].copy_(eng.cb0_ok[st.c0:st.c0 + G], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s)
                got[t & 1][i] = ev

            eng.step(h2d_q, d2h_tokens)

        eng.draw_q = False          # the depth frame's draws come from the host in this run
        for t in range(a.warmup):
            e2e_step(t)
        torch.cuda.synchronize(dev)
        got = [[None] * S, [None] * S]
        barrier()
        w0 = torch.cuda.Event(enable_timing=True)
        w1 = torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for t in range(a.steps):
            e2e_step(t)
        w1.record(stream)
        for e in got[0] + got[1]:
            if e is not None:
                e.synchronize()     # the last two steps' tokens are on the host
        barrier()
        e_ms = maxred(w0.elapsed_time(w1))
        eng.draw_q = True
        e2e = dict(value=round(frames / (e_ms / 1e3), 3), unit='frames/s', h2d_bytes_per_step=h2d,
                   d2h_bytes_per_step=d2h, ms_per_step=round(e_ms / a.steps, 3))

    # ---- CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and case == 'frame':
        r = cpu_frames(seconds=a.cpu_seconds, prompt=a.prompt)
        cpu = dict(value=round(r['value'], 4), unit='frames/s', cores=r['threads'], kind='port',
                   sample=cpu_sample(r, a.prompt))

    # frame latency of ONE stream (its own single-stream slot on the same weights), graph-replayed back to back
    lat = None
    if case == 'frame' and eng.single is not None:
        for _ in range(3):
            eng.frame('single')
        barrier()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for _ in range(LAT_FRAMES):
            eng.frame('single')
        l1.record(stream)
        barrier()
        lat = round(maxred(l0.elapsed_time(l1) / LAT_FRAMES), 4)
    prefill = measure_prefill(dev, world, rank) if case == 'frame' else None
    per_config = measure_per_config(dev) if case == 'frame' and not a.no_per_config else None
    launches = eng.launches_per_frame() if case == 'frame' else (
        1 if case == 'depth' else eng.launches_per_frame() - 1)
    if rank == 0:
        line = dict(
            metric='frames/s', value=round(value, 3), unit='frames/s', n_gpus=world, steps=a.steps,
            warmup=a.warmup, ms_per_step=round(ms_max / a.steps, 3), higher_is_better=True, scaling='weak',
            vs_baseline=None, dtype='bf16', data='synthetic (seeded random bf16 weights, random prompt KV)',
            config=frame_config(a, world, my_streams, lanes, eng.shared,
                                eng.lane_sms or torch.cuda.get_device_properties(dev).multi_processor_count,
                                [kv0, kv1], case),
            frames_per_s_per_gpu=round(value / world, 3), tokens_per_s=round(value * 17, 1),
            frame_ms_single_stream=lat,
            roofline=roof, roofline_backbone=roof_bb, prefill=prefill, per_config=per_config, cpu_baseline=cpu,
            e2e=e2e,
            gpu_launches=int(launches * frames / a.group), clocks=clk)
        print(json.dumps(line), flush=True)
    if world > 1:
        for st in eng.streams + ([eng.single] if eng.single is not None else []):
            st.graph = None
        eng.bb_graph = None
        barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
