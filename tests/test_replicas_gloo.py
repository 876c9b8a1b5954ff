"""The N > 1 host logic of the replica bench, on CPU with two gloo ranks: every stream is served by exactly one
rank, the job time is the maximum over ranks and the frame count their sum, and a rank that raises fails the run
instead of hanging it (short process-group timeout)."""
import datetime
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), 'breeze-tts-2-flash_b200')


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_streams, out, fail_rank):
    sys.path.insert(0, PKG)
    import torch.distributed as dist
    from flashb import replicas
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        mine = replicas.streams_for_rank(n_streams, rank, world)
        replicas.barrier()
        if rank == fail_rank:
            raise RuntimeError('injected failure on the host')
        t = replicas.max_over_ranks(1.0 + rank)
        n = replicas.sum_over_ranks(len(mine))
        out.put((rank, mine, t, n))
    finally:
        dist.destroy_process_group()


def _run(world, n_streams, fail_rank=-1):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_streams, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    return codes, sorted(res)


def test_two_ranks_partition_streams_and_reduce():
    codes, res = _run(2, 64)
    assert codes == [0, 0]
    assert len(res) == 2
    served = sorted(s for _, mine, _, _ in res for s in mine)
    assert served == list(range(64))
    for _, mine, t, n in res:
        assert t == 2.0 and n == 64 and len(mine) == 32


def test_rank_failure_surfaces_instead_of_hanging():
    codes, res = _run(2, 8, fail_rank=1)
    assert codes[1] not in (0, None)   # the failing rank exits with an error
    assert codes[0] not in (0, None)   # its peer's next collective errors out (peer gone / timeout); no hang
    assert res == []                   # no rank reports a result for a failed job


def test_streams_for_rank_rejects_bad_rank():
    sys.path.insert(0, PKG)
    from flashb import replicas
    with pytest.raises(ValueError):
        replicas.streams_for_rank(8, 2, 2)
    assert replicas.streams_for_rank(5, 1, 4) == [1]


def _prefill_worker(rank, world, port, out):
    """Two CPU ranks: each computes its KV-head group's q heads with the oracle (the stand-in for the kernel on a
    GPU rank) and the shards are gathered with flashb.prefill_attn.gather_head_shards."""
    sys.path.insert(0, PKG)
    sys.path.insert(0, os.path.dirname(HERE))
    import numpy as np
    import torch
    import torch.distributed as dist
    from flashb import prefill_attn
    from oracle import prefill as opf
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        g = torch.Generator().manual_seed(3)
        B, NH, NKV, L = 1, 8, 2, 24
        q = torch.randn(B, NH, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        k = torch.randn(B, NKV, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        v = torch.randn(B, NKV, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        mask = np.where(np.arange(L)[None, :] <= np.arange(L)[:, None], 0.0, -3.3895313892515355e38)
        mask = mask.astype(np.float32)[None, None]
        h0, h1 = prefill_attn.shard_heads(NH, NKV, world, rank)
        G = NH // NKV
        kv0, kv1 = h0 // G, h1 // G
        part = opf.prefill_attention(q[:, h0:h1], k[:, kv0:kv1], v[:, kv0:kv1], mask, 128 ** -0.5)
        full = prefill_attn.gather_head_shards(torch.from_numpy(np.ascontiguousarray(part)))
        ref = opf.prefill_attention(q, k, v, mask, 128 ** -0.5)
        out.put((rank, bool(np.array_equal(full.numpy(), ref)), (h0, h1)))
    finally:
        dist.destroy_process_group()


def test_prefill_head_shards_gather_to_the_full_output():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_prefill_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert [p.exitcode for p in procs] == [0, 0]
    res = sorted(q.get() for _ in range(2))
    assert res == [(0, True, (0, 4)), (1, True, (4, 8))]


def _row_worker(rank, world, port, out):
    """CPU ranks: each computes its causal-balanced range of query-row tiles with the oracle (the stand-in for the
    kernel on a GPU rank), the ranges are gathered with flashb.prefill_attn.gather_row_shards (one
    all_gather_into_tensor of padded parts)."""
    sys.path.insert(0, PKG)
    sys.path.insert(0, os.path.dirname(HERE))
    import numpy as np
    import torch
    import torch.distributed as dist
    from flashb import prefill_attn
    from oracle import decode as dec
    from oracle import prefill as opf
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        g = torch.Generator().manual_seed(4)
        B, NH, NKV, L = 2, 4, 2, 300
        q = torch.randn(B, NH, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        k = torch.randn(B, NKV, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        v = torch.randn(B, NKV, L, 128, generator=g).to(torch.bfloat16).float().numpy()
        mask = np.where(np.arange(L)[None, :] <= np.arange(L)[:, None], 0.0, -3.3895313892515355e38)
        mask = mask.astype(np.float32)[None, None]
        ranges = prefill_attn.row_shards(L, world)
        t0, t1 = ranges[rank]
        rows = max(min(L, b * 128) - a * 128 for a, b in ranges)
        part = np.zeros((B, rows, NH, 128), np.float32)
        r0, r1 = t0 * 128, min(L, t1 * 128)
        if r1 > r0:
            # a shard's rows attend to every key of the (already trimmed) cache: the eager attention, no re-trim
            part[:, :r1 - r0] = dec.attention_eager(q[:, :, r0:r1], k, v, mask[:, :, r0:r1], 128 ** -0.5)
        full = prefill_attn.gather_row_shards(torch.from_numpy(part), ranges, L)
        ref = opf.prefill_attention(q, k, v, mask, 128 ** -0.5)
        out.put((rank, bool(np.array_equal(full.numpy(), ref)), (t0, t1)))
    finally:
        dist.destroy_process_group()


def test_prefill_row_shards_gather_to_the_full_output():
    """The N > NKV split (e.g. 8 ranks over 4 KV heads) by query rows, here 3 ranks over 300 rows (3 tiles): each
    rank's causal-balanced tile range, gathered to the full output on every rank."""
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert [p.exitcode for p in procs] == [0, 0, 0]
    res = sorted(q.get() for _ in range(3))
    assert all(ok for _, ok, _ in res)
    assert [r for _, _, r in res] == [(0, 2), (2, 3), (3, 3)] or [r for _, _, r in res] == [(0, 1), (1, 2), (2, 3)]


def test_row_shards_balance_the_causal_work():
    sys.path.insert(0, PKG)
    from flashb.prefill_attn import row_shards
    for L, n in ((4096, 8), (4096, 4), (4096, 2), (512, 8), (1000, 3), (100, 4)):
        r = row_shards(L, n)
        T = (L + 127) // 128
        assert len(r) == n and r[0][0] == 0 and r[-1][1] == T
        assert all(a <= b for a, b in r) and all(r[i][1] == r[i + 1][0] for i in range(n - 1))
        work = [sum(t + 1 for t in range(a, b)) for a, b in r]
        ideal = T * (T + 1) / 2 / n
        # within one tile's work (the largest, T) of the ideal share
        assert max(work) <= ideal + T
