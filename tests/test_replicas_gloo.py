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
