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
