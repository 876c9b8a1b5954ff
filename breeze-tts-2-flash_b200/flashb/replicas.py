"""Multi-GPU plumbing of the streaming decode: one replica per rank, independent streams, no collective on the
decode path.

Streams are independent (``flash/main_loop.py`` serves one request at a time per GPU), so N GPUs run N replicas:
every rank holds its own copy of the weights and the streams assigned to it.  The only cross-rank traffic is
bookkeeping: a barrier around the timed region and the reductions of timings and frame counts.
"""
import torch
import torch.distributed as dist


def streams_for_rank(n_streams, rank, world):
    """Round-robin assignment: rank r serves streams r, r + world, r + 2 world, ...  Every stream exactly once."""
    if not (0 <= rank < world):
        raise ValueError(f'rank {rank} outside world {world}')
    return list(range(rank, n_streams, world))


def _device_for(group_backend, device):
    return torch.device('cpu') if group_backend == 'gloo' else device


def reduce_scalar(x, op, device=None):
    """All-reduce one float over the default process group (MAX or SUM); identity when not distributed."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    dev = _device_for(dist.get_backend(), device)
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(x, device=None):
    """The job's time is the slowest rank's."""
    return reduce_scalar(x, dist.ReduceOp.MAX, device)


def sum_over_ranks(x, device=None):
    return reduce_scalar(x, dist.ReduceOp.SUM, device)


def barrier(device=None):
    """Synchronise this rank's device, then every rank."""
    if device is not None and device.type == 'cuda':
        torch.cuda.synchronize(device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    if device is not None and device.type == 'cuda':
        torch.cuda.synchronize(device)
