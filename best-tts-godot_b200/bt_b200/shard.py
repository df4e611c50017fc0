"""Utterance sharding for one process per GPU.

The decoder-stage stream is independent per utterance (every op of the
stream works within one utterance's rows), so N GPUs split the utterances
and exchange nothing on the data path: rank r runs its own utterances
through its own FusedDecoder and copies its own results to its own pinned
host buffer.  The only collectives are host-side bookkeeping outside the
timed work (a barrier and the max of the per-rank times).  These helpers
work with any torch.distributed backend (NCCL on the GPU box, gloo in the
CPU tests).
"""
import torch
import torch.distributed as dist


def world_and_rank():
    """(world size, rank) of the initialised process group, (1, 0) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def utterance_range(per_rank, rank):
    """Global ids [start, start + per_rank) of rank's utterances (weak
    scaling: every rank takes the same number)."""
    if per_rank < 0 or rank < 0:
        raise ValueError("per_rank and rank must be non-negative")
    return rank * per_rank, per_rank


def split_utterances(total, world, rank):
    """Global ids [start, start + count) of rank's share of a fixed total
    (strong scaling): contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("need world >= 1, 0 <= rank < world, total >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def rank_seed(base, rank):
    """Seed of rank's synthetic inputs (distinct per rank)."""
    return int(base) + int(rank)


def max_over_ranks(value, device=None):
    """Maximum of a float over all ranks (the job's time is its slowest
    rank's).  device: where the reduction tensor lives (a CUDA device for
    NCCL, None -> CPU for gloo)."""
    world, _ = world_and_rank()
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, device=None):
    """Sum of a number over all ranks (bytes moved by the whole job)."""
    world, _ = world_and_rank()
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(device=None):
    """Barrier across ranks, then (on a GPU) a device synchronize."""
    world, _ = world_and_rank()
    if world > 1:
        dist.barrier()
    if device is not None and torch.cuda.is_available():
        torch.cuda.synchronize(device)
