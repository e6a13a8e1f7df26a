"""Clip sharding across GPUs: one encoder replica per GPU, one process per
GPU, no collective on the data path.

The reference runs one encoder on one NPU and serialises requests
(serve/npu_stt_server.py:131); clips are independent, so on N GPUs each rank
encodes its own contiguous slice of the clip batch. torch.distributed is used
only for the barrier around a timed region and the max-over-ranks of the
measured time (gloo on CPU in the tests, nccl on the GPUs).
"""
import torch
import torch.distributed as dist


def shard(n_items, world, rank):
    """Contiguous slice [start, stop) of n_items for `rank` of `world`; the
    first n_items % world ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def barrier():
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(value, device=None):
    """Largest `value` over all ranks (the job's time is its slowest rank's)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    if device is None:
        device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, device=None):
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    if device is None:
        device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_to_all(obj):
    """Every rank's `obj` (picklable), in rank order, on every rank; [obj] when
    not distributed. Used for the per-rank timing and clock records the
    benchmark prints beside the max-over-ranks time."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out
