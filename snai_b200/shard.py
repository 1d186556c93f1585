"""Host-side plumbing for one process per GPU.

Sequences are independent (no state is shared between them in
core/cortex.nim:487-563), so N ranks split them into N contiguous shards and
never exchange tensors on the decode path.  torch.distributed is used only
for barriers, the max-over-ranks of timings, and gathering sampled ids to
rank 0 when a caller wants them in one place.
"""
import torch
import torch.distributed as dist


def shard_range(total, rank, world):
    """[start, stop) of rank's contiguous share; shares differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _device():
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(x):
    """The maximum of a float over all ranks (x itself without a group)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_ids(local_ids, total):
    """Concatenates every rank's int32 ids (in rank order) on every rank."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return torch.as_tensor(local_ids).to(torch.int32).cpu()
    world = dist.get_world_size()
    dev = _device()
    sizes = [shard_range(total, r, world) for r in range(world)]
    width = max(b - a for a, b in sizes)
    buf = torch.full((width,), -1, dtype=torch.int32, device=dev)
    loc = torch.as_tensor(local_ids, dtype=torch.int32)
    buf[:loc.numel()] = loc.to(dev)
    out = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(out, buf)
    return torch.cat([o[:b - a].cpu() for o, (a, b) in zip(out, sizes)])
