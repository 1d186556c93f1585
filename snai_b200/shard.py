"""Host-side plumbing for one process per GPU.

Sequences are independent (no state is shared between them in
core/cortex.nim:487-563), so N ranks split them into N contiguous shards and
never exchange tensors on the decode path.  torch.distributed is used only
for barriers and the max-over-ranks of timings; sampled ids are gathered
to the host through a gloo group (never NCCL) when a caller wants them in
one place.
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


_gloo = None


def host_group():
    """A gloo process group over every rank (made once, on first use; every
    rank must call this in the same order as its other group calls).  Host
    gathers go through it, so no id ever crosses NCCL."""
    global _gloo
    if _gloo is None:
        _gloo = dist.new_group(backend="gloo") if dist.get_backend() != "gloo" else dist.group.WORLD
    return _gloo


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


def _padded(local_ids, total):
    world = dist.get_world_size()
    sizes = [shard_range(total, r, world) for r in range(world)]
    width = max(b - a for a, b in sizes)
    buf = torch.full((width,), -1, dtype=torch.int32)
    loc = torch.as_tensor(local_ids, dtype=torch.int32).cpu().reshape(-1)
    buf[:loc.numel()] = loc
    return buf, sizes


def gather_ids_host(local_ids, total):
    """Rank 0 receives every rank's int32 ids (host memory, rank order) as one
    tensor of `total` ids; other ranks get None.  Goes through the gloo group
    (host_group()), never NCCL."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return torch.as_tensor(local_ids).to(torch.int32).cpu().reshape(-1)
    buf, sizes = _padded(local_ids, total)
    out = [torch.empty_like(buf) for _ in sizes] if dist.get_rank() == 0 else None
    dist.gather(buf, out, dst=0, group=host_group())
    if out is None:
        return None
    return torch.cat([o[:b - a] for o, (a, b) in zip(out, sizes)])


def gather_ids(local_ids, total):
    """Every rank receives every rank's int32 ids (host memory, rank order),
    through the gloo group."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return torch.as_tensor(local_ids).to(torch.int32).cpu().reshape(-1)
    buf, sizes = _padded(local_ids, total)
    out = [torch.empty_like(buf) for _ in sizes]
    dist.all_gather(out, buf, group=host_group())
    return torch.cat([o[:b - a] for o, (a, b) in zip(out, sizes)])
