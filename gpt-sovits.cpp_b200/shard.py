"""Session sharding across ranks (one process per GPU) and the scalar reductions the benchmark
needs.  Sessions are independent, so a rank only ever touches its own contiguous shard; the
reductions carry timing and token counts, never data of the decode path."""
from __future__ import annotations


def session_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the sessions owned by `rank`: contiguous, sizes differ by at most one."""
    if world <= 0 or not (0 <= rank < world) or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _reduce(v: float, op: str, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(v)
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(v: float, device=None) -> float:
    return _reduce(v, "max", device)


def sum_over_ranks(v: float, device=None) -> float:
    return _reduce(v, "sum", device)
