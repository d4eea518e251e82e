"""Partitioning pages across GPUs (one process per GPU, no collective on the data path).

Pages are independent -- one SipHash chain and one keystream per page -- so ranks never exchange page
data.  Two forms:

* strong: a fixed list of pages (e.g. a 4,096-token x 64-layer prefix addressed through a shuffled block
  table) split into contiguous, balanced per-rank ranges (``shard_range``);
* weak: every rank processes its own batches; ``global_page_base`` gives each (rank, batch) a disjoint
  global page range, so sequence nonces ``base + global page index`` never repeat across ranks.

``max_over_ranks`` is the only collective the benchmark uses (timings), and works with the gloo backend
on CPU as with NCCL on GPU.
"""
from __future__ import annotations


def shard_range(n_pages: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, start + count) of `n_pages` for `rank`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if n_pages < 0:
        raise ValueError("n_pages must be non-negative")
    base, extra = divmod(n_pages, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def global_page_base(rank: int, batch: int, batches_per_rank: int, pages_per_batch: int) -> int:
    """First global page index of `batch` on `rank` when every rank owns `batches_per_rank` batches."""
    if not 0 <= batch < batches_per_rank:
        raise ValueError("batch must lie in [0, batches_per_rank)")
    return (rank * batches_per_rank + batch) * pages_per_batch


def max_over_ranks(values, device=None):
    """Element-wise maximum of a list of floats over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]
