"""Host-side work distribution across GPUs (one process per GPU, no collective on the data path).

Images and recognizer crops are independent, so every rank runs the whole
model on its own share: detector images round-robin, recognizer crops split
evenly and then bucketed by width into fixed-size batches (one compiled plan
per bucket width, as the reference caches one session per input shape,
src/ocr.rs:648-685).  The only cross-rank traffic is the timing reduction.
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Tuple


def round_robin(count: int, world: int, rank: int) -> List[int]:
    """Indices of the items rank `rank` owns when `count` items are dealt round-robin."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return list(range(rank, count, world))


def even_split(count: int, world: int, rank: int) -> range:
    """Contiguous share of `count` items; the first count % world ranks take one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(count, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def width_buckets(widths: Sequence[int], buckets: Sequence[int], batch: int) -> List[Tuple[int, List[int]]]:
    """Group crop indices by the smallest bucket width that holds them, in batches of at most `batch`.

    Returns [(bucket_width, indices)] ordered by bucket width, then by index.
    A crop wider than the largest bucket is an error (the caller resizes first).
    """
    if batch <= 0:
        raise ValueError("batch must be positive")
    order = sorted(buckets)
    groups: Dict[int, List[int]] = {b: [] for b in order}
    for i, w in enumerate(widths):
        for b in order:
            if w <= b:
                groups[b].append(i)
                break
        else:
            raise ValueError(f"crop {i} width {w} exceeds the largest bucket {order[-1]}")
    out = []
    for b in order:
        idx = groups[b]
        for s in range(0, len(idx), batch):
            out.append((b, idx[s:s + batch]))
    return out


def max_over_ranks(value: float) -> float:
    """Max of a per-rank scalar (the device time of the timed region) over the process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
