"""Partitioning of the fused-operator workloads across the GPUs of one node.

Every configuration except the tensor-parallel block shards into independent
problems, so ranks exchange nothing on the data path:

* GEMM / SwiGLU: token rows (``row_range``), weights replicated;
* dense attention: heads (``row_range`` over the head axis) — a head slice of
  [B, S, H, D] storage is a strided view that the kernel reads in place;
* varlen attention: whole sequences, balanced by tokens (``balance_sequences``).

Timing across ranks takes the maximum device time (``max_over_ranks``).
"""

from __future__ import annotations

import heapq
from typing import Sequence


def row_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) slice of n units for ``rank``; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def balance_sequences(lengths: Sequence[int], world: int, cost: str = "tokens") -> list[list[int]]:
    """Assign whole sequences to ``world`` ranks, longest first, each to the least-loaded rank.

    ``cost`` is "tokens" (load = sum of lengths: the token-balanced partition) or
    "quadratic" (load = sum of squared lengths: causal attention work).
    Returns the sequence indices of each rank, each list in ascending order.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    weight = (lambda n: n) if cost == "tokens" else (lambda n: n * n)
    heap = [(0, r) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + weight(lengths[i]), r))
    return [sorted(p) for p in parts]


def cu_seqlens(lengths: Sequence[int]) -> list[int]:
    out = [0]
    for n in lengths:
        out.append(out[-1] + int(n))
    return out


def max_over_ranks(value: float, group=None) -> float:
    """Maximum of a per-rank scalar (e.g. device milliseconds) over the process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
