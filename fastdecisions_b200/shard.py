"""Request-level data parallelism across the GPUs of one node.

Every rank holds a full model replica; independent decision requests are split into
length-balanced bins (LPT: longest processing time first, onto the least-loaded rank, with the
request's forward FLOPs as its cost), each rank runs its own bins with no collective on the hot
path, and only the final answer probabilities are gathered to rank 0.  The reference serves from
one process and one GPU thread (src/decider/serve.py:365,401); this is the scale-out it lacks.
"""
from __future__ import annotations

import heapq
from typing import Sequence

import numpy as np
import torch


def lpt_partition(costs: Sequence[float], n_ranks: int) -> list:
    """Indices of the items each rank gets; greedy longest-first onto the least-loaded rank."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    heap = [(0.0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    bins = [[] for _ in range(n_ranks)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    for b in bins:
        b.sort()
    return bins


def bin_loads(costs: Sequence[float], bins: list) -> list:
    return [float(sum(costs[i] for i in b)) for b in bins]


def gather_probs(local_ids: np.ndarray, local_probs: torch.Tensor, n_total: int, group=None):
    """Gather ``(request id, probability row)`` pairs of every rank to rank 0 (all ranks call).

    Rows are padded to the largest local count, exchanged with one all_gather (NCCL on GPUs or
    Gloo on CPU tensors), and rank 0 returns the ``[n_total, K]`` matrix in request order; other
    ranks return None.  With no process group it just reorders the local rows.
    """
    import torch.distributed as dist
    K = local_probs.shape[1]
    dev = local_probs.device
    if not (dist.is_available() and dist.is_initialized()):
        out = torch.zeros(n_total, K, dtype=local_probs.dtype, device=dev)
        out[torch.as_tensor(local_ids, device=dev, dtype=torch.long)] = local_probs
        return out
    world = dist.get_world_size(group)
    n_local = torch.tensor([len(local_ids)], device=dev, dtype=torch.int64)
    counts = [torch.zeros_like(n_local) for _ in range(world)]
    dist.all_gather(counts, n_local, group=group)
    m = int(max(c.item() for c in counts))
    buf = torch.full((m, K + 1), -1.0, device=dev, dtype=torch.float32)
    buf[:len(local_ids), 0] = torch.as_tensor(local_ids, device=dev, dtype=torch.float32)
    buf[:len(local_ids), 1:] = local_probs.float()
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    if dist.get_rank(group) != 0:
        return None
    allb = torch.cat(parts)
    valid = allb[:, 0] >= 0
    ids = allb[valid, 0].long()
    out = torch.zeros(n_total, K, device=dev, dtype=torch.float32)
    out[ids] = allb[valid, 1:]
    return out
