"""Sequence sharding across GPUs (one process per GPU).

The paged KV cache shards by sequence: each rank owns whole sequences, its own
block pool and block tables, so append, gather, decode and checkpoints never
touch another rank's memory and the data path has no collective.  These are the
host-side pieces around that: the partition (balanced by context tokens, since
lengths span 512x), the throughput aggregation (sum of work / max of time over
ranks), and a gather of per-rank outputs to rank 0 in global sequence order,
used only for checking.  They work on any torch.distributed backend (NCCL on
the GPUs, gloo on CPU in the tests).
"""
from __future__ import annotations

import numpy as np


def lpt_partition(lens, n_parts):
    """Greedy LPT: the longest sequence first, each to the least-loaded part
    (ties to the lower rank).  Returns (sorted sequence ids per part, tokens per part)."""
    lens = np.asarray(lens, np.int64)
    if n_parts < 1:
        raise ValueError("n_parts must be >= 1")
    order = np.argsort(-lens, kind="stable")
    loads = [0] * n_parts
    parts = [[] for _ in range(n_parts)]
    for s in order:
        k = min(range(n_parts), key=lambda i: (loads[i], i))
        parts[k].append(int(s))
        loads[k] += int(lens[s])
    return [sorted(p) for p in parts], loads


def aggregate_throughput(work, seconds, dist=None, device=None):
    """Whole-job (total work, job time): work summed over ranks, time = the
    slowest rank's.  Single-process when `dist` is None or not initialised."""
    if dist is None or not dist.is_available() or not dist.is_initialized():
        return float(work), float(seconds)
    import torch

    w = torch.tensor([float(work)], dtype=torch.float64, device=device)
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(w, op=dist.ReduceOp.SUM)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return w.item(), t.item()


def gather_to_root(local, parts, dist):
    """Collect each rank's rows (one row per owned sequence, in the order of
    parts[rank]) into rank 0 as one array in global sequence order.  `local` is
    a torch tensor [len(parts[rank]), ...]; ranks are padded to the largest
    part for the all-gather.  Returns the full tensor on rank 0, None elsewhere."""
    import torch

    rank, world = dist.get_rank(), dist.get_world_size()
    if len(parts) != world:
        raise ValueError(f"{len(parts)} parts for {world} ranks")
    if local.shape[0] != len(parts[rank]):
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, owns {len(parts[rank])} sequences")
    cap = max(len(p) for p in parts)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    if rank != 0:
        return None
    n = sum(len(p) for p in parts)
    out = torch.empty((n,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    for r, p in enumerate(parts):
        if p:
            out[torch.as_tensor(p, device=local.device)] = bufs[r][: len(p)]
    return out
