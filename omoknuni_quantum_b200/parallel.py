"""Multi-GPU plumbing for the wave search: one process per GPU, independent trees per GPU.

The search itself has no cross-GPU exchange: roots (or self-play games) are partitioned across
ranks and every rank runs its own trees, leaf queues and ResNet. The only collectives are
  * a one-time broadcast of the evaluator weights from rank 0 (NCCL over NVLink on B200; any
    torch.distributed backend works, the CPU tests use gloo), and
  * scalar reductions for reporting (max of the device-timed step time over ranks, sums of
    simulation counts) and an optional gather of per-root results.
The reference has no distributed code at all (its self-play parallelism is CPU processes
feeding one evaluator, python/mcts/neural_networks/self_play_manager.py:552-598).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist


def world() -> tuple:
    """(world_size, rank, local_rank) from the torchrun environment (1, 0, 0 without it)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def shard_range(total: int, world_size: int, rank: int) -> range:
    """Contiguous block of item indices owned by `rank` (sizes differ by at most one)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad world_size / rank")
    base, extra = divmod(total, world_size)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def broadcast_state_dict(sd: Optional[Dict[str, torch.Tensor]], device, src: int = 0,
                         keys: Optional[Sequence[str]] = None) -> Dict[str, torch.Tensor]:
    """Broadcast rank `src`'s state_dict to all ranks in ONE collective: the tensors (sorted key
    order) are packed byte for byte into a single uint8 buffer on `device`, broadcast, and cut
    apart again, so every dtype arrives bit-exact. Every rank passes a state_dict of the
    source's keys, shapes and dtypes (a template built from the same spec)."""
    if not initialized() or dist.get_world_size() == 1:
        return dict(sd)
    if sd is None:
        raise ValueError("every rank needs a template state_dict with the source's shapes")
    names = sorted(sd if keys is None else keys)
    tensors = [sd[k].detach().contiguous() for k in names]
    sizes = [t.numel() * t.element_size() for t in tensors]
    buf = torch.empty(sum(sizes), dtype=torch.uint8, device=device)
    if dist.get_rank() == src:
        off = 0
        for t, n in zip(tensors, sizes):
            buf[off:off + n].copy_(t.reshape(-1).view(torch.uint8))
            off += n
    dist.broadcast(buf, src=src)
    host = buf.cpu()
    out, off = {}, 0
    for k, t, n in zip(names, tensors, sizes):
        out[k] = host[off:off + n].clone().view(t.dtype).reshape(t.shape)
        off += n
    return out


def max_over_ranks(value: float, device) -> float:
    """Maximum of a per-rank scalar (e.g. the device-timed elapsed ms of the timed region)."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device) -> float:
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_results(local: np.ndarray, device) -> Optional[np.ndarray]:
    """Concatenate equally shaped per-rank result arrays on rank 0 (None elsewhere)."""
    if not initialized() or dist.get_world_size() == 1:
        return local
    t = torch.from_numpy(np.ascontiguousarray(local)).to(device)
    parts: List[torch.Tensor] = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    if dist.get_rank() != 0:
        return None
    return torch.cat(parts).cpu().numpy()
