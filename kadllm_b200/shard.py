"""Request sharding across ranks (one process per GPU) and the result exchange.

GRBeam requests are independent, so N ranks each run their own batch of
requests with a replicated model (weak scaling) and no collective between
them; the finished beams (tokens and scores) can be all-gathered into one
result afterwards, and the timing takes the max over ranks.  NCCL over NVLink
on the GPU box; the same functions run on ``gloo`` for the CPU tests.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def rank_prompts(rank: int, batch: int, prompt: int, vocab: int) -> np.ndarray:
    """This rank's shard of synthetic requests: [batch, prompt] token ids seeded by rank."""
    from .synthetic import random_prompts

    return random_prompts(batch, prompt, vocab, seed=rank)


def _all_gather(t: torch.Tensor) -> torch.Tensor:
    world = dist.get_world_size()
    t = t.contiguous()
    if dist.get_backend() == "nccl":
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t)
        return out
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return torch.cat(parts)


def gather_beams(tokens: torch.Tensor, scores: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """All ranks' finished beams in rank order: tokens [world*B, W, D], scores [world*B, W].

    Without an initialised process group (one GPU) the inputs are returned."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return tokens, scores
    return _all_gather(tokens), _all_gather(scores)


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """The largest value over ranks (every rank gets it); identity on one process."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(value: float, device: torch.device | str = "cpu") -> list[float]:
    """Every rank's value, in rank order (every rank gets the list); [value] on one process."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(value)]
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    return [float(x) for x in _all_gather(t).tolist()]
