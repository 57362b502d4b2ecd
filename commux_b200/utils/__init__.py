"""Utilities: clock sampling, rank-max device timing, rendezvous helpers."""

from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def env_rank() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from torchrun's environment (defaults 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def rank_max(values, group=None) -> list[float]:
    """Element-wise max over ranks of a list of floats (host collective)."""
    t = torch.tensor([float(v) for v in values], dtype=torch.float64)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()


def rank_sum(values, group=None) -> list[float]:
    t = torch.tensor([float(v) for v in values], dtype=torch.float64)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t.tolist()
