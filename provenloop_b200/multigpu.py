"""Sharding of independent users across ranks (one process per GPU).

Users -- each a hidden state with its own encryption stream and, optionally,
its own secret key -- have no data dependence on each other (the reference's
_he_lora_delta treats every token independently,
demonstrator/server/inference_engine.py:1197-1405).  So ranks take disjoint
blocks of users and run the whole pipeline locally; the only exchange is
gathering the decrypted deltas to rank 0, one collective per step.
"""
from __future__ import annotations


def user_block(n_users: int, world: int, rank: int):
    """[start, stop) of the users rank `rank` owns: contiguous blocks, the
    first n_users % world ranks get one extra user."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n_users, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def stream_seed(user: int, step: int, n_users: int, seed0: int = 1) -> int:
    """Encryption seed of `user` at `step`: unique per (user, step) and the
    same whichever rank owns the user, so results do not depend on the
    number of GPUs."""
    return seed0 + step * n_users + user


def stream_seeds(users, step: int, n_users: int, seed0: int = 1):
    """stream_seed for an array of users at once (uint64; the per-call cost of
    a whole batch is one vector operation, not a Python loop per user)."""
    import numpy as np

    u = np.asarray(users, dtype=np.uint64)
    return u + np.uint64(seed0 + step * n_users)


def gather_rows(rows, world: int, rank: int, dst: int = 0):
    """Gather each rank's [n_local, d] tensor to `dst` (torch.distributed;
    NCCL for CUDA tensors, gloo on CPU).  All ranks must hold the same
    n_local.  Returns the list of per-rank tensors on dst, else None."""
    import torch
    import torch.distributed as dist

    if world == 1:
        return [rows]
    out = [torch.empty_like(rows) for _ in range(world)] if rank == dst else None
    dist.gather(rows, gather_list=out, dst=dst)
    return out
