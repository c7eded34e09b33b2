"""Data parallelism for the LoRA-linear path: tokens shard across ranks (one
process per GPU); the forward needs no communication; training averages the
LoRA gradients (the only state that differs between ranks) with one
all-reduce over the flat gradient buffer.  The reference is single-device; this
is the multi-GPU layer of this implementation."""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n_tokens: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of this rank's contiguous token shard (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n_tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of a [tokens, ...] (or [batch, seq, ...], flattened) tensor."""
    flat = x.reshape(-1, *x.shape[2:]) if x.dim() > 2 else x
    b, e = shard_bounds(flat.shape[0], rank, world)
    return flat[b:e]


def average_gradients(flat_grad: torch.Tensor, group=None) -> None:
    """In-place mean of a flat gradient buffer over the process group (AVG on
    NCCL; SUM then scale elsewhere)."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    if dist.get_backend(group) == "nccl":
        dist.all_reduce(flat_grad, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(flat_grad, group=group)
        flat_grad.mul_(1.0 / world)


def replicas_in_sync(t: torch.Tensor, group=None) -> bool:
    """True when every rank holds a bitwise-identical copy of ``t`` (checked
    through an all-gathered checksum)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return True
    v = t.detach().reshape(-1).view(torch.int32) if t.element_size() == 4 else \
        t.detach().reshape(-1).to(torch.float32).view(torch.int32)
    chk = torch.stack([v.sum(dtype=torch.int64), (v.to(torch.int64) * 31).sum()]).to(t.device)
    out = [torch.zeros_like(chk) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, chk, group=group)
    return all(torch.equal(o, out[0]) for o in out)
