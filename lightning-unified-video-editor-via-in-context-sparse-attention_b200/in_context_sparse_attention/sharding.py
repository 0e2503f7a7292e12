"""Multi-GPU plumbing for the in-context sparse attention call.

The call is independent per (batch, head): every stage of the reference is
computed per (b, h) (editing_sparse_attention.py:126-136 for the in-context
top-K, :161-172 for the split, and the kernels are gridded over B*H).  Heads
are therefore split across ranks with no collective on the data path; the
helpers here only place work, time it (maximum over ranks) and, for
verification, gather results.

For a DiT that keeps the sequence sharded across ranks (the full-model
configuration), `seq_to_heads` / `heads_to_seq` are the Ulysses-style
all-to-all exchanges around the call: [B, S/n, H, D] per rank <->
[B, S, H/n, D] per rank, one NCCL all_to_all_single each way.

One process per GPU, torch.distributed for the plumbing (NCCL on GPUs; the
tests run the same code on CPU with gloo).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_range(num_heads: int, rank: int, world: int) -> range:
    """Heads owned by `rank`: contiguous, equal shares (num_heads % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split evenly over {world} ranks")
    per = num_heads // world
    return range(rank * per, (rank + 1) * per)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Maximum of a per-rank scalar (the slowest rank sets a step's time)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t[0])


def gather_heads(x_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather [B, S, H/n, D] head shards into [B, S, H, D] (verification only)."""
    world = dist.get_world_size(group)
    parts = [torch.empty_like(x_local) for _ in range(world)]
    dist.all_gather(parts, x_local.contiguous(), group=group)
    return torch.cat(parts, dim=2)


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, S/n, H, D] (sequence shard) -> [B, S, H/n, D] (head shard).

    Rank r sends head group g of its sequence shard to rank g; the received
    pieces are the sequence shards of head group r in rank order.
    """
    world = dist.get_world_size(group)
    B, s, H, D = x.shape
    if H % world:
        raise ValueError(f"{H} heads do not split over {world} ranks")
    hp = H // world
    # [B, s, n, hp, D] -> [n, B, s, hp, D]: chunk g goes to rank g
    send = x.reshape(B, s, world, hp, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[r] = sequence shard r of my head group -> [B, n*s, hp, D]
    return recv.permute(1, 0, 2, 3, 4).reshape(B, world * s, hp, D)


def heads_to_seq(y: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of seq_to_heads: [B, S, H/n, D] -> [B, S/n, H, D]."""
    world = dist.get_world_size(group)
    B, S, hp, D = y.shape
    if S % world:
        raise ValueError(f"sequence of {S} does not split over {world} ranks")
    s = S // world
    send = y.reshape(B, world, s, hp, D).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[g] = head group g of my sequence shard -> [B, s, n*hp, D]
    return recv.permute(1, 2, 0, 3, 4).reshape(B, s, world * hp, D)
