"""Expert-ID sharding of the stack over the GPUs of one node (one process per GPU).

Rank r of `world` holds experts [r*E/world, (r+1)*E/world) of every layer
(`shard_range`). The banks exchange CUDA IPC handles of their exchange regions over the
process group (host plumbing only: torch.distributed with any backend) and then run the
stack together: every rank calls `stack_decode*` with the same token, computes the picks
it owns, and the rows of every pick reach every GPU through peer stores inside the
persistent kernel (clb_bank_connect). Mirrors the lane split of crosslane's
`warm_execute` (runtime.cpp:121-189), with GPUs in place of lanes.

The batched stack (`stack_batch_device`, a batch of tokens per step) exchanges per layer
the [T*k][dim] expert rows: each rank fills the rows of the picks it owns (the others are
zero), an all-reduce (sum) over the process group (NCCL on GPUs) gives every rank every
row exactly, and every rank runs the same ascending-id combine.
"""
from __future__ import annotations

from .bank import ExpertBank


def shard_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous expert block of `rank`: [rank*E//world, (rank+1)*E//world)."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside [0, {world})")
    return rank * n_experts // world, (rank + 1) * n_experts // world


def owner_of(expert: int, n_experts: int, world: int) -> int:
    """Rank whose block holds `expert` (inverse of shard_range)."""
    for r in range(world):
        b, e = shard_range(n_experts, r, world)
        if b <= expert < e:
            return r
    raise ValueError(f"expert {expert} outside [0, {n_experts})")


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' 64-byte handles, indexed by rank (torch.distributed all_gather_object)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class ShardedBank(ExpertBank):
    """An ExpertBank holding this rank's expert block, connected to its peers."""

    def __init__(self, *, n_layers: int, n_experts: int, dim: int, ff: int, max_picks: int = 6,
                 limit: float = 0.0, device: int = 0, rank: int, world: int, exact_order: bool = False,
                 group=None):
        b, e = shard_range(n_experts, rank, world)
        super().__init__(n_layers=n_layers, n_experts=n_experts, dim=dim, ff=ff, max_picks=max_picks, limit=limit,
                         device=device, expert_begin=b, expert_end=e, exact_order=exact_order)
        self.rank, self.world = rank, world
        if world > 1:
            self.connect(rank, world, exchange_handles(self.exchange_handle(), group))

    def stack_batch_device(self, first_layer: int, n_layers: int, d_h, d_logits, d_ws, d_rows, group=None) -> None:
        """d_h [T][dim] (identical on every rank, updated in place), d_logits [n_layers][T][E],
        d_ws (stack_batch_workspace_bytes), d_rows float32 [T*k][dim]; all on this rank's GPU,
        enqueued on the bank stream (the all-reduce is ordered on it too, which makes torch's
        allocator record that stream on d_rows: free d_rows before closing the bank)."""
        import torch
        import torch.distributed as dist

        stream = torch.cuda.ExternalStream(self.stream)
        with torch.cuda.stream(stream):
            for l in range(n_layers):
                self.stack_batch_layer_device(first_layer + l, d_h, d_logits[l], d_rows, d_ws, 1)
                if self.world > 1:
                    dist.all_reduce(d_rows, group=group)
                self.stack_batch_layer_device(first_layer + l, d_h, d_logits[l], d_rows, d_ws, 2)
