"""(batch x head) sharding of the attention forward over GPUs.

Every (b, h) slice of the problem is independent, so ranks split the
flattened B*H range into contiguous near-equal blocks and compute their
block with no communication.  The only cross-GPU step is the optional
gather of the output shards (NCCL all-gather over NVLink), which is not part
of the hot path.

One process per GPU (torchrun); the process group is the caller's.
"""

import torch
import torch.distributed as dist

from .sparse_attention import sparse_attention


def shard_range(total, world, rank):
    """[lo, hi) of rank's contiguous block of `total` items; block sizes
    differ by at most one and earlier ranks get the larger blocks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def shard_heads(x, world, rank):
    """Rank's slice of a [B, H, ...] tensor over the flattened B*H range, as
    a [1, hi-lo, ...] view (contiguous when x is)."""
    B, H = x.shape[:2]
    lo, hi = shard_range(B * H, world, rank)
    return x.reshape((B * H,) + tuple(x.shape[2:]))[lo:hi].unsqueeze(0)


def gather_heads(local, total_heads, group=None):
    """All-gather rank outputs [1, h_r, ...] into [1, total_heads, ...] on
    every rank.  Uneven blocks are padded to the largest block for the
    collective and trimmed afterwards."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    max_h = shard_range(total_heads, world, 0)[1]
    lo, hi = shard_range(total_heads, world, rank)
    assert local.shape[1] == hi - lo, f"rank {rank} holds {local.shape[1]} heads, expected {hi - lo}"
    tail = tuple(local.shape[2:])
    padded = local.new_zeros((max_h,) + tail)
    padded[: hi - lo] = local[0]
    if dist.get_backend(group) == "nccl":
        buf = local.new_empty((world * max_h,) + tail)
        dist.all_gather_into_tensor(buf, padded, group=group)
        parts = list(buf.view((world, max_h) + tail))
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
    pieces = []
    for r in range(world):
        rlo, rhi = shard_range(total_heads, world, r)
        pieces.append(parts[r][: rhi - rlo])
    return torch.cat(pieces).unsqueeze(0)


def sharded_sparse_attention(q, k, v, mask, group=None, gather=False, total_heads=None, attention=sparse_attention):
    """Attention on this rank's shard ([1, h_r, N, D] inputs, e.g. from
    shard_heads); with gather=True every rank returns the full
    [1, total_heads, N, D] output.  `attention` is the per-shard function
    (the CUDA path by default)."""
    out = attention(q, k, v, mask)
    if not gather:
        return out
    if total_heads is None:
        total_heads = torch.tensor([q.shape[1]], device=out.device)
        dist.all_reduce(total_heads, group=group)
        total_heads = int(total_heads.item())
    return gather_heads(out, total_heads, group=group)
