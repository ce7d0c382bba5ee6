"""Multi-GPU host plumbing (one process per GPU, torch.distributed).

Sequence sharding needs no collective: each rank runs cottus_paged_decode on
its own sequences.  The long-context path splits every sequence's pages
into contiguous ranges, one per rank; each rank computes normalised partial
outputs with their log-sum-exp (cottus_paged_decode in partial mode), the
partials are all-gathered (NCCL over NVLink on GPUs, gloo on CPU), and every
rank merges them with cottus_lse_combine.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .ops import lse_combine, paged_decode


def all_gather_partials(out: torch.Tensor, lse: torch.Tensor, group=None):
    """[B][H][D] fp32 partials and [B][H] lses from every rank, stacked by rank."""
    world = dist.get_world_size(group)
    out, lse = out.contiguous(), lse.contiguous()
    if out.is_cuda:
        outs = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=out.device)
        lses = torch.empty((world,) + tuple(lse.shape), dtype=lse.dtype, device=lse.device)
        dist.all_gather_into_tensor(outs, out, group=group)
        dist.all_gather_into_tensor(lses, lse, group=group)
        return outs, lses
    outs = [torch.empty_like(out) for _ in range(world)]
    lses = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(outs, out, group=group)
    dist.all_gather(lses, lse, group=group)
    return torch.stack(outs), torch.stack(lses)


def split_kv_decode(query, kv_pool, block_table, context_lens, *, num_kv_heads, head_dim, block_size,
                    num_layers=1, layer=0, num_physical_blocks=None, out_dtype=torch.float16, group=None,
                    part=None, lse=None, stream=None):
    """Decode attention over a context split across the ranks of `group`.
    Inputs are this rank's page range (its pool shard, block table and
    per-sequence token counts); returns the merged output on every rank."""
    B, H, D = query.shape
    if part is None:
        part = torch.empty((B, H, D), dtype=torch.float32, device=query.device)
    if lse is None:
        lse = torch.empty((B, H), dtype=torch.float32, device=query.device)
    paged_decode(query, kv_pool, block_table, context_lens, num_kv_heads=num_kv_heads, head_dim=head_dim,
                 block_size=block_size, num_layers=num_layers, layer=layer, out=part, lse_out=lse,
                 num_physical_blocks=num_physical_blocks, stream=stream)
    parts, lses = all_gather_partials(part, lse, group)
    return lse_combine(parts, lses, out_dtype=out_dtype, stream=stream)
