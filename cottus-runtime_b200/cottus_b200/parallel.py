"""Multi-GPU host plumbing (one process per GPU, torch.distributed).

Sequence sharding needs no collective: each rank runs cottus_paged_decode on
its own sequences.  The long-context path splits every sequence's pages
into contiguous ranges, one per rank; each rank computes normalised partial
outputs with their log-sum-exp (cottus_paged_decode in partial mode), the
partials are all-gathered (NCCL over NVLink on GPUs, gloo on CPU), and every
rank merges them with cottus_lse_combine.  PeerExchange/split_kv_decode_peer
do the same exchange without a collective library call: partials are read
from the other ranks' memory over NVLink after a completion flag that the
decode kernel itself raises (cottus_split_decode).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from ._lib import check, lib
from .ops import _stream, lse_combine, make_decode_params, paged_decode, workspace


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


def gather_head_outputs(out: torch.Tensor, group=None) -> torch.Tensor:
    """Outputs [B][H/world][D] of every rank's kv-head shard
    (workloads.shard_kv_heads) gathered into [B][H][D], rank r's query heads
    at [r*H/world, (r+1)*H/world).  The partition itself needs no exchange:
    each rank's outputs are final for its heads; this assembles them (for a
    caller that wants every head on every rank, and for the tests)."""
    world = dist.get_world_size(group)
    out = out.contiguous()
    parts = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(parts, out, group=group)
    return torch.cat(parts, dim=1)


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


class PeerExchange:
    """Exchange buffers of a split-context decode, one per rank, mapped by
    every other rank through CUDA IPC (cottus_peer_exchange_*).  Collective
    at construction (handles all-gathered over `group`).  `wait_cycles`
    sets the combine's wait limit in GPU clock cycles (default about 1 s).
    `absent` lists ranks that take no part (their handles are replaced by
    all-zero ones): every combine then waits out its limit and reports
    COTTUS_STATUS_TIMEOUT, which is how failure handling is exercised."""

    def __init__(self, batch: int, num_heads: int, head_dim: int, group=None, wait_cycles: int | None = None,
                 absent=()):
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        handle = (C.c_uint8 * 64)()
        h = C.c_void_p()
        check(lib().cottus_peer_exchange_create(world, rank, batch, num_heads, head_dim, C.byref(h), handle))
        self._h = h
        dev = torch.device("cuda", torch.cuda.current_device())
        mine = torch.tensor(bytearray(bytes(handle)), dtype=torch.uint8, device=dev)
        every = torch.empty(world * 64, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(every, mine, group=group)
        blob = np.ascontiguousarray(every.cpu().numpy())
        self._open(blob, absent, rank, wait_cycles)
        dist.barrier(group=group)  # every rank mapped every buffer before first use
        self.group, self._collective = group, True

    @classmethod
    def alone(cls, world: int, rank: int, batch: int, num_heads: int, head_dim: int, wait_cycles: int | None = None):
        """This process as rank `rank` of `world` ranks of which no other takes
        part (no process group needed): every combine waits out its limit and
        reports COTTUS_STATUS_TIMEOUT (world 1: an ordinary one-rank split)."""
        self = cls.__new__(cls)
        handle = (C.c_uint8 * 64)()
        h = C.c_void_p()
        check(lib().cottus_peer_exchange_create(world, rank, batch, num_heads, head_dim, C.byref(h), handle))
        self._h = h
        self.group, self._collective = None, False
        self._open(np.zeros(world * 64, np.uint8), range(world), rank, wait_cycles)
        return self

    def _open(self, blob, absent, rank, wait_cycles):
        blob = blob.copy()
        for r in absent:
            if r != rank:
                blob[r * 64:(r + 1) * 64] = 0
        try:
            check(lib().cottus_peer_exchange_open(self._h, blob.ctypes.data))
            if wait_cycles is not None:
                check(lib().cottus_peer_exchange_set_wait_cycles(self._h, int(wait_cycles)))
        except Exception:
            lib().cottus_peer_exchange_destroy(self._h)
            self._h = None
            raise

    def close(self):
        """Collective (when made with a group): every rank stops using the
        exchange, then frees it."""
        if self._h:
            if self._collective:
                dist.barrier(group=self.group)
            lib().cottus_peer_exchange_destroy(self._h)
            self._h = None


def split_kv_decode_peer(query, kv_pool, block_table, context_lens, exchange: PeerExchange, *, num_kv_heads,
                         head_dim, block_size, num_layers=1, layer=0, num_physical_blocks=None,
                         out_dtype=torch.float16, out=None, lse_out=None, status=None, stream=None):
    """split_kv_decode with the exchange through peer memory, no collective
    call: on the tensor-core path (grouped queries) one decode kernel per
    rank that also merges every rank's partials; otherwise a decode kernel
    and a combine kernel per rank."""
    B, H, D = query.shape
    if out is None:
        out = torch.empty((B, H, D), dtype=out_dtype, device=query.device)
    p = make_decode_params(out, query, kv_pool, block_table, context_lens, num_kv_heads=num_kv_heads,
                           head_dim=head_dim, block_size=block_size, num_layers=num_layers, layer=layer,
                           num_physical_blocks=num_physical_blocks, lse_out=lse_out, status=status)
    need = lib().cottus_split_decode_workspace_size(C.byref(p))
    if need:
        ws = workspace(need, query.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().cottus_split_decode(C.byref(p), exchange._h, _stream(stream)))
    return out
