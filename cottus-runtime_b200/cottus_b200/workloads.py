"""Seeded synthetic decode workloads with the shapes of the five reference
configurations (no public dataset is involved; all inputs are synthetic).

  tinyllama_f32   H32/Hkv4/D64 fp32, B4, context U[128,512], pool = seeded
                  permutation of the needed blocks
  llama3_8b       H32/Hkv8/D128 fp16, B64, context 2048, 8192-block pool,
                  seeded shuffle
  ragged_mha      H32/Hkv32/D128 fp16, B256, context log-uniform [16,8192],
                  block table from a seeded 10k-op alloc/free churn on the
                  BlockAllocator, then interleaved per-sequence allocation
  long_ctx_70b    H64/Hkv8/D128 fp16, B8, context 131072 (split-KV across
                  GPUs by contiguous page ranges)
  fused_tinyllama H32/Hkv4/D64 fp16, B32, new-token positions U[0,4095],
                  RoPE theta 1e4; the new token's block is freshly
                  allocated when position % 16 == 0

KV values are fp32 N(0,1) draws stored through the reference's truncating
fp16 encoder (what the reference pipeline writes into its cache); they are
generated on the target device from per-segment seeds so that any shard of
the pool can be rebuilt independently.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

BLOCK = 16
N_SEGMENTS = 8  # page segments of long_ctx_70b (finest split across GPUs)


@dataclass
class Workload:
    name: str
    H: int
    Hkv: int
    D: int
    bs: int
    L: int
    layer: int
    q_dtype: torch.dtype
    out_dtype: torch.dtype
    ctx: np.ndarray            # int32 [B] tokens attended per sequence
    block_table: np.ndarray    # int32 [B, max_blocks]
    num_blocks: int
    seed: int
    positions: np.ndarray | None = None  # fused: new-token position (ctx = positions + 1)
    theta: float = 10000.0
    segment_blocks: int = 0   # >0: pool is generated per contiguous segment of this many blocks
    meta: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return len(self.ctx)

    @property
    def fused(self) -> bool:
        return self.positions is not None

    def block_elems(self) -> int:
        return 2 * self.L * self.bs * self.Hkv * self.D

    def kv_bytes(self) -> int:
        """KV bytes attention must read once (K and V rows of every context token)."""
        return int(np.sum(self.ctx.astype(np.int64))) * 2 * self.Hkv * self.D * 2

    def io_bytes(self) -> int:
        qb = 4 if self.q_dtype == torch.float32 else 2
        ob = 4 if self.out_dtype == torch.float32 else 2
        n = self.B * self.H * self.D
        extra = self.block_table.size * 4 + self.B * 4
        if self.fused:
            extra += 2 * self.B * self.Hkv * self.D * (qb + 2)  # new k, v read; encoded k, v written
            extra += self.B * (self.D // 2) * 8                 # (cos, sin) rows
        return n * qb + n * ob + extra


# -- device tensors -------------------------------------------------------------------

def trunc_f16_bits(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> fp16 bit patterns by truncation (generic_transformer.cpp:255-262), as int16."""
    b = x.contiguous().view(torch.int32)
    sign = (b >> 16) & 0x8000
    e = ((b >> 23) & 0xFF) - 112
    m = (b >> 13) & 0x3FF
    r = torch.where(e <= 0, sign, torch.where(e >= 31, sign | 0x7C00, sign | (e.clamp(0, 31) << 10) | m))
    return r.to(torch.int16)


def f16_bits_to_f32(h: torch.Tensor) -> torch.Tensor:
    return h.view(torch.float16).float()


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def fill_pool(pool: torch.Tensor, w: Workload, first_block: int = 0, chunk_elems: int = 1 << 26) -> None:
    """Fills pool (int16, [n_blocks * block_elems]) with encoded N(0,1) values
    for global blocks [first_block, first_block + n_blocks).  Each segment of
    w.segment_blocks blocks (the whole pool when 0) has its own generator, so
    a segment-aligned shard rebuilds exactly its part of the global pool."""
    per = w.block_elems()
    n_blocks = pool.numel() // per
    seg = w.segment_blocks or n_blocks
    if first_block % seg or n_blocks % seg:
        raise ValueError("pool shard must be aligned to generator segments")
    for i in range(n_blocks // seg):
        s = first_block // seg + i
        g = _gen(w.seed * 1000003 + 7919 * s, pool.device)
        base = i * seg * per
        for off in range(0, seg * per, chunk_elems):
            n = min(chunk_elems, seg * per - off)
            x = torch.randn(n, generator=g, device=pool.device, dtype=torch.float32)
            pool[base + off: base + off + n] = trunc_f16_bits(x)


def device_tensors(w: Workload, device, pool_blocks: tuple[int, int] | None = None) -> dict:
    """Builds the step's device inputs.  pool_blocks=(first, count) restricts
    the pool to a contiguous range of global blocks (block ids in the table
    must then be rebased by the caller)."""
    first, count = pool_blocks if pool_blocks else (0, w.num_blocks)
    per = w.block_elems()
    pool = torch.empty(count * per, dtype=torch.int16, device=device)
    fill_pool(pool, w, first_block=first)
    g = _gen(w.seed * 31 + 5, device)
    qf = torch.randn((w.B, w.H, w.D), generator=g, device=device, dtype=torch.float32)
    t = dict(kv_pool=pool,
             block_table=torch.from_numpy(w.block_table).to(device),
             context_lens=torch.from_numpy(w.ctx).to(device))
    if w.q_dtype == torch.float16:
        t["query"] = qf.half()
    else:
        t["query"] = qf
    if w.fused:
        t["key"] = torch.randn((w.B, w.Hkv, w.D), generator=g, device=device).to(w.q_dtype)
        t["value"] = torch.randn((w.B, w.Hkv, w.D), generator=g, device=device).to(w.q_dtype)
        t["positions"] = torch.from_numpy(w.positions).to(device)
    return t


# -- block tables ---------------------------------------------------------------------

def _pages(ctx) -> np.ndarray:
    return (np.asarray(ctx, np.int64) + BLOCK - 1) // BLOCK


def _permuted_tables(rng, ctx, extra_blocks=0):
    pages = _pages(ctx)
    total = int(pages.sum()) + extra_blocks
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(ctx), max(int(pages.max()), 1)), np.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n]
        off += n
    return bt, total


def churn_tables(rng, ctx, n_ops=10000, slack=4096, allocator_cls=None):
    """Seeded alloc/free churn on a LIFO BlockAllocator, then interleaved
    allocation of every sequence's pages (one page per sequence per round,
    as concurrent decodes grow).  Returns (block_table, pool_size)."""
    if allocator_cls is None:
        from .ops import BlockAllocator as allocator_cls
    pages = _pages(ctx)
    total = int(pages.sum()) + slack
    a = allocator_cls(total, BLOCK)
    live = []
    for _ in range(n_ops):
        if not live or (len(live) < slack and rng.random() < 0.5):
            live.append(a.allocate())
        else:
            k = int(rng.integers(0, len(live)))
            a.free(live[k])
            live[k] = live[-1]
            live.pop()
    bt = np.zeros((len(ctx), max(int(pages.max()), 1)), np.int32)
    for r in range(int(pages.max())):
        for b in np.nonzero(pages > r)[0]:
            bt[b, r] = a.allocate()
    return bt, total


# -- the five configurations ----------------------------------------------------------

def tinyllama_f32(seed=1, B=4, lo=128, hi=512):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(lo, hi + 1, B).astype(np.int32)
    bt, total = _permuted_tables(rng, ctx, extra_blocks=3)
    return Workload("tinyllama_f32", 32, 4, 64, BLOCK, 1, 0, torch.float32, torch.float32, ctx, bt, total, seed)


def llama3_8b(seed=2, B=64, context=2048, pool=None):
    rng = np.random.default_rng(seed)
    ctx = np.full(B, context, np.int32)
    pages = int(_pages(ctx).sum())
    bt, total = _permuted_tables(rng, ctx, extra_blocks=(pool - pages) if pool else 0)
    return Workload("llama3_8b", 32, 8, 128, BLOCK, 1, 0, torch.float16, torch.float16, ctx, bt, total, seed)


def ragged_mha(seed=3, B=256, lo=16, hi=8192, n_ops=10000, allocator_cls=None):
    rng = np.random.default_rng(seed)
    ctx = np.rint(np.exp(rng.uniform(math.log(lo), math.log(hi), B))).astype(np.int32)
    bt, total = churn_tables(rng, ctx, n_ops=n_ops, allocator_cls=allocator_cls)
    return Workload("ragged_mha", 32, 32, 128, BLOCK, 1, 0, torch.float16, torch.float16, ctx, bt, total, seed)


def long_ctx_70b(seed=4, B=8, context=131072):
    """Pages of every sequence are cut into N_SEGMENTS contiguous segments;
    segment s uses physical ids [s*B*P/8, (s+1)*B*P/8) (shuffled inside), so
    any 1/2/4/8-way split of the pages is a contiguous range of the pool."""
    rng = np.random.default_rng(seed)
    ctx = np.full(B, context, np.int32)
    P = int(_pages(ctx)[0])
    assert P % N_SEGMENTS == 0
    ps = P // N_SEGMENTS
    seg_blocks = B * ps
    bt = np.zeros((B, P), np.int32)
    for s in range(N_SEGMENTS):
        perm = (rng.permutation(seg_blocks) + s * seg_blocks).astype(np.int32)
        bt[:, s * ps:(s + 1) * ps] = perm.reshape(B, ps)
    w = Workload("long_ctx_70b", 64, 8, 128, BLOCK, 1, 0, torch.float16, torch.float16, ctx, bt, B * P, seed,
                 segment_blocks=seg_blocks)
    w.meta["pages_per_segment"] = ps
    return w


def fused_tinyllama(seed=5, B=32, max_pos=4095, allocator_cls=None):
    """Engine-style allocation: blocks for positions [0, pos) are allocated
    interleaved across sequences; the new token's block is allocated at the
    step itself when pos % 16 == 0 (engine.cpp:73-77)."""
    if allocator_cls is None:
        from .ops import BlockAllocator as allocator_cls
    rng = np.random.default_rng(seed)
    pos = rng.integers(0, max_pos + 1, B).astype(np.int32)
    ctx = pos + 1
    pages_prefix = (pos.astype(np.int64) + BLOCK - 1) // BLOCK  # blocks holding tokens [0, pos)
    pages = _pages(ctx)
    total = int(pages.sum()) + 8
    a = allocator_cls(total, BLOCK)
    bt = np.zeros((B, int(pages.max())), np.int32)
    for r in range(int(pages_prefix.max(initial=0))):
        for b in np.nonzero(pages_prefix > r)[0]:
            bt[b, r] = a.allocate()
    for b in np.nonzero(pos % BLOCK == 0)[0]:
        bt[b, pos[b] // BLOCK] = a.allocate()
    w = Workload("fused_tinyllama", 32, 4, 64, BLOCK, 1, 0, torch.float16, torch.float16, ctx, bt, total, seed,
                 positions=pos)
    return w


BUILDERS = {
    "tinyllama_f32": tinyllama_f32,
    "llama3_8b": llama3_8b,
    "ragged_mha": ragged_mha,
    "long_ctx_70b": long_ctx_70b,
    "fused_tinyllama": fused_tinyllama,
}


def shard_long_context(w: Workload, rank: int, world: int) -> Workload:
    """Rank `rank` of `world` keeps pages [rank*P/world, (rank+1)*P/world) of
    every sequence; block ids are rebased to its local pool, which is the
    contiguous global range returned in meta['pool_range']."""
    assert N_SEGMENTS % world == 0
    P = w.block_table.shape[1]
    p0, p1 = rank * P // world, (rank + 1) * P // world
    seg_per_rank = N_SEGMENTS // world
    first = rank * seg_per_rank * w.segment_blocks
    count = seg_per_rank * w.segment_blocks
    bt = np.ascontiguousarray(w.block_table[:, p0:p1] - first).astype(np.int32)
    ctx = np.clip(w.ctx - p0 * w.bs, 0, (p1 - p0) * w.bs).astype(np.int32)
    s = Workload(w.name, w.H, w.Hkv, w.D, w.bs, w.L, w.layer, w.q_dtype, torch.float32, ctx, bt, count, w.seed,
                 segment_blocks=w.segment_blocks)
    s.meta = dict(w.meta, pool_range=(first, count), page_range=(p0, p1))
    return s


def shard_kv_heads(w: Workload, t: dict, rank: int, world: int) -> tuple[Workload, dict]:
    """Rank `rank` of `world` keeps kv heads [rank*Hkv/world, (rank+1)*Hkv/world)
    of every page of the pool in t, and the query heads of their GQA groups
    (h * Hkv / H falls in the rank's range, paged_attention_cpu.cpp:48): the
    attention of those query heads is complete on the rank, so no partial
    is exchanged.  Returns the shard's workload (H/world query heads,
    Hkv/world kv heads; same block table, lengths and block ids) and its
    device tensors: the pool [blocks][L][K|V][bs][Hkv/world][D] and the
    query [B][H/world][D], both contiguous copies."""
    if w.Hkv % world or w.H % w.Hkv:
        raise ValueError("kv heads must divide evenly over the ranks, query heads over the kv heads")
    if w.fused:
        raise ValueError("a fused step's new k and v are not sharded by this helper")
    hk, G = w.Hkv // world, w.H // w.Hkv
    h0 = rank * hk
    pool = t["kv_pool"].view(w.num_blocks, w.L, 2, w.bs, w.Hkv, w.D)[:, :, :, :, h0:h0 + hk].contiguous()
    s = Workload(w.name, w.H // world, hk, w.D, w.bs, w.L, w.layer, w.q_dtype, w.out_dtype, w.ctx, w.block_table,
                 w.num_blocks, w.seed, positions=w.positions, theta=w.theta)
    s.meta = dict(w.meta, kv_heads=(h0, h0 + hk), query_heads=(h0 * G, (h0 + hk) * G))
    ts = dict(t, kv_pool=pool.view(-1), query=t["query"][:, h0 * G:(h0 + hk) * G].contiguous())
    return s, ts


def host_subpool(w: Workload, kv_pool: torch.Tensor, seqs):
    """Copies the blocks used by `seqs` to the host and renumbers them densely;
    returns (pool uint16, block table int32 [len(seqs), max_blocks], ctx)."""
    per = w.block_elems()
    pages = (w.ctx[seqs].astype(np.int64) + w.bs - 1) // w.bs
    maxb = max(int(pages.max(initial=0)), 1)
    ids = np.unique(np.concatenate([w.block_table[b, :n] for b, n in zip(seqs, pages)] + [np.zeros(0, np.int32)]))
    lookup = np.zeros(max(int(ids.max(initial=0)) + 1, 1), np.int64)
    lookup[ids] = np.arange(len(ids))
    bt = np.zeros((len(seqs), maxb), np.int32)
    for i, (b, n) in enumerate(zip(seqs, pages)):
        bt[i, :n] = lookup[w.block_table[b, :n]]
    if len(ids):
        idx = torch.from_numpy(ids.astype(np.int64)).to(kv_pool.device)
        sub = kv_pool.view(-1, per).index_select(0, idx).cpu().numpy().view(np.uint16).ravel()
    else:
        sub = np.zeros(per, np.uint16)
    return sub, bt, w.ctx[seqs].astype(np.int32)
