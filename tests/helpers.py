"""Shared test helpers: run the oracle on (a subset of) a device workload,
and a plain torch fp32 attention reference for full-size checks."""
from __future__ import annotations

import numpy as np
import torch

from cottus_b200.workloads import host_subpool  # noqa: F401  (re-exported for tests)

TOL_F32 = 1e-5   # max-abs error bound for fp32 outputs
TOL_F16 = 2e-3   # max-abs error bound for fp16 outputs


def tol_for(dtype) -> float:
    return TOL_F32 if dtype == torch.float32 else TOL_F16


def oracle_outputs(oracle, w, t, seqs, query=None):
    """Oracle (C restatement of pagedAttentionCPU) outputs for `seqs`."""
    seqs = list(seqs)
    sub, bt, ctx = host_subpool(w, t["kv_pool"], seqs)
    q = (t["query"] if query is None else query)[seqs].float().cpu().numpy()
    return oracle.paged_attention_batch(q, sub, bt, ctx, w.layer, w.H, w.Hkv, w.D, w.bs, w.L)


def torch_reference(w, t, query=None, seqs=None):
    """fp32 attention on the GPU from a dense torch gather of the pages
    (GQA groups kept as a separate axis, so K/V are not replicated)."""
    pool = t["kv_pool"].view(-1, w.L, 2, w.bs, w.Hkv, w.D)[:, w.layer]
    q = (t["query"] if query is None else query).float()
    G = w.H // w.Hkv
    scale = 1.0 / np.sqrt(w.D)
    outs = []
    seqs = range(w.B) if seqs is None else seqs
    bt = torch.from_numpy(w.block_table).to(pool.device).long()
    for b in seqs:
        n = int(w.ctx[b])
        if n == 0:
            outs.append(torch.zeros(w.H, w.D, device=pool.device))
            continue
        pages = (n + w.bs - 1) // w.bs
        blk = pool.index_select(0, bt[b, :pages])                  # [pages, 2, bs, Hkv, D]
        k = blk[:, 0].reshape(-1, w.Hkv, w.D)[:n].view(torch.float16).float()
        v = blk[:, 1].reshape(-1, w.Hkv, w.D)[:n].view(torch.float16).float()
        qg = q[b].view(w.Hkv, G, w.D)
        s = torch.einsum("kgd,nkd->kgn", qg, k) * scale
        p = torch.softmax(s, dim=-1)
        outs.append(torch.einsum("kgn,nkd->kgd", p, v).reshape(w.H, w.D))
    return torch.stack(outs)


def max_abs(a, b) -> float:
    a = a.float().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float32)
    b = b.float().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float32)
    return float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64)))) if a.size else 0.0


class BatchReplica:
    """Host model of the batched decode-step driver, built on the oracle's
    allocator (the restated reference BlockAllocator): Engine::generate's
    bookkeeping (engine.cpp:52-95) for many sequences, rows in addition
    order, a released row taken by the last one."""

    def __init__(self, oracle, num_blocks, block_size, max_batch, max_blocks):
        self.alloc = oracle.allocator(num_blocks, block_size)
        self.bs, self.max_batch, self.max_blocks = block_size, max_batch, max_blocks
        self.rows = []   # sequence ids in row order
        self.seq = {}    # id -> [position, blocks]

    def add(self, sid):
        self.rows.append(sid)
        self.seq[sid] = [0, []]

    def release(self, sid):
        for blk in self.seq[sid][1]:  # allocation order (engine.cpp:88-90)
            assert self.alloc.free(blk) == 0
        r = self.rows.index(sid)
        last = self.rows.pop()
        if last != sid:
            self.rows[r] = last
        del self.seq[sid]

    def begin_step(self):
        """True if the step's blocks were allocated, False (nothing changed) on exhaustion."""
        grown = []
        for sid in self.rows:
            pos, blocks = self.seq[sid]
            if pos % self.bs == 0:
                blk = self.alloc.alloc()
                if blk < 0:
                    for g in reversed(grown):
                        assert self.alloc.free(self.seq[g][1].pop()) == 0
                    return False
                blocks.append(blk)
                grown.append(sid)
        return True

    def end_step(self):
        for sid in self.rows:
            self.seq[sid][0] += 1
