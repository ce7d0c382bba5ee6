"""World-size-2 host logic of the multi-GPU long-context paths on CPU
(gloo), checked against the un-split oracle:
  * split-KV: page-range sharding, the all-gather of (normalised partial,
    lse) pairs and the log-sum-exp merge;
  * kv-head partition: each rank keeps some kv heads of every page and
    their query heads, and its outputs are final for those heads (gathered
    here only to compare), bit for bit the oracle's.
The per-rank results come from the oracle, so this runs without a GPU; the
device kernels are tested on the GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _small_long_ctx():
    from cottus_b200 import workloads as W

    return W.long_ctx_70b(seed=61, B=2, context=2048)


def _partial(oracle, w, s, pool_all):
    """Oracle output + lse over one shard (lse from the oracle's own scores)."""
    from cases import fp16_bits_to_f32

    per = w.block_elems()
    first, count = s.meta["pool_range"]
    pool = pool_all[first * per:(first + count) * per]
    q = _query(w)
    out = np.zeros((w.B, w.H, w.D), np.float32)
    lse = np.full((w.B, w.H), -np.inf, np.float32)
    G = w.H // w.Hkv
    for b in range(w.B):
        n = int(s.ctx[b])
        if n == 0:
            continue
        nb = (n + 15) // 16
        out[b] = oracle.paged_attention(q[b], pool, s.block_table[b, :nb], n, 0, w.H, w.Hkv, w.D, 16, 1)
        k, _ = oracle.gather_kv(pool, s.block_table[b, :nb], n, 0, w.Hkv, w.D, 16, 1)
        kf = fp16_bits_to_f32(k).astype(np.float64)
        for h in range(w.H):
            sc = kf[:, h // G] @ q[b, h].astype(np.float64) / np.sqrt(w.D)
            m = sc.max()
            lse[b, h] = m + np.log(np.exp(sc - m).sum())
    return out, lse


def _query(w):
    rng = np.random.default_rng(w.seed + 99)
    from cases import fp16_bits_to_f32, fp32_to_fp16_trunc

    return fp16_bits_to_f32(fp32_to_fp16_trunc(rng.standard_normal((w.B, w.H, w.D), dtype=np.float32)))


def _pool(w):
    from cottus_b200 import workloads as W

    pool = torch.empty(w.num_blocks * w.block_elems(), dtype=torch.int16)
    W.fill_pool(pool, w)
    return pool.numpy().view(np.uint16)


def lse_merge_host(parts, lses):
    """Reference log-sum-exp merge in float64 (test-side)."""
    m = lses.max(axis=0)
    wts = np.exp(lses.astype(np.float64) - m)
    return ((wts[..., None] * parts).sum(0) / wts.sum(0)[..., None]).astype(np.float32)


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    for p in (root, root / "cottus-runtime_b200", root / "tests" / "golden", root / "tests"):
        sys.path.insert(0, str(p))
    from oracle.oracle import Oracle

    from cottus_b200 import parallel
    from cottus_b200 import workloads as W

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _small_long_ctx()
        s = W.shard_long_context(w, rank, world)
        oracle = Oracle()
        out, lse = _partial(oracle, w, s, _pool(w))
        parts, lses = parallel.all_gather_partials(torch.from_numpy(out), torch.from_numpy(lse))
        merged = lse_merge_host(parts.numpy(), lses.numpy())
        result_q.put((rank, merged))
    finally:
        dist.destroy_process_group()


def test_split_kv_two_ranks_gloo():
    from oracle.oracle import Oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, m = q.get(timeout=240)
        res[r] = m
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = _small_long_ctx()
    oracle = Oracle()
    pool = _pool(w)
    qv = _query(w)
    ref = np.stack([oracle.paged_attention(qv[b], pool, w.block_table[b], int(w.ctx[b]), 0, w.H, w.Hkv, w.D, 16, 1)
                    for b in range(w.B)])
    for r in range(world):
        assert np.max(np.abs(res[r] - ref)) < 1e-5
    np.testing.assert_array_equal(res[0], res[1])


def test_shard_plan_covers_every_page_once():
    from cottus_b200 import workloads as W

    w = W.long_ctx_70b(seed=3, B=3, context=4096)
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            s = W.shard_long_context(w, r, world)
            first, count = s.meta["pool_range"]
            assert s.block_table.min() >= 0 and s.block_table.max() < count
            seen.append(s.block_table + first)
            assert int(s.ctx.sum()) == int(w.ctx.sum()) // world
        np.testing.assert_array_equal(np.concatenate(seen, axis=1), w.block_table)


def _heads_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    for p in (root, root / "cottus-runtime_b200", root / "tests" / "golden", root / "tests"):
        sys.path.insert(0, str(p))
    from helpers import oracle_outputs
    from oracle.oracle import Oracle

    from cottus_b200 import parallel
    from cottus_b200 import workloads as W

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _small_long_ctx()
        t = W.device_tensors(w, "cpu")
        s, ts = W.shard_kv_heads(w, t, rank, world)
        mine = torch.from_numpy(oracle_outputs(Oracle(), s, ts, range(s.B)))
        result_q.put((rank, parallel.gather_head_outputs(mine).numpy()))
    finally:
        dist.destroy_process_group()


def test_kv_head_partition_two_ranks_gloo():
    from helpers import oracle_outputs
    from oracle.oracle import Oracle

    from cottus_b200 import workloads as W

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_heads_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, m = q.get(timeout=240)
        res[r] = m
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = _small_long_ctx()
    full = oracle_outputs(Oracle(), w, W.device_tensors(w, "cpu"), range(w.B))
    for r in range(world):
        np.testing.assert_array_equal(res[r].view(np.uint32), full.view(np.uint32))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_shards_are_slices_of_the_pool(oracle, world):
    """Each shard's pool holds exactly its kv heads' rows of every page, its
    query exactly its query heads, and the oracle over the shard gives the
    un-split oracle's rows of those heads bit for bit."""
    from helpers import oracle_outputs

    from cottus_b200 import workloads as W

    w = _small_long_ctx()
    t = W.device_tensors(w, "cpu")
    full = oracle_outputs(oracle, w, t, range(w.B))
    view = t["kv_pool"].view(w.num_blocks, w.L, 2, w.bs, w.Hkv, w.D)
    for rank in range(world):
        s, ts = W.shard_kv_heads(w, t, rank, world)
        h0, h1 = s.meta["kv_heads"]
        q0, q1 = s.meta["query_heads"]
        assert (s.H, s.Hkv) == (w.H // world, w.Hkv // world)
        assert torch.equal(ts["kv_pool"].view(w.num_blocks, w.L, 2, w.bs, s.Hkv, w.D), view[:, :, :, :, h0:h1])
        assert torch.equal(ts["query"], t["query"][:, q0:q1])
        got = oracle_outputs(oracle, s, ts, range(w.B))
        np.testing.assert_array_equal(got.view(np.uint32), full[:, q0:q1].view(np.uint32))
