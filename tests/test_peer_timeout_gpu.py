"""Failure detection of the split-context exchange (cottus_split_decode) on
one GPU.  Rank 1 of a two-rank exchange never takes part (its handle is
all-zero, so its flag is a word on this GPU that nothing raises): rank 0's
combine kernel must give up after its wait limit, set
COTTUS_STATUS_TIMEOUT, leave the output untouched and return, and the
exchange must then refuse every later step at once.  A new exchange then
decodes correctly (checked against the oracle, pagedAttentionCPU restated).
The reference has no device-side failure path: it throws and frees
(engine.cpp:97-104)."""
import time

import pytest
import torch

import cottus_b200 as cb
from cottus_b200 import parallel
from cottus_b200 import workloads as W
from helpers import TOL_F16, max_abs, oracle_outputs

pytestmark = pytest.mark.gpu

TIMEOUT = 0x8


def _shard(w, rank, world, dev):
    s = W.shard_long_context(w, rank, world)
    t = W.device_tensors(s, dev, pool_blocks=s.meta["pool_range"])
    t["block_table"] = torch.from_numpy(s.block_table).to(dev)
    t["context_lens"] = torch.from_numpy(s.ctx).to(dev)
    return s, t


def _step(w, s, t, ex, out, status):
    parallel.split_kv_decode_peer(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], ex,
                                  num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, num_physical_blocks=s.num_blocks,
                                  out_dtype=torch.float16, out=out, status=status)


def test_absent_peer_times_out_and_exchange_stays_broken(oracle):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = W.long_ctx_70b(seed=91, B=2, context=4096)
    s, t = _shard(w, 0, 2, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.full((w.B, w.H, w.D), 7.0, dtype=torch.float16, device=dev)

    # a short limit (2e6 cycles, about 1 ms at the boost clock) for the wait that must run out
    ex = parallel.PeerExchange.alone(2, 0, w.B, w.H, w.D, wait_cycles=2_000_000)
    try:
        _step(w, s, t, ex, out, status)
        torch.cuda.synchronize(dev)
        assert int(status.item()) & TIMEOUT, "the combine's wait for the absent rank did not run out"
        assert bool(torch.all(out == 7.0)), "a combine that timed out wrote output"

        # broken from now on: with the default limit (about a second) restored, the next
        # step must still report the timeout, at once and without writing
        cb._lib.check(cb._lib.lib().cottus_peer_exchange_set_wait_cycles(ex._h, 2_000_000_000))
        status.zero_()
        out2 = torch.full_like(out, 5.0)
        t0 = time.perf_counter()
        _step(w, s, t, ex, out2, status)
        torch.cuda.synchronize(dev)
        elapsed = time.perf_counter() - t0
        assert int(status.item()) & TIMEOUT
        assert bool(torch.all(out2 == 5.0))
        assert elapsed < 0.5, f"a broken exchange waited {elapsed:.2f} s"
    finally:
        ex.close()

    # recovery: a new exchange (here one rank over the whole context) decodes correctly
    full = W.device_tensors(w, dev)
    ex1 = parallel.PeerExchange.alone(1, 0, w.B, w.H, w.D)
    try:
        status.zero_()
        out3 = torch.empty_like(out)
        parallel.split_kv_decode_peer(full["query"], full["kv_pool"], full["block_table"], full["context_lens"], ex1,
                                      num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                      num_physical_blocks=w.num_blocks, out_dtype=torch.float16, out=out3,
                                      status=status)
        torch.cuda.synchronize(dev)
        assert int(status.item()) == 0
        ref = oracle_outputs(oracle, w, full, range(w.B))
        assert max_abs(out3, ref) <= TOL_F16
    finally:
        ex1.close()


def test_wait_limit_rejects_out_of_range_values():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with pytest.raises(cb.CottusError):
        parallel.PeerExchange.alone(2, 0, 1, 8, 64, wait_cycles=10)
    ex = parallel.PeerExchange.alone(2, 0, 1, 8, 64)
    try:
        assert cb._lib.lib().cottus_peer_exchange_set_wait_cycles(ex._h, 10 ** 13) != 0
        assert cb._lib.lib().cottus_peer_exchange_set_wait_cycles(ex._h, 10 ** 6) == 0
    finally:
        ex.close()
