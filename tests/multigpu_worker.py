"""Worker for tests/test_multigpu_nccl.py (one process per GPU, launched by
torch.distributed.run): the long-context split-KV decode across GPUs.

Every rank holds one contiguous page range of every sequence.

mode "parity":
  Path 1 computes LSE partials with cottus_paged_decode, all-gathers them
  over NCCL and merges them with cottus_lse_combine.  Path 2
  (cottus_split_decode) exchanges the same partials through peer memory:
  the decode kernel flags completion to every rank, the combine kernel
  reads the other ranks' partials over NVLink.  Path 2 runs many steps in
  a row with no barrier between steps and a random host delay before each
  step on each rank, so ranks run up to a step ahead of each other; every
  step must give the bits of path 1 and no timeout.  Rank 0 compares the
  merged output with the oracle (pagedAttentionCPU restated) on one
  sequence and with a torch fp32 attention on every sequence, both over
  the whole, un-split context.

mode "skip":
  Rank 1 skips one step.  Rank 0's combine must time out (short wait limit)
  with its output untouched; the next step must fail at once on both ranks
  (the exchange is broken everywhere); after every rank recreates the
  exchange, a step is correct again.

mode "heads":
  The kv-head partition: every rank keeps Hkv/world kv heads of every page
  and the query heads of their groups, and decodes them with
  cottus_paged_decode; its outputs are final for those heads (no
  exchange).  The ranks' outputs are gathered only to compare them with
  the oracle on one sequence and with a torch fp32 attention on all.

Rank 0 writes the results as JSON."""
import json
import os
import random
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "cottus-runtime_b200", ROOT / "tests"):
    sys.path.insert(0, str(p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

TIMEOUT = 0x8


def _setup(dev, rank, world, B, context):
    from cottus_b200 import workloads as W

    w = W.long_ctx_70b(seed=81, B=B, context=context)
    s = W.shard_long_context(w, rank, world)
    t = W.device_tensors(s, dev, pool_blocks=s.meta["pool_range"])
    t["block_table"] = torch.from_numpy(s.block_table).to(dev)
    t["context_lens"] = torch.from_numpy(s.ctx).to(dev)
    return w, s, t


def _peer_step(parallel, w, s, t, ex, out, status):
    return parallel.split_kv_decode_peer(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], ex,
                                         num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                         num_physical_blocks=s.num_blocks, out_dtype=torch.float16, out=out,
                                         status=status)


def parity(out_path, rank, world, dev):
    from cottus_b200 import parallel
    from cottus_b200 import workloads as W
    from helpers import max_abs, oracle_outputs, torch_reference
    from oracle.oracle import Oracle

    w, s, t = _setup(dev, rank, world, B=3, context=32768)
    merged = parallel.split_kv_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"],
                                      num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                      num_physical_blocks=s.num_blocks, out_dtype=torch.float16)
    torch.cuda.synchronize(dev)
    ex = parallel.PeerExchange(w.B, w.H, w.D)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rng = random.Random(1234 + rank)
    steps, peer_equal = 40, True
    outs = [torch.empty_like(merged) for _ in range(2)]
    for i in range(steps):
        time.sleep(rng.uniform(0.0, 0.002))  # host skew: ranks drift up to a step apart
        _peer_step(parallel, w, s, t, ex, outs[i % 2], status)
        if i % 2 == 1:
            torch.cuda.synchronize(dev)
            peer_equal = peer_equal and torch.equal(outs[0], merged) and torch.equal(outs[1], merged)
    torch.cuda.synchronize(dev)
    ex.close()
    peer_status = int(status.item())
    gathered = [torch.empty_like(merged) for _ in range(world)]
    dist.all_gather(gathered, merged)
    flags = torch.tensor([int(peer_equal), peer_status], dtype=torch.int64, device=dev)
    every = [torch.empty_like(flags) for _ in range(world)]
    dist.all_gather(every, flags)
    if rank == 0:
        full = W.device_tensors(w, dev)
        err_torch = max_abs(merged, torch_reference(w, full))
        err_oracle = max_abs(merged[1:2], oracle_outputs(Oracle(), w, full, [1]))
        Path(out_path).write_text(json.dumps({
            "max_abs_torch_fp32": err_torch, "max_abs_oracle": err_oracle, "oracle_sequences": [1],
            "ranks_agree": all(torch.equal(g, gathered[0]) for g in gathered), "world": world,
            "peer_steps": steps, "peer_equal_all_ranks": all(int(f[0]) == 1 for f in every),
            "peer_status": [int(f[1]) for f in every]}))


def skip(out_path, rank, world, dev):
    from cottus_b200 import parallel
    from cottus_b200 import workloads as W
    from helpers import max_abs, oracle_outputs
    from oracle.oracle import Oracle

    w, s, t = _setup(dev, rank, world, B=2, context=8192)
    wait = 20_000_000  # about 10 ms at the boost clock
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    record = []

    def gather_status():
        x = torch.tensor([int(status.item())], dtype=torch.int64, device=dev)
        every = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(every, x)
        return [int(e.item()) for e in every]

    ex = parallel.PeerExchange(w.B, w.H, w.D, wait_cycles=wait)
    out = torch.empty((w.B, w.H, w.D), dtype=torch.float16, device=dev)
    # step 0: every rank takes part
    _peer_step(parallel, w, s, t, ex, out, status)
    torch.cuda.synchronize(dev)
    record.append(gather_status())
    # step 1: rank 1 skips it; the others' combines run out of time and leave their output alone
    status.zero_()
    out.fill_(3.0)
    if rank != 1:
        _peer_step(parallel, w, s, t, ex, out, status)
    torch.cuda.synchronize(dev)
    untouched = bool(torch.all(out == 3.0)) if rank != 1 else True
    record.append(gather_status())
    # step 2: the exchange is broken on every rank: each step fails at once
    status.zero_()
    t0 = time.perf_counter()
    _peer_step(parallel, w, s, t, ex, out, status)
    torch.cuda.synchronize(dev)
    fast = time.perf_counter() - t0 < 0.5
    record.append(gather_status())
    # recovery: every rank is done with the exchange (streams synchronised above), recreate it
    ex.close()
    ex = parallel.PeerExchange(w.B, w.H, w.D, wait_cycles=wait)
    status.zero_()
    _peer_step(parallel, w, s, t, ex, out, status)
    torch.cuda.synchronize(dev)
    record.append(gather_status())
    ex.close()
    flags = torch.tensor([int(untouched), int(fast)], dtype=torch.int64, device=dev)
    every = [torch.empty_like(flags) for _ in range(world)]
    dist.all_gather(every, flags)
    if rank == 0:
        full = W.device_tensors(w, dev)
        err = max_abs(out, oracle_outputs(Oracle(), w, full, range(w.B)))
        Path(out_path).write_text(json.dumps({
            "status_per_step": record, "timed_out_untouched": all(int(f[0]) for f in every),
            "broken_fails_fast": all(int(f[1]) for f in every), "recovered_max_abs_oracle": err, "world": world}))


def heads(out_path, rank, world, dev):
    import cottus_b200 as cb
    from cottus_b200 import parallel
    from cottus_b200 import workloads as W
    from helpers import max_abs, oracle_outputs, torch_reference
    from oracle.oracle import Oracle

    w = W.long_ctx_70b(seed=82, B=3, context=32768)
    t = W.device_tensors(w, dev)
    s, st = W.shard_kv_heads(w, t, rank, world)
    mine = cb.paged_decode(st["query"], st["kv_pool"], st["block_table"], st["context_lens"], num_kv_heads=s.Hkv,
                           head_dim=s.D, block_size=s.bs, num_physical_blocks=s.num_blocks,
                           out_dtype=torch.float16)
    torch.cuda.synchronize(dev)
    joined = parallel.gather_head_outputs(mine)
    if rank == 0:
        Path(out_path).write_text(json.dumps({
            "max_abs_torch_fp32": max_abs(joined, torch_reference(w, t)),
            "max_abs_oracle": max_abs(joined[1:2], oracle_outputs(Oracle(), w, t, [1])), "oracle_sequences": [1],
            "heads_per_rank": s.H, "world": world}))


def main():
    out_path, mode = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        {"parity": parity, "skip": skip, "heads": heads}[mode](out_path, rank, world, dev)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
