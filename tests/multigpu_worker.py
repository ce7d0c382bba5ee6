"""Worker for tests/test_multigpu_nccl.py (one process per GPU, launched by
torch.distributed.run): the long-context split-KV decode across GPUs.

Every rank holds one contiguous page range of every sequence.  Path 1
computes LSE partials with cottus_paged_decode, all-gathers them over NCCL
and merges them with cottus_lse_combine.  Path 2 (cottus_split_decode)
exchanges the same partials through peer memory: the decode kernel flags
completion to every rank, the combine kernel reads the other ranks'
partials over NVLink; it runs three steps in a row (both exchange slots)
and must give the same bits as path 1.  Rank 0 compares the merged output
with the un-split kernel on the whole pool (built on rank 0's GPU) and
writes a JSON verdict."""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "cottus-runtime_b200", ROOT / "tests"):
    sys.path.insert(0, str(p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        import cottus_b200 as cb
        from cottus_b200 import parallel
        from cottus_b200 import workloads as W
        from helpers import max_abs

        w = W.long_ctx_70b(seed=81, B=3, context=32768)
        s = W.shard_long_context(w, rank, world)
        t = W.device_tensors(s, dev, pool_blocks=s.meta["pool_range"])
        merged = parallel.split_kv_decode(t["query"], t["kv_pool"], torch.from_numpy(s.block_table).to(dev),
                                          torch.from_numpy(s.ctx).to(dev), num_kv_heads=w.Hkv, head_dim=w.D,
                                          block_size=w.bs, num_physical_blocks=s.num_blocks,
                                          out_dtype=torch.float16)
        torch.cuda.synchronize(dev)
        ex = parallel.PeerExchange(w.B, w.H, w.D)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        peer_equal = True
        for _ in range(3):
            peer = parallel.split_kv_decode_peer(t["query"], t["kv_pool"], torch.from_numpy(s.block_table).to(dev),
                                                 torch.from_numpy(s.ctx).to(dev), ex, num_kv_heads=w.Hkv,
                                                 head_dim=w.D, block_size=w.bs, num_physical_blocks=s.num_blocks,
                                                 out_dtype=torch.float16, status=status)
            torch.cuda.synchronize(dev)
            peer_equal = peer_equal and torch.equal(peer, merged)
        ex.close()
        peer_status = int(status.item())
        gathered = [torch.empty_like(merged) for _ in range(world)]
        dist.all_gather(gathered, merged)
        flags = torch.tensor([int(peer_equal), peer_status], dtype=torch.int64, device=dev)
        every = [torch.empty_like(flags) for _ in range(world)]
        dist.all_gather(every, flags)
        if rank == 0:
            full = W.device_tensors(w, dev)
            ref = cb.paged_decode(full["query"], full["kv_pool"], full["block_table"], full["context_lens"],
                                  num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                  num_physical_blocks=w.num_blocks)
            torch.cuda.synchronize(dev)
            err = max_abs(merged, ref)
            same = all(torch.equal(g, gathered[0]) for g in gathered)
            Path(out_path).write_text(json.dumps({
                "max_abs": err, "ranks_agree": same, "world": world,
                "peer_equal_all_ranks": all(int(f[0]) == 1 for f in every),
                "peer_status": [int(f[1]) for f in every]}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
