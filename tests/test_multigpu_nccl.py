"""Split-KV decode across GPUs (needs two or more GPUs): each rank holds a
contiguous page range of every sequence.  The merged output must match the
oracle (pagedAttentionCPU restated, paged_attention_cpu.cpp:24-103) and a
torch fp32 attention over the un-split context within the fp16 bound on
every rank, over NCCL and, bit for bit the same, through peer memory
(cottus_split_decode) over many steps with the ranks drifting up to a step
apart.  A rank that skips a step makes the others time out, the exchange
then refuses every step on every rank, and a recreated exchange is correct
again.  The kv-head partition (each rank's final outputs for its query
heads, no exchange) matches the oracle and torch fp32 as well."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from helpers import TOL_F16

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(tmp_path, world, mode):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / f"result_{mode}_{world}.json"
    # NVLS off: a rank that leaves must not be bound to an NVLink multicast object
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "multigpu_worker.py"), str(out), mode]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=360, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.loads(out.read_text())


@pytest.mark.parametrize("world", [2, 4, 8])
def test_split_kv_parity(tmp_path, world):
    v = _run(tmp_path, world, "parity")
    assert v["ranks_agree"]
    assert v["max_abs_oracle"] <= TOL_F16
    assert v["max_abs_torch_fp32"] <= TOL_F16
    assert v["peer_equal_all_ranks"]
    assert v["peer_status"] == [0] * world


@pytest.mark.parametrize("world", [2, 4])
def test_split_kv_rank_skips_a_step(tmp_path, world):
    v = _run(tmp_path, world, "skip")
    st = v["status_per_step"]
    timeout = 0x8
    assert st[0] == [0] * world
    assert all(s & timeout for r, s in enumerate(st[1]) if r != 1) and st[1][1] == 0
    assert all(s & timeout for s in st[2])
    assert v["timed_out_untouched"] and v["broken_fails_fast"]
    assert st[3] == [0] * world
    assert v["recovered_max_abs_oracle"] <= TOL_F16


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_partition_parity(tmp_path, world):
    v = _run(tmp_path, world, "heads")
    assert v["max_abs_oracle"] <= TOL_F16
    assert v["max_abs_torch_fp32"] <= TOL_F16
