"""bench.py's reference arm on the host cores (no GPU): it runs the
reference's own CPU path and prints the one JSON line the bench contract
asks for, with the reference arm's extra keys."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _reference_line(config):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", config,
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=240, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


@pytest.mark.parametrize("config", ["tinyllama_f32", "oproj_llama3_8b"])
def test_reference_arm_json(config):
    pytest.importorskip("oracle.oracle")
    d = _reference_line(config)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]
    if config == "tinyllama_f32":
        # the reference arm describes the workload with the same config object as the GPU arm
        sys.path.insert(0, str(ROOT))
        import argparse

        import bench
        args = argparse.Namespace(config=config, batch=None, exchange="peer")
        assert d["config"] == bench.decode_config(args, 1)[1]


def test_l2_plan_keeps_every_step_off_l2_resident_kv():
    """Workloads smaller than 2 x L2 per step cycle enough layers' KV that a
    cycle covers 3 x L2; below 8 MB per layer the timed steps are replayed
    from a CUDA graph (the kernel is shorter than a host-side call)."""
    sys.path.insert(0, str(ROOT))
    import bench

    l2 = bench.L2_BYTES
    assert bench.l2_plan(2 * l2) == (1, False)
    assert bench.l2_plan(536870912) == (1, False)  # Llama-3-8B shape, batch 64
    for kv in (64 << 20, 8 << 20, 1380352, 4096):
        layers, graph = bench.l2_plan(kv)
        assert layers * kv >= 3 * l2 and (layers - 1) * kv < 3 * l2
        assert graph == (kv < 8 << 20)
