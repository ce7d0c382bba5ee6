"""Runs the C++ drop-in check (tests/cpp/test_shim_parity.cpp), built by
__graft_entry__.build() against libcottus_b200.so and the oracle."""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
EXE = ROOT / "tests" / "cpp" / "_build" / "test_shim_parity"


def test_cpp_shim_parity():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not EXE.exists():
        pytest.fail(f"{EXE} not built: run __graft_entry__.build()")
    r = subprocess.run([str(EXE)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS" in r.stdout
