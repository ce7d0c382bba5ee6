"""The C-ABI library without a GPU: it loads, exports every symbol the
headers declare, rejects bad arguments before touching CUDA, and its host
components (block pool, RoPE table) match the reference bit for bit."""
import ctypes as C
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import cases

ROOT = Path(__file__).resolve().parent.parent
cb = pytest.importorskip("cottus_b200")
from cottus_b200 import _lib  # noqa: E402


def _declared_c_functions():
    text = (ROOT / "include" / "cottus_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cottus_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_c_abi():
    L = _lib.lib()
    names = _declared_c_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(L, n), n
    assert L.cottus_version() >= 10000


@pytest.mark.skipif(shutil.which("nm") is None, reason="nm not available")
def test_library_exports_cxx_shims():
    out = subprocess.run(["nm", "-D", "-C", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    for sym in ["cottus::pagedAttentionCUDA(float*, float const*, void const*, cottus::PageTable const&, int, int, "
                "int, int, int, int, int)",
                "cottus::ropeCUDA(float*, float const*, int, int, int, float)",
                "cottus::PageTable::appendBlock(int)", "cottus::PageTable::getBlock(int) const",
                "cottus::BlockAllocator::allocateBlock()", "cottus::BlockAllocator::freeBlock(int)"]:
        assert sym in out, sym


def test_invalid_arguments_rejected_without_gpu():
    L = _lib.lib()
    p = _lib.PagedDecodeParams()
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size, p.num_layers = 1, 4, 2, 64, 16, 1
    p.q_dtype = p.out_dtype = _lib.F32
    for field, val, msg in [("layer", -1, "layerIdx must be non-negative"), ("num_heads", 0, "numHeads must be positive"),
                            ("head_dim", 0, "headDim"), ("block_size", 0, "blockSize must be positive"),
                            ("layer", 1, "numLayers"), ("q_dtype", 7, "dtype")]:
        q = _lib.PagedDecodeParams.from_buffer_copy(p)
        setattr(q, field, val)
        rc = L.cottus_paged_decode(C.byref(q), None)
        assert rc == _lib.COTTUS_ERR_INVALID_ARGUMENT
        assert msg in L.cottus_last_error().decode()
    # NULL pointers with a non-empty batch
    assert L.cottus_paged_decode(C.byref(p), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    assert L.cottus_paged_decode(None, None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    assert L.cottus_status_string(-5) == b"workspace"
    # the allocation-free variant checks its arguments the same way, before sizing or queueing anything
    for field, val in [("batch", -1), ("layer", 1), ("out_dtype", 9)]:
        q = _lib.PagedDecodeParams.from_buffer_copy(p)
        setattr(q, field, val)
        assert L.cottus_paged_decode_static_scratch(C.byref(q), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    assert L.cottus_paged_decode_static_scratch(None, None) == _lib.COTTUS_ERR_INVALID_ARGUMENT


def test_projection_arguments_rejected_without_gpu():
    L = _lib.lib()
    p = _lib.OProjParams()
    p.in_features, p.out_features, p.batch, p.out_dtype = 128, 256, 3, _lib.F32
    assert L.cottus_o_proj_residual(None, None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    assert L.cottus_o_proj_residual(C.byref(p), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT  # NULL pointers
    assert "NULL" in L.cottus_last_error().decode()
    p.x, p.weight, p.residual, p.out = 0x1000, 0x2000, 0x3000, 0x4008
    assert L.cottus_o_proj_residual(C.byref(p), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    assert "16-byte" in L.cottus_last_error().decode()
    p.out, p.out_dtype = 0x4000, 9
    assert L.cottus_o_proj_residual(C.byref(p), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT
    for fin, fout in [(96, 256), (128, 200)]:
        q = _lib.OProjParams.from_buffer_copy(p)
        q.in_features, q.out_features = fin, fout
        assert L.cottus_o_proj_residual(C.byref(q), None) == _lib.COTTUS_ERR_UNSUPPORTED
    p.batch = 0
    assert L.cottus_o_proj_residual(C.byref(p), None) == _lib.COTTUS_OK  # nothing to do
    p.batch = -1
    assert L.cottus_o_proj_residual(C.byref(p), None) == _lib.COTTUS_ERR_INVALID_ARGUMENT


def test_rope_table_bit_exact(golden):
    r = cases.rope_cases()
    for D, key in ((64, "rope/cos_sin_d64"), (128, "rope/cos_sin_d128")):
        tab = cb.rope_cos_sin_table(4096, D).numpy()
        np.testing.assert_array_equal(tab[r["positions"]], golden[key])
    with pytest.raises(cb.CottusError):
        cb.rope_cos_sin_table(16, 7)


def test_block_allocator_matches_reference_trace(golden):
    ops, total = cases.allocator_ops()

    class A:
        def __init__(self):
            self.a = cb.BlockAllocator(total, 16)

        def alloc(self):
            return self.a.allocate()

        def free(self, i):
            self.a.free(i)
            return 0

    a = A()
    trace, _ = cases.run_allocator_ops(a, ops)
    np.testing.assert_array_equal(trace, golden["allocator/trace"])
    assert a.a.num_free() == golden["allocator/num_free"][0]


def test_block_allocator_errors():
    a = cb.BlockAllocator(2, 16)
    assert a.total_blocks() == 2
    with pytest.raises(cb.CottusError) as e:
        a.free(5)
    assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT and "Invalid block ID" in e.value.message
    x = a.allocate()
    assert x == 0
    a.free(x)
    with pytest.raises(cb.CottusError) as e:
        a.free(x)
    assert e.value.code == cb.COTTUS_ERR_DOUBLE_FREE and "Double free" in e.value.message
    a.allocate(), a.allocate()
    with pytest.raises(cb.CottusError) as e:
        a.allocate()
    assert e.value.code == cb.COTTUS_ERR_OUT_OF_MEMORY and "Out of memory" in e.value.message
    with pytest.raises(cb.CottusError):
        cb.BlockAllocator(0, 16)


def test_workload_tables_are_valid():
    from cottus_b200 import workloads as W

    for name, f in W.BUILDERS.items():
        w = f()
        pages = (w.ctx.astype(np.int64) + w.bs - 1) // w.bs
        used = np.concatenate([w.block_table[b, :n] for b, n in enumerate(pages)])
        assert used.min() >= 0 and used.max() < w.num_blocks, name
        assert len(np.unique(used)) == len(used), name  # no block shared between live pages
    w = W.ragged_mha()
    assert w.ctx.min() >= 16 and w.ctx.max() <= 8192 and w.B == 256
    # churn leaves the table fragmented: consecutive pages are rarely consecutive ids
    d = np.diff(w.block_table[np.argmax(w.ctx)][: (w.ctx.max() + 15) // 16])
    assert np.mean(d == 1) < 0.5
