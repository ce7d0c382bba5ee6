"""cottus_paged_decode_static_scratch: the decode entry point for callers that
cannot allocate device memory while attention runs (allocator or memory-pool
callbacks, engines that reserve all device memory up front, plugin hosts that
pass only a stream and the call's tensors).  It uses a scratch array built
into the library instead of a caller workspace.

Called through the C ABI and checked against cottus_paged_decode (which gets
a normal workspace) on two calls in a row, within the tolerances the other
tests use.  This file is collected last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes as C

import pytest
import torch

from helpers import max_abs, tol_for

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")
from cottus_b200 import _lib  # noqa: E402
from cottus_b200 import workloads as W  # noqa: E402
from cottus_b200.ops import make_decode_params  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _static_scratch_call(w, t, out_dtype):
    out = torch.full((w.B, w.H, w.D), float("nan"), dtype=out_dtype, device=DEV)
    p = make_decode_params(out, t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                           head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=w.layer,
                           num_physical_blocks=w.num_blocks)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib().cottus_paged_decode_static_scratch(C.byref(p), stream))
    torch.cuda.synchronize()
    return out


CASES = {
    # fp16 output, group of 4 (tensor-core kernel), pairs cut across workers
    "llama3_8b_f16": lambda: W.llama3_8b(seed=71, B=16, context=1500),
    # fp32 output (SIMT kernel), fp32 queries
    "tinyllama_f32": lambda: W.tinyllama_f32(seed=72),
    # ragged MHA with empty slots handled by the kernel
    "ragged_mha": lambda: W.ragged_mha(seed=73, B=24, lo=1, hi=2500, n_ops=500),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_static_scratch_matches_workspace_entry_point(name):
    w = CASES[name]()
    t = W.device_tensors(w, DEV)
    ref = cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                          head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=w.layer, out_dtype=w.out_dtype,
                          num_physical_blocks=w.num_blocks)
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row share (and reuse) the scratch
        got = _static_scratch_call(w, t, w.out_dtype)
        assert torch.isfinite(got).all()
        assert max_abs(got, ref) <= tol_for(w.out_dtype)


def test_static_scratch_rejects_oversized_calls():
    """A batch whose arrival counters alone exceed the 32 MiB scratch is
    refused before anything runs (the pointers are never dereferenced)."""
    p = _lib.PagedDecodeParams()
    p.out = p.query = p.kv_pool = p.block_table = p.context_lens = 256
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size = 600_000, 8, 8, 128, 16
    p.num_layers, p.layer, p.max_blocks_per_seq, p.num_physical_blocks = 1, 0, 1, 1
    p.q_dtype = p.out_dtype = _lib.F16
    rc = _lib.lib().cottus_paged_decode_static_scratch(C.byref(p), None)
    assert rc == cb.COTTUS_ERR_WORKSPACE
    assert "static scratch" in _lib.lib().cottus_last_error().decode()
