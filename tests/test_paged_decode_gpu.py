"""Parity of cottus_paged_decode (through the C ABI) with the oracle.

Bounds: max-abs error <= 1e-5 for fp32 outputs and <= 2e-3 for fp16
outputs (helpers.TOL_F32 / TOL_F16).  Sizes the oracle finishes in seconds
are compared in full; full-size workloads are compared on sampled sequences
against the oracle and on every sequence against a torch fp32 reference.
"""
import numpy as np
import pytest
import torch

import cases
from helpers import TOL_F16, TOL_F32, max_abs, oracle_outputs, tol_for, torch_reference

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")
from cottus_b200 import workloads as W  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def run(w, t, out_dtype=None, **kw):
    out = cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                          head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=w.layer,
                          out_dtype=out_dtype or w.out_dtype, num_physical_blocks=w.num_blocks, **kw)
    torch.cuda.synchronize()
    return out


def case_tensors(c, q_dtype=torch.float32):
    return dict(query=torch.from_numpy(c["q"]).to(DEV).to(q_dtype),
                kv_pool=torch.from_numpy(c["kv"].view(np.int16)).to(DEV),
                block_table=torch.from_numpy(np.ascontiguousarray(c["tables"])).to(DEV),
                context_lens=torch.from_numpy(c["ctx"]).to(DEV))


def case_run(c, t, out_dtype):
    nb = c["kv"].size // (2 * c["L"] * c["bs"] * c["Hkv"] * c["D"])
    out = cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=c["Hkv"],
                          head_dim=c["D"], block_size=c["bs"], num_layers=c["L"], layer=c["layer"],
                          out_dtype=out_dtype, num_physical_blocks=nb)
    torch.cuda.synchronize()
    return out


# -- known-answer and golden cases ----------------------------------------------------

@pytest.mark.parametrize("name", sorted(cases.kat_cases()))
def test_kat_vs_golden(golden, name):
    c = cases.kat_cases()[name]
    out = case_run(c, case_tensors(c), torch.float32)
    assert max_abs(out, golden[f"{name}/out"]) <= TOL_F32


def test_kat_expected_values():
    c = cases.kat_cases()
    o = case_run(c["kat_single_head"], case_tensors(c["kat_single_head"]), torch.float32).cpu().numpy().ravel()
    np.testing.assert_allclose(o, 0.622 + 0.378 * 2, atol=0.01)
    o = case_run(c["kat_multi_head"], case_tensors(c["kat_multi_head"]), torch.float32).cpu().numpy().ravel()
    np.testing.assert_allclose(o, [2, 0, 0, 3], atol=0.01)
    o = case_run(c["kat_multi_block"], case_tensors(c["kat_multi_block"]), torch.float32).cpu().numpy().ravel()
    assert abs(o[0] - 2.0) < 0.1


@pytest.mark.parametrize("name", sorted(cases.SHAPE_CASES))
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_shape_cases_vs_golden(golden, name, out_dtype):
    c = cases.make_shape_case(name)
    q_dtype = torch.float16 if c["q_fp16"] else torch.float32
    out = case_run(c, case_tensors(c, q_dtype), out_dtype)
    assert max_abs(out, golden[f"{name}/out"]) <= tol_for(out_dtype)


def test_determinism_bitwise():
    """tests/test_paged_attention_parity.cpp:178-215: repeated runs are bit-identical."""
    w = W.ragged_mha(seed=11, B=24, lo=16, hi=2048, n_ops=500)
    t = W.device_tensors(w, DEV)
    ref = run(w, t).clone()
    for _ in range(9):
        assert torch.equal(run(w, t), ref)


# -- seeded workloads at oracle-friendly sizes ----------------------------------------

SMALL = {
    "tinyllama_f32": lambda: W.tinyllama_f32(seed=21),
    "llama3_8b": lambda: W.llama3_8b(seed=22, B=6, context=1000),
    "ragged_mha": lambda: W.ragged_mha(seed=23, B=20, lo=1, hi=3000, n_ops=2000),
    "long_ctx_70b": lambda: W.long_ctx_70b(seed=24, B=2, context=16384),
}


@pytest.mark.parametrize("name,out_dtype", [("llama3_8b", torch.float16), ("ragged_mha", torch.float32)])
def test_replayed_from_a_cuda_graph(oracle, name, out_dtype):
    """One launch captured in a CUDA graph and replayed with new queries: the
    arrival counters of the cut pairs return to zero at the end of every
    launch, so each replay (same launch tag) merges its pairs again.  Covers
    the tensor-core kernel (fp16, G=4) and the SIMT kernel (G=1, fp32 out)."""
    w = SMALL[name]()
    t = W.device_tensors(w, DEV)
    out = torch.empty(t["query"].shape, dtype=out_dtype, device=DEV)
    run(w, t, out=out)  # outside the capture: the cached workspace is sized here
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                        head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=w.layer, out=out,
                        num_physical_blocks=w.num_blocks)
    gen = torch.Generator().manual_seed(31)
    for _ in range(3):
        t["query"].copy_(torch.randn(tuple(t["query"].shape), generator=gen).to(t["query"].dtype))
        g.replay()
        torch.cuda.synchronize()
        assert max_abs(out, oracle_outputs(oracle, w, t, range(w.B))) <= tol_for(out_dtype)
    del g


@pytest.mark.parametrize("name", sorted(SMALL))
def test_workload_vs_oracle(oracle, name):
    w = SMALL[name]()
    t = W.device_tensors(w, DEV)
    out = run(w, t)
    ref = oracle_outputs(oracle, w, t, range(w.B))
    assert max_abs(out, ref) <= tol_for(w.out_dtype)


def test_fp32_query_fp16_out_and_reverse(oracle):
    w = W.llama3_8b(seed=25, B=3, context=333)
    t = W.device_tensors(w, DEV)
    ref = oracle_outputs(oracle, w, t, range(w.B))
    assert max_abs(run(w, t, out_dtype=torch.float32), ref) <= TOL_F32
    t32 = dict(t, query=t["query"].float())
    assert max_abs(run(w, t32, out_dtype=torch.float16), ref) <= TOL_F16


# -- full-size workloads ---------------------------------------------------------------

def test_full_llama3_8b(oracle):
    w = W.llama3_8b()
    t = W.device_tensors(w, DEV)
    out = run(w, t)
    seqs = [0, 17, 63]
    assert max_abs(out[seqs], oracle_outputs(oracle, w, t, seqs)) <= TOL_F16
    assert max_abs(out, torch_reference(w, t)) <= TOL_F16


def test_full_ragged_mha(oracle):
    w = W.ragged_mha()
    t = W.device_tensors(w, DEV)
    out = run(w, t)
    order = np.argsort(w.ctx)
    seqs = [int(order[0]), int(order[1]), int(order[len(order) // 2]), int(order[-1])]
    assert max_abs(out[seqs], oracle_outputs(oracle, w, t, seqs)) <= TOL_F16
    assert max_abs(out, torch_reference(w, t)) <= TOL_F16


def test_full_long_context_split_kv(oracle):
    """Full 131072-token contexts: the un-split kernel, the 2/4/8-way
    page-range split (LSE partials on one GPU, then cottus_lse_combine), and
    the 2/4/8-way kv-head partition (each shard's final outputs for its
    query heads, the shards run one after another on one GPU), against the
    oracle on one sequence and torch fp32 on all."""
    w = W.long_ctx_70b()
    t = W.device_tensors(w, DEV)
    out = run(w, t)
    ref = oracle_outputs(oracle, w, t, [5])
    assert max_abs(out[5:6], ref) <= TOL_F16
    tref = torch_reference(w, t)
    assert max_abs(out, tref) <= TOL_F16
    for world in (2, 4, 8):
        parts, lses = [], []
        for r in range(world):
            s = W.shard_long_context(w, r, world)
            first, count = s.meta["pool_range"]
            per = w.block_elems()
            st = dict(query=t["query"], kv_pool=t["kv_pool"][first * per:(first + count) * per],
                      block_table=torch.from_numpy(s.block_table).to(DEV),
                      context_lens=torch.from_numpy(s.ctx).to(DEV))
            lse = torch.empty((w.B, w.H), dtype=torch.float32, device=DEV)
            parts.append(run(s, st, out_dtype=torch.float32, lse_out=lse))
            lses.append(lse)
        merged = cb.lse_combine(torch.stack(parts), torch.stack(lses), out_dtype=torch.float16)
        torch.cuda.synchronize()
        assert max_abs(merged, tref) <= TOL_F16
        assert max_abs(merged[5:6], ref) <= TOL_F16
    for world in (2, 4, 8):
        heads = []
        for r in range(world):
            s, st = W.shard_kv_heads(w, t, r, world)
            heads.append(run(s, st))
            del st
        joined = torch.cat(heads, dim=1)
        assert max_abs(joined, tref) <= TOL_F16
        assert max_abs(joined[5:6], ref) <= TOL_F16


# -- edge cases ------------------------------------------------------------------------

def _custom(ctx, maxb=None, H=8, Hkv=2, D=128, seed=31, pool_extra=3):
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    pages = (ctx.astype(np.int64) + 15) // 16
    maxb = maxb or max(int(pages.max(initial=1)), 1)
    total = int(pages.sum()) + pool_extra
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(ctx), maxb), np.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n]
        off += n
    return W.Workload("custom", H, Hkv, D, 16, 1, 0, torch.float16, torch.float32, ctx, bt, total, seed)


def test_ragged_edges(oracle):
    w = _custom([0, 1, 15, 16, 17, 31, 32, 33, 0, 1000, 2049])
    t = W.device_tensors(w, DEV)
    out = run(w, t)
    ref = oracle_outputs(oracle, w, t, range(w.B))
    assert max_abs(out, ref) <= TOL_F32
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[8]) == 0


def test_max_context_and_single_sequence(oracle):
    """One sequence filling its whole table (every worker of the grid shares it)."""
    w = _custom([4096], maxb=256)
    t = W.device_tensors(w, DEV)
    assert max_abs(run(w, t), oracle_outputs(oracle, w, t, [0])) <= TOL_F32


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_group_and_head_dim_grid(oracle, G, D, out_dtype):
    """Every (group, head_dim) instantiation: fp32 outputs use the SIMT
    kernel, fp16 outputs the tensor-core kernel (head_dim 64/128)."""
    w = _custom([5, 77, 300, 16], H=2 * G, Hkv=2, D=D, seed=G * 1000 + D)
    t = W.device_tensors(w, DEV)
    got = run(w, t, out_dtype=out_dtype)
    assert max_abs(got, oracle_outputs(oracle, w, t, range(w.B))) <= tol_for(out_dtype)
    t32 = dict(t, query=t["query"].float())  # fp32 queries: split into fp16 hi/lo on the tensor-core path
    assert max_abs(run(w, t32, out_dtype=out_dtype), oracle_outputs(oracle, w, t32, range(w.B))) <= tol_for(out_dtype)


@pytest.mark.parametrize("H,Hkv,D,bs", [(6, 4, 64, 16), (4, 4, 40, 16), (16, 2, 128, 32), (2, 1, 96, 7)])
def test_generic_shapes(oracle, H, Hkv, D, bs):
    """Shapes outside the fast path (uneven GQA map, odd head_dim, other block sizes)."""
    rng = np.random.default_rng(H * 100 + D + bs)
    ctx = np.array([1, bs, 3 * bs + 1, 200], np.int32)
    pages = (ctx + bs - 1) // bs
    total = int(pages.sum()) + 2
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((4, int(pages.max())), np.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n]
        off += n
    w = W.Workload("generic", H, Hkv, D, bs, 2, 1, torch.float32, torch.float32, ctx, bt, total, 77)
    t = W.device_tensors(w, DEV)
    assert max_abs(run(w, t), oracle_outputs(oracle, w, t, range(4))) <= TOL_F32


def test_lse_output(oracle):
    w = _custom([50, 700], H=8, Hkv=2, D=64)
    t = W.device_tensors(w, DEV)
    lse = torch.empty((w.B, w.H), dtype=torch.float32, device=DEV)
    run(w, t, lse_out=lse)
    pool = t["kv_pool"].view(-1, 2, 16, w.Hkv, w.D)
    for b in range(w.B):
        n = int(w.ctx[b])
        pages = (n + 15) // 16
        blk = pool.index_select(0, torch.from_numpy(w.block_table[b, :pages]).long().to(DEV))
        k = blk[:, 0].reshape(-1, w.Hkv, w.D)[:n].view(torch.float16).double()
        q = t["query"][b].double()
        s = torch.einsum("hd,nhd->hn", q, k.repeat_interleave(w.H // w.Hkv, 1)) / np.sqrt(w.D)
        assert max_abs(lse[b], torch.logsumexp(s, -1)) < 1e-4


def test_status_bad_block_and_context():
    w = _custom([40, 40, 40])
    t = W.device_tensors(w, DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    bt = t["block_table"].clone()
    bt[1, 1] = w.num_blocks + 5
    ctx = t["context_lens"].clone()
    ctx[2] = 10 ** 6
    out = cb.paged_decode(t["query"], t["kv_pool"], bt, ctx, num_kv_heads=w.Hkv, head_dim=w.D, block_size=16,
                          out_dtype=torch.float32, num_physical_blocks=w.num_blocks, status=status)
    torch.cuda.synchronize()
    s = int(status.item())
    assert s & cb.STATUS_BAD_BLOCK_ID and s & cb.STATUS_BAD_CONTEXT
    assert torch.count_nonzero(out[2]) == 0
    assert torch.isfinite(out).all()


def test_invalid_arguments_raise():
    w = _custom([10])
    t = W.device_tensors(w, DEV)
    with pytest.raises(cb.CottusError) as e:
        cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                        head_dim=w.D, block_size=0)
    assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT and "blockSize must be positive" in e.value.message
    with pytest.raises(cb.CottusError) as e:
        cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                        head_dim=w.D, block_size=16, num_layers=1, layer=1)
    assert e.value.code == cb.COTTUS_ERR_INVALID_ARGUMENT


def test_workspace_required():
    import ctypes as C

    from cottus_b200 import _lib
    from cottus_b200.ops import make_decode_params

    w = _custom([100])
    t = W.device_tensors(w, DEV)
    out = torch.empty(t["query"].shape, dtype=torch.float32, device=DEV)
    p = make_decode_params(out, t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                           head_dim=w.D, block_size=16, num_physical_blocks=w.num_blocks)
    need = _lib.lib().cottus_paged_decode_workspace_size(C.byref(p))
    assert need > 0
    rc = _lib.lib().cottus_paged_decode(C.byref(p), None)
    assert rc == cb.COTTUS_ERR_WORKSPACE


def test_batch_zero_is_noop():
    q = torch.empty((0, 8, 128), dtype=torch.float16, device=DEV)
    pool = torch.zeros(2 * 16 * 2 * 128, dtype=torch.int16, device=DEV)
    bt = torch.zeros((0, 1), dtype=torch.int32, device=DEV)
    ctx = torch.zeros(0, dtype=torch.int32, device=DEV)
    out = cb.paged_decode(q, pool, bt, ctx, num_kv_heads=2, head_dim=128, block_size=16)
    assert out.shape == (0, 8, 128)
