"""RoPE, KV append, the fused RoPE + append + decode step, and the
block-table gather, through the C ABI, against the oracle.

RoPE outputs and every KV byte written by the append are compared bit for
bit; attention outputs use the fp32/fp16 bounds of helpers.py.
"""
import numpy as np
import pytest
import torch

import cases
from helpers import TOL_F16, TOL_F32, host_subpool, max_abs, tol_for

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")
from cottus_b200 import workloads as W  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_rope_bit_exact_vs_golden(golden):
    r = cases.rope_cases()
    tab = cb.rope_cos_sin_table(4096, 64).to(DEV)
    pos = torch.from_numpy(r["positions"]).to(DEV)
    x = torch.from_numpy(np.broadcast_to(r["x64"], (len(r["positions"]), 4, 64)).copy()).to(DEV)
    out = cb.rope(x, pos, tab)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().reshape(len(r["positions"]), -1), golden["rope/x64_out"])
    # in place
    y = x.clone()
    cb.rope(y, pos, tab, out=y)
    torch.cuda.synchronize()
    assert torch.equal(y, out)
    # the reference parity test's input (pos 5, H 2, D 8)
    tab8 = cb.rope_cos_sin_table(8, 8).to(DEV)
    k = torch.from_numpy(r["kat_in"].reshape(1, 2, 8)).to(DEV)
    o = cb.rope(k, torch.tensor([5], dtype=torch.int32, device=DEV), tab8)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o.cpu().numpy().ravel(), golden["rope/kat_out"])


def _fused_inputs(w, t):
    tab = cb.rope_cos_sin_table(int(w.positions.max()) + 1, w.D, w.theta).to(DEV)
    return tab


def _oracle_step(oracle, w, t, pool_before):
    """Oracle of one decode step: ropeCPU(q), ropeCPU(k), restated append,
    pagedAttentionCPU over pos+1 tokens.  Returns (pool after, out, q_rot)."""
    pool = pool_before.copy()
    B = w.B
    q = t["query"].float().cpu().numpy()
    k = t["key"].float().cpu().numpy()
    v = t["value"].float().cpu().numpy()
    outs, qrs = [], []
    for b in range(B):
        p = int(w.positions[b])
        qr = oracle.rope(q[b], p, w.H, w.D, w.theta).reshape(w.H, w.D)
        kr = oracle.rope(k[b], p, w.Hkv, w.D, w.theta)
        nblk = p // w.bs + 1
        oracle.kv_append(pool, kr, v[b], w.block_table[b, :nblk], p, w.layer, w.Hkv, w.D, w.bs, w.L)
        outs.append(oracle.paged_attention(qr, pool, w.block_table[b, :nblk], p + 1, w.layer, w.H, w.Hkv, w.D,
                                           w.bs, w.L))
        qrs.append(qr)
    return pool, np.stack(outs), np.stack(qrs)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_rope_append_bit_exact(oracle, dtype):
    w = W.fused_tinyllama(seed=41, B=12, max_pos=700)
    w.q_dtype = dtype
    t = W.device_tensors(w, DEV)
    pool_before = t["kv_pool"].cpu().numpy().view(np.uint16).copy()
    tab = _fused_inputs(w, t)
    q_out = torch.empty_like(t["query"])
    cb.rope_append(t["query"], t["key"], t["value"], t["positions"], tab, t["kv_pool"], t["block_table"],
                   num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, query_out=q_out)
    torch.cuda.synchronize()
    pool_ref, _, q_ref = _oracle_step(oracle, w, t, pool_before)
    np.testing.assert_array_equal(t["kv_pool"].cpu().numpy().view(np.uint16), pool_ref)
    if dtype == torch.float32:
        np.testing.assert_array_equal(q_out.cpu().numpy(), q_ref)
    else:
        np.testing.assert_array_equal(q_out.cpu().numpy(), q_ref.astype(np.float16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("B,max_pos", [(32, 4095), (7, 40)])
def test_fused_step_vs_oracle(oracle, dtype, B, max_pos):
    w = W.fused_tinyllama(seed=42 + B, B=B, max_pos=max_pos)
    w.q_dtype = dtype
    w.out_dtype = dtype
    t = W.device_tensors(w, DEV)
    pool_before = t["kv_pool"].cpu().numpy().view(np.uint16).copy()
    tab = _fused_inputs(w, t)
    q_out = torch.empty_like(t["query"])
    out = cb.rope_append_decode(t["query"], t["key"], t["value"], t["positions"], tab, t["kv_pool"],
                                t["block_table"], num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                query_out=q_out)
    torch.cuda.synchronize()
    pool_ref, out_ref, q_ref = _oracle_step(oracle, w, t, pool_before)
    np.testing.assert_array_equal(t["kv_pool"].cpu().numpy().view(np.uint16), pool_ref)
    assert max_abs(out, out_ref) <= tol_for(dtype)
    if dtype == torch.float32:
        np.testing.assert_array_equal(q_out.cpu().numpy(), q_ref)


def test_fused_step_generic_path(oracle):
    """head_dim 40 is outside the fast path: append kernel + generic decode."""
    rng = np.random.default_rng(9)
    B, H, Hkv, D = 5, 4, 2, 40
    pos = np.array([0, 15, 16, 33, 100], np.int32)
    pages = pos // 16 + 1
    total = int(pages.sum()) + 2
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((B, int(pages.max())), np.int32)
    off = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[off:off + n]
        off += n
    w = W.Workload("g", H, Hkv, D, 16, 1, 0, torch.float32, torch.float32, pos + 1, bt, total, 3, positions=pos)
    t = W.device_tensors(w, DEV)
    pool_before = t["kv_pool"].cpu().numpy().view(np.uint16).copy()
    tab = cb.rope_cos_sin_table(128, D).to(DEV)
    out = cb.rope_append_decode(t["query"], t["key"], t["value"], t["positions"], tab, t["kv_pool"],
                                t["block_table"], num_kv_heads=Hkv, head_dim=D, block_size=16)
    torch.cuda.synchronize()
    pool_ref, out_ref, _ = _oracle_step(oracle, w, t, pool_before)
    np.testing.assert_array_equal(t["kv_pool"].cpu().numpy().view(np.uint16), pool_ref)
    assert max_abs(out, out_ref) <= TOL_F32


def test_bad_position_status():
    w = W.fused_tinyllama(seed=43, B=4, max_pos=100)
    t = W.device_tensors(w, DEV)
    tab = cb.rope_cos_sin_table(int(w.positions.max()) + 1, w.D).to(DEV)
    pos = t["positions"].clone()
    pos[2] = 10 ** 6
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = cb.rope_append_decode(t["query"], t["key"], t["value"], pos, tab, t["kv_pool"], t["block_table"],
                                num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & cb.STATUS_BAD_POSITION
    assert torch.count_nonzero(out[2]) == 0


@pytest.mark.parametrize("name", ["ragged_mha", "llama3_8b"])
def test_gather_bit_exact(oracle, name):
    w = W.ragged_mha(seed=51, B=16, lo=1, hi=900, n_ops=1000) if name == "ragged_mha" else \
        W.llama3_8b(seed=52, B=4, context=300)
    t = W.device_tensors(w, DEV)
    maxc = int(w.ctx.max())
    k, v = cb.paged_gather(t["kv_pool"], t["block_table"], t["context_lens"], max_context=maxc,
                           num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, num_physical_blocks=w.num_blocks)
    torch.cuda.synchronize()
    k = k.cpu().numpy()
    v = v.cpu().numpy()
    seqs = list(range(w.B))
    sub, bt, ctx = host_subpool(w, t["kv_pool"], seqs)
    for b in seqs:
        kr, vr = oracle.gather_kv(sub, bt[b], int(ctx[b]), w.layer, w.Hkv, w.D, w.bs, w.L)
        np.testing.assert_array_equal(k[b, :ctx[b]], kr)
        np.testing.assert_array_equal(v[b, :ctx[b]], vr)
        assert not k[b, ctx[b]:].any()


def test_lse_combine_empty_shard():
    P, B, H, D = 3, 2, 4, 64
    g = torch.Generator(device=DEV).manual_seed(1)
    parts = torch.randn((P, B, H, D), generator=g, device=DEV)
    lse = torch.randn((P, B, H), generator=g, device=DEV)
    lse[1] = -float("inf")
    out = cb.lse_combine(parts, lse)
    torch.cuda.synchronize()
    w = torch.softmax(lse, dim=0)
    ref = (w.unsqueeze(-1) * parts.nan_to_num()).sum(0)
    assert max_abs(out, ref) < 1e-5
