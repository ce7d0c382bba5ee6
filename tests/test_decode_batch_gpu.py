"""Batched decode steps through the device-resident block table of
cottus_decode_batch_*, against the oracle.

Sequences join and leave a running batch (a released row is taken by the
last one, blocks are reused LIFO).  Each step: begin_step (blocks for rows
whose next token starts one, changed table entries and positions sent to
the device), then per layer cottus_rope_append_decode over the device table
and positions, then end_step.  A host replica runs the same schedule on the
oracle: ropeCPU, the restated append and pagedAttentionCPU per sequence
(generic_transformer.cpp:196-291 for each token of Engine::generate,
engine.cpp:52-95).  Attention outputs are compared within the fp16/fp32
bounds; at the end the KV pool is compared bit for bit, and the device
table and positions with the host mirror.
"""
import numpy as np
import pytest
import torch

from helpers import BatchReplica, max_abs, tol_for

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_batched_steps_with_joins_and_releases(oracle, dtype):
    H, Hkv, D, bs, L = 8, 2, 64, 16, 2
    nb, mb, maxb = 40, 5, 8
    per_block = 2 * L * bs * Hkv * D
    rng = np.random.default_rng(17 if dtype == torch.float16 else 18)
    pool = torch.zeros(nb * per_block, dtype=torch.int16, device=DEV)
    hpool = np.zeros(nb * per_block, np.uint16)
    tab = cb.rope_cos_sin_table(maxb * bs, D).to(DEV)
    batch = cb.DecodeBatch(nb, bs, mb, maxb, device=DEV)
    rep = BatchReplica(oracle, nb, bs, mb, maxb)
    next_id, worst = 0, 0.0
    for step in range(60):
        if len(rep.rows) < mb and (not rep.rows or rng.random() < 0.25):
            batch.add(next_id)
            rep.add(next_id)
            next_id += 1
        if len(rep.rows) > 1 and rng.random() < 0.07:
            sid = int(rng.choice(rep.rows))
            batch.release(sid)
            rep.release(sid)
        for sid in [s for s in rep.rows if rep.seq[s][0] >= maxb * bs]:
            batch.release(sid)
            rep.release(sid)
        if not rep.begin_step():  # pool exhausted: the oldest sequence ends first
            sid = rep.rows[0]
            batch.release(sid)
            rep.release(sid)
            assert rep.begin_step()
        batch.begin_step()
        rows = batch.rows()
        assert rows == rep.rows
        n = len(rows)
        q = torch.from_numpy(rng.standard_normal((n, H, D), dtype=np.float32)).to(DEV).to(dtype)
        k = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).to(DEV).to(dtype)
        v = torch.from_numpy(rng.standard_normal((n, Hkv, D), dtype=np.float32)).to(DEV).to(dtype)
        qh, kh, vh = q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy()
        for layer in range(L):
            out = cb.rope_append_decode(q, k, v, batch.positions[:n], tab, pool, batch.block_table[:n],
                                        num_kv_heads=Hkv, head_dim=D, block_size=bs, num_layers=L, layer=layer,
                                        out_dtype=dtype)
            torch.cuda.synchronize()
            for r, sid in enumerate(rows):
                pos, blocks = rep.seq[sid]
                qr = oracle.rope(qh[r], pos, H, D)
                kr = oracle.rope(kh[r], pos, Hkv, D)
                oracle.kv_append(hpool, kr, vh[r], blocks, pos, layer, Hkv, D, bs, L)
                ref = oracle.paged_attention(qr, hpool, blocks, pos + 1, layer, H, Hkv, D, bs, L)
                err = max_abs(out[r].float().cpu(), ref.reshape(H, D))
                worst = max(worst, err)
                assert err <= tol_for(dtype), (step, layer, sid, err)
        batch.end_step()
        rep.end_step()
    assert next_id >= 8  # the schedule had joins, releases and block reuse
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.cpu().numpy().view(np.uint16), hpool)
    tbl, posd = batch.block_table.cpu().numpy(), batch.positions.cpu().numpy()
    for r, sid in enumerate(rep.rows):
        pos, blocks = rep.seq[sid]
        assert posd[r] == pos - 1  # the device holds the last step's positions
        np.testing.assert_array_equal(tbl[r, :len(blocks)], blocks)


PROJ_TOL = 2e-4  # |projection - gemmCPU| for N(0,1) activations and N(0, 1/in) weights


def test_attention_block_steps_vs_oracle(oracle):
    """attention_block over a running batch: the QKV projection with RoPE
    and append, attention over position + 1 tokens through the device
    context lengths, and the O-projection added to the residual, for two
    layers per step while sequences join and leave.  Every stage is checked
    against the oracle on the kernel's own inputs to that stage: the rotated
    query and the new K/V against gemmCPU + ropeCPU (+ the truncating
    encoder), the attention output against pagedAttentionCPU over the pool
    the kernels wrote, and the residual against gemmCPU + residualAddCPU on
    that attention output (generic_transformer.cpp:169-327)."""
    hidden, H, Hkv, D, bs, L = 512, 8, 2, 64, 16, 2
    N, HD, KD = (H + 2 * Hkv) * D, H * D, Hkv * D
    nb, mb, maxb = 48, 5, 8
    per_block = 2 * L * bs * Hkv * D
    rng = np.random.default_rng(41)
    w_qkv = [torch.from_numpy(rng.standard_normal((N, hidden), dtype=np.float32) / np.float32(hidden ** 0.5)).half()
             for _ in range(L)]
    w_o = [torch.from_numpy(rng.standard_normal((hidden, HD), dtype=np.float32) / np.float32(HD ** 0.5)).half()
           for _ in range(L)]
    wq_dev, wo_dev = [w.to(DEV) for w in w_qkv], [w.to(DEV) for w in w_o]
    wq_ref = [np.ascontiguousarray(w.float().numpy().T) for w in w_qkv]
    wo_ref = [np.ascontiguousarray(w.float().numpy().T) for w in w_o]
    pool = torch.zeros(nb * per_block, dtype=torch.int16, device=DEV)
    tab = cb.rope_cos_sin_table(maxb * bs, D).to(DEV)
    batch = cb.DecodeBatch(nb, bs, mb, maxb, device=DEV)
    rep = BatchReplica(oracle, nb, bs, mb, maxb)
    next_id = 0
    for step in range(24):
        if len(rep.rows) < mb and (not rep.rows or rng.random() < 0.4):
            batch.add(next_id)
            rep.add(next_id)
            next_id += 1
        if len(rep.rows) > 1 and rng.random() < 0.1:
            sid = int(rng.choice(rep.rows))
            batch.release(sid)
            rep.release(sid)
        assert rep.begin_step()
        batch.begin_step()
        rows = batch.rows()
        n = len(rows)
        for layer in range(L):
            x = torch.from_numpy(rng.standard_normal((n, hidden), dtype=np.float32)).half()
            res0 = rng.standard_normal((n, hidden), dtype=np.float32)
            res = torch.from_numpy(res0).to(DEV)
            q = torch.empty((n, H, D), dtype=torch.float16, device=DEV)
            att = cb.attention_block(batch, x.to(DEV), wq_dev[layer], wo_dev[layer], res, pool, tab, num_heads=H,
                                     num_kv_heads=Hkv, head_dim=D, num_layers=L, layer=layer, query_out=q)
            torch.cuda.synchronize()
            hpool = pool.cpu().numpy().view(np.uint16)
            qh, ah = q.float().cpu().numpy().reshape(n, HD), att.float().cpu().numpy()
            proj = oracle.gemm(x.float().numpy(), wq_ref[layer])
            for r, sid in enumerate(rows):
                pos, blocks = rep.seq[sid]
                # 1. projection + RoPE: fp16 rounding of the query on top of the projection bound
                qr = oracle.rope(proj[r, :HD], pos, H, D)
                assert np.all(np.abs(qh[r] - qr) <= 2 * PROJ_TOL + np.abs(qr) * 2.0 ** -11), (step, layer, sid)
                # 2. the appended K/V row: truncation loses up to one fp16 ulp
                kr = oracle.rope(proj[r, HD:HD + KD], pos, Hkv, D)
                for kv, ref in ((0, kr), (1, proj[r, HD + KD:])):
                    # elem(blk, layer, kv, t, h, d), paged_attention_cpu.cpp:63-67
                    o = (((blocks[pos // bs] * L + layer) * 2 + kv) * bs + pos % bs) * KD
                    got = hpool[o:o + KD].view(np.float16).astype(np.float32)
                    assert np.all(np.abs(got - ref) <= 2 * PROJ_TOL + np.abs(ref) * 2.0 ** -9), (step, layer, kv)
                # 3. attention over the pool the kernels wrote, with the kernel's rotated query
                ref = oracle.paged_attention(qh[r], hpool, blocks, pos + 1, layer, H, Hkv, D, bs, L)
                assert max_abs(ah[r], ref.reshape(-1)) <= tol_for(torch.float16), (step, layer, sid)
            # 4. O-projection + residual on the kernel's attention output
            exp = oracle.gemm(ah, wo_ref[layer]) + res0
            assert max_abs(res.cpu().numpy(), exp) <= PROJ_TOL, (step, layer)
        batch.end_step()
        rep.end_step()
    assert next_id >= 6
