"""The fused QKV projection + RoPE + KV append (cottus_qkv_rope_append)
against the oracle: gemmCPU restated (pinned to the reference's own by the
golden vectors), ropeCPU and the restated append (generic_transformer.cpp:
169-284 per token).

The projection sums in a different order than gemmCPU (fp32 tensor-core
accumulation over k-tiles and K splits), so the projections are compared
within PROJ_TOL; the epilogue is then checked bit for bit: the rotated query
and every KV byte equal ropeCPU and the restated append applied to the
kernel's own projections.  Finally the attention over the appended cache
(cottus_paged_decode on the rotated query) is compared with the oracle.
"""
import numpy as np
import pytest
import torch

from helpers import TOL_F16, max_abs

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")

DEV = "cuda"
PROJ_TOL = 2e-4  # |projection - gemmCPU| for N(0,1) activations and N(0, 1/hidden) weights


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


SHAPES = {
    # hidden, H, Hkv, D, batch
    "tinyllama_b1": (2048, 32, 4, 64, 1),
    "tinyllama_b7": (2048, 32, 4, 64, 7),
    "tinyllama_b70": (2048, 32, 4, 64, 70),  # two launches of at most 64 tokens
    "llama3_8b_b16": (4096, 32, 8, 128, 16),
    "llama3_8b_b64": (4096, 32, 8, 128, 64),  # the benchmark's shape
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_qkv_rope_append_vs_oracle(oracle, name):
    hidden, H, Hkv, D, B = SHAPES[name]
    bs, L, layer, maxb = 16, 2, 1, 8
    N = (H + 2 * Hkv) * D
    rng = np.random.default_rng(sum(map(ord, name)))
    x16 = torch.from_numpy(rng.standard_normal((B, hidden), dtype=np.float32)).half()
    w16 = torch.from_numpy(rng.standard_normal((N, hidden), dtype=np.float32) / np.float32(np.sqrt(hidden))).half()
    nb = B * maxb + 3
    tables = rng.permutation(nb)[:B * maxb].reshape(B, maxb).astype(np.int32)
    pos = rng.integers(0, maxb * bs, size=B).astype(np.int32)
    per_block = 2 * L * bs * Hkv * D
    pool0 = cb_encode(rng.standard_normal(nb * per_block, dtype=np.float32))
    tab = cb.rope_cos_sin_table(maxb * bs, D).to(DEV)
    pool = torch.from_numpy(pool0.view(np.int16).copy()).to(DEV)
    qkv = torch.zeros((B, N), dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    qf32 = cb.qkv_rope_append(x16.to(DEV), w16.to(DEV), torch.from_numpy(pos).to(DEV), tab, pool,
                              torch.from_numpy(tables).to(DEV), num_heads=H, num_kv_heads=Hkv, head_dim=D,
                              block_size=bs, num_layers=L, layer=layer, query_out_dtype=torch.float32,
                              qkv_out=qkv, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = qkv.cpu().numpy()
    # 1. the projection against gemmCPU on the same fp16 values (reference layout [hidden][out])
    ref = oracle.gemm(x16.float().numpy(), np.ascontiguousarray(w16.float().numpy().T))
    assert max_abs(got, ref) <= PROJ_TOL
    # 2. the epilogue, bit for bit, from the kernel's own projections
    HD, KD = H * D, Hkv * D
    hpool = pool0.copy()
    qrot = np.zeros((B, HD), np.float32)
    for b in range(B):
        p = int(pos[b])
        qrot[b] = oracle.rope(got[b, :HD], p, H, D)
        kr = oracle.rope(got[b, HD:HD + KD], p, Hkv, D)
        oracle.kv_append(hpool, kr, got[b, HD + KD:], tables[b, :p // bs + 1], p, layer, Hkv, D, bs, L)
    np.testing.assert_array_equal(qf32.cpu().numpy().reshape(B, HD).view(np.uint32), qrot.view(np.uint32))
    np.testing.assert_array_equal(pool.cpu().numpy().view(np.uint16), hpool)
    # 3. attention over the appended cache with the fp16 rotated query, as a decode step would run it
    q16 = cb.qkv_rope_append(x16.to(DEV), w16.to(DEV), torch.from_numpy(pos).to(DEV), tab, pool,
                             torch.from_numpy(tables).to(DEV), num_heads=H, num_kv_heads=Hkv, head_dim=D,
                             block_size=bs, num_layers=L, layer=layer, query_out_dtype=torch.float16)
    out = cb.paged_decode(q16.view(B, H, D), pool, torch.from_numpy(tables).to(DEV),
                          torch.from_numpy(pos + 1).to(DEV), num_kv_heads=Hkv, head_dim=D, block_size=bs,
                          num_layers=L, layer=layer, num_physical_blocks=nb)
    torch.cuda.synchronize()
    q16h = q16.float().cpu().numpy().reshape(B, HD)
    for b in range(B):
        p = int(pos[b])
        r = oracle.paged_attention(q16h[b], hpool, tables[b, :p // bs + 1], p + 1, layer, H, Hkv, D, bs, L)
        assert max_abs(out[b].float().cpu(), r.reshape(H, D)) <= TOL_F16


def test_rejects_unsupported_shapes():
    x = torch.zeros((2, 96), dtype=torch.float16, device=DEV)  # hidden not a multiple of 64
    w = torch.zeros((3 * 64, 96), dtype=torch.float16, device=DEV)
    tab = cb.rope_cos_sin_table(32, 64).to(DEV)
    pool = torch.zeros(4 * 2 * 16 * 64, dtype=torch.int16, device=DEV)
    with pytest.raises(cb.CottusError) as e:
        cb.qkv_rope_append(x, w, torch.zeros(2, dtype=torch.int32, device=DEV), tab, pool,
                           torch.zeros((2, 2), dtype=torch.int32, device=DEV), num_heads=1, num_kv_heads=1,
                           head_dim=64, block_size=16)
    assert e.value.code == cb.COTTUS_ERR_UNSUPPORTED


def cb_encode(f):
    import cases
    return cases.fp32_to_fp16_trunc(f)
