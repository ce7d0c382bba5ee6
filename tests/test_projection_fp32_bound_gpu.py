"""The projections against the reference's fp32 arithmetic.

The reference keeps its weights in fp32 and multiplies in fp32 (gemmCUDA is
cuBLAS SGEMM, compute_primitives_cuda.cu:30-55; its CPU twin gemmCPU,
called at generic_transformer.cpp:169-176 and 305-307).  cottus_qkv_rope_append
and cottus_o_proj_residual take fp16 weights and activations and accumulate
in fp32 on the tensor cores.  Here the inputs are drawn in fp32, the GPU
gets their fp16 roundings, and the result is compared with gemmCPU
(restated, pinned to the reference's own) on the UNROUNDED fp32 values.

Elementwise bound: with u = 2^-11 (fp16 rounding) and v = 2^-24 (fp32),
each product x~ w~ differs from x w by at most |x w| (2u + u^2), plus the
absolute error of a weight or activation that rounds into the fp16
subnormal range (at most 2^-25, times the other factor); both sums are
fp32 accumulations of K terms in different orders, each within K v of
sum |x w|.  So for every output n

    |gpu_n - ref_n| <= sum_k |x_k w_nk| (2u + u^2 + 2 K v)
                       + 2^-25 sum_k (|x_k| + |w_nk|) (1 + 2u)

The test asserts this bound for every output, and a max-abs error of at
most 5e-3 at these shapes (N(0,1) activations, N(0, 1/K) weights; about
4.5 standard deviations of the rounding error's random walk over K = 4096
terms).  The residual add of the O-projection is exact in fp32 up to v.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")

DEV = "cuda"
U16, U32 = 2.0 ** -11, 2.0 ** -24
MAX_ABS_FP32_REF = 5e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _bound(x, w):
    """Elementwise worst-case error bound [B][N] for x [B][K] @ w[N][K]^T."""
    K = x.shape[1]
    ax, aw = np.abs(x.astype(np.float64)), np.abs(w.astype(np.float64))
    rel = 2 * U16 + U16 * U16 + 2 * K * U32
    sub = 2.0 ** -25 * (ax.sum(1, keepdims=True) + aw.sum(1)[None, :]) * (1 + 2 * U16)
    return (ax @ aw.T) * rel + sub


def _draw(seed, B, K, N):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(K))
    return x, w


def test_qkv_projection_vs_fp32_reference_llama3_8b_b64(oracle):
    hidden, H, Hkv, D, B = 4096, 32, 8, 128, 64  # the benchmark's shape
    N = (H + 2 * Hkv) * D
    x, w = _draw(41, B, hidden, N)
    bs, L, maxb = 16, 1, 4
    nb = B * maxb
    tables = np.arange(nb, dtype=np.int32).reshape(B, maxb)
    pos = np.full(B, 5, np.int32)
    pool = torch.zeros(nb * 2 * L * bs * Hkv * D, dtype=torch.int16, device=DEV)
    tab = cb.rope_cos_sin_table(maxb * bs, D).to(DEV)
    qkv = torch.zeros((B, N), dtype=torch.float32, device=DEV)
    cb.qkv_rope_append(torch.from_numpy(x).half().to(DEV), torch.from_numpy(w).half().to(DEV),
                       torch.from_numpy(pos).to(DEV), tab, pool, torch.from_numpy(tables).to(DEV), num_heads=H,
                       num_kv_heads=Hkv, head_dim=D, block_size=bs, num_layers=L, qkv_out=qkv)
    torch.cuda.synchronize()
    got = qkv.cpu().numpy().astype(np.float64)
    ref = oracle.gemm(x, np.ascontiguousarray(w.T)).astype(np.float64)
    err = np.abs(got - ref)
    assert np.all(err <= _bound(x, w)), f"rounding bound exceeded by {float(np.max(err - _bound(x, w)))}"
    assert float(err.max()) <= MAX_ABS_FP32_REF, float(err.max())


def test_o_projection_vs_fp32_reference_llama3_8b_b64(oracle):
    fin, fout, B = 4096, 4096, 64  # the benchmark's shape
    x, w = _draw(43, B, fin, fout)
    res = np.random.default_rng(44).standard_normal((B, fout), dtype=np.float32)
    out = cb.o_proj_residual(torch.from_numpy(x).half().to(DEV), torch.from_numpy(w).half().to(DEV),
                             torch.from_numpy(res).to(DEV))
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    ref = (oracle.gemm(x, np.ascontiguousarray(w.T)) + res).astype(np.float64)
    err = np.abs(got - ref)
    bound = _bound(x, w) + (np.abs(ref) + np.abs(res)) * 2 * U32
    assert np.all(err <= bound), f"rounding bound exceeded by {float(np.max(err - bound))}"
    assert float(err.max()) <= MAX_ABS_FP32_REF, float(err.max())
