"""Output projection + residual add (cottus_o_proj_residual) against the
oracle: gemmCPU restated (pinned to the reference's own by the golden
vectors), then residualAddCPU (compute_primitives_cpu.cpp:74-82), the two
steps of generic_transformer.cpp:305-327 per layer and token.

The projection sums in a different order than gemmCPU (fp32 tensor-core
accumulation over k-tiles and K splits), so results are compared within
PROJ_TOL, plus half an fp16 ulp of the result when the output is fp16.
"""
import numpy as np
import pytest
import torch

from helpers import max_abs

pytestmark = pytest.mark.gpu

cb = pytest.importorskip("cottus_b200")

DEV = "cuda"
PROJ_TOL = 2e-4  # |projection - gemmCPU| for N(0,1) activations and N(0, 1/in) weights


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


SHAPES = {
    # in_features (num_heads * head_dim), out_features (hidden), batch
    "tinyllama_b1": (2048, 2048, 1),
    "tinyllama_b13": (2048, 2048, 13),
    "tinyllama_b70": (2048, 2048, 70),  # two launches of at most 64 tokens
    "llama3_8b_b32": (4096, 4096, 32),
    "llama3_8b_b64": (4096, 4096, 64),  # the benchmark's shape
    "narrow_b5": (64, 128, 5),  # one k-tile, one row tile
}


def _inputs(name, fin, fout, B):
    rng = np.random.default_rng(sum(map(ord, name)))
    x16 = torch.from_numpy(rng.standard_normal((B, fin), dtype=np.float32)).half()
    w16 = torch.from_numpy(rng.standard_normal((fout, fin), dtype=np.float32) / np.float32(np.sqrt(fin))).half()
    res = rng.standard_normal((B, fout), dtype=np.float32)
    return x16, w16, res


def _expected(oracle, x16, w16, res):
    # reference layout: wo is [in][out], x = att . wo, then x = x + xb
    proj = oracle.gemm(x16.float().numpy(), np.ascontiguousarray(w16.float().numpy().T))
    return proj + res


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_o_proj_residual_vs_oracle(oracle, name):
    fin, fout, B = SHAPES[name]
    x16, w16, res = _inputs(name, fin, fout, B)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = cb.o_proj_residual(x16.to(DEV), w16.to(DEV), torch.from_numpy(res).to(DEV), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert max_abs(out.cpu().numpy(), _expected(oracle, x16, w16, res)) <= PROJ_TOL


def test_o_proj_residual_in_place_and_fp16(oracle):
    fin, fout, B = 2048, 2048, 9
    x16, w16, res = _inputs("in_place", fin, fout, B)
    exp = _expected(oracle, x16, w16, res)
    xd, wd = x16.to(DEV), w16.to(DEV)
    # in place on the residual stream, as residualAddCUDA(d_x, d_x, d_xb) runs
    stream = torch.from_numpy(res.copy()).to(DEV)
    got = cb.o_proj_residual(xd, wd, stream, out=stream)
    torch.cuda.synchronize()
    assert got.data_ptr() == stream.data_ptr()
    assert max_abs(stream.cpu().numpy(), exp) <= PROJ_TOL
    # fp16 output: the fp32 result rounded once
    h = cb.o_proj_residual(xd, wd, torch.from_numpy(res).to(DEV), out_dtype=torch.float16)
    torch.cuda.synchronize()
    tol = PROJ_TOL + np.abs(exp) * 2.0 ** -11
    assert np.all(np.abs(h.float().cpu().numpy() - exp) <= tol)


def test_o_proj_residual_deterministic():
    fin, fout, B = 4096, 4096, 17
    x16, w16, res = _inputs("det", fin, fout, B)
    xd, wd, rd = x16.to(DEV), w16.to(DEV), torch.from_numpy(res).to(DEV)
    a = cb.o_proj_residual(xd, wd, rd)
    b = cb.o_proj_residual(xd, wd, rd)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_o_proj_residual_rejects_bad_shapes():
    x = torch.zeros((2, 96), dtype=torch.float16, device=DEV)
    w = torch.zeros((128, 96), dtype=torch.float16, device=DEV)
    r = torch.zeros((2, 128), dtype=torch.float32, device=DEV)
    with pytest.raises(cb.CottusError) as e:
        cb.o_proj_residual(x, w, r)
    assert e.value.code == cb.COTTUS_ERR_UNSUPPORTED
    x = torch.zeros((2, 64), dtype=torch.float16, device=DEV)
    w = torch.zeros((100, 64), dtype=torch.float16, device=DEV)
    with pytest.raises(cb.CottusError) as e:
        cb.o_proj_residual(x, w, torch.zeros((2, 100), dtype=torch.float32, device=DEV))
    assert e.value.code == cb.COTTUS_ERR_UNSUPPORTED
