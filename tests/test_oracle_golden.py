"""Pins the C restatement (oracle/oracle.c) against the reference.

Golden outputs in tests/golden/golden.npz come from the reference's own CPU
code (tests/golden/make_golden.py).  Where the compiled reference library is
present (oracle/_ref/), the restatement is also compared with it directly on
fresh seeded inputs.  Everything here is bit-exact: the restatement performs
the same fp32 operations in the same order as the reference.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import cases
from oracle.oracle import OracleError, Reference, reference_available

MANIFEST = json.loads((Path(__file__).parent / "golden" / "golden_manifest.json").read_text())


def _oracle_attention(oracle, c):
    out = np.zeros((len(c["ctx"]), c["H"], c["D"]), np.float32)
    for b, n in enumerate(c["ctx"]):
        nblk = (int(n) + c["bs"] - 1) // c["bs"]
        out[b] = oracle.paged_attention(c["q"][b], c["kv"], c["tables"][b][:nblk], int(n), c["layer"], c["H"],
                                        c["Hkv"], c["D"], c["bs"], c["L"])
    return out


@pytest.mark.parametrize("name", sorted(cases.kat_cases()))
def test_kat_bit_exact(oracle, golden, name):
    c = cases.kat_cases()[name]
    assert cases.sha(c["q"], c["kv"], c["tables"], c["ctx"]) == MANIFEST[name]["input_sha"]
    got = _oracle_attention(oracle, c)
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"{name}/out"].view(np.uint32))


def test_kat_expected_values(golden):
    # hand-computed expectations of tests/test_paged_attention_cpu.cpp:67-76, :120-126, :167-169
    np.testing.assert_allclose(golden["kat_single_head/out"].ravel(), 0.622 + 0.378 * 2, atol=0.01)
    np.testing.assert_allclose(golden["kat_multi_head/out"].ravel(), [2, 0, 0, 3], atol=0.01)
    assert abs(golden["kat_multi_block/out"].ravel()[0] - 2.0) < 0.1


@pytest.mark.parametrize("name", sorted(cases.SHAPE_CASES))
def test_shape_cases_bit_exact(oracle, golden, name):
    c = cases.make_shape_case(name)
    assert cases.sha(c["q"], c["kv"], c["tables"], c["ctx"]) == MANIFEST[name]["input_sha"]
    got = _oracle_attention(oracle, c)
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"{name}/out"].view(np.uint32))


def test_rope_bit_exact(oracle, golden):
    r = cases.rope_cases()
    assert cases.sha(r["positions"], r["kat_in"], r["x64"]) == MANIFEST["rope"]["input_sha"]
    np.testing.assert_array_equal(oracle.rope(r["kat_in"], 5, 2, 8), golden["rope/kat_out"])
    for i, p in enumerate(r["positions"]):
        np.testing.assert_array_equal(oracle.rope(r["x64"], int(p), 4, 64), golden["rope/x64_out"][i])
        cs = np.array([oracle.rope_cos_sin(int(p), d, 64) for d in range(32)], np.float32)
        np.testing.assert_array_equal(cs, golden["rope/cos_sin_d64"][i])
        cs = np.array([oracle.rope_cos_sin(int(p), d, 128) for d in range(64)], np.float32)
        np.testing.assert_array_equal(cs, golden["rope/cos_sin_d128"][i])


@pytest.mark.parametrize("name", sorted(cases.gemm_cases()))
def test_gemm_bit_exact(oracle, golden, name):
    """gemmCPU restated (the fused QKV projection's oracle) against the reference's own."""
    a, b = cases.gemm_cases()[name]
    assert cases.sha(a, b) == MANIFEST[f"gemm/{name}"]["input_sha"]
    np.testing.assert_array_equal(oracle.gemm(a, b).view(np.uint32), golden[f"gemm/{name}"].view(np.uint32))


def test_allocator_trace(oracle, golden):
    ops, total = cases.allocator_ops()
    a = oracle.allocator(total, 16)
    trace, _ = cases.run_allocator_ops(a, ops)
    np.testing.assert_array_equal(trace, golden["allocator/trace"])
    assert a.num_free() == golden["allocator/num_free"][0]
    b = oracle.allocator(2, 16)
    errs = [b.free(5), b.free(-1)]
    x = b.alloc()
    errs += [b.free(x), b.free(x)]
    b.alloc(); b.alloc()
    errs += [b.alloc()]
    np.testing.assert_array_equal(errs, golden["allocator/errors"])


def test_first_allocation_is_zero(oracle):
    a = oracle.allocator(8, 16)
    assert [a.alloc() for _ in range(3)] == [0, 1, 2]


def test_kv_append_matches_forward_token(oracle, golden):
    """The restated encoder + scatter reproduces, bit for bit, the cache that
    the reference's GenericTransformer::forwardToken wrote."""
    if "engine_append/kv_cache" not in golden:
        pytest.skip("engine golden not generated")
    e = cases.ENGINE_CASE
    per_block = 2 * e["bs"] * e["Hkv"] * e["D"]
    kv = np.zeros(e["pool_blocks"] * per_block, np.uint16)
    table = np.array(e["table"], np.int32)
    for pos in range(len(e["tokens"])):
        oracle.kv_append(kv, golden["engine_append/k_rot"][pos], golden["engine_append/v"][pos], table, pos, 0,
                         e["Hkv"], e["D"], e["bs"], 1)
    np.testing.assert_array_equal(kv, golden["engine_append/kv_cache"])
    assert np.count_nonzero(kv) > 0


def test_encoder_edge_cases(oracle):
    vals = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65536.0, 1e-5, -1e-8, np.inf, -np.inf, np.nan, 1.0009765625,
                     1.00048828125, 6.103515625e-05, 6.1e-05], np.float32)
    got = oracle.fp32_to_fp16_trunc(vals)
    want = np.array([oracle.lib.oracle_fp32_to_fp16_trunc(float(v)) for v in vals], np.uint16)
    np.testing.assert_array_equal(got, want)
    # truncation, not round-to-nearest; subnormal range flushes to signed zero; overflow/NaN -> inf
    assert got[2] == 0x3C00 and got[12] == 0x3C00  # 1 + 2^-11 truncates to 1.0
    assert got[6] == 0x0000 and got[7] == 0x8000
    assert got[5] == 0x7C00 and got[10] == 0x7C00 and got[9] == 0xFC00
    # decoder: subnormals and zero decode to +0, exp 31 decodes finite
    h = np.array([0x0001, 0x8001, 0x7C00, 0x3C00], np.uint16)
    d = oracle.fp16_to_fp32(h)
    assert d[0] == 0 and d[1] == 0 and np.isfinite(d[2]) and d[3] == 1.0
    np.testing.assert_array_equal(d, [oracle.lib.oracle_fp16_to_fp32(int(x)) for x in h])


def test_out_of_range_and_invalid(oracle):
    kv = np.zeros(64, np.uint16)
    q = np.zeros(4, np.float32)
    with pytest.raises(OracleError) as e:
        oracle.paged_attention(q, kv, [0], 3, 0, 1, 1, 4, 2, 1)  # 3 tokens, one block of 2
    assert e.value.rc == -2
    with pytest.raises(OracleError) as e:
        oracle.paged_attention(q, kv, [0], 0, 0, 1, 1, 4, 2, 1)
    assert e.value.rc == -1


@pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")
def test_restatement_vs_reference_random():
    """Fresh random inputs, restatement vs the compiled reference, bit for bit."""
    from oracle.oracle import Oracle

    o, r = Oracle(), Reference()
    rng = np.random.default_rng(7)
    for trial in range(6):
        H, Hkv = [(4, 1), (8, 2), (6, 3), (16, 16), (32, 4), (12, 4)][trial]
        D, bs, L = [16, 32, 24, 64, 64, 128][trial], [1, 4, 16, 8, 16, 16][trial], 1 + trial % 3
        layer = trial % L
        n = int(rng.integers(1, 90))
        nblk = (n + bs - 1) // bs
        pool = nblk + 3
        table = rng.permutation(pool)[:nblk].astype(np.int32)
        kv = cases.fp32_to_fp16_trunc(rng.standard_normal(pool * 2 * L * bs * Hkv * D, dtype=np.float32))
        q = rng.standard_normal(H * D, dtype=np.float32) * 2
        a = o.paged_attention(q, kv, table, n, layer, H, Hkv, D, bs, L)
        b = r.paged_attention(q, kv, table, n, layer, H, Hkv, D, bs, L)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        x = rng.standard_normal(H * D, dtype=np.float32)
        p = int(rng.integers(0, 10000))
        np.testing.assert_array_equal(o.rope(x, p, H, D), r.rope(x, p, H, D))
