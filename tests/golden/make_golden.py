"""Generates tests/golden/golden.npz from the reference's own CPU code.

Run where the reference tree exists (it is compiled by `make -C oracle ref
engine` into oracle/_ref/):

    python tests/golden/make_golden.py

Everything stored comes out of the reference library (paged attention,
RoPE, gemmCPU, block allocator, page-table bounds, and the KV cache written
by GenericTransformer::forwardToken); inputs are regenerated from cases.py and
only their SHA-256 is stored.
"""
from __future__ import annotations

import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402
from oracle.oracle import REF_ENGINE_SO, Reference  # noqa: E402


def attention_via_ref(ref: Reference, c):
    out = np.zeros((len(c["ctx"]), c["H"], c["D"]), np.float32)
    for b, n in enumerate(c["ctx"]):
        nblk = (int(n) + c["bs"] - 1) // c["bs"]
        out[b] = ref.paged_attention(c["q"][b], c["kv"], c["tables"][b][:nblk], int(n), c["layer"], c["H"],
                                     c["Hkv"], c["D"], c["bs"], c["L"])
    return out


def engine_append_golden():
    e = cases.ENGINE_CASE
    w = cases.engine_weights(e)
    lib = C.CDLL(str(REF_ENGINE_SO))
    fp = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
    lib.ref_forward_token_kv.restype = C.c_int
    lib.ref_forward_token_kv.argtypes = ([C.c_int32] * 7 + [C.c_float, C.c_float] + [fp] * 12 +
                                         [C.c_int32, C.c_int32,
                                          np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"), C.c_int32,
                                          np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"), fp, fp])
    per_block = 2 * 1 * e["bs"] * e["Hkv"] * e["D"]
    kv = np.zeros(e["pool_blocks"] * per_block, np.uint16)
    table = np.array(e["table"], np.int32)
    ks, vs = [], []
    for pos, tok in enumerate(e["tokens"]):
        k = np.zeros(e["Hkv"] * e["D"], np.float32)
        v = np.zeros_like(k)
        rc = lib.ref_forward_token_kv(e["vocab"], e["hidden"], e["H"], e["Hkv"], e["D"], e["inter"], e["bs"],
                                      e["theta"], e["eps"], w["embed"], w["attn_norm"], w["wq"], w["wk"], w["wv"],
                                      w["wo"], w["w1"], w["w2"], w["w3"], w["ffn_norm"], w["out_norm"],
                                      w["lm_head"], tok, pos, table, len(table), kv, k, v)
        assert rc == 0, rc
        ks.append(k)
        vs.append(v)
    return np.stack(ks), np.stack(vs), kv


def main():
    ref = Reference()
    out, meta = {}, {}

    for name, c in cases.kat_cases().items():
        o = attention_via_ref(ref, c)
        out[f"{name}/out"] = o
        meta[name] = dict(kind="kat", input_sha=cases.sha(c["q"], c["kv"], c["tables"], c["ctx"]))

    for name in cases.SHAPE_CASES:
        c = cases.make_shape_case(name)
        out[f"{name}/out"] = attention_via_ref(ref, c)
        meta[name] = dict(kind="shape", input_sha=cases.sha(c["q"], c["kv"], c["tables"], c["ctx"]))

    r = cases.rope_cases()
    out["rope/kat_out"] = ref.rope(r["kat_in"], 5, 2, 8)
    # (cos, sin) of the reference formula via unit inputs: x0=1, x1=0 gives (cos, sin) exactly
    unit = np.zeros(64, np.float32)
    unit[0::2] = 1.0
    out["rope/cos_sin_d64"] = np.stack([ref.rope(unit, int(p), 1, 64).reshape(32, 2) for p in r["positions"]])
    unit128 = np.zeros(128, np.float32)
    unit128[0::2] = 1.0
    out["rope/cos_sin_d128"] = np.stack([ref.rope(unit128, int(p), 1, 128).reshape(64, 2)
                                         for p in r["positions"]])
    out["rope/x64_out"] = np.stack([ref.rope(r["x64"], int(p), 4, 64) for p in r["positions"]])
    meta["rope"] = dict(input_sha=cases.sha(r["positions"], r["kat_in"], r["x64"]))

    for name, (a, b) in cases.gemm_cases().items():
        out[f"gemm/{name}"] = ref.gemm(a, b)
        meta[f"gemm/{name}"] = dict(input_sha=cases.sha(a, b))

    ops, total = cases.allocator_ops()
    a = ref.allocator(total, 16)
    trace, live = cases.run_allocator_ops(a, ops)
    out["allocator/trace"] = trace
    out["allocator/num_free"] = np.array([a.num_free()], np.int64)
    # error behaviour: invalid id, double free, exhaustion
    b = ref.allocator(2, 16)
    errs = [b.free(5), b.free(-1)]
    x = b.alloc()
    errs += [b.free(x), b.free(x)]
    b.alloc(); b.alloc()
    errs += [b.alloc()]
    out["allocator/errors"] = np.array(errs, np.int64)
    meta["allocator"] = dict(input_sha=cases.sha(ops))

    blocks = np.array([4, 9, 2], np.int32)
    out["page_table/get"] = np.array([ref.page_table_get(blocks, 16, i) for i in (-1, 0, 1, 2, 3, 100)], np.int64)

    if REF_ENGINE_SO.exists():
        k, v, kv = engine_append_golden()
        out["engine_append/k_rot"] = k
        out["engine_append/v"] = v
        out["engine_append/kv_cache"] = kv
        meta["engine_append"] = dict(input_sha=cases.sha(*cases.engine_weights().values()))

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden_manifest.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} arrays, {(HERE / 'golden.npz').stat().st_size} bytes")


if __name__ == "__main__":
    main()
