"""Seeded input definitions for the golden fixtures.

The inputs are regenerated from these definitions (numpy PCG64 seeds), so the
fixture file only stores the reference's outputs plus a SHA-256 of every
input, which the tests check first to catch generator drift.

KV values are fp32 N(0,1) draws stored through the reference's truncating
fp16 encoder (generic_transformer.cpp:255-262), i.e. exactly what the
reference pipeline would have written into its cache.
"""
from __future__ import annotations

import hashlib

import numpy as np


def fp32_to_fp16_trunc(f: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32)
    sign = (bits & 0x80000000) >> 16
    e = ((bits & 0x7F800000) >> 23).astype(np.int64) - 112
    m = (bits & 0x007FFFFF) >> 13
    out = np.where(e <= 0, sign, np.where(e >= 31, sign | 0x7C00, sign | (np.clip(e, 0, 31) << 10) | m))
    return out.astype(np.uint16)


def fp16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.asarray(h, dtype=np.uint16).astype(np.uint32)
    sign = (h & 0x8000) << 16
    e = (h & 0x7C00) >> 10
    m = h & 0x03FF
    bits = np.where(e == 0, 0, sign | ((e + 112) << 23) | (m << 13)).astype(np.uint32)
    return bits.view(np.float32)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# -- known-answer cases of the reference tests ------------------------------------
# tests/test_paged_attention_cpu.cpp:26-172 and tests/test_paged_attention_parity.cpp:178-215.

def kat_cases():
    enc = lambda x: int(fp32_to_fp16_trunc(np.array([x], np.float32))[0])
    cases = {}
    # single head, single block, bs 2, D 4 (expected ~1.378)
    kv = np.full(16, enc(0.0), np.uint16)
    kv[0] = enc(1.0); kv[4] = enc(0.0); kv[5] = enc(1.0)
    kv[8:12] = enc(1.0); kv[12:16] = enc(2.0)
    cases["kat_single_head"] = dict(H=1, Hkv=1, D=4, bs=2, L=1, layer=0, q=np.array([[1, 0, 0, 0]], np.float32),
                                    kv=kv, tables=[[0]], ctx=[2])
    # two heads, one token: output == V
    kv = np.zeros(8, np.uint16)
    kv[0] = enc(1.0); kv[1] = enc(0.0); kv[2] = enc(0.0); kv[3] = enc(1.0)
    kv[4] = enc(2.0); kv[5] = enc(0.0); kv[6] = enc(0.0); kv[7] = enc(3.0)
    cases["kat_multi_head"] = dict(H=2, Hkv=2, D=2, bs=1, L=1, layer=0, q=np.array([[1, 0, 0, 1]], np.float32),
                                   kv=kv, tables=[[0]], ctx=[1])
    # three tokens over two blocks: mean of V == 2
    kv = np.zeros(16, np.uint16)
    kv[0] = enc(1.0); kv[2] = enc(1.0); kv[4] = enc(1.0); kv[6] = enc(2.0)
    kv[8] = enc(1.0); kv[12] = enc(3.0)
    cases["kat_multi_block"] = dict(H=1, Hkv=1, D=2, bs=2, L=1, layer=0, q=np.array([[1, 0]], np.float32),
                                    kv=kv, tables=[[0, 1]], ctx=[3])
    # determinism case: everything 1.0, H=Hkv=2, D=4, bs 2, 3 tokens
    kv = np.full(2 * 2 * 2 * 2 * 4, enc(1.0), np.uint16)
    cases["kat_determinism"] = dict(H=2, Hkv=2, D=4, bs=2, L=1, layer=0, q=np.ones((1, 8), np.float32),
                                    kv=kv, tables=[[0, 1]], ctx=[3])
    for c in cases.values():
        c["tables"] = np.array(c["tables"], np.int32)
        c["ctx"] = np.array(c["ctx"], np.int32)
        c["q"] = c["q"].reshape(len(c["ctx"]), c["H"], c["D"])
    return cases


# -- seeded shape cases (reduced sizes of the five workloads) ---------------------

SHAPE_CASES = {
    # TinyLlama fp32 shape, shuffled pool, contexts not multiples of 16
    "tinyllama_f32": dict(H=32, Hkv=4, D=64, bs=16, L=1, layer=0, ctx=[130, 77, 16, 1], extra_blocks=5, seed=101,
                          q_fp16=False),
    # Llama-3-8B GQA shape, fp16-representable Q
    "llama3_8b_f16": dict(H=32, Hkv=8, D=128, bs=16, L=1, layer=0, ctx=[48, 33], extra_blocks=3, seed=102,
                          q_fp16=True),
    # MHA shape, two layers in the pool, attention on layer 1
    "mha_two_layer": dict(H=8, Hkv=8, D=128, bs=16, L=2, layer=1, ctx=[16, 5, 100], extra_blocks=4, seed=103,
                          q_fp16=True),
    # Llama-3-70B shape (group of 8)
    "llama3_70b_f16": dict(H=64, Hkv=8, D=128, bs=16, L=1, layer=0, ctx=[200], extra_blocks=2, seed=104,
                           q_fp16=True),
    # odd sizes: block size 8, D 32, group of 4
    "odd_block8": dict(H=8, Hkv=2, D=32, bs=8, L=3, layer=2, ctx=[9, 64, 3], extra_blocks=7, seed=105,
                       q_fp16=False),
}


def pool_elems(c, num_blocks):
    return num_blocks * 2 * c["L"] * c["bs"] * c["Hkv"] * c["D"]


def make_shape_case(name: str):
    c = dict(SHAPE_CASES[name])
    rng = np.random.default_rng(c["seed"])
    bs = c["bs"]
    nblk = [(x + bs - 1) // bs for x in c["ctx"]]
    total = sum(nblk) + c["extra_blocks"]
    perm = rng.permutation(total).astype(np.int32)
    maxb = max(nblk)
    tables = np.full((len(nblk), maxb), -1, np.int32)
    off = 0
    for b, n in enumerate(nblk):
        tables[b, :n] = perm[off:off + n]
        off += n
    kv = fp32_to_fp16_trunc(rng.standard_normal(pool_elems(c, total), dtype=np.float32))
    q = rng.standard_normal((len(nblk), c["H"], c["D"]), dtype=np.float32)
    if c["q_fp16"]:
        q = fp16_bits_to_f32(fp32_to_fp16_trunc(q))
    c.update(kv=kv, q=q, tables=tables, ctx=np.array(c["ctx"], np.int32), num_blocks=total)
    return c


# -- RoPE -----------------------------------------------------------------------

ROPE_POSITIONS = [0, 1, 2, 5, 15, 16, 17, 100, 1023, 1024, 2047, 4095]


def rope_cases():
    rng = np.random.default_rng(201)
    pos = ROPE_POSITIONS + sorted(rng.integers(0, 4096, 36).tolist())
    # tests/test_compute_primitives_parity.cpp:118-160 input: (i % 10) * 0.1, pos 5, H 2, D 8
    kat_in = np.array([(i % 10) * 0.1 for i in range(16)], np.float32)
    x64 = rng.standard_normal((4, 64), dtype=np.float32)
    return dict(positions=np.array(pos, np.int32), kat_in=kat_in, x64=x64)


# -- allocator churn --------------------------------------------------------------

def gemm_cases():
    """Inputs of gemmCPU (compute_primitives_cpu.cpp:6-23) golden vectors:
    decode-shaped products (one to a few tokens x a projection), fp16-valued
    operands stored as float, as the fused QKV step uses them."""
    rng = np.random.default_rng(401)
    out = {}
    for name, (m, k, n) in {"m1": (1, 256, 192), "m5": (5, 128, 320)}.items():
        a = fp16_bits_to_f32(fp32_to_fp16_trunc(rng.standard_normal((m, k), dtype=np.float32)))
        b = fp16_bits_to_f32(fp32_to_fp16_trunc(rng.standard_normal((k, n), dtype=np.float32) / np.float32(16)))
        out[name] = (a.reshape(m, k), b.reshape(k, n))
    return out


def allocator_ops(seed=301, n_ops=10000, total=512):
    """Seeded alloc/free op list: +1 = alloc, -k-1 = free the k-th live block."""
    rng = np.random.default_rng(seed)
    ops = []
    live = 0
    for _ in range(n_ops):
        if live == 0 or (live < total and rng.random() < 0.55):
            ops.append(1)
            live += 1
        else:
            ops.append(-int(rng.integers(0, live)) - 1)
            live -= 1
    return np.array(ops, np.int64), total


def run_allocator_ops(alloc, ops):
    """Replays `ops` on an allocator object with alloc()/free(); returns the
    id sequence (alloc results, then freed ids as -(id+1))."""
    live, trace = [], []
    for op in ops:
        if op == 1:
            i = alloc.alloc()
            trace.append(i)
            live.append(i)
        else:
            k = -op - 1
            i = live.pop(k)
            rc = alloc.free(i)
            assert rc == 0
            trace.append(-(i + 1))
    return np.array(trace, np.int64), live


# -- engine-driven KV append (reference GenericTransformer) -----------------------

ENGINE_CASE = dict(vocab=16, hidden=32, H=4, Hkv=2, D=8, inter=64, bs=4, theta=10000.0, eps=1e-5,
                   tokens=[3, 7, 1, 0, 9, 12, 5, 5, 2, 15], table=[5, 2, 7], pool_blocks=8, seed=401)


def engine_weights(c=ENGINE_CASE):
    rng = np.random.default_rng(c["seed"])
    h, H, Hkv, D, it, V = c["hidden"], c["H"], c["Hkv"], c["D"], c["inter"], c["vocab"]
    w = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.2).astype(np.float32)
    return dict(embed=w(V, h), attn_norm=1.0 + w(h), wq=w(h, H * D), wk=w(h, Hkv * D), wv=w(h, Hkv * D),
                wo=w(H * D, h), w1=w(h, it), w2=w(it, h), w3=w(h, it), ffn_norm=1.0 + w(h),
                out_norm=1.0 + w(h), lm_head=w(h, V))
