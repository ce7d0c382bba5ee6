"""ctypes bindings for the CPU oracle (test infrastructure only).

`Oracle` wraps oracle/liboracle.so, the C restatement of the reference's CPU
path (oracle.c).  `Reference` wraps oracle/_ref/libcottus_ref.so, the
reference's own CPU sources compiled by oracle/Makefile.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module,
as the checker; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libcottus_ref.so"
REF_ENGINE_SO = HERE / "_ref" / "libcottus_ref_engine.so"

OK, INVALID_ARGUMENT, OUT_OF_RANGE, RUNTIME_ERROR = 0, -1, -2, -3

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i32, _f32, _i64 = C.c_int32, C.c_float, C.c_int64


def _sig(fn, res, *args):
    fn.restype = res
    fn.argtypes = list(args)
    return fn


class OracleError(RuntimeError):
    def __init__(self, rc: int):
        super().__init__({INVALID_ARGUMENT: "invalid_argument", OUT_OF_RANGE: "out_of_range",
                          RUNTIME_ERROR: "runtime_error"}.get(rc, f"rc={rc}"))
        self.rc = rc


def _check(rc):
    if rc != OK:
        raise OracleError(rc)


class Oracle:
    """The C restatement (liboracle.so)."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = C.CDLL(str(path))
        self.lib = L
        _sig(L.oracle_fp16_to_fp32, _f32, C.c_uint16)
        _sig(L.oracle_fp32_to_fp16_trunc, C.c_uint16, _f32)
        _sig(L.oracle_paged_attention, C.c_int, _f32p, _f32p, _u16p, _i32p, _i32, _i32, _i32, _i32,
             _i32, _i32, _i32, _i32)
        _sig(L.oracle_paged_attention_batch, C.c_int, _f32p, _f32p, C.c_void_p, _i32p, _i32, _i32p,
             _i32, _i32, _i32, _i32, _i32, _i32, _i32)
        _sig(L.oracle_rope, None, _f32p, _f32p, _i32, _i32, _i32, _f32)
        _sig(L.oracle_gemm, None, _f32p, _f32p, _f32p, _i32, _i32, _i32)
        _sig(L.oracle_rope_cos_sin, None, _i32, _i32, _i32, _f32, C.POINTER(_f32), C.POINTER(_f32))
        _sig(L.oracle_kv_append, C.c_int, _u16p, _f32p, _f32p, _i32p, _i32, _i32, _i32, _i32, _i32,
             _i32, _i32)
        _sig(L.oracle_gather_kv, C.c_int, _u16p, _u16p, C.c_void_p, _i32p, _i32, _i32, _i32, _i32,
             _i32, _i32, _i32)
        _sig(L.oracle_allocator_create, C.c_void_p, _i32, _i32)
        _sig(L.oracle_allocator_destroy, None, C.c_void_p)
        _sig(L.oracle_allocator_alloc, _i32, C.c_void_p)
        _sig(L.oracle_allocator_free, C.c_int, C.c_void_p, _i32)
        _sig(L.oracle_allocator_num_free, _i32, C.c_void_p)

    # -- elementwise ---------------------------------------------------------
    def fp16_to_fp32(self, h: np.ndarray) -> np.ndarray:
        """Vectorised restatement of paged_attention_cpu.cpp:10-22 (numpy)."""
        h = np.asarray(h, dtype=np.uint16).astype(np.uint32)
        sign = (h & 0x8000) << 16
        e = (h & 0x7C00) >> 10
        m = h & 0x03FF
        bits = sign | ((e + 112) << 23) | (m << 13)
        bits = np.where(e == 0, 0, bits).astype(np.uint32)
        return bits.view(np.float32)

    def fp32_to_fp16_trunc(self, f: np.ndarray) -> np.ndarray:
        """Vectorised restatement of generic_transformer.cpp:255-262 (numpy)."""
        bits = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32)
        sign = (bits & 0x80000000) >> 16
        e = ((bits & 0x7F800000) >> 23).astype(np.int64) - 112
        m = (bits & 0x007FFFFF) >> 13
        out = np.where(e <= 0, sign, np.where(e >= 31, sign | 0x7C00, sign | (np.clip(e, 0, 31) << 10) | m))
        return out.astype(np.uint16)

    # -- attention -----------------------------------------------------------
    def paged_attention(self, query, kv, block_table, seq_len, layer, num_heads, num_kv_heads, head_dim,
                        block_size, num_layers):
        out = np.zeros(num_heads * head_dim, np.float32)
        bt = np.ascontiguousarray(block_table, np.int32)
        _check(self.lib.oracle_paged_attention(out, np.ascontiguousarray(query, np.float32).ravel(),
                                               np.ascontiguousarray(kv, np.uint16).ravel(), bt, len(bt),
                                               seq_len, layer, num_heads, num_kv_heads, head_dim,
                                               block_size, num_layers))
        return out.reshape(num_heads, head_dim)

    def paged_attention_batch(self, query, kv, block_table, context_lens, layer, num_heads, num_kv_heads,
                              head_dim, block_size, num_layers, threads: int | None = None,
                              seqs=None):
        """Per-sequence oracle over a batch; sequences run on host threads
        (ctypes drops the GIL).  `seqs` restricts the work to a subset."""
        from concurrent.futures import ThreadPoolExecutor

        q = np.ascontiguousarray(query, np.float32).reshape(len(context_lens), num_heads * head_dim)
        kvf = np.ascontiguousarray(kv, np.uint16).ravel()
        bt = np.ascontiguousarray(block_table, np.int32)
        out = np.zeros_like(q)
        seqs = range(len(context_lens)) if seqs is None else seqs

        def one(b):
            if context_lens[b] == 0:
                return
            row = np.ascontiguousarray(bt[b])
            o = np.zeros(num_heads * head_dim, np.float32)
            _check(self.lib.oracle_paged_attention(o, np.ascontiguousarray(q[b]), kvf, row, len(row),
                                                   int(context_lens[b]), layer, num_heads, num_kv_heads,
                                                   head_dim, block_size, num_layers))
            out[b] = o

        threads = threads or min(32, os.cpu_count() or 1)
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(one, seqs))
        return out.reshape(len(context_lens), num_heads, head_dim)

    # -- rope / append / gather ---------------------------------------------
    def rope(self, x, pos, num_heads, head_dim, theta=10000.0):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        self.lib.oracle_rope(out, x, pos, num_heads, head_dim, theta)
        return out

    def gemm(self, a, b):
        """gemmCPU restated: a [M][K] @ b [K][N] in float, k increasing."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        self.lib.oracle_gemm(c, a, b, a.shape[0], b.shape[1], a.shape[1])
        return c

    def rope_cos_sin(self, pos, pair, head_dim, theta=10000.0):
        c, s = _f32(), _f32()
        self.lib.oracle_rope_cos_sin(pos, pair, head_dim, theta, C.byref(c), C.byref(s))
        return c.value, s.value

    def rope_table(self, max_pos, head_dim, theta=10000.0):
        """[max_pos][head_dim/2][2] (cos, sin) table from the reference formula."""
        t = np.empty((max_pos, head_dim // 2, 2), np.float32)
        for p in range(max_pos):
            for d in range(head_dim // 2):
                t[p, d] = self.rope_cos_sin(p, d, head_dim, theta)
        return t

    def kv_append(self, kv, k, v, block_table, pos, layer, num_kv_heads, head_dim, block_size, num_layers):
        bt = np.ascontiguousarray(block_table, np.int32)
        _check(self.lib.oracle_kv_append(kv, np.ascontiguousarray(k, np.float32).ravel(),
                                         np.ascontiguousarray(v, np.float32).ravel(), bt, len(bt), pos,
                                         layer, num_kv_heads, head_dim, block_size, num_layers))

    def gather_kv(self, kv, block_table, seq_len, layer, num_kv_heads, head_dim, block_size, num_layers):
        bt = np.ascontiguousarray(block_table, np.int32)
        k = np.zeros((seq_len, num_kv_heads, head_dim), np.uint16)
        v = np.zeros_like(k)
        kvf = np.ascontiguousarray(kv, np.uint16)
        _check(self.lib.oracle_gather_kv(k, v, kvf.ctypes.data, bt, len(bt), seq_len, layer, num_kv_heads,
                                         head_dim, block_size, num_layers))
        return k, v

    # -- allocator -----------------------------------------------------------
    def allocator(self, total_blocks, block_size):
        return _Alloc(self.lib, "oracle_allocator", total_blocks, block_size)


class _Alloc:
    def __init__(self, lib, prefix, total, bs):
        self.lib, self.p = lib, prefix
        self.h = getattr(lib, f"{prefix}_create")(total, bs)
        if not self.h:
            raise OracleError(INVALID_ARGUMENT)

    def alloc(self) -> int:
        return int(getattr(self.lib, f"{self.p}_alloc")(self.h))

    def free(self, i) -> int:
        return int(getattr(self.lib, f"{self.p}_free")(self.h, int(i)))

    def num_free(self) -> int:
        return int(getattr(self.lib, f"{self.p}_num_free")(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            getattr(self.lib, f"{self.p}_destroy")(self.h)
            self.h = None


class Reference:
    """The reference's own CPU code (oracle/_ref/libcottus_ref.so)."""

    def __init__(self, path: Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference exists")
        L = C.CDLL(str(path))
        self.lib = L
        _sig(L.ref_paged_attention_cpu, C.c_int, _f32p, _f32p, C.c_void_p, _i32p, _i32, _i32, _i32, _i32,
             _i32, _i32, _i32, _i32)
        _sig(L.ref_paged_attention_cpu_batch, C.c_int, _f32p, _f32p, C.POINTER(C.c_void_p), _i32p, _i32,
             _i32p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32)
        _sig(L.ref_rope_cpu, None, _f32p, _f32p, _i32, _i32, _i32, _f32)
        _sig(L.ref_gemm_cpu, None, _f32p, _f32p, _f32p, _i32, _i32, _i32)
        _sig(L.ref_allocator_create, C.c_void_p, _i32, _i32)
        _sig(L.ref_allocator_destroy, None, C.c_void_p)
        _sig(L.ref_allocator_alloc, _i32, C.c_void_p)
        _sig(L.ref_allocator_free, C.c_int, C.c_void_p, _i32)
        _sig(L.ref_allocator_num_free, _i32, C.c_void_p)
        _sig(L.ref_page_table_get, _i32, _i32p, _i32, _i32, _i32)

    def paged_attention(self, query, kv, block_table, seq_len, layer, num_heads, num_kv_heads, head_dim,
                        block_size, num_layers, kv_base_elems: int = 0):
        """One sequence through cottus::pagedAttentionCPU.  `kv_base_elems`
        rebases the pool pointer (block ids must then be relative to it)."""
        out = np.zeros(num_heads * head_dim, np.float32)
        kvf = np.ascontiguousarray(kv, np.uint16)
        bt = np.ascontiguousarray(block_table, np.int32)
        _check(self.lib.ref_paged_attention_cpu(out, np.ascontiguousarray(query, np.float32).ravel(),
                                                kvf.ctypes.data + 2 * kv_base_elems, bt, len(bt), seq_len,
                                                layer, num_heads, num_kv_heads, head_dim, block_size,
                                                num_layers))
        return out.reshape(num_heads, head_dim)

    def paged_attention_batch_rebased(self, out, query, kv_bases, block_table, context_lens, layer,
                                      num_heads, num_kv_heads, head_dim, block_size, num_layers, threads):
        """Batch through the reference, one sequence per call, spread over
        `threads` host threads inside the library.  kv_bases: per-sequence
        pool base addresses (ints); block_table ids relative to them."""
        arr = (C.c_void_p * len(kv_bases))(*[C.c_void_p(int(a)) for a in kv_bases])
        bt = np.ascontiguousarray(block_table, np.int32)
        _check(self.lib.ref_paged_attention_cpu_batch(out, np.ascontiguousarray(query, np.float32).ravel(),
                                                      arr, bt, bt.shape[1],
                                                      np.ascontiguousarray(context_lens, np.int32),
                                                      len(context_lens), layer, num_heads, num_kv_heads,
                                                      head_dim, block_size, num_layers, threads))

    def rope(self, x, pos, num_heads, head_dim, theta=10000.0):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        self.lib.ref_rope_cpu(out, x, pos, num_heads, head_dim, theta)
        return out

    def gemm(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        self.lib.ref_gemm_cpu(c, a, b, a.shape[0], b.shape[1], a.shape[1])
        return c

    def allocator(self, total_blocks, block_size):
        return _Alloc(self.lib, "ref_allocator", total_blocks, block_size)

    def page_table_get(self, blocks, block_size, idx):
        b = np.ascontiguousarray(blocks, np.int32)
        return int(self.lib.ref_page_table_get(b, len(b), block_size, idx))


def reference_available() -> bool:
    return REF_SO.exists()
