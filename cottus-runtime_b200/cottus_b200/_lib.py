"""ctypes binding of libcottus_b200.so (the C ABI in include/cottus_b200.h).

There is no fallback: if the shared library is missing or cannot be loaded,
importing the ops raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("COTTUS_B200_LIB", PKG_ROOT / "libcottus_b200.so"))

COTTUS_OK = 0
COTTUS_ERR_INVALID_ARGUMENT = -1
COTTUS_ERR_OUT_OF_RANGE = -2
COTTUS_ERR_CUDA = -3
COTTUS_ERR_UNSUPPORTED = -4
COTTUS_ERR_WORKSPACE = -5
COTTUS_ERR_OUT_OF_MEMORY = -6
COTTUS_ERR_DOUBLE_FREE = -7

STATUS_BAD_BLOCK_ID = 0x1
STATUS_BAD_CONTEXT = 0x2
STATUS_BAD_POSITION = 0x4
STATUS_TIMEOUT = 0x8

F32, F16 = 0, 1

_vp, _i32, _i64, _f32, _sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t


class PagedDecodeParams(C.Structure):
    _fields_ = [
        ("out", _vp), ("query", _vp), ("kv_pool", _vp), ("block_table", _vp), ("context_lens", _vp),
        ("num_physical_blocks", _i64),
        ("batch", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32), ("block_size", _i32),
        ("num_layers", _i32), ("layer", _i32), ("max_blocks_per_seq", _i32), ("q_dtype", _i32), ("out_dtype", _i32),
        ("scale", _f32),
        ("lse_out", _vp), ("workspace", _vp), ("workspace_bytes", _sz), ("status", _vp),
    ]


class LseCombineParams(C.Structure):
    _fields_ = [
        ("out", _vp), ("lse_out", _vp), ("partial_out", _vp), ("partial_lse", _vp),
        ("num_parts", _i32), ("batch", _i32), ("num_heads", _i32), ("head_dim", _i32), ("out_dtype", _i32),
    ]


class DecodeStepParams(C.Structure):
    _fields_ = [
        ("query", _vp), ("key", _vp), ("value", _vp), ("qkv_dtype", _i32), ("positions", _vp),
        ("cos_sin", _vp), ("max_position", _i32),
        ("kv_pool", _vp), ("block_table", _vp), ("num_physical_blocks", _i64),
        ("batch", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32), ("block_size", _i32),
        ("num_layers", _i32), ("layer", _i32), ("max_blocks_per_seq", _i32),
        ("query_out", _vp), ("out", _vp), ("out_dtype", _i32), ("scale", _f32),
        ("workspace", _vp), ("workspace_bytes", _sz), ("status", _vp),
    ]


class DecodeBatchDesc(C.Structure):
    _fields_ = [
        ("num_blocks", _i32), ("block_size", _i32), ("max_batch", _i32), ("max_blocks_per_seq", _i32),
        ("device_block_table", _vp), ("device_positions", _vp), ("device_context_lens", _vp),
    ]


class QkvParams(C.Structure):
    _fields_ = [
        ("x", _vp), ("weight", _vp), ("hidden", _i32), ("positions", _vp), ("cos_sin", _vp), ("max_position", _i32),
        ("kv_pool", _vp), ("block_table", _vp), ("num_physical_blocks", _i64),
        ("batch", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32), ("block_size", _i32),
        ("num_layers", _i32), ("layer", _i32), ("max_blocks_per_seq", _i32),
        ("query_out", _vp), ("query_out_dtype", _i32), ("qkv_out", _vp),
        ("workspace", _vp), ("workspace_bytes", _sz), ("status", _vp),
    ]


class OProjParams(C.Structure):
    _fields_ = [
        ("x", _vp), ("weight", _vp), ("in_features", _i32), ("out_features", _i32), ("batch", _i32),
        ("residual", _vp), ("out", _vp), ("out_dtype", _i32),
        ("workspace", _vp), ("workspace_bytes", _sz), ("status", _vp),
    ]


class CottusError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (code {code})")
        self.code = code
        self.message = message


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C cottus-runtime_b200` "
                          "(or __graft_entry__.build()); there is no fallback path")
    L = C.CDLL(str(LIB_PATH))
    P = C.POINTER
    sig = [
        ("cottus_last_error", C.c_char_p, []),
        ("cottus_status_string", C.c_char_p, [C.c_int]),
        ("cottus_version", C.c_int, []),
        ("cottus_paged_decode_workspace_size", _sz, [P(PagedDecodeParams)]),
        ("cottus_paged_decode", C.c_int, [P(PagedDecodeParams), _vp]),
        ("cottus_paged_decode_static_scratch", C.c_int, [P(PagedDecodeParams), _vp]),
        ("cottus_lse_combine", C.c_int, [P(LseCombineParams), _vp]),
        ("cottus_rope_cos_sin_fill", C.c_int, [_vp, _i32, _i32, _f32]),
        ("cottus_rope", C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _vp, _i32, _vp]),
        ("cottus_rope_append", C.c_int, [P(DecodeStepParams), _vp]),
        ("cottus_rope_append_decode_workspace_size", _sz, [P(DecodeStepParams)]),
        ("cottus_rope_append_decode", C.c_int, [P(DecodeStepParams), _vp]),
        ("cottus_paged_gather", C.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                          _i32, _vp, _vp]),
        ("cottus_block_allocator_create", C.c_int, [_i32, _i32, P(_vp)]),
        ("cottus_block_allocator_destroy", None, [_vp]),
        ("cottus_block_allocator_allocate", C.c_int, [_vp, P(_i32)]),
        ("cottus_block_allocator_free", C.c_int, [_vp, _i32]),
        ("cottus_block_allocator_num_free", _i32, [_vp]),
        ("cottus_block_allocator_total_blocks", _i32, [_vp]),
        ("cottus_qkv_rope_append_workspace_size", _sz, [P(QkvParams)]),
        ("cottus_qkv_rope_append", C.c_int, [P(QkvParams), _vp]),
        ("cottus_o_proj_residual_workspace_size", _sz, [P(OProjParams)]),
        ("cottus_o_proj_residual", C.c_int, [P(OProjParams), _vp]),
        ("cottus_peer_exchange_create", C.c_int, [_i32, _i32, _i32, _i32, _i32, P(_vp), _vp]),
        ("cottus_peer_exchange_open", C.c_int, [_vp, _vp]),
        ("cottus_peer_exchange_set_wait_cycles", C.c_int, [_vp, _i64]),
        ("cottus_peer_exchange_destroy", None, [_vp]),
        ("cottus_split_decode_workspace_size", _sz, [P(PagedDecodeParams)]),
        ("cottus_split_decode", C.c_int, [P(PagedDecodeParams), _vp, _vp]),
        ("cottus_decode_batch_create", C.c_int, [P(DecodeBatchDesc), P(_vp)]),
        ("cottus_decode_batch_destroy", None, [_vp]),
        ("cottus_decode_batch_add", C.c_int, [_vp, _i64, P(_i32)]),
        ("cottus_decode_batch_release", C.c_int, [_vp, _i64]),
        ("cottus_decode_batch_begin_step", C.c_int, [_vp, _vp]),
        ("cottus_decode_batch_end_step", C.c_int, [_vp]),
        ("cottus_decode_batch_size", _i32, [_vp]),
        ("cottus_decode_batch_free_blocks", _i32, [_vp]),
        ("cottus_decode_batch_rows", C.c_int, [_vp, P(_i64), _i32]),
        ("cottus_decode_batch_sequence", C.c_int, [_vp, _i64, P(_i32), P(_i32), P(_i32), _i32, P(_i32)]),
    ]
    for name, res, args in sig:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = L
    return L


def check(rc: int) -> None:
    if rc != COTTUS_OK:
        msg = lib().cottus_last_error().decode(errors="replace")
        raise CottusError(rc, msg)
