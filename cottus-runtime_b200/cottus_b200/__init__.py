"""cottus_b200: B200-native decode hot path of cottus-runtime.

Paged decode attention, fused RoPE + KV append, split-KV LSE merge and the
block pool, implemented in libcottus_b200.so (sm_100a CUDA + C ABI).  This
Python package is a thin ctypes layer for tests, benchmarks and Python
callers; C/C++ callers use include/cottus_b200.h directly.
"""
from ._lib import (COTTUS_ERR_CUDA, COTTUS_ERR_DOUBLE_FREE, COTTUS_ERR_INVALID_ARGUMENT, COTTUS_ERR_OUT_OF_MEMORY,
                   COTTUS_ERR_OUT_OF_RANGE, COTTUS_ERR_UNSUPPORTED, COTTUS_ERR_WORKSPACE, COTTUS_OK, LIB_PATH,
                   STATUS_BAD_BLOCK_ID, STATUS_BAD_CONTEXT, STATUS_BAD_POSITION, STATUS_TIMEOUT, CottusError, lib)
from .ops import (BlockAllocator, DecodeBatch, attention_block, lse_combine, o_proj_residual, paged_decode, paged_gather,
                  qkv_rope_append, rope,
                  rope_append, rope_append_decode, rope_cos_sin_table)

__all__ = [
    "BlockAllocator", "CottusError", "attention_block", "DecodeBatch", "LIB_PATH", "lib", "lse_combine", "o_proj_residual", "paged_decode", "paged_gather",
    "qkv_rope_append", "rope",
    "rope_append", "rope_append_decode", "rope_cos_sin_table", "COTTUS_OK", "COTTUS_ERR_INVALID_ARGUMENT",
    "COTTUS_ERR_OUT_OF_RANGE", "COTTUS_ERR_CUDA", "COTTUS_ERR_UNSUPPORTED", "COTTUS_ERR_WORKSPACE",
    "COTTUS_ERR_OUT_OF_MEMORY", "COTTUS_ERR_DOUBLE_FREE", "STATUS_BAD_BLOCK_ID", "STATUS_BAD_CONTEXT",
    "STATUS_BAD_POSITION", "STATUS_TIMEOUT",
]
