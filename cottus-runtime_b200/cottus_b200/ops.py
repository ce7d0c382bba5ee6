"""Torch-facing wrappers over the C ABI.

torch is used only for device memory and the current CUDA stream; all
arithmetic runs in libcottus_b200.so.  Tensors must be contiguous CUDA
tensors on the current device (the block pool helpers are host-only).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import (F16, F32, CottusError, DecodeBatchDesc, DecodeStepParams, LseCombineParams, PagedDecodeParams,
                   OProjParams, QkvParams, check, lib)

_DT = {torch.float32: F32, torch.float16: F16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; use float32 or float16") from None


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def _require(t: torch.Tensor, name: str, dtype=None):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


_WS: dict = {}


def workspace(nbytes: int, device: torch.device, kind: str = "decode") -> torch.Tensor:
    """Cached scratch buffer (a convenience of this Python layer; the C ABI
    itself only takes caller-provided workspace).  One buffer per kind: the
    decode kernels keep the counter words at the start of theirs at zero
    between calls, while the projections ("proj") overwrite all of theirs
    with split partials, so the two never share one."""
    key = (device.type, device.index, kind)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def make_decode_params(out, query, kv_pool, block_table, context_lens, *, num_kv_heads, head_dim, block_size,
                       num_layers=1, layer=0, num_physical_blocks=None, scale=0.0, lse_out=None, status=None,
                       ws=None) -> PagedDecodeParams:
    B, H = query.shape[0], query.shape[1]
    if num_physical_blocks is None:
        per_block = 2 * num_layers * block_size * num_kv_heads * head_dim
        num_physical_blocks = kv_pool.numel() // per_block if per_block > 0 else 0
    p = PagedDecodeParams()
    p.out, p.query, p.kv_pool = out.data_ptr(), query.data_ptr(), kv_pool.data_ptr()
    p.block_table, p.context_lens = block_table.data_ptr(), context_lens.data_ptr()
    p.num_physical_blocks = int(num_physical_blocks)
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim = B, H, num_kv_heads, head_dim
    p.block_size, p.num_layers, p.layer = block_size, num_layers, layer
    p.max_blocks_per_seq = block_table.shape[1] if block_table.dim() == 2 else 0
    p.q_dtype, p.out_dtype = _dtype_code(query), _dtype_code(out)
    p.scale = float(scale)
    p.lse_out = lse_out.data_ptr() if lse_out is not None else None
    p.status = status.data_ptr() if status is not None else None
    if ws is not None:
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel() * ws.element_size()
    return p


def paged_decode(query: torch.Tensor, kv_pool: torch.Tensor, block_table: torch.Tensor, context_lens: torch.Tensor,
                 *, num_kv_heads: int, head_dim: int, block_size: int, num_layers: int = 1, layer: int = 0,
                 out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None, scale: float = 0.0,
                 lse_out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                 num_physical_blocks: int | None = None, stream=None) -> torch.Tensor:
    """Batched paged decode attention (cottus_paged_decode)."""
    _require(query, "query")
    _require(kv_pool, "kv_pool")
    _require(block_table, "block_table", torch.int32)
    _require(context_lens, "context_lens", torch.int32)
    if out is None:
        out = torch.empty(query.shape, dtype=out_dtype or query.dtype, device=query.device)
    p = make_decode_params(out, query, kv_pool, block_table, context_lens, num_kv_heads=num_kv_heads,
                           head_dim=head_dim, block_size=block_size, num_layers=num_layers, layer=layer,
                           num_physical_blocks=num_physical_blocks, scale=scale, lse_out=lse_out, status=status)
    need = lib().cottus_paged_decode_workspace_size(C.byref(p))
    if need:
        ws = workspace(need, query.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().cottus_paged_decode(C.byref(p), _stream(stream)))
    return out


def decode_workspace_size(p: PagedDecodeParams) -> int:
    return int(lib().cottus_paged_decode_workspace_size(C.byref(p)))


def lse_combine(partial_out: torch.Tensor, partial_lse: torch.Tensor, *, out: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.float32, lse_out: torch.Tensor | None = None, stream=None):
    """Merge [P][B][H][D] normalised partials with their [P][B][H] LSEs."""
    _require(partial_out, "partial_out", torch.float32)
    _require(partial_lse, "partial_lse", torch.float32)
    P, B, H, D = partial_out.shape
    if out is None:
        out = torch.empty((B, H, D), dtype=out_dtype, device=partial_out.device)
    p = LseCombineParams()
    p.out, p.partial_out, p.partial_lse = out.data_ptr(), partial_out.data_ptr(), partial_lse.data_ptr()
    p.lse_out = lse_out.data_ptr() if lse_out is not None else None
    p.num_parts, p.batch, p.num_heads, p.head_dim, p.out_dtype = P, B, H, D, _dtype_code(out)
    check(lib().cottus_lse_combine(C.byref(p), _stream(stream)))
    return out


def rope_cos_sin_table(max_position: int, head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Host (cos, sin) table [max_position][head_dim/2][2] from the reference formula."""
    t = torch.empty((max_position, head_dim // 2, 2), dtype=torch.float32)
    check(lib().cottus_rope_cos_sin_fill(C.c_void_p(t.data_ptr()), max_position, head_dim, float(theta)))
    return t


def rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, *, out: torch.Tensor | None = None,
         stream=None) -> torch.Tensor:
    """RoPE of fp32 x[num_tokens][num_heads][head_dim] (in place when out is x)."""
    _require(x, "x", torch.float32)
    _require(positions, "positions", torch.int32)
    _require(cos_sin, "cos_sin", torch.float32)
    T, H, D = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(lib().cottus_rope(_ptr(out), _ptr(x), _ptr(positions), T, H, D, _ptr(cos_sin), cos_sin.shape[0],
                            _stream(stream)))
    return out


def make_step_params(query, key, value, positions, cos_sin, kv_pool, block_table, *, num_kv_heads, head_dim,
                     block_size, num_layers=1, layer=0, num_physical_blocks=None, query_out=None, out=None,
                     scale=0.0, status=None) -> DecodeStepParams:
    B, H = query.shape[0], query.shape[1]
    if num_physical_blocks is None:
        num_physical_blocks = kv_pool.numel() // (2 * num_layers * block_size * num_kv_heads * head_dim)
    p = DecodeStepParams()
    p.query, p.key, p.value = query.data_ptr(), key.data_ptr(), value.data_ptr()
    p.qkv_dtype = _dtype_code(query)
    p.positions = positions.data_ptr()
    p.cos_sin = cos_sin.data_ptr() if cos_sin is not None else None
    p.max_position = cos_sin.shape[0] if cos_sin is not None else 0
    p.kv_pool, p.block_table = kv_pool.data_ptr(), block_table.data_ptr()
    p.num_physical_blocks = int(num_physical_blocks)
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim = B, H, num_kv_heads, head_dim
    p.block_size, p.num_layers, p.layer = block_size, num_layers, layer
    p.max_blocks_per_seq = block_table.shape[1]
    p.query_out = query_out.data_ptr() if query_out is not None else None
    if out is not None:
        p.out, p.out_dtype = out.data_ptr(), _dtype_code(out)
    p.scale = float(scale)
    p.status = status.data_ptr() if status is not None else None
    return p


def rope_append(query, key, value, positions, cos_sin, kv_pool, block_table, *, num_kv_heads, head_dim, block_size,
                num_layers=1, layer=0, query_out=None, status=None, stream=None):
    """RoPE on the new token's q/k and KV append (cottus_rope_append)."""
    for t, n in ((query, "query"), (key, "key"), (value, "value"), (kv_pool, "kv_pool")):
        _require(t, n)
    p = make_step_params(query, key, value, positions, cos_sin, kv_pool, block_table, num_kv_heads=num_kv_heads,
                         head_dim=head_dim, block_size=block_size, num_layers=num_layers, layer=layer,
                         query_out=query_out, status=status)
    check(lib().cottus_rope_append(C.byref(p), _stream(stream)))
    return query_out


def rope_append_decode(query, key, value, positions, cos_sin, kv_pool, block_table, *, num_kv_heads, head_dim,
                       block_size, num_layers=1, layer=0, out=None, out_dtype=None, query_out=None, scale=0.0,
                       status=None, stream=None):
    """RoPE + KV append + paged attention over positions+1 tokens (one kernel)."""
    for t, n in ((query, "query"), (key, "key"), (value, "value"), (kv_pool, "kv_pool")):
        _require(t, n)
    if out is None:
        out = torch.empty(query.shape, dtype=out_dtype or query.dtype, device=query.device)
    p = make_step_params(query, key, value, positions, cos_sin, kv_pool, block_table, num_kv_heads=num_kv_heads,
                         head_dim=head_dim, block_size=block_size, num_layers=num_layers, layer=layer,
                         query_out=query_out, out=out, scale=scale, status=status)
    need = lib().cottus_rope_append_decode_workspace_size(C.byref(p))
    if need:
        ws = workspace(need, query.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().cottus_rope_append_decode(C.byref(p), _stream(stream)))
    return out


def qkv_rope_append(x, weight, positions, cos_sin, kv_pool, block_table, *, num_heads, num_kv_heads, head_dim,
                    block_size, num_layers=1, layer=0, num_physical_blocks=None, query_out=None,
                    query_out_dtype=torch.float16, qkv_out=None, status=None, stream=None):
    """QKV projection + RoPE + KV append in one kernel (cottus_qkv_rope_append).
    x [B][hidden] fp16, weight [(H + 2 Hkv) D][hidden] fp16; returns the rotated query."""
    for t, n in ((x, "x"), (weight, "weight"), (kv_pool, "kv_pool")):
        _require(t, n)
    B, hidden = x.shape
    if num_physical_blocks is None:
        num_physical_blocks = kv_pool.numel() // (2 * num_layers * block_size * num_kv_heads * head_dim)
    if query_out is None:
        query_out = torch.empty((B, num_heads, head_dim), dtype=query_out_dtype, device=x.device)
    p = QkvParams()
    p.x, p.weight, p.hidden = x.data_ptr(), weight.data_ptr(), hidden
    p.positions, p.cos_sin, p.max_position = positions.data_ptr(), cos_sin.data_ptr(), cos_sin.shape[0]
    p.kv_pool, p.block_table, p.num_physical_blocks = kv_pool.data_ptr(), block_table.data_ptr(), int(num_physical_blocks)
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim = B, num_heads, num_kv_heads, head_dim
    p.block_size, p.num_layers, p.layer, p.max_blocks_per_seq = block_size, num_layers, layer, block_table.shape[1]
    p.query_out, p.query_out_dtype = query_out.data_ptr(), _dtype_code(query_out)
    p.qkv_out = qkv_out.data_ptr() if qkv_out is not None else None
    p.status = status.data_ptr() if status is not None else None
    need = lib().cottus_qkv_rope_append_workspace_size(C.byref(p))
    if need:
        ws = workspace(need, x.device, "proj")
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().cottus_qkv_rope_append(C.byref(p), _stream(stream)))
    return query_out


def o_proj_residual(x, weight, residual, *, out=None, out_dtype=torch.float32, status=None, stream=None):
    """Output projection + residual add (cottus_o_proj_residual):
    out = x . weight^T + residual.  x [B][in] fp16, weight [out][in] fp16,
    residual [B][out] fp32; out may be the residual tensor itself (fp32)."""
    for t, n in ((x, "x"), (weight, "weight"), (residual, "residual")):
        _require(t, n)
    B, fin = x.shape
    fout = weight.shape[0]
    if out is None:
        out = torch.empty((B, fout), dtype=out_dtype, device=x.device)
    p = OProjParams()
    p.x, p.weight, p.in_features, p.out_features, p.batch = x.data_ptr(), weight.data_ptr(), fin, fout, B
    p.residual, p.out, p.out_dtype = residual.data_ptr(), out.data_ptr(), _dtype_code(out)
    p.status = status.data_ptr() if status is not None else None
    need = lib().cottus_o_proj_residual_workspace_size(C.byref(p))
    if need:
        ws = workspace(need, x.device, "proj")
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().cottus_o_proj_residual(C.byref(p), _stream(stream)))
    return out


def attention_block(batch, x, w_qkv, w_o, residual, kv_pool, cos_sin, *, num_heads, num_kv_heads, head_dim,
                    num_layers=1, layer=0, query_out=None, att_out=None, status=None, stream=None):
    """The attention half of one decoder layer for the step tokens of a
    DecodeBatch (generic_transformer.cpp:169-327 per token), as three
    launches of this library: the QKV projection with RoPE and the KV append
    (cottus_qkv_rope_append), paged decode attention over the device block
    table with context = position + 1 (cottus_paged_decode), and the output
    projection added to the residual stream in place (cottus_o_proj_residual).

    x [n][hidden] fp16 (the normalised hidden state of each row's token, n =
    len(batch)), w_qkv [(H + 2 Hkv) D][hidden] fp16, w_o [hidden][H D] fp16,
    residual [n][hidden] fp32 (updated in place).  Returns the attention
    output [n][H D] fp16 (the O-projection's input)."""
    n = len(batch)
    if x.shape[0] != n or residual.shape[0] != n:
        raise ValueError(f"x and residual need one row per active sequence ({n})")
    nb = batch.num_blocks
    q = qkv_rope_append(x, w_qkv, batch.positions[:n], cos_sin, kv_pool, batch.block_table[:n], num_heads=num_heads,
                        num_kv_heads=num_kv_heads, head_dim=head_dim, block_size=batch.block_size,
                        num_layers=num_layers, layer=layer, num_physical_blocks=nb, query_out=query_out,
                        query_out_dtype=torch.float16, status=status, stream=stream)
    if att_out is None:
        att_out = torch.empty((n, num_heads, head_dim), dtype=torch.float16, device=x.device)
    paged_decode(q, kv_pool, batch.block_table[:n], batch.context_lens[:n], num_kv_heads=num_kv_heads,
                 head_dim=head_dim, block_size=batch.block_size, num_layers=num_layers, layer=layer, out=att_out,
                 status=status, num_physical_blocks=nb, stream=stream)
    att = att_out.view(n, num_heads * head_dim)
    o_proj_residual(att, w_o, residual, out=residual, status=status, stream=stream)
    return att


def paged_gather(kv_pool, block_table, context_lens, *, max_context, num_kv_heads, head_dim, block_size,
                 num_layers=1, layer=0, num_physical_blocks=None, status=None, k_out=None, v_out=None, stream=None):
    """Dense copy of the K and V rows named by the block table (bit-exact)."""
    B = block_table.shape[0]
    if num_physical_blocks is None:
        num_physical_blocks = kv_pool.numel() // (2 * num_layers * block_size * num_kv_heads * head_dim)
    if k_out is None:
        k_out = torch.zeros((B, max_context, num_kv_heads, head_dim), dtype=torch.uint16, device=kv_pool.device)
    if v_out is None:
        v_out = torch.zeros_like(k_out)
    check(lib().cottus_paged_gather(_ptr(k_out), _ptr(v_out), _ptr(kv_pool), _ptr(block_table), _ptr(context_lens),
                                    int(num_physical_blocks), B, max_context, num_kv_heads, head_dim, block_size,
                                    num_layers, layer, block_table.shape[1], _ptr(status), _stream(stream)))
    return k_out, v_out


class BlockAllocator:
    """The product's LIFO block pool (cottus_block_allocator_*), same
    semantics as the reference cottus::BlockAllocator."""

    def __init__(self, total_blocks: int, block_size: int):
        h = C.c_void_p()
        check(lib().cottus_block_allocator_create(total_blocks, block_size, C.byref(h)))
        self._h = h

    def allocate(self) -> int:
        bid = C.c_int32()
        check(lib().cottus_block_allocator_allocate(self._h, C.byref(bid)))
        return bid.value

    def free(self, block_id: int) -> None:
        check(lib().cottus_block_allocator_free(self._h, int(block_id)))

    def num_free(self) -> int:
        return int(lib().cottus_block_allocator_num_free(self._h))

    def total_blocks(self) -> int:
        return int(lib().cottus_block_allocator_total_blocks(self._h))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().cottus_block_allocator_destroy(h)
            self._h = None


class DecodeBatch:
    """Batched decode-step driver (cottus_decode_batch_*): the block
    bookkeeping of Engine::generate (engine.cpp:52-95) for many sequences,
    with the block table and positions resident on the device.

    `device` None keeps the host bookkeeping only.  Per step:
    ``begin_step()``, then per layer ``rope_append_decode(...)`` with
    ``block_table=self.block_table[:n]``, ``positions=self.positions[:n]``
    (n = len(self)), or ``attention_block(...)``, then ``end_step()``."""

    def __init__(self, num_blocks: int, block_size: int, max_batch: int, max_blocks_per_seq: int, device=None):
        self.block_table = self.positions = self.context_lens = None
        d = DecodeBatchDesc()
        d.num_blocks, d.block_size, d.max_batch, d.max_blocks_per_seq = num_blocks, block_size, max_batch, \
            max_blocks_per_seq
        if device is not None:
            self.block_table = torch.zeros((max_batch, max_blocks_per_seq), dtype=torch.int32, device=device)
            self.positions = torch.zeros(max_batch, dtype=torch.int32, device=device)
            self.context_lens = torch.zeros(max_batch, dtype=torch.int32, device=device)
            d.device_block_table, d.device_positions = self.block_table.data_ptr(), self.positions.data_ptr()
            d.device_context_lens = self.context_lens.data_ptr()
        h = C.c_void_p()
        check(lib().cottus_decode_batch_create(C.byref(d), C.byref(h)))
        self._h = h
        self.num_blocks, self.block_size = num_blocks, block_size
        self.max_batch, self.max_blocks_per_seq = max_batch, max_blocks_per_seq

    def add(self, seq_id: int) -> int:
        row = C.c_int32()
        check(lib().cottus_decode_batch_add(self._h, int(seq_id), C.byref(row)))
        return row.value

    def release(self, seq_id: int) -> None:
        check(lib().cottus_decode_batch_release(self._h, int(seq_id)))

    def begin_step(self, stream=None) -> None:
        check(lib().cottus_decode_batch_begin_step(self._h, _stream(stream) if self.block_table is not None
                                                    else None))

    def end_step(self) -> None:
        check(lib().cottus_decode_batch_end_step(self._h))

    def __len__(self) -> int:
        return int(lib().cottus_decode_batch_size(self._h))

    def free_blocks(self) -> int:
        return int(lib().cottus_decode_batch_free_blocks(self._h))

    def rows(self) -> list:
        n = len(self)
        ids = (C.c_int64 * max(n, 1))()
        lib().cottus_decode_batch_rows(self._h, ids, n)
        return [int(ids[i]) for i in range(n)]

    def sequence(self, seq_id: int):
        """(row, next position, blocks) of an active sequence (host mirror)."""
        row, pos, nb = C.c_int32(), C.c_int32(), C.c_int32()
        check(lib().cottus_decode_batch_sequence(self._h, int(seq_id), C.byref(row), C.byref(pos), None, 0,
                                                 C.byref(nb)))
        blocks = (C.c_int32 * max(nb.value, 1))()
        check(lib().cottus_decode_batch_sequence(self._h, int(seq_id), None, None, blocks, nb.value, None))
        return row.value, pos.value, [int(blocks[i]) for i in range(nb.value)]

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().cottus_decode_batch_destroy(h)
            self._h = None
