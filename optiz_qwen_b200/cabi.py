"""Tensor-level wrappers over the C ABI.

Each function validates shapes/dtypes on the host, takes raw pointers from
torch tensors and enqueues the kernel on the current CUDA stream of the
tensors' device.  No function here synchronises or allocates except where it
creates the output tensor the caller asked for (through torch's caching
allocator, so calls are CUDA-graph capturable).
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import call, dtype_code, ptr, require_cuda, stream_ptr

HEAD_DIM_ATTN = 256
PAGE_SIZE = 64


class PagedKvPool:
    """Device storage of one layer's paged INT4 (or INT8) KV cache.

    ``kv_codes`` uint8 ``[num_pages, Hkv, 2, page_size, D * bits / 8]`` (0 = K, 1 = V) and
    ``kv_meta`` fp16 ``[num_pages, Hkv, 4, page_size]`` (k_scale, k_min, v_scale, v_min).
    Pages are zero-filled on creation.  The append, attention and gather wrappers below
    pick the 4- or 8-bit entry point from ``bits``.
    """

    def __init__(self, num_pages: int, num_kv_heads: int, head_dim: int, page_size: int = PAGE_SIZE,
                 device: torch.device | str = "cuda", bits: int = 4):
        if head_dim % 2:
            raise ValueError("head_dim must be even")
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.num_pages = int(num_pages)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        self.bits = int(bits)
        self.device = torch.device(device)
        self.kv_codes = torch.zeros((num_pages, num_kv_heads, 2, page_size, head_dim * bits // 8),
                                    dtype=torch.uint8, device=self.device)
        self.kv_meta = torch.zeros((num_pages, num_kv_heads, 4, page_size), dtype=torch.float16, device=self.device)

    @property
    def nbytes(self) -> int:
        return self.kv_codes.numel() + 2 * self.kv_meta.numel()

    def grow(self, num_pages: int) -> None:
        """Enlarge the pool to ``num_pages`` pages, keeping page contents and ids."""
        if num_pages <= self.num_pages:
            return
        codes = torch.zeros((num_pages, *self.kv_codes.shape[1:]), dtype=torch.uint8, device=self.device)
        meta = torch.zeros((num_pages, *self.kv_meta.shape[1:]), dtype=torch.float16, device=self.device)
        codes[: self.num_pages].copy_(self.kv_codes)
        meta[: self.num_pages].copy_(self.kv_meta)
        self.kv_codes, self.kv_meta, self.num_pages = codes, meta, int(num_pages)


def _check_table(block_table: torch.Tensor, seq_lens: torch.Tensor, batch: int) -> None:
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be an int32 [batch, max_pages] tensor with contiguous rows")
    if seq_lens.dtype != torch.int32 or seq_lens.dim() != 1 or not seq_lens.is_contiguous():
        raise ValueError("seq_lens must be a contiguous int32 [batch] tensor")
    if block_table.shape[0] < batch or seq_lens.shape[0] < batch:
        raise ValueError("block_table / seq_lens have fewer rows than the batch")


def _bits_entry(base: str, pool: PagedKvPool, bits: int | None) -> str:
    """The entry point ``oq_<base>_int<bits>`` for ``pool``; ``bits`` (when given) must match it."""
    if bits is not None and bits != pool.bits:
        raise ValueError(f"this is the {bits}-bit entry point but the pool holds {pool.bits}-bit codes")
    return f"oq_{base}_int{pool.bits}"


def append_quant(key: torch.Tensor, value: torch.Tensor, pool: PagedKvPool, block_table: torch.Tensor,
                 seq_lens: torch.Tensor, *, advance: bool = True, device_status: torch.Tensor | None = None,
                 _bits: int | None = None) -> None:
    """Quantise ``key``/``value`` ``[B, Hkv, n, D]`` into ``pool`` at positions ``seq_lens[b] + t``
    (4- or 8-bit codes, as the pool holds)."""
    require_cuda(key, value, block_table, seq_lens)
    entry = _bits_entry("append_quant", pool, _bits)
    if key.shape != value.shape or key.dim() != 4:
        raise ValueError("key and value must both be [batch, num_kv_heads, num_new, head_dim]")
    if key.dtype != value.dtype:
        raise ValueError("key and value must share a dtype")
    b, h, n, d = key.shape
    if h != pool.num_kv_heads or d != pool.head_dim:
        raise ValueError(f"key shape {tuple(key.shape)} does not match the pool ({pool.num_kv_heads} heads, "
                         f"head_dim {pool.head_dim})")
    if key.stride(3) != 1 or value.stride(3) != 1:
        key, value = key.contiguous(), value.contiguous()
    _check_table(block_table, seq_lens, b)
    call(entry, ptr(key), ptr(value), dtype_code(key.dtype), b, h, n, d,
         key.stride(0), key.stride(1), key.stride(2), value.stride(0), value.stride(1), value.stride(2),
         ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
         ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens), int(advance),
         ptr(device_status), stream_ptr(key.device))


def append_quant_int4(key, value, pool, block_table, seq_lens, **kw) -> None:
    """:func:`append_quant` into a 4-bit pool (``oq_append_quant_int4``)."""
    append_quant(key, value, pool, block_table, seq_lens, _bits=4, **kw)


def append_quant_int8(key, value, pool, block_table, seq_lens, **kw) -> None:
    """:func:`append_quant` into an 8-bit pool (``oq_append_quant_int8``)."""
    append_quant(key, value, pool, block_table, seq_lens, _bits=8, **kw)


def advance_seq_lens(seq_lens: torch.Tensor, delta: int = 1) -> None:
    require_cuda(seq_lens)
    call("oq_advance_seq_lens", ptr(seq_lens), seq_lens.shape[0], int(delta), stream_ptr(seq_lens.device))


def choose_splits(batch: int, num_kv_heads: int, max_pages: int, sm_count: int = 148, ctas_per_sm: int = 1) -> int:
    """Split count used when ``num_splits <= 0`` (a mirror of the C plan, for host-side sizing):
    enough KV ranges per (sequence, KV head) to fill ~7/8 of one wave of resident CTAs (one per
    SM for the 4-bit kernel; the C side reads SM count and occupancy from the device), at least
    4 pages per range, ranges of equal length."""
    units = batch * num_kv_heads
    splits = min(max(1, (sm_count * ctas_per_sm * 7 // 8) // units), max(1, max_pages // 4), max_pages, 512)
    pps = -(-max_pages // splits)
    return -(-max_pages // pps)


def decode_workspace_bytes(batch: int, num_heads: int, num_kv_heads: int, max_splits: int,
                           head_dim: int = HEAD_DIM_ATTN) -> int:
    return int(_lib.load().oq_decode_attn_workspace_bytes(batch, num_heads, num_kv_heads, head_dim, max_splits))


def new_decode_workspace(batch: int, num_heads: int, num_kv_heads: int, max_pages: int,
                         device: torch.device) -> torch.Tensor:
    """Zero-filled workspace large enough for any split count of this batch shape."""
    nbytes = decode_workspace_bytes(batch, num_heads, num_kv_heads, max(1, max_pages))
    return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)


def decode_attention(query: torch.Tensor, pool: PagedKvPool, block_table: torch.Tensor,
                     seq_lens: torch.Tensor, scaling: float, *, out: torch.Tensor | None = None,
                     out_f32: torch.Tensor | None = None, out_lse: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None, num_splits: int = 0,
                     device_status: torch.Tensor | None = None, want_out: bool = True,
                     gate: torch.Tensor | None = None, exchange: tuple | None = None,
                     new_key: torch.Tensor | None = None, new_value: torch.Tensor | None = None,
                     early: bool = False, _bits: int | None = None):
    """One-token attention of ``query`` ``[B, Hq, D]`` over the paged cache (4- or 8-bit codes,
    as the pool holds: ``oq_decode_attn_int{4,8}_paged``).

    Returns ``out`` (query dtype, ``[B, Hq, D]``) unless ``want_out`` is False.  With
    ``gate`` ``[B, Hq, D]`` (query dtype, unit stride along D) the output is gated in the
    kernel: ``out = attn * sigmoid(gate)`` (``oq_decode_attn_int{4,8}_paged_gated``); fp32 /
    lse outputs are not available then.  With ``exchange = (peer_table, rank, world)`` (4-bit
    pools; ``peer_table``: int64 device tensor of the ``world`` NVLink receive buffers of this
    call site) this rank's KV range is attended and the split merge exchanges every merged row
    with the other ranks in the same launch: the outputs are the merge over all ranks
    (``oq_decode_attn_int4_paged_xrank``).  With ``new_key`` / ``new_value`` ``[B, Hkv, D]`` (query
    dtype) the launch first quantises that token into the cache at position ``seq_lens[b]`` and
    attends over ``seq_lens[b] + 1`` tokens; ``seq_lens`` is left as it is
    (``oq_decode_attn_paged_ex``, which also serves ``early`` alone).  ``early``: launch before the kernel
    ahead in the stream
    has finished and read the lengths, the block table and the cached pages meanwhile; only
    when that kernel writes none of them (``OQ_ATTN_EARLY``).
    """
    require_cuda(query, block_table, seq_lens)
    entry = _bits_entry("decode_attn", pool, _bits) + "_paged"
    if query.dim() != 3:
        raise ValueError("query must be [batch, num_heads, head_dim]")
    if query.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("query must be bf16 or fp16")
    b, hq, d = query.shape
    if query.stride(2) != 1:
        query = query.contiguous()
    if pool.num_kv_heads <= 0 or hq % pool.num_kv_heads:
        raise ValueError("Qwen GQA decode requires an integer query-to-KV head ratio.")
    _check_table(block_table, seq_lens, b)
    if want_out and out is None:
        out = torch.empty((b, hq, d), dtype=query.dtype, device=query.device)
    if workspace is None:
        workspace = new_decode_workspace(b, hq, pool.num_kv_heads, block_table.shape[1], query.device)
    for t, shape in ((out_f32, (b, hq, d)), (out_lse, (b, hq))):
        if t is not None and (t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous()):
            raise ValueError("out_f32 / out_lse must be contiguous fp32 of shape [B, Hq, D] / [B, Hq]")
    flags = _lib.OQ_ATTN_EARLY if early else 0
    if gate is not None:
        require_cuda(gate)
        if gate.dtype != query.dtype or tuple(gate.shape) != (b, hq, d) or gate.stride(2) != 1:
            raise ValueError("gate must be [B, Hq, D] in the query dtype with unit stride along D")
        if out is None or out_f32 is not None or out_lse is not None:
            raise ValueError("a gated call writes the query-dtype output only")
    if new_key is not None or new_value is not None or (early and exchange is None):
        if exchange is not None:
            raise ValueError("an appended token with the cross-GPU exchange is not supported")
        require_cuda(new_key, new_value)
        hkv = pool.num_kv_heads
        if new_key is not None or new_value is not None:
            for t in (new_key, new_value):
                if (t is None or t.dtype != query.dtype or t.dim() != 3 or tuple(t.shape) != (b, hkv, d)
                        or t.stride(2) != 1):
                    raise ValueError("new_key / new_value must be [B, Hkv, D] in the query dtype with unit stride "
                                     "along D")
        ks = (new_key.stride(0), new_key.stride(1)) if new_key is not None else (0, 0)
        vs = (new_value.stride(0), new_value.stride(1)) if new_value is not None else (0, 0)
        call("oq_decode_attn_paged_ex", pool.bits, ptr(query), dtype_code(query.dtype), query.stride(0),
             query.stride(1), ptr(new_key), ks[0], ks[1], ptr(new_value), vs[0], vs[1], ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
             ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens),
             b, hq, hkv, d, float(scaling), ptr(gate), gate.stride(0) if gate is not None else 0,
             gate.stride(1) if gate is not None else 0,
             ptr(out), out.stride(0) if out is not None else 0, out.stride(1) if out is not None else 0,
             ptr(out_f32), ptr(out_lse), ptr(workspace), workspace.numel(), int(num_splits), flags,
             ptr(device_status), stream_ptr(query.device))
        return out
    if gate is not None:
        call(entry + "_gated", ptr(query), dtype_code(query.dtype), query.stride(0),
             query.stride(1), ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
             ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens),
             b, hq, pool.num_kv_heads, d, float(scaling), ptr(gate), gate.stride(0), gate.stride(1),
             ptr(out), out.stride(0), out.stride(1), ptr(workspace), workspace.numel(), int(num_splits),
             ptr(device_status), stream_ptr(query.device))
        return out
    if exchange is not None:
        peer_table, rank, world = exchange
        require_cuda(peer_table)
        if entry != "oq_decode_attn_int4_paged":
            raise ValueError("the cross-GPU exchange needs the 4-bit cache")
        if peer_table.dtype != torch.int64 or peer_table.numel() != world:
            raise ValueError("peer_table must be int64 [world]")
        call(entry + "_xrank", ptr(query), dtype_code(query.dtype), query.stride(0), query.stride(1),
             ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
             ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens),
             b, hq, pool.num_kv_heads, d, float(scaling),
             ptr(out), out.stride(0) if out is not None else 0, out.stride(1) if out is not None else 0,
             ptr(out_f32), ptr(out_lse), ptr(workspace), workspace.numel(), int(num_splits),
             ptr(peer_table), int(rank), int(world), flags, ptr(device_status), stream_ptr(query.device))
        return out
    call(entry, ptr(query), dtype_code(query.dtype), query.stride(0), query.stride(1),
         ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
         ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens),
         b, hq, pool.num_kv_heads, d, float(scaling),
         ptr(out), out.stride(0) if out is not None else 0, out.stride(1) if out is not None else 0,
         ptr(out_f32), ptr(out_lse), ptr(workspace), workspace.numel(), int(num_splits),
         ptr(device_status), stream_ptr(query.device))
    return out


def decode_attention_int4(query, pool, block_table, seq_lens, scaling, **kw):
    """:func:`decode_attention` over a 4-bit pool."""
    return decode_attention(query, pool, block_table, seq_lens, scaling, _bits=4, **kw)


def decode_attention_int8(query, pool, block_table, seq_lens, scaling, **kw):
    """:func:`decode_attention` over an 8-bit pool."""
    return decode_attention(query, pool, block_table, seq_lens, scaling, _bits=8, **kw)


def lse_merge(part_out: torch.Tensor, part_lse: torch.Tensor, dtype: torch.dtype = torch.bfloat16,
              out: torch.Tensor | None = None, out_lse: torch.Tensor | None = None) -> torch.Tensor:
    """Merge ``part_out`` ``[N, R, D]`` / ``part_lse`` ``[N, R]`` (fp32) into ``[R, D]``."""
    require_cuda(part_out, part_lse)
    if part_out.dtype != torch.float32 or part_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    part_out, part_lse = part_out.contiguous(), part_lse.contiguous()
    n, rows, d = part_out.shape
    if tuple(part_lse.shape) != (n, rows):
        raise ValueError("part_lse must be [num_parts, rows]")
    if out is None:
        out = torch.empty((rows, d), dtype=dtype, device=part_out.device)
    call("oq_lse_merge", ptr(part_out), ptr(part_lse), n, rows, d, ptr(out), dtype_code(out.dtype), ptr(out_lse),
         stream_ptr(part_out.device))
    return out


def xrank_buffer_bytes(rows: int, head_dim: int, world: int) -> int:
    """Bytes of one call site's NVLink receive buffer (``oq_xrank_buffer_bytes``)."""
    n = int(_lib.load().oq_xrank_buffer_bytes(rows, head_dim, world))
    if n == 0:
        raise ValueError(f"bad exchange sizes: rows={rows}, head_dim={head_dim}, world={world}")
    return n


def ipc_export(buf: torch.Tensor) -> tuple[bytes, int]:
    """IPC handle of the device allocation holding ``buf`` and ``buf``'s byte offset in it."""
    require_cuda(buf)
    import ctypes

    handle = ctypes.create_string_buffer(int(_lib.load().oq_ipc_handle_bytes()))
    off = ctypes.c_int64(0)
    call("oq_ipc_export", ptr(buf), ctypes.addressof(handle), ctypes.addressof(off))
    return handle.raw, off.value


def ipc_import(handle: bytes, offset: int) -> int:
    """Map a peer's allocation into this process; returns the device address at ``offset``."""
    import ctypes

    out = ctypes.c_void_p(0)
    call("oq_ipc_import", handle, int(offset), ctypes.addressof(out))
    return int(out.value)


def ipc_close(address: int, offset: int) -> None:
    call("oq_ipc_close", int(address), int(offset))


def xrank_lse_merge(part_out: torch.Tensor, part_lse: torch.Tensor, peer_table: torch.Tensor, rank: int,
                    world: int, *, dtype: torch.dtype = torch.bfloat16,
                    out: torch.Tensor | None = None, out_lse: torch.Tensor | None = None,
                    device_status: torch.Tensor | None = None) -> torch.Tensor:
    """Exchange this rank's partial ``part_out`` ``[R, D]`` / ``part_lse`` ``[R]`` over NVLink and merge
    every rank's into ``[R, D]`` (``oq_xrank_lse_merge``).  ``peer_table``: int64 device tensor of
    the ``world`` buffer addresses of this call site."""
    require_cuda(part_out, part_lse, peer_table)
    if part_out.dtype != torch.float32 or part_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    if peer_table.dtype != torch.int64 or peer_table.numel() != world:
        raise ValueError("peer_table must be int64 [world]")
    part_out, part_lse = part_out.contiguous(), part_lse.contiguous()
    rows, d = part_out.shape
    if tuple(part_lse.shape) != (rows,):
        raise ValueError("part_lse must be [rows]")
    if out is None:
        out = torch.empty((rows, d), dtype=dtype, device=part_out.device)
    call("oq_xrank_lse_merge", ptr(part_out), ptr(part_lse), rows, d, ptr(peer_table), int(rank), int(world),
         ptr(out), dtype_code(out.dtype), ptr(out_lse), ptr(device_status), stream_ptr(part_out.device))
    return out


def gather_dequant(pool: PagedKvPool, block_table: torch.Tensor, seq_lens: torch.Tensor, max_len: int,
                   dtype: torch.dtype, *, device_status: torch.Tensor | None = None, _bits: int | None = None):
    """Dequantised ``(keys, values)`` ``[B, Hkv, max_len, D]`` (rows past a sequence's length are 0)."""
    require_cuda(block_table, seq_lens)
    entry = _bits_entry("gather_dequant", pool, _bits)
    b = block_table.shape[0]
    _check_table(block_table, seq_lens, b)
    shape = (b, pool.num_kv_heads, int(max_len), pool.head_dim)
    keys = torch.zeros(shape, dtype=dtype, device=pool.device)
    values = torch.zeros(shape, dtype=dtype, device=pool.device)
    call(entry, ptr(pool.kv_codes), ptr(pool.kv_meta), pool.num_pages, pool.page_size,
         ptr(block_table), block_table.stride(0), block_table.shape[1], ptr(seq_lens), b, pool.num_kv_heads,
         pool.head_dim, int(max_len), ptr(keys), ptr(values), dtype_code(dtype), ptr(device_status),
         stream_ptr(pool.device))
    return keys, values


def gather_dequant_int4(pool, block_table, seq_lens, max_len, dtype, **kw):
    """:func:`gather_dequant` of a 4-bit pool."""
    return gather_dequant(pool, block_table, seq_lens, max_len, dtype, _bits=4, **kw)


def gather_dequant_int8(pool, block_table, seq_lens, max_len, dtype, **kw):
    """:func:`gather_dequant` of an 8-bit pool."""
    return gather_dequant(pool, block_table, seq_lens, max_len, dtype, _bits=8, **kw)


def gdn_recurrent(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, *,
                  scale: float | None = None, initial_state: torch.Tensor | None = None,
                  final_state: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  use_qk_l2norm: bool = False, prefetch_state: bool = False, z: torch.Tensor | None = None,
                  norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
                  norm_workspace: torch.Tensor | None = None,
                  device_status: torch.Tensor | None = None) -> torch.Tensor:
    """Gated delta rule over ``T`` tokens: q, k ``[B, T, H, Dk]``, v ``[B, T, H, Dv]``, g/beta ``[B, T, H]``.

    Writes ``final_state`` (may alias ``initial_state``) and returns ``out`` ``[B, T, H, Dv]``.
    With ``z`` ``[B, T, H, Dv]`` and ``norm_weight`` ``[Dv]`` (qkv dtype) the layer's gated
    RMSNorm is fused in (``oq_gdn_recurrent_norm``): ``out = RMSNormGated(o, z)``; its zeroed
    counter workspace (:func:`new_gdn_norm_workspace`) is allocated when not given.
    ``prefetch_state`` (``OQ_GDN_STATE_PREFETCH``) lets the kernel read the state while the
    preceding kernel in the stream is still running: only for callers that know no such
    kernel writes it (a decode step, where layer l's state was written one step earlier).
    ``device_status`` (int32 ``[1]``, optional; the step without the fused norm) collects
    ``OQ_DEV_TIMEOUT`` if a bounded wait on a state copy gives up.
    """
    require_cuda(q, k, v, g, beta, initial_state, final_state)
    if q.dim() != 4 or k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError("q, k must be [B, T, H, Dk] and v [B, T, H, Dv]")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share a dtype")
    bsz, t, h, dk = q.shape
    dv = v.shape[-1]
    q, k, v = (x if x.stride(3) == 1 else x.contiguous() for x in (q, k, v))
    g, beta = g.contiguous(), beta.contiguous()
    if tuple(g.shape) != (bsz, t, h) or tuple(beta.shape) != (bsz, t, h):
        raise ValueError("g and beta must be [B, T, H]")
    for s in (initial_state, final_state):
        if s is not None and (s.dtype != torch.float32 or tuple(s.shape) != (bsz, h, dk, dv) or not s.is_contiguous()):
            raise ValueError("states must be contiguous fp32 [B, H, Dk, Dv]")
    if out is None:
        out = torch.empty((bsz, t, h, dv), dtype=q.dtype, device=q.device)
    scale = dk ** -0.5 if scale is None else float(scale)
    if (z is None) != (norm_weight is None):
        raise ValueError("z and norm_weight come together")
    if z is not None:
        require_cuda(z, norm_weight)
        if z.dtype != q.dtype or tuple(z.shape) != (bsz, t, h, dv) or z.stride(3) != 1:
            raise ValueError("z must be [B, T, H, Dv] in the qkv dtype with unit stride along Dv")
        norm_weight = norm_weight.to(q.dtype).contiguous()
        if norm_workspace is None:
            norm_workspace = new_gdn_norm_workspace(bsz, h, q.device)
        call("oq_gdn_recurrent_norm", ptr(q), ptr(k), ptr(v), dtype_code(q.dtype),
             q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
             v.stride(0), v.stride(1), v.stride(2),
             ptr(g), dtype_code(g.dtype), ptr(beta), dtype_code(beta.dtype),
             ptr(initial_state), ptr(final_state), ptr(out), bsz, t, h, dk, dv, float(scale), int(use_qk_l2norm),
             ptr(z), z.stride(0), z.stride(1), z.stride(2), ptr(norm_weight), float(norm_eps),
             ptr(norm_workspace), norm_workspace.numel(), GDN_STATE_PREFETCH if prefetch_state else 0,
             stream_ptr(q.device))
        return out
    call("oq_gdn_recurrent", ptr(q), ptr(k), ptr(v), dtype_code(q.dtype),
         q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
         v.stride(0), v.stride(1), v.stride(2),
         ptr(g), dtype_code(g.dtype), ptr(beta), dtype_code(beta.dtype),
         ptr(initial_state), ptr(final_state), ptr(out), bsz, t, h, dk, dv, float(scale), int(use_qk_l2norm),
         GDN_STATE_PREFETCH if prefetch_state else 0, ptr(device_status), stream_ptr(q.device))
    return out


def gdn_recurrent_gates(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                        A_log: torch.Tensor, dt_bias: torch.Tensor, *, scale: float | None = None,
                        initial_state: torch.Tensor | None = None, final_state: torch.Tensor | None = None,
                        out: torch.Tensor | None = None, use_qk_l2norm: bool = False, prefetch_state: bool = False,
                        device_status: torch.Tensor | None = None) -> torch.Tensor:
    """:func:`gdn_recurrent` with the layer's gate arithmetic in the kernel (``oq_gdn_recurrent_gates``):
    from the raw projections ``a``, ``b`` ``[B, T, H]`` and the layer's ``A_log``, ``dt_bias`` ``[H]``
    it computes ``beta = sigmoid(b)`` (in b's dtype) and ``g = -exp(A_log) * softplus(a + dt_bias)``
    in fp32, as Qwen3_5GatedDeltaNet's decode branch does before calling the hook
    (transformers models/qwen3_5/modeling_qwen3_5.py:492-493)."""
    require_cuda(q, k, v, a, b, A_log, dt_bias, initial_state, final_state)
    if q.dim() != 4 or k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError("q, k must be [B, T, H, Dk] and v [B, T, H, Dv]")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share a dtype")
    bsz, t, h, dk = q.shape
    dv = v.shape[-1]
    q, k, v = (x if x.stride(3) == 1 else x.contiguous() for x in (q, k, v))
    a, b = a.contiguous(), b.contiguous()
    if tuple(a.shape) != (bsz, t, h) or b.shape != a.shape or a.dtype != b.dtype:
        raise ValueError("a and b must be [B, T, H] of one dtype")
    A_log, dt_bias = A_log.contiguous(), dt_bias.contiguous()
    if A_log.numel() != h or dt_bias.numel() != h:
        raise ValueError("A_log and dt_bias must have one value per head")
    for s in (initial_state, final_state):
        if s is not None and (s.dtype != torch.float32 or tuple(s.shape) != (bsz, h, dk, dv) or not s.is_contiguous()):
            raise ValueError("states must be contiguous fp32 [B, H, Dk, Dv]")
    if out is None:
        out = torch.empty((bsz, t, h, dv), dtype=q.dtype, device=q.device)
    scale = dk ** -0.5 if scale is None else float(scale)
    call("oq_gdn_recurrent_gates", ptr(q), ptr(k), ptr(v), dtype_code(q.dtype),
         q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
         v.stride(0), v.stride(1), v.stride(2),
         ptr(a), ptr(b), dtype_code(a.dtype), ptr(A_log), dtype_code(A_log.dtype), ptr(dt_bias),
         dtype_code(dt_bias.dtype), ptr(initial_state), ptr(final_state), ptr(out), bsz, t, h, dk, dv, float(scale),
         int(use_qk_l2norm), GDN_STATE_PREFETCH if prefetch_state else 0, ptr(device_status), stream_ptr(q.device))
    return out


GDN_STATE_PREFETCH = 1
CHUNK_SIZE = 64


def new_gdn_norm_workspace(batch: int, num_heads: int, device: torch.device) -> torch.Tensor:
    """Zeroed counters for the fused gated-RMSNorm epilogue of ``batch x num_heads`` heads."""
    nbytes = int(_lib.load().oq_gdn_norm_workspace_bytes(batch, num_heads))
    return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)


def causal_conv1d_update(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None = None, silu: bool = True,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal depthwise conv1d update: x ``[B, C, T]``, conv_state ``[B, C, W]`` (updated in place),
    weight ``[C, K]``; returns ``[B, C, T]`` in x's dtype."""
    require_cuda(x, conv_state, weight, bias)
    if x.dim() != 3 or conv_state.dim() != 3 or conv_state.shape[:2] != x.shape[:2]:
        raise ValueError("x must be [B, C, T] and conv_state [B, C, W]")
    if conv_state.dtype != x.dtype or not conv_state.is_contiguous():
        raise ValueError("conv_state must be contiguous in x's dtype")
    bsz, ch, t = x.shape
    weight = weight.reshape(ch, -1).contiguous()
    if bias is not None:
        bias = bias.to(weight.dtype).contiguous()
    if out is None:
        out = torch.empty((bsz, ch, t), dtype=x.dtype, device=x.device)
    call("oq_causal_conv1d_update", ptr(x), dtype_code(x.dtype), x.stride(0), x.stride(1), x.stride(2),
         ptr(conv_state), ptr(weight), ptr(bias), dtype_code(weight.dtype), ptr(out), bsz, ch, t,
         conv_state.shape[-1], weight.shape[-1], int(silu), stream_ptr(x.device))
    return out


def gdn_conv_step(qkv: torch.Tensor, conv_state: torch.Tensor, conv_weight: torch.Tensor,
                  conv_bias: torch.Tensor | None, g: torch.Tensor, beta: torch.Tensor, *, num_heads: int,
                  scale: float | None = None, initial_state: torch.Tensor | None = None,
                  final_state: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  use_qk_l2norm: bool = True, prefetch_state: bool = False, z: torch.Tensor | None = None,
                  norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
                  norm_workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One GDN decode token with the causal conv1d update fused in: qkv ``[B, C]`` (the projection
    output, q heads | k heads | v heads), conv_state ``[B, C, W]`` and the recurrent state are updated
    in place; returns ``out`` ``[B, 1, H, 128]``.  With ``z`` ``[B, H, 128]`` and ``norm_weight`` the
    layer's gated RMSNorm is fused in as well (``oq_gdn_conv_step_norm``)."""
    require_cuda(qkv, conv_state, conv_weight, conv_bias, g, beta, initial_state, final_state)
    dk = dv = 128
    bsz = qkv.shape[0]
    ch = num_heads * (2 * dk + dv)
    if qkv.dim() != 2 or qkv.shape[1] != ch or qkv.stride(1) != 1:
        raise ValueError(f"qkv must be [B, {ch}] with contiguous channels")
    if conv_state.shape[:2] != (bsz, ch) or conv_state.dtype != qkv.dtype or not conv_state.is_contiguous():
        raise ValueError("conv_state must be contiguous [B, C, W] in qkv's dtype")
    conv_weight = conv_weight.reshape(ch, -1).contiguous()
    if conv_bias is not None:
        conv_bias = conv_bias.to(conv_weight.dtype).contiguous()
    g, beta = g.contiguous(), beta.contiguous()
    for s in (initial_state, final_state):
        if s is not None and (s.dtype != torch.float32 or tuple(s.shape) != (bsz, num_heads, dk, dv)
                              or not s.is_contiguous()):
            raise ValueError("states must be contiguous fp32 [B, H, Dk, Dv]")
    if out is None:
        out = torch.empty((bsz, 1, num_heads, dv), dtype=qkv.dtype, device=qkv.device)
    scale = dk ** -0.5 if scale is None else float(scale)
    if (z is None) != (norm_weight is None):
        raise ValueError("z and norm_weight come together")
    if z is not None:
        require_cuda(z, norm_weight)
        if z.dtype != qkv.dtype or tuple(z.shape) != (bsz, num_heads, dv) or z.stride(2) != 1:
            raise ValueError("z must be [B, H, 128] in the qkv dtype with unit stride along the last dim")
        norm_weight = norm_weight.to(qkv.dtype).contiguous()
        if norm_workspace is None:
            norm_workspace = new_gdn_norm_workspace(bsz, num_heads, qkv.device)
        call("oq_gdn_conv_step_norm", ptr(qkv), dtype_code(qkv.dtype), qkv.stride(0), ptr(conv_state),
             ptr(conv_weight), ptr(conv_bias), dtype_code(conv_weight.dtype), conv_state.shape[-1],
             conv_weight.shape[-1], ptr(g), dtype_code(g.dtype), ptr(beta), dtype_code(beta.dtype),
             ptr(initial_state), ptr(final_state), ptr(out), bsz, num_heads, dk, dv, float(scale),
             int(use_qk_l2norm), ptr(z), z.stride(0), z.stride(1), ptr(norm_weight), float(norm_eps),
             ptr(norm_workspace), norm_workspace.numel(), GDN_STATE_PREFETCH if prefetch_state else 0,
             stream_ptr(qkv.device))
        return out
    call("oq_gdn_conv_step", ptr(qkv), dtype_code(qkv.dtype), qkv.stride(0), ptr(conv_state), ptr(conv_weight),
         ptr(conv_bias), dtype_code(conv_weight.dtype), conv_state.shape[-1], conv_weight.shape[-1],
         ptr(g), dtype_code(g.dtype), ptr(beta), dtype_code(beta.dtype), ptr(initial_state), ptr(final_state),
         ptr(out), bsz, num_heads, dk, dv, float(scale), int(use_qk_l2norm),
         GDN_STATE_PREFETCH if prefetch_state else 0, stream_ptr(qkv.device))
    return out


def rmsnorm_gated(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3_5RMSNormGated over the last dim: ``x``, ``z`` ``[..., D]`` (same dtype, D <= 1024),
    ``weight`` ``[D]``; returns ``rnd(rnd(rnd(x * rsqrt(mean(x^2) + eps)) * w) * silu(z))``."""
    require_cuda(x, z, weight)
    if z.shape != x.shape or z.dtype != x.dtype:
        raise ValueError("x and z must share shape and dtype")
    d = x.shape[-1]
    x2, z2 = x.reshape(-1, d), z.reshape(-1, d)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    if z2.stride(1) != 1:
        z2 = z2.contiguous()
    weight = weight.to(x.dtype).contiguous()
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    o2 = out.view(-1, d)
    call("oq_rmsnorm_gated", ptr(x2), x2.stride(0), ptr(z2), z2.stride(0), ptr(weight), ptr(o2), o2.stride(0),
         dtype_code(x.dtype), x2.shape[0], d, float(eps), stream_ptr(x.device))
    return out


def gdn_chunk_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, *,
                  scale: float | None = None, initial_state: torch.Tensor | None = None,
                  final_state: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  use_qk_l2norm: bool = False, device_status: torch.Tensor | None = None,
                  two_phase: bool = True, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Chunked gated delta rule (prefill) on the tensor cores; same contract as :func:`gdn_recurrent`.

    q, k, v must be bf16 with unit stride along the head dim and 16-byte-multiple
    strides (a slice of a fused projection qualifies); Dk = Dv = 128.  ``two_phase``
    (default) runs ``oq_gdn_chunk_fwd_ws``: the state-independent per-chunk work for all
    chunks in one parallel launch, then the sequential state walk; ``workspace`` (uint8,
    :func:`gdn_chunk_workspace_bytes` bytes) is allocated when not given.  With
    ``two_phase=False`` one launch does both (``oq_gdn_chunk_fwd``).  Results are identical.
    """
    require_cuda(q, k, v, g, beta, initial_state, final_state)
    if q.dim() != 4 or k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError("q, k must be [B, T, H, Dk] and v [B, T, H, Dv]")
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise ValueError("q, k, v must be bf16")
    bsz, t, h, dk = q.shape
    dv = v.shape[-1]
    q, k, v = (x if x.stride(3) == 1 and all((s * 2) % 16 == 0 and s > 0 for s in x.stride()[:3])
               and x.data_ptr() % 16 == 0 else x.contiguous() for x in (q, k, v))
    g, beta = g.contiguous(), beta.contiguous()
    if tuple(g.shape) != (bsz, t, h) or tuple(beta.shape) != (bsz, t, h):
        raise ValueError("g and beta must be [B, T, H]")
    for s in (initial_state, final_state):
        if s is not None and (s.dtype != torch.float32 or tuple(s.shape) != (bsz, h, dk, dv) or not s.is_contiguous()):
            raise ValueError("states must be contiguous fp32 [B, H, Dk, Dv]")
    if out is None:
        out = torch.empty((bsz, t, h, dv), dtype=q.dtype, device=q.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (bsz, t, h, dv) or not out.is_contiguous():
        raise ValueError("out must be contiguous bf16 [B, T, H, Dv]")
    scale = dk ** -0.5 if scale is None else float(scale)
    args = (ptr(q), ptr(k), ptr(v), dtype_code(q.dtype),
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2),
            ptr(g), dtype_code(g.dtype), ptr(beta), dtype_code(beta.dtype),
            ptr(initial_state), ptr(final_state), ptr(out), bsz, t, h, dk, dv, float(scale), int(use_qk_l2norm),
            CHUNK_SIZE)
    if two_phase and t > 0:
        need = gdn_chunk_workspace_bytes(bsz, t, h)
        if workspace is None:
            workspace = torch.empty(max(need, 128), dtype=torch.uint8, device=q.device)
        require_cuda(workspace)
        call("oq_gdn_chunk_fwd_ws", *args, ptr(workspace), workspace.numel() * workspace.element_size(),
             ptr(device_status), stream_ptr(q.device))
    else:
        call("oq_gdn_chunk_fwd", *args, ptr(device_status), stream_ptr(q.device))
    return out


def gdn_chunk_workspace_bytes(batch: int, seq_len: int, num_heads: int) -> int:
    """Bytes of the two-phase chunked form's workspace (about 49 KB per 64-token chunk and head)."""
    return int(_lib.load().oq_gdn_chunk_workspace_bytes(batch, seq_len, num_heads))


def pages_for(length: int, page_size: int = PAGE_SIZE) -> int:
    return max(0, math.ceil(length / page_size))
