"""Long-context decode attention split across the GPUs of one box.

One sequence's KV cache is cut into contiguous, page-aligned token ranges, one
per rank (``kv_ranges``).  Each rank stores only its range in its own paged
INT4 pool and runs the split-KV decode kernel over it, producing the
normalised fp32 partial output and the natural-log log-sum-exp of its scores
(``oq_decode_attn_int4_paged`` with ``out_f32`` / ``out_lse``).  One all-gather
over NCCL (NVLink / NVSwitch) exchanges the partials -- B x Hq x (D + 1) fp32
per rank, 8,224 B for one sequence with 8 heads of 256 -- and every rank
combines them with ``oq_lse_merge``:

    out = sum_r exp(lse_r - L) * out_r,   L = log sum_r exp(lse_r).

New decode tokens are appended to the last rank's range (the tail of the
sequence).  The reference decodes on one GPU; this module has no counterpart
there.

Two exchanges.  The NCCL path packs the partial, all-gathers it through
torch.distributed and merges with ``oq_lse_merge``.  The NVLink path
(``PeerExchange``) stores each merged row into every rank's receive buffer with
plain 8-byte stores over NVLink (CUDA IPC mappings, no multicast), each value
tagged with its call's epoch, polls (bounded) until every rank's row has arrived
and merges in the same order as ``oq_lse_merge``.  By default it runs inside the
attention launch's split merge (``oq_decode_attn_int4_paged_xrank``: one launch
pair per layer); ``oq_xrank_lse_merge`` is the same exchange as a kernel of its
own after the partial, bit-identical to the NCCL path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


def kv_ranges(length: int, world: int, page_size: int = 64) -> list[tuple[int, int]]:
    """Even split of ``[0, length)`` into ``world`` page-aligned contiguous ranges (may be empty)."""
    if world <= 0:
        raise ValueError("world must be positive")
    pages = -(-int(length) // page_size)
    per = -(-pages // world) if pages else 0
    out = []
    for r in range(world):
        lo = min(length, r * per * page_size)
        hi = min(length, (r + 1) * per * page_size)
        out.append((lo, hi))
    return out


def pack_partial(out_f32: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """[B, Hq, D] fp32 + [B, Hq] fp32 -> one contiguous [B * Hq, D + 1] message."""
    b, h, d = out_f32.shape
    msg = torch.empty((b * h, d + 1), dtype=torch.float32, device=out_f32.device)
    msg[:, :d].copy_(out_f32.reshape(b * h, d))
    msg[:, d].copy_(lse.reshape(b * h))
    return msg


def unpack_partials(gathered: torch.Tensor, head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """[world, R, D + 1] -> (part_out [world, R, D], part_lse [world, R]), both contiguous."""
    return gathered[..., :head_dim].contiguous(), gathered[..., head_dim].contiguous()


@dataclass
class PartialFns:
    """The compute a rank plugs in: partial attention over its range, and the merge."""

    partial: Callable[[torch.Tensor], tuple[torch.Tensor, torch.Tensor]]  # q [B,Hq,D] -> (out_f32, lse)
    merge: Callable[[torch.Tensor, torch.Tensor], torch.Tensor]          # (part_out, part_lse) -> out [R, D]
    # optional, one rank: q -> out [B, Hq, D] straight from the attention kernel.  The merge of a
    # single partial is the identity, so the fp32 partial, its packing and the merge are skipped.
    single: Callable[[torch.Tensor], torch.Tensor] | None = None
    # optional, several ranks: (out_f32 [B, Hq, D], lse [B, Hq]) -> out [B * Hq, D] merged over every
    # rank by the NVLink exchange kernel, in place of pack + all-gather + unpack + merge.
    exchange: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None


def context_parallel_attention(q: torch.Tensor, fns: PartialFns, group=None) -> torch.Tensor:
    """Attention of ``q`` ``[B, Hq, D]`` over the KV ranges of every rank of ``group``; returns ``[B, Hq, D]``.

    Every rank takes the same exchange step (one all-gather, or one NVLink exchange kernel) per call.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1 and fns.single is not None:
        return fns.single(q).reshape(q.shape)
    out_f32, lse = fns.partial(q)
    if world > 1 and fns.exchange is not None:
        return fns.exchange(out_f32, lse).reshape(q.shape)
    msg = pack_partial(out_f32, lse)
    if world == 1:
        part_out, part_lse = unpack_partials(msg.view(1, *msg.shape), q.shape[-1])
        return fns.merge(part_out, part_lse).reshape(q.shape)
    gathered = torch.empty((world * msg.shape[0], msg.shape[1]), dtype=msg.dtype, device=msg.device)
    dist.all_gather_into_tensor(gathered, msg, group=group)
    part_out, part_lse = unpack_partials(gathered.view(world, *msg.shape), q.shape[-1])
    return fns.merge(part_out, part_lse).reshape(q.shape)


class PeerExchange:
    """NVLink receive buffers for ``sites`` call sites (e.g. one per attention layer) of ``rows`` x
    ``head_dim`` partials, mapped into every rank of ``group``.

    Construction is collective: each rank allocates one zeroed buffer for all sites, exports its
    CUDA IPC handle, all-gathers the handles over ``group`` and maps every peer's buffer.  Each
    site's buffer keeps its own per-row call counters on the device, so calls of one site may be
    captured in a CUDA graph and replayed.  A site serves either the standalone exchange
    (``merge``) or the attention launch that exchanges in its split merge (``table``), with the
    same rows.  ``close()`` is collective too: it waits for every rank's last exchange, then
    unmaps the peers' buffers.
    """

    def __init__(self, rows: int, head_dim: int, *, rank: int, world: int, device, group=None, sites: int = 1):
        from . import cabi

        self.cabi = cabi
        self.rows, self.head_dim, self.rank, self.world, self.sites = int(rows), int(head_dim), rank, world, sites
        self.device = torch.device(device)
        self.site_bytes = cabi.xrank_buffer_bytes(rows, head_dim, world)
        self.buf = torch.zeros(self.site_bytes * sites, dtype=torch.uint8, device=self.device)
        self._imported: list[tuple[int, int]] = []
        bases = [0] * world
        bases[rank] = self.buf.data_ptr()
        if world > 1:
            import torch.distributed as dist

            handle, off = cabi.ipc_export(self.buf)
            nh = len(handle)
            msg = torch.zeros(nh + 8, dtype=torch.uint8)
            msg[:nh] = torch.frombuffer(bytearray(handle), dtype=torch.uint8)
            msg[nh:] = torch.tensor([off], dtype=torch.int64).view(torch.uint8)
            gathered = torch.empty(world * msg.numel(), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(gathered, msg.to(self.device), group=group)
            g = gathered.cpu().view(world, nh + 8)
            for r in range(world):
                if r == rank:
                    continue
                peer_off = int(g[r, nh:].clone().view(torch.int64)[0])
                addr = cabi.ipc_import(bytes(g[r, :nh].tolist()), peer_off)
                self._imported.append((addr, peer_off))
                bases[r] = addr
            dist.barrier(group=group)        # every buffer is zeroed and mapped before any rank's first store
        self.group = group
        self.peer_tables = torch.tensor([[b + s * self.site_bytes for b in bases] for s in range(sites)],
                                        dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def table(self, site: int) -> tuple[torch.Tensor, int, int]:
        """``(peer_table, rank, world)`` of ``site``: the ``exchange`` argument of ``cabi.decode_attention``."""
        return self.peer_tables[site], self.rank, self.world

    def merge(self, site: int, part_out: torch.Tensor, part_lse: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
        """This rank's partial ``[R, D]`` / ``[R]`` in, every rank's merged output ``[R, D]`` out."""
        return self.cabi.xrank_lse_merge(part_out.reshape(self.rows, self.head_dim), part_lse.reshape(self.rows),
                                         self.peer_tables[site], self.rank, self.world, dtype=dtype,
                                         device_status=self.status)

    def close(self) -> None:
        if self._imported:
            import torch.distributed as dist

            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)   # no rank still stores into a buffer that is about to go
            for addr, off in self._imported:
                self.cabi.ipc_close(addr, off)
            self._imported = []


class ContextParallelDecoder:
    """One attention layer's share of a long sequence on this rank, backed by the sm_100a kernels.

    ``keys`` / ``values`` passed to ``prefill`` are the whole sequence's K/V
    ``[B, Hkv, T, D]``; each rank keeps only its own range.  ``decode(q)`` runs
    the partial attention, the all-gather and the merge; ``append`` adds one new
    token on the last rank.
    """

    def __init__(self, num_kv_heads: int, head_dim: int, *, rank: int, world: int, device, group=None,
                 page_size: int = 64, out_dtype=torch.bfloat16, exchange: PeerExchange | None = None,
                 site: int = 0):
        from . import cabi

        self.cabi = cabi
        self.rank, self.world, self.group = rank, world, group
        self.num_kv_heads, self.head_dim, self.page_size = num_kv_heads, head_dim, page_size
        self.device = torch.device(device)
        self.out_dtype = out_dtype
        self.paged = None
        self.range = (0, 0)
        self._ws = None
        # the NVLink exchange (call site `site` of it) in place of the NCCL all-gather, when given:
        # inside the attention's split merge (fused_exchange) or as its own kernel after it
        self.exchange, self.site = exchange, site
        self.fused_exchange = True
        # early: launch the attention before the kernel ahead of it finishes, loading the cached
        # pages meanwhile -- only when that kernel writes none of this decoder's cache (e.g. the
        # previous layer's attention and merge)
        self.early = False

    def prefill(self, keys: torch.Tensor, values: torch.Tensor, *, capacity_tokens: int | None = None,
                page_seed: int | None = None) -> None:
        from .compression.paged_kv import PageAllocator, PagedKvState

        b, h, t, d = keys.shape
        lo, hi = kv_ranges(t, self.world, self.page_size)[self.rank]
        self.range = (lo, hi)
        extra = (capacity_tokens or 0) if self.rank == self.world - 1 else 0
        cap = (hi - lo) + extra
        pages = max(1, self.cabi.pages_for(max(cap, 1), self.page_size))
        pool = self.cabi.PagedKvPool(b * pages, h, d, self.page_size, self.device)
        self.paged = PagedKvState(pool, b, max_pages=pages, allocator=PageAllocator(b * pages, page_seed))
        self.paged.reserve([max(cap, 1)] * b)
        if hi > lo:
            self.paged.append(keys[:, :, lo:hi].to(self.device), values[:, :, lo:hi].to(self.device))

    def prefill_random(self, length: int, *, generator: torch.Generator, capacity_tokens: int = 0,
                       page_seed: int | None = None, batch: int = 1, dtype=torch.bfloat16) -> None:
        """Fill this rank's range of a ``length``-token sequence with N(0,1) K/V (synthetic workloads);
        only the rank's own slice is generated and stored."""
        from .compression.paged_kv import PageAllocator, PagedKvState

        lo, hi = kv_ranges(length, self.world, self.page_size)[self.rank]
        self.range = (lo, hi)
        extra = capacity_tokens if self.rank == self.world - 1 else 0
        cap = max(1, (hi - lo) + extra)
        pages = self.cabi.pages_for(cap, self.page_size)
        pool = self.cabi.PagedKvPool(batch * pages, self.num_kv_heads, self.head_dim, self.page_size, self.device)
        self.paged = PagedKvState(pool, batch, max_pages=pages, allocator=PageAllocator(batch * pages, page_seed))
        self.paged.reserve([cap] * batch)
        chunk = 8192
        for start in range(lo, hi, chunk):
            m = min(chunk, hi - start)
            shp = (batch, self.num_kv_heads, m, self.head_dim)
            k = torch.randn(shp, generator=generator, device=self.device, dtype=torch.float32).to(dtype)
            v = torch.randn(shp, generator=generator, device=self.device, dtype=torch.float32).to(dtype)
            self.paged.append(k, v)

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append new tokens ``[B, Hkv, n, D]`` to the sequence tail (held by the last rank)."""
        if self.rank == self.world - 1:
            self.paged.append(key, value)
            self.range = (self.range[0], self.range[1] + int(key.shape[-2]))

    def _workspace(self, q: torch.Tensor) -> torch.Tensor:
        if self._ws is None:
            b, hq, _ = q.shape
            self._ws = self.cabi.new_decode_workspace(b, hq, self.num_kv_heads, self.paged.max_pages, self.device)
        return self._ws

    def _partial(self, q: torch.Tensor):
        b, hq, d = q.shape
        out_f32 = torch.empty((b, hq, d), dtype=torch.float32, device=self.device)
        lse = torch.empty((b, hq), dtype=torch.float32, device=self.device)
        self.cabi.decode_attention_int4(q, self.paged.pool, self.paged.block_table, self.paged.seq_lens,
                                        self.head_dim ** -0.5, out_f32=out_f32, out_lse=lse,
                                        workspace=self._workspace(q), want_out=False, early=self.early)
        return out_f32, lse

    def _single(self, q: torch.Tensor) -> torch.Tensor:
        return self.cabi.decode_attention_int4(q, self.paged.pool, self.paged.block_table, self.paged.seq_lens,
                                               self.head_dim ** -0.5, workspace=self._workspace(q), early=self.early)

    def _merge(self, part_out: torch.Tensor, part_lse: torch.Tensor) -> torch.Tensor:
        return self.cabi.lse_merge(part_out, part_lse, dtype=self.out_dtype)

    def _exchange(self, out_f32: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
        return self.exchange.merge(self.site, out_f32, lse, dtype=self.out_dtype)

    def _fused(self, q: torch.Tensor) -> torch.Tensor:
        """Partial attention whose split merge exchanges the rows over NVLink: one launch pair."""
        return self.cabi.decode_attention_int4(q, self.paged.pool, self.paged.block_table, self.paged.seq_lens,
                                               self.head_dim ** -0.5, workspace=self._workspace(q),
                                               exchange=self.exchange.table(self.site),
                                               device_status=self.exchange.status, early=self.early)

    def decode(self, q: torch.Tensor) -> torch.Tensor:
        if self.exchange is not None and self.world > 1 and q.dtype == self.out_dtype and self.fused_exchange:
            return self._fused(q).reshape(q.shape)
        # one rank with the output in the query's dtype: the kernel writes the output itself
        single = self._single if q.dtype == self.out_dtype else None
        exchange = self._exchange if self.exchange is not None else None
        return context_parallel_attention(q, PartialFns(self._partial, self._merge, single, exchange), self.group)
