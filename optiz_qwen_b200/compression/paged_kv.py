"""Host-side bookkeeping of the paged INT4 KV cache: page allocation and block tables.

The reference stores each layer's packed KV as one contiguous tensor grown by
``torch.cat`` (optiz_qwen/compression/qserve_kv_cache.py:374-377), which copies
the whole cache every ``residual_length`` tokens and moves its address.  Here a
layer owns a fixed pool of 64-token pages (``cabi.PagedKvPool``) and a block
table; appending a token touches only its page slot, and the device addresses
stay put, so a decode step can be captured in a CUDA graph.

Page hand-out order is a free list, optionally a seeded permutation (numpy
PCG64); ``oracle.kv_quant.page_permutation`` restates the same policy.
"""

from __future__ import annotations

from collections import deque

import numpy as np
import torch

from .. import cabi


class PageAllocator:
    """Free list of physical page ids."""

    def __init__(self, num_pages: int, seed: int | None = None):
        order = (np.arange(num_pages) if seed is None
                 else np.random.default_rng(seed).permutation(num_pages))
        self._free = deque(int(x) for x in order)
        self.num_pages = int(num_pages)

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"page pool exhausted: need {n} pages, {len(self._free)} free")
        return [self._free.popleft() for _ in range(n)]

    def free(self, pages) -> None:
        self._free.extend(int(p) for p in pages)

    def grow(self, num_pages: int) -> None:
        """Add the new ids ``[old, num_pages)`` to the end of the free list."""
        self._free.extend(range(self.num_pages, num_pages))
        self.num_pages = int(num_pages)


class PagedKvState:
    """One batch of sequences stored in a ``PagedKvPool``.

    ``block_table`` (int32 ``[batch, max_pages]``, -1 = no page) and ``seq_lens``
    (int32 ``[batch]``) live on the device; ``host_lens`` / ``host_pages`` mirror
    them on the host so page reservations never read the device.
    """

    def __init__(self, pool: cabi.PagedKvPool, batch: int, *, max_pages: int = 1,
                 allocator: PageAllocator | None = None):
        self.pool = pool
        self.allocator = allocator or PageAllocator(pool.num_pages)
        self.batch = int(batch)
        self.host_lens = [0] * self.batch
        self.host_pages: list[list[int]] = [[] for _ in range(self.batch)]
        self.block_table = torch.full((self.batch, max(1, max_pages)), -1, dtype=torch.int32, device=pool.device)
        self.seq_lens = torch.zeros(self.batch, dtype=torch.int32, device=pool.device)

    @property
    def page_size(self) -> int:
        return self.pool.page_size

    @property
    def max_pages(self) -> int:
        return self.block_table.shape[1]

    def reserve(self, lengths) -> None:
        """Make sure row ``b`` has pages for ``lengths[b]`` tokens (growing pool / table as needed)."""
        need = [cabi.pages_for(int(n), self.page_size) for n in lengths]
        extra = sum(max(0, n - len(p)) for n, p in zip(need, self.host_pages))
        if extra == 0:
            return
        if extra > self.allocator.num_free:
            new_total = max(self.pool.num_pages * 2, self.pool.num_pages + extra - self.allocator.num_free)
            self.pool.grow(new_total)
            self.allocator.grow(new_total)
        width = max(need + [self.max_pages])
        if width > self.max_pages:
            table = torch.full((self.batch, max(width, 2 * self.max_pages)), -1, dtype=torch.int32,
                               device=self.pool.device)
            table[:, : self.max_pages].copy_(self.block_table)
            self.block_table = table
        for b, n in enumerate(need):
            if n > len(self.host_pages[b]):
                self.host_pages[b].extend(self.allocator.allocate(n - len(self.host_pages[b])))
        self._upload_table()

    def _upload_table(self) -> None:
        host = np.full((self.batch, self.max_pages), -1, dtype=np.int32)
        for b, pages in enumerate(self.host_pages):
            host[b, : len(pages)] = pages
        self.block_table.copy_(torch.from_numpy(host), non_blocking=False)

    def append(self, key: torch.Tensor, value: torch.Tensor, *, device_status: torch.Tensor | None = None) -> None:
        """Quantise ``[batch, Hkv, n, D]`` tokens onto the end of every row."""
        n = int(key.shape[-2])
        self.reserve([length + n for length in self.host_lens])
        cabi.append_quant(key, value, self.pool, self.block_table, self.seq_lens, advance=True,
                          device_status=device_status)
        self.host_lens = [length + n for length in self.host_lens]

    def append_attend(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float, *,
                      workspace: torch.Tensor, gate: torch.Tensor | None = None,
                      device_status: torch.Tensor | None = None) -> torch.Tensor:
        """One decode token per row in one launch: ``key`` / ``value`` ``[batch, Hkv, D]`` go into the
        cache at the end of every row and ``query`` ``[batch, Hq, D]`` attends over the rows with them
        (``oq_decode_attn_paged_ex``); returns ``[batch, Hq, D]`` in the query dtype (gated when
        ``gate`` is given).  The row lengths then advance by one."""
        self.reserve([length + 1 for length in self.host_lens])
        out = cabi.decode_attention(query, self.pool, self.block_table, self.seq_lens, scaling, workspace=workspace,
                                    gate=gate, new_key=key, new_value=value, device_status=device_status)
        cabi.advance_seq_lens(self.seq_lens, 1)
        self.host_lens = [length + 1 for length in self.host_lens]
        return out

    def set_lengths(self, lengths) -> None:
        """Truncate rows (crop); pages past the new end go back to the free list."""
        for b, n in enumerate(lengths):
            keep = cabi.pages_for(int(n), self.page_size)
            if keep < len(self.host_pages[b]):
                self.allocator.free(self.host_pages[b][keep:])
                del self.host_pages[b][keep:]
            self.host_lens[b] = int(n)
        self.seq_lens.copy_(torch.tensor(self.host_lens, dtype=torch.int32))
        self._upload_table()

    def select_rows(self, indices) -> None:
        """Rebuild the batch from rows ``indices`` (may repeat); every new row gets its own pages."""
        indices = [int(i) for i in indices]
        old_pages, old_lens = self.host_pages, self.host_lens
        needed = sum(len(old_pages[i]) for i in indices)
        if needed > self.allocator.num_free:
            new_total = max(self.pool.num_pages * 2, self.pool.num_pages + needed - self.allocator.num_free)
            self.pool.grow(new_total)
            self.allocator.grow(new_total)
        new_pages = []
        src, dst = [], []
        for i in indices:
            pages = self.allocator.allocate(len(old_pages[i])) if old_pages[i] else []
            new_pages.append(pages)
            src.extend(old_pages[i])
            dst.extend(pages)
        if src:
            s = torch.tensor(src, dtype=torch.long, device=self.pool.device)
            d = torch.tensor(dst, dtype=torch.long, device=self.pool.device)
            self.pool.kv_codes.index_copy_(0, d, self.pool.kv_codes.index_select(0, s))
            self.pool.kv_meta.index_copy_(0, d, self.pool.kv_meta.index_select(0, s))
        for pages in old_pages:
            self.allocator.free(pages)
        self.batch = len(indices)
        self.host_pages = new_pages
        self.host_lens = [old_lens[i] for i in indices]
        self.block_table = torch.full((self.batch, self.max_pages), -1, dtype=torch.int32, device=self.pool.device)
        self.seq_lens = torch.tensor(self.host_lens, dtype=torch.int32, device=self.pool.device)
        self._upload_table()

    def release(self) -> None:
        for pages in self.host_pages:
            self.allocator.free(pages)
        self.host_pages = [[] for _ in range(self.batch)]
        self.host_lens = [0] * self.batch
        self.seq_lens.zero_()
        self.block_table.fill_(-1)
