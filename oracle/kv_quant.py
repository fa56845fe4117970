"""Oracle: asymmetric uint4 KV quantisation and the paged INT4 layout (numpy).

TEST INFRASTRUCTURE ONLY -- imported by tests, smoke() and bench.py's CPU legs,
never by the product path.

Reference algorithm: ``QServeAttentionLayer._quantize_groupwise`` /
``_dequantize_groupwise`` / ``_pack_uint4`` / ``_unpack_uint4`` in
optiz_qwen/compression/qserve_kv_cache.py:313-372.

* min/max per group in fp32 (:321-325),
* ``scale = (max - min) / 15`` in fp32, replaced by 1 where it is not > 0 (:326-328),
* ``code = clamp(round_half_even((x - min) / scale), 0, 15)`` (:329),
* even index in the low nibble, odd index in the high nibble (:356-362),
* dequant ``min + code * scale`` (:349-352).

The B200 cache stores one group per token per KV head (group = head_dim) and
keeps scale/min as fp16 (round-to-nearest-even of the fp32 values).  Codes are
computed with the fp32 scale/min exactly as the reference does; dequantisation
uses the stored fp16 values.
"""

from __future__ import annotations

import math

import numpy as np

# --------------------------------------------------------------------------- bf16 helpers


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = 0x7FC0
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------------------- reference quantiser


def quantize_groupwise(x: np.ndarray, group_size: int, bits: int):
    """Restates qserve_kv_cache.py:313-335.

    Returns ``(codes_packed_or_raw, scale_f32, min_f32)`` with scale/min of shape
    ``x.shape[:-1] + (groups,)`` -- the reference's squeezed outputs.
    """
    x = np.asarray(x, dtype=np.float32)
    last = x.shape[-1]
    if last % group_size != 0:
        raise ValueError(f"last dimension {last} must be divisible by group_size={group_size}")
    groups = last // group_size
    grouped = x.reshape(*x.shape[:-1], groups, group_size)
    gmin = grouped.min(axis=-1, keepdims=True)
    gmax = grouped.max(axis=-1, keepdims=True)
    levels = (1 << bits) - 1
    scale = (gmax - gmin) / np.float32(levels)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    codes = np.clip(np.rint((grouped - gmin) / scale), 0, levels).astype(np.uint8)
    flat = codes.reshape(*x.shape[:-1], last)
    packed = pack_uint4(flat) if bits == 4 else flat
    return packed, scale[..., 0], gmin[..., 0]


def pack_uint4(codes: np.ndarray) -> np.ndarray:
    """Restates qserve_kv_cache.py:356-362 (even index -> low nibble)."""
    codes = np.asarray(codes, dtype=np.uint8)
    if codes.shape[-1] % 2:
        codes = np.concatenate([codes, np.zeros(codes.shape[:-1] + (1,), np.uint8)], axis=-1)
    pairs = codes.reshape(*codes.shape[:-1], -1, 2)
    return ((pairs[..., 0] & 0x0F) | ((pairs[..., 1] & 0x0F) << 4)).astype(np.uint8)


def unpack_uint4(packed: np.ndarray, last_dim: int) -> np.ndarray:
    """Restates qserve_kv_cache.py:365-372."""
    packed = np.asarray(packed, dtype=np.uint8)
    low = packed & 0x0F
    high = (packed >> 4) & 0x0F
    vals = np.stack([low, high], axis=-1).reshape(*packed.shape[:-1], -1)
    return vals[..., :last_dim]


def dequantize_groupwise(packed, scale, gmin, group_size: int, last_dim: int, bits: int = 4):
    """Restates qserve_kv_cache.py:338-353 in fp32 (``dtype=float32``)."""
    codes = unpack_uint4(packed, last_dim) if bits == 4 else np.asarray(packed, np.uint8)
    groups = last_dim // group_size
    codes = codes.reshape(*codes.shape[:-1], groups, group_size).astype(np.float32)
    scale = np.asarray(scale, np.float32)[..., None]
    gmin = np.asarray(gmin, np.float32)[..., None]
    out = gmin + codes * scale
    return out.reshape(*out.shape[:-2], last_dim)


# --------------------------------------------------------------------------- B200 token format


def quantize_tokens_int4(x: np.ndarray):
    """Per-token per-head quantisation as stored by the B200 cache.

    ``x``: float32 ``[..., D]``.  Returns ``(packed u8 [..., D/2], scale f16 [...], min f16 [...])``.
    The group is the whole head (group_size = D); scale/min are the reference's
    fp32 values rounded to fp16 (RNE).
    """
    d = x.shape[-1]
    packed, scale, gmin = quantize_groupwise(x, d, 4)
    return packed, scale[..., 0].astype(np.float16), gmin[..., 0].astype(np.float16)


def dequantize_tokens_int4(packed, scale16, min16) -> np.ndarray:
    """fp32 dequantisation with the stored fp16 scale/min: ``min + code * scale``."""
    d = packed.shape[-1] * 2
    codes = unpack_uint4(packed, d).astype(np.float32)
    return np.asarray(min16, np.float32)[..., None] + codes * np.asarray(scale16, np.float32)[..., None]


def quantize_tokens_int8(x: np.ndarray):
    """The 8-bit variant of :func:`quantize_tokens_int4` (the reference's ``bits=8`` path of
    ``_quantize_groupwise``, qserve_kv_cache.py:313-335: 255 levels, codes unpacked).

    Returns ``(codes u8 [..., D], scale f16 [...], min f16 [...])``.
    """
    d = x.shape[-1]
    codes, scale, gmin = quantize_groupwise(x, d, 8)
    return codes, scale[..., 0].astype(np.float16), gmin[..., 0].astype(np.float16)


def dequantize_tokens_int8(codes, scale16, min16) -> np.ndarray:
    """fp32 dequantisation of 8-bit codes with the stored fp16 scale/min."""
    c = np.asarray(codes, np.uint8).astype(np.float32)
    return np.asarray(min16, np.float32)[..., None] + c * np.asarray(scale16, np.float32)[..., None]


# --------------------------------------------------------------------------- paged layout

META_K_SCALE, META_K_MIN, META_V_SCALE, META_V_MIN = 0, 1, 2, 3


def page_permutation(num_pages: int, seed: int | None) -> np.ndarray:
    """Order in which the page allocator hands out physical pages.

    ``seed=None`` -> identity order; otherwise a numpy PCG64 permutation.  The
    product allocator (``optiz_qwen_b200.compression.paged_kv.PageAllocator``)
    uses the same policy, so block tables can be compared bit for bit.
    """
    if seed is None:
        return np.arange(num_pages, dtype=np.int32)
    return np.random.default_rng(seed).permutation(num_pages).astype(np.int32)


def build_block_table(lengths, page_size: int, num_pages: int, max_pages_per_seq: int, seed=None):
    """Give each sequence, in batch order, ``ceil(len/page_size)`` pages from the permuted free list."""
    order = page_permutation(num_pages, seed)
    table = np.full((len(lengths), max_pages_per_seq), -1, dtype=np.int32)
    cursor = 0
    for b, length in enumerate(lengths):
        need = -(-int(length) // page_size)
        if need > max_pages_per_seq or cursor + need > num_pages:
            raise ValueError("page pool too small for the requested lengths")
        table[b, :need] = order[cursor:cursor + need]
        cursor += need
    return table


class PagedKvOracle:
    """numpy mirror of the paged INT4 (or INT8) pool.

    ``kv_codes``: uint8 ``[num_pages, Hkv, 2, page_size, D * bits / 8]`` (index 0 = K, 1 = V)
    ``kv_meta`` : float16 ``[num_pages, Hkv, 4, page_size]`` (k_scale, k_min, v_scale, v_min)
    """

    def __init__(self, num_pages, num_kv_heads, head_dim, page_size, block_table, seq_lens, bits: int = 4):
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        self.page_size = page_size
        self.head_dim = head_dim
        self.bits = bits
        self.kv_codes = np.zeros((num_pages, num_kv_heads, 2, page_size, head_dim * bits // 8), np.uint8)
        self.kv_meta = np.zeros((num_pages, num_kv_heads, 4, page_size), np.float16)
        self.block_table = np.asarray(block_table, np.int32)
        self.seq_lens = np.asarray(seq_lens, np.int64).copy()

    def append(self, keys: np.ndarray, values: np.ndarray, rows=None) -> None:
        """Append ``[B, Hkv, n, D]`` float32 tokens at each sequence's current length.

        ``rows`` names the batch rows the tokens belong to (default: all rows in order).
        """
        quant = quantize_tokens_int4 if self.bits == 4 else quantize_tokens_int8
        kp, ks, km = quant(keys)
        vp, vs, vm = quant(values)
        batch, _, n, _ = keys.shape
        rows = range(batch) if rows is None else rows
        for i, b in enumerate(rows):
            pos = int(self.seq_lens[b]) + np.arange(n)
            pages = self.block_table[b, pos // self.page_size]
            if np.any(pages < 0):
                raise ValueError("block table has no page for an appended position")
            slots = pos % self.page_size
            self.kv_codes[pages, :, 0, slots] = kp[i].transpose(1, 0, 2)
            self.kv_codes[pages, :, 1, slots] = vp[i].transpose(1, 0, 2)
            self.kv_meta[pages, :, META_K_SCALE, slots] = ks[i].T
            self.kv_meta[pages, :, META_K_MIN, slots] = km[i].T
            self.kv_meta[pages, :, META_V_SCALE, slots] = vs[i].T
            self.kv_meta[pages, :, META_V_MIN, slots] = vm[i].T
            self.seq_lens[b] += n

    def gather(self, b: int):
        """Dequantised fp32 ``(K, V)`` of sequence ``b``: ``[Hkv, T, D]`` each."""
        length = int(self.seq_lens[b])
        npages = -(-length // self.page_size)
        pages = self.block_table[b, :npages]
        codes = self.kv_codes[pages]                     # [np, H, 2, P, D/2]
        meta = self.kv_meta[pages]                       # [np, H, 4, P]
        codes = codes.transpose(1, 2, 0, 3, 4).reshape(codes.shape[1], 2, -1, codes.shape[-1])[:, :, :length]
        meta = meta.transpose(1, 2, 0, 3).reshape(meta.shape[1], 4, -1)[:, :, :length]
        deq = dequantize_tokens_int4 if self.bits == 4 else dequantize_tokens_int8
        k = deq(codes[:, 0], meta[:, META_K_SCALE], meta[:, META_K_MIN])
        v = deq(codes[:, 1], meta[:, META_V_SCALE], meta[:, META_V_MIN])
        return k, v


def fill_paged_cache(rng: np.random.Generator, lengths, num_kv_heads, head_dim, page_size,
                     num_pages=None, max_pages_per_seq=None, seed_pages=None, chunk=4096, bits: int = 4):
    """Build a populated ``PagedKvOracle`` with bf16-valued N(0,1) K/V (config-0 distribution).

    Returns the oracle; its pool arrays can be uploaded to the device as-is.
    """
    lengths = [int(x) for x in lengths]
    need = sum(-(-n // page_size) for n in lengths)
    num_pages = num_pages or need
    max_pages_per_seq = max_pages_per_seq or max(1, max(-(-n // page_size) for n in lengths))
    table = build_block_table(lengths, page_size, num_pages, max_pages_per_seq, seed_pages)
    cache = PagedKvOracle(num_pages, num_kv_heads, head_dim, page_size, table, np.zeros(len(lengths)), bits=bits)
    for b, n in enumerate(lengths):
        start = 0
        while start < n:
            m = min(chunk, n - start)
            k = round_bf16(rng.standard_normal((1, num_kv_heads, m, head_dim), dtype=np.float32))
            v = round_bf16(rng.standard_normal((1, num_kv_heads, m, head_dim), dtype=np.float32))
            cache.append(k, v, rows=[b])
            start += m
    return cache


def pages_needed(length: int, page_size: int) -> int:
    return int(math.ceil(length / page_size))
