"""Shared helpers for the parity tests (tolerances are the contract's)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import kv_quant as kq

# Attention: max-abs 2e-3 and rel 1e-2 vs fp32 attention over the dequantised cache.
ATTN_ATOL = 2e-3
ATTN_RTOL = 1e-2
# GDN state and outputs: rel 1e-4 in fp32 (normwise, plus an elementwise bound of the same size
# relative to the tensor's largest magnitude).
GDN_RTOL = 1e-4


def attn_margin(actual: np.ndarray, expected: np.ndarray) -> float:
    """Largest |err| / (ATTN_ATOL + ATTN_RTOL |ref|): the share of the tolerance used (<= 1 passes)."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    return float(np.max(np.abs(actual - expected) / (ATTN_ATOL + ATTN_RTOL * np.abs(expected))))


def assert_attn_close(actual: np.ndarray, expected: np.ndarray) -> float:
    """Asserts the attention tolerance; returns the share of it used (see :func:`attn_margin`)."""
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    err = np.abs(actual - expected)
    bound = ATTN_ATOL + ATTN_RTOL * np.abs(expected)
    assert np.all(np.isfinite(actual)), "non-finite attention output"
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), (
        f"attention mismatch: max |err| {err.max():.3e} at {worst}: {actual[worst]} vs {expected[worst]}")
    return attn_margin(actual, expected)


def random_paged_cache(rng: np.random.Generator, lengths, num_kv_heads: int, head_dim: int, page_size: int,
                       seed_pages=None, *, k_scale=(0.30, 0.42), k_min=(-3.1, -2.3), v_scale=(0.30, 0.42),
                       v_min=(-3.1, -2.3)) -> kq.PagedKvOracle:
    """A populated INT4 ``PagedKvOracle`` without running the quantiser: codes uniform on [0, 15] and
    fp16 scale / min uniform on the given ranges (the defaults are what per-token groups of 256
    N(0,1) values give: min about -2.7, scale about 0.36).  Used for long contexts, where
    quantising N(0,1) data in numpy would dominate the test's time; the attention oracle
    dequantises the stored codes and fp16 values either way."""
    lengths = [int(x) for x in lengths]
    need = sum(-(-n // page_size) for n in lengths)
    max_pages = max(1, max(-(-n // page_size) for n in lengths))
    table = kq.build_block_table(lengths, page_size, need, max_pages, seed_pages)
    cache = kq.PagedKvOracle(need, num_kv_heads, head_dim, page_size, table, lengths)
    cache.kv_codes[...] = rng.integers(0, 256, cache.kv_codes.shape, dtype=np.uint8)
    meta = np.empty(cache.kv_meta.shape, np.float32)
    for idx, (lo, hi) in enumerate((k_scale, k_min, v_scale, v_min)):
        meta[:, :, idx] = rng.uniform(lo, hi, meta[:, :, idx].shape)
    cache.kv_meta[...] = meta.astype(np.float16)
    return cache


def oracle_from_device(pool, block_table: torch.Tensor, seq_lens: torch.Tensor, rows) -> kq.PagedKvOracle:
    """The sequences ``rows`` of a device pool as a ``PagedKvOracle`` (their pages downloaded and
    renumbered in order; row i of the result is sequence rows[i])."""
    rows = [int(r) for r in rows]
    table = block_table.cpu().numpy()
    lens = seq_lens.cpu().numpy().astype(np.int64)
    page = pool.page_size
    pages = [table[r, : -(-int(lens[r]) // page)] for r in rows]
    flat = np.concatenate(pages) if pages else np.zeros(0, np.int64)
    idx = torch.from_numpy(flat.astype(np.int64)).to(pool.kv_codes.device)
    max_pages = max(1, max(len(x) for x in pages))
    new_table = np.full((len(rows), max_pages), -1, np.int32)
    off = 0
    for i, x in enumerate(pages):
        new_table[i, : len(x)] = np.arange(off, off + len(x))
        off += len(x)
    cache = kq.PagedKvOracle(max(1, len(flat)), pool.num_kv_heads, pool.head_dim, page, new_table,
                             [int(lens[r]) for r in rows], bits=pool.bits)
    if len(flat):
        cache.kv_codes[...] = pool.kv_codes.index_select(0, idx).cpu().numpy()
        cache.kv_meta[...] = pool.kv_meta.index_select(0, idx).cpu().numpy()
    return cache


def assert_gdn_close(actual: np.ndarray, expected: np.ndarray, rtol: float = GDN_RTOL) -> None:
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert np.all(np.isfinite(actual)), "non-finite GDN output"
    scale = max(np.abs(expected).max(), 1e-30)
    max_err = np.abs(actual - expected).max()
    norm_err = np.linalg.norm(actual - expected) / max(np.linalg.norm(expected), 1e-30)
    assert norm_err <= rtol, f"GDN normwise rel err {norm_err:.3e} > {rtol}"
    assert max_err <= rtol * scale, f"GDN max err {max_err:.3e} > {rtol} x max|ref| ({scale:.3e})"


def bf16_tensor(x: np.ndarray, device="cuda") -> torch.Tensor:
    """float32 numpy (bf16-representable values) -> bf16 torch tensor."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(device=device, dtype=torch.bfloat16)


def upload_pool(cache: kq.PagedKvOracle, device="cuda"):
    """Copy an oracle cache into a device PagedKvPool + block table + seq_lens."""
    from optiz_qwen_b200.cabi import PagedKvPool

    num_pages, hkv, _, page, _ = cache.kv_codes.shape
    pool = PagedKvPool(num_pages, hkv, cache.head_dim, page, device, bits=cache.bits)
    pool.kv_codes.copy_(torch.from_numpy(cache.kv_codes))
    pool.kv_meta.copy_(torch.from_numpy(cache.kv_meta))
    table = torch.from_numpy(cache.block_table.astype(np.int32)).to(device)
    lens = torch.from_numpy(cache.seq_lens.astype(np.int32)).to(device)
    return pool, table, lens


def oracle_attention(cache: kq.PagedKvOracle, q: np.ndarray, scaling: float):
    from oracle.attention import decode_attention

    keys, values = [], []
    for b in range(q.shape[0]):
        if int(cache.seq_lens[b]) == 0:
            hkv = cache.kv_codes.shape[1]
            keys.append(np.zeros((hkv, 0, q.shape[-1]), np.float32))
            values.append(np.zeros((hkv, 0, q.shape[-1]), np.float32))
            continue
        k, v = cache.gather(b)
        keys.append(k)
        values.append(v)
    return decode_attention(q, keys, values, scaling)
