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


def assert_attn_close(actual: np.ndarray, expected: np.ndarray) -> None:
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    err = np.abs(actual - expected)
    bound = ATTN_ATOL + ATTN_RTOL * np.abs(expected)
    assert np.all(np.isfinite(actual)), "non-finite attention output"
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), (
        f"attention mismatch: max |err| {err.max():.3e} at {worst}: {actual[worst]} vs {expected[worst]}")


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
