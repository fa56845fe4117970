"""Oracle: fp32 decode attention over the dequantised INT4 cache, and LSE merging (numpy).

TEST INFRASTRUCTURE ONLY -- imported by tests, smoke() and bench.py's CPU legs.

Reference semantics: ``qserve_int4_split_decode_attention(query, layer, scaling=...)``
(optiz_qwen/kernels/qserve_int4_attention.py:576-620) computes one-token
attention of every query head over its KV head's whole cache (GQA: query head
``h`` reads KV head ``h // (Hq // Hkv)``, :34/:399-407), softmax over
``scaling * q.k``, output ``[B, 1, Hq, D]``.  The reference's own test checks it
against ``F.scaled_dot_product_attention`` over the dequantised cache with
``repeat_interleave`` (tests/test_qserve_kv_cache.py:175-195); this oracle is
that comparison in fp32 over the fp32-dequantised cache (stored fp16 scale/min).
"""

from __future__ import annotations

import numpy as np


def decode_attention(q: np.ndarray, keys, values, scaling: float):
    """One-token attention.

    ``q``: ``[B, Hq, D]`` float32.  ``keys[b]`` / ``values[b]``: ``[Hkv, T_b, D]`` float32
    (ragged per sequence).  Returns ``(out [B, Hq, D], lse [B, Hq])`` where ``lse`` is the
    natural-log log-sum-exp of ``scaling * q.k`` (``-inf`` and a zero row for T_b = 0).
    """
    q = np.asarray(q, np.float32)
    batch, num_heads, head_dim = q.shape
    out = np.zeros((batch, num_heads, head_dim), np.float32)
    lse = np.full((batch, num_heads), -np.inf, np.float32)
    for b in range(batch):
        k = np.asarray(keys[b], np.float32)
        v = np.asarray(values[b], np.float32)
        hkv, t, _ = k.shape
        if t == 0:
            continue
        group = num_heads // hkv
        qg = q[b].reshape(hkv, group, head_dim)
        scores = np.einsum("hgd,htd->hgt", qg, k) * np.float32(scaling)
        m = scores.max(axis=-1, keepdims=True)
        p = np.exp(scores - m)
        denom = p.sum(axis=-1, keepdims=True)
        o = np.einsum("hgt,htd->hgd", p, v) / denom
        out[b] = o.reshape(num_heads, head_dim)
        lse[b] = (m[..., 0] + np.log(denom[..., 0])).reshape(num_heads)
    return out, lse


def lse_merge(parts_out: np.ndarray, parts_lse: np.ndarray):
    """Merge partial attention results computed over disjoint KV ranges.

    ``parts_out``: ``[N, R, D]`` normalised partial outputs, ``parts_lse``: ``[N, R]``.
    ``out = sum_i exp(lse_i - lse) * out_i`` with ``lse = log sum_i exp(lse_i)``.
    Rows whose partials are all empty (``-inf``) merge to zeros / ``-inf``.
    """
    parts_out = np.asarray(parts_out, np.float32)
    parts_lse = np.asarray(parts_lse, np.float32)
    m = parts_lse.max(axis=0)
    safe_m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    w = np.where(np.isfinite(parts_lse), np.exp(parts_lse - safe_m[None]), 0.0).astype(np.float32)
    denom = w.sum(axis=0)
    out = np.einsum("nr,nrd->rd", w, parts_out)
    ok = denom > 0
    out[ok] /= denom[ok, None]
    out[~ok] = 0.0
    lse = np.where(ok, safe_m + np.log(np.where(ok, denom, 1.0)), -np.inf).astype(np.float32)
    return out.astype(np.float32), lse


def split_kv_ranges(length: int, parts: int, page_size: int):
    """Even split of ``[0, length)`` into ``parts`` page-aligned contiguous ranges."""
    pages = -(-length // page_size)
    per = -(-pages // parts)
    ranges = []
    for i in range(parts):
        lo = min(length, i * per * page_size)
        hi = min(length, (i + 1) * per * page_size)
        ranges.append((lo, hi))
    return ranges
