"""Oracle: the gated delta rule (Gated DeltaNet) in numpy fp32.

TEST INFRASTRUCTURE ONLY -- imported by tests, smoke() and bench.py's CPU legs.

The reference's GDN arithmetic is third-party: its hook falls back to
``torch_recurrent_gated_delta_rule`` / ``torch_chunk_gated_delta_rule`` /
``torch_causal_conv1d_update`` from transformers
(models/qwen3_5/modeling_qwen3_5.py:210-353; the reference pins transformers
5.10.1, this container carries 5.5.0 with the same functions), or to
fla-core 0.5.1's Triton kernels.  These restatements follow the transformers
functions line by line; ``tests/golden/make_golden.py`` pins them against the
transformers code itself.

Shapes follow the hook convention: ``q, k`` ``[B, T, H, Dk]``, ``v`` ``[B, T, H, Dv]``,
``g, beta`` ``[B, T, H]``, state ``[B, H, Dk, Dv]``.
"""

from __future__ import annotations

import numpy as np


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """modeling_qwen3_5.py:228-231: ``x * rsqrt(sum(x*x) + eps)`` along the last axis."""
    x = np.asarray(x, np.float32)
    inv = np.float32(1.0) / np.sqrt((x * x).sum(axis=-1, keepdims=True) + np.float32(eps))
    return (x * inv).astype(np.float32)


def decay_gates(a, b, a_log, dt_bias, rnd=None):
    """The decode branch's gate arithmetic (modeling_qwen3_5.py:492-493), ahead of the hook call.

    ``beta = b.sigmoid()`` in b's dtype (``rnd`` rounds to it; None: fp32) and, in fp32,
    ``g = -exp(A_log) * softplus(a + dt_bias)`` with torch's softplus (threshold 20: the
    identity above it).  ``a``, ``b`` ``[B, T, H]``; ``a_log``, ``dt_bias`` ``[H]``.
    Returns ``(g, beta)`` as float32.
    """
    a, b, a_log, dt_bias = (np.asarray(x, np.float32) for x in (a, b, a_log, dt_bias))
    beta = (np.float32(1.0) / (np.float32(1.0) + np.exp(-b))).astype(np.float32)
    if rnd is not None:
        beta = rnd(beta)
    x = (a + dt_bias).astype(np.float32)
    with np.errstate(over="ignore"):
        softplus = np.where(x > np.float32(20.0), x, np.log1p(np.exp(x))).astype(np.float32)
    g = (-np.exp(a_log) * softplus).astype(np.float32)
    return g, beta


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, output_final_state=True,
                               use_qk_l2norm_in_kernel=False, scale=None):
    """modeling_qwen3_5.py:314-353 in fp32.

    Per token and head: ``S *= exp(g)``; ``kv = S^T k``; ``delta = beta (v - kv)``;
    ``S += k delta^T``; ``o = S^T (q * scale)``.
    """
    q, k, v, g, beta = (np.asarray(x, np.float32) for x in (q, k, v, g, beta))
    if use_qk_l2norm_in_kernel:
        q, k = l2norm(q), l2norm(k)
    batch, seq, heads, dk = k.shape
    dv = v.shape[-1]
    scale = np.float32(dk ** -0.5 if scale is None else scale)
    q = q * scale
    state = (np.zeros((batch, heads, dk, dv), np.float32) if initial_state is None
             else np.array(initial_state, np.float32, copy=True))
    out = np.zeros((batch, seq, heads, dv), np.float32)
    for t in range(seq):
        q_t, k_t, v_t = q[:, t], k[:, t], v[:, t]                 # [B, H, D]
        state *= np.exp(g[:, t])[:, :, None, None]
        kv_mem = np.einsum("bhkv,bhk->bhv", state, k_t)
        delta = (v_t - kv_mem) * beta[:, t][:, :, None]
        state += k_t[:, :, :, None] * delta[:, :, None, :]
        out[:, t] = np.einsum("bhkv,bhk->bhv", state, q_t)
    return out, (state if output_final_state else None)


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None,
                           output_final_state=True, use_qk_l2norm_in_kernel=False, scale=None):
    """modeling_qwen3_5.py:234-311 in fp32 (chunked WY form, zero padding to a chunk multiple)."""
    q, k, v, g, beta = (np.asarray(x, np.float32) for x in (q, k, v, g, beta))
    if use_qk_l2norm_in_kernel:
        q, k = l2norm(q), l2norm(k)
    # [B, T, H, D] -> [B, H, T, D]
    q, k, v = (x.transpose(0, 2, 1, 3) for x in (q, k, v))
    g, beta = (x.transpose(0, 2, 1) for x in (g, beta))
    batch, heads, seq, dk = k.shape
    dv = v.shape[-1]
    c = chunk_size
    pad = (c - seq % c) % c
    if pad:
        q, k, v = (np.pad(x, ((0, 0), (0, 0), (0, pad), (0, 0))) for x in (q, k, v))
        g, beta = (np.pad(x, ((0, 0), (0, 0), (0, pad))) for x in (g, beta))
    total = seq + pad
    nchunks = total // c
    scale = np.float32(dk ** -0.5 if scale is None else scale)
    q = q * scale
    v_beta = v * beta[..., None]
    k_beta = k * beta[..., None]
    q, k, v, k_beta, v_beta = (x.reshape(batch, heads, nchunks, c, x.shape[-1])
                               for x in (q, k, v, k_beta, v_beta))
    g = g.reshape(batch, heads, nchunks, c).cumsum(axis=-1, dtype=np.float32)
    tril_incl = np.tril(np.ones((c, c), bool))
    decay = np.where(tril_incl, np.exp(np.where(tril_incl, g[..., :, None] - g[..., None, :], 0.0)), 0.0)
    decay = decay.astype(np.float32)
    attn = -(k_beta @ k.swapaxes(-1, -2)) * decay
    attn = np.where(np.tril(np.ones((c, c), bool), -1), attn, 0.0).astype(np.float32)
    for i in range(1, c):
        row = attn[..., i, :i].copy()
        sub = attn[..., :i, :i].copy()
        attn[..., i, :i] = row + (row[..., :, None] * sub).sum(axis=-2)
    attn = attn + np.eye(c, dtype=np.float32)
    value = attn @ v_beta
    k_cumdecay = attn @ (k_beta * np.exp(g)[..., None])
    state = (np.zeros((batch, heads, dk, dv), np.float32) if initial_state is None
             else np.array(initial_state, np.float32, copy=True))
    out = np.zeros_like(value)
    causal = np.tril(np.ones((c, c), bool))
    for i in range(nchunks):
        q_i, k_i, v_i = q[:, :, i], k[:, :, i], value[:, :, i]
        a = np.where(causal, (q_i @ k_i.swapaxes(-1, -2)) * decay[:, :, i], 0.0).astype(np.float32)
        v_prime = k_cumdecay[:, :, i] @ state
        v_new = v_i - v_prime
        attn_inter = (q_i * np.exp(g[:, :, i])[..., None]) @ state
        out[:, :, i] = attn_inter + a @ v_new
        g_last = g[:, :, i, -1]
        state = (state * np.exp(g_last)[..., None, None]
                 + (k_i * np.exp(g_last[..., None] - g[:, :, i])[..., None]).swapaxes(-1, -2) @ v_new)
    out = out.reshape(batch, heads, total, dv)[:, :, :seq].transpose(0, 2, 1, 3)
    return np.ascontiguousarray(out, np.float32), (state if output_final_state else None)


def causal_conv1d_update(x, conv_state, weight, bias=None, silu=True):
    """modeling_qwen3_5.py:210-225: depthwise causal conv over ``[state | x]`` then SiLU.

    ``x``: ``[B, C, T]``, ``conv_state``: ``[B, C, W]`` (updated in place with the
    last ``W`` inputs), ``weight``: ``[C, K]``.  Returns ``[B, C, T]`` float32.
    """
    x = np.asarray(x, np.float32)
    batch, channels, seq = x.shape
    width = conv_state.shape[-1]
    ksize = weight.shape[-1]
    full = np.concatenate([conv_state.astype(np.float32), x], axis=-1)
    conv_state[...] = full[:, :, -width:]
    out = np.zeros((batch, channels, seq), np.float32)
    w = np.asarray(weight, np.float32)
    for t in range(seq):
        end = width + t + 1
        window = full[:, :, end - ksize:end]
        out[:, :, t] = (window * w[None]).sum(-1)
    if bias is not None:
        out += np.asarray(bias, np.float32)[None, :, None]
    if silu:
        out = out / (1.0 + np.exp(-out))
    return out.astype(np.float32)
