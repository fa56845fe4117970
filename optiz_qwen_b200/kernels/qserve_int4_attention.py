"""INT4 / INT8 paged-KV decode attention launchers (drop-in for optiz_qwen/kernels/qserve_int4_attention.py).

Signatures, return shapes and error behaviour follow the reference launchers
(:516-660): ``fn(query [B, Hq, 1, D] CUDA, layer, *, scaling) -> [B, 1, Hq, D]``
in the query dtype; ``RuntimeError`` when the query is not a one-token CUDA
tensor or the layer holds no packed KV; ``ValueError`` on a non-integer GQA
ratio.  The INT4 launchers run one sm_100a kernel (C ABI
``oq_decode_attn_int4_paged``): the one-pass backend gives each (sequence, KV
head) a single CTA, the split backend cuts the KV range over CTAs and merges
the partials by log-sum-exp in the same launch.  The INT8 launcher runs the
8-bit instance of the same kernel (``oq_decode_attn_int8_paged``), split-KV.
"""

from __future__ import annotations

from typing import Any

import torch

from .. import _lib, cabi


def triton_int4_decode_available(query: torch.Tensor) -> bool:
    """Reference name kept for the fused-forward dispatch: a one-token CUDA query and a built library."""
    return bool(query.is_cuda and query.shape[-2] == 1 and _lib.available())


int4_decode_available = triton_int4_decode_available


def _paged_decode(query: torch.Tensor, layer: Any, scaling: float, num_splits: int, what: str,
                  gate: torch.Tensor | None = None, bits: int = 4) -> torch.Tensor:
    if not (query.is_cuda and query.shape[-2] == 1):
        raise RuntimeError(f"{what} requires a CUDA query with sequence length 1.")
    paged = getattr(layer, "paged", None)
    if paged is None or getattr(layer, "_key_code", None) is None:
        raise RuntimeError("Fused qserve attention requires packed KV tensors.")
    batch, num_heads, _, head_dim = query.shape
    num_kv_heads = paged.pool.num_kv_heads
    if num_heads % num_kv_heads:
        raise ValueError("Qwen GQA decode requires an integer query-to-KV head ratio.")
    q = query[:, :, 0, :]
    if gate is not None:  # the decode forward's output gate, [B, 1, Hq * D] -> [B, Hq, D]
        gate = gate.reshape(batch, num_heads, head_dim)
    if paged.pool.bits != bits:
        raise RuntimeError(f"{what} requires a {bits}-bit cache; this layer holds {paged.pool.bits}-bit codes.")
    out = cabi.decode_attention(q, paged.pool, paged.block_table, paged.seq_lens, scaling,
                                workspace=layer.decode_workspace(num_heads), num_splits=num_splits, gate=gate)
    return out.unsqueeze(1)


def qserve_int4_decode_attention(query: torch.Tensor, layer: Any, *, scaling: float,
                                 gate: torch.Tensor | None = None) -> torch.Tensor:
    """Attend to the packed cache with one KV range per (sequence, KV head).

    ``gate`` (``[B, 1, Hq * D]``, optional, an addition to the reference's signature)
    fuses the decode forward's ``* sigmoid(gate)`` into the kernel's output store."""
    return _paged_decode(query, layer, scaling, 1, "INT4 decode attention", gate)


def qserve_int4_split_decode_attention(query: torch.Tensor, layer: Any, *, scaling: float,
                                       gate: torch.Tensor | None = None) -> torch.Tensor:
    """Split-KV decode: KV ranges spread over the SMs, partials merged by log-sum-exp in-launch.

    ``gate``: as for :func:`qserve_int4_decode_attention`."""
    return _paged_decode(query, layer, scaling, 0, "INT4 split decode", gate)


def qserve_int8_decode_attention(query: torch.Tensor, layer: Any, *, scaling: float,
                                 gate: torch.Tensor | None = None) -> torch.Tensor:
    """Attend to an 8-bit packed cache (reference :548-573); split-KV with the in-launch merge.

    ``gate``: as for :func:`qserve_int4_decode_attention`."""
    return _paged_decode(query, layer, scaling, 0, "INT8 decode attention", gate, bits=8)
