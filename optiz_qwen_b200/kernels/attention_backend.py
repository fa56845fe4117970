"""Attention-backend switch for prefill vs captured decode (mirrors optiz_qwen/kernels/attention_backend.py).

transformers resolves the attention kernel from ``config._attn_implementation``
on every forward call, and a captured CUDA graph freezes whichever kernels ran
at capture time; so a decode graph captured under one backend can coexist with
prefill dispatched to another.  This module only mutates the config.  The paged
INT4 path needs no backend entry: its cache keeps fixed device addresses and
its launches are graph-capturable on their own.
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Any, Iterator

#: backends known to survive CUDA-graph capture of the decode step
GRAPH_SAFE_BACKENDS = ("sdpa", "flash_attention_2")
#: backends accepted for the (uncaptured) prefill pass
PREFILL_BACKENDS = ("sdpa", "flash_attention_2", "eager")
DEFAULT_PREFILL_BACKEND = "sdpa"
DEFAULT_DECODE_BACKEND = "flash_attention_2"
ATTENTION_BACKEND_ENV_KEYS = ("OPTIZ_QWEN_ATTN_PREFILL", "OPTIZ_QWEN_ATTN_DECODE")


def resolved_prefill_backend() -> str:
    """Prefill backend from ``OPTIZ_QWEN_ATTN_PREFILL``, else the default."""
    return os.environ.get("OPTIZ_QWEN_ATTN_PREFILL", "").strip().lower() or DEFAULT_PREFILL_BACKEND


def resolved_decode_backend() -> str:
    """Decode backend from ``OPTIZ_QWEN_ATTN_DECODE``, else the default."""
    return os.environ.get("OPTIZ_QWEN_ATTN_DECODE", "").strip().lower() or DEFAULT_DECODE_BACKEND


def current_attention_backend(model: Any) -> str | None:
    config = getattr(model, "config", None)
    return None if config is None else getattr(config, "_attn_implementation", None)


def set_attention_backend(model: Any, backend: str) -> str | None:
    """Select ``backend`` on the model config and its text config; return the previous one."""
    normalized = str(backend).strip().lower()
    if not normalized:
        raise ValueError("attention backend must be a non-empty string")
    config = getattr(model, "config", None)
    if config is None:
        raise ValueError("model has no config; cannot select an attention backend")
    previous = getattr(config, "_attn_implementation", None)
    config._attn_implementation = normalized
    text_config = getattr(config, "text_config", None)
    if text_config is not None:
        text_config._attn_implementation = normalized
    return previous


@contextmanager
def attention_backend(model: Any, backend: str | None) -> Iterator[str | None]:
    """Temporarily select ``backend`` (``None`` is a no-op), restoring the previous one on exit."""
    if backend is None:
        yield current_attention_backend(model)
        return
    previous = set_attention_backend(model, backend)
    try:
        yield previous
    finally:
        if previous is not None:
            set_attention_backend(model, previous)


def validate_graph_backend(backend: str) -> str:
    """Reject decode backends that cannot survive CUDA-graph capture."""
    normalized = str(backend).strip().lower()
    if normalized not in GRAPH_SAFE_BACKENDS:
        raise ValueError(f"attention backend {normalized!r} is not graph-safe; choose one of {GRAPH_SAFE_BACKENDS}.")
    return normalized
