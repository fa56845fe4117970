"""Decode attention for the paged INT4 cache, behind the reference's kernel-module names."""

from .attention_backend import (
    ATTENTION_BACKEND_ENV_KEYS,
    DEFAULT_DECODE_BACKEND,
    DEFAULT_PREFILL_BACKEND,
    GRAPH_SAFE_BACKENDS,
    attention_backend,
    current_attention_backend,
    resolved_decode_backend,
    resolved_prefill_backend,
    set_attention_backend,
    validate_graph_backend,
)
from .qserve_int4_attention import (
    int4_decode_available,
    qserve_int4_decode_attention,
    qserve_int4_split_decode_attention,
    qserve_int8_decode_attention,
    triton_int4_decode_available,
)
from .qwen35_fused_attention import install_qwen35_fused_attention

__all__ = [
    "ATTENTION_BACKEND_ENV_KEYS",
    "DEFAULT_DECODE_BACKEND",
    "DEFAULT_PREFILL_BACKEND",
    "GRAPH_SAFE_BACKENDS",
    "attention_backend",
    "current_attention_backend",
    "install_qwen35_fused_attention",
    "int4_decode_available",
    "qserve_int4_decode_attention",
    "qserve_int4_split_decode_attention",
    "qserve_int8_decode_attention",
    "resolved_decode_backend",
    "resolved_prefill_backend",
    "set_attention_backend",
    "triton_int4_decode_available",
    "validate_graph_backend",
]
