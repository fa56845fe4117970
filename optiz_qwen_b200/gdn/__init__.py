"""Gated-DeltaNet hooks (recurrent step, chunked prefill) on sm_100a kernels."""

from .gated_delta_rule import (
    chunk_gated_delta_rule,
    fused_recurrent_gated_delta_rule,
    install_gdn_fastpath,
    recurrent_gated_delta_rule,
)

__all__ = [
    "chunk_gated_delta_rule",
    "fused_recurrent_gated_delta_rule",
    "install_gdn_fastpath",
    "recurrent_gated_delta_rule",
]
