"""KV-chain builder (mirrors optiz_qwen/scheduling/kv_chain.py:15-63).

Only the retained chain ``qserve_deferred_split_fused_kv`` exists; it now
builds the paged INT4 cache served by the sm_100a kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from ..compression import QServeKvConfig, build_qserve_deferred_split_fused_kv_cache


@dataclass(frozen=True)
class KVChainReport:
    """Metadata describing which KV optimisation chain ran."""

    chain_name: str
    enabled: bool
    k_bits: int | None = None
    v_bits: int | None = None
    group_size: int | None = None
    residual_length: int | None = None
    activation_threshold: int | None = None
    decode_warmup_tokens: int | None = None
    attention_backend: str | None = None
    implementation: str | None = None


def build_kv_chain(*, chain_name: str, model_config: Any, enabled: bool,
                   qserve_config: QServeKvConfig | None = None) -> tuple[Any | None, KVChainReport]:
    """Build the selected KV chain object and a compact report."""
    normalized = chain_name.strip().lower()
    if not enabled:
        return None, KVChainReport(chain_name=normalized, enabled=False)
    if normalized == "qserve_deferred_split_fused_kv":
        cfg = qserve_config or QServeKvConfig()
        cache = build_qserve_deferred_split_fused_kv_cache(model_config, cfg)
        return cache, KVChainReport(
            chain_name=normalized, enabled=True, k_bits=cfg.k_bits, v_bits=cfg.v_bits, group_size=cfg.group_size,
            residual_length=cfg.residual_length, activation_threshold=cfg.activation_threshold,
            decode_warmup_tokens=cfg.decode_warmup_tokens, attention_backend=cfg.attention_backend,
            implementation="qserve_triton_int4_deferred_split_decode",
        )
    raise ValueError(f"unsupported KV chain: {chain_name}. Only qserve_deferred_split_fused_kv is retained.")
