"""Paged INT4 KV cache behind the reference's QServe cache API (optiz_qwen.compression)."""

from .paged_kv import PageAllocator, PagedKvState
from .qserve_kv_cache import (
    VALID_BACKENDS,
    QServeAttentionLayer,
    QServeDeferredSplitFusedAttentionLayer,
    QServeDeferredSplitFusedKvCache,
    QServeFusedAttentionLayer,
    QServeFusedKvCache,
    QServeKvCache,
    QServeKvCacheReport,
    QServeKvConfig,
    QServeSplitFusedKvCache,
    build_qserve_deferred_split_fused_kv_cache,
)

__all__ = [
    "PageAllocator",
    "PagedKvState",
    "QServeAttentionLayer",
    "QServeDeferredSplitFusedAttentionLayer",
    "QServeDeferredSplitFusedKvCache",
    "QServeFusedAttentionLayer",
    "QServeFusedKvCache",
    "QServeKvCache",
    "QServeKvCacheReport",
    "QServeKvConfig",
    "QServeSplitFusedKvCache",
    "VALID_BACKENDS",
    "build_qserve_deferred_split_fused_kv_cache",
]
