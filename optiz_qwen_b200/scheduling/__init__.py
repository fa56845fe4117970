"""KV-chain selection (caller of the cache API, kept so existing call sites work)."""

from .kv_chain import KVChainReport, build_kv_chain

__all__ = ["KVChainReport", "build_kv_chain"]
