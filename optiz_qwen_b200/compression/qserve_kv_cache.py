"""Drop-in QServe packed-KV cache for Qwen3.5, stored as paged INT4 (or INT8) on the GPU.

Same public surface as optiz_qwen/compression/qserve_kv_cache.py (config,
layer and cache classes, builder, report, counters), with a different storage
engine behind it:

* every token is quantised when it is appended, by the fused CUDA
  append-quantize kernel, into 64-token pages of a per-layer pool
  (the reference keeps a dense bf16 window of ``residual_length`` tokens and
  re-concatenates the whole code tensor with ``torch.cat``, :210-232, :374-377);
* one group per token per KV head (``group_size`` must equal ``head_dim``),
  scale/min stored as fp16 (the reference keeps fp32, :325-331);
* codes are bit-identical to the reference quantiser on the same token
  (round-half-even of ``(x - min) / scale`` in fp32, :313-335).

Because a token's codes depend only on that token, appending is exactly
equivalent to the reference's "rebuild from full" re-quantisation (:116-124),
so multi-token updates append instead of rebuilding.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .. import cabi
from .paged_kv import PageAllocator, PagedKvState

try:  # the cache classes plug into transformers like the reference's do
    from transformers.cache_utils import CacheLayerMixin, DynamicCache
except Exception:  # pragma: no cover - transformers is a runtime dependency of the model path
    class CacheLayerMixin:  # minimal stand-in so the module imports without transformers
        is_compileable = False

        def __init__(self):
            self.keys = None
            self.values = None
            self.is_initialized = False

    DynamicCache = None

VALID_BACKENDS = ("triton_int4_decode", "triton_int4_split_decode", "triton_int8_decode")


@dataclass(frozen=True)
class QServeKvConfig:
    """Runtime preset (mirrors qserve_kv_cache.py:24-54).

    Backend names are the reference's own, kept so existing configuration and
    the fused-forward dispatch work unchanged; they now select the sm_100a
    kernels (``*_int4_decode`` -> one KV range per CTA, ``*_int4_split_decode``
    -> split-KV with an in-launch log-sum-exp merge).  ``group_size`` must equal
    the model's head_dim (per-token groups).  ``residual_length`` is validated
    as in the reference but no dense window is kept: per-token groups need none.
    """

    k_bits: int = 4
    v_bits: int = 4
    group_size: int = 256
    residual_length: int = 256
    activation_threshold: int = 1024
    decode_warmup_tokens: int = 4
    attention_backend: str = "triton_int4_split_decode"
    page_size: int = 64
    page_seed: int | None = None

    def validate(self) -> None:
        if self.k_bits not in {4, 8} or self.v_bits != self.k_bits:
            raise ValueError("qserve_kv supports matched 4-bit or 8-bit K/V only.")
        if self.group_size <= 0:
            raise ValueError("qserve_kv group_size must be positive.")
        if self.residual_length <= 0:
            raise ValueError("qserve_kv residual_length must be positive.")
        if self.residual_length % self.group_size != 0:
            raise ValueError("qserve_kv residual_length must be divisible by group_size.")
        if self.activation_threshold < self.residual_length:
            raise ValueError("qserve_kv activation_threshold must be at least residual_length.")
        if self.decode_warmup_tokens < 0:
            raise ValueError("qserve_kv decode_warmup_tokens must be non-negative.")
        if self.attention_backend not in VALID_BACKENDS:
            raise ValueError("qserve_kv attention_backend must be a retained Triton decode backend.")
        if self.k_bits == 8 and self.attention_backend != "triton_int8_decode":
            raise ValueError("8-bit QServe KV requires triton_int8_decode.")
        if self.k_bits == 4 and self.attention_backend == "triton_int8_decode":
            raise ValueError("triton_int8_decode requires 8-bit QServe KV.")
        if self.page_size != cabi.PAGE_SIZE:
            raise ValueError(f"qserve_kv page_size must be {cabi.PAGE_SIZE} on this build.")


@dataclass(frozen=True)
class QServeKvCacheReport:
    enabled: bool
    full_attention_layers: tuple[int, ...]
    k_bits: int
    v_bits: int
    group_size: int
    residual_length: int
    activation_threshold: int
    decode_warmup_tokens: int
    attention_backend: str
    implementation: str = "qserve_deferred_split_packed_kv"


class QServeAttentionLayer(CacheLayerMixin):
    """Full-attention layer cache backed by a paged INT4 (or INT8, ``k_bits = 8``) pool
    (qserve_kv_cache.py:71-377)."""

    is_compileable = False
    supports_early_init = True
    is_sliding = False

    def __init__(self, config: QServeKvConfig) -> None:
        super().__init__()
        config.validate()
        self.config = config
        self.keys = None
        self.values = None
        self.device = None
        self.dtype = None
        self.is_initialized = False
        self._seq_length = 0
        self.paged: PagedKvState | None = None
        self._workspace: torch.Tensor | None = None
        self._workspace_key = None

    # ------------------------------------------------------------------ reference surface
    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype = key_states.dtype
        self.device = key_states.device
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        key_states = key_states.contiguous()
        value_states = value_states.contiguous()
        if self._seq_length == 0:
            self._rebuild_from_full(key_states, value_states)
            return key_states, value_states
        if key_states.shape[-2] == 1:
            self._append_decode_token(key_states, value_states)
            return self.materialize()
        previous_keys, previous_values = self.materialize()
        self._append(key_states, value_states)
        return (torch.cat([previous_keys, key_states], dim=-2), torch.cat([previous_values, value_states], dim=-2))

    def materialize(self) -> tuple[torch.Tensor, torch.Tensor]:
        if not self.is_initialized or self._seq_length == 0 or self.paged is None:
            raise ValueError("qserve_kv cache layer is empty and cannot be materialized.")
        keys, values = cabi.gather_dequant(self.paged.pool, self.paged.block_table, self.paged.seq_lens,
                                           self._seq_length, self.dtype)
        self.keys, self.values = keys, values
        return keys, values

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.get_seq_length() + query_length, 0

    def get_seq_length(self) -> int:
        return self._seq_length

    def get_max_length(self) -> int:
        return -1

    def get_max_cache_shape(self) -> int:
        return self.get_max_length()

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.get_seq_length() - abs(max_length)
        if self.get_seq_length() <= max_length or self.paged is None:
            return
        self.paged.set_lengths([max_length] * self.paged.batch)
        self._seq_length = int(max_length)

    def batch_repeat_interleave(self, repeats: int) -> None:
        if self.get_seq_length() == 0 or self.paged is None:
            return
        self.paged.select_rows([b for b in range(self.paged.batch) for _ in range(int(repeats))])

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        if self.get_seq_length() == 0 or self.paged is None:
            return
        self.paged.select_rows(torch.as_tensor(indices).reshape(-1).tolist())

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        self.batch_select_indices(beam_idx)

    def reset(self) -> None:
        if self.paged is not None:
            self.paged.release()
        self.paged = None
        self._seq_length = 0
        self.keys = None
        self.values = None
        self.is_initialized = False

    # ------------------------------------------------------------------ storage engine
    def _rebuild_from_full(self, keys: torch.Tensor, values: torch.Tensor, extra_tokens: int = 0) -> None:
        if keys.shape[-1] != self.config.group_size:
            raise ValueError(
                f"qserve_kv paged cache keeps one group per token: group_size ({self.config.group_size}) "
                f"must equal head_dim ({keys.shape[-1]}).")
        self.dtype = keys.dtype
        self.device = keys.device
        self.is_initialized = True
        batch, heads, seq, dim = keys.shape
        if self.paged is not None:
            self.paged.release()
        if self.paged is None or self.paged.batch != batch or self.paged.pool.num_kv_heads != heads:
            cap = seq + 1 + int(extra_tokens)
            pages = max(4, 2 * batch * cabi.pages_for(cap, self.config.page_size))
            pool = cabi.PagedKvPool(pages, heads, dim, self.config.page_size, keys.device, bits=self.config.k_bits)
            self.paged = PagedKvState(pool, batch, max_pages=cabi.pages_for(cap, self.config.page_size),
                                      allocator=PageAllocator(pages, self.config.page_seed))
        self._seq_length = 0
        self._append(keys, values)
        self.keys = None
        self.values = None

    def _append_decode_token(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype = key_states.dtype
        self.device = key_states.device
        self.is_initialized = True
        self._append(key_states, value_states)
        self.keys = None
        self.values = None

    def _append(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        if self.paged is None:
            self._rebuild_from_full(keys, values)
            return
        self.paged.append(keys, values)
        self._seq_length += int(keys.shape[-2])

    def decode_workspace(self, num_heads: int) -> torch.Tensor:
        """Zeroed split-KV workspace for this layer's batch shape (grown on demand)."""
        key = (self.paged.batch, num_heads, self.paged.pool.num_kv_heads, self.paged.max_pages)
        if self._workspace is None or self._workspace_key != key:
            self._workspace = cabi.new_decode_workspace(*key, self.paged.pool.device)
            self._workspace_key = key
        return self._workspace

    # reference attribute names: packed storage views (None until something is packed)
    @property
    def _key_code(self):
        return None if self.paged is None or self._seq_length == 0 else self.paged.pool.kv_codes[:, :, 0]

    @property
    def _value_code(self):
        return None if self.paged is None or self._seq_length == 0 else self.paged.pool.kv_codes[:, :, 1]

    @property
    def _key_scale(self):
        return None if self.paged is None else self.paged.pool.kv_meta[:, :, 0]

    @property
    def _key_min(self):
        return None if self.paged is None else self.paged.pool.kv_meta[:, :, 1]

    @property
    def _value_scale(self):
        return None if self.paged is None else self.paged.pool.kv_meta[:, :, 2]

    @property
    def _value_min(self):
        return None if self.paged is None else self.paged.pool.kv_meta[:, :, 3]


class QServeFusedAttentionLayer(QServeAttentionLayer):
    """Decode returns the new token's dense K/V; attention reads the packed pool (:422-446)."""

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        key_states = key_states.contiguous()
        value_states = value_states.contiguous()
        if self._seq_length == 0:
            self._rebuild_from_full(key_states, value_states)
            return key_states, value_states
        if key_states.shape[-2] == 1:
            self._append_decode_token(key_states, value_states)
            return key_states, value_states
        previous_keys, previous_values = self.materialize()
        self._append(key_states, value_states)
        return (torch.cat([previous_keys, key_states], dim=-2), torch.cat([previous_values, value_states], dim=-2))


    def packed_ready(self) -> bool:
        """Whether the next decode token can go through :meth:`append_and_attend` (packed storage
        holds the layer's history)."""
        return self.is_initialized and self.paged is not None and self._seq_length > 0

    def prepare_decode(self) -> bool:
        """Called before a one-token decode step: :meth:`packed_ready` (the deferred layer packs
        here the history that the coming token's ``update`` would pack)."""
        return self.packed_ready()

    def append_and_attend(self, query: torch.Tensor, key_states: torch.Tensor, value_states: torch.Tensor, *,
                          scaling: float, gate: torch.Tensor | None = None) -> torch.Tensor:
        """The decode step's cache update and attention in one launch: ``key_states`` /
        ``value_states`` ``[B, Hkv, 1, D]`` are quantised into the packed pool and ``query``
        ``[B, Hq, 1, D]`` attends over the cache with them, gated by ``gate`` ``[B, Hq, D]`` when
        given.  Returns ``[B, 1, Hq, D]`` in the query dtype.  Equivalent to ``update`` followed by
        the packed attention launcher (and the gate multiply), bit for bit."""
        if not self.packed_ready():
            raise RuntimeError("append_and_attend needs a packed qserve cache layer")
        if query.shape[-2] != 1 or key_states.shape[-2] != 1:
            raise RuntimeError("append_and_attend takes one decode token")
        q = query[:, :, 0, :]
        out = self.paged.append_attend(q, key_states[:, :, 0, :], value_states[:, :, 0, :], scaling,
                                       workspace=self.decode_workspace(q.shape[1]), gate=gate)
        self._seq_length += 1
        self.keys = None
        self.values = None
        return out.unsqueeze(1)


class QServeDeferredSplitFusedAttentionLayer(QServeFusedAttentionLayer):
    """Dense until ``activation_threshold`` tokens, then packed once (:473-547)."""

    def __init__(self, config: QServeKvConfig) -> None:
        super().__init__(config)
        self._deferred_prefill = False

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        key_states = key_states.contiguous()
        value_states = value_states.contiguous()
        if self._seq_length == 0:
            # prefill stays dense: quantisation is moved out of time-to-first-token
            self.dtype = key_states.dtype
            self.device = key_states.device
            self._seq_length = int(key_states.shape[-2])
            self.keys = key_states
            self.values = value_states
            self._deferred_prefill = True
            return key_states, value_states
        if self._deferred_prefill:
            if self.keys is None or self.values is None:
                raise RuntimeError("deferred qserve prefill cache is missing dense KV tensors.")
            dense_keys = torch.cat([self.keys, key_states], dim=-2).contiguous()
            dense_values = torch.cat([self.values, value_states], dim=-2).contiguous()
            self._seq_length = int(dense_keys.shape[-2])
            if self._seq_length < self.config.activation_threshold:
                self.keys = dense_keys
                self.values = dense_values
                return dense_keys, dense_values
            self._deferred_prefill = False
            self._seq_length = 0
            self._rebuild_from_full(dense_keys, dense_values)
            return key_states, value_states
        return super().update(key_states, value_states, *args, **kwargs)

    def adopt_prefill(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        """Adopt dense KV produced by the native prefill cache without repacking it."""
        self.lazy_initialization(key_states, value_states)
        self._seq_length = int(key_states.shape[-2])
        self.keys = key_states.contiguous()
        self.values = value_states.contiguous()
        self._deferred_prefill = True

    def materialize(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._deferred_prefill:
            if self.keys is None or self.values is None:
                raise RuntimeError("deferred qserve prefill cache is missing dense KV tensors.")
            return self.keys, self.values
        return super().materialize()

    def reset(self) -> None:
        super().reset()
        self._deferred_prefill = False

    def packed_ready(self) -> bool:
        return not self._deferred_prefill and super().packed_ready()

    def prepare_decode(self) -> bool:
        # ``update`` packs once the dense length with the new token reaches the threshold; packing
        # the history before that token gives the same pages (tokens are quantised one by one)
        if (self._deferred_prefill and self.keys is not None
                and self._seq_length + 1 >= self.config.activation_threshold):
            keys, values = self.keys, self.values
            self._deferred_prefill = False
            self._seq_length = 0
            self._rebuild_from_full(keys, values, extra_tokens=1)  # (sized as update sizes it, token included)
        return self.packed_ready()

    @property
    def _key_code(self):
        return None if self._deferred_prefill else super()._key_code


def _cache_base():
    if DynamicCache is None:
        raise ImportError("transformers is required for the QServe cache containers")
    return DynamicCache


class QServeKvCache(DynamicCache if DynamicCache is not None else object):
    """DynamicCache whose full-attention layers are paged INT4 layers (:380-419)."""

    layer_class = QServeAttentionLayer

    def __init__(self, model_config: Any, qserve_config: QServeKvConfig | None = None) -> None:
        _cache_base()
        self.qserve_config = qserve_config or QServeKvConfig()
        self.qserve_config.validate()
        super().__init__(config=model_config)
        decoder_config = (model_config.get_text_config(decoder=True)
                          if hasattr(model_config, "get_text_config") else model_config)
        self.layer_types = tuple(getattr(decoder_config, "layer_types", ()))
        self.full_attention_layers = tuple(
            idx for idx, layer_type in enumerate(self.layer_types) if layer_type == "full_attention")
        for layer_idx in self.full_attention_layers:
            self.layers[layer_idx] = self.layer_class(self.qserve_config)

    def report(self) -> QServeKvCacheReport:
        c = self.qserve_config
        return QServeKvCacheReport(
            enabled=True, full_attention_layers=self.full_attention_layers, k_bits=c.k_bits, v_bits=c.v_bits,
            group_size=c.group_size, residual_length=c.residual_length,
            activation_threshold=c.activation_threshold, decode_warmup_tokens=c.decode_warmup_tokens,
            attention_backend=c.attention_backend)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if (layer_idx == 0 and self.layer_types and self.layer_types[0] == "linear_attention"
                and self.full_attention_layers):
            layer_idx = self.full_attention_layers[0]
        return super().get_seq_length(layer_idx)

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.report()})"


class QServeFusedKvCache(QServeKvCache):
    """Full-attention decode reads the packed pool directly (:449-461)."""

    layer_class = QServeFusedAttentionLayer

    def __init__(self, model_config: Any, qserve_config: QServeKvConfig | None = None) -> None:
        super().__init__(model_config=model_config, qserve_config=qserve_config)
        self.attention_backend = self.qserve_config.attention_backend
        self.kernel_calls = 0
        self.fallback_calls = 0


class QServeSplitFusedKvCache(QServeFusedKvCache):
    """Selects the split-KV decode backend (:464-470)."""

    attention_backend = "triton_int4_split_decode"


class QServeDeferredSplitFusedKvCache(QServeSplitFusedKvCache):
    """Split decode cache that keeps prefill dense until the activation threshold (:550-594)."""

    attention_backend = "triton_int4_split_decode"
    defer_prefill_cache_injection = True
    layer_class = QServeDeferredSplitFusedAttentionLayer

    def adopt_native_prefill_cache(self, native_cache: Any) -> None:
        """Transfer native prefill state, replacing only full-attention cache layers."""
        native_layers = getattr(native_cache, "layers", None)
        if native_layers is None:
            raise TypeError("native prefill cache does not expose cache layers.")
        if len(native_layers) != len(self.layers):
            raise ValueError("native prefill cache depth does not match the Qwen3.5 cache.")
        for layer_idx, native_layer in enumerate(native_layers):
            if layer_idx not in self.full_attention_layers:
                self.layers[layer_idx] = native_layer
                continue
            key_states = getattr(native_layer, "keys", None)
            value_states = getattr(native_layer, "values", None)
            if key_states is None or value_states is None:
                raise RuntimeError(f"native full-attention layer {layer_idx} has no dense KV to adopt.")
            layer = self.layers[layer_idx]
            if not isinstance(layer, QServeDeferredSplitFusedAttentionLayer):
                raise TypeError("deferred split cache lost its full-attention layer type.")
            layer.adopt_prefill(key_states, value_states)
        for attribute in ("_seen_tokens", "_max_batch_size", "_max_cache_len"):
            if hasattr(native_cache, attribute):
                setattr(self, attribute, getattr(native_cache, attribute))

    def packed_decode_active(self) -> bool:
        """Whether every adapted full-attention layer has crossed the threshold."""
        return bool(self.full_attention_layers) and all(
            getattr(self.layers[i], "_key_code", None) is not None for i in self.full_attention_layers)


def build_qserve_deferred_split_fused_kv_cache(model_config: Any,
                                               qserve_config: QServeKvConfig | None = None
                                               ) -> QServeDeferredSplitFusedKvCache:
    return QServeDeferredSplitFusedKvCache(model_config=model_config, qserve_config=qserve_config)
