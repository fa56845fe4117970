"""Host-side behaviour of the drop-in API (mirrors the reference's tests/test_qserve_kv_cache.py:32-172).

Everything here runs on CPU: config validation, the cache builder, dense-phase
behaviour of the deferred layer, the page allocator policy, and loud failure of the
kernels on CPU tensors.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from optiz_qwen_b200.compression import (
    PageAllocator,
    QServeDeferredSplitFusedAttentionLayer,
    QServeDeferredSplitFusedKvCache,
    QServeKvConfig,
    build_qserve_deferred_split_fused_kv_cache,
)


class MinimalQwenConfig:
    layer_types = ("linear_attention", "full_attention", "linear_attention")
    num_hidden_layers = 3

    def get_text_config(self, decoder: bool = True):
        return self


CFG16 = QServeKvConfig(k_bits=4, v_bits=4, group_size=16, residual_length=16, activation_threshold=32)


def test_deferred_split_cache_preserves_prefill_dense_until_decode():
    layer = QServeDeferredSplitFusedAttentionLayer(CFG16)
    prefill_keys = torch.randn(1, 2, 16, 16)
    prefill_values = torch.randn_like(prefill_keys)
    layer.update(prefill_keys, prefill_values)
    assert layer._deferred_prefill is True
    assert layer._key_code is None
    assert torch.equal(layer.materialize()[0], prefill_keys)
    decode_key = torch.randn(1, 2, 1, 16)
    layer.update(decode_key, torch.randn_like(decode_key))
    assert layer._deferred_prefill is True
    assert layer._key_code is None
    assert torch.equal(layer.materialize()[0], torch.cat([prefill_keys, decode_key], dim=-2))
    assert layer.get_seq_length() == 17


def test_deferred_split_layer_can_adopt_native_prefill_tensors():
    layer = QServeDeferredSplitFusedAttentionLayer(CFG16)
    prefill_keys = torch.randn(1, 2, 16, 16)
    prefill_values = torch.randn_like(prefill_keys)
    layer.adopt_prefill(prefill_keys, prefill_values)
    assert layer._deferred_prefill is True
    assert layer.get_seq_length() == 16
    assert torch.equal(layer.materialize()[1], prefill_values)


def test_packing_cpu_tensors_fails_loudly():
    """Crossing the activation threshold on CPU tensors must not silently fall back."""
    layer = QServeDeferredSplitFusedAttentionLayer(CFG16)
    layer.update(torch.randn(1, 2, 31, 16), torch.randn(1, 2, 31, 16))
    with pytest.raises((RuntimeError, ValueError)):
        layer.update(torch.randn(1, 2, 1, 16), torch.randn(1, 2, 1, 16))


def test_deferred_split_cache_builder_places_packed_layers_on_full_attention():
    """What the reference's chain builder (scheduling/kv_chain.py) receives from the cache builder."""
    cache = build_qserve_deferred_split_fused_kv_cache(MinimalQwenConfig(), CFG16)
    assert isinstance(cache, QServeDeferredSplitFusedKvCache)
    assert cache.full_attention_layers == (1,)
    assert isinstance(cache.layers[1], QServeDeferredSplitFusedAttentionLayer)
    assert cache.kernel_calls == 0 and cache.fallback_calls == 0
    assert cache.packed_decode_active() is False


def test_qserve_config_rejects_unknown_attention_backend():
    with pytest.raises(ValueError, match="attention_backend"):
        QServeKvConfig(attention_backend="unknown").validate()


def test_qserve_config_requires_int8_backend_for_8bit_kv():
    with pytest.raises(ValueError, match="requires triton_int8_decode"):
        QServeKvConfig(k_bits=8, v_bits=8).validate()


@pytest.mark.parametrize("kwargs", [dict(group_size=0), dict(residual_length=0), dict(residual_length=100),
                                    dict(activation_threshold=8), dict(decode_warmup_tokens=-1),
                                    dict(k_bits=3, v_bits=3), dict(k_bits=4, v_bits=8), dict(page_size=32)])
def test_qserve_config_validation(kwargs):
    with pytest.raises(ValueError):
        QServeKvConfig(**kwargs).validate()


def test_8bit_layers_build_an_8bit_pool_and_dispatch_to_the_8bit_entry_points():
    from optiz_qwen_b200 import cabi

    cfg = QServeKvConfig(k_bits=8, v_bits=8, attention_backend="triton_int8_decode")
    cfg.validate()
    layer = QServeDeferredSplitFusedAttentionLayer(cfg)
    assert layer.config.k_bits == 8
    pool8 = cabi.PagedKvPool(2, 2, 256, 64, "cpu", bits=8)
    pool4 = cabi.PagedKvPool(2, 2, 256, 64, "cpu")
    assert tuple(pool8.kv_codes.shape) == (2, 2, 2, 64, 256)
    assert tuple(pool4.kv_codes.shape) == (2, 2, 2, 64, 128)
    assert cabi._bits_entry("decode_attn", pool8, None) == "oq_decode_attn_int8"
    assert cabi._bits_entry("append_quant", pool4, 4) == "oq_append_quant_int4"
    with pytest.raises(ValueError, match="8-bit codes"):
        cabi._bits_entry("gather_dequant", pool8, 4)
    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        cabi.PagedKvPool(2, 2, 256, 64, "cpu", bits=2)


def test_builder_and_report():
    cache = build_qserve_deferred_split_fused_kv_cache(MinimalQwenConfig(), CFG16)
    rep = cache.report()
    assert rep.group_size == 16 and rep.attention_backend == "triton_int4_split_decode"
    assert "QServeDeferredSplitFusedKvCache" in repr(cache)


def test_page_allocator_policy_matches_the_oracle():
    from oracle import kv_quant as kq

    alloc = PageAllocator(37, seed=3)
    got = alloc.allocate(37)
    assert got == kq.page_permutation(37, 3).tolist()
    alloc.free(got[:5])
    assert alloc.num_free == 5
    alloc.grow(40)
    assert alloc.allocate(8) == got[:5] + [37, 38, 39]
    with pytest.raises(MemoryError):
        alloc.allocate(1)


def test_block_table_policy_matches_the_oracle_allocator():
    from oracle import kv_quant as kq

    lengths = [130, 1, 64, 65]
    alloc = PageAllocator(20, seed=11)
    rows = [alloc.allocate(-(-n // 64)) for n in lengths]
    table = kq.build_block_table(lengths, 64, 20, 3, seed=11)
    for b, row in enumerate(rows):
        assert row == table[b, : len(row)].tolist()


def test_kernels_refuse_cpu_tensors():
    from optiz_qwen_b200 import cabi

    pool = cabi.PagedKvPool.__new__(cabi.PagedKvPool)
    with pytest.raises(RuntimeError, match="CUDA"):
        cabi.decode_attention_int4(torch.zeros(1, 8, 256, dtype=torch.bfloat16), pool,
                                   torch.zeros(1, 1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32), 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        cabi.gdn_recurrent(*(torch.zeros(1, 1, 1, 128) for _ in range(3)), torch.zeros(1, 1, 1),
                           torch.zeros(1, 1, 1))


def test_gdn_hooks_refuse_cpu_and_unsupported_options():
    from optiz_qwen_b200.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule

    q = torch.zeros(1, 2, 1, 128)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_recurrent_gated_delta_rule(q, q, q, g=torch.zeros(1, 2, 1), beta=torch.ones(1, 2, 1))
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(q, q, q, torch.zeros(1, 2, 1), torch.ones(1, 2, 1), cu_seqlens=torch.tensor([0, 2]))
    with pytest.raises(NotImplementedError):
        fused_recurrent_gated_delta_rule(q, q, q, g=torch.zeros(1, 2, 1), beta=torch.ones(1, 2, 1),
                                         use_gate_in_kernel=True)


def test_attention_launchers_error_behaviour():
    from optiz_qwen_b200.kernels import qserve_int4_split_decode_attention

    layer = QServeDeferredSplitFusedAttentionLayer(CFG16)
    with pytest.raises(RuntimeError, match="CUDA query"):
        qserve_int4_split_decode_attention(torch.zeros(1, 8, 1, 256), layer, scaling=1.0)


def test_install_gdn_fastpath_binds_hooks():
    from optiz_qwen_b200.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule, install_gdn_fastpath
    from optiz_qwen_b200.gdn.gated_delta_rule import causal_conv1d_update

    class Qwen3_5GatedDeltaNet(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.recurrent_gated_delta_rule = None
            self.chunk_gated_delta_rule = None
            self.causal_conv1d_update = None

    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNormGated

    model = torch.nn.Sequential(Qwen3_5GatedDeltaNet(), torch.nn.Linear(2, 2), Qwen3_5GatedDeltaNet())
    model[2].norm = Qwen3_5RMSNormGated(8)
    assert install_gdn_fastpath(model) == 2
    assert model[0].recurrent_gated_delta_rule is fused_recurrent_gated_delta_rule
    assert model[2].chunk_gated_delta_rule is chunk_gated_delta_rule
    assert model[2].causal_conv1d_update is causal_conv1d_update
    # the output norm now runs the kernel: on CPU tensors it refuses loudly
    with pytest.raises(RuntimeError, match="CUDA"):
        model[2].norm(torch.zeros(2, 8), torch.zeros(2, 8))


def test_conv_hook_rejects_unsupported_arguments():
    from optiz_qwen_b200.gdn.gated_delta_rule import causal_conv1d_update

    x, st, w = torch.zeros(1, 4, 1), torch.zeros(1, 4, 4), torch.zeros(4, 4)
    with pytest.raises(NotImplementedError):
        causal_conv1d_update(x, st, w, None, "gelu")
    with pytest.raises(NotImplementedError):
        causal_conv1d_update(x, st, w, None, "silu", cache_seqlens=torch.zeros(1))
    with pytest.raises(RuntimeError, match="CUDA"):
        causal_conv1d_update(x, st, w, None, "silu")


def test_workspace_split_heuristic_matches_the_c_side():
    from optiz_qwen_b200 import cabi

    assert cabi.choose_splits(64, 2, 66) == 1          # 128 units already fill the 148 SMs
    assert cabi.choose_splits(1, 2, 2048) == 64        # one long sequence: 64 ranges of 32 pages
    assert cabi.choose_splits(1, 2, 256) == 64         # ... of 4 pages (the floor)
    assert cabi.choose_splits(1024, 2, 128) == 1
