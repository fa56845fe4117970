"""The reference-facing API on the GPU: cache layers, attention launchers and GDN hooks.

Mirrors tests/test_qserve_kv_cache.py:175-195 of the reference (kernel vs SDPA over
the materialised cache) on the paged INT4 layer, plus the deferred-activation
flow, cache surgery (crop / select / repeat) and the GDN hooks.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import gdn as ogdn
from oracle import kv_quant as kq
from tests._util import assert_attn_close, assert_gdn_close

pytestmark = pytest.mark.gpu


def _sdpa_over_cache(query, layer, hq, hkv):
    keys, values = layer.materialize()
    return F.scaled_dot_product_attention(query.float(), keys.float().repeat_interleave(hq // hkv, dim=1),
                                          values.float().repeat_interleave(hq // hkv, dim=1)).transpose(1, 2)


def _oracle_over_layer(query, layer):
    """fp32 attention over the fp32-dequantised pool (stored fp16 scale/min)."""
    from oracle.attention import decode_attention

    codes = layer.paged.pool.kv_codes.cpu().numpy()
    meta = layer.paged.pool.kv_meta.cpu().numpy()
    table = layer.paged.block_table.cpu().numpy()
    lens = layer.paged.seq_lens.cpu().numpy()
    cache = kq.PagedKvOracle.__new__(kq.PagedKvOracle)
    cache.kv_codes, cache.kv_meta, cache.block_table, cache.seq_lens = codes, meta, table, lens.astype(np.int64)
    cache.bits = layer.paged.pool.bits
    cache.page_size, cache.head_dim = 64, codes.shape[-1] * 8 // cache.bits
    keys, values = zip(*(cache.gather(b) for b in range(len(lens))))
    out, _ = decode_attention(query.float().cpu().numpy()[:, :, 0], keys, values, 256 ** -0.5)
    return out


@pytest.mark.parametrize("launcher", ["qserve_int4_split_decode_attention", "qserve_int4_decode_attention"])
def test_layer_kernel_matches_sdpa_over_the_same_quantized_kv(launcher):
    import optiz_qwen_b200.kernels as K
    from optiz_qwen_b200.compression import QServeAttentionLayer, QServeKvConfig

    torch.manual_seed(31)
    layer = QServeAttentionLayer(QServeKvConfig())
    keys = torch.randn(1, 2, 300, 256, device="cuda", dtype=torch.bfloat16)
    values = torch.randn_like(keys)
    query = torch.randn(1, 8, 1, 256, device="cuda", dtype=torch.bfloat16)
    layer.update(keys, values)
    actual = getattr(K, launcher)(query, layer, scaling=1 / (256 ** 0.5))
    assert actual.shape == (1, 1, 8, 256) and actual.dtype == torch.bfloat16
    # the reference test's own oracle: SDPA over materialize() (model dtype)
    expected = _sdpa_over_cache(query, layer, 8, 2)
    torch.testing.assert_close(actual.float(), expected, rtol=1e-2, atol=2e-2)
    # the contract's oracle: fp32 attention over the fp32-dequantised cache
    assert_attn_close(actual[:, 0].float().cpu().numpy(), _oracle_over_layer(query, layer))


def test_deferred_cache_flow_through_threshold_and_decode():
    from optiz_qwen_b200.compression import QServeDeferredSplitFusedAttentionLayer, QServeKvConfig
    from optiz_qwen_b200.kernels import qserve_int4_split_decode_attention

    torch.manual_seed(5)
    cfg = QServeKvConfig(activation_threshold=512, residual_length=256)
    layer = QServeDeferredSplitFusedAttentionLayer(cfg)
    dense_k = torch.randn(2, 2, 500, 256, device="cuda", dtype=torch.bfloat16)
    dense_v = torch.randn_like(dense_k)
    layer.update(dense_k, dense_v)
    assert layer._key_code is None
    for step in range(20):
        k = torch.randn(2, 2, 1, 256, device="cuda", dtype=torch.bfloat16)
        v = torch.randn_like(k)
        layer.update(k, v)
        dense_k = torch.cat([dense_k, k], dim=-2)
        dense_v = torch.cat([dense_v, v], dim=-2)
        if layer._key_code is not None:
            q = torch.randn(2, 8, 1, 256, device="cuda", dtype=torch.bfloat16)
            out = qserve_int4_split_decode_attention(q, layer, scaling=1 / 16)
            assert_attn_close(out[:, 0].float().cpu().numpy(), _oracle_over_layer(q, layer))
    assert layer._key_code is not None and layer.get_seq_length() == 520
    # the packed cache holds the reference quantiser's codes for every token
    keys, _ = layer.materialize()
    ref = kq.dequantize_tokens_int4(*kq.quantize_tokens_int4(dense_k.float().cpu().numpy()))
    np.testing.assert_allclose(keys.float().cpu().numpy(), ref, rtol=8e-3, atol=8e-3)


def test_cache_surgery_crop_select_repeat():
    from optiz_qwen_b200.compression import QServeAttentionLayer, QServeKvConfig

    torch.manual_seed(7)
    layer = QServeAttentionLayer(QServeKvConfig(page_seed=4))
    keys = torch.randn(3, 2, 150, 256, device="cuda", dtype=torch.bfloat16)
    layer.update(keys, keys.clone())
    full_k, _ = layer.materialize()
    layer.batch_select_indices(torch.tensor([2, 0, 2]))
    sel_k, _ = layer.materialize()
    assert torch.equal(sel_k, full_k[[2, 0, 2]])
    layer.batch_repeat_interleave(2)
    rep_k, _ = layer.materialize()
    assert torch.equal(rep_k, full_k[[2, 2, 0, 0, 2, 2]])
    layer.crop(100)
    crop_k, _ = layer.materialize()
    assert layer.get_seq_length() == 100 and torch.equal(crop_k, full_k[[2, 2, 0, 0, 2, 2], :, :100])
    # appending after surgery writes each row's own pages
    k = torch.randn(6, 2, 1, 256, device="cuda", dtype=torch.bfloat16)
    layer.update(k, k)
    after, _ = layer.materialize()
    assert torch.equal(after[:, :, :100], crop_k)


def test_gdn_hooks_match_the_oracle():
    from optiz_qwen_b200.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule

    rng = np.random.default_rng(3)
    b, t, h, d = 2, 70, 4, 128
    q, k, v = (kq.round_bf16(rng.standard_normal((b, t, h, d), dtype=np.float32)) for _ in range(3))
    g = (-np.logaddexp(0, rng.standard_normal((b, t, h)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, h))))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d))).astype(np.float32)
    tt = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    ref_o, ref_s = ogdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    o, s = chunk_gated_delta_rule(tt(q), tt(k), tt(v), tt(g), tt(beta), initial_state=tt(s0),
                                  output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert_gdn_close(o.cpu().numpy(), ref_o)
    assert_gdn_close(s.cpu().numpy(), ref_s)
    # decode continuation through the recurrent hook, state carried over
    q1, k1, v1 = (kq.round_bf16(rng.standard_normal((b, 1, h, d), dtype=np.float32)) for _ in range(3))
    g1 = (-np.logaddexp(0, rng.standard_normal((b, 1, h)))).astype(np.float32)
    b1 = (1 / (1 + np.exp(-rng.standard_normal((b, 1, h))))).astype(np.float32)
    ro, rs = ogdn.recurrent_gated_delta_rule(q1, k1, v1, g1, b1, ref_s, True, True)
    o1, s1 = fused_recurrent_gated_delta_rule(tt(q1), tt(k1), tt(v1), g=tt(g1), beta=tt(b1), initial_state=s,
                                              output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert_gdn_close(o1.cpu().numpy(), ro)
    assert_gdn_close(s1.cpu().numpy(), rs)
    o2, s2 = fused_recurrent_gated_delta_rule(tt(q1), tt(k1), tt(v1), g=tt(g1), beta=tt(b1), initial_state=s,
                                              output_final_state=False, use_qk_l2norm_in_kernel=True)
    assert s2 is None and torch.equal(o2, o1)


def test_attention_launch_is_graph_capturable():
    """The decode step (append + attention) replays from a CUDA graph with fixed addresses."""
    from optiz_qwen_b200.compression import QServeFusedAttentionLayer, QServeKvConfig
    from optiz_qwen_b200.kernels import qserve_int4_split_decode_attention

    torch.manual_seed(9)
    layer = QServeFusedAttentionLayer(QServeKvConfig())
    keys = torch.randn(4, 2, 200, 256, device="cuda", dtype=torch.bfloat16)
    layer.update(keys, keys.clone())
    layer.paged.reserve([260] * 4)          # pages for the captured steps
    k_new = torch.randn(4, 2, 1, 256, device="cuda", dtype=torch.bfloat16)
    q = torch.randn(4, 8, 1, 256, device="cuda", dtype=torch.bfloat16)
    from optiz_qwen_b200 import cabi

    paged = layer.paged
    ws = layer.decode_workspace(8)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        cabi.append_quant_int4(k_new, k_new, paged.pool, paged.block_table, paged.seq_lens)
        out = cabi.decode_attention_int4(q[:, :, 0], paged.pool, paged.block_table, paged.seq_lens, 1 / 16,
                                         workspace=ws)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cabi.append_quant_int4(k_new, k_new, paged.pool, paged.block_table, paged.seq_lens)
        out = cabi.decode_attention_int4(q[:, :, 0], paged.pool, paged.block_table, paged.seq_lens, 1 / 16,
                                         workspace=ws)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert paged.seq_lens.tolist() == [204] * 4
    paged.host_lens = [204] * 4
    layer._seq_length = 204
    assert_attn_close(out.float().cpu().numpy(), _oracle_over_layer(q, layer))
