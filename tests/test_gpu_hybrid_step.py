"""One decode step of the hybrid stack (the graph bench.py times), against the oracle.

An 8-layer stack (6 GDN + 2 full-attention layers, 3:1 as in Qwen3.5) over three
ragged sequences: after one graph replay, every GDN layer's state and output and
every attention layer's output match the oracle run on the same inputs, and the new
token's codes in each attention cache are the reference quantiser's.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import kv_quant as kq
from tests._util import assert_attn_close, assert_gdn_close, oracle_attention

pytestmark = pytest.mark.gpu


def _gates(layer):
    """g and beta of a GDN layer of the stack: given, or (raw-gate layers) the oracle of the
    decode branch's gate arithmetic on the layer's a, b, A_log and dt_bias."""
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    if layer.g is not None:
        return f(layer.g), f(layer.beta)
    return ogdn.decay_gates(f(layer.a), f(layer.b), f(layer.A_log), f(layer.dt_bias), rnd=kq.round_bf16)


@pytest.mark.parametrize("gates,fused_append", [("given", True), ("fused", True), ("given", False)])
def test_graph_step_matches_oracle(gates, fused_append):
    """The captured step against the oracle: fused or separate append, given or computed gates
    (the fused append's attention launches start early after each GDN layer)."""
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape

    shape = HybridShape(batch=3, context=[70, 130, 5], num_layers=8)
    stack = HybridDecodeStack(shape, device="cuda", seed=3, gates=gates, fused_append=fused_append)
    stack.fill_inputs()
    states0 = [layer.state.cpu().numpy().copy() for layer in stack.gdn]
    graph = stack.capture()          # (the capture runs one eager step first)
    # restore the states the eager step advanced, then run the captured step once
    for layer, s0 in zip(stack.gdn, states0):
        layer.state.copy_(torch.from_numpy(s0))
    graph.replay()
    torch.cuda.synchronize()

    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    for layer, s0 in zip(stack.gdn, states0):
        ro, rs = ogdn.recurrent_gated_delta_rule(f(layer.q), f(layer.k), f(layer.v), *_gates(layer), s0,
                                                 True, True)
        assert_gdn_close(layer.state.cpu().numpy(), rs)
        got = f(layer.out)
        assert np.all(np.abs(got - ro) <= 2.0 ** -8 * np.abs(ro) + 1e-4 * np.abs(ro).max())

    for layer in stack.attn:
        p = layer.paged
        lens = layer.attend_lens.cpu().numpy()
        table = p.block_table.cpu().numpy()
        cache = kq.PagedKvOracle(p.pool.kv_codes.shape[0], shape.num_kv_heads, shape.head_dim, shape.page_size,
                                 table, lens)
        cache.kv_codes[...] = p.pool.kv_codes.cpu().numpy()
        cache.kv_meta[...] = p.pool.kv_meta.cpu().numpy()
        # the appended token (slot = context) holds the reference quantiser's codes of k / v
        kp, ks, km = kq.quantize_tokens_int4(f(layer.k))
        for b, pos in enumerate(shape.lengths):
            page, slot = table[b, pos // shape.page_size], pos % shape.page_size
            assert np.array_equal(cache.kv_codes[page, :, 0, slot], kp[b, :, 0])
            assert np.array_equal(cache.kv_meta[page, :, 0, slot], ks[b, :, 0])
            assert np.array_equal(cache.kv_meta[page, :, 1, slot], km[b, :, 0])
        ref, _ = oracle_attention(cache, f(layer.q), shape.head_dim ** -0.5)
        assert_attn_close(f(layer.out), ref)


@pytest.mark.parametrize("conv", ["separate", "fused"])
def test_graph_step_with_conv_matches_conv_then_recurrence(conv):
    """Same step with every GDN layer fed its raw projection output: the conv states and the
    GDN states / outputs match the oracle's conv update followed by its recurrence."""
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape

    shape = HybridShape(batch=2, context=[40, 90], num_layers=4)
    stack = HybridDecodeStack(shape, device="cuda", seed=5, conv=conv)
    stack.fill_inputs()
    states0 = [layer.state.cpu().numpy().copy() for layer in stack.gdn]
    conv0 = [layer.conv_state.float().cpu().numpy().copy() for layer in stack.gdn]
    graph = stack.capture()
    for layer, s0, c0 in zip(stack.gdn, states0, conv0):
        layer.state.copy_(torch.from_numpy(s0))
        layer.conv_state.copy_(torch.from_numpy(c0).to(layer.conv_state.dtype))
    graph.replay()
    torch.cuda.synchronize()

    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    h, d = shape.gdn_heads, shape.gdn_dim
    for layer, s0, c0 in zip(stack.gdn, states0, conv0):
        cst = c0.copy()
        conv = kq.round_bf16(ogdn.causal_conv1d_update(f(layer.qkv)[:, :, None], cst, f(layer.conv_w), f(layer.conv_b),
                                                       silu=True)[:, :, 0])
        b = conv.shape[0]
        q, k, v = (conv[:, i * h * d:(i + 1) * h * d].reshape(b, 1, h, d) for i in range(3))
        ro, rs = ogdn.recurrent_gated_delta_rule(q, k, v, *_gates(layer), s0, True, True)
        assert np.array_equal(f(layer.conv_state), cst)
        assert_gdn_close(layer.state.cpu().numpy(), rs)
        got = f(layer.out)
        assert np.all(np.abs(got - ro) <= 2.0 ** -8 * np.abs(ro) + 1e-4 * np.abs(ro).max())


@pytest.mark.parametrize("conv", [None, "fused"])
def test_graph_step_with_epilogues(conv):
    """The step with the output epilogues fused in: attention outputs are the oracle attention
    times sigmoid(gate), GDN outputs the oracle recurrence through Qwen3_5RMSNormGated(o, z)."""
    from oracle import epilogue as ep
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape

    shape = HybridShape(batch=2, context=[40, 131], num_layers=4)
    stack = HybridDecodeStack(shape, device="cuda", seed=9, conv=conv, epilogues=True)
    stack.fill_inputs()
    states0 = [layer.state.cpu().numpy().copy() for layer in stack.gdn]
    conv0 = [layer.conv_state.float().cpu().numpy().copy() for layer in stack.gdn] if conv else None
    graph = stack.capture()
    for j, (layer, s0) in enumerate(zip(stack.gdn, states0)):
        layer.state.copy_(torch.from_numpy(s0))
        if conv:
            layer.conv_state.copy_(torch.from_numpy(conv0[j]).to(layer.conv_state.dtype))
    graph.replay()
    torch.cuda.synchronize()

    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    h, d = shape.gdn_heads, shape.gdn_dim
    for j, (layer, s0) in enumerate(zip(stack.gdn, states0)):
        if conv:
            cst = conv0[j].copy()
            y = kq.round_bf16(ogdn.causal_conv1d_update(f(layer.qkv)[:, :, None], cst, f(layer.conv_w),
                                                        f(layer.conv_b), silu=True)[:, :, 0])
            b = y.shape[0]
            q, k, v = (y[:, i * h * d:(i + 1) * h * d].reshape(b, 1, h, d) for i in range(3))
        else:
            q, k, v = f(layer.q), f(layer.k), f(layer.v)
        ro, rs = ogdn.recurrent_gated_delta_rule(q, k, v, *_gates(layer), s0, True, True)
        assert_gdn_close(layer.state.cpu().numpy(), rs)
        ref = ep.rmsnorm_gated(kq.round_bf16(ro), f(layer.z), f(layer.norm_w), 1e-6, rnd=kq.round_bf16)
        got = f(layer.out)
        # o carries the recurrence's 1e-4-of-max error into the norm: bf16 rounding plus that, at output scale
        assert np.all(np.abs(got - ref) <= 3 * 2.0 ** -7 * np.abs(ref) + 2e-3 * np.abs(ref).max())

    for layer in stack.attn:
        p = layer.paged
        cache = kq.PagedKvOracle(p.pool.kv_codes.shape[0], shape.num_kv_heads, shape.head_dim, shape.page_size,
                                 p.block_table.cpu().numpy(), layer.attend_lens.cpu().numpy())
        cache.kv_codes[...] = p.pool.kv_codes.cpu().numpy()
        cache.kv_meta[...] = p.pool.kv_meta.cpu().numpy()
        ref, _ = oracle_attention(cache, f(layer.q), shape.head_dim ** -0.5)
        assert_attn_close(f(layer.out), ep.sigmoid_gate(ref, f(layer.gate), rnd=kq.round_bf16))


def test_host_facing_step_copies_overlap_and_match_the_device_graph():
    """`step()` (one graph: per-layer input copies from pinned host memory, the kernels, per-layer
    output copies back) gives the device-only graph's outputs and states bit for bit; the device
    input buffer and the host output buffer are cleared first, so only the step's own copies can
    produce the match."""
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape

    shape = HybridShape(batch=3, context=[70, 130, 5], num_layers=8)
    stack = HybridDecodeStack(shape, device="cuda", seed=5)
    stack.fill_inputs()
    states0 = [layer.state.clone() for layer in stack.gdn]
    graph = stack.capture()
    for layer, s0 in zip(stack.gdn, states0):
        layer.state.copy_(s0)
    graph.replay()
    torch.cuda.synchronize()
    want_out = stack.out_dev.clone()
    want_states = [layer.state.clone() for layer in stack.gdn]

    stack.io_graph = stack.capture_io()  # (runs one eager step first)
    for layer, s0 in zip(stack.gdn, states0):
        layer.state.copy_(s0)
    stack.in_dev.zero_()  # (g lives in the input buffer too)
    stack.out_host.zero_()
    torch.cuda.synchronize()
    got = stack.step()
    torch.cuda.synchronize()
    assert torch.equal(got.to("cuda"), want_out)
    for layer, s in zip(stack.gdn, want_states):
        assert torch.equal(layer.state, s)
