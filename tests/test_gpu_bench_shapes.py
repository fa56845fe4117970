"""Parity at the shapes the benchmarks run, and at adversarial attention inputs.

* Hybrid decode step, B = 64 at context 4096 (4097 attended): the real ``HybridDecodeStack``
  the bench times, one step through the product path; every attention layer and two GDN
  layers are compared with the oracle on a sample of sequences (all heads).
* One long-context layer, B = 1 at context 131072: 2048 pages over 74 KV ranges, so the
  separate split-merge kernel runs.
* One ragged serving shard: the sequences rank 0 of 8 gets from ``serving.shard_by_cost``
  for 1024 contexts drawn from U[256, 8192] (seed 3), with permuted pages.
* Adversarial: q scaled x8 (a peaky softmax), and values with a large |min| and wide range,
  at 4097 and 131072 tokens.

Each attention check prints the share of the tolerance it used (``attn_margin``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import kv_quant as kq
from tests._util import (assert_attn_close, assert_gdn_close, oracle_attention, oracle_from_device,
                         random_paged_cache, upload_pool)

pytestmark = pytest.mark.gpu


def _gates(layer):
    """g and beta of a GDN layer of the stack: given, or (raw-gate layers) the oracle of the
    decode branch's gate arithmetic on the layer's a, b, A_log and dt_bias."""
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    if layer.g is not None:
        return f(layer.g), f(layer.beta)
    return ogdn.decay_gates(f(layer.a), f(layer.b), f(layer.A_log), f(layer.dt_bias), rnd=kq.round_bf16)


SCALING = 256 ** -0.5


def _report(name, margin):
    print(f"[attention margin] {name}: {margin:.3f} of the tolerance")


def test_hybrid_step_b64_ctx4096_sampled():
    from optiz_qwen_b200.hybrid import HybridDecodeStack, HybridShape

    shape = HybridShape(batch=64, context=4096)
    stack = HybridDecodeStack(shape, device="cuda", seed=1, page_seed=1)
    stack.fill_inputs()
    rows = [0, 17, 42, 63]
    gdn_layers = [0, len(stack.gdn) - 1]
    states0 = {i: stack.gdn[i].state[rows].cpu().numpy().copy() for i in gdn_layers}
    stack.step_device()
    torch.cuda.synchronize()

    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    worst = 0.0
    for layer in stack.attn:
        p = layer.paged
        cache = oracle_from_device(p.pool, p.block_table, layer.attend_lens, rows)
        assert list(cache.seq_lens) == [4097] * len(rows)
        ref, _ = oracle_attention(cache, f(layer.q)[rows], SCALING)
        worst = max(worst, assert_attn_close(f(layer.out)[rows], ref))
    _report("hybrid B=64 ctx 4097, 6 layers x 4 sequences", worst)
    for i in gdn_layers:
        layer = stack.gdn[i]
        ro, rs = ogdn.recurrent_gated_delta_rule(f(layer.q)[rows], f(layer.k)[rows], f(layer.v)[rows],
                                                 *(x[rows] for x in _gates(layer)), states0[i], True, True)
        assert_gdn_close(layer.state[rows].cpu().numpy(), rs)
        got = f(layer.out)[rows]
        assert np.all(np.abs(got - ro) <= 2.0 ** -8 * np.abs(ro) + 1e-4 * np.abs(ro).max())


def _long_context(rng, q_mult=1.0, **meta):
    from optiz_qwen_b200 import cabi

    cache = random_paged_cache(rng, [131072], 2, 256, 64, seed_pages=2, **meta)
    pool, table, lens = upload_pool(cache)
    q = kq.round_bf16(q_mult * rng.standard_normal((1, 8, 256), dtype=np.float32))
    out_f32 = torch.empty((1, 8, 256), dtype=torch.float32, device="cuda")
    out = cabi.decode_attention_int4(torch.from_numpy(q).cuda().to(torch.bfloat16), pool, table, lens, SCALING,
                                     out_f32=out_f32)
    torch.cuda.synchronize()
    ref, _ = oracle_attention(cache, q, SCALING)
    return out.float().cpu().numpy(), out_f32.cpu().numpy(), ref


def test_long_context_layer_ctx131072():
    out, out_f32, ref = _long_context(np.random.default_rng(2))
    _report("long context 131072 (fp32 output)", assert_attn_close(out_f32, ref))
    assert_attn_close(out, ref)


def test_serving_shard_ragged():
    from bench import serving_lengths
    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.serving import shard_by_cost

    lengths = serving_lengths()
    mine = [lengths[i] for i in shard_by_cost(lengths, 8)[0]]
    rng = np.random.default_rng(3)
    cache = random_paged_cache(rng, mine, 2, 256, 64, seed_pages=3)
    pool, table, lens = upload_pool(cache)
    q = kq.round_bf16(rng.standard_normal((len(mine), 8, 256), dtype=np.float32))
    out = cabi.decode_attention_int4(torch.from_numpy(q).cuda().to(torch.bfloat16), pool, table, lens, SCALING)
    torch.cuda.synchronize()
    order = np.argsort(mine)
    rows = sorted({int(order[0]), int(order[-1]), *map(int, rng.choice(len(mine), 6, replace=False))})
    sub = oracle_from_device(pool, table, lens, rows)
    ref, _ = oracle_attention(sub, q[rows], SCALING)
    _report(f"serving shard ({len(mine)} ragged sequences, 8 sampled)",
            assert_attn_close(out.float().cpu().numpy()[rows], ref))


def test_adversarial_peaky_softmax_ctx4097():
    """q x 8 over N(0,1) keys: scores of standard deviation ~8, a few tokens dominate."""
    from optiz_qwen_b200 import cabi

    rng = np.random.default_rng(5)
    cache = kq.fill_paged_cache(rng, [4097] * 4, 2, 256, 64, seed_pages=5)
    pool, table, lens = upload_pool(cache)
    q = kq.round_bf16(8.0 * rng.standard_normal((4, 8, 256), dtype=np.float32))
    out_f32 = torch.empty((4, 8, 256), dtype=torch.float32, device="cuda")
    cabi.decode_attention_int4(torch.from_numpy(q).cuda().to(torch.bfloat16), pool, table, lens, SCALING,
                               out_f32=out_f32, want_out=False)
    torch.cuda.synchronize()
    ref, _ = oracle_attention(cache, q, SCALING)
    _report("peaky softmax (q x 8), ctx 4097", assert_attn_close(out_f32.cpu().numpy(), ref))


def test_adversarial_wide_values_ctx131072():
    """q x 8 and values with |min| in [15, 30] and a range of 22-45 (scale 1.5-3 per code)."""
    out, out_f32, ref = _long_context(np.random.default_rng(6), q_mult=8.0, v_scale=(1.5, 3.0),
                                      v_min=(-30.0, -15.0))
    _report("peaky softmax + wide values, ctx 131072 (fp32 output)", assert_attn_close(out_f32, ref))
    assert_attn_close(out, ref)


def test_gdn_step_serving_shard_batch():
    """The GDN step at a serving shard's batch (128 sequences x 16 heads)."""
    from optiz_qwen_b200 import cabi

    rng = np.random.default_rng(7)
    b, h, d = 128, 16, 128
    q, k, v = (kq.round_bf16(rng.standard_normal((b, 1, h, d), dtype=np.float32)) for _ in range(3))
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, 1, h))))).astype(np.float32)
    g = (-np.logaddexp(0, rng.standard_normal((b, 1, h)))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d))).astype(np.float32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    s = t(s0)
    out = cabi.gdn_recurrent(t(q).to(torch.bfloat16), t(k).to(torch.bfloat16), t(v).to(torch.bfloat16), t(g),
                             t(beta), initial_state=s, final_state=s, use_qk_l2norm=True)
    torch.cuda.synchronize()
    ro, rs = ogdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)
    assert_gdn_close(s.cpu().numpy(), rs)
    got = out.float().cpu().numpy()
    assert np.all(np.abs(got - ro) <= 2.0 ** -8 * np.abs(ro) + 1e-4 * np.abs(ro).max())
