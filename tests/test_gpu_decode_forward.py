"""The one-launch decode forward of Qwen3.5's attention modules (``install_paged_decode_forward``).

A small random Qwen3.5 text config (hidden 512, 8 query / 2 KV heads of 256, layer 3 full
attention) and transformers' own ``Qwen3_5Attention`` module.  Against the unfused path over a
second copy of the same cache -- the cache layer's ``update``, the package's attention launcher,
the module's own ``attn * sigmoid(gate)`` and ``o_proj`` -- the decode forward must leave the
same cache bytes and give the same output bits; its attention must match the fp32 oracle over
the dequantised cache; and every other call (prefill, a deferred dense layer) must run the
module's own forward.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests._util import assert_attn_close

pytestmark = pytest.mark.gpu


def _setup(batch=3, prefix=300, seed=0, deferred=False, threshold=1024):
    import transformers.models.qwen3_5.configuration_qwen3_5 as c
    import transformers.models.qwen3_5.modeling_qwen3_5 as m

    from optiz_qwen_b200.compression import QServeKvConfig
    from optiz_qwen_b200.compression.qserve_kv_cache import QServeDeferredSplitFusedKvCache, QServeFusedKvCache

    torch.manual_seed(seed)
    cfg = c.Qwen3_5TextConfig(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=256,
                              num_hidden_layers=4, intermediate_size=1024, vocab_size=1000)
    attn = m.Qwen3_5Attention(cfg, 3).cuda().to(torch.bfloat16).eval()
    with torch.no_grad():
        for p in attn.parameters():
            p.normal_(0.0, 0.05)
    rotary = m.Qwen3_5TextRotaryEmbedding(cfg).cuda()
    qcfg = QServeKvConfig(activation_threshold=threshold)
    caches = []
    for _ in range(2):
        cache = (QServeDeferredSplitFusedKvCache if deferred else QServeFusedKvCache)(cfg, qcfg)
        caches.append(cache)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    k = torch.randn((batch, 2, prefix, 256), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((batch, 2, prefix, 256), generator=g, device="cuda").to(torch.bfloat16)
    for cache in caches:
        cache.layers[3].update(k, v)
    return attn, rotary, caches, g


def _step_inputs(rotary, g, batch, pos):
    h = (torch.randn((batch, 1, 512), generator=g, device="cuda") * 2.0).to(torch.bfloat16)
    ids = torch.full((batch, 1), pos, dtype=torch.long, device="cuda")
    return h, rotary(h, ids)


def _unfused(attn, hidden, pe, cache):
    """transformers' projections around the cache update and the package's launcher: the
    output with the gate fused into the launcher (as the reference adapter passes it), the
    output with transformers' own ``attn * sigmoid(gate)``, and the query."""
    import sys

    from optiz_qwen_b200.kernels import qserve_int4_split_decode_attention

    bsz, d = hidden.shape[0], attn.head_dim
    q, gate = torch.chunk(attn.q_proj(hidden).view(bsz, 1, -1, 2 * d), 2, dim=-1)
    gate = gate.reshape(bsz, 1, -1)
    q = attn.q_norm(q).transpose(1, 2)
    k = attn.k_norm(attn.k_proj(hidden).view(bsz, 1, -1, d)).transpose(1, 2)
    v = attn.v_proj(hidden).view(bsz, 1, -1, d).transpose(1, 2)
    q, k = sys.modules[type(attn).__module__].apply_rotary_pos_emb(q, k, *pe)
    cache.layers[3].update(k, v)
    fused_gate = qserve_int4_split_decode_attention(q, cache.layers[3], scaling=attn.scaling, gate=gate)
    o = qserve_int4_split_decode_attention(q, cache.layers[3], scaling=attn.scaling)
    torch_gate = o.reshape(bsz, 1, -1) * torch.sigmoid(gate)
    return attn.o_proj(fused_gate.reshape(bsz, 1, -1)), attn.o_proj(torch_gate), q


@torch.no_grad()
def test_decode_forward_matches_unfused_path_and_oracle():
    from optiz_qwen_b200 import cabi
    from optiz_qwen_b200.kernels import install_paged_decode_forward
    from oracle.attention import decode_attention

    batch, prefix = 3, 300
    attn, rotary, (fused_cache, plain_cache), g = _setup(batch, prefix)
    assert install_paged_decode_forward(attn) == 1
    for step in range(70):             # crosses a page edge (300 + 70 > 320)
        hidden, pe = _step_inputs(rotary, g, batch, prefix + step)
        out, weights = attn(hidden, pe, None, past_key_values=fused_cache)
        ref, ref_torch_gate, q = _unfused(attn, hidden, pe, plain_cache)
        assert weights is None and out.shape == ref.shape
        assert torch.equal(out, ref), f"step {step}"
        torch.testing.assert_close(out.float(), ref_torch_gate.float(), rtol=2e-2, atol=2e-2)
    lf, lp = fused_cache.layers[3], plain_cache.layers[3]
    assert lf.get_seq_length() == lp.get_seq_length() == prefix + 70
    assert torch.equal(lf.paged.seq_lens, lp.paged.seq_lens)
    assert torch.equal(lf.paged.pool.kv_codes, lp.paged.pool.kv_codes)
    assert torch.equal(lf.paged.pool.kv_meta.view(torch.int16), lp.paged.pool.kv_meta.view(torch.int16))
    # the last step's attention (before the gate and o_proj) against the fp32 oracle
    n = prefix + 70
    keys, values = cabi.gather_dequant(lf.paged.pool, lf.paged.block_table, lf.paged.seq_lens, n, torch.float32)
    qn = q[:, :, 0, :].float().cpu().numpy()
    expected, _ = decode_attention(qn, [keys[b].cpu().numpy() for b in range(batch)],
                                   [values[b].cpu().numpy() for b in range(batch)], attn.scaling)
    got = cabi.decode_attention_int4(q[:, :, 0, :], lf.paged.pool, lf.paged.block_table, lf.paged.seq_lens,
                                     attn.scaling).float().cpu().numpy()
    assert_attn_close(got, expected)


@torch.no_grad()
def test_other_calls_run_the_module_forward_and_the_deferred_layer_switches():
    """Prefill-shaped calls take the module's own forward (identical output).  A deferred layer
    decodes through the module's forward while it is dense, and through one launch from the
    step that crosses its threshold on: against a twin cache driven by the module's forward
    (dense steps) and by update + launcher (packed steps), outputs and cache bytes identical."""
    from transformers import DynamicCache

    from optiz_qwen_b200.kernels import install_paged_decode_forward

    batch, prefix, threshold = 2, 240, 256
    attn, rotary, (cache, twin), g = _setup(batch, prefix=prefix, deferred=True, threshold=threshold)
    hidden = (torch.randn((batch, 5, 512), generator=g, device="cuda")).to(torch.bfloat16)
    ids = torch.arange(5, device="cuda").expand(batch, 5)
    pe = rotary(hidden, ids)
    ref, _ = attn(hidden, pe, None, past_key_values=DynamicCache())
    install_paged_decode_forward(attn)
    out, _ = attn(hidden, pe, None, past_key_values=DynamicCache())
    assert torch.equal(out, ref)
    layer = cache.layers[3]
    assert not layer.packed_ready()                  # dense (deferred) below the threshold
    for step in range(30):                           # 240 + 30 crosses the threshold of 256
        h1, pe1 = _step_inputs(rotary, g, batch, prefix + step)
        o, _ = attn(h1, pe1, None, past_key_values=cache)
        if prefix + step + 1 < threshold:
            r, _ = attn._oq_module_forward(h1, pe1, None, past_key_values=twin)
        else:
            r, _, _ = _unfused(attn, h1, pe1, twin)
        assert torch.equal(o, r), f"step {step}"
    lt = twin.layers[3]
    assert layer.packed_ready() and layer.get_seq_length() == lt.get_seq_length() == prefix + 30
    assert np.array_equal(layer.paged.seq_lens.cpu().numpy(), [prefix + 30] * batch)
    assert torch.equal(layer.paged.pool.kv_codes, lt.paged.pool.kv_codes)
    assert torch.equal(layer.paged.pool.kv_meta.view(torch.int16), lt.paged.pool.kv_meta.view(torch.int16))
