"""The CPU oracle reproduces the reference's own outputs (golden vectors from tests/golden/make_golden.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import attention as oattn
from oracle import gdn as ogdn
from oracle import kv_quant as kq

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def quant():
    return np.load(GOLD / "quant_golden.npz")


@pytest.mark.parametrize("group", [256, 32])
def test_quantizer_bit_exact(quant, group):
    x = kq.bf16_bits_to_f32(quant["x_bf16"])
    packed, scale, mn = kq.quantize_groupwise(x, group, 4)
    np.testing.assert_array_equal(packed, quant[f"g{group}_packed"])
    np.testing.assert_array_equal(scale, quant[f"g{group}_scale"])
    np.testing.assert_array_equal(mn, quant[f"g{group}_min"])
    np.testing.assert_array_equal(scale.astype(np.float16), quant[f"g{group}_scale_f16"])
    np.testing.assert_array_equal(mn.astype(np.float16), quant[f"g{group}_min_f16"])
    np.testing.assert_array_equal(kq.dequantize_groupwise(packed, scale, mn, group, 256), quant[f"g{group}_dequant"])


def test_quantizer_8bit_codes(quant):
    x = kq.bf16_bits_to_f32(quant["x_bf16"])
    codes, scale, mn = kq.quantize_groupwise(x, 32, 8)
    np.testing.assert_array_equal(codes, quant["g32_b8_codes"])
    np.testing.assert_array_equal(scale, quant["g32_b8_scale"])


def test_edge_rows(quant):
    x = kq.bf16_bits_to_f32(quant["x_bf16"])
    packed, scale, mn = kq.quantize_groupwise(x, 256, 4)
    assert scale[0, 0, 0, 0] == 1.0                      # constant row: scale 0 -> 1
    assert np.all(kq.unpack_uint4(packed[0, 0, 0], 256) == 0)
    codes = kq.unpack_uint4(packed[0, 0, 1], 256)         # ties at .5 round to even
    assert codes[2] == 0 and codes[3] == 2 and codes[4] == 2 and codes[5] == 4


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, (3, 5, 256), dtype=np.uint8)
    np.testing.assert_array_equal(kq.unpack_uint4(kq.pack_uint4(codes), 256), codes)


def test_paged_oracle_gather_matches_dense():
    rng = np.random.default_rng(1)
    lengths = [130, 64, 1]
    cache = kq.fill_paged_cache(rng, lengths, 2, 256, 64, seed_pages=9)
    for b, n in enumerate(lengths):
        k, v = cache.gather(b)
        assert k.shape == (2, n, 256) and v.shape == (2, n, 256)
        assert np.all(np.isfinite(k)) and np.all(np.isfinite(v))


def test_attention_oracle_matches_reference_sdpa():
    gold = np.load(GOLD / "attention_golden.npz")
    for name in "abc":
        k = kq.bf16_bits_to_f32(gold[f"{name}_k_bf16"])[0]
        v = kq.bf16_bits_to_f32(gold[f"{name}_v_bf16"])[0]
        q = kq.bf16_bits_to_f32(gold[f"{name}_q_bf16"])[0, :, 0]
        kp, ks, km = kq.quantize_tokens_int4(k)
        vp, vs, vm = kq.quantize_tokens_int4(v)
        out, _ = oattn.decode_attention(q[None], [kq.dequantize_tokens_int4(kp, ks, km)],
                                        [kq.dequantize_tokens_int4(vp, vs, vm)], float(gold[f"{name}_scaling"]))
        np.testing.assert_allclose(out[0], gold[f"{name}_out"][0, 0], rtol=1e-5, atol=1e-6)


def test_lse_merge_equals_full_attention():
    rng = np.random.default_rng(2)
    cache = kq.fill_paged_cache(rng, [1000], 2, 256, 64)
    k, v = cache.gather(0)
    q = rng.standard_normal((1, 8, 256)).astype(np.float32)
    full, full_lse = oattn.decode_attention(q, [k], [v], 0.0625)
    parts = oattn.split_kv_ranges(1000, 4, 64)
    outs, lses = [], []
    for lo, hi in parts:
        o, l = oattn.decode_attention(q, [k[:, lo:hi]], [v[:, lo:hi]], 0.0625)
        outs.append(o.reshape(8, 256))
        lses.append(l.reshape(8))
    merged, lse = oattn.lse_merge(np.stack(outs), np.stack(lses))
    np.testing.assert_allclose(merged, full[0], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lse, full_lse[0], rtol=1e-6, atol=1e-6)


def test_lse_merge_empty_parts():
    out, lse = oattn.lse_merge(np.zeros((2, 3, 4), np.float32), np.full((2, 3), -np.inf, np.float32))
    assert np.all(out == 0) and np.all(np.isneginf(lse))


@pytest.fixture(scope="module")
def gdn_gold():
    return np.load(GOLD / "gdn_golden.npz")


@pytest.mark.parametrize("name", ["step", "multi"])
def test_recurrent_matches_transformers(gdn_gold, name):
    g = gdn_gold
    o, s = ogdn.recurrent_gated_delta_rule(g[f"{name}_q"], g[f"{name}_k"], g[f"{name}_v"], g[f"{name}_g"],
                                           g[f"{name}_beta"], g[f"{name}_s0"], True, True)
    np.testing.assert_allclose(o, g[f"{name}_o"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s, g[f"{name}_s"], rtol=1e-5, atol=1e-6)


def test_chunk_matches_transformers_and_recurrent(gdn_gold):
    g = gdn_gold
    o, s = ogdn.chunk_gated_delta_rule(g["chunk_q"], g["chunk_k"], g["chunk_v"], g["chunk_g"], g["chunk_beta"],
                                       64, g["chunk_s0"], True, True)
    np.testing.assert_allclose(o, g["chunk_o"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(s, g["chunk_s"], rtol=1e-4, atol=1e-5)
    # the chunked form equals the token-by-token recurrence (transformers' own two functions)
    np.testing.assert_allclose(g["chunk_o"], g["chunk_o_rec"], rtol=1e-4, atol=1e-5)


def test_causal_conv1d_update_matches_transformers(gdn_gold):
    g = gdn_gold
    state = g["conv_state"].copy()
    y = ogdn.causal_conv1d_update(g["conv_x"], state, g["conv_w"])
    np.testing.assert_allclose(y, g["conv_y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(state, g["conv_state_after"])


# ---- output epilogues (gated RMSNorm of the GDN output, sigmoid gate of the attention output)
def _bf16_from_bits(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_rmsnorm_gated_matches_transformers():
    from oracle import epilogue as ep
    from oracle import kv_quant as kq

    g = np.load(GOLD / "epilogue_golden.npz")
    x, z, w = (_bf16_from_bits(g[k]) for k in ("norm_x", "norm_z", "norm_w"))
    want = _bf16_from_bits(g["norm_y"])
    got = ep.rmsnorm_gated(x, z, w, float(g["norm_eps"]), rnd=kq.round_bf16)
    assert np.array_equal(got, want)


def test_sigmoid_gate_matches_reference_expression():
    from oracle import epilogue as ep
    from oracle import kv_quant as kq

    g = np.load(GOLD / "epilogue_golden.npz")
    got = ep.sigmoid_gate(_bf16_from_bits(g["gate_attn"]), _bf16_from_bits(g["gate_g"]), rnd=kq.round_bf16)
    want = _bf16_from_bits(g["gate_y"])
    assert np.array_equal(got, want)


def test_int8_token_format_matches_the_reference_quantiser(quant):
    """The B200 8-bit token format = the reference's bits=8 quantiser with group = head_dim,
    scale/min rounded to fp16; the paged oracle round-trips it."""
    x = kq.bf16_bits_to_f32(quant["x_bf16"])
    codes, scale, mn = kq.quantize_tokens_int8(x)
    ref_codes, ref_scale, ref_min = kq.quantize_groupwise(x, x.shape[-1], 8)
    np.testing.assert_array_equal(codes, ref_codes)
    np.testing.assert_array_equal(scale, ref_scale[..., 0].astype(np.float16))
    deq = kq.dequantize_tokens_int8(codes, scale, mn)
    assert np.all(np.abs(deq - x) <= 0.51 * scale.astype(np.float32)[..., None] + 2e-3 * np.abs(x).max())
    rng = np.random.default_rng(2)
    cache = kq.fill_paged_cache(rng, [70, 5], 2, 256, 64, seed_pages=3, bits=8)
    assert cache.kv_codes.shape[-1] == 256
    k, v = cache.gather(0)
    assert k.shape == (2, 70, 256) and v.shape == (2, 70, 256)


def test_decay_gates_match_transformers():
    """The decode branch's g / beta (transformers modeling_qwen3_5.py:492-493) on bf16 inputs:
    beta bit-exact in bf16 (torch rounds sigmoid to b's dtype), g within a few fp32 ulps."""
    gold = np.load(GOLD / "gates_golden.npz")
    f = kq.bf16_bits_to_f32
    g, beta = ogdn.decay_gates(f(gold["a"]), f(gold["b"]), f(gold["A_log"]), f(gold["dt_bias"]), rnd=kq.round_bf16)
    assert np.array_equal(kq.f32_to_bf16_bits(beta), gold["beta"])
    np.testing.assert_allclose(g, gold["g"], rtol=1e-6, atol=0)
