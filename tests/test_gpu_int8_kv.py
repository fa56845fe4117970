"""The 8-bit paged KV cache (the reference's ``k_bits = v_bits = 8`` / ``triton_int8_decode`` path).

* append-quantize: codes, fp16 scale/min, page slots and lengths bit-exact against the
  oracle's 8-bit quantiser (255 levels, round-half-even of (x - min) / scale in fp32);
* gather-dequantise: bit-exact against the oracle's dequantisation rounded to the dtype;
* decode attention (``oq_decode_attn_int8_paged``): within the attention tolerance
  (max-abs 2e-3, rel 1e-2) of fp32 attention over the dequantised cache, for every
  split path, GQA ratio and query dtype; the gated variant equals the oracle gate on
  the kernel's own ungated output bit for bit;
* the cache layer with ``k_bits = 8`` through the reference-facing launcher.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogue as ep
from oracle import kv_quant as kq
from tests._util import assert_attn_close, bf16_tensor, oracle_attention, upload_pool

pytestmark = pytest.mark.gpu

LSE_TOL = 1e-3


# ---------------------------------------------------------------- append-quantize
def _setup(lengths, capacity_tokens, hkv=2, d=256, seed_pages=7, extra_pages=3):
    from optiz_qwen_b200.cabi import PagedKvPool

    page = 64
    max_pages = -(-capacity_tokens // page)
    num_pages = max_pages * len(lengths) + extra_pages
    table = kq.build_block_table([capacity_tokens] * len(lengths), page, num_pages, max_pages, seed_pages)
    oracle = kq.PagedKvOracle(num_pages, hkv, d, page, table, lengths, bits=8)
    pool = PagedKvPool(num_pages, hkv, d, page, "cuda", bits=8)
    t = torch.from_numpy(table).cuda()
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    return oracle, pool, t, lens


def _compare(oracle, pool, lens):
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.kv_codes.cpu().numpy(), oracle.kv_codes)
    np.testing.assert_array_equal(pool.kv_meta.cpu().numpy().view(np.uint16), oracle.kv_meta.view(np.uint16))
    np.testing.assert_array_equal(lens.cpu().numpy(), oracle.seq_lens)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_bulk_append_bit_exact(dtype):
    from optiz_qwen_b200.cabi import append_quant_int8

    rng = np.random.default_rng(10)
    oracle, pool, table, lens = _setup([0, 5, 63], capacity_tokens=200)
    k = rng.standard_normal((3, 2, 70, 256), dtype=np.float32)
    v = rng.standard_normal((3, 2, 70, 256), dtype=np.float32) * 3.0
    kt, vt = torch.from_numpy(k).cuda().to(dtype), torch.from_numpy(v).cuda().to(dtype)
    append_quant_int8(kt, vt, pool, table, lens)
    oracle.append(kt.float().cpu().numpy(), vt.float().cpu().numpy())
    _compare(oracle, pool, lens)


def test_decode_appends_cross_pages_bit_exact():
    from optiz_qwen_b200.cabi import append_quant

    rng = np.random.default_rng(11)
    oracle, pool, table, lens = _setup([0, 17, 64, 127], capacity_tokens=320)
    for _ in range(70):
        k = kq.round_bf16(rng.standard_normal((4, 2, 1, 256), dtype=np.float32))
        v = kq.round_bf16(rng.standard_normal((4, 2, 1, 256), dtype=np.float32))
        append_quant(bf16_tensor(k), bf16_tensor(v), pool, table, lens)  # dispatches on pool.bits
        oracle.append(k, v)
    _compare(oracle, pool, lens)


@pytest.mark.parametrize("d", [64, 128, 512])
def test_other_head_dims_and_strided_inputs(d):
    from optiz_qwen_b200.cabi import append_quant_int8

    rng = np.random.default_rng(d)
    oracle, pool, table, lens = _setup([3, 0], capacity_tokens=128, hkv=4, d=d)
    # [B, T, H, D] storage viewed as [B, H, T, D]
    k = kq.round_bf16(rng.standard_normal((2, 9, 4, d), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((2, 9, 4, d), dtype=np.float32))
    append_quant_int8(bf16_tensor(k).transpose(1, 2), bf16_tensor(v).transpose(1, 2), pool, table, lens)
    oracle.append(k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3))
    _compare(oracle, pool, lens)


def test_constant_rows_use_unit_scale():
    """A row whose max equals its min quantises with scale 1 (qserve_kv_cache.py:326-328): codes 0."""
    from optiz_qwen_b200.cabi import append_quant_int8

    oracle, pool, table, lens = _setup([0], capacity_tokens=64, hkv=1)
    k = np.full((1, 1, 3, 256), 0.375, np.float32)
    v = np.full((1, 1, 3, 256), -2.0, np.float32)
    append_quant_int8(bf16_tensor(k), bf16_tensor(v), pool, table, lens)
    oracle.append(k, v)
    _compare(oracle, pool, lens)
    assert not pool.kv_codes.any()


def test_entry_point_rejects_the_other_width():
    from optiz_qwen_b200.cabi import append_quant_int4

    _, pool, table, lens = _setup([0], capacity_tokens=64, hkv=1)
    x = torch.zeros(1, 1, 1, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="8-bit codes"):
        append_quant_int4(x, x, pool, table, lens)


# ---------------------------------------------------------------- gather-dequantise
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gather_dequant_bit_exact(dtype):
    from optiz_qwen_b200.cabi import gather_dequant_int8

    rng = np.random.default_rng(5)
    lengths = [130, 0, 64, 7]
    cache = kq.fill_paged_cache(rng, lengths, 2, 256, 64, seed_pages=3, bits=8)
    pool, table, lens = upload_pool(cache)
    max_len = max(lengths) + 5
    keys, values = gather_dequant_int8(pool, table, lens, max_len, dtype)
    torch.cuda.synchronize()
    rnd = kq.round_bf16 if dtype == torch.bfloat16 else (lambda a: a)
    for b, n in enumerate(lengths):
        got_k = keys[b].float().cpu().numpy()
        got_v = values[b].float().cpu().numpy()
        assert not got_k[:, n:].any() and not got_v[:, n:].any()
        if n == 0:
            continue
        k, v = cache.gather(b)
        np.testing.assert_array_equal(got_k[:, :n], rnd(k))
        np.testing.assert_array_equal(got_v[:, :n], rnd(v))


# ---------------------------------------------------------------- decode attention
def _run(lengths, hq=8, hkv=2, seed=0, splits=0, qdtype=torch.bfloat16, seed_pages=11, extra=True):
    from optiz_qwen_b200.cabi import decode_attention_int8

    rng = np.random.default_rng(seed)
    cache = kq.fill_paged_cache(rng, lengths, hkv, 256, 64, seed_pages=seed_pages, bits=8,
                                max_pages_per_seq=max(1, -(-max(lengths) // 64)) + (1 if extra else 0))
    q = kq.round_bf16(rng.standard_normal((len(lengths), hq, 256), dtype=np.float32))
    pool, table, lens = upload_pool(cache)
    qt = torch.from_numpy(q).cuda().to(qdtype)
    out_f32 = torch.empty((len(lengths), hq, 256), dtype=torch.float32, device="cuda")
    lse = torch.empty((len(lengths), hq), dtype=torch.float32, device="cuda")
    out = decode_attention_int8(qt, pool, table, lens, 256 ** -0.5, out_f32=out_f32, out_lse=lse, num_splits=splits)
    torch.cuda.synchronize()
    ref, ref_lse = oracle_attention(cache, qt.float().cpu().numpy(), 256 ** -0.5)
    return out.float().cpu().numpy(), out_f32.cpu().numpy(), lse.cpu().numpy(), ref, ref_lse


def test_config0_shapes():
    out, out32, lse, ref, ref_lse = _run([512, 512], seed=0)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


@pytest.mark.parametrize("length", [1, 15, 16, 17, 63, 64, 65, 129, 1000])
def test_edge_lengths(length):
    out, out32, lse, ref, ref_lse = _run([length], seed=length)
    assert_attn_close(out32, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


def test_many_units_one_group_form():
    """256 short ragged sequences: the 8-bit launch takes the one-warp-group form; every row
    against the oracle."""
    lengths = [int(x) for x in np.random.default_rng(6).integers(1, 600, 256)]
    out, out32, lse, ref, ref_lse = _run(lengths, seed=6)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)


@pytest.mark.parametrize("splits", [1, 2, 3, 0])
def test_forced_splits_ragged_batch(splits):
    out, out32, lse, ref, ref_lse = _run([700, 64, 1, 333, 129], seed=3, splits=splits)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (6, 2), (16, 2), (8, 1)])
def test_gqa_ratios(hq, hkv):
    out, out32, lse, ref, ref_lse = _run([300, 77], hq=hq, hkv=hkv, seed=hq)
    assert_attn_close(out32, ref)


def test_fp16_query():
    out, out32, lse, ref, ref_lse = _run([450, 3], seed=9, qdtype=torch.float16)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)


def test_empty_sequence_gives_zero_row_and_neg_inf_lse():
    out, out32, lse, ref, ref_lse = _run([0, 100], seed=4)
    assert not out[0].any() and not out32[0].any()
    assert np.all(np.isneginf(lse[0]))
    assert_attn_close(out32[1:], ref[1:])


def test_long_context_many_splits():
    out, out32, lse, ref, ref_lse = _run([8192, 5000], seed=12, seed_pages=None)
    assert_attn_close(out32, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


def test_int8_is_closer_to_the_unquantised_attention_than_int4():
    """The point of the 8-bit cache: the same K/V quantised to 255 levels lands nearer fp32
    attention over the unquantised values than 15 levels do."""
    from oracle.attention import decode_attention

    from optiz_qwen_b200.cabi import decode_attention as attn

    rng = np.random.default_rng(21)
    n = 600
    k = kq.round_bf16(rng.standard_normal((1, 2, n, 256), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((1, 2, n, 256), dtype=np.float32))
    q = kq.round_bf16(rng.standard_normal((1, 8, 256), dtype=np.float32))
    exact, _ = decode_attention(q, [k[0]], [v[0]], 256 ** -0.5)
    errs = {}
    for bits in (4, 8):
        table = kq.build_block_table([n], 64, 10, 10, 2)
        cache = kq.PagedKvOracle(10, 2, 256, 64, table, [0], bits=bits)
        cache.append(k, v)
        pool, tt, lens = upload_pool(cache)
        f32 = torch.empty(1, 8, 256, device="cuda")
        attn(bf16_tensor(q), pool, tt, lens, 256 ** -0.5, out_f32=f32, want_out=False)
        torch.cuda.synchronize()
        errs[bits] = float(np.abs(f32.cpu().numpy() - exact).max())
    assert errs[8] < errs[4] / 4, errs


@pytest.mark.parametrize("splits", [1, 3])
def test_gated_attention(splits):
    from optiz_qwen_b200.cabi import decode_attention_int8

    rng = np.random.default_rng(60 + splits)
    lengths = [700, 64, 1, 1333]
    hq, hkv, d = 8, 2, 256
    cache = kq.fill_paged_cache(rng, lengths, hkv, d, 64, seed_pages=7, bits=8,
                                max_pages_per_seq=-(-max(lengths) // 64) + 1)
    q = kq.round_bf16(rng.standard_normal((len(lengths), hq, d), dtype=np.float32))
    gate = kq.round_bf16(2.0 * rng.standard_normal((len(lengths), hq, d), dtype=np.float32))
    pool, table, lens = upload_pool(cache)
    qt, gt = bf16_tensor(q), bf16_tensor(gate)
    plain = decode_attention_int8(qt, pool, table, lens, d ** -0.5, num_splits=splits)
    gated = decode_attention_int8(qt, pool, table, lens, d ** -0.5, num_splits=splits, gate=gt)
    torch.cuda.synchronize()
    got = gated.float().cpu().numpy()
    assert np.array_equal(got, ep.sigmoid_gate(plain.float().cpu().numpy(), gate, rnd=kq.round_bf16))
    ref, _ = oracle_attention(cache, q, d ** -0.5)
    assert_attn_close(got, ep.sigmoid_gate(ref, gate, rnd=kq.round_bf16))


# ---------------------------------------------------------------- the cache layer
def test_8bit_layer_decode_through_the_reference_launcher():
    from oracle.attention import decode_attention

    from optiz_qwen_b200.compression import QServeAttentionLayer, QServeKvConfig
    from optiz_qwen_b200.kernels import qserve_int4_decode_attention, qserve_int8_decode_attention

    torch.manual_seed(41)
    layer = QServeAttentionLayer(QServeKvConfig(k_bits=8, v_bits=8, attention_backend="triton_int8_decode"))
    keys = torch.randn(2, 2, 300, 256, device="cuda", dtype=torch.bfloat16)
    values = torch.randn_like(keys)
    layer.update(keys, values)
    for _ in range(3):  # decode appends, then attention over the grown cache
        k1 = torch.randn(2, 2, 1, 256, device="cuda", dtype=torch.bfloat16)
        layer.update(k1, torch.randn_like(k1))
    assert layer.paged.pool.bits == 8 and layer.get_seq_length() == 303
    query = torch.randn(2, 8, 1, 256, device="cuda", dtype=torch.bfloat16)
    out = qserve_int8_decode_attention(query, layer, scaling=1 / 16)
    assert out.shape == (2, 1, 8, 256) and out.dtype == torch.bfloat16
    # fp32 attention over the layer's own dequantised cache (materialize = the gather kernel)
    mk, mv = layer.materialize()
    torch.cuda.synchronize()
    qn = query.float().cpu().numpy()[:, :, 0]
    ref, _ = decode_attention(qn, list(mk.float().cpu().numpy()), list(mv.float().cpu().numpy()), 1 / 16)
    # the materialised K/V are bf16-rounded: compare with the rounding's own slack added
    np.testing.assert_allclose(out[:, 0].float().cpu().numpy(), ref, rtol=2e-2, atol=1e-2)
    with pytest.raises(RuntimeError, match="4-bit cache"):
        qserve_int4_decode_attention(query, layer, scaling=1 / 16)
