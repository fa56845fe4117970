"""Parity of the split-KV INT4 paged decode attention kernel against the fp32 oracle.

Tolerance (the contract's): max-abs 2e-3 and rel 1e-2 vs fp32 attention over the
dequantised cache (stored fp16 scale/min).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_quant as kq
from oracle.attention import decode_attention
from tests._util import assert_attn_close, bf16_tensor, oracle_attention, upload_pool

pytestmark = pytest.mark.gpu

# Natural-log LSE of the scores.  q enters the q.k dot products as 21-bit fixed point
# (relative error <= 2^-21 of the head's largest element), and P' as fp16 plus its fp16
# remainder; an LSE error d scales merge weights by exp(d), i.e. a relative output
# error d, so 1e-3 stays an order of magnitude inside the 1e-2 output tolerance.
LSE_TOL = 1e-3


def _run(lengths, hq=8, hkv=2, seed=0, splits=0, qdtype=torch.bfloat16, seed_pages=11, extra=True):
    from optiz_qwen_b200.cabi import decode_attention_int4

    rng = np.random.default_rng(seed)
    cache = kq.fill_paged_cache(rng, lengths, hkv, 256, 64, seed_pages=seed_pages,
                                max_pages_per_seq=max(1, -(-max(lengths) // 64)) + (1 if extra else 0))
    q = kq.round_bf16(rng.standard_normal((len(lengths), hq, 256), dtype=np.float32))
    pool, table, lens = upload_pool(cache)
    qt = torch.from_numpy(q).cuda().to(qdtype)
    out_f32 = torch.empty((len(lengths), hq, 256), dtype=torch.float32, device="cuda")
    lse = torch.empty((len(lengths), hq), dtype=torch.float32, device="cuda")
    out = decode_attention_int4(qt, pool, table, lens, 256 ** -0.5, out_f32=out_f32, out_lse=lse, num_splits=splits)
    torch.cuda.synchronize()
    ref, ref_lse = oracle_attention(cache, qt.float().cpu().numpy(), 256 ** -0.5)
    return out.float().cpu().numpy(), out_f32.cpu().numpy(), lse.cpu().numpy(), ref, ref_lse


def test_config0_shapes():
    """Config 0: batch 2, 8 query heads, 2 KV heads, head_dim 256, context 512, page 64."""
    out, out32, lse, ref, ref_lse = _run([512, 512], seed=0)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


@pytest.mark.parametrize("length", [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 1000])
def test_edge_lengths(length):
    out, out32, lse, ref, ref_lse = _run([length], seed=length)
    assert_attn_close(out32, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 0])
def test_forced_splits_ragged_batch(splits):
    out, out32, lse, ref, ref_lse = _run([700, 64, 1, 333, 129], seed=3, splits=splits)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (8, 1), (16, 2), (6, 3)])
def test_gqa_ratios(hq, hkv):
    out, out32, lse, ref, ref_lse = _run([300, 77], hq=hq, hkv=hkv, seed=hq + hkv)
    assert_attn_close(out32, ref)


def test_fp16_query():
    out, out32, lse, ref, ref_lse = _run([450, 200], seed=5, qdtype=torch.float16)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)


def test_empty_sequence_gives_zero_row_and_neg_inf_lse():
    out, out32, lse, ref, ref_lse = _run([0, 70], seed=9)
    assert np.all(out32[0] == 0.0)
    assert np.all(np.isneginf(lse[0]))
    assert_attn_close(out32[1], ref[1])


def test_long_context_many_splits():
    out, out32, lse, ref, ref_lse = _run([8192], seed=12)
    assert_attn_close(out32, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)


def test_reference_golden_attention():
    """The kernel reproduces the reference test's oracle (SDPA over the dequantised cache)."""
    from optiz_qwen_b200.cabi import decode_attention_int4

    gold = np.load(__file__.replace("test_gpu_decode_attention.py", "golden/attention_golden.npz"))
    for name in "abc":
        k = kq.bf16_bits_to_f32(gold[f"{name}_k_bf16"])      # [1, 2, T, 256]
        v = kq.bf16_bits_to_f32(gold[f"{name}_v_bf16"])
        q = kq.bf16_bits_to_f32(gold[f"{name}_q_bf16"])[:, :, 0]  # [1, 8, 256]
        t = k.shape[2]
        pages = -(-t // 64)
        table = kq.build_block_table([t], 64, pages + 2, pages, seed=3)
        cache = kq.PagedKvOracle(pages + 2, 2, 256, 64, table, [0])
        cache.append(k, v)
        pool, tbl, lens = upload_pool(cache)
        out = decode_attention_int4(bf16_tensor(q), pool, tbl, lens, float(gold[f"{name}_scaling"]))
        torch.cuda.synchronize()
        assert_attn_close(out.float().cpu().numpy(), gold[f"{name}_out"][:, 0])


def test_repeated_launches_reuse_workspace():
    """Counters are left at zero: back-to-back launches on one workspace agree."""
    from optiz_qwen_b200.cabi import decode_attention_int4, new_decode_workspace

    rng = np.random.default_rng(21)
    cache = kq.fill_paged_cache(rng, [900, 1300, 40], 2, 256, 64, seed_pages=2)
    pool, table, lens = upload_pool(cache)
    q = bf16_tensor(kq.round_bf16(rng.standard_normal((3, 8, 256), dtype=np.float32)))
    ws = new_decode_workspace(3, 8, 2, table.shape[1], q.device)
    first = decode_attention_int4(q, pool, table, lens, 0.0625, workspace=ws, num_splits=4)
    for _ in range(5):
        again = decode_attention_int4(q, pool, table, lens, 0.0625, workspace=ws, num_splits=4)
        torch.cuda.synchronize()
        assert torch.equal(first, again)
    ref, _ = oracle_attention(cache, q.float().cpu().numpy(), 0.0625)
    assert_attn_close(first.float().cpu().numpy(), ref)


def test_bad_page_is_skipped_and_reported():
    from optiz_qwen_b200._lib import OQ_DEV_BAD_PAGE
    from optiz_qwen_b200.cabi import decode_attention_int4

    rng = np.random.default_rng(4)
    cache = kq.fill_paged_cache(rng, [192], 2, 256, 64, seed_pages=1)
    pool, table, lens = upload_pool(cache)
    table[0, 1] = -7
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    q = bf16_tensor(kq.round_bf16(rng.standard_normal((1, 8, 256), dtype=np.float32)))
    out = decode_attention_int4(q, pool, table, lens, 0.0625, device_status=status, num_splits=1)
    torch.cuda.synchronize()
    assert int(status.item()) & OQ_DEV_BAD_PAGE
    # the remaining pages (0 and 2) still give a finite result equal to attention over them
    k, v = cache.gather(0)
    keep = np.r_[0:64, 128:192]
    ref, _ = decode_attention(q.float().cpu().numpy(), [k[:, keep]], [v[:, keep]], 0.0625)
    assert_attn_close(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16])
def test_many_units_one_group_form(qdtype):
    """256 short ragged sequences (512 sequence x KV-head units, many waves): the launch takes the
    one-warp-group form, three CTAs per SM.  Every row against the oracle."""
    lengths = [int(x) for x in np.random.default_rng(5).integers(1, 600, 256)]
    out, out32, lse, ref, ref_lse = _run(lengths, seed=5, qdtype=qdtype)
    assert_attn_close(out32, ref)
    assert_attn_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=LSE_TOL, atol=LSE_TOL)
