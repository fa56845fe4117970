"""Parity of the fused append-quantize kernel: codes, scales, mins and page slots bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_quant as kq
from tests._util import bf16_tensor

pytestmark = pytest.mark.gpu


def _setup(lengths, capacity_tokens, hkv=2, d=256, seed_pages=7, extra_pages=3):
    from optiz_qwen_b200.cabi import PagedKvPool

    page = 64
    max_pages = -(-capacity_tokens // page)
    num_pages = max_pages * len(lengths) + extra_pages
    table = kq.build_block_table([capacity_tokens] * len(lengths), page, num_pages, max_pages, seed_pages)
    oracle = kq.PagedKvOracle(num_pages, hkv, d, page, table, lengths)
    pool = PagedKvPool(num_pages, hkv, d, page, "cuda")
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
    from optiz_qwen_b200.cabi import append_quant_int4

    rng = np.random.default_rng(0)
    oracle, pool, table, lens = _setup([0, 5, 63], capacity_tokens=200)
    k = rng.standard_normal((3, 2, 70, 256), dtype=np.float32)
    v = rng.standard_normal((3, 2, 70, 256), dtype=np.float32) * 3.0
    kt = torch.from_numpy(k).cuda().to(dtype)
    vt = torch.from_numpy(v).cuda().to(dtype)
    append_quant_int4(kt, vt, pool, table, lens)
    oracle.append(kt.float().cpu().numpy(), vt.float().cpu().numpy())
    _compare(oracle, pool, lens)


def test_decode_appends_cross_pages_bit_exact():
    from optiz_qwen_b200.cabi import append_quant_int4

    rng = np.random.default_rng(1)
    oracle, pool, table, lens = _setup([0, 17, 64, 127], capacity_tokens=320)
    for _ in range(130):
        k = kq.round_bf16(rng.standard_normal((4, 2, 1, 256), dtype=np.float32))
        v = kq.round_bf16(rng.standard_normal((4, 2, 1, 256), dtype=np.float32))
        append_quant_int4(bf16_tensor(k), bf16_tensor(v), pool, table, lens)
        oracle.append(k, v)
    _compare(oracle, pool, lens)


def test_strided_inputs_and_head_dim_128():
    from optiz_qwen_b200.cabi import append_quant_int4

    rng = np.random.default_rng(2)
    oracle, pool, table, lens = _setup([3, 0], capacity_tokens=128, hkv=4, d=128)
    # [B, T, H, D] storage viewed as [B, H, T, D] (the layout a projection produces)
    k = kq.round_bf16(rng.standard_normal((2, 9, 4, 128), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((2, 9, 4, 128), dtype=np.float32))
    kt = bf16_tensor(k).transpose(1, 2)
    vt = bf16_tensor(v).transpose(1, 2)
    append_quant_int4(kt, vt, pool, table, lens)
    oracle.append(k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3))
    _compare(oracle, pool, lens)


def test_reference_golden_codes():
    """The kernel reproduces the reference quantiser's own outputs (per-token groups, fp16 scale/min)."""
    from optiz_qwen_b200.cabi import append_quant_int4

    gold = np.load(__file__.replace("test_gpu_append_quant.py", "golden/quant_golden.npz"))
    x = kq.bf16_bits_to_f32(gold["x_bf16"])            # [2, 2, 48, 256]
    oracle, pool, table, lens = _setup([0, 0], capacity_tokens=64)
    xt = bf16_tensor(x)
    append_quant_int4(xt, xt, pool, table, lens)
    torch.cuda.synchronize()
    codes = pool.kv_codes.cpu().numpy()
    meta = pool.kv_meta.cpu().numpy()
    tbl = table.cpu().numpy()
    for b in range(2):
        page = tbl[b, 0]
        for kv in (0, 1):
            np.testing.assert_array_equal(codes[page, :, kv, :48], gold["g256_packed"][b])
            np.testing.assert_array_equal(meta[page, :, 2 * kv, :48], gold["g256_scale_f16"][b][..., 0])
            np.testing.assert_array_equal(meta[page, :, 2 * kv + 1, :48], gold["g256_min_f16"][b][..., 0])


def test_bad_page_reports_and_skips():
    from optiz_qwen_b200._lib import OQ_DEV_BAD_PAGE, OQ_DEV_OVERFLOW
    from optiz_qwen_b200.cabi import append_quant_int4

    oracle, pool, table, lens = _setup([0, 60], capacity_tokens=64)
    table[0, 0] = pool.num_pages + 5          # corrupt entry: must be skipped, not written
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    k = torch.randn(2, 2, 8, 256, device="cuda", dtype=torch.bfloat16)
    append_quant_int4(k, k, pool, table, lens, device_status=status)
    torch.cuda.synchronize()
    bits = int(status.item())
    assert bits & OQ_DEV_BAD_PAGE
    assert bits & OQ_DEV_OVERFLOW            # row 1 runs past its single page
    assert lens.tolist() == [8, 68]
