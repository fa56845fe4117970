"""Append + attend in one launch (``oq_decode_attn_paged_ex``) against the separate launches.

The fused launch must leave the cache bit-identical to ``oq_append_quant_int4`` / ``_int8``
and the oracle's quantiser, and give the same output bits as the append launch followed by
the attention launch over ``seq_lens + 1`` tokens, whose parity with the fp32 oracle the other
attention tests establish (checked here too).  Cases: ragged lengths with the new token at the
start, middle and end of a page; split counts that put the new page in a later split, another
warp group, and beyond the first four pages of a group; both cache widths and query dtypes; a
gate; and early launches (``OQ_ATTN_EARLY``) captured in a CUDA graph behind another kernel.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_quant as kq
from tests._util import assert_attn_close, oracle_attention

pytestmark = pytest.mark.gpu

HKV, HQ, D, PAGE = 2, 8, 256, 64


def _cache(lengths, bits, seed, capacity_extra=64):
    """A device pool holding `lengths` tokens of random codes (page table permuted), twice."""
    from optiz_qwen_b200.cabi import PagedKvPool

    rng = np.random.default_rng(seed)
    cap = [n + capacity_extra for n in lengths]
    max_pages = max(-(-c // PAGE) for c in cap)
    num_pages = max_pages * len(lengths) + 2
    table = kq.build_block_table(cap, PAGE, num_pages, max_pages, seed)
    pools = []
    codes = rng.integers(0, 256, (num_pages, HKV, 2, PAGE, D * bits // 8), dtype=np.uint8)
    meta = np.empty((num_pages, HKV, 4, PAGE), np.float32)
    meta[:, :, 0::2] = rng.uniform(0.2, 0.4, meta[:, :, 0::2].shape)
    meta[:, :, 1::2] = rng.uniform(-3.0, -2.0, meta[:, :, 1::2].shape)
    meta = meta.astype(np.float16)
    for _ in range(2):
        pool = PagedKvPool(num_pages, HKV, D, PAGE, "cuda", bits=bits)
        pool.kv_codes.copy_(torch.from_numpy(codes))
        pool.kv_meta.copy_(torch.from_numpy(meta))
        pools.append(pool)
    t = torch.from_numpy(table).cuda()
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    return pools, t, lens, rng


def _inputs(rng, b, dtype):
    q = kq.round_bf16(rng.standard_normal((b, HQ, D), dtype=np.float32))
    k = kq.round_bf16(rng.standard_normal((b, HKV, D), dtype=np.float32))
    v = kq.round_bf16(rng.standard_normal((b, HKV, D), dtype=np.float32) * 2.0)
    g = kq.round_bf16(rng.standard_normal((b, HQ, D), dtype=np.float32))
    return [torch.from_numpy(x).cuda().to(dtype) for x in (q, k, v, g)]


def _separate(pool, table, lens, q, k, v, ws, num_splits, gate=None):
    from optiz_qwen_b200 import cabi

    cabi.append_quant(k.unsqueeze(2), v.unsqueeze(2), pool, table, lens.clone(), advance=False)
    return cabi.decode_attention(q, pool, table, lens + 1, D ** -0.5, workspace=ws, num_splits=num_splits, gate=gate)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("lengths,num_splits", [
    ([100, 64, 4095, 0], 0),          # mid-page, page start, page end, empty sequence
    ([4096, 1000], 4),                # the new page in the last split, in-launch merge
    ([4096, 1000], 64),               # many splits, merge kernel
    ([2000, 3000], 1),                # one range: the new page beyond a group's first four pages
    ([int(x) for x in np.random.default_rng(2).integers(0, 700, 200)], 0),  # many units: one-group form
])
def test_fused_append_matches_separate_launches(bits, lengths, num_splits):
    from optiz_qwen_b200 import cabi

    dtype = torch.bfloat16
    (pa, pb), table, lens, rng = _cache(lengths, bits, seed=len(lengths) * 7 + num_splits + bits)
    q, k, v, _ = _inputs(rng, len(lengths), dtype)
    ws_a = cabi.new_decode_workspace(len(lengths), HQ, HKV, table.shape[1], "cuda")
    ws_b = cabi.new_decode_workspace(len(lengths), HQ, HKV, table.shape[1], "cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = _separate(pa, table, lens, q, k, v, ws_a, num_splits)
    out = cabi.decode_attention(q, pb, table, lens, D ** -0.5, workspace=ws_b, num_splits=num_splits,
                                new_key=k, new_value=v, device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(pa.kv_codes, pb.kv_codes)
    assert torch.equal(pa.kv_meta.view(torch.int16), pb.kv_meta.view(torch.int16))
    assert torch.equal(out, ref)
    assert torch.equal(lens, torch.tensor(lengths, dtype=torch.int32, device="cuda"))  # seq_lens untouched
    # the appended rows are the oracle quantiser's, and the output the fp32 oracle's
    quant = kq.quantize_tokens_int4 if bits == 4 else kq.quantize_tokens_int8
    kc, ks, km = quant(k.float().cpu().numpy()[:, :, None])
    tbl = table.cpu().numpy()
    for bi, n in enumerate(lengths):
        pg, slot = int(tbl[bi, n // PAGE]), n % PAGE
        np.testing.assert_array_equal(pb.kv_codes[pg, :, 0, slot].cpu().numpy(), kc[bi, :, 0])
        np.testing.assert_array_equal(pb.kv_meta[pg, :, 0, slot].cpu().numpy(), ks[bi, :, 0])
        np.testing.assert_array_equal(pb.kv_meta[pg, :, 1, slot].cpu().numpy(), km[bi, :, 0])
    if bits == 4:
        from tests._util import oracle_from_device

        cache = oracle_from_device(pb, table, lens + 1, range(len(lengths)))
        expected, _ = oracle_attention(cache, q.float().cpu().numpy(), D ** -0.5)
        assert_attn_close(out.float().cpu().numpy(), expected)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_append_gated_fp16_and_graph_early(dtype):
    """Gated output, both query dtypes, and early launches replayed in a CUDA graph behind an
    unrelated kernel (the contract of OQ_ATTN_EARLY: the kernel ahead writes no cache data)."""
    from optiz_qwen_b200 import cabi

    lengths = [700, 64, 1]
    (pa, pb), table, lens, rng = _cache(lengths, 4, seed=11)
    q, k, v, g = _inputs(rng, len(lengths), dtype)
    ws_a = cabi.new_decode_workspace(len(lengths), HQ, HKV, table.shape[1], "cuda")
    ws_b = cabi.new_decode_workspace(len(lengths), HQ, HKV, table.shape[1], "cuda")
    ref = _separate(pa, table, lens, q, k, v, ws_a, 0, gate=g)
    out = torch.empty_like(q)
    scratch = torch.zeros(1 << 20, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        scratch.mul_(0.5)          # the kernel ahead: touches none of the cache data
        cabi.decode_attention(q, pb, table, lens, D ** -0.5, out=out, workspace=ws_b, gate=g, new_key=k,
                              new_value=v, early=True)
    for _ in range(3):             # every replay rewrites the same slot with the same bits
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(pa.kv_codes, pb.kv_codes)
        assert torch.equal(pa.kv_meta.view(torch.int16), pb.kv_meta.view(torch.int16))


def test_fused_append_rejects_bad_arguments():
    from optiz_qwen_b200 import cabi

    (pa, _), table, lens, rng = _cache([10], 4, seed=3)
    q, k, v, _ = _inputs(rng, 1, torch.bfloat16)
    with pytest.raises(ValueError):
        cabi.decode_attention(q, pa, table, lens, 1 / 16, new_key=k, new_value=None)
    with pytest.raises(ValueError):
        cabi.decode_attention(q, pa, table, lens, 1 / 16, new_key=k[:, :1], new_value=v[:, :1])
    with pytest.raises(ValueError):
        cabi.decode_attention(q, pa, table, lens, 1 / 16, new_key=k.half(), new_value=v.half())


@pytest.mark.parametrize("lengths,num_splits", [([3000, 64, 1], 0), ([20000], 0)])
def test_early_launch_without_append_matches_plain(lengths, num_splits):
    """OQ_ATTN_EARLY alone (no appended token), in a CUDA graph behind another kernel: the same
    bits as the plain launch, with one range per CTA and with the split merge kernel."""
    from optiz_qwen_b200 import cabi

    (pa, _), table, lens, rng = _cache(lengths, 4, seed=21)
    q, _, _, _ = _inputs(rng, len(lengths), torch.bfloat16)
    ws = cabi.new_decode_workspace(len(lengths), HQ, HKV, table.shape[1], "cuda")
    ref = cabi.decode_attention(q, pa, table, lens, D ** -0.5, workspace=ws, num_splits=num_splits)
    out = torch.empty_like(q)
    scratch = torch.zeros(1 << 20, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        scratch.mul_(0.5)
        cabi.decode_attention(q, pa, table, lens, D ** -0.5, out=out, workspace=ws, num_splits=num_splits,
                              early=True)
    for _ in range(2):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
