"""The allocation-free decode-attention entry point agrees with the regular one.

oq_decode_attn_int4_paged_noalloc exists for callers that cannot call
cudaMalloc (a host runtime whose own arena owns the device memory, or a
foreign-language caller that only holds buffers allocated elsewhere): it takes
its split-KV scratch from a fixed 8 MiB array inside the library instead of a
caller workspace.  This file is collected last so a failure here leaves every
other test already run; it passes alone in a fresh process too.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_quant as kq
from tests._util import assert_attn_close, oracle_attention, random_paged_cache, upload_pool

pytestmark = pytest.mark.gpu


def _noalloc(q, pool, table, lens, scaling, out, num_splits=0, out_f32=None):
    from optiz_qwen_b200 import _lib

    lib = _lib.load()
    return lib.oq_decode_attn_int4_paged_noalloc(
        q.data_ptr(), _lib.dtype_code(q.dtype), q.stride(0), q.stride(1), pool.kv_codes.data_ptr(),
        pool.kv_meta.data_ptr(), pool.num_pages, pool.page_size, table.data_ptr(), table.stride(0), table.shape[1],
        lens.data_ptr(), q.shape[0], q.shape[1], pool.num_kv_heads, q.shape[2], float(scaling), out.data_ptr(),
        out.stride(0), out.stride(1), None if out_f32 is None else out_f32.data_ptr(), None, int(num_splits), None,
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_the_workspace_entry_point_on_consecutive_calls():
    from optiz_qwen_b200 import _lib, cabi

    rng = np.random.default_rng(77)
    lengths = [4096, 1000, 64, 3000]
    cache = kq.fill_paged_cache(rng, lengths, 2, 256, 64, seed_pages=5)
    pool, table, lens = upload_pool(cache)
    q = torch.from_numpy(kq.round_bf16(rng.standard_normal((4, 8, 256), dtype=np.float32))).cuda().to(torch.bfloat16)
    scaling = 256 ** -0.5
    expected = cabi.decode_attention_int4(q, pool, table, lens, scaling)       # caller-provided workspace
    ref, _ = oracle_attention(cache, q.float().cpu().numpy(), scaling)
    for _ in range(2):                                                       # two calls in a row
        out = torch.empty_like(q)
        assert _noalloc(q, pool, table, lens, scaling, out) == _lib.OQ_OK
        torch.cuda.synchronize()
        assert_attn_close(out.float().cpu().numpy(), expected.float().cpu().numpy())
        assert_attn_close(out.float().cpu().numpy(), ref)


def test_noalloc_rejects_scratch_beyond_its_fixed_size():
    from optiz_qwen_b200 import _lib

    rng = np.random.default_rng(78)
    cache = random_paged_cache(rng, [2048] * 64, 2, 256, 64, seed_pages=6)
    pool, table, lens = upload_pool(cache)
    q = torch.zeros((64, 8, 256), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(q)
    # 32 pages per sequence, so 32 splits stay 32 after the clamps: 64 sequences x 2 KV heads x
    # 32 ranges of 8 heads x 258 fp32 is ~34 MB > 8 MiB
    assert _noalloc(q, pool, table, lens, 0.0625, out, num_splits=32) == _lib.OQ_ERR_WORKSPACE
    assert b"scratch" in _lib.load().oq_last_error()
    # the automatic split count always fits
    assert _noalloc(q, pool, table, lens, 0.0625, out) == _lib.OQ_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("lengths", [[4097] * 64, [131072]], ids=["b64_ctx4097", "b1_ctx131072"])
def test_noalloc_runs_the_regular_partition(lengths):
    """Both entry points pick the same split count (the regular heuristic) whenever its scratch
    fits, so their fp32 outputs are bit-identical: one range per CTA at the hybrid bench shape,
    64 ranges and the merge kernel at 131072 tokens."""
    from optiz_qwen_b200 import _lib, cabi

    rng = np.random.default_rng(79)
    cache = random_paged_cache(rng, lengths, 2, 256, 64, seed_pages=7)
    pool, table, lens = upload_pool(cache)
    b = len(lengths)
    q = torch.from_numpy(kq.round_bf16(rng.standard_normal((b, 8, 256), dtype=np.float32))).cuda().to(torch.bfloat16)
    regular = torch.empty((b, 8, 256), dtype=torch.float32, device="cuda")
    cabi.decode_attention_int4(q, pool, table, lens, 256 ** -0.5, out_f32=regular, want_out=False)
    for _ in range(2):
        mine = torch.full_like(regular, float("nan"))
        out = torch.empty_like(q)
        assert _noalloc(q, pool, table, lens, 256 ** -0.5, out, out_f32=mine) == _lib.OQ_OK
        torch.cuda.synchronize()
        assert torch.equal(mine, regular)
