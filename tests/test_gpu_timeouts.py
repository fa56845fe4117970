"""Failure detection on the device: a bounded wait that runs out.

Every kernel that waits on an asynchronous copy (TMA / bulk copy into shared memory, or a
tensor-core MMA) bounds the wait and reports OQ_DEV_TIMEOUT in the caller's status word
instead of hanging.  These tests make the waits run out without faulting or hanging
anything: ``oq_debug_set_wait_polls(0)`` lets every wait give up at its first poll while
the copies themselves are ordinary in-bounds copies that do land.  Each kernel must then
report the timeout, let its copies land before its CTAs exit, keep its workspace
consistent (merge counters back at zero), and the next normal call on the same buffers
must match the oracle.
"""

from __future__ import annotations

import contextlib

import numpy as np
import pytest
import torch

from oracle import gdn
from oracle import kv_quant as kq
from tests._util import assert_attn_close, assert_gdn_close, oracle_attention, upload_pool

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def wait_polls(n):
    from optiz_qwen_b200 import _lib

    lib = _lib.load()
    prev = lib.oq_debug_set_wait_polls(int(n))
    try:
        yield
    finally:
        lib.oq_debug_set_wait_polls(prev)


def _status():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def test_poll_limit_hook_round_trips():
    from optiz_qwen_b200 import _lib

    lib = _lib.load()
    default = lib.oq_debug_set_wait_polls(-1)
    assert default > 0
    assert lib.oq_debug_set_wait_polls(7) == default
    assert lib.oq_debug_set_wait_polls(-1) == 7
    assert lib.oq_debug_set_wait_polls(-1) == default


@pytest.mark.parametrize("num_splits,many", [(1, False), (4, False), (16, False), (64, False), (1, True)])
def test_attention_timeout_reports_and_leaves_workspace_consistent(num_splits, many):
    """1 split (single range per CTA), 4 (last-CTA merge through the counters), 16 (units of
    13 and 8 ranges, merged by the merge kernel), 64 (the merge kernel); and 300 short
    sequences, whose launch takes the one-warp-group form."""
    from optiz_qwen_b200 import _lib, cabi

    rng = np.random.default_rng(91)
    lengths = [int(x) for x in rng.integers(1, 400, 300)] if many else [4097, 300, 1, 2500]
    cache = kq.fill_paged_cache(rng, lengths, 2, 256, 64, seed_pages=3)
    pool, table, lens = upload_pool(cache)
    b = len(lengths)
    q = torch.from_numpy(kq.round_bf16(rng.standard_normal((b, 8, 256), dtype=np.float32))).cuda().to(torch.bfloat16)
    scaling = 256 ** -0.5
    ws = cabi.new_decode_workspace(b, 8, 2, table.shape[1], q.device)
    st = _status()
    with wait_polls(0):
        out = cabi.decode_attention_int4(q, pool, table, lens, scaling, workspace=ws, num_splits=num_splits,
                                         device_status=st)
        torch.cuda.synchronize()
    assert int(st.item()) & _lib.OQ_DEV_TIMEOUT
    assert torch.isfinite(out.float()).all()
    # every merge counter is back at zero, so the next launch on this workspace merges correctly
    counters = ws[: b * 2 * 4].view(torch.int32)
    assert int(counters.abs().sum().item()) == 0
    st.zero_()
    out = cabi.decode_attention_int4(q, pool, table, lens, scaling, workspace=ws, num_splits=num_splits,
                                     device_status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref, _ = oracle_attention(cache, q.float().cpu().numpy(), scaling)
    assert_attn_close(out.float().cpu().numpy(), ref)


def _gdn_inputs(rng, b=4, h=16, d=128):
    q, k, v = (kq.round_bf16(rng.standard_normal((b, 1, h, d), dtype=np.float32)) for _ in range(3))
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, 1, h))))).astype(np.float32)
    g = (-np.logaddexp(0, rng.standard_normal((b, 1, h)))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d))).astype(np.float32)
    return q, k, v, g, beta, s0


def test_gdn_step_timeout_leaves_state_and_output_untouched():
    from optiz_qwen_b200 import _lib, cabi

    rng = np.random.default_rng(92)
    q, k, v, g, beta, s0 = _gdn_inputs(rng)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    s = t(s0)
    sentinel = torch.full((4, 1, 16, 128), 7.0, device="cuda")
    st = _status()
    with wait_polls(0):
        cabi.gdn_recurrent(t(q), t(k), t(v), t(g), t(beta), initial_state=s, final_state=s, out=sentinel,
                           use_qk_l2norm=True, device_status=st)
        torch.cuda.synchronize()
    assert int(st.item()) & _lib.OQ_DEV_TIMEOUT
    assert torch.equal(s.cpu(), torch.from_numpy(s0))          # the state in place: unchanged
    assert bool((sentinel == 7.0).all())                       # no output written
    st.zero_()
    out = cabi.gdn_recurrent(t(q), t(k), t(v), t(g), t(beta), initial_state=s, final_state=s, use_qk_l2norm=True,
                             device_status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ro, rs = gdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)
    assert_gdn_close(out.cpu().numpy(), ro)
    assert_gdn_close(s.cpu().numpy(), rs)


@pytest.mark.parametrize("two_phase", [True, False])
def test_chunked_gdn_timeout_then_clean_run(two_phase):
    from optiz_qwen_b200 import _lib, cabi

    rng = np.random.default_rng(93)
    b, tp, h, d = 2, 130, 16, 128
    q, k, v = (kq.round_bf16(rng.standard_normal((b, tp, h, d), dtype=np.float32)) for _ in range(3))
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, tp, h))))).astype(np.float32)
    g = (-np.logaddexp(0, rng.standard_normal((b, tp, h)))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d))).astype(np.float32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    bf = lambda x: t(x).to(torch.bfloat16)  # noqa: E731
    sf = torch.empty((b, h, d, d), dtype=torch.float32, device="cuda")
    st = _status()
    with wait_polls(0):
        cabi.gdn_chunk_fwd(bf(q), bf(k), bf(v), t(g), t(beta), initial_state=t(s0), final_state=sf,
                           use_qk_l2norm=True, device_status=st, two_phase=two_phase)
        torch.cuda.synchronize()
    assert int(st.item()) & _lib.OQ_DEV_TIMEOUT
    st.zero_()
    out = cabi.gdn_chunk_fwd(bf(q), bf(k), bf(v), t(g), t(beta), initial_state=t(s0), final_state=sf,
                             use_qk_l2norm=True, device_status=st, two_phase=two_phase)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    _, rs = gdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    assert_gdn_close(sf.cpu().numpy(), rs)
    assert np.isfinite(out.float().cpu().numpy()).all()


def test_exchange_wait_timeout_reports_and_next_call_is_clean():
    """The NVLink exchange's wait for tagged words (one rank: its own words, stored before it polls) given no
    polls reports OQ_DEV_TIMEOUT and returns; the next call (the other slot parity) is clean."""
    from optiz_qwen_b200 import _lib, cabi
    from optiz_qwen_b200.context_parallel import PeerExchange

    gen = torch.Generator(device="cuda").manual_seed(9)
    ex = PeerExchange(8, 256, rank=0, world=1, device="cuda")
    part = torch.randn((8, 256), generator=gen, device="cuda")
    lse = torch.randn((8,), generator=gen, device="cuda")
    ref = cabi.lse_merge(part.view(1, 8, 256), lse.view(1, 8), dtype=torch.bfloat16)
    with wait_polls(0):
        ex.merge(0, part, lse)
        torch.cuda.synchronize()
    assert int(ex.status.item()) & _lib.OQ_DEV_TIMEOUT
    ex.status.zero_()
    out = ex.merge(0, part, lse)
    torch.cuda.synchronize()
    assert int(ex.status.item()) == 0 and torch.equal(out, ref)
