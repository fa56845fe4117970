"""Parity of the chunked GDN prefill kernel (tcgen05 / TMEM).

The state is fp32 and must match the fp32 references within rel 1e-4 (normwise and
max-abs relative to max|ref|).  The output is bf16 like the model's: every element
is within bf16 rounding (half an ulp: at most 2^-8 relative, plus the fp32 tolerance)
of the fp32 reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn
from oracle import kv_quant as kq
from tests._util import GDN_RTOL, assert_gdn_close

pytestmark = pytest.mark.gpu

GOLD = __file__.replace("test_gpu_gdn_chunk.py", "golden/gdn_golden.npz")


def _t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dtype)


def _inputs(rng, b, t, h, d=128, normalise=False):
    """Config-0 distributions: q,k,v bf16 N(0,1); beta = sigmoid(N); g = -softplus(N); S = 0.02 N.
    With ``normalise`` q and k are L2-normalised before the bf16 rounding (for runs without
    the in-kernel normalisation)."""
    q = rng.standard_normal((b, t, h, d), dtype=np.float32)
    k = rng.standard_normal((b, t, h, d), dtype=np.float32)
    if normalise:
        q, k = gdn.l2norm(q), gdn.l2norm(k)
    q, k = kq.round_bf16(q), kq.round_bf16(k)
    v = kq.round_bf16(rng.standard_normal((b, t, h, d), dtype=np.float32))
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((b, t, h), dtype=np.float32)))).astype(np.float32)
    g = -np.logaddexp(0.0, rng.standard_normal((b, t, h), dtype=np.float32)).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d), dtype=np.float32)).astype(np.float32)
    return q, k, v, g, beta, s0


def _assert_bf16_out(out: torch.Tensor, ref: np.ndarray) -> None:
    got = out.float().cpu().numpy().astype(np.float64)
    ref = ref.astype(np.float64)
    assert np.all(np.isfinite(got))
    bound = 2.0 ** -8 * np.abs(ref) + GDN_RTOL * np.abs(ref).max()
    excess = np.abs(got - ref) - bound
    assert excess.max() <= 0, f"bf16 output off by {excess.max():.3e} beyond rounding + tolerance"


def _run(q, k, v, g, beta, s0, l2norm=True, final=True):
    from optiz_qwen_b200.cabi import gdn_chunk_fwd

    b, t, h, d = q.shape
    s_out = torch.empty((b, h, d, d), dtype=torch.float32, device="cuda") if final else None
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = gdn_chunk_fwd(_t(q, torch.bfloat16), _t(k, torch.bfloat16), _t(v, torch.bfloat16), _t(g), _t(beta),
                        initial_state=None if s0 is None else _t(s0), final_state=s_out, use_qk_l2norm=l2norm,
                        device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, s_out


def test_transformers_golden_partial_chunk():
    """T = 130 (two full chunks and a 2-token tail) against transformers' torch_chunk_gated_delta_rule."""
    gold = np.load(GOLD)
    out, s = _run(gold["chunk_q"], gold["chunk_k"], gold["chunk_v"], gold["chunk_g"], gold["chunk_beta"],
                  gold["chunk_s0"])
    assert_gdn_close(s.cpu().numpy(), gold["chunk_s"])
    _assert_bf16_out(out, gold["chunk_o"])


@pytest.mark.parametrize("t", [1, 63, 64, 65, 200, 512])
def test_lengths_vs_chunk_oracle(t):
    rng = np.random.default_rng(100 + t)
    q, k, v, g, beta, s0 = _inputs(rng, 2, t, 3)
    ref_o, ref_s = gdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    out, s = _run(q, k, v, g, beta, s0)
    assert_gdn_close(s.cpu().numpy(), ref_s)
    _assert_bf16_out(out, ref_o)


def test_long_prompt_vs_token_by_token_oracle():
    """1024 tokens (16 chunks): the chunked kernel against the token-by-token recurrence."""
    rng = np.random.default_rng(4)
    q, k, v, g, beta, s0 = _inputs(rng, 1, 1024, 2)
    ref_o, ref_s = gdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)
    out, s = _run(q, k, v, g, beta, s0)
    assert_gdn_close(s.cpu().numpy(), ref_s)
    _assert_bf16_out(out, ref_o)


def test_no_initial_state_no_l2norm():
    rng = np.random.default_rng(7)
    q, k, v, g, beta, _ = _inputs(rng, 2, 150, 2, normalise=True)
    ref_o, ref_s = gdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, None, True, False, scale=0.125)
    from optiz_qwen_b200.cabi import gdn_chunk_fwd

    s = torch.empty((2, 2, 128, 128), dtype=torch.float32, device="cuda")
    out = gdn_chunk_fwd(_t(q, torch.bfloat16), _t(k, torch.bfloat16), _t(v, torch.bfloat16), _t(g), _t(beta),
                        scale=0.125, final_state=s, use_qk_l2norm=False)
    torch.cuda.synchronize()
    assert_gdn_close(s.cpu().numpy(), ref_s)
    _assert_bf16_out(out, ref_o)


def test_strided_slices_of_a_fused_projection_and_bf16_beta():
    """q, k, v as views into one [B, T, 3, H, 128] buffer (no copies); beta in bf16, g fp32."""
    from optiz_qwen_b200.cabi import gdn_chunk_fwd

    rng = np.random.default_rng(11)
    q, k, v, g, beta, s0 = _inputs(rng, 2, 96, 4)
    beta = kq.round_bf16(beta)
    fused = torch.empty((2, 96, 3, 4, 128), dtype=torch.bfloat16, device="cuda")
    for i, x in enumerate((q, k, v)):
        fused[:, :, i] = _t(x, torch.bfloat16)
    qv, kv_, vv = fused[:, :, 0], fused[:, :, 1], fused[:, :, 2]
    assert not qv.is_contiguous()
    s = _t(s0)
    out = gdn_chunk_fwd(qv, kv_, vv, _t(g), _t(beta, torch.bfloat16), initial_state=s, final_state=s,
                        use_qk_l2norm=True)
    torch.cuda.synchronize()
    ref_o, ref_s = gdn.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    assert_gdn_close(s.cpu().numpy(), ref_s)
    _assert_bf16_out(out, ref_o)


def test_empty_prompt_copies_the_state():
    from optiz_qwen_b200.cabi import gdn_chunk_fwd

    rng = np.random.default_rng(3)
    q, k, v, g, beta, s0 = _inputs(rng, 2, 0, 2)
    s = torch.empty((2, 2, 128, 128), dtype=torch.float32, device="cuda")
    out = gdn_chunk_fwd(_t(q, torch.bfloat16), _t(k, torch.bfloat16), _t(v, torch.bfloat16), _t(g), _t(beta),
                        initial_state=_t(s0), final_state=s, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert out.shape == (2, 0, 2, 128)
    assert np.array_equal(s.cpu().numpy(), s0)


def test_hook_signature_and_prefill_then_decode():
    """The GDN hook pair as Qwen3_5GatedDeltaNet calls it: prefill 300 tokens with
    chunk_gated_delta_rule, then 3 decode steps with recurrent_gated_delta_rule, against
    the token-by-token oracle over all 303 tokens."""
    from optiz_qwen_b200.gdn.gated_delta_rule import chunk_gated_delta_rule, recurrent_gated_delta_rule

    rng = np.random.default_rng(5)
    q, k, v, g, beta, s0 = _inputs(rng, 1, 303, 2)
    ref_o, ref_s = gdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)
    bt = lambda x: _t(x, torch.bfloat16)  # noqa: E731
    o1, s = chunk_gated_delta_rule(bt(q[:, :300]), bt(k[:, :300]), bt(v[:, :300]), g=_t(g[:, :300]),
                                   beta=_t(beta[:, :300]), initial_state=_t(s0), output_final_state=True,
                                   use_qk_l2norm_in_kernel=True)
    outs = [o1]
    for t in range(300, 303):
        o, s = recurrent_gated_delta_rule(bt(q[:, t:t + 1]), bt(k[:, t:t + 1]), bt(v[:, t:t + 1]), _t(g[:, t:t + 1]),
                                          _t(beta[:, t:t + 1]), initial_state=s, output_final_state=True,
                                          use_qk_l2norm_in_kernel=True)
        outs.append(o)
    torch.cuda.synchronize()
    assert_gdn_close(s.cpu().numpy(), ref_s)
    _assert_bf16_out(torch.cat(outs, dim=1), ref_o)


def test_config4_shape_matches_recurrent_kernel():
    """Full prefill shape of the tensor-core workload (B=8, T=8192, H=16): the chunked
    kernel's final state against the recurrent kernel's on the same device inputs."""
    from optiz_qwen_b200.cabi import gdn_chunk_fwd, gdn_recurrent

    gen = torch.Generator(device="cuda").manual_seed(4)
    b, t, h, d = 8, 8192, 16, 128
    q, k, v = (torch.randn((b, t, h, d), generator=gen, device="cuda").to(torch.bfloat16) for _ in range(3))
    beta = torch.sigmoid(torch.randn((b, t, h), generator=gen, device="cuda"))
    g = -torch.nn.functional.softplus(torch.randn((b, t, h), generator=gen, device="cuda"))
    s0 = 0.02 * torch.randn((b, h, d, d), generator=gen, device="cuda")
    s_chunk = torch.empty_like(s0)
    s_rec = torch.empty_like(s0)
    o_chunk = gdn_chunk_fwd(q, k, v, g, beta, initial_state=s0, final_state=s_chunk, use_qk_l2norm=True)
    o_rec = gdn_recurrent(q, k, v, g, beta, initial_state=s0, final_state=s_rec, use_qk_l2norm=True)
    torch.cuda.synchronize()
    assert_gdn_close(s_chunk.cpu().numpy(), s_rec.cpu().numpy())
    # both outputs are bf16 roundings of fp32 values that agree to ~1e-5: at most one bf16 step apart
    diff = (o_chunk.float() - o_rec.float()).abs()
    assert (diff <= 2.0 ** -7 * o_rec.float().abs() + 1e-3).all()


@pytest.mark.parametrize("b,t,h,init", [(1, 1, 2, True), (2, 63, 3, True), (1, 64, 2, False), (2, 65, 2, True),
                                        (3, 300, 4, True), (1, 1000, 2, False)])
def test_two_phase_form_matches_the_single_kernel_bit_for_bit(b, t, h, init):
    """oq_gdn_chunk_fwd_ws (state-independent work for all chunks first, then the state walk)
    gives the single-kernel form's outputs and final state exactly."""
    from optiz_qwen_b200.cabi import gdn_chunk_fwd, gdn_chunk_workspace_bytes

    gen = torch.Generator(device="cuda").manual_seed(b * 1000 + t)
    q, k, v = (torch.randn((b, t, h, 128), generator=gen, device="cuda").to(torch.bfloat16) for _ in range(3))
    g = -torch.nn.functional.softplus(torch.randn((b, t, h), generator=gen, device="cuda"))
    beta = torch.sigmoid(torch.randn((b, t, h), generator=gen, device="cuda"))
    s0 = 0.05 * torch.randn((b, h, 128, 128), generator=gen, device="cuda") if init else None
    results = []
    for two_phase in (False, True):
        s_out = torch.empty((b, h, 128, 128), device="cuda")
        ws = None
        if two_phase:  # a dirty, exactly sized workspace: nothing in it may be read before written
            ws = torch.full((gdn_chunk_workspace_bytes(b, t, h),), 0x7F, dtype=torch.uint8, device="cuda")
        out = gdn_chunk_fwd(q, k, v, g, beta, initial_state=s0, final_state=s_out, use_qk_l2norm=True,
                            two_phase=two_phase, workspace=ws)
        results.append((out, s_out))
    torch.cuda.synchronize()
    assert torch.equal(results[0][0], results[1][0])
    assert torch.equal(results[0][1], results[1][1])


def test_two_phase_form_rejects_a_short_workspace():
    from optiz_qwen_b200.cabi import gdn_chunk_fwd, gdn_chunk_workspace_bytes

    q = torch.zeros((1, 130, 2, 128), dtype=torch.bfloat16, device="cuda")
    g = torch.zeros((1, 130, 2), device="cuda")
    need = gdn_chunk_workspace_bytes(1, 130, 2)
    assert need == 3 * 2 * 50176
    with pytest.raises(ValueError, match="workspace of 301056 bytes needed"):
        gdn_chunk_fwd(q, q, q, g, g, workspace=torch.empty(need - 128, dtype=torch.uint8, device="cuda"))
