"""Causal conv1d update (the GDN layer's short convolution), standalone and fused into
the GDN decode step, against transformers' golden vectors and the oracle.

The conv state is copied bit-exactly; outputs are fp32 within 1e-5 for fp32 inputs and
within bf16 rounding (half an ulp, at most 2^-8 relative, plus 1e-4 of the row scale)
for bf16 inputs.  The fused step's GDN state matches the oracle within rel 1e-4.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from oracle import kv_quant as kq
from tests._util import assert_gdn_close

pytestmark = pytest.mark.gpu

GOLD = __file__.replace("test_gpu_conv1d.py", "golden/gdn_golden.npz")


def _t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dtype)


def _close_bf16(got: np.ndarray, ref: np.ndarray) -> None:
    got, ref = got.astype(np.float64), ref.astype(np.float64)
    assert np.all(np.abs(got - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-4 * np.abs(ref).max() + 1e-30)


def test_transformers_golden_fp32():
    from optiz_qwen_b200.cabi import causal_conv1d_update

    g = np.load(GOLD)
    state = _t(g["conv_state"])
    out = causal_conv1d_update(_t(g["conv_x"]), state, _t(g["conv_w"]), None, silu=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), g["conv_y"], rtol=1e-5, atol=1e-6)
    assert np.array_equal(state.cpu().numpy(), g["conv_state_after"])


@pytest.mark.parametrize("t", [1, 2, 4, 5])
def test_bf16_against_oracle(t):
    from optiz_qwen_b200.cabi import causal_conv1d_update

    rng = np.random.default_rng(40 + t)
    b, c, w = 3, 6144, 4
    x = kq.round_bf16(rng.standard_normal((b, c, t), dtype=np.float32))
    st = kq.round_bf16(rng.standard_normal((b, c, w), dtype=np.float32))
    wt = kq.round_bf16(0.5 * rng.standard_normal((c, w), dtype=np.float32))
    bias = kq.round_bf16(0.1 * rng.standard_normal(c, dtype=np.float32))
    st_ref = st.copy()
    ref = ogdn.causal_conv1d_update(x, st_ref, wt, bias, silu=True)
    state = _t(st, torch.bfloat16)
    out = causal_conv1d_update(_t(x, torch.bfloat16), state, _t(wt, torch.bfloat16), _t(bias, torch.bfloat16))
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16
    assert np.array_equal(state.float().cpu().numpy(), st_ref)
    _close_bf16(out.float().cpu().numpy(), ref)


def test_hook_on_a_transposed_projection_output():
    """The call site passes mixed_qkv.transpose(1, 2): a [B, C, T] view of the [B, T, C] projection."""
    from optiz_qwen_b200.gdn.gated_delta_rule import causal_conv1d_update

    rng = np.random.default_rng(9)
    b, c, w = 2, 768, 4
    proj = kq.round_bf16(rng.standard_normal((b, 2, c), dtype=np.float32))
    st = kq.round_bf16(rng.standard_normal((b, c, w), dtype=np.float32))
    wt = kq.round_bf16(0.5 * rng.standard_normal((c, w), dtype=np.float32))
    st_ref = st.copy()
    ref = ogdn.causal_conv1d_update(proj.transpose(0, 2, 1), st_ref, wt, None, silu=True)
    state = _t(st, torch.bfloat16)
    x = _t(proj, torch.bfloat16).transpose(1, 2)
    assert x.stride() == (2 * c, 1, c)
    out = causal_conv1d_update(x, state, _t(wt, torch.bfloat16).unsqueeze(1), None, "silu")
    torch.cuda.synchronize()
    assert np.array_equal(state.float().cpu().numpy(), st_ref)
    _close_bf16(out.float().cpu().numpy(), ref)


def test_fused_conv_gdn_step_matches_conv_then_recurrence():
    from optiz_qwen_b200.cabi import gdn_conv_step

    rng = np.random.default_rng(21)
    b, h, d, w = 3, 16, 128, 4
    c = h * 3 * d
    qkv = kq.round_bf16(rng.standard_normal((b, c), dtype=np.float32))
    cst = kq.round_bf16(rng.standard_normal((b, c, w), dtype=np.float32))
    wt = kq.round_bf16(0.5 * rng.standard_normal((c, w), dtype=np.float32))
    bias = kq.round_bf16(0.1 * rng.standard_normal(c, dtype=np.float32))
    beta = kq.round_bf16((1.0 / (1.0 + np.exp(-rng.standard_normal((b, 1, h), dtype=np.float32)))).astype(np.float32))
    g = (-np.logaddexp(0.0, rng.standard_normal((b, 1, h), dtype=np.float32))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d), dtype=np.float32)).astype(np.float32)
    # oracle: conv (output rounded to bf16 like the unfused layer), split, recurrent step
    cst_ref = cst.copy()
    conv = kq.round_bf16(ogdn.causal_conv1d_update(qkv[:, :, None], cst_ref, wt, bias, silu=True)[:, :, 0])
    q = conv[:, :h * d].reshape(b, 1, h, d)
    k = conv[:, h * d:2 * h * d].reshape(b, 1, h, d)
    v = conv[:, 2 * h * d:].reshape(b, 1, h, d)
    ro, rs = ogdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)

    conv_state = _t(cst, torch.bfloat16)
    state = _t(s0)
    out = gdn_conv_step(_t(qkv, torch.bfloat16), conv_state, _t(wt, torch.bfloat16), _t(bias, torch.bfloat16),
                        _t(g), _t(beta, torch.bfloat16), num_heads=h, initial_state=state, final_state=state)
    torch.cuda.synchronize()
    assert np.array_equal(conv_state.float().cpu().numpy(), cst_ref)
    assert_gdn_close(state.cpu().numpy(), rs)
    _close_bf16(out.float().cpu().numpy(), ro)
