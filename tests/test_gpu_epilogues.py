"""Output epilogues fused into the decode kernels, against the oracle and transformers' golden.

* Attention: ``attn * sigmoid(gate)`` in the kernel's store (every store path: one KV
  range, in-launch split merge, separate merge kernel).  The gated output equals the
  oracle gate applied to the kernel's own ungated output bit for bit, and the oracle
  attention + gate within the attention tolerance.
* GDN: Qwen3_5RMSNormGated(o, z) fused into the recurrent step and into the conv step
  (4-CTA clusters); the state is unchanged by the epilogue (bit-exact), the output
  matches the oracle recurrence + norm within bf16 rounding, and the standalone
  gated-RMSNorm kernel on the unfused output within one bf16 ulp.
* Standalone gated RMSNorm against transformers' module (golden vectors) and the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import epilogue as ep
from oracle import gdn as ogdn
from oracle import kv_quant as kq
from tests._util import assert_attn_close, assert_gdn_close, oracle_attention, upload_pool

pytestmark = pytest.mark.gpu

GOLD = __file__.replace("test_gpu_epilogues.py", "golden/epilogue_golden.npz")


def _bf16_from_bits(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _t(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(dtype)


def _ulp_close(got: np.ndarray, ref: np.ndarray, ulps: int = 1) -> None:
    """Within `ulps` bf16 units in the last place (2^-7 relative per ulp at most)."""
    got, ref = got.astype(np.float64), ref.astype(np.float64)
    assert np.all(np.abs(got - ref) <= ulps * 2.0 ** -7 * np.abs(ref) + 1e-30)


# ---------------------------------------------------------------- attention output gate
@pytest.mark.parametrize("splits", [1, 3, 16])
def test_gated_attention(splits):
    from optiz_qwen_b200.cabi import decode_attention_int4

    rng = np.random.default_rng(60 + splits)
    lengths = [700, 64, 1, 1333]
    hq, hkv, d = 8, 2, 256
    cache = kq.fill_paged_cache(rng, lengths, hkv, d, 64, seed_pages=7, max_pages_per_seq=-(-max(lengths) // 64) + 1)
    q = kq.round_bf16(rng.standard_normal((len(lengths), hq, d), dtype=np.float32))
    gate = kq.round_bf16(2.0 * rng.standard_normal((len(lengths), 1, hq * d), dtype=np.float32))
    pool, table, lens = upload_pool(cache)
    qt, gt = _t(q), _t(gate)
    plain = decode_attention_int4(qt, pool, table, lens, d ** -0.5, num_splits=splits)
    gated = decode_attention_int4(qt, pool, table, lens, d ** -0.5, num_splits=splits,
                                  gate=gt.reshape(len(lengths), hq, d))
    torch.cuda.synchronize()
    g = gate.reshape(len(lengths), hq, d)
    got = gated.float().cpu().numpy()
    # the epilogue is exactly the reference's unfused expression on the kernel's own output
    assert np.array_equal(got, ep.sigmoid_gate(plain.float().cpu().numpy(), g, rnd=kq.round_bf16))
    ref, _ = oracle_attention(cache, q, d ** -0.5)
    assert_attn_close(got, ep.sigmoid_gate(ref, g, rnd=kq.round_bf16))


def test_gated_attention_rejects_fp32_outputs():
    from optiz_qwen_b200.cabi import decode_attention_int4

    rng = np.random.default_rng(1)
    cache = kq.fill_paged_cache(rng, [64], 2, 256, 64, seed_pages=1, max_pages_per_seq=2)
    pool, table, lens = upload_pool(cache)
    q = torch.zeros(1, 8, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="query-dtype output only"):
        decode_attention_int4(q, pool, table, lens, 0.0625, gate=q.clone(),
                              out_f32=torch.empty(1, 8, 256, device="cuda"))


# ---------------------------------------------------------------- GDN gated RMSNorm
def _gdn_inputs(rng, b, t, h, d=128):
    q, k, v, z = (kq.round_bf16(rng.standard_normal((b, t, h, d), dtype=np.float32)) for _ in range(4))
    beta = kq.round_bf16((1.0 / (1.0 + np.exp(-rng.standard_normal((b, t, h), dtype=np.float32)))).astype(np.float32))
    g = (-np.logaddexp(0.0, rng.standard_normal((b, t, h), dtype=np.float32))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d), dtype=np.float32)).astype(np.float32)
    w = kq.round_bf16((1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32))
    return q, k, v, z, g, beta, s0, w


@pytest.mark.parametrize("b,t,h", [(3, 1, 16), (2, 3, 4)])
def test_gdn_recurrent_with_gated_norm(b, t, h):
    from optiz_qwen_b200.cabi import gdn_recurrent, rmsnorm_gated

    rng = np.random.default_rng(70 + t)
    q, k, v, z, g, beta, s0, w = _gdn_inputs(rng, b, t, h)
    args = (_t(q), _t(k), _t(v), _t(g, torch.float32), _t(beta))
    s_plain, s_norm = _t(s0, torch.float32), _t(s0, torch.float32)
    plain = gdn_recurrent(*args, initial_state=s_plain, final_state=s_plain, use_qk_l2norm=True)
    normed = gdn_recurrent(*args, initial_state=s_norm, final_state=s_norm, use_qk_l2norm=True, z=_t(z),
                           norm_weight=_t(w), norm_eps=1e-6)
    unfused = rmsnorm_gated(plain, _t(z), _t(w), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(s_plain, s_norm)  # the epilogue leaves the state alone
    got = normed.float().cpu().numpy()
    _ulp_close(got, unfused.float().cpu().numpy())
    ro, rs = ogdn.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, True)
    assert_gdn_close(s_norm.cpu().numpy(), rs)
    ref = ep.rmsnorm_gated(kq.round_bf16(ro), z, w, 1e-6, rnd=kq.round_bf16)
    # o agrees with the fp32 oracle to 1e-4 of its largest element, which the norm carries to the output
    # scale: bf16 rounding plus that error
    assert np.all(np.abs(got - ref) <= 3 * 2.0 ** -7 * np.abs(ref) + 2e-3 * np.abs(ref).max())


def test_gdn_conv_step_with_gated_norm():
    from optiz_qwen_b200.cabi import gdn_conv_step, rmsnorm_gated

    rng = np.random.default_rng(81)
    b, h, d, width = 2, 16, 128, 4
    c = h * 3 * d
    qkv = kq.round_bf16(rng.standard_normal((b, c), dtype=np.float32))
    cst = kq.round_bf16(rng.standard_normal((b, c, width), dtype=np.float32))
    cw = kq.round_bf16(0.5 * rng.standard_normal((c, width), dtype=np.float32))
    z = kq.round_bf16(rng.standard_normal((b, h, d), dtype=np.float32))
    w = kq.round_bf16((1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32))
    beta = kq.round_bf16((1.0 / (1.0 + np.exp(-rng.standard_normal((b, 1, h), dtype=np.float32)))).astype(np.float32))
    g = (-np.logaddexp(0.0, rng.standard_normal((b, 1, h), dtype=np.float32))).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((b, h, d, d), dtype=np.float32)).astype(np.float32)
    outs, states = [], []
    for norm in (False, True):
        st, conv = _t(s0, torch.float32), _t(cst)
        kw = dict(z=_t(z), norm_weight=_t(w)) if norm else {}
        outs.append(gdn_conv_step(_t(qkv), conv, _t(cw), None, _t(g, torch.float32), _t(beta), num_heads=h,
                                  initial_state=st, final_state=st, **kw))
        states.append(st)
    unfused = rmsnorm_gated(outs[0].reshape(b, h, d), _t(z), _t(w), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(states[0], states[1])
    _ulp_close(outs[1].reshape(b, h, d).float().cpu().numpy(), unfused.float().cpu().numpy())


# ---------------------------------------------------------------- standalone gated RMSNorm
def test_rmsnorm_gated_transformers_golden():
    from optiz_qwen_b200.cabi import rmsnorm_gated

    g = np.load(GOLD)
    x, z, w = (_bf16_from_bits(g[k]) for k in ("norm_x", "norm_z", "norm_w"))
    want = _bf16_from_bits(g["norm_y"])
    got = rmsnorm_gated(_t(x), _t(z), _t(w), float(g["norm_eps"]))
    torch.cuda.synchronize()
    got = got.float().cpu().numpy()
    _ulp_close(got, want)
    assert np.mean(got == want) > 0.99


@pytest.mark.parametrize("rows,dim,dtype", [(1, 32, torch.bfloat16), (37, 128, torch.bfloat16),
                                            (9, 1000, torch.float16), (64, 256, torch.float32)])
def test_rmsnorm_gated_against_oracle(rows, dim, dtype):
    from optiz_qwen_b200.cabi import rmsnorm_gated

    rng = np.random.default_rng(rows + dim)
    rnd = {torch.bfloat16: kq.round_bf16, torch.float16: lambda a: np.asarray(a, np.float16).astype(np.float32),
           torch.float32: lambda a: np.asarray(a, np.float32)}[dtype]
    x, z = (rnd(rng.standard_normal((rows, dim), dtype=np.float32)) for _ in range(2))
    w = rnd((1.0 + 0.1 * rng.standard_normal(dim, dtype=np.float32)).astype(np.float32))
    # a strided view: every other row of a wider buffer
    xb = torch.zeros(rows, 2 * dim, dtype=dtype, device="cuda")
    xb[:, :dim] = _t(x, dtype)
    got = rmsnorm_gated(xb[:, :dim], _t(z, dtype), _t(w, dtype), 1e-5)
    torch.cuda.synchronize()
    ref = ep.rmsnorm_gated(x, z, w, 1e-5, rnd=rnd)
    got = got.float().cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
    else:
        # three chained roundings to the model dtype: at most 2 ulps apart from the oracle's
        tol = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -9
        assert np.all(np.abs(got - ref) <= tol * np.abs(ref) + 1e-30)


def test_installed_norm_hook_matches_the_module():
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNormGated

    from optiz_qwen_b200.gdn.gated_delta_rule import rmsnorm_gated_forward

    rng = np.random.default_rng(3)
    norm = Qwen3_5RMSNormGated(128, eps=1e-6).to("cuda", torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(_t(1.0 + 0.1 * rng.standard_normal(128, dtype=np.float32)))
    x = _t(rng.standard_normal((5, 16, 128), dtype=np.float32))
    z = _t(rng.standard_normal((5, 16, 128), dtype=np.float32))
    with torch.no_grad():
        want = norm(x, z)
        got = rmsnorm_gated_forward(norm, x, z)
    torch.cuda.synchronize()
    _ulp_close(got.float().cpu().numpy(), want.float().cpu().numpy())
