"""Generate the golden vectors that pin the numpy oracle to the reference's own code.

Run in a container that has the reference checkout (read-only is fine) and
transformers installed:

    python tests/golden/make_golden.py --reference /root/reference

It imports the reference quantiser ``QServeAttentionLayer._quantize_groupwise`` /
``_dequantize_groupwise`` (optiz_qwen/compression/qserve_kv_cache.py:313-353) and
the GDN functions the reference's hook falls back to
(transformers models/qwen3_5/modeling_qwen3_5.py:210-353), feeds them seeded
inputs and stores inputs + outputs as small ``.npz`` files next to this script.
The GPU box never runs this script; tests only read the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _bf16_bits(t):
    import torch

    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def make_quant(layer_cls, torch):
    rng = np.random.default_rng(20240601)
    x = torch.from_numpy(rng.standard_normal((2, 2, 48, 256), dtype=np.float32)).to(torch.bfloat16)
    # edge rows: constant (scale 0 -> 1), exact .5 ties, a wide range, tiny values
    x[0, 0, 0] = 0.75
    ties = torch.zeros(256)
    ties[1] = 15.0
    ties[2:] = torch.tensor([0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5, 7.5, 8.5, 9.5, 10.5, 11.5, 12.5, 13.5]).repeat(19)[:254]
    x[0, 0, 1] = ties.to(torch.bfloat16)
    x[0, 1, 2] = (x[0, 1, 2].float() * 1000.0).to(torch.bfloat16)
    x[1, 0, 3] = (x[1, 0, 3].float() * 1e-5).to(torch.bfloat16)
    x[1, 1, 4] = -3.0
    x[1, 1, 4, 7] = 2.0
    out = {"x_bf16": _bf16_bits(x)}
    for gs in (256, 32):
        packed, scale, mn = layer_cls._quantize_groupwise(x, gs, 4)
        deq = layer_cls._dequantize_groupwise(packed, scale, mn, gs, 256, torch.float32, 4)
        out[f"g{gs}_packed"] = packed.numpy()
        out[f"g{gs}_scale"] = scale.numpy()
        out[f"g{gs}_min"] = mn.numpy()
        out[f"g{gs}_scale_f16"] = scale.to(torch.float16).numpy()
        out[f"g{gs}_min_f16"] = mn.to(torch.float16).numpy()
        out[f"g{gs}_dequant"] = deq.numpy()
    # 8-bit path of the same quantiser (the INT8 backend's storage)
    packed8, scale8, mn8 = layer_cls._quantize_groupwise(x, 32, 8)
    out["g32_b8_codes"] = packed8.numpy()
    out["g32_b8_scale"] = scale8.numpy()
    out["g32_b8_min"] = mn8.numpy()
    np.savez_compressed(HERE / "quant_golden.npz", **out)


def make_attention(layer_cls, torch):
    """The reference test's oracle (tests/test_qserve_kv_cache.py:175-195) on per-token groups:
    SDPA over the cache dequantised with the stored fp16 scale/min, GQA by repeat_interleave."""
    import torch.nn.functional as F

    rng = np.random.default_rng(31)
    out = {}
    for name, (t, hq, hkv, d) in {"a": (200, 8, 2, 256), "b": (65, 8, 2, 256), "c": (1, 8, 2, 256)}.items():
        k = torch.from_numpy(rng.standard_normal((1, hkv, t, d), dtype=np.float32)).to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((1, hkv, t, d), dtype=np.float32)).to(torch.bfloat16)
        q = torch.from_numpy(rng.standard_normal((1, hq, 1, d), dtype=np.float32)).to(torch.bfloat16)
        kp, ks, km = layer_cls._quantize_groupwise(k, d, 4)
        vp, vs, vm = layer_cls._quantize_groupwise(v, d, 4)
        ks16, km16, vs16, vm16 = (x.to(torch.float16).to(torch.float32) for x in (ks, km, vs, vm))
        kd = layer_cls._dequantize_groupwise(kp, ks16, km16, d, d, torch.float32, 4)
        vd = layer_cls._dequantize_groupwise(vp, vs16, vm16, d, d, torch.float32, 4)
        scaling = 1.0 / d ** 0.5
        ref = F.scaled_dot_product_attention(
            q.float(), kd.repeat_interleave(hq // hkv, dim=1), vd.repeat_interleave(hq // hkv, dim=1),
            is_causal=False, scale=scaling,
        ).transpose(1, 2)
        out[f"{name}_k_bf16"] = _bf16_bits(k)
        out[f"{name}_v_bf16"] = _bf16_bits(v)
        out[f"{name}_q_bf16"] = _bf16_bits(q)
        out[f"{name}_out"] = ref.numpy()
        out[f"{name}_scaling"] = np.float32(scaling)
    np.savez_compressed(HERE / "attention_golden.npz", **out)


def make_gdn(torch):
    import torch.nn.functional as F
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m

    rng = np.random.default_rng(4)
    out = {}

    def inputs(b, t, h, d):
        q = torch.from_numpy(rng.standard_normal((b, t, h, d), dtype=np.float32)).to(torch.bfloat16).float()
        k = torch.from_numpy(rng.standard_normal((b, t, h, d), dtype=np.float32)).to(torch.bfloat16).float()
        v = torch.from_numpy(rng.standard_normal((b, t, h, d), dtype=np.float32)).to(torch.bfloat16).float()
        beta = torch.sigmoid(torch.from_numpy(rng.standard_normal((b, t, h), dtype=np.float32)))
        g = -F.softplus(torch.from_numpy(rng.standard_normal((b, t, h), dtype=np.float32)))
        s0 = 0.02 * torch.from_numpy(rng.standard_normal((b, h, d, d), dtype=np.float32))
        return q, k, v, g, beta, s0

    for name, (b, t, h) in {"step": (2, 1, 2), "multi": (1, 5, 2)}.items():
        q, k, v, g, beta, s0 = inputs(b, t, h, 128)
        o, s = m.torch_recurrent_gated_delta_rule(
            q, k, v, g=g, beta=beta, initial_state=s0.clone(), output_final_state=True,
            use_qk_l2norm_in_kernel=True,
        )
        for key, val in dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, o=o, s=s).items():
            out[f"{name}_{key}"] = val.numpy()

    q, k, v, g, beta, s0 = inputs(1, 130, 2, 128)
    oc, sc = m.torch_chunk_gated_delta_rule(
        q, k, v, g=g, beta=beta, chunk_size=64, initial_state=s0.clone(), output_final_state=True,
        use_qk_l2norm_in_kernel=True,
    )
    orr, sr = m.torch_recurrent_gated_delta_rule(
        q, k, v, g=g, beta=beta, initial_state=s0.clone(), output_final_state=True,
        use_qk_l2norm_in_kernel=True,
    )
    for key, val in dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, o=oc, s=sc, o_rec=orr, s_rec=sr).items():
        out[f"chunk_{key}"] = val.numpy()

    # causal conv1d update (decode branch, modeling_qwen3_5.py:210-225, call site :454)
    x = torch.from_numpy(rng.standard_normal((2, 96, 1), dtype=np.float32))
    state = torch.from_numpy(rng.standard_normal((2, 96, 4), dtype=np.float32))
    w = torch.from_numpy(rng.standard_normal((96, 4), dtype=np.float32)) * 0.5
    st = state.clone()
    y = m.torch_causal_conv1d_update(x, st, w, None, "silu")
    out.update(conv_x=x.numpy(), conv_state=state.numpy(), conv_w=w.numpy(), conv_y=y.numpy(),
               conv_state_after=st.numpy())
    np.savez_compressed(HERE / "gdn_golden.npz", **out)


def make_epilogue(torch):
    """The output epilogues around the two decode kernels, in bf16 as the model runs them:
    Qwen3_5RMSNormGated on the GDN output (transformers modeling_qwen3_5.py:175-190, call
    site :527-529) and the attention output gate ``attn_output * torch.sigmoid(gate)``
    (optiz_qwen/kernels/qwen35_fused_attention.py:96-97)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m

    rng = np.random.default_rng(5)
    out = {}
    rows, dim = 48, 128
    x = torch.from_numpy(rng.standard_normal((rows, dim), dtype=np.float32)).to(torch.bfloat16)
    z = torch.from_numpy(rng.standard_normal((rows, dim), dtype=np.float32)).to(torch.bfloat16)
    norm = m.Qwen3_5RMSNormGated(dim, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(1.0 + 0.1 * rng.standard_normal(dim, dtype=np.float32)))
        y = norm(x, z)
    out.update(norm_x=_bf16_bits(x), norm_z=_bf16_bits(z), norm_w=_bf16_bits(norm.weight.detach()),
               norm_y=_bf16_bits(y), norm_eps=np.float32(1e-6))
    attn = torch.from_numpy(rng.standard_normal((3, 1, 8 * 256), dtype=np.float32)).to(torch.bfloat16)
    gate = torch.from_numpy(2.0 * rng.standard_normal((3, 1, 8 * 256), dtype=np.float32)).to(torch.bfloat16)
    gated = attn * torch.sigmoid(gate)
    out.update(gate_attn=_bf16_bits(attn), gate_g=_bf16_bits(gate), gate_y=_bf16_bits(gated))
    np.savez_compressed(HERE / "epilogue_golden.npz", **out)


def make_gates(torch):
    """The GDN decode branch's gate arithmetic ahead of the hook (transformers
    modeling_qwen3_5.py:492-493), on bf16 projections and bf16 parameters as a bf16 model
    holds them: ``beta = b.sigmoid()``, ``g = -A_log.float().exp() * F.softplus(a.float() + dt_bias)``."""
    import torch.nn.functional as F

    rng = np.random.default_rng(6)
    bsz, t, h = 4, 3, 16
    a = torch.from_numpy(3.0 * rng.standard_normal((bsz, t, h), dtype=np.float32)).to(torch.bfloat16)
    b = torch.from_numpy(3.0 * rng.standard_normal((bsz, t, h), dtype=np.float32)).to(torch.bfloat16)
    a[0, 0, :4] = torch.tensor([25.0, -30.0, 19.5, 0.0])          # softplus threshold and tails
    A_log = torch.log(torch.from_numpy(rng.uniform(1.0, 16.0, h).astype(np.float32))).to(torch.bfloat16)
    dt_bias = torch.ones(h, dtype=torch.bfloat16) + 0.1 * torch.from_numpy(
        rng.standard_normal(h, dtype=np.float32)).to(torch.bfloat16)
    beta = b.sigmoid()
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias)
    np.savez_compressed(HERE / "gates_golden.npz", a=_bf16_bits(a), b=_bf16_bits(b), A_log=_bf16_bits(A_log),
                        dt_bias=_bf16_bits(dt_bias), beta=_bf16_bits(beta), g=g.numpy().astype(np.float32))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (its src/ holds the optiz_qwen package)")
    ap.add_argument("--only", choices=["quant", "attention", "gdn", "epilogue", "gates"], default=None,
                    help="regenerate one fixture file only")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch

    torch.manual_seed(0)
    from optiz_qwen.compression.qserve_kv_cache import QServeAttentionLayer

    if args.only in (None, "quant"):
        make_quant(QServeAttentionLayer, torch)
    if args.only in (None, "attention"):
        make_attention(QServeAttentionLayer, torch)
    if args.only in (None, "gdn"):
        make_gdn(torch)
    if args.only in (None, "epilogue"):
        make_epilogue(torch)
    if args.only in (None, "gates"):
        make_gates(torch)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
