"""Oracle: the output epilogues around the decode kernels, in numpy.

TEST INFRASTRUCTURE ONLY -- imported by tests, smoke() and bench.py's CPU legs.

* ``rmsnorm_gated`` restates transformers' ``Qwen3_5RMSNormGated.forward``
  (models/qwen3_5/modeling_qwen3_5.py:175-190), applied by the GDN layer to the
  recurrent output with the ``z`` projection as gate (:527-529).
* ``sigmoid_gate`` restates the attention output gate of the reference's fused decode
  forward, ``attn_output * torch.sigmoid(gate)``
  (optiz_qwen/kernels/qwen35_fused_attention.py:96-97).

Both follow the reference's dtype steps: ``rnd`` rounds to the model dtype (bf16 via
``oracle.kv_quant.round_bf16``, or the identity for fp32 models).
``tests/golden/make_golden.py`` pins them against the transformers module and the
reference's torch expression.
"""

from __future__ import annotations

import numpy as np


def _identity(x):
    return np.asarray(x, np.float32)


def rmsnorm_gated(x, z, weight, eps: float = 1e-6, rnd=_identity) -> np.ndarray:
    """``y = rnd(rnd(rnd(x * rsqrt(mean(x^2) + eps)) * w) * silu(z))`` over the last axis.

    ``x``, ``z``, ``weight`` hold model-dtype values (as float32); the variance, the
    normalisation and the gate are computed in float32 as the module does.
    """
    x = np.asarray(x, np.float32)
    z = np.asarray(z, np.float32)
    w = np.asarray(weight, np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    h = rnd(x * inv)
    h = rnd(w * h)
    silu = z / (np.float32(1.0) + np.exp(-z))
    return rnd(h * silu)


def sigmoid_gate(o, gate, rnd=_identity) -> np.ndarray:
    """``rnd(rnd(o) * rnd(sigmoid(gate)))``: the model-dtype product of the attention
    output and the sigmoid of its gate, each operand in the model dtype."""
    g = np.asarray(gate, np.float32)
    sig = rnd(np.float32(1.0) / (np.float32(1.0) + np.exp(-g)))
    return rnd(rnd(o) * sig)
