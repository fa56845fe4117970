"""Gated DeltaNet hooks backed by the sm_100a kernels.

Qwen3_5GatedDeltaNet calls its instance attributes ``recurrent_gated_delta_rule``
(decode) and ``chunk_gated_delta_rule`` (prefill) as
``f(q, k, v, g=g, beta=beta, initial_state=S | None, output_final_state=bool,
use_qk_l2norm_in_kernel=True)`` (transformers models/qwen3_5/modeling_qwen3_5.py:499-520)
and expects ``(o [B, T, H, Dv] in q's dtype, S_final [B, H, Dk, Dv] fp32 | None)``.
The reference binds fla 0.5.1's Triton kernels there (or transformers' torch
loops, :234-353); these functions take their place with fla's keyword
signature.  The state stays fp32; q/k L2 normalisation is done in fp32 inside
the kernel (as fla does).
"""

from __future__ import annotations

import torch

from .. import cabi


def _check_unsupported(cu_seqlens, use_gate_in_kernel, kwargs):
    if cu_seqlens is not None:
        raise NotImplementedError("variable-length (cu_seqlens) inputs are not supported; pass [B, T, H, D] batches")
    if use_gate_in_kernel:
        raise NotImplementedError("use_gate_in_kernel is not supported; pass the log-space decay g")
    if kwargs.get("transpose_state_layout"):
        raise NotImplementedError("transpose_state_layout is not supported; the state layout is [B, H, Dk, Dv]")


def _expand_value_heads(q, k, v):
    """GVA (more value heads than q/k heads): repeat q/k heads on the device."""
    h, hv = q.shape[2], v.shape[2]
    if hv == h:
        return q, k
    if hv % h:
        raise ValueError(f"value heads ({hv}) must be a multiple of q/k heads ({h})")
    return q.repeat_interleave(hv // h, dim=2), k.repeat_interleave(hv // h, dim=2)


def fused_recurrent_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                     g: torch.Tensor | None = None, gk=None, gv=None,
                                     beta: torch.Tensor | None = None, scale: float | None = None,
                                     initial_state: torch.Tensor | None = None, output_final_state: bool = False,
                                     use_qk_l2norm_in_kernel: bool = False, use_gate_in_kernel: bool = False,
                                     A_log=None, dt_bias=None, cu_seqlens=None, **kwargs):
    """Token-by-token gated delta rule (fla/ops/gated_delta_rule/fused_recurrent.py:291 signature)."""
    _check_unsupported(cu_seqlens, use_gate_in_kernel, kwargs)
    if gk is not None or gv is not None:
        raise NotImplementedError("per-channel decays (gk / gv) are not supported")
    q, k = _expand_value_heads(q, k, v)
    if g is None:
        g = torch.zeros(q.shape[:3], dtype=torch.float32, device=q.device)
    if beta is None:
        beta = torch.ones(q.shape[:3], dtype=q.dtype, device=q.device)
    batch, _, heads, dk = q.shape
    dv = v.shape[-1]
    if initial_state is not None:
        initial_state = initial_state.to(torch.float32).contiguous()
    final = (torch.empty((batch, heads, dk, dv), dtype=torch.float32, device=q.device)
             if output_final_state else None)
    out = cabi.gdn_recurrent(q, k, v, g, beta, scale=scale, initial_state=initial_state, final_state=final,
                             use_qk_l2norm=use_qk_l2norm_in_kernel)
    return out, final


def recurrent_gated_delta_rule(query, key, value, g, beta, initial_state=None, output_final_state=False,
                               use_qk_l2norm_in_kernel=False, scale=None):
    """Same operation with transformers' torch-fallback argument order
    (``torch_recurrent_gated_delta_rule``, modeling_qwen3_5.py:314)."""
    return fused_recurrent_gated_delta_rule(query, key, value, g=g, beta=beta, scale=scale,
                                            initial_state=initial_state, output_final_state=output_final_state,
                                            use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)


def chunk_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                           beta: torch.Tensor, scale: float | None = None,
                           initial_state: torch.Tensor | None = None, output_final_state: bool = False,
                           use_qk_l2norm_in_kernel: bool = False, cu_seqlens=None, chunk_size: int = 64,
                           **kwargs):
    """Prefill form (fla/ops/gated_delta_rule/chunk.py:365 signature).

    bf16 inputs with 128-wide heads run the chunked WY form of
    ``torch_chunk_gated_delta_rule`` (modeling_qwen3_5.py:234-311) on the tensor
    cores (``oq_gdn_chunk_fwd``, 64-token chunks, fp32 state in tensor memory).
    Other input dtypes run the same recurrence token by token through the
    recurrent kernel, which reads fp16 / fp32 directly.
    """
    _check_unsupported(cu_seqlens, kwargs.pop("use_gate_in_kernel", False), kwargs)
    if chunk_size != cabi.CHUNK_SIZE:
        raise ValueError(f"chunk_size must be {cabi.CHUNK_SIZE}")
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16) or q.shape[-1] != 128 or v.shape[-1] != 128:
        return fused_recurrent_gated_delta_rule(q, k, v, g=g, beta=beta, scale=scale, initial_state=initial_state,
                                                output_final_state=output_final_state,
                                                use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    q, k = _expand_value_heads(q, k, v)
    batch, _, heads, dk = q.shape
    dv = v.shape[-1]
    if initial_state is not None:
        initial_state = initial_state.to(torch.float32).contiguous()
    final = (torch.empty((batch, heads, dk, dv), dtype=torch.float32, device=q.device)
             if output_final_state else None)
    out = cabi.gdn_chunk_fwd(q, k, v, g, beta, scale=scale, initial_state=initial_state, final_state=final,
                             use_qk_l2norm=use_qk_l2norm_in_kernel)
    return out, final


def causal_conv1d_update(x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None = None, activation: str | None = None, cache_seqlens=None,
                         conv_state_indices=None, **kwargs) -> torch.Tensor:
    """The layer's short convolution on the decode path (causal-conv1d 1.6.2 ``causal_conv1d_update``
    signature; transformers torch_causal_conv1d_update, modeling_qwen3_5.py:210-225): x ``[B, C, T]``,
    conv_state ``[B, C, W]`` updated in place, weight ``[C, K]``; activation None or "silu"/"swish"."""
    if cache_seqlens is not None or conv_state_indices is not None:
        raise NotImplementedError("cache_seqlens / conv_state_indices are not supported")
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError(f"activation {activation!r} is not supported")
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(-1)
    out = cabi.causal_conv1d_update(x, conv_state, weight, bias, silu=activation is not None)
    return out.squeeze(-1) if squeeze else out


def rmsnorm_gated_forward(self, hidden_states: torch.Tensor, gate: torch.Tensor | None = None) -> torch.Tensor:
    """``Qwen3_5RMSNormGated.forward`` (transformers models/qwen3_5/modeling_qwen3_5.py:181-190) on
    the ``oq_rmsnorm_gated`` kernel: same dtype steps, bound per module by :func:`install_gdn_fastpath`."""
    if gate is None:
        raise NotImplementedError("the gated RMSNorm hook needs the gate (the GDN layer always passes z)")
    if not hidden_states.is_cuda:
        raise RuntimeError("rmsnorm_gated requires CUDA tensors")
    return cabi.rmsnorm_gated(hidden_states, gate.to(hidden_states.dtype), self.weight,
                              float(self.variance_epsilon))


def install_gdn_fastpath(model) -> int:
    """Bind the hooks on every Gated-DeltaNet module of ``model``; returns how many were patched.

    This replaces the reference's PYTHONPATH overlay that makes fla importable
    before transformers binds its fast path (scripts/run_v11_cuda_matrix.py:285-289).
    The module's output norm (a Qwen3_5RMSNormGated at ``module.norm``) gets the gated
    RMSNorm kernel as its forward.
    """
    from types import MethodType

    patched = 0
    for module in model.modules():
        if "GatedDeltaNet" in type(module).__name__ and hasattr(module, "recurrent_gated_delta_rule"):
            module.recurrent_gated_delta_rule = fused_recurrent_gated_delta_rule
            module.chunk_gated_delta_rule = chunk_gated_delta_rule
            module.causal_conv1d_update = causal_conv1d_update
            norm = getattr(module, "norm", None)
            if norm is not None and "RMSNormGated" in type(norm).__name__:
                norm.forward = MethodType(rmsnorm_gated_forward, norm)
            patched += 1
    return patched
