"""Decode forward of Qwen3.5's full-attention layers over the paged cache: one launch per layer.

transformers' ``Qwen3_5Attention.forward`` (models/qwen3_5/modeling_qwen3_5.py:647-692) runs, per
decode token, the q / gate / k / v projections, the q / k RMS norms, the rotary embedding, the
cache update, the attention, the output gate ``* sigmoid(gate)`` and ``o_proj``.  With a packed
cache layer of this package the middle three are one kernel launch here
(``oq_decode_attn_paged_ex``): the new token is quantised into its page, the query attends over
the cache with it, and the gate is applied as the output is stored.  The projections, the norms,
the rotary embedding and ``o_proj`` are the module's own.  Any other call -- prefill, a layer that
the deferred policy still keeps dense, another cache type, training -- runs the module's own
forward unchanged.

The reference gets to the same kernels through its adapter
(optiz_qwen/kernels/qwen35_fused_attention.py), which dispatches on an attention-backend name and
then calls the cache update and the attention launcher separately.  Here there is no backend
name to consult: whether the layer's cache is packed decides, and the update rides in the
attention launch.
"""

from __future__ import annotations

import sys
import types

import torch


def _packed_layer(cache, layer_idx: int):
    """The cache layer of `layer_idx` when it is one of this package's packed layers, else None."""
    layers = getattr(cache, "layers", None)
    if layers is None or not 0 <= layer_idx < len(layers):
        return None
    layer = layers[layer_idx]
    prepare = getattr(layer, "prepare_decode", None)
    return layer if prepare is not None and prepare() else None


def paged_decode_forward(module, hidden_states: torch.Tensor, position_embeddings, attention_mask=None,
                         past_key_values=None, **kwargs):
    """``Qwen3_5Attention.forward`` for ``module``; a one-token call over a packed layer takes the
    one-launch path, every other call the module's own forward."""
    layer = None
    if hidden_states.dim() == 3 and hidden_states.shape[1] == 1 and not module.training:
        layer = _packed_layer(past_key_values, module.layer_idx)
    if layer is None:
        return module._oq_module_forward(hidden_states, position_embeddings, attention_mask, past_key_values,
                                         **kwargs)
    bsz, d = hidden_states.shape[0], module.head_dim
    # q_proj holds (query, gate) per head, 2 x head_dim wide
    qg = module.q_proj(hidden_states).view(bsz, 1, -1, 2 * d)
    query = module.q_norm(qg[..., :d]).transpose(1, 2)                                   # [B, Hq, 1, D]
    gate = qg[:, 0, :, d:]                                                              # [B, Hq, D]
    key = module.k_norm(module.k_proj(hidden_states).view(bsz, 1, -1, d)).transpose(1, 2)  # [B, Hkv, 1, D]
    value = module.v_proj(hidden_states).view(bsz, 1, -1, d).transpose(1, 2)
    cos, sin = position_embeddings
    rotary = sys.modules[type(module).__module__].apply_rotary_pos_emb  # the model file's own rotary
    query, key = rotary(query, key, cos, sin)
    out = layer.append_and_attend(query, key, value, scaling=module.scaling, gate=gate)  # [B, 1, Hq, D]
    return module.o_proj(out.reshape(bsz, 1, -1)), None


def install_paged_decode_forward(model) -> int:
    """Give every ``Qwen3_5Attention`` module of ``model`` the one-launch decode forward (its own
    forward stays as ``_oq_module_forward`` for every other call); returns how many were set."""
    count = 0
    for mod in model.modules():
        if type(mod).__name__ == "Qwen3_5Attention" and not hasattr(mod, "_oq_module_forward"):
            mod._oq_module_forward = mod.forward
            mod.forward = types.MethodType(paged_decode_forward, mod)
            count += 1
    return count
