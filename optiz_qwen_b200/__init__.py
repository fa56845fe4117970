"""B200 (sm_100a) decode hot path for the optiz-qwen Qwen3.5 hybrid LM.

Drop-in replacements behind the reference's own Python surface:

* ``optiz_qwen_b200.compression`` -- the QServe packed-KV cache API
  (``QServeKvConfig``, ``QServeAttentionLayer`` ... ``QServeDeferredSplitFusedKvCache``)
  backed by a paged INT4 pool and the fused append-quantize kernel;
* ``optiz_qwen_b200.kernels`` -- ``qserve_int4_decode_attention`` /
  ``qserve_int4_split_decode_attention`` (split-KV INT4 decode attention) and
  ``qserve_int8_decode_attention``, the launchers the reference's decode-attention
  adapter imports;
* ``optiz_qwen_b200.gdn`` -- the Gated-DeltaNet hooks
  (``fused_recurrent_gated_delta_rule``, ``chunk_gated_delta_rule``) and
  ``install_gdn_fastpath``.

All compute runs in ``liboptiz_qwen_b200.so`` (hand-written CUDA for sm_100a,
C ABI in ``include/optiz_qwen_b200.h``).  There is no CPU fallback.
"""

from ._lib import available as library_available  # noqa: F401

__version__ = "0.1.0"
