"""Decode attention for the paged INT4 / INT8 cache, behind the reference's launcher names.

The reference's decode-attention adapter (optiz_qwen/kernels/qwen35_fused_attention.py)
imports these four names from its ``qserve_int4_attention`` module; pointing that import
here is the whole switch.  ``install_paged_decode_forward`` is this package's own decode
forward for Qwen3.5's attention modules, with the cache update, attention and output gate in
one launch.
"""

from .decode_forward import install_paged_decode_forward, paged_decode_forward
from .qserve_int4_attention import (
    int4_decode_available,
    qserve_int4_decode_attention,
    qserve_int4_split_decode_attention,
    qserve_int8_decode_attention,
    triton_int4_decode_available,
)

__all__ = [
    "install_paged_decode_forward",
    "paged_decode_forward",
    "int4_decode_available",
    "qserve_int4_decode_attention",
    "qserve_int4_split_decode_attention",
    "qserve_int8_decode_attention",
    "triton_int4_decode_available",
]
