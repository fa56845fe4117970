"""ctypes binding of ``liboptiz_qwen_b200.so`` (the C ABI in include/optiz_qwen_b200.h).

The library is loaded from the package directory.  If it is missing, every op
raises: there is no Python or CPU fallback for the hot path.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "liboptiz_qwen_b200.so"

OQ_OK = 0
OQ_ERR_INVALID_ARGUMENT = 1
OQ_ERR_UNSUPPORTED = 2
OQ_ERR_MISALIGNED = 3
OQ_ERR_WORKSPACE = 4
OQ_ERR_CUDA = 5

OQ_F32, OQ_F16, OQ_BF16 = 0, 1, 2
OQ_DEV_BAD_PAGE, OQ_DEV_OVERFLOW, OQ_DEV_TIMEOUT = 1, 2, 4
OQ_ATTN_EARLY = 1

_DTYPES = {torch.float32: OQ_F32, torch.float16: OQ_F16, torch.bfloat16: OQ_BF16}

p, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); mirrors include/optiz_qwen_b200.h
SIGNATURES = {
    "oq_status_string": (C.c_char_p, [i32]),
    "oq_last_error": (C.c_char_p, []),
    "oq_abi_version": (i32, []),
    "oq_append_quant_int4": (i32, [p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                   p, p, i64, i64, p, i64, i64, p, i32, p, p]),
    "oq_append_quant_int8": (i32, [p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                   p, p, i64, i64, p, i64, i64, p, i32, p, p]),
    "oq_advance_seq_lens": (i32, [p, i64, C.c_int32, p]),
    "oq_decode_attn_workspace_bytes": (sz, [i64, i64, i64, i64, i64]),
    "oq_decode_attn_int4_paged": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                        i64, i64, i64, i64, f32, p, i64, i64, p, p, p, sz, i32, p, p]),
    "oq_decode_attn_int8_paged": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                        i64, i64, i64, i64, f32, p, i64, i64, p, p, p, sz, i32, p, p]),
    "oq_decode_attn_int4_paged_noalloc": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                                i64, i64, i64, i64, f32, p, i64, i64, p, p, i32, p, p]),
    "oq_decode_attn_int4_paged_gated": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                              i64, i64, i64, i64, f32, p, i64, i64, p, i64, i64, p, sz, i32, p,
                                              p]),
    "oq_decode_attn_int8_paged_gated": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                              i64, i64, i64, i64, f32, p, i64, i64, p, i64, i64, p, sz, i32, p,
                                              p]),
    "oq_lse_merge": (i32, [p, p, i64, i64, i64, p, i32, p, p]),
    "oq_xrank_buffer_bytes": (sz, [i64, i64, i64]),
    "oq_ipc_handle_bytes": (sz, []),
    "oq_ipc_export": (i32, [p, p, p]),
    "oq_ipc_import": (i32, [p, i64, p]),
    "oq_ipc_close": (i32, [p, i64]),
    "oq_xrank_lse_merge": (i32, [p, p, i64, i64, p, i32, i32, p, i32, p, p, p]),
    "oq_decode_attn_int4_paged_xrank": (i32, [p, i32, i64, i64, p, p, i64, i64, p, i64, i64, p,
                                              i64, i64, i64, i64, f32, p, i64, i64, p, p, p, sz, i32, p, i32, i32,
                                              i32, p, p]),
    "oq_decode_attn_paged_ex": (i32, [i32, p, i32, i64, i64, p, i64, i64, p, i64, i64, p, p, i64, i64,
                                          p, i64, i64, p, i64, i64, i64, i64, f32, p, i64, i64, p, i64, i64,
                                          p, p, p, sz, i32, i32, p, p]),
    "oq_gather_dequant_int4": (i32, [p, p, i64, i64, p, i64, i64, p, i64, i64, i64, i64, p, p, i32, p, p]),
    "oq_gather_dequant_int8": (i32, [p, p, i64, i64, p, i64, i64, p, i64, i64, i64, i64, p, p, i32, p, p]),
    "oq_gdn_recurrent": (i32, [p, p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                               p, i32, p, i32, p, p, p, i64, i64, i64, i64, i64, f32, i32, i32, p, p]),
    "oq_gdn_recurrent_gates": (i32, [p, p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                     p, p, i32, p, i32, p, i32, p, p, p, i64, i64, i64, i64, i64, f32, i32, i32,
                                     p, p]),
    "oq_debug_set_wait_polls": (i32, [i32]),
    "oq_gdn_recurrent_norm": (i32, [p, p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                    p, i32, p, i32, p, p, p, i64, i64, i64, i64, i64, f32, i32,
                                    p, i64, i64, i64, p, f32, p, sz, i32, p]),
    "oq_gdn_norm_workspace_bytes": (sz, [i64, i64]),
    "oq_gdn_conv_step_norm": (i32, [p, i32, i64, p, p, p, i32, i64, i64, p, i32, p, i32, p, p, p, i64, i64, i64,
                                    i64, f32, i32, p, i64, i64, p, f32, p, sz, i32, p]),
    "oq_rmsnorm_gated": (i32, [p, i64, p, i64, p, p, i64, i32, i64, i64, f32, p]),
    "oq_causal_conv1d_update": (i32, [p, i32, i64, i64, i64, p, p, p, i32, p, i64, i64, i64, i64, i64, i32, p]),
    "oq_gdn_conv_step": (i32, [p, i32, i64, p, p, p, i32, i64, i64, p, i32, p, i32, p, p, p, i64, i64, i64, i64,
                               f32, i32, i32, p]),
    "oq_gdn_chunk_fwd": (i32, [p, p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                               p, i32, p, i32, p, p, p, i64, i64, i64, i64, i64, f32, i32, i64, p, p]),
    "oq_gdn_chunk_workspace_bytes": (sz, [i64, i64, i64]),
    "oq_gdn_chunk_fwd_ws": (i32, [p, p, p, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                  p, i32, p, i32, p, p, p, i64, i64, i64, i64, i64, f32, i32, i64, p, sz, p, p]),
}

_lib = None
_lock = threading.Lock()


class OqError(RuntimeError):
    """A C-ABI entry point returned a non-zero oq_status."""

    def __init__(self, name: str, status: int, detail: str):
        super().__init__(f"{name} failed ({status}): {detail}")
        self.status = status


def load() -> C.CDLL:
    """Load the shared library (once); raise ImportError when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m optiz_qwen_b200.build` "
                    "(the CUDA kernels are the only implementation of this path)"
                )
            lib = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def available() -> bool:
    try:
        load()
    except (ImportError, OSError):
        return False
    return True


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != OQ_OK:
        detail = (lib.oq_last_error() or b"").decode(errors="replace")
        if status in (OQ_ERR_INVALID_ARGUMENT, OQ_ERR_UNSUPPORTED, OQ_ERR_MISALIGNED, OQ_ERR_WORKSPACE):
            raise ValueError(f"{name}: {detail}")
        raise OqError(name, status, detail)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("optiz_qwen_b200 kernels need CUDA tensors (there is no CPU path)")
