"""The shared library loads and exports every entry point declared in include/*.h (no GPU calls)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(oq_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("oq_append_quant_int4", "oq_decode_attn_int4_paged", "oq_lse_merge", "oq_gdn_recurrent",
                     "oq_append_quant_int8", "oq_decode_attn_int8_paged", "oq_gather_dequant_int8"):
        assert required in names


def test_library_exports_every_declared_symbol():
    import ctypes

    from optiz_qwen_b200 import _lib

    if not _lib.LIB_PATH.exists():
        pytest.fail(f"{_lib.LIB_PATH} is not built; run `python -m optiz_qwen_b200.build`")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, f"symbols declared but not exported: {missing}"


def test_binding_signatures_cover_the_header():
    from optiz_qwen_b200 import _lib

    assert declared_symbols() <= set(_lib.SIGNATURES), set(declared_symbols()) - set(_lib.SIGNATURES)


def test_host_only_entry_points():
    from optiz_qwen_b200 import _lib

    lib = _lib.load()
    assert lib.oq_abi_version() >= 1
    assert lib.oq_status_string(0) == b"ok"
    # workspace sizing is pure host arithmetic: counters + splits x heads x (D + 2) floats
    assert lib.oq_decode_attn_workspace_bytes(64, 8, 2, 256, 7) == 512 + 64 * 2 * 7 * 4 * 258 * 4
    assert lib.oq_decode_attn_workspace_bytes(0, 8, 2, 256, 7) == 0


def test_argument_validation_needs_no_gpu():
    """Bad arguments are rejected on the host before anything is launched."""
    from optiz_qwen_b200 import _lib

    lib = _lib.load()
    status = lib.oq_decode_attn_int4_paged(None, _lib.OQ_F32, 0, 0, None, None, 1, 64, None, 1, 1, None,
                                           1, 8, 2, 256, 1.0, None, 0, 0, None, None, None, 0, 0, None, None)
    assert status == _lib.OQ_ERR_UNSUPPORTED          # fp32 query
    status = lib.oq_gdn_recurrent(None, None, None, _lib.OQ_BF16, 0, 0, 0, 0, 0, 0, 0, 0, 0, None, 0, None, 0,
                                  None, None, None, 1, 1, 1, 64, 64, 1.0, 0, 0, None, None)
    assert status == _lib.OQ_ERR_UNSUPPORTED          # head dims other than 128
    assert b"128" in lib.oq_last_error()
