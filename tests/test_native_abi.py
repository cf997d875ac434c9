"""The C-ABI library loads on a machine without a GPU and exports every entry
point declared in include/forgeml_b200.h (no kernel is launched here)."""

import ctypes
import re
from pathlib import Path

from forgeml_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "forgeml_b200.h"


def declared_symbols() -> set[str]:
    return set(re.findall(r"FML_API\s+[\w\s\*]+?\b((?:fml|neb)_\w+)\s*\(", HEADER.read_text()))


def test_header_declares_the_expected_entry_points():
    syms = declared_symbols()
    for s in ("fml_gemm", "fml_gemm_workspace_size", "fml_gemm_noalloc", "fml_layernorm", "fml_sdpa",
              "neb_attention", "neb_kv_append", "neb_embed", "neb_argmax", "neb_add", "fml_pack_weight",
              "fml_linear_packed", "fml_packed_weight_bytes", "fml_last_error", "fml_device_status",
              "fml_launch_count", "fml_version"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    for s in declared_symbols():
        assert hasattr(lib, s), s
    # and the Python binding declares a signature for each of them
    assert declared_symbols() <= set(_native.EXPORTED)


def test_library_metadata_without_gpu():
    lib = _native.load()
    assert "sm_100a" in _native.version()
    assert lib.fml_last_error() is not None
    assert _native.launch_count() >= 0
