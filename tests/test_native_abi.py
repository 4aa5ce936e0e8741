"""The C-ABI library loads and exports every entry point include/wgd.h declares
(no GPU needed: nothing here launches a kernel)."""
import ctypes
import os
import re

from webgpu_b200 import _native
from webgpu_b200._build_paths import REPO_DIR


def declared_symbols():
    text = open(os.path.join(REPO_DIR, "include", "wgd.h")).read()
    return sorted(set(re.findall(r"\b(wgd_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for name in ("wgd_create", "wgd_model_begin", "wgd_tensor_register", "wgd_model_end", "wgd_tensor_upload",
                 "wgd_forward", "wgd_truncate_kv", "wgd_cancel", "wgd_stats_get", "wgd_destroy", "wgd_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(os.path.join(REPO_DIR, "webgpu_b200", "_build", "libwgd.so"))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_every_symbol_and_abi_version():
    assert set(declared_symbols()) <= set(_native.SIGNATURES)
    assert _native.lib().wgd_abi_version() == 1


def test_row_layout_sizes_without_gpu():
    L = _native.lib()
    assert L.wgd_dev_row_bytes(12, 4096) == 16 * 144
    assert L.wgd_dev_row_bytes(14, 5376) == (21 * 210 + 15) // 16 * 16
    assert L.wgd_dev_row_bytes(2, 896) == (28 * 18 + 15) // 16 * 16
    assert L.wgd_dev_row_bytes(12, 100) == -1
