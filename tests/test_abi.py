"""The C-ABI library loads and exports every function include/fmoe.h declares
(no device calls)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "fmoe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fmoe_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "fmoe_moe_block_forward" in names and "fmoe_last_error" in names


def test_library_exports_every_declared_symbol(fm):
    lib = ctypes.CDLL(fm.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(fm):
    assert set(declared_functions()) <= set(fm.SIGNATURES)


def test_no_cuda_calls_needed_for_errors(fm):
    # argument validation runs on the host and reports through fmoe_last_error
    rc = fm.lib().fmoe_dequantize(None, None, None)
    assert rc == -1 and "null" in fm.last_error()
    assert fm.lib().fmoe_version() >= 100
