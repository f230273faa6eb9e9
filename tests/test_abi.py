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


def test_kv_cache_layout_host_only(fm):
    """fmoe_kv_cache_bytes / fmoe_kv_cache_init carve a buffer on the host."""
    import ctypes

    L = fm.lib()
    B, H, D, cap = 2, 8, 256, 1024
    rows = B * H * cap
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    assert L.fmoe_kv_cache_bytes(0, B, H, D, cap) == 2 * up(rows * D * 2)
    aff = up(rows * D // 2) + up(rows * D) + 4 * up(rows * (D // 64) * 2)
    assert L.fmoe_kv_cache_bytes(1, B, H, D, cap) == aff
    assert L.fmoe_kv_cache_bytes(1, B, H, 128, cap) == 0          # head_dim not compiled
    assert L.fmoe_kv_cache_bytes(1, B, H, D, 1000) == 0           # capacity not a multiple of 16
    c = fm.KvCacheC()
    base = 1 << 40  # never dereferenced: init only does pointer arithmetic
    assert L.fmoe_kv_cache_init(ctypes.byref(c), 1, B, H, D, cap, base, aff) == 0
    assert (c.k_bits, c.v_bits, c.group_size) == (4, 8, 64)
    assert c.k == base and c.k_scales == base + up(rows * D // 2)
    assert c.v == base + up(rows * D // 2) + 2 * up(rows * (D // 64) * 2)
    assert L.fmoe_kv_cache_init(ctypes.byref(c), 1, B, H, D, cap, base, aff - 1) == -3
    assert L.fmoe_kv_cache_init(ctypes.byref(c), 1, B, H, D, cap, base + 8, aff) == -2


def test_kv_entry_points_validate_before_launch(fm):
    import ctypes

    L = fm.lib()
    c = fm.KvCacheC()
    base = 1 << 40
    n = L.fmoe_kv_cache_bytes(1, 1, 8, 256, 64)
    assert L.fmoe_kv_cache_init(ctypes.byref(c), 1, 1, 8, 256, 64, base, n) == 0
    # 3 query heads per kv head is not a compiled configuration
    assert L.fmoe_attn_decode(ctypes.byref(c), base, 24, 10, None, 1.0, base, base, 1 << 20, None) == -5
    # workspace too small
    assert L.fmoe_attn_decode(ctypes.byref(c), base, 16, 10, None, 1.0, base, base, 16, None) == -3
    assert "workspace" in fm.last_error()
    # turbo bits only with the bf16 storage mode
    assert L.fmoe_kv_append(ctypes.byref(c), base, base, 1, 0, None, 3, None) == -1
    assert L.fmoe_turbo_round_trip(base, 4, 256, 5, base, None) == -1
    assert L.fmoe_turbo_round_trip(base, 4, 384, 3, base, None) == -5
