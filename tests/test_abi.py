"""CPU: the C-ABI library loads and exports exactly what include/lisa_attn.h
declares (no compute calls: there is no GPU here)."""
import ctypes
import os
import re
import subprocess

import lisa_attn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lisa_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lisa_attn_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "lisa_attn_decode" in names and "lisa_attn_prefill_chunk" in names
    assert "lisa_attn_commit_verified_prefix" in names and "lisa_attn_trim_state" in names


def test_library_exports_every_declared_symbol():
    lib = lisa_attn.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", lisa_attn.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(lisa_attn_\w+)\b", out))
    assert exported == set(declared_functions())


def test_python_bindings_cover_header():
    assert set(lisa_attn.SIGNATURES) == set(declared_functions())


def test_cpu_safe_calls():
    lib = lisa_attn.load_library()
    assert b"sm_100a" in lib.lisa_attn_build_info()
    assert lib.lisa_attn_window_workspace_bytes(0, 1) == 0
    assert lib.lisa_attn_window_workspace_bytes(1024, 4) == 0
    # at least one chunk's per-(kv head) O partials, growing with the window and rows
    one = lib.lisa_attn_window_workspace_bytes(1024, 1)
    assert one >= 4 * 2048 * 4
    assert lib.lisa_attn_window_workspace_bytes(65536, 1) > one
    assert lib.lisa_attn_window_workspace_bytes(1024, 3) > one
    # null contexts are rejected before any CUDA call
    assert lib.lisa_attn_destroy(None) == lisa_attn.EINVAL
    assert lib.lisa_attn_commit_verified_prefix(None, 1) == lisa_attn.EINVAL
    assert lib.lisa_attn_position(None) == 0
    assert lib.lisa_attn_merge_windows(0, 1, None, None, 0, None, None, None) == lisa_attn.EINVAL
    h = ctypes.c_void_p()
    assert lib.lisa_attn_create(0, 0, 16, ctypes.byref(h)) == lisa_attn.EINVAL
    assert lib.lisa_attn_create(0, 1, 0, ctypes.byref(h)) == lisa_attn.EINVAL

