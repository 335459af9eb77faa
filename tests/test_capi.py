"""The C-ABI library loads without a GPU and exports every declared symbol."""

import ctypes
import os
import re
import subprocess

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "splat200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(splat_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "splat_render_forward" in names and "splat_bin_emit" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    from dsl_splat_b200 import _native

    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (splat_\w+)", out))
    assert set(declared_functions()) <= exported


def test_python_binding_covers_header():
    from dsl_splat_b200 import _native

    assert set(declared_functions()) == set(_native.SIGNATURES)
    assert _native.lib.splat_abi_version() == 1


def test_workspace_queries_without_gpu():
    from dsl_splat_b200._native import lib

    small = lib.splat_bin_workspace_bytes(10, 256, 256, 0)
    big = lib.splat_bin_workspace_bytes(1_000_000, 1920, 1080, 0)
    assert 0 < small < big
    # tile grids that fit the chunked scatter need no pair workspace; the
    # onesweep fallback (65,536 tiles here) sorts 8-byte pairs, and accutile
    # (mode 2) materialises its pairs plus a ping-pong copy
    assert lib.splat_bin_pairs_workspace_bytes(8_800_000, 1920, 1080, 0) == 0
    assert lib.splat_bin_pairs_workspace_bytes(8_800_000, 1920, 1080, 1) == 0
    assert lib.splat_bin_pairs_workspace_bytes(8_800_000, 4096, 4096, 0) >= 8 * 8_800_000
    assert lib.splat_bin_pairs_workspace_bytes(8_800_000, 1920, 1080, 2) >= 16 * 8_800_000
    assert lib.splat_scan_workspace_bytes(1_000_000) > 0


def test_invalid_arguments_fail_before_any_launch():
    from dsl_splat_b200._native import lib

    assert lib.splat_render_forward(0, 10, None, None, 0, 0, None, None, None, 3, 3, None, 0, 0,
                                    1, None, None, 4, 1, None, None, None, None, None) == -1
    assert b"bad render sizes" in lib.splat_last_error()
    assert lib.splat_bin_emit(10, 1 << 31, 64, 64, 0, None, None, None, None, 0, None, 0, None,
                              None) == -4
    assert lib.splat_bin_prepare(10, None, None, None, None, None, 64, 64, 0, None, 0, None, None,
                                 None) == -5
    # tile modes: unknown mode, and snugbox/accutile without conics
    assert lib.splat_bin_prepare(10, None, None, None, None, None, 64, 64, 3, None, 0, None, None,
                                 None) == -1
    assert lib.splat_bin_prepare(10, None, None, None, None, None, 64, 64, 1, None, 0, None, None,
                                 None) == -1
    assert b"require projected conics" in lib.splat_last_error()
