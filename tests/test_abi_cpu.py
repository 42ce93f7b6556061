"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/dmoe_b200.h declares (no compute calls)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dmoe_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dmoe_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = _declared()
    for required in ["dmoe_router", "dmoe_route_plan", "dmoe_permute_rows", "dmoe_grouped_gated_mlp",
                     "dmoe_combine", "dmoe_ipc_export", "dmoe_ipc_open", "dmoe_ipc_close", "dmoe_flag_signal",
                     "dmoe_flag_wait", "dmoe_last_error"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    # the Python binding covers the whole header
    assert set(_declared()) <= set(N.SIGNATURES)


def test_pure_host_entry_points():
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    assert b"sm_100a" in lib.dmoe_version()
    assert lib.dmoe_route_plan_workspace_size(4096, 2, 8) == 4 * 8 * 4
    assert lib.dmoe_grouped_mlp_workspace_size(8192, 14336, 2) >= 8192 * 14336 * 2


def test_argument_validation_without_gpu():
    """Validation runs before any CUDA call, so it works here."""
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    rc = lib.dmoe_router(None, None, 2, None, None, None, 16, 64, 300, 2, 0, 0, 1.0, 1, 1, None, None, None, 2, None)
    assert rc == 1 and b"E <=" in lib.dmoe_last_error()
    rc = lib.dmoe_grouped_gated_mlp(None, None, None, None, 8, 100, 64, 2, None, None, 1, 0, 10, 0, None, None, 0,
                                    None, None)
    assert rc == 1


def test_more_argument_checks_without_gpu():
    """Every entry point rejects malformed requests with DMOE_ERR_INVALID and a message
    before touching the GPU."""
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    # tensor-core router logits: d and E must be multiples of 8
    assert lib.dmoe_router_logits(None, None, 2, 16, 100, 256, None, None, None) == 1
    assert b"multiples of 8" in lib.dmoe_last_error()
    assert lib.dmoe_router_logits(None, None, 0, 16, 128, 256, None, None, None) == 1  # fp32 inputs
    # SM reserve range, then back to 0
    assert lib.dmoe_grouped_mlp_set_sm_reserve(65) == 1
    assert lib.dmoe_grouped_mlp_set_sm_reserve(-1) == 1
    assert lib.dmoe_grouped_mlp_set_sm_reserve(0) == 0
    # combine: k above the kernel's bound
    assert lib.dmoe_combine(None, None, None, 2, 8, 17, 64, 2, 0, None, None) == 1
    # gather: more segments than one launch takes
    assert lib.dmoe_permute_rows(None, None, 64, None, None, None, None, 5000, None) == 1
    # completion flag: misaligned flag and an out-of-range timeout
    assert lib.dmoe_flag_signal(ctypes.c_void_p(12), 1, None) == 1
    assert lib.dmoe_flag_wait(ctypes.c_void_p(16), 1, 0, None, None) == 1
    assert lib.dmoe_flag_wait(ctypes.c_void_p(16), 1, 61 * 10**9, None, None) == 1
    # router: bad mode and a group split that cannot hold k experts
    assert lib.dmoe_router(None, None, 2, None, None, None, 16, 64, 8, 2, 7, 0, 1.0, 1, 1, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), 2, None) == 1
    assert lib.dmoe_router(None, None, 2, None, None, None, 16, 64, 8, 4, 1, 0, 1.0, 4, 1, None,
                           ctypes.c_void_p(16), ctypes.c_void_p(16), 2, None) == 1


def test_fp8_argument_checks_without_gpu():
    """The 8-bit entry points reject rows that TMA cannot tile and bad arguments before any
    CUDA call."""
    from distributedmoe_b200 import _native as N
    lib = N.lib()
    p16 = ctypes.c_void_p(16)
    # quantisation: cols a multiple of 16 (16-byte e4m3 rows), dtype f32/f16/bf16, strides
    assert lib.dmoe_quantize_rows_e4m3(p16, 2, 4, 24, p16, 32, p16, 1, None) == 1
    assert b"multiple of 16" in lib.dmoe_last_error()
    assert lib.dmoe_quantize_rows_e4m3(p16, 3, 4, 32, p16, 32, p16, 1, None) == 1
    assert lib.dmoe_quantize_rows_e4m3(p16, 2, 4, 32, p16, 40, p16, 1, None) == 1  # q_ld not a multiple of 16
    assert lib.dmoe_quantize_rows_e4m3(p16, 2, 4, 32, p16, 32, p16, 0, None) == 1  # scale_ld < 1
    assert lib.dmoe_quantize_rows_e4m3(None, 2, 0, 32, None, 32, None, 1, None) == 0  # nothing to do
    # grouped MLP: d a multiple of 16, activation, tile policy, then the pointers
    args = [None] * 7 + [4, 200, 128, None, None, 1, 0, 64, 1, None, None, 0, None, 0, None]
    assert lib.dmoe_grouped_gated_mlp_fp8(*args) == 1 and b"multiple of 16" in lib.dmoe_last_error()
    args[8] = 256
    args[15] = 9
    assert lib.dmoe_grouped_gated_mlp_fp8(*args) == 1 and b"activation" in lib.dmoe_last_error()
    args[15] = 1
    args[20] = 7
    assert lib.dmoe_grouped_gated_mlp_fp8(*args) == 1 and b"tile policy" in lib.dmoe_last_error()
    args[20] = 0
    assert lib.dmoe_grouped_gated_mlp_fp8(*args) == 1 and b"null pointer" in lib.dmoe_last_error()
    # exchange expert step: d a multiple of 16, then the window table
    assert lib.dmoe_ep_expert_mlp_fp8(None, None, None, None, None, None, 4, 200, 128, None, None, 1, 64, 1, None, 0,
                                      None, 0, None) == 1
    assert b"multiple of 16" in lib.dmoe_last_error()
    assert lib.dmoe_ep_expert_mlp_fp8(None, None, None, None, None, None, 4, 256, 128, None, None, 1, 64, 1, None, 0,
                                      None, 0, None) == 1
    assert b"window" in lib.dmoe_last_error()

def test_no_cpu_fallback_in_product():
    """The product never imports the oracle."""
    pkg = os.path.join(ROOT, "distributedmoe_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", src, flags=re.M), f
