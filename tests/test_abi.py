"""CPU checks of the C-ABI library: it loads, exports exactly what the header
declares, and rejects bad arguments with status codes (no GPU calls)."""

import ctypes
import os
import re

import pytest

from flashmap_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashmap_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^FM_API [^;(]*?\b(fm_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_header_function():
    lib = _lib.load()
    declared = header_functions()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/flashmap_b200.h but not exported"
    assert sorted(_lib.exported_symbols()) == declared


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.fm_version() >= 1
    assert isinstance(lib.fm_last_error(), bytes)


def test_invalid_arguments_return_status_codes():
    lib = _lib.load()
    st = lib.fm_gemm_bf16(None, None, None, 16, 16, 64, 16, None, None, 0, None, 0, None, None)
    assert st == 1  # FM_ERR_INVALID
    assert b"null" in lib.fm_last_error()
    assert lib.fm_rmsnorm(None, None, None, 1, 1, 1e-6, None) == 1
    assert lib.fm_accept_greedy(None, 0, None, 1, 1, 1, None, None, None, 0, None) == 1
    st = lib.fm_gemm_bf16(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 16, 16, 60, 16, None,
                          None, 0, ctypes.c_void_p(16), 1 << 20, None, None)
    assert st in (2, 3)  # K % 8 != 0 -> shape / alignment error, before any CUDA call


def test_workspace_size_queries_are_pure():
    lib = _lib.load()
    assert lib.fm_gemm_workspace_size(2048, 16, 2048) > 0
    assert lib.fm_cross_attn_workspace_size(1, 16, 128, 19) >= 16 * 19 * (16 * 128 + 32) * 4
    assert lib.fm_accept_workspace_size(64, 16) >= 64 * 17 * 16


def test_plan_validation_without_gpu():
    lib = _lib.load()
    desc = _lib.ModelDesc()
    cfg = _lib.PlanConfig()
    size = ctypes.c_size_t(0)
    desc.hidden, desc.heads, desc.head_dim, desc.block = 2048, 16, 96, 16
    st = lib.fm_plan_workspace_size(ctypes.byref(desc), ctypes.byref(cfg), ctypes.byref(size))
    assert st != 0  # heads * head_dim != hidden


@pytest.mark.parametrize("name", ["fm_check_device"])
def test_device_check_fails_cleanly_without_gpu(name):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert getattr(_lib.load(), name)() != 0
