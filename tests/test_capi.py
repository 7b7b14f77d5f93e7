"""CPU checks of the C ABI: the library builds, loads, exports every symbol
include/paris_moe.h declares, and its host-only entry points behave (no GPU
compute is called here)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import PM, ROOT

HEADER = os.path.join(ROOT, "include", "paris_moe.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pmoe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from paris_moe_b200 import build, _lib
    build.build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert "pmoe_block_forward" in names and "pmoe_route" in names
    for n in names:
        assert hasattr(lib, n), n
    from paris_moe_b200 import _lib
    assert set(names) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"


def test_version_and_status_strings(lib):
    assert lib.pmoe_version().decode().startswith("paris_moe")
    assert lib.pmoe_status_string(0) == b"ok"
    assert b"workspace" in lib.pmoe_status_string(-3)
    assert lib.pmoe_status_string(12345) == b"unknown status"


def test_workspace_size_contract(lib):
    from paris_moe_b200 import _lib
    a = _lib.workspace_size(64, 2048, 256, 8, 512, 512)
    b = _lib.workspace_size(8192, 2048, 256, 8, 512, 512)
    assert 0 < a < b
    assert a % 256 == 0
    assert _lib.workspace_size(0, 2048, 256, 8, 512, 512) > 0
    with pytest.raises(_lib.PmoeError):
        _lib.workspace_size(4, 2048, 512, 8, 512, 512)    # E > 256 unsupported
    with pytest.raises(_lib.PmoeError):
        _lib.workspace_size(4, 2000, 256, 8, 512, 512)    # H % 128 != 0
    with pytest.raises(_lib.PmoeError):
        _lib.workspace_size(4, 2048, 8, 9, 512, 512)      # K > E
    out = ctypes.c_size_t(0)
    assert lib.pmoe_workspace_size(-1, 2048, 256, 8, 512, 512, ctypes.byref(out)) == -1


def test_forward_rejects_bad_args_before_touching_gpu(lib):
    # Argument validation runs before any CUDA call, so this is safe on CPU.
    null = None
    st = lib.pmoe_block_forward(null, 4, 2048, 256, 8, 512, 512, *([null] * 7), 0, 256, 3,
                                null, null, 0, null)
    assert st == -1
    st = lib.pmoe_block_forward(null, 4, 2048, 256, 8, 512, 512, *([null] * 7), 10, 5, 3,
                                null, null, 0, null)
    assert st == -1
    st = lib.pmoe_block_forward(null, 0, 2048, 256, 8, 512, 512, *([null] * 7), 0, 256, 3,
                                null, null, 0, null)
    assert st == 0        # T == 0 is a no-op
    st = lib.pmoe_block_forward(null, 4, 2048, 256, 8, 512, 512, *([null] * 7), 0, 256, 64,
                                null, null, 0, null)
    assert st == -1       # unknown flag


def test_rows_fused_buffer_layout(lib):
    """The fused row-exchange buffer is the partial-sum buffer (header + two
    T_max x H bf16 slice regions) followed by two regions of T_max*(K+1) rows."""
    def r256(n):
        return (n + 255) // 256 * 256
    T, H, K = 8192, 2048, 8
    a, b = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.pmoe_rows_buffer_bytes(T, H, ctypes.byref(a)) == 0
    assert lib.pmoe_rows_fused_buffer_bytes(T, H, K, ctypes.byref(b)) == 0
    assert a.value == 1024 + 2 * r256(T * H * 2)
    assert b.value == a.value + 2 * r256(T * (K + 1) * H * 2)
    assert lib.pmoe_rows_fused_buffer_bytes(T, H, 0, ctypes.byref(b)) == -1
    assert lib.pmoe_rows_fused_buffer_bytes(T, 2047, K, ctypes.byref(b)) == -1
    assert lib.pmoe_rows_fused_buffer_bytes(0, H, K, ctypes.byref(b)) == -1


def test_rows_fused_rejects_bad_args_before_touching_gpu(lib):
    null = None
    fake = (ctypes.c_void_p * 2)(0x10000, 0x20000)   # never dereferenced: checks fail first

    def call(bufs=fake, rank=0, world=2, T=4, T_max=4, epoch=1, flags=3, x=null):
        return lib.pmoe_block_forward_rows_fused(
            x, T, 2048, 256, 8, 512, 512, *([null] * 7), rank, world, bufs, T_max, epoch, flags,
            null, null, 0, null, null, 0)
    assert call(bufs=None) == -1
    assert call(rank=2) == -1
    assert call(world=9) == -1
    assert call(epoch=0) == -1
    assert call(T=8, T_max=4) == -1
    assert call(flags=2) == -1          # the slice combine needs routed and shared rows
    assert call() == -1                 # null x / weights / y / workspace
    assert call(T=0) == 0               # empty batch: no-op
