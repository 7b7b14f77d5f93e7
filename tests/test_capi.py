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
