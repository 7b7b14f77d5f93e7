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
    # + two parity regions of rows, + two of routing slices (idx, w: K each; the gate)
    assert b.value == a.value + 2 * r256(T * (K + 1) * H * 2) + 2 * r256(T * (2 * K + 1) * 4)
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


def test_communicator_host_logic(lib):
    """pmoe_comm_*: registration, the row exchange's epoch (restarted when
    buffers are re-registered), and the capacity refusal, which
    pmoe_block_forward_comm returns before touching any pointer."""
    P = ctypes.c_void_p
    c = P()
    assert lib.pmoe_comm_create(0, 9, ctypes.byref(c)) == -1        # more than 8 ranks
    assert lib.pmoe_comm_create(2, 2, ctypes.byref(c)) == -1
    assert lib.pmoe_comm_create(1, 2, ctypes.byref(c)) == 0
    r, w, et, rt = (ctypes.c_int() for _ in range(4))
    assert lib.pmoe_comm_info(c, *(ctypes.byref(v) for v in (r, w, et, rt))) == 0
    assert (r.value, w.value, et.value, rt.value) == (1, 2, 0, 0)
    bufs = (P * 2)(0x10000, 0x20000)
    assert lib.pmoe_comm_set_ep(c, (P * 2)(0x10000, 0x20008), 4096, 64) == -1  # misaligned
    assert lib.pmoe_comm_set_ep(c, bufs, 4096, 64) == 0
    assert lib.pmoe_comm_set_rows(c, bufs, 1000) == 0
    assert lib.pmoe_comm_info(c, *(ctypes.byref(v) for v in (r, w, et, rt))) == 0
    assert (et.value, rt.value) == (64, 1000)
    e = ctypes.c_int()
    for want in (1, 2, 3):
        assert lib.pmoe_comm_next_rows_epoch(c, ctypes.byref(e)) == 0 and e.value == want
    assert lib.pmoe_comm_set_rows(c, bufs, 1000) == 0                 # fresh buffers
    assert lib.pmoe_comm_next_rows_epoch(c, ctypes.byref(e)) == 0 and e.value == 1
    ws = [None] * 7
    assert lib.pmoe_block_forward_comm(c, None, 1001, 2048, 256, 8, 512, 512, *ws, 3, None,
                                       None, 0, None, None, 0) == -9
    # shared or routed alone cannot use the row exchange
    assert lib.pmoe_block_forward_comm(c, None, 100, 2048, 256, 8, 512, 512, *ws, 1, None,
                                       None, 0, None, None, 0) == -9
    assert b"exchange buffers" in lib.pmoe_status_string(-9)
    assert lib.pmoe_comm_destroy(c) == 0
    assert lib.pmoe_comm_destroy(None) == -1


def test_torch_ops_registered_with_the_boundary_schema():
    """torch.ops.paris_moe.* come from the C++ library, with the ep_rank /
    ep_size / comm_handle keyword arguments; Meta kernels give the shapes;
    CPU tensors raise instead of computing."""
    import torch
    from paris_moe_b200 import ops
    sch = torch.ops.paris_moe.moe_block.default._schema
    kw = [a.name for a in sch.arguments if a.kwarg_only]
    assert kw == ["ep_rank", "ep_size", "comm_handle"]
    assert os.path.basename(ops.OPS_LIB_PATH) == "libparis_moe_torch.so"
    H, E, I, Is, T = 64, 8, 32, 32, 5
    m = dict(device="meta", dtype=torch.bfloat16)
    x = torch.empty(T, H, **m)
    w = (torch.empty(E, H, **m), torch.empty(E, 2 * I, H, **m), torch.empty(E, H, I, **m),
         torch.empty(Is, H, **m), torch.empty(Is, H, **m), torch.empty(H, Is, **m),
         torch.empty(1, H, **m))
    assert ops.moe_block(x, *w, 2, ep_rank=1, ep_size=2).shape == (T, H)
    outs = ops.moe_route(x, w[0], w[6], 2)
    assert [tuple(o.shape) for o in outs] == [(T, 2), (T, 2), (E + 1,), (2 * T,), (2 * T,), (T,)]
    assert [o.dtype for o in outs] == [torch.int32, torch.float32, torch.int32, torch.int32,
                                       torch.int32, torch.float32]
    c = torch.zeros(T, H, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.rmsnorm(c, torch.zeros(H, dtype=torch.bfloat16), 1e-6)


def test_route_slice_flag_only_with_the_row_exchange(lib):
    """PMOE_F_ROUTE_SLICE is refused (before any pointer or device use) by the
    entry points without the fused row exchange."""
    ws = [None] * 7
    assert lib.pmoe_block_forward(None, 64, 2048, 256, 8, 512, 512, *ws, 0, 256, 3 | 16,
                                  None, None, 0, None) == -1
