"""The no-allocation entry point, pmoe_block_forward_noalloc.

It exists for callers that cannot allocate device memory when they call the
MoE block -- a serving engine that has reserved all of HBM in advance and
allows no allocation on its decode path, or a foreign-language host calling
the C ABI with no device allocator -- so it takes no workspace and uses a
fixed scratch array inside the library instead.  These tests call it through
the C ABI and check it against pmoe_block_forward, which gets a workspace
from the caller.  The file name sorts last so a run that stops at the first
failure has run every other test already; it also passes on its own.
"""
from __future__ import annotations

import pytest
import torch

from conftest import PM

pytestmark = pytest.mark.gpu


def _args(x, wts, flags=3):
    S = wts.shape
    return (x.data_ptr(), x.shape[0], S.H, S.E, S.K, S.I, S.Is,
            *[t.data_ptr() for t in wts.tensors()], 0, S.E, flags)


def _with_workspace(lib, x, wts, stream):
    from paris_moe_b200 import _lib
    S = wts.shape
    n = _lib.workspace_size(x.shape[0], S.H, S.E, S.K, S.I, S.Is)
    ws = torch.empty(n, dtype=torch.uint8, device=x.device)
    y = torch.empty_like(x)
    _lib.check("pmoe_block_forward",
               lib.pmoe_block_forward(*_args(x, wts), y.data_ptr(), ws.data_ptr(), n, stream))
    return y


def _noalloc(lib, x, wts, stream):
    from paris_moe_b200 import _lib
    y = torch.empty_like(x)
    _lib.check("pmoe_block_forward_noalloc",
               lib.pmoe_block_forward_noalloc(*_args(x, wts), y.data_ptr(), stream))
    return y


@pytest.mark.parametrize("T", [64, 5])
def test_noalloc_matches_workspace_entry_twice(T):
    from paris_moe_b200 import _lib, workload as W
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wts = W.make_weights(W.MoEShape(), seed=3, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    x1 = W.make_hidden(T, W.MoEShape(), seed=3, device=dev)
    x2 = W.make_hidden(T, W.MoEShape(), seed=4, device=dev)
    for x in (x1, x2):      # two calls in a row, different inputs
        want = _with_workspace(lib, x, wts, stream)
        got = _noalloc(lib, x, wts, stream)
        torch.cuda.synchronize()
        # the same kernels on the same inputs, deterministic: bit for bit
        # (a tolerance would let stale scratch contents slip through)
        assert torch.equal(got, want), f"noalloc T={T}"


def test_noalloc_rejects_oversized_shape():
    from paris_moe_b200 import _lib, workload as W
    lib = _lib.load()
    S = W.MoEShape()
    assert lib.pmoe_noalloc_scratch_bytes() >= _lib.workspace_size(64, S.H, S.E, S.K, S.I, S.Is)
    assert _lib.workspace_size(4096, S.H, S.E, S.K, S.I, S.Is) > lib.pmoe_noalloc_scratch_bytes()
    null = None
    st = lib.pmoe_block_forward_noalloc(null, 4096, S.H, S.E, S.K, S.I, S.Is, *([null] * 7),
                                        0, S.E, 3, null, null)
    assert st == -8
    assert b"scratch" in lib.pmoe_status_string(st)
