"""The PyTorch operators ``torch.ops.paris_moe.*``, registered in C++
(csrc/torch_ops.cpp, built into libparis_moe_torch.so) over the C ABI.

    moe_block(x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec,
              top_k=8, expert_lo=0, expert_hi=-1, flags=3, *, ep_rank=0, ep_size=1,
              comm_handle=0) -> y
    moe_route(x, w_router, w_sh_gvec, k) -> (topk_idx, topk_w, offsets, sorted_tok,
                                            sorted_slot, shared_gate)
    moe_layer(x, w_norm, eps, <7 weights>, top_k=8, flags=3) -> y
    rmsnorm(x, w_norm, eps) -> y

The ops run on the current CUDA stream, allocate their outputs and workspace
through PyTorch's caching allocator, never synchronise the host, and have
Meta kernels, so they can be captured in CUDA graphs at fixed T.  The CPU
kernels only raise (no fallback), a missing library raises at
import, and a kernel status other than 0 raises RuntimeError naming it.
``comm_handle`` is an ``EPGroup.comm_handle`` (pmoe_comm_create).
"""
from __future__ import annotations

import os

import torch

from . import _lib

OPS_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libparis_moe_torch.so")


if not os.path.exists(OPS_LIB_PATH):
    raise RuntimeError(
        f"{OPS_LIB_PATH} is missing: build it with `python "
        f"{os.path.dirname(OPS_LIB_PATH)}/build.py` (no CPU or Python fallback)")
_lib.load()  # the C ABI first, so the operator library's dependency resolves to it
torch.ops.load_library(OPS_LIB_PATH)

moe_block = torch.ops.paris_moe.moe_block
moe_route = torch.ops.paris_moe.moe_route
moe_layer = torch.ops.paris_moe.moe_layer
rmsnorm = torch.ops.paris_moe.rmsnorm
