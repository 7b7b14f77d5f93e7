"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as O

# Output tolerance of the north-star spec, against the fp32-accumulate oracle.
REL_L2_TOL = 5e-3
MAX_ABS_TOL = 3e-2


def bits(t):
    return O.torch_bf16_bits(t)


def weight_bits(wts):
    return [bits(getattr(wts, n)) for n in wts.shape.weight_names()]


def oracle_y(x, wts, route=None, expert_range=None, with_shared=True, rows=None):
    """fp32 oracle output for rows `rows` of x (all when None), optionally
    with a given routing (idx, w) restricted to the same rows."""
    xb = bits(x)
    if rows is not None:
        xb = xb[rows]
        if route is not None:
            route = (route[0][rows], route[1][rows])
    y, idx, w = O.moe_block(xb, *weight_bits(wts), k=wts.shape.K, route=route,
                            expert_range=expert_range, with_shared=with_shared)
    return y


def assert_close(y_gpu, y_ref, what=""):
    y = y_gpu.float().cpu().numpy() if isinstance(y_gpu, torch.Tensor) else y_gpu
    r, m = O.rel_l2(y, y_ref), O.max_abs(y, y_ref)
    assert r <= REL_L2_TOL and m <= MAX_ABS_TOL, f"{what}: rel_l2={r:.3e} max_abs={m:.3e}"
    return r, m


def exact_logits(x, w_router):
    """float64 router logits (products exact, sum within ~1e-12 of the exact value)."""
    return O.bf16_to_f32(bits(x)).astype(np.float64) @ O.bf16_to_f32(bits(w_router)).astype(np.float64).T
