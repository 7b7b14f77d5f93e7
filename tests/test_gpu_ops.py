"""The C++ operator boundary (torch.ops.paris_moe.*) on the GPU: its argument
checks raise before any kernel runs, and the empty batch returns an empty
output."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    from paris_moe_b200 import workload as W
    S = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    return S, W.make_weights(S, seed=4, device="cuda")


def test_empty_batch(small):
    from paris_moe_b200 import ops
    S, w = small
    x = torch.empty((0, S.H), dtype=torch.bfloat16, device="cuda")
    y = ops.moe_block(x, *w.tensors(), S.K)
    assert y.shape == (0, S.H) and y.dtype == torch.bfloat16
    idx, wt, offs, *_ = ops.moe_route(x, w.w_router, w.w_sh_gvec, S.K)
    assert idx.shape == (0, S.K) and int(offs.abs().sum()) == 0


def test_bad_arguments_raise(small):
    from paris_moe_b200 import ops, workload as W
    S, w = small
    t = w.tensors()
    x = W.make_hidden(8, S, seed=1, device="cuda")
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.moe_block(torch.cat([x, x], 1)[:, ::2], *t, S.K)
    with pytest.raises(RuntimeError, match="bf16"):
        ops.moe_block(x.float(), *t, S.K)
    with pytest.raises(RuntimeError, match="weight shapes"):
        ops.moe_block(x, t[0], t[1][:, :64].contiguous(), *t[2:], S.K)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.moe_block(x, t[0].cpu(), *t[1:], S.K)
    with pytest.raises(RuntimeError, match="ep_rank"):
        ops.moe_block(x, *t, S.K, ep_rank=2, ep_size=2)


def test_comm_handle_must_match_ep_arguments(small):
    from paris_moe_b200 import ops, workload as W
    from paris_moe_b200.ep import EPGroup
    S, w = small
    g = EPGroup.emulated(S.E, S.H, S.K, 0, 1)
    x = W.make_hidden(8, S, seed=2, device="cuda")
    with pytest.raises(RuntimeError, match="differ from the communicator"):
        ops.moe_block(x, *w.tensors(), S.K, ep_rank=0, ep_size=2, comm_handle=g.comm_handle)
    with pytest.raises(RuntimeError, match="expert range"):
        ops.moe_block(x, *w.tensors(), S.K, 0, 4, ep_rank=0, ep_size=1, comm_handle=g.comm_handle)
    g.close()
