"""The drop-in as the reference's engine uses it, on the GPU: a full-shape HF
Qwen3_5MoeSparseMoeBlock on CUDA with ``patch_qwen3_5_moe`` installed (the
reference installs its patch from load_model, engine/model/qwen3_next.py:117-126,
via engine/kernels/patch.py:43-84), its CUDA-graph capture at the decode
buckets of engine/runtime/cuda_graphs.py:142, and the tensor-parallel shared
expert of engine/model/tp_shard.py."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PM
from gpu_util import assert_close, bits, oracle_y
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

BUCKETS = [1, 2, 4, 8, 16, 32, 64]   # engine/runtime/cuda_graphs.py:142


def hf_block(wts, device="cuda"):
    """The HF module of the full shape holding ``wts`` (bf16, eval mode)."""
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    S = wts.shape
    cfg = Qwen3_5MoeTextConfig(hidden_size=S.H, num_experts=S.E, num_experts_per_tok=S.K,
                               moe_intermediate_size=S.I, shared_expert_intermediate_size=S.Is)
    cfg._experts_implementation = "eager"     # HF's per-expert loop: runs on any GPU
    with torch.device("meta"):
        blk = M.Qwen3_5MoeSparseMoeBlock(cfg)
    blk = blk.to_empty(device=device).to(torch.bfloat16).eval()
    with torch.no_grad():
        blk.gate.weight.copy_(wts.w_router)
        blk.experts.gate_up_proj.copy_(wts.w_gate_up)
        blk.experts.down_proj.copy_(wts.w_down)
        blk.shared_expert.gate_proj.weight.copy_(wts.w_sh_gate)
        blk.shared_expert.up_proj.weight.copy_(wts.w_sh_up)
        blk.shared_expert.down_proj.weight.copy_(wts.w_sh_down)
        blk.shared_expert_gate.weight.copy_(wts.w_sh_gvec)
    return blk


@pytest.fixture(scope="module")
def setup():
    from paris_moe_b200 import workload as W
    wts = W.make_weights(W.MoEShape(), seed=0)
    return wts, hf_block(wts)


@pytest.mark.parametrize("B,S", [(1, 1), (2, 20), (1, 300)])
def test_patched_hf_module_matches_oracle_and_hf(setup, B, S):
    from paris_moe_b200 import moe, workload as W
    wts, blk = setup
    x = W.make_hidden(B * S, wts.shape, seed=B * 1000 + S)
    x3 = x.view(B, S, -1).cuda()
    with torch.inference_mode():
        want_hf = blk(x3)
        if isinstance(want_hf, tuple):
            want_hf = want_hf[0]
        try:
            assert moe.patch_qwen3_5_moe()
            got = blk(x3)
        finally:
            moe.unpatch_qwen3_5_moe()
    assert isinstance(got, torch.Tensor) and got.shape == x3.shape and got.dtype == torch.bfloat16
    ref = oracle_y(x, wts)                 # the oracle's own routing
    assert_close(got.reshape(B * S, -1), ref, f"patched B={B} S={S}")
    # HF's own CUDA path rounds every intermediate to bf16 (rel-L2 ~5e-3 vs fp32)
    hf = want_hf.reshape(B * S, -1).float().cpu().numpy()
    assert O.rel_l2(got.reshape(B * S, -1).float().cpu().numpy(), hf) <= 1e-2


def test_patched_hf_module_cuda_graph_buckets(setup):
    """Capture the patched module at every decode bucket and replay with new
    inputs: bit-identical to eager calls."""
    from paris_moe_b200 import moe, workload as W
    wts, blk = setup
    try:
        assert moe.patch_qwen3_5_moe()
        with torch.inference_mode():
            for B in BUCKETS:
                xs = W.make_hidden(B, wts.shape, seed=50 + B).view(B, 1, -1).cuda()
                static = xs.clone()
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    for _ in range(2):
                        blk(static)
                torch.cuda.current_stream().wait_stream(side)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    out = blk(static)
                for seed in (1, 2):
                    xn = W.make_hidden(B, wts.shape, seed=900 + 10 * B + seed).view(B, 1, -1)
                    static.copy_(xn.cuda())
                    g.replay()
                    torch.cuda.synchronize()
                    eager = blk(xn.cuda())
                    assert torch.equal(out, eager), f"bucket {B}"
                del g
    finally:
        moe.unpatch_qwen3_5_moe()


# ---- tensor-parallel shared expert ------------------------------------------

def test_tp_shared_shards_sum_to_full():
    """Each TP rank's shared-expert shard (Is/2 rows of gate/up, Is/2 columns of
    down), run one after another on one GPU and summed with the routed experts,
    equals the unsharded block (the RowParallel sum of tp_shard.py:95-100)."""
    from paris_moe_b200 import ops, workload as W
    S = W.MoEShape()
    wts = W.make_weights(S, seed=9)
    g = wts.to("cuda")
    x = W.make_hidden(32, S, seed=9)
    xg = x.cuda()
    y = ops.moe_block(xg, *g.tensors(), S.K, 0, S.E, 2).float()       # routed only
    h = S.Is // 2
    for r in range(2):
        t = list(g.tensors())
        t[3] = g.w_sh_gate[r * h:(r + 1) * h].contiguous()
        t[4] = g.w_sh_up[r * h:(r + 1) * h].contiguous()
        t[5] = g.w_sh_down[:, r * h:(r + 1) * h].contiguous()
        y += ops.moe_block(xg, *t, S.K, 0, S.E, 1).float()              # shared shard r
    assert_close(y, oracle_y(x, wts), "routed + sum of shared shards")


class _Shard(torch.nn.Module):
    """Attribute contract of tp_shard's Column/RowParallelLinear (tp_shard.py:25-100)."""

    def __init__(self, lin, tp, rank, dim):
        super().__init__()
        n = lin.weight.shape[dim] // tp
        self.weight = torch.nn.Parameter(
            lin.weight.data.narrow(dim, rank * n, n).contiguous().clone(), requires_grad=False)
        self.bias = None
        self.tp_size, self.tp_rank = tp, rank


def _tp_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from paris_moe_b200 import moe, workload as W
        wts = W.make_weights(W.MoEShape(), seed=0)
        blk = hf_block(wts)
        se = blk.shared_expert
        se.gate_proj = _Shard(se.gate_proj, world, rank, 0)
        se.up_proj = _Shard(se.up_proj, world, rank, 0)
        se.down_proj = _Shard(se.down_proj, world, rank, 1)
        x = W.make_hidden(24, wts.shape, seed=4).view(2, 12, -1).cuda()
        try:
            moe.patch_qwen3_5_moe()
            with torch.inference_mode():
                y = blk(x)
        finally:
            moe.unpatch_qwen3_5_moe()
        torch.save(y.cpu(), os.path.join(out_dir, f"y{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_tp_sharded_shared_expert_drop_in(tmp_path):
    """Two TP ranks (processes, gloo for the host collective, both on cuda:0)
    with the shared expert sharded as tp_shard._replace_mlp does: the patched
    module returns the full block on every rank, never a partial."""
    from paris_moe_b200 import workload as W
    mp.spawn(_tp_worker, args=(2, 29641, str(tmp_path)), nprocs=2, join=True)
    y0 = torch.load(tmp_path / "y0.pt")
    y1 = torch.load(tmp_path / "y1.pt")
    assert torch.equal(y0, y1)
    wts = W.make_weights(W.MoEShape(), seed=0)
    x = W.make_hidden(24, wts.shape, seed=4)
    assert_close(y0.reshape(24, -1), oracle_y(x, wts), "TP=2 drop-in")
