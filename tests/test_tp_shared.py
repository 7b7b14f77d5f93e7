"""The drop-in under the reference's tensor-parallel shared expert, on CPU.

engine/model/tp_shard.py:_replace_mlp (tp_shard.py:144-159) replaces a
block's shared_expert gate/up with column shards and down with a row shard
whose forward all-reduces (tp_shard.py:95-100).  The block op must see the
whole shared expert: ``moe.shared_weights`` assembles it from the shards of
every rank (2 gloo ranks here) and refuses shapes it cannot handle."""
from __future__ import annotations

import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PM
from test_host_logic import tiny_block

REF = "/root/reference"


class _Shard(torch.nn.Module):
    """Stand-in with the attribute contract of tp_shard's ColumnParallelLinear
    (dim 0: output rows) / RowParallelLinear (dim 1: input columns)."""

    def __init__(self, lin, tp, rank, dim):
        super().__init__()
        n = lin.weight.shape[dim] // tp
        w = lin.weight.data.narrow(dim, rank * n, n).contiguous().clone()
        self.weight = torch.nn.Parameter(w, requires_grad=False)
        self.bias = None
        self.tp_size, self.tp_rank = tp, rank


def shard_shared(se, tp, rank, use_reference):
    if use_reference:
        sys.path.insert(0, REF)
        from engine.model import tp_shard
        assert tp_shard._replace_mlp(se, tp, rank)
        return
    se.gate_proj = _Shard(se.gate_proj, tp, rank, 0)
    se.up_proj = _Shard(se.up_proj, tp, rank, 0)
    se.down_proj = _Shard(se.down_proj, tp, rank, 1)


def _worker(rank, world, port, use_reference):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from paris_moe_b200 import moe
        _, blk = tiny_block()                   # seeded: identical on both ranks
        se = blk.shared_expert
        full = [se.gate_proj.weight.detach().clone(), se.up_proj.weight.detach().clone(),
                se.down_proj.weight.detach().clone()]
        shard_shared(se, world, rank, use_reference)
        assert se.gate_proj.weight.shape[0] == full[0].shape[0] // world
        got = moe.shared_weights(blk)
        for a, b in zip(got, full):
            assert torch.equal(a, b)
        again = moe.shared_weights(blk)         # cached: no second collective
        assert all(a is b for a, b in zip(got, again))
        ws = moe.block_weights(blk)
        assert all(a is b for a, b in zip(ws[3:6], got))
        assert ws[0] is blk.gate.weight and ws[1] is blk.experts.gate_up_proj
        # a shard that changes in place invalidates the cache
        with torch.no_grad():
            se.up_proj.weight.add_(1)
        upd = moe.shared_weights(blk)
        assert upd[1] is not got[1]
        # a TP degree other than the group's cannot be assembled: raise
        se.down_proj.tp_size = se.gate_proj.tp_size = se.up_proj.tp_size = 4
        with pytest.raises(RuntimeError, match="TP-sharded 4 ways"):
            moe.shared_weights(blk)
        se.down_proj.tp_size = world
        with pytest.raises(ValueError, match="different TP degrees"):
            moe.shared_weights(blk)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("use_reference", [False, True])
def test_tp_shared_expert_assembled_gloo(use_reference):
    if use_reference and not os.path.isdir(os.path.join(REF, "engine", "model")):
        pytest.skip("reference checkout not present")
    mp.spawn(_worker, args=(2, 29621 + int(use_reference), use_reference), nprocs=2, join=True)


def test_tp_shard_without_group_raises():
    """A sharded shared expert with no process group: raise, never compute a
    partial."""
    from paris_moe_b200 import moe
    _, blk = tiny_block()
    shard_shared(blk.shared_expert, 2, 0, False)
    with pytest.raises(RuntimeError, match="cannot assemble"):
        moe.block_weights(blk)


def test_block_weights_shape_mismatch_raises():
    from paris_moe_b200 import moe
    _, blk = tiny_block()
    se = blk.shared_expert
    se.down_proj.weight = torch.nn.Parameter(se.down_proj.weight.data[:, :16].clone())
    with pytest.raises(ValueError, match="shared_expert.down_proj"):
        moe.block_weights(blk)
