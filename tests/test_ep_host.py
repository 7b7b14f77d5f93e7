"""Host-side EP logic on CPU: the expert / token partitions and the IPC
handle exchange over a 2-rank gloo group."""
from __future__ import annotations

import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PM


def test_expert_range_partitions():
    from paris_moe_b200.ep import expert_range, token_range
    for n, w in [(256, 1), (256, 2), (256, 8), (257, 3), (10, 4)]:
        ranges = [expert_range(n, r, w) for r in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert max(h - l for l, h in ranges) - min(h - l for l, h in ranges) <= 1
        assert token_range(n, 1, w) == expert_range(n, 1, w) if w > 1 else True
    assert expert_range(256, 3, 8) == (96, 128)      # ep.py:78-86 formula


def _worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from paris_moe_b200.ep import exchange_handles
    got = exchange_handles(bytes([rank]) * 64)
    assert [g[0] for g in got] == list(range(world))
    assert all(len(g) == 64 for g in got)
    dist.destroy_process_group()


def test_handle_exchange_gloo():
    mp.spawn(_worker, args=(2, 29611), nprocs=2, join=True)


def test_a2a_plan_sends_each_token_once_per_owning_rank():
    """Token-dispatch plan: a token goes to every rank owning one of its
    experts, once, grouped by destination rank."""
    import torch
    from paris_moe_b200.ep import a2a_plan, expert_owner, expert_range
    E, world = 16, 4
    idx = torch.tensor([[0, 1, 4, 5], [15, 14, 13, 12], [3, 7, 11, 15], [2, 2, 2, 2]])
    owner = expert_owner(idx, E, world)
    for r in range(world):
        lo, hi = expert_range(E, r, world)
        assert torch.equal((owner == r), (idx >= lo) & (idx < hi))
    send, counts = a2a_plan(idx, E, world)
    assert counts.tolist() == [3, 2, 1, 2]
    assert send.tolist() == [0, 2, 3, 0, 2, 2, 1, 2]


def test_prefill_exchange_default_by_world_size():
    """The row exchange below 8 ranks, the partial-sum exchange from 8 on (the
    measured faster one at each size); a communicator exists either way."""
    from paris_moe_b200.ep import EPGroup
    for world, want in ((2, "rows"), (4, "rows"), (8, "partial")):
        g = EPGroup.emulated(256, 2048, 8, 0, world)
        assert g.prefill == want
        assert g.comm_handle != 0
        g.close()
