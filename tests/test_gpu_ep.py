"""Expert parallelism on the GPU: multi-GPU parity (when the box has two or
more GPUs) and the bounded peer wait, which a single GPU can exercise."""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
import time

import pytest
import torch

from conftest import PM, ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ep_two_gpus_matches_single_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={min(torch.cuda.device_count(), 8)}",
           "--master-addr", "127.0.0.1", "--master-port", "29531",
           os.path.join(ROOT, "tests", "ep_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(p.stdout[-4000:], p.stderr[-2000:])
    assert p.returncode == 0
    assert p.stdout.count("EP_OK") == min(torch.cuda.device_count(), 8)


def test_missing_peer_times_out_without_hanging():
    """A 2-rank exchange where rank 1 never runs: rank 0's combine gives up on
    the absent flag after its bounded wait and reports status 4 (peer
    timeout); the GPU context stays usable."""
    from paris_moe_b200 import _lib, workload as W
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(S, seed=1, device="cuda")
    x = W.make_hidden(8, S, seed=1, device="cuda")
    T = x.shape[0]
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_ep_buffer_bytes(T, S.H, S.K, ctypes.byref(nb)) == 0
    bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    arr = (ctypes.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    t0 = time.time()
    st = lib.pmoe_block_forward_ep(x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is,
                                   *[t.data_ptr() for t in wts.tensors()], 0, S.E // 2, 0, T, 3,
                                   arr, nb.value, 0, 2, 1, y.data_ptr(), ws.data_ptr(), n,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    status = ctypes.c_int(-1)
    assert lib.pmoe_read_status(ws.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is,
                                ctypes.byref(status)) == 0
    assert status.value == 4
    assert time.time() - t0 < 60
    # the context still works
    from paris_moe_b200 import ops
    z = ops.moe_block(x, *wts.tensors(), S.K, 0, S.E, 3)
    torch.cuda.synchronize()
    assert torch.isfinite(z.float()).all()


def test_missing_peer_raises_through_epgroup():
    """The same lost peer seen by the product path: EPGroup reads the sticky
    status asynchronously and raises PmoeError(PMOE_ERR_PEER_TIMEOUT) at the
    next call, at check() and at close()."""
    from paris_moe_b200 import _lib, workload as W
    from paris_moe_b200.ep import EPGroup
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(S, seed=1, device="cuda")
    x = W.make_hidden(8, S, seed=1, device="cuda")
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_ep_buffer_bytes(64, S.H, S.K, ctypes.byref(nb)) == 0
    bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    g = EPGroup.emulated(S.E, S.H, S.K, 0, 2, peer_bufs=[b.data_ptr() for b in bufs])
    t0 = time.time()
    g.forward(x, wts.tensors())                # rank 1 never runs: the combine gives up
    with pytest.raises(_lib.PmoeError) as ei:
        g.check()
    assert ei.value.status == _lib.PMOE_ERR_PEER_TIMEOUT
    with pytest.raises(_lib.PmoeError):        # sticky: the next call refuses
        g.forward(x, wts.tensors())
    with pytest.raises(_lib.PmoeError):
        g.close()
    assert time.time() - t0 < 60


@pytest.mark.parametrize("T,flags", [(200, 3), (64, 3), (64, 3 | 4), (200, 2), (200, 1)])
def test_rank_partials_sum_to_full(T, flags):
    """What each of 4 ranks returns without the exchange (its experts, its
    shared-expert tokens) sums to the single-GPU block (the NCCL-comparator
    semantics of ep_forward, engine/runtime/ep.py:97-143)."""
    from oracle import moe_oracle as O
    from paris_moe_b200 import _lib, ops, workload as W
    from paris_moe_b200.ep import expert_range, token_range
    lib = _lib.load()
    S = W.MoEShape()
    wts = W.make_weights(S, seed=5, device="cuda")
    x = W.make_hidden(T, S, seed=7, device="cuda")
    full = ops.moe_block(x, *wts.tensors(), S.K, 0, S.E, flags).float()
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    acc = torch.zeros_like(full)
    for r in range(4):
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        y = torch.empty_like(x)
        lo, hi = expert_range(S.E, r, 4)
        slo, shi = token_range(T, r, 4)
        st = lib.pmoe_block_forward_ep(x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is,
                                       *[t.data_ptr() for t in wts.tensors()], lo, hi, slo, shi,
                                       flags, None, 0, r, 4, 0, y.data_ptr(), ws.data_ptr(), n,
                                       torch.cuda.current_stream().cuda_stream)
        assert st == 0
        acc += y.float()
    torch.cuda.synchronize()
    assert O.rel_l2(acc.cpu().numpy(), full.cpu().numpy()) < 5e-3


@pytest.mark.parametrize("world", [2, 4])
def test_row_split_partials_sum_to_full(world):
    """Row-split EP for prefill-sized batches, its ranks run one after another
    on one GPU: sliced routing equals full routing bit for bit, and the
    ranks' row-share partials sum to the single-GPU block."""
    from oracle import moe_oracle as O
    from paris_moe_b200 import _lib, ops, workload as W
    lib = _lib.load()
    S = W.MoEShape()
    wts = W.make_weights(S, seed=5, device="cuda", zipf_s=1.1)
    T = 1000
    x = W.make_hidden(T, S, seed=8, device="cuda", zipf=True)
    full = ops.moe_block(x, *wts.tensors(), S.K, 0, S.E, 3).float()
    ref_idx, ref_w, *_ = ops.moe_route(x, wts.w_router, wts.w_sh_gvec, S.K)
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    wp = [t.data_ptr() for t in wts.tensors()]
    idx = torch.empty((T, S.K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, S.K), dtype=torch.float32, device="cuda")
    gate = torch.empty((T,), dtype=torch.float32, device="cuda")
    chunk = (T + world - 1) // world
    for r in range(world):
        t0, t1 = min(r * chunk, T), min((r + 1) * chunk, T)
        assert lib.pmoe_route_slice(x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, t0, t1, wp[0],
                                    wp[6], idx.data_ptr(), w.data_ptr(), gate.data_ptr(),
                                    ws.data_ptr(), n, st) == 0
    assert torch.equal(idx.long(), ref_idx.long())
    assert torch.equal(w, ref_w)
    total = torch.zeros_like(full)
    for r in range(world):
        y = torch.empty((T, S.H), dtype=torch.bfloat16, device="cuda")
        assert lib.pmoe_block_forward_rows(x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, *wp,
                                           idx.data_ptr(), w.data_ptr(), gate.data_ptr(), 0,
                                           S.E, r, world, 3, y.data_ptr(), ws.data_ptr(), n,
                                           st) == 0
        total += y.float()
    assert O.rel_l2(total.cpu().numpy(), full.cpu().numpy()) < 5e-3
    # the same split with each rank routing all tokens itself (null routing)
    total2 = torch.zeros_like(full)
    for r in range(world):
        y = torch.empty((T, S.H), dtype=torch.bfloat16, device="cuda")
        assert lib.pmoe_block_forward_rows(x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, *wp,
                                           None, None, None, 0, S.E, r, world, 3, y.data_ptr(),
                                           ws.data_ptr(), n, st) == 0
        total2 += y.float()
    assert torch.equal(total2, total)


def test_rows_fused_missing_peer_times_out():
    """The fused row exchange for 2 ranks where rank 1 never runs: rank 0's
    waits for rank 1's flags give up after their bounded budget and leave
    status 4 (peer timeout) in its buffer; the GPU context stays usable."""
    from paris_moe_b200 import _lib, ops, workload as W
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=128, Is=128)
    wts = W.make_weights(S, seed=2, device="cuda")
    T = 200
    x = W.make_hidden(T, S, seed=2, device="cuda")
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_rows_fused_buffer_bytes(T, S.H, S.K, ctypes.byref(nb)) == 0
    bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    arr = (ctypes.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    t0 = time.time()
    assert lib.pmoe_block_forward_rows_fused(
        x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, *[t.data_ptr() for t in wts.tensors()], 0, 2,
        arr, T, 1, 3, y.data_ptr(), ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream,
        None, 0) == 0
    torch.cuda.synchronize()
    status = ctypes.c_int(-1)
    assert lib.pmoe_rows_status(bufs[0].data_ptr(), ctypes.byref(status)) == 0
    assert status.value == 4
    assert time.time() - t0 < 60
    z = ops.moe_block(x, *wts.tensors(), S.K, 0, S.E, 3)
    torch.cuda.synchronize()
    assert torch.isfinite(z.float()).all()


def test_rows_fused_missing_peer_raises_through_epgroup():
    """Prefill row exchange with rank 1 absent, through EPGroup: rank 0's
    waits give up, its combine, slice push and copy are skipped (y is left
    as it was), and the group raises PMOE_ERR_PEER_TIMEOUT."""
    from paris_moe_b200 import _lib, workload as W
    from paris_moe_b200.ep import EPGroup
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=128, Is=128)
    wts = W.make_weights(S, seed=2, device="cuda")
    T = 200
    x = W.make_hidden(T, S, seed=2, device="cuda")
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_rows_fused_buffer_bytes(T, S.H, S.K, ctypes.byref(nb)) == 0
    bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    g = EPGroup.emulated(S.E, S.H, S.K, 0, 2, rows_bufs=[b.data_ptr() for b in bufs],
                         rows_t_max=T)
    y = torch.full_like(x, 7.0)
    g.forward(x, wts.tensors(), out=y)
    with pytest.raises(_lib.PmoeError) as ei:
        g.check()
    assert ei.value.status == _lib.PMOE_ERR_PEER_TIMEOUT
    assert bool((y == 7.0).all())             # nothing was copied out
    # and no slice was pushed into the absent peer's slice region (epoch 1:
    # parity region 1 after the 1 KiB header); the down GEMM's row stores
    # into its rows region happen before any wait and are expected
    region = (T * S.H * 2 + 255) // 256 * 256
    assert int(bufs[1][1024 + region:1024 + 2 * region].count_nonzero()) == 0
    with pytest.raises(_lib.PmoeError):
        g.close()


@pytest.mark.parametrize("T,slices", [(200, False), (1000, False), (200, True), (1000, True)])
def test_rows_fused_single_rank_matches_block(T, slices):
    """The fused row exchange with world = 1 runs all of its kernels on one GPU
    (down-GEMM stores to the owner's buffer, both flag rounds, the slice
    combine's push, the final copy; with routing slices also the routing push,
    its flag round and the dispatch from the exchanged routing): y equals
    pmoe_block_forward bit for bit, for two calls (both buffer parities)."""
    from paris_moe_b200 import _lib, ops, workload as W
    lib = _lib.load()
    S = W.MoEShape()
    wts = W.make_weights(S, seed=6, device="cuda", zipf_s=1.1)
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_rows_fused_buffer_bytes(T, S.H, S.K, ctypes.byref(nb)) == 0
    buf = torch.zeros(nb.value, dtype=torch.uint8, device="cuda")
    arr = (ctypes.c_void_p * 1)(buf.data_ptr())
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for epoch in (1, 2):
        x = W.make_hidden(T, S, seed=30 + epoch, device="cuda", zipf=True)
        ref = ops.moe_block(x, *wts.tensors(), S.K, 0, S.E, 3)
        y = torch.empty_like(x)
        assert lib.pmoe_block_forward_rows_fused(
            x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, *[t.data_ptr() for t in wts.tensors()],
            0, 1, arr, T, epoch, 3 | (_lib.PMOE_F_ROUTE_SLICE if slices else 0), y.data_ptr(),
            ws.data_ptr(), n, st, None, 0) == 0
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    status = ctypes.c_int(-1)
    assert lib.pmoe_rows_status(buf.data_ptr(), ctypes.byref(status)) == 0
    assert status.value == 0


def test_op_ep_partials_match_c_abi():
    """torch.ops.paris_moe.moe_block(..., ep_rank=r, ep_size=4) without a
    communicator is rank r's partial (its experts, its shared-expert tokens):
    the same bits as pmoe_block_forward_ep with those ranges, and the four
    partials sum to the whole block."""
    from oracle import moe_oracle as O
    from paris_moe_b200 import _lib, ops, workload as W
    from paris_moe_b200.ep import expert_range, token_range
    lib = _lib.load()
    S = W.MoEShape()
    wts = W.make_weights(S, seed=5, device="cuda")
    T = 48
    x = W.make_hidden(T, S, seed=8, device="cuda")
    full = ops.moe_block(x, *wts.tensors(), S.K).float()
    n = _lib.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
    acc = torch.zeros_like(full)
    for r in range(4):
        got = ops.moe_block(x, *wts.tensors(), S.K, ep_rank=r, ep_size=4)
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        want = torch.empty_like(x)
        lo, hi = expert_range(S.E, r, 4)
        slo, shi = token_range(T, r, 4)
        assert lib.pmoe_block_forward_ep(
            x.data_ptr(), T, S.H, S.E, S.K, S.I, S.Is, *[t.data_ptr() for t in wts.tensors()],
            lo, hi, slo, shi, 3, None, 0, r, 4, 0, want.data_ptr(), ws.data_ptr(), n,
            torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        acc += got.float()
    assert O.rel_l2(acc.cpu().numpy(), full.cpu().numpy()) < 5e-3


def test_op_comm_handle_world1_is_the_block():
    """A one-rank communicator: the operator with comm_handle is the block."""
    from paris_moe_b200 import ops, workload as W
    from paris_moe_b200.ep import EPGroup
    S = W.MoEShape()
    wts = W.make_weights(S, seed=3, device="cuda")
    g = EPGroup.emulated(S.E, S.H, S.K, 0, 1)
    for T in (16, 300):
        x = W.make_hidden(T, S, seed=T, device="cuda")
        y = ops.moe_block(x, *wts.tensors(), S.K, ep_rank=0, ep_size=1,
                          comm_handle=g.comm_handle)
        assert torch.equal(y, ops.moe_block(x, *wts.tensors(), S.K))
    g.close()


def test_op_comm_handle_missing_peer_raises():
    """The operator over a communicator whose rank 1 never runs (decode
    exchange, then the row exchange): the bounded waits give up, and the
    group raises PMOE_ERR_PEER_TIMEOUT through the patched module's path
    (EPGroup.op_forward); a batch above the registered buffers is refused by
    the communicator with PMOE_ERR_COMM_CAPACITY."""
    from paris_moe_b200 import _lib, ops, workload as W
    from paris_moe_b200.ep import EPGroup
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=128, Is=128)
    wts = W.make_weights(S, seed=2, device="cuda")
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_ep_buffer_bytes(64, S.H, S.K, ctypes.byref(nb)) == 0
    ep_bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    assert lib.pmoe_rows_fused_buffer_bytes(200, S.H, S.K, ctypes.byref(nb)) == 0
    rx_bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    for T in (8, 200):
        g = EPGroup.emulated(S.E, S.H, S.K, 0, 2, peer_bufs=[b.data_ptr() for b in ep_bufs],
                             rows_bufs=[b.data_ptr() for b in rx_bufs], rows_t_max=200)
        x = W.make_hidden(T, S, seed=T, device="cuda")
        t0 = time.time()
        g.op_forward(x, wts.tensors())
        with pytest.raises(_lib.PmoeError) as ei:
            g.check()
        assert ei.value.status == _lib.PMOE_ERR_PEER_TIMEOUT
        assert time.time() - t0 < 60
        with pytest.raises(RuntimeError, match="status -9"):
            ops.moe_block(W.make_hidden(201, S, seed=1, device="cuda"), *wts.tensors(), S.K,
                          ep_rank=0, ep_size=2, comm_handle=g.comm_handle)
        with pytest.raises(_lib.PmoeError):
            g.close()
        for b in ep_bufs + rx_bufs:
            b.zero_()


def test_capture_after_an_exchange_call_skips_the_status_poll():
    """An exchange call records a status event; capturing the next call in a
    CUDA graph must not query it (CUDA forbids event queries during capture).
    Rank 1 of the emulated group never runs, so the eager call times out and
    the sticky word is raised at check() after the capture.  The graph is
    not replayed."""
    from paris_moe_b200 import _lib, workload as W
    from paris_moe_b200.ep import EPGroup
    lib = _lib.load()
    S = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(S, seed=1, device="cuda")
    x = W.make_hidden(8, S, seed=1, device="cuda")
    nb = ctypes.c_size_t(0)
    assert lib.pmoe_ep_buffer_bytes(64, S.H, S.K, ctypes.byref(nb)) == 0
    bufs = [torch.zeros(nb.value, dtype=torch.uint8, device="cuda") for _ in range(2)]
    g = EPGroup.emulated(S.E, S.H, S.K, 0, 2, peer_bufs=[b.data_ptr() for b in bufs])
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g.op_forward(x, wts.tensors())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        g.op_forward(x, wts.tensors())
    with pytest.raises(_lib.PmoeError) as ei:
        g.check()
    assert ei.value.status == _lib.PMOE_ERR_PEER_TIMEOUT
    del graph
    with pytest.raises(_lib.PmoeError):
        g.close()
