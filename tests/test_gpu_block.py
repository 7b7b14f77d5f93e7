"""GPU parity of the whole MoE block against the fp32 oracle
(rel-L2 <= 5e-3 and max-abs <= 3e-2)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import PM, golden_inputs, load_golden
from gpu_util import assert_close, bits, oracle_y
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

F_SH, F_RT, F_STREAM, F_TC = 1, 2, 4, 8


def block(x, wts, lo=0, hi=None, flags=F_SH | F_RT):
    from paris_moe_b200 import ops
    hi = wts.shape.E if hi is None else hi
    return ops.moe_block(x, *wts.tensors(), wts.shape.K, lo, hi, flags)


def route_of(x, wts):
    from paris_moe_b200 import ops
    idx, w, *_ = ops.moe_route(x, wts.w_router, wts.w_sh_gvec, wts.shape.K)
    return idx.cpu().numpy(), w.cpu().numpy()


@pytest.fixture(scope="module")
def full():
    from paris_moe_b200 import workload as W
    wts = W.make_weights(W.MoEShape(), seed=0)        # CPU generator: same as the fixtures
    x = W.make_hidden(64, W.MoEShape(), seed=0)
    return wts, wts.to("cuda"), x


@pytest.mark.parametrize("name", ["tiny_T1", "tiny_T5", "tiny_T33", "tiny_T200_zipf"])
def test_block_tiny_golden(name):
    d, meta = load_golden(name)
    shape, wts, x = golden_inputs(meta)
    g = wts.to("cuda")
    xg = x.cuda()
    y = block(xg, g)
    route = route_of(xg, g)
    assert_close(y, oracle_y(x, wts, route=route), name)


@pytest.mark.parametrize("T", [1, 2, 4, 8, 16, 32, 64])
def test_block_decode_sweep(full, T):
    wts, g, x = full
    xg = x[:T].cuda()
    y = block(xg, g)
    route = route_of(xg, g)
    assert_close(y, oracle_y(x[:T], wts, route=route), f"T={T}")


def test_block_c1_against_reference_outputs(full):
    """Config 1 (T=16): the kernel is at least as close to the fp32 oracle as
    the reference's own bf16 paths are."""
    wts, g, x = full
    d, meta = load_golden("c1_T16")
    xg = x[:16].cuda()
    y = block(xg, g).float().cpu().numpy()
    route = route_of(xg, g)
    ref32 = oracle_y(x[:16], wts, route=route)
    ours = O.rel_l2(y, ref32)
    # Only compare against the references on tokens routed identically.
    hidx = d["hf_idx"].astype(np.int32)
    same = np.all(np.sort(route[0], -1) == np.sort(hidx, -1), -1)
    ref_fused = O.bf16_to_f32(d["y_ref_fused"])
    assert ours <= 5e-3
    assert O.rel_l2(y[same], ref_fused[same]) <= 8e-3


def test_block_deterministic(full):
    wts, g, x = full
    xg = x.cuda()
    a = block(xg, g)
    b = block(xg, g)
    assert torch.equal(a, b)


def test_block_partials_sum(full):
    """EP partials: routed [0,128) + routed [128,256) + shared == full."""
    wts, g, x = full
    xg = x[:32].cuda()
    y = block(xg, g).float()
    p0 = block(xg, g, 0, 128, F_RT).float()
    p1 = block(xg, g, 128, 256, F_RT).float()
    sh = block(xg, g, 0, 0, F_SH).float()
    route = route_of(xg, g)
    assert_close(p0, oracle_y(x[:32], wts, route=route, expert_range=(0, 128),
                              with_shared=False), "rank0 partial")
    assert_close(sh, oracle_y(x[:32], wts, route=route, expert_range=(0, 0)), "shared only")
    s = (p0 + p1 + sh).cpu().numpy()
    assert O.rel_l2(s, y.cpu().numpy()) < 5e-3


def test_block_empty():
    from paris_moe_b200 import workload as W
    sh = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    g = W.make_weights(sh, device="cuda")
    x = torch.empty((0, 256), dtype=torch.bfloat16, device="cuda")
    assert block(x, g).shape == (0, 256)


@pytest.fixture(scope="module")
def zipf8192():
    """T=8192 Zipf workload and the oracle's output on its OWN routing (every
    row; the GPU routing is bit-identical to it, checked here first)."""
    from paris_moe_b200 import workload as W
    wts = W.make_weights(W.MoEShape(), seed=0, zipf_s=1.1)
    x = W.make_hidden(8192, W.MoEShape(), seed=0, zipf=True)
    g = wts.to("cuda")
    xg = x.cuda()
    y, oidx, _ = O.moe_block(bits(x), *[bits(t) for t in wts.tensors()], k=wts.shape.K)
    idx, _ = route_of(xg, g)
    assert np.array_equal(idx, oidx)
    return wts, g, x, xg, y


def test_block_prefill_zipf_streaming(zipf8192):
    """T=8192 skewed routing through the streaming kernels, every row."""
    wts, g, x, xg, ref = zipf8192
    y = block(xg, g, flags=F_SH | F_RT | F_STREAM)
    assert_close(y, ref, "T=8192 streaming")


@pytest.mark.parametrize("T", [1, 16, 64])
def test_block_oracle_routing(full, T):
    """End to end against the oracle's own routing (route=None): the GPU's
    exactly rounded top-k makes the two routings identical."""
    wts, g, x = full
    xg = x[:T].cuda()
    y = block(xg, g)
    assert_close(y, oracle_y(x[:T], wts), f"T={T} oracle routing")


@pytest.mark.parametrize("name", ["tiny_T1", "tiny_T5", "tiny_T33", "tiny_T200_zipf"])
def test_block_tiny_golden_oracle_routing(name):
    d, meta = load_golden(name)
    shape, wts, x = golden_inputs(meta)
    y = block(x.cuda(), wts.to("cuda"))
    assert_close(y, oracle_y(x, wts), name)


# ---- tcgen05 grouped-GEMM path (prefill) -----------------------------------

TC_SHAPE = dict(H=256, E=16, K=4, I=128, Is=128)


@pytest.mark.parametrize("T", [1, 5, 64, 200, 777])
def test_block_tc_small_shape(T):
    """Forced tensor-core path on a small shape: ragged M tiles, empty experts."""
    from paris_moe_b200 import workload as W
    sh = W.MoEShape(**TC_SHAPE)
    wts = W.make_weights(sh, seed=21)
    x = W.make_hidden(T, sh, seed=21)
    g = wts.to("cuda")
    xg = x.cuda()
    y = block(xg, g, flags=F_SH | F_RT | F_TC)
    route = route_of(xg, g)
    assert_close(y, oracle_y(x, wts, route=route), f"tc T={T}")


def test_block_tc_partials(full):
    """Forced tensor-core path, EP partial + shared-only at the full shape."""
    wts, g, x = full
    xg = x[:48].cuda()
    route = route_of(xg, g)
    p0 = block(xg, g, 0, 100, F_RT | F_TC)
    assert_close(p0, oracle_y(x[:48], wts, route=route, expert_range=(0, 100),
                              with_shared=False), "tc rank partial")
    sh = block(xg, g, 0, 0, F_SH | F_TC)
    assert_close(sh, oracle_y(x[:48], wts, route=route, expert_range=(0, 0)), "tc shared")


def test_block_tc_matches_stream(full):
    """Both expert paths agree at the full shape (T=64 decode batch)."""
    wts, g, x = full
    xg = x.cuda()
    a = block(xg, g, flags=F_SH | F_RT | F_TC).float().cpu().numpy()
    b = block(xg, g, flags=F_SH | F_RT | F_STREAM).float().cpu().numpy()
    assert O.rel_l2(a, b) < 3e-3


def test_block_prefill_tc_deterministic():
    """The tensor-core path has no atomics: repeated calls are bit-identical."""
    from paris_moe_b200 import workload as W
    wts = W.make_weights(W.MoEShape(), seed=0, zipf_s=1.1)
    g = wts.to("cuda")
    xg = W.make_hidden(2048, W.MoEShape(), seed=0, zipf=True).cuda()
    a = block(xg, g)
    b = block(xg, g)
    assert torch.equal(a, b)


def test_block_prefill_zipf_tc(zipf8192):
    """Default path at T=8192 (tensor cores), skewed routing, every row."""
    wts, g, x, xg, ref = zipf8192
    y = block(xg, g)
    assert_close(y, ref, "tc T=8192")


@pytest.mark.parametrize("up_first", [False, True])
def test_block_prefill_shared_weights_adjacent(up_first):
    """Shared gate and up weights that lie in one buffer (either one first) take
    the single 5-D tensor-map load of the shared expert; the result equals the
    one with separately allocated tensors bit for bit."""
    from paris_moe_b200 import ops, workload as W
    S = W.MoEShape()
    g = W.make_weights(S, seed=3).to("cuda")
    x = W.make_hidden(1024, S, seed=3).cuda()
    ref = block(x, g)
    pair = torch.empty((2, S.Is, S.H), dtype=torch.bfloat16, device="cuda")
    gate, up = (pair[1], pair[0]) if up_first else (pair[0], pair[1])
    gate.copy_(g.w_sh_gate)
    up.copy_(g.w_sh_up)
    t = list(g.tensors())
    t[3], t[4] = gate, up
    y = ops.moe_block(x, *t, S.K, 0, S.E, F_SH | F_RT)
    assert torch.equal(y, ref)
    wc = W.make_weights(S, seed=3)
    rows = np.arange(0, 1024, 16)
    assert_close(y.float().cpu().numpy()[rows],
                 oracle_y(x.cpu(), wc, route=route_of(x, g), rows=rows), "shared adjacent")


def test_block_prefill_shared_gate_is_up():
    """Shared gate and up passed as one tensor (distance 0, no 5-D map): the
    eight 2-D loads per stage give the same bits as two separate copies."""
    from paris_moe_b200 import ops, workload as W
    S = W.MoEShape()
    g = W.make_weights(S, seed=4).to("cuda")
    x = W.make_hidden(512, S, seed=4).cuda()
    t = list(g.tensors())
    t[4] = t[3]
    same = ops.moe_block(x, *t, S.K, 0, S.E, F_SH | F_RT)
    t[4] = t[3].clone()
    apart = ops.moe_block(x, *t, S.K, 0, S.E, F_SH | F_RT)
    assert torch.equal(same, apart)
