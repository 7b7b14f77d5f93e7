"""GPU parity of the router / top-k / dispatch kernels against the oracle
and the reference's golden outputs.

Router logits are defined as the bf16 values nearest to the exact dot
products; the kernels select on those values exactly, so the top-k indices
must equal the oracle's for every token (ties to the lower expert)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import PM, golden_inputs, load_golden
from gpu_util import bits, exact_logits
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

CASES = ["tiny_T1", "tiny_T5", "tiny_T33", "tiny_T200_zipf", "c1_T16", "c2_T64",
         "c3_T8192_route"]


def run_route(x, wts):
    from paris_moe_b200 import ops
    out = ops.moe_route(x.cuda(), wts.w_router.cuda(), wts.w_sh_gvec.cuda(), wts.shape.K)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in out]


def check_route(x, wts, idx, w):
    """idx bit-exact against the oracle; weights to fp32 rounding (a weight
    uses the approximate logit's rounding where the bound did not require an
    exact evaluation, which can move a rare row by one bf16 ulp)."""
    logits = O.router_logits(bits(x), bits(wts.w_router))
    oidx, ow = O.topk_route(logits, wts.shape.K)
    bad = np.nonzero(np.any(idx != oidx, axis=-1))[0]
    assert bad.size == 0, f"{bad.size} tokens differ, first {bad[:5]}: {idx[bad[:2]]} vs {oidx[bad[:2]]}"
    close = np.all(np.isclose(w, ow, rtol=1e-5, atol=1e-7), axis=-1)
    # a weight uses the approximate logit's rounding where the bound did not call for
    # an exact evaluation; that moves the rare row by one bf16 ulp of a logit
    assert close.mean() >= 0.99, close.mean()
    np.testing.assert_allclose(w, ow, atol=0.05)
    return oidx


@pytest.mark.parametrize("name", CASES)
def test_route_matches_oracle(name):
    d, meta = load_golden(name)
    shape, wts, x = golden_inputs(meta)
    idx, w, offs, stok, sslot, sg = run_route(x, wts)
    oidx = check_route(x, wts, idx, w)
    o_offs, o_tok, o_slot = O.dispatch(oidx, shape.E)
    np.testing.assert_array_equal(offs, o_offs)
    np.testing.assert_array_equal(stok, o_tok)
    np.testing.assert_array_equal(sslot, o_slot)
    gate = O.bf16_to_f32(bits(x)) @ O.bf16_to_f32(bits(wts.w_sh_gvec)).reshape(-1)
    np.testing.assert_allclose(sg, 1 / (1 + np.exp(-gate)), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", CASES)
def test_route_matches_reference_topk(name):
    """Against the reference's own (HF) top-k: HF's CPU GEMM rounds its fp32
    sum in another order and breaks exact ties arbitrarily, so a disagreement
    must swap experts whose exact logits are equal or one bf16 ulp apart."""
    d, meta = load_golden(name)
    shape, wts, x = golden_inputs(meta)
    idx, w, *_ = run_route(x, wts)
    hidx = d["hf_idx"].astype(np.int32)
    logits = O.router_logits(bits(x), bits(wts.w_router))
    for t in np.nonzero(np.any(idx != hidx, axis=-1))[0]:
        a = np.sort(logits[t][idx[t]])
        b = np.sort(logits[t][hidx[t]])
        ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(a), 1e-30))) - 7)
        assert np.all(np.abs(a - b) <= ulp), t


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("T", [7, 64, 300])
def test_route_exact_random(seed, T):
    """Full shape, Zipf-biased and plain logits, decode and prefill paths."""
    from paris_moe_b200 import workload as W
    zipf = 1.1 if seed % 2 else None
    wts = W.make_weights(W.MoEShape(), seed=100 + seed, zipf_s=zipf)
    x = W.make_hidden(T, W.MoEShape(), seed=100 + seed, zipf=zipf is not None)
    idx, w, *_ = run_route(x, wts)
    check_route(x, wts, idx, w)


def _diag(x, wts):
    from paris_moe_b200 import _lib
    lib = _lib.load()
    S = wts.shape
    T = x.shape[0]
    xg, wr, gv = x.cuda(), wts.w_router.cuda(), wts.w_sh_gvec.cuda()
    n = _lib.workspace_size(T, S.H, S.E, S.K, 64, 64)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    Rpad = (S.E + 1 + 15) // 16 * 16
    idx = torch.empty((T, S.K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, S.K), dtype=torch.float32, device="cuda")
    lg = torch.empty((T, Rpad), dtype=torch.float32, device="cuda")
    gamma = ctypes.c_float(0)
    stats = (ctypes.c_int * 2)()
    _lib.check("pmoe_route_diag", lib.pmoe_route_diag(
        xg.data_ptr(), T, S.H, S.E, S.K, wr.data_ptr(), gv.data_ptr(), idx.data_ptr(),
        w.data_ptr(), lg.data_ptr(), ctypes.byref(gamma), stats, ws.data_ptr(), n,
        torch.cuda.current_stream().cuda_stream))
    return (idx.cpu().numpy(), w.cpu().numpy(), lg.cpu().numpy()[:, :S.E], gamma.value,
            list(stats))


@pytest.mark.parametrize("case", ["decode_T64", "zipf_T8192", "tc_T300", "mma_K10_T200"])
def test_route_error_bound_holds(case):
    """The accumulation bound the exact selection relies on,
    |approx - exact| <= gamma * ||x|| * ||w||, holds with a factor 16 to spare
    on every logit of each routing path (fused decode router, tensor-core
    prefill router, mma.sync router for K > 8)."""
    from paris_moe_b200 import workload as W
    if case == "decode_T64":
        S, T, z = W.MoEShape(), 64, None
    elif case == "zipf_T8192":
        S, T, z = W.MoEShape(), 8192, 1.1
    elif case == "tc_T300":
        S, T, z = W.MoEShape(), 300, None
    else:
        S, T, z = W.MoEShape(H=1024, E=64, K=10, I=64, Is=64), 200, None
    wts = W.make_weights(S, seed=7, zipf_s=z)
    x = W.make_hidden(T, S, seed=7, zipf=z is not None)
    idx, w, approx, gamma, stats = _diag(x, wts)
    ex = exact_logits(x, wts.w_router)
    xf = O.bf16_to_f32(bits(x)).astype(np.float64)
    wf = O.bf16_to_f32(bits(wts.w_router)).astype(np.float64)
    bound = gamma * np.linalg.norm(xf, axis=1)[:, None] * np.linalg.norm(wf, axis=1)[None, :]
    ratio = np.abs(approx - ex) / bound
    print(f"{case}: gamma=2^{np.log2(gamma):.2f} max err/bound={ratio.max():.2e} "
          f"exact evaluations={stats[0]} ({stats[0] / T:.3f}/token)")
    assert ratio.max() <= 1 / 16
    assert stats[1] == 0
    check_route(x, wts, idx, w)


def test_route_exact_midpoints():
    """Logits that are exactly bf16 midpoints (ties to even) or lie within
    2^-40 of one: the fp32 approximations cannot tell these apart, the exact
    evaluation must."""
    from paris_moe_b200 import workload as W
    S = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(S, seed=5)
    f = lambda v: torch.tensor(v, dtype=torch.float32).to(torch.bfloat16)
    wr = torch.zeros((S.E, S.H), dtype=torch.bfloat16)
    x = torch.zeros((4, S.H), dtype=torch.bfloat16)
    x[:, 0], x[:, 1], x[:, 2] = f(1.0), f(2.0 ** -8), f(2.0 ** -40)
    x[1, 2] = f(-2.0 ** -40)
    x[2, 1] = f(3 * 2.0 ** -8)
    x[3, 1] = f(-2.0 ** -8)
    for e in range(S.E):
        # logits 1 + c * 2^-8 (+ d * 2^-40), all within two bf16 values of 1
        wr[e, 0] = f(1.0)
        wr[e, 1] = f(float(e % 4))
        wr[e, 2] = f(float((e // 4) - 1))
    wts.w_router = wr
    idx, w, *_ = run_route(x, wts)
    check_route(x, wts, idx, w)


def test_route_empty():
    from paris_moe_b200 import ops, workload as W
    sh = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(sh, device="cuda")
    x = torch.empty((0, 256), dtype=torch.bfloat16, device="cuda")
    idx, w, offs, stok, sslot, sg = ops.moe_route(x, wts.w_router, wts.w_sh_gvec, 4)
    assert idx.shape == (0, 4) and offs.cpu().tolist() == [0] * 17


@pytest.mark.parametrize("T", [9, 200])
def test_route_all_tied_logits(T):
    """Zero router weights: every logit ties, the top-k is experts 0..K-1."""
    from paris_moe_b200 import ops, workload as W
    sh = W.MoEShape(H=256, E=32, K=8, I=64, Is=64)
    wts = W.make_weights(sh, device="cuda")
    wts.w_router.zero_()
    x = W.make_hidden(T, sh, device="cuda")
    idx, w, offs, stok, sslot, sg = ops.moe_route(x, wts.w_router, wts.w_sh_gvec, 8)
    assert (idx.cpu() == torch.arange(8, dtype=torch.int32)).all()
    assert torch.allclose(w.cpu(), torch.full((T, 8), 1 / 8))


def _exact_logits_gpu(x, w):
    from paris_moe_b200 import _lib
    lib = _lib.load()
    T, H = x.shape
    E = w.shape[0]
    xg, wg = x.cuda().contiguous(), w.cuda().contiguous()
    out = torch.empty((T, E), dtype=torch.float32, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check("pmoe_exact_logits", lib.pmoe_exact_logits(
        xg.data_ptr(), T, H, E, wg.data_ptr(), out.data_ptr(), bad.data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out.cpu().numpy(), int(bad.item())


def test_exact_logits_all_pairs_bit_exact():
    """The GPU's exact evaluation on every (token, expert) pair equals the
    oracle's exactly rounded logits bit for bit: the full decode batch, Zipf
    rows, and rows that take the general (integer-field) path -- bf16
    subnormals, exact zeros, huge and tiny entries, exact midpoints."""
    from paris_moe_b200 import workload as W
    S = W.MoEShape()
    wts = W.make_weights(S, seed=11, zipf_s=1.1)
    x = W.make_hidden(64, S, seed=11, zipf=True)
    got, bad = _exact_logits_gpu(x, wts.w_router)
    want = O.router_logits(bits(x), bits(wts.w_router))
    diff = np.argwhere(got != want)
    assert diff.size == 0, (diff[:5], got[tuple(diff[:5].T)], want[tuple(diff[:5].T)])
    assert bad == 0
    f = lambda v: torch.tensor(v, dtype=torch.float32).to(torch.bfloat16)
    xs = torch.zeros((6, 256), dtype=torch.bfloat16)
    ws = (torch.randn((40, 256), generator=torch.Generator().manual_seed(3)) * 0.02).bfloat16()
    xs[0] = (torch.randn(256, generator=torch.Generator().manual_seed(4))).bfloat16()
    xs[1] = (xs[0].float() * 2.0 ** -122).bfloat16()                          # subnormals
    xs[2] = xs[0] * f(2.0 ** 60)                                               # huge
    xs[3, :2] = f(1.0)
    xs[3, 2] = f(2.0 ** -8)                                                    # midpoints
    xs[4] = xs[0]
    xs[4, 5] = f(2.0 ** -60)                                                   # wide spread
    ws[0, :3] = f(1.0)
    got, bad = _exact_logits_gpu(xs, ws)
    want = O.router_logits(bits(xs), bits(ws))
    diff = np.argwhere(got != want)
    assert diff.size == 0, (diff[:5], got[tuple(diff[:5].T)], want[tuple(diff[:5].T)])
    assert bad == 0
