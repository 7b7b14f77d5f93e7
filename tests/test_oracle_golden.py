"""Pin the CPU oracle against outputs of the reference's own code
(HF Qwen3_5MoeSparseMoeBlock grouped_mm/eager and the reference's
fused_moe_forward / _torch_dispatch), stored by tests/golden/make_golden.py."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import golden_inputs, load_golden
from oracle import moe_oracle as O

ALL = ["tiny_T1", "tiny_T5", "tiny_T33", "tiny_T200_zipf", "c1_T16", "c2_T64",
       "c3_T8192_route"]
FULL = ["tiny_T1", "tiny_T5", "tiny_T33", "tiny_T200_zipf", "c1_T16", "c2_T64"]

_cache = {}


def case(name):
    if name not in _cache:
        d, meta = load_golden(name)
        shape, wts, x = golden_inputs(meta)
        wb = {n: O.torch_bf16_bits(getattr(wts, n)) for n in shape.weight_names()}
        _cache.clear()
        _cache[name] = (d, meta, shape, wb, O.torch_bf16_bits(x))
    return _cache[name]


def ties_only(idx_a, idx_b, logits):
    """True when every top-k disagreement swaps experts whose bf16 logits are
    equal or one bf16 ulp apart (a rounding flip of an fp32 accumulation in
    another order; HF's own logits are not stored for the largest case)."""
    for t in np.nonzero(np.any(idx_a != idx_b, axis=-1))[0]:
        va = np.sort(logits[t][idx_a[t]])
        vb = np.sort(logits[t][idx_b[t]])
        ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(va), 1e-30))) - 7)
        if np.any(np.abs(va - vb) > ulp):
            return False
    return True


@pytest.mark.parametrize("name", ALL)
def test_generator_digests(name):
    d, meta, shape, wb, xb = case(name)
    for n, dig in meta["weights_sha256_16"].items():
        assert hashlib.sha256(wb[n].tobytes()).hexdigest()[:16] == dig, n
    assert hashlib.sha256(xb.tobytes()).hexdigest()[:16] == meta["x_sha256_16"]


@pytest.mark.parametrize("name", ALL)
def test_routing_matches_hf(name):
    d, meta, shape, wb, xb = case(name)
    logits = O.router_logits(xb, wb["w_router"])
    if "hf_logits" in d:
        # HF's CPU bf16 GEMM accumulates in another order: allow rare 1-ulp flips.
        same = (O.f32_to_bf16(logits) == d["hf_logits"]).mean()
        assert same >= 0.999, same
    idx, w = O.topk_route(logits, shape.K)
    hidx = d["hf_idx"].astype(np.int32)
    assert ties_only(idx, hidx, logits)
    agree = np.all(idx == hidx, axis=-1)
    assert agree.mean() > 0.5
    close = np.all(np.isclose(w, d["hf_w"], rtol=2e-6, atol=1e-7), axis=-1)
    # Rows whose logits all agree with HF's match to fp32 rounding; the rare
    # row with a 1-ulp logit flip moves its weights by a few percent.
    assert close[agree].mean() >= 0.995, close[agree].mean()
    np.testing.assert_allclose(w[agree], d["hf_w"][agree], atol=0.05)


@pytest.mark.parametrize("name", ALL)
def test_dispatch_matches_reference(name):
    d, meta, shape, wb, xb = case(name)
    offs, stok, sslot = O.dispatch(d["hf_idx"].astype(np.int32), shape.E)
    np.testing.assert_array_equal(offs, d["ref_offsets"])
    if "ref_sorted_tok" in d:
        np.testing.assert_array_equal(stok, d["ref_sorted_tok"])
        np.testing.assert_array_equal(sslot, d["ref_sorted_slot"])


@pytest.mark.parametrize("name", FULL)
def test_block_matches_reference(name):
    """Same routing as HF, fp32 oracle vs the references' bf16 outputs.

    The references round every intermediate to bf16, which alone costs
    rel-L2 4.8e-3..5.3e-3 against fp32; the bound here is 6e-3."""
    d, meta, shape, wb, xb = case(name)
    route = (d["hf_idx"].astype(np.int32), d["hf_w"])
    y, _, _ = O.moe_block(xb, *[wb[n] for n in shape.weight_names()], k=shape.K, route=route)
    for key in ("y_hf_grouped", "y_hf_eager", "y_ref_fused"):
        ref = O.bf16_to_f32(d[key])
        assert O.rel_l2(ref, y) <= 6e-3, (key, O.rel_l2(ref, y))
        assert O.max_abs(ref, y) <= 3e-2, (key, O.max_abs(ref, y))


def test_bf16_rounding_rne():
    v = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 0.0], dtype=np.float32)
    out = O.bf16_to_f32(O.f32_to_bf16(v))
    np.testing.assert_array_equal(out, np.array([1.0, 1.0, 1.0 + 4 * 2 ** -8, -2.5, 0.0],
                                                dtype=np.float32))


def test_topk_ties_lower_index():
    logits = np.array([[0.5, 1.0, 1.0, 0.25, 1.0]], dtype=np.float32)
    idx, w = O.topk_route(logits, 2)
    assert idx.tolist() == [[1, 2]]
    np.testing.assert_allclose(w, [[0.5, 0.5]])


def test_dispatch_empty_and_ragged():
    offs, st, ss = O.dispatch(np.zeros((0, 4), np.int32), 8)
    assert offs.tolist() == [0] * 9 and st.size == 0
    idx = np.array([[3, 1], [1, 7], [3, 0]], np.int32)
    offs, st, ss = O.dispatch(idx, 8)
    assert offs.tolist() == [0, 1, 3, 3, 5, 5, 5, 5, 6]
    assert st.tolist() == [2, 0, 1, 0, 2, 1] and ss.tolist() == [1, 1, 0, 0, 0, 1]


def test_router_logits_exactly_rounded():
    """The oracle's logits equal the integer-arithmetic exact rounding, on
    random rows and on crafted exact midpoints (ties to even) and near-midpoints."""
    rng = np.random.default_rng(3)
    x = O.f32_to_bf16(rng.standard_normal((6, 512)).astype(np.float32))
    w = O.f32_to_bf16((rng.standard_normal((40, 512)) * 0.02).astype(np.float32))
    lg = O.router_logits(x, w)
    for t in range(6):
        for e in range(0, 40, 3):
            assert lg[t, e] == O.exact_logit_bf16(x[t], w[e])
    one, eps, tiny = [O.f32_to_bf16(np.float32(v)) for v in (1.0, 2.0 ** -8, 2.0 ** -40)]
    xx = np.zeros((3, 256), np.uint16)
    ww = np.zeros((1, 256), np.uint16)
    xx[:, 0], xx[:, 1] = one, eps                    # exact sum 1 + 2^-8: a midpoint
    xx[1, 2] = tiny                                  # just above it
    xx[2, 2] = tiny | 0x8000                         # just below it
    ww[0, 0] = ww[0, 1] = ww[0, 2] = one
    np.testing.assert_array_equal(O.router_logits(xx, ww)[:, 0], [1.0, 1.0 + 2 ** -7, 1.0])
