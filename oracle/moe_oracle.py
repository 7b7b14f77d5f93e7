"""CPU oracle for the Qwen3.5-35B-A3B sparse-MoE block (TEST INFRASTRUCTURE ONLY).

This module is the checker for the CUDA path, never the thing measured or
shipped: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` leg may import it.  It is a plain numpy restatement of the
arithmetic the reference executes:

* the reference patches ``Qwen3_5MoeSparseMoeBlock.forward``
  (``engine/kernels/patch.py:43-84``) with ``fused_moe_forward``
  (``engine/kernels/moe_grouped_mlp.py:166-186``);
* the math itself lives in the third-party ``transformers`` package
  (the reference's ``uv.lock:4282-4283`` pins 4.57.6, which has no
  ``qwen3_5_moe`` module; the code requires >= 5.5 and 5.5.0 is what is
  installed and used here): ``modeling_qwen3_5_moe.py:698-792`` and
  ``integrations/moe.py:350-429``.

Parity is pinned: ``tests/golden/make_golden.py`` imports the HF block and
the reference's ``fused_moe_forward`` in a container that has the reference
checked out, runs them on seeded inputs, and stores their outputs; the
``-m "not gpu"`` tests check this oracle against those fixtures.

Numerics.  bf16 tensors are carried as ``uint16`` bit patterns and widened
exactly to fp32.  Router logits are the bf16 values nearest (ties to even)
to the exact dot products -- the value a "fp32-accumulate, round once" GEMM
approximates -- computed in float64 with a rigorous error bound and, where
the bound leaves the rounding open, in integer arithmetic; top-k ties are
broken to the lower expert index.  Everything after routing is fp32 ("the
fp32-accumulate reference" the output tolerance is stated against).
"""
from __future__ import annotations

import numpy as np


# ---------------------------------------------------------------- bf16 bits --

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits with round-to-nearest-even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    return ((u + bias) >> 16).astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(np.asarray(x, dtype=np.float32)))


def torch_bf16_bits(t) -> np.ndarray:
    """bf16 torch tensor (any device) -> numpy uint16 bits (copy on host)."""
    import torch
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


# ----------------------------------------------------------------- routing --

def _rn_bf16_f64(v: np.ndarray) -> np.ndarray:
    """Nearest bf16 value (ties to even) of float64 values, as float64.

    |v| in [2^(e-1), 2^e) has bf16 spacing 2^(e-8); subnormal bf16 spacing is
    2^-133.  Scaling by a power of two is exact, so one ``rint`` (half to
    even) rounds correctly."""
    v = np.asarray(v, dtype=np.float64)
    _, e = np.frexp(v)
    q = np.maximum(e - 8, -133)
    return np.ldexp(np.rint(np.ldexp(v, -q)), q)


def _bf16_int(b: int):
    """bf16 bit pattern -> (signed integer significand M, exponent k): value = M * 2^k."""
    sign = -1 if b & 0x8000 else 1
    E = (b >> 7) & 0xFF
    frac = b & 0x7F
    if E == 0:
        return sign * frac, -133
    return sign * (128 + frac), E - 134


def exact_logit_bf16(x_row_bits: np.ndarray, w_row_bits: np.ndarray) -> float:
    """bf16 nearest (ties to even) to the exact dot product of two bf16 rows,
    in Python integer arithmetic (no rounding before the final one)."""
    terms = []
    for xb, wb in zip(x_row_bits.tolist(), w_row_bits.tolist()):
        mx, kx = _bf16_int(xb)
        mw, kw = _bf16_int(wb)
        if mx and mw:
            terms.append((mx * mw, kx + kw))
    if not terms:
        return 0.0
    base = min(k for _, k in terms)
    n = sum(m << (k - base) for m, k in terms)
    if n == 0:
        return 0.0
    sign, n = (-1 if n < 0 else 1), abs(n)
    shift = max(n.bit_length() - 8, -133 - base)
    if shift > 0:
        qv, rem = n >> shift, n & ((1 << shift) - 1)
        half = 1 << (shift - 1)
        if rem > half or (rem == half and (qv & 1)):
            qv += 1
        n, base = qv, base + shift
    import math
    return float(sign * math.ldexp(n, base))


def router_logits(x_bits: np.ndarray, w_router_bits: np.ndarray) -> np.ndarray:
    """bf16 router logits as fp32 values.

    Follows ``Qwen3_5MoeTopKRouter.forward`` (modeling_qwen3_5_moe.py:762-764):
    ``F.linear(hidden_states, self.weight)`` in bf16.  The value taken is the
    bf16 nearest (ties to even) to the EXACT dot product -- the one rounding
    every fp32-accumulating bf16 GEMM approximates, and the definition the CUDA
    kernels implement.  Products of bf16 values are exact in float64; the
    float64 sum has |error| <= n * 2^-52 * sum|x_i w_i| (twice the textbook
    bound for any summation order); where that interval still straddles a bf16
    rounding boundary the logit is recomputed in integer arithmetic
    (``exact_logit_bf16``).
    """
    x = bf16_to_f32(x_bits).astype(np.float64)
    w = bf16_to_f32(w_router_bits).astype(np.float64)
    a = x @ w.T
    bound = (np.abs(x) @ np.abs(w).T) * (x.shape[1] * 2.0 ** -52)
    r = _rn_bf16_f64(a)
    amb = _rn_bf16_f64(a - bound) != _rn_bf16_f64(a + bound)
    xb = np.asarray(x_bits, dtype=np.uint16)
    wb = np.asarray(w_router_bits, dtype=np.uint16)
    for t, e in zip(*np.nonzero(amb)):
        r[t, e] = exact_logit_bf16(xb[t], wb[e])
    return r.astype(np.float32)


def topk_route(logits: np.ndarray, k: int):
    """Top-k experts per token with renormalised fp32 weights.

    Follows modeling_qwen3_5_moe.py:765-768: softmax in fp32 over all
    experts, ``topk(k)`` sorted by value, divide by the sum of the k values.
    Ties (equal bf16 logits) go to the lower expert index.
    Returns (idx int32 [T,k], weights fp32 [T,k]).
    """
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    # lexsort: last key is primary -> sort by -logit, then by index.
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -logits), axis=-1)
    idx = order[:, :k].astype(np.int32)
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32))
    probs = e / e.sum(axis=-1, keepdims=True)
    top = np.take_along_axis(probs, idx.astype(np.int64), axis=-1)
    w = (top / top.sum(axis=-1, keepdims=True)).astype(np.float32)
    return idx, w


def dispatch(idx: np.ndarray, E: int):
    """CSR dispatch of the (token, slot) pairs by expert.

    Follows ``_torch_dispatch`` (engine/kernels/moe_dispatch.py:119-137):
    stable sort of the flattened expert ids, ``sorted_token_idx = perm // K``,
    ``sorted_slot_idx = perm % K``, bincount + exclusive cumsum for offsets.
    Returns (offsets int32 [E+1], sorted_tok int32 [T*K], sorted_slot int32 [T*K]).
    """
    T, K = idx.shape
    flat = idx.reshape(-1).astype(np.int64)
    perm = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=E)
    offsets = np.zeros(E + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    return offsets, (perm // K).astype(np.int32), (perm % K).astype(np.int32)


# ------------------------------------------------------------------ block ---

def _silu(x):
    return x / (1.0 + np.exp(-x))


def swiglu(x: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
           round_h: bool = False) -> np.ndarray:
    """``down(act(gate(x)) * up(x))`` in fp32 (modeling_qwen3_5_moe.py:709-711,
    and the per-expert body at :743-747).  ``round_h`` rounds the SiLU*up
    intermediate to bf16, as every bf16 implementation of the block does."""
    g = x @ w_gate.T
    u = x @ w_up.T
    h = (_silu(g) * u).astype(np.float32)
    if round_h:
        h = round_bf16(h)
    return h @ w_down.T


def moe_block(x_bits, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up, w_sh_down,
              w_sh_gvec, k: int, expert_range=None, with_shared=True, round_h=False,
              route=None):
    """fp32 restatement of ``Qwen3_5MoeSparseMoeBlock.forward``.

    modeling_qwen3_5_moe.py:781-792 (and the patched equivalent
    engine/kernels/moe_grouped_mlp.py:166-186):
    ``y = experts(x, topk) + sigmoid(shared_expert_gate(x)) * shared_expert(x)``.
    The expert combine ``y_t = sum_k w_tk * down_k(t)`` is accumulated in fp32
    (the HF grouped_mm path, integrations/moe.py:417-429).

    ``expert_range=(lo, hi)`` keeps only the routed contributions of experts
    in [lo, hi) -- the per-rank partial of ``ep_forward``
    (engine/runtime/ep.py:97-143).  All weight args are bf16 bit arrays.
    Returns (y fp32 [T,H], idx, weights).
    """
    x = bf16_to_f32(x_bits)
    T, H = x.shape
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    if route is None:
        logits = router_logits(x_bits, w_router)
        idx, wts = topk_route(logits, k)
    else:
        idx, wts = route
    y = np.zeros((T, H), dtype=np.float32)
    lo, hi = (0, E) if expert_range is None else expert_range
    for e in np.unique(idx):
        if not (lo <= e < hi):
            continue
        tok, slot = np.nonzero(idx == e)
        wgu = bf16_to_f32(w_gate_up[e])
        wd = bf16_to_f32(w_down[e])
        out = swiglu(x[tok], wgu[:I], wgu[I:], wd, round_h=round_h)
        y[tok] += out * wts[tok, slot][:, None]      # tokens are distinct within an expert
    if with_shared:
        sh = swiglu(x, bf16_to_f32(w_sh_gate), bf16_to_f32(w_sh_up),
                    bf16_to_f32(w_sh_down), round_h=round_h)
        gate = x @ bf16_to_f32(w_sh_gvec).reshape(-1)
        y += (1.0 / (1.0 + np.exp(-gate)))[:, None].astype(np.float32) * sh
    return y, idx, wts


def rmsnorm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """``Qwen3_5MoeRMSNorm.forward`` (modeling_qwen3_5_moe.py:795-812):
    fp32 ``x * rsqrt(mean(x^2) + eps) * (1 + w)`` then cast to bf16 (bits)."""
    x = bf16_to_f32(x_bits)
    w = bf16_to_f32(w_bits)
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + np.float32(eps))
    return f32_to_bf16((x * r * (1.0 + w)).astype(np.float32))


def decoder_layer(x_bits: np.ndarray, w_norm_bits: np.ndarray, block_weights, k: int,
                  eps: float = 1e-6, route=None):
    """MoE-only ``Qwen3_5MoeDecoderLayer`` half (modeling_qwen3_5_moe.py:862-868):
    ``residual + mlp(post_attention_layernorm(x))`` in bf16, i.e.
    bf16(x + bf16(moe_block(rmsnorm(x)))).  ``route`` (optional) is the routing
    of the normalised input.  Returns (y fp32 values of the bf16 result, xn bits)."""
    xn = rmsnorm(x_bits, w_norm_bits, eps)
    y, _, _ = moe_block(xn, *block_weights, k=k, route=route)
    out = round_bf16(bf16_to_f32(x_bits) + round_bf16(y.astype(np.float32)))
    return out, xn


# ------------------------------------------------------------- comparisons --

def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
