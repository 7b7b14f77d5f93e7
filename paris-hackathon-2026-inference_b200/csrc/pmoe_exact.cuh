// Exactly rounded router logits and the top-k selection built on them.
//
// The router of Qwen3_5MoeTopKRouter.forward (modeling_qwen3_5_moe.py:762-770)
// computes bf16 logits F.linear(x, W_r) and selects the top K.  Which experts
// win depends on the last bit of those logits, so "the" logit is defined here
// as the bf16 value nearest (ties to even) to the EXACT dot product of the
// bf16 operands.  The tensor-core GEMMs produce an fp32 approximation `a`;
// this file turns it into a provably correct selection:
//
//  1. Error model.  Every product of two bf16 values is exact in fp32; each
//     tensor-core MMA step (k = 16) and each fp32 addition of partial sums is
//     taken to add at most 2^-22 * S to the error, S = sum_i |x_i w_i| (the
//     published measurements of fp32-accumulating tensor cores, Fasi, Higham,
//     Mikaitis, Pranesh, "Numerical behavior of NVIDIA tensor cores", PeerJ
//     CS 2021, show at most one unit in the last place of fp32 per step).  A
//     path whose accumulation has depth D therefore has |a - exact| <=
//     D * 2^-22 * S <= gamma * ||x||_2 * ||w||_2 (Cauchy-Schwarz), gamma =
//     D * 2^-22 (with slack for the fp32 norms).  The GPU tests check the
//     observed error against this bound with a wide margin.
//  2. Interval selection.  Each expert's logit lies in [RN(a - d), RN(a + d)]
//     (RN = round to bf16, monotone), d = gamma * ||x|| * ||w_e||.  The K
//     largest lower ends (ties to the lower expert) are the answer when no
//     other expert's upper end reaches the K-th lower end and consecutive
//     winners' intervals are ordered; otherwise every expert whose interval
//     is wider than one value and reaches the K-th lower end is evaluated
//     exactly (step 3) and the selection is redone on exact keys.
//  3. Exact evaluation (one warp): products in double (exact), summed with
//     TwoSum (Knuth) into a value s and a compensation c, so the partial sum
//     is s + c exactly as long as c stays representable.  That holds when
//     span(x) + span(w) + log2((n + 64) n) <= 88, span = largest minus
//     smallest exponent of the non-zero entries; a row outside it is counted
//     in a statistics word (the result is then still far more accurate than
//     the fp32 approximation).  The final rounding to bf16 uses h = RN64(s+c)
//     and the exact remainder l = (s + c) - h to decide a midpoint.
#pragma once
#include "pmoe_common.cuh"

namespace pmoe {

// Per-step error unit of the model above, and the slack factor on top of it
// that covers the fp32 arithmetic of the norms and of d itself.
constexpr float kAccStepErr = 0x1p-22f;
constexpr float kBoundSlack = 1.0f + 0x1p-8f;

// Statistics words of the exact selection (in the workspace status array).
struct ExactStats {
  int* n_exact;    // exact evaluations run
  int* n_inexact;  // of which outside the exactness condition
};

__device__ __forceinline__ void two_sum(double a, double b, double& s, double& e) {
  s = __dadd_rn(a, b);
  const double bb = __dsub_rn(s, a);
  e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
}

// Exponent of a non-zero finite bf16 (subnormals count as -126: their last
// place is 2^-133, like a normal value of exponent -126).  Zero: no entry.
__device__ __forceinline__ void bf16_exp_range(uint32_t b, int& emin, int& emax, bool& finite) {
  if ((b & 0x7FFFu) == 0) return;
  const int E = int((b >> 7) & 0xFFu);
  if (E == 0xFF) finite = false;
  const int ex = E == 0 ? -126 : E - 127;
  emin = min(emin, ex);
  emax = max(emax, ex);
}

// bf16 nearest (ties to even) to h + l, where h = RN64(h + l) (so a bf16
// midpoint can only be hit by h itself, and then l decides).
__device__ __forceinline__ float round_bf16_pair(double h, double l) {
  if (h == 0.0) return 0.0f;
  const int e = int((__double2hiint(h) >> 20) & 0x7FF) - 1023;
  const int q = max(e - 7, -133);
  const double sc = scalbn(h, -q);  // |sc| in [128, 256): exact
  const double fl = floor(sc);
  double r;
  if (__dsub_rn(sc, fl) == 0.5 && l != 0.0)
    r = l > 0.0 ? fl + 1.0 : fl;
  else
    r = rint(sc);                      // round half to even
  return float(scalbn(r, q));          // <= 9 significant bits: exact in fp32
}

// Exact x . w (bf16 rows of length n, n % 256 == 0, 16-byte aligned), rounded
// to bf16; all lanes of the warp return the same value.  `ok` is false when
// the exactness condition of step 3 fails.
static __device__ __noinline__ float warp_exact_dot(const __nv_bfloat16* __restrict__ x,
                                             const __nv_bfloat16* __restrict__ w, int n,
                                             bool& ok) {
  const int lane = threadIdx.x & 31;
  double s0 = 0.0, c0 = 0.0, s1 = 0.0, c1 = 0.0;
  int xmin = 1 << 20, xmax = -(1 << 20), wmin = 1 << 20, wmax = -(1 << 20);
  bool finite = true;
  for (int i = lane * 8; i < n; i += 256) {
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + i));
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + i));
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        const uint32_t xb = (xs[j] >> (16 * hlf)) & 0xFFFFu;
        const uint32_t wb = (ws[j] >> (16 * hlf)) & 0xFFFFu;
        bf16_exp_range(xb, xmin, xmax, finite);
        bf16_exp_range(wb, wmin, wmax, finite);
        const double p = __dmul_rn(double(__uint_as_float(xb << 16)),
                                   double(__uint_as_float(wb << 16)));  // exact
        double t, e;
        if (hlf == 0) {
          two_sum(s0, p, t, e);
          s0 = t;
          c0 = __dadd_rn(c0, e);
        } else {
          two_sum(s1, p, t, e);
          s1 = t;
          c1 = __dadd_rn(c1, e);
        }
      }
    }
  }
  double s, c, e;
  two_sum(s0, s1, s, e);
  c = __dadd_rn(__dadd_rn(c0, c1), e);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const double c2 = __shfl_xor_sync(0xffffffffu, c, o);
    double t;
    two_sum(s, s2, t, e);
    s = t;
    c = __dadd_rn(__dadd_rn(c, c2), e);
  }
  xmin = __reduce_min_sync(0xffffffffu, xmin);
  xmax = __reduce_max_sync(0xffffffffu, xmax);
  wmin = __reduce_min_sync(0xffffffffu, wmin);
  wmax = __reduce_max_sync(0xffffffffu, wmax);
  finite = __all_sync(0xffffffffu, finite);
  double h, l;
  two_sum(s, c, h, l);
  // ceil(log2((n + 64) * n)) by integer arithmetic
  const unsigned long long nn = (unsigned long long)(n + 64) * (unsigned long long)n;
  const int lg = 64 - __clzll((long long)(nn - 1));
  const int span = (xmax >= xmin ? xmax - xmin : 0) + (wmax >= wmin ? wmax - wmin : 0);
  ok = finite && span + lg <= 88;
  return round_bf16_pair(h, l);
}

// Order-preserving 16-bit key of a bf16-exact float, ties to the lower expert:
// (key << 16) | (0xFFFF - e) is unique per expert and larger is better.
__device__ __forceinline__ uint32_t logit_key(float v, int e) {
  uint32_t b = __float_as_uint(v) >> 16;
  if (b == 0x8000u) b = 0;  // -0 == +0
  b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (b << 16) | uint32_t(0xFFFF - e);
}
__device__ __forceinline__ float logit_key_value(uint32_t key) {
  const uint32_t s = key >> 16;
  const uint32_t b = (s & 0x8000u) ? (s & 0x7FFFu) : (~s & 0xFFFFu);
  return __uint_as_float(b << 16);
}

// Per-warp top-K of one token from its approximate logits (see the file
// comment).  `lg(e)` returns the fp32 approximation of expert e's logit,
// `wn` the experts' row norms, `nx` the token's norm, `gamma` the path's
// bound factor; x_row / w_router (row stride H) feed the exact evaluations.
// Lane k < K receives the k-th expert (descending) in `e_out` and its bf16
// logit in `v_out`; the weights follow from those (caller).
template <typename LogitFn>
__device__ __forceinline__ void warp_select_exact(LogitFn lg, const float* __restrict__ wn,
                                                  float nx, float gamma, int E, int K,
                                                  const __nv_bfloat16* __restrict__ x_row,
                                                  const __nv_bfloat16* __restrict__ w_router,
                                                  int H, ExactStats stats, int& e_out,
                                                  float& v_out) {
  const int lane = threadIdx.x & 31;
  uint32_t klo[8], khi[8];
  float val[8];
  const float gx = gamma * kBoundSlack * nx;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = j * 32 + lane;
    klo[j] = khi[j] = 0u;
    val[j] = 0.f;
    if (e < E) {
      const float a = lg(e);
      const float d = gx * wn[e];
      klo[j] = logit_key(bf16_round(__fsub_rd(a, d)), e);
      khi[j] = logit_key(bf16_round(__fadd_ru(a, d)), e);
      val[j] = bf16_round(a);
    }
  }
  // K largest lower ends; for each winner also its upper end.
  uint32_t mine_lo = 0u, mine_hi = 0u, sel = 0u;
  for (int k = 0; k < K; ++k) {
    uint32_t m = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (!(sel >> j & 1u)) m = max(m, klo[j]);
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, m);
    uint32_t hk = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (klo[j] == wmax && !(sel >> j & 1u)) {
        sel |= 1u << j;
        hk = khi[j];
      }
    hk = __reduce_max_sync(0xffffffffu, hk);
    if (lane == k) {
      mine_lo = wmax;
      mine_hi = hk;
    }
  }
  const uint32_t Lk = __shfl_sync(0xffffffffu, mine_lo, K - 1);
  uint32_t mo = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (!(sel >> j & 1u)) mo = max(mo, khi[j]);
  mo = __reduce_max_sync(0xffffffffu, mo);
  const uint32_t prev_lo = __shfl_up_sync(0xffffffffu, mine_lo, 1);
  const bool bad_order = lane >= 1 && lane < K && !(prev_lo > mine_hi);
  const bool certain = mo < Lk && !__any_sync(0xffffffffu, bad_order);
  uint32_t mine = mine_lo;
  if (!certain) {
    // Evaluate exactly every candidate whose interval holds more than one value.
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      const int e = j * 32 + lane;
      const bool unc = e < E && khi[j] >= Lk && (khi[j] >> 16) != (klo[j] >> 16);
      unsigned mask = __ballot_sync(0xffffffffu, unc);
      while (mask) {
        const int l = __ffs(mask) - 1;
        mask &= mask - 1;
        const int ee = j * 32 + l;
        bool ok = true;
        const float r = warp_exact_dot(x_row, w_router + size_t(ee) * H, H, ok);
        if (lane == l) {
          klo[j] = khi[j] = logit_key(r, ee);
          val[j] = r;
        }
        if (lane == 0) {
          atomicAdd(stats.n_exact, 1);
          if (!ok) atomicAdd(stats.n_inexact, 1);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (khi[j] < Lk) klo[j] = 0u;  // cannot be among the K largest
    sel = 0u;
    mine = 0u;
    for (int k = 0; k < K; ++k) {
      uint32_t m = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (!(sel >> j & 1u)) m = max(m, klo[j]);
      const uint32_t wmax = __reduce_max_sync(0xffffffffu, m);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (klo[j] == wmax) sel |= 1u << j;
      if (lane == k) mine = wmax;
    }
  }
  e_out = 0xFFFF - int(mine & 0xFFFFu);
  // value of the selected expert: exact where evaluated, else RN(a) (equal to
  // the exact value when the interval is one value wide)
  float v = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float vj = __shfl_sync(0xffffffffu, val[j], e_out & 31);
    if ((e_out >> 5) == j) v = vj;
  }
  v_out = v;
}

// Renormalised top-K weights (router :765-768): softmax over all experts,
// top K, divided by their sum == exp(l_k - l_0) / sum_j exp(l_j - l_0) over
// the K selected.  Lanes >= K return 0.
__device__ __forceinline__ float warp_topk_weight(float v, int K) {
  const int lane = threadIdx.x & 31;
  const float l0 = __shfl_sync(0xffffffffu, v, 0);
  const float ex = lane < K ? __expf(v - l0) : 0.f;
  float den = ex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  return ex / den;
}

// Sum of squares of a bf16 row (n % 256 == 0) by one warp; all lanes get it.
__device__ __forceinline__ float warp_row_sumsq(const __nv_bfloat16* __restrict__ r, int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int i = lane * 8; i < n; i += 256) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(r + i));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(u[j] << 16), hi = __uint_as_float(u[j] & 0xFFFF0000u);
      s = fmaf(lo, lo, s);
      s = fmaf(hi, hi, s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Upper bound of the 2-norm from an fp32 sum of squares of n terms.
__device__ __forceinline__ float norm_from_sumsq(float ss) {
  return sqrtf(ss * kBoundSlack);
}

// ---------------------------------------------------------------------------
// Warp-per-token top-k with exactly rounded logits (above): `row`
// holds the token's fp32 approximate logits (entry E = the raw shared-gate
// sum), nx its norm, wn the router rows' norms, gamma the accumulation
// bound of the GEMM that produced `row`.  Writes the K experts (descending,
// ties to the lower expert), their renormalised weights, sigmoid(gate), and
// counts each expert in cnt.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_topk_token(const float* row, float nx,
                                                const float* __restrict__ wn, float gamma, int t,
                                                int E, int K, const __nv_bfloat16* __restrict__ x,
                                                const __nv_bfloat16* __restrict__ w_router, int H,
                                                ExactStats stats, int32_t* __restrict__ topk_idx,
                                                float* __restrict__ topk_w,
                                                float* __restrict__ shared_gate, int* cnt) {
  const int lane = threadIdx.x & 31;
  int e;
  float v;
  warp_select_exact([&](int ee) { return row[ee]; }, wn, nx, gamma, E, K, x + size_t(t) * H,
                    w_router, H, stats, e, v);
  const float wk = warp_topk_weight(v, K);
  if (lane < K) {
    topk_idx[size_t(t) * K + lane] = e;
    topk_w[size_t(t) * K + lane] = wk;
    atomicAdd(&cnt[e], 1);
  }
  if (lane == 0) shared_gate[t] = 1.0f / (1.0f + __expf(-row[E]));
}

}  // namespace pmoe
