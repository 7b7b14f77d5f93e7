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
//     tensor-core MMA step (k = 16) is taken to add at most 2^-22 * S to the
//     error, S = sum_i |x_i w_i| (two units in the last place of fp32: the
//     published measurements of fp32-accumulating tensor cores, Fasi, Higham,
//     Mikaitis, Pranesh, "Numerical behavior of NVIDIA tensor cores", PeerJ
//     CS 2021, show at most one per step), and each fp32 addition of partial
//     sums (round to nearest) at most 2^-24 * S.  A path with M steps and A
//     additions therefore has |a - exact| <= (M 2^-22 + A 2^-24) S <=
//     gamma * ||x||_2 * ||w||_2 (Cauchy-Schwarz), with slack for the fp32
//     norms.  The GPU tests check the observed error against this bound with
//     a wide margin.
//  2. Interval selection.  Each expert's logit lies in [RN(a - d), RN(a + d)]
//     (RN = round to bf16, monotone), d = gamma * ||x|| * ||w_e||.  The K
//     largest lower ends (ties to the lower expert) are the answer when no
//     other expert's upper end reaches the K-th lower end and consecutive
//     winners' intervals are ordered; otherwise every expert whose interval
//     is wider than one value and reaches the K-th lower end is evaluated
//     exactly (step 3) and the selection is redone on exact keys.
//  3. Exact evaluation (one warp), in integer arithmetic: a product of two
//     bf16 values is a 16-bit integer times a power of two; relative to the
//     smallest exponent the two rows allow, every product is an integer,
//     summed exactly in 128 bits (positive and negative parts), then rounded
//     once to bf16.  Exact whenever the rows' exponent spread leaves the
//     room (the smallest non-zero entries within 2^90 or so of the largest);
//     a row outside it is counted in a statistics word.  (FP64 is avoided:
//     on this part double-precision throughput is a small fraction of the
//     integer rate.)
// The token rows are read through L2 (ld.global.cg), not the read-only
// path: the decode routing kernel evaluates rows of the RMSNorm output that
// other CTAs of the same launch wrote.
#pragma once
#include "pmoe_common.cuh"

namespace pmoe {

// Error units of the model above -- a tensor-core MMA step, an fp32 addition
// rounded to nearest (at most half an ulp: 2^-24 of its result) -- and the
// slack factor on top that covers the fp32 arithmetic of the norms and of d.
constexpr float kAccStepErr = 0x1p-22f;
constexpr float kAddErr = 0x1p-24f;
constexpr float kBoundSlack = 1.0f + 0x1p-8f;

// gamma of an accumulation of `mma_steps` tensor-core steps followed by
// `adds` fp32 additions of partial sums.
__host__ __device__ constexpr float accumulation_gamma(int mma_steps, int adds) {
  return float(mma_steps) * kAccStepErr + float(adds) * kAddErr;
}

// Statistics words of the exact selection (in the workspace status array).
struct ExactStats {
  int* n_exact;    // exact evaluations run
  int* n_inexact;  // of which outside the exactness condition
};

// bf16 bit pattern -> sign, integer significand and exponent: |value| =
// mag * 2^k (subnormals: exponent field 0 counts as 1, no implicit bit).
__device__ __forceinline__ void bf16_parts(uint32_t b, uint32_t& mag, int& k, bool& neg) {
  const uint32_t E = (b >> 7) & 0xFFu, f = b & 0x7Fu;
  neg = (b >> 15) & 1u;
  mag = E ? (f | 0x80u) : f;
  k = (E ? int(E) : 1) - 134;
}

// 128-bit unsigned accumulator (hi, lo).
struct U128 {
  unsigned long long hi, lo;
};
__device__ __forceinline__ void u128_add(U128& a, const U128& b) {
  const unsigned long long lo = a.lo + b.lo;
  a.hi += b.hi + (lo < a.lo ? 1ull : 0ull);
  a.lo = lo;
}
// a += m * 2^sh, 0 <= sh <= 111, m < 2^16
__device__ __forceinline__ void u128_add_shifted(U128& a, unsigned long long m, int sh) {
  U128 v;
  if (sh >= 64) {
    v.lo = 0ull;
    v.hi = m << (sh - 64);
  } else {
    v.lo = m << sh;
    v.hi = sh > 48 ? m >> (64 - sh) : 0ull;
  }
  u128_add(a, v);
}
__device__ __forceinline__ U128 u128_shfl_xor(const U128& a, int o) {
  U128 r;
  r.hi = __shfl_xor_sync(0xffffffffu, a.hi, o);
  r.lo = __shfl_xor_sync(0xffffffffu, a.lo, o);
  return r;
}
__device__ __forceinline__ int u128_bitlen(const U128& a) {
  return a.hi ? 128 - __clzll((long long)a.hi) : (a.lo ? 64 - __clzll((long long)a.lo) : 0);
}
// bit i of a, and a >> d (0 < d < 128)
__device__ __forceinline__ unsigned long long u128_shr_low(const U128& a, int d) {
  if (d >= 64) return a.hi >> (d - 64);
  return (a.lo >> d) | (a.hi << (64 - d));
}
__device__ __forceinline__ bool u128_low_bits_nonzero(const U128& a, int d) {  // a mod 2^d != 0
  if (d >= 128) return a.hi || a.lo;
  if (d >= 64) return a.lo || (a.hi & ((1ull << (d - 64)) - 1ull));
  return d > 0 && (a.lo & ((1ull << d) - 1ull));
}
__device__ __forceinline__ bool u128_bit(const U128& a, int i) {
  return i >= 64 ? (a.hi >> (i - 64)) & 1ull : (a.lo >> i) & 1ull;
}

// Exponent of a bf16 magnitude pattern (sign cleared, non-zero): |value| =
// mag * 2^k, mag the integer significand (subnormals: field 0 counts as 1).
__device__ __forceinline__ int bf16_k(uint32_t a) {
  const int E = int(a >> 7);
  return (E ? E : 1) - 134;
}

// bf16 nearest (ties to even) to mag * 2^kb, mag a 128-bit magnitude; the
// sign is applied after.
__device__ __forceinline__ float round_mag_bf16(const U128& mag, bool negative, int kb) {
  const int bl = u128_bitlen(mag);
  if (bl == 0) return 0.0f;
  // keep 8 significant bits, or the bf16 subnormal grid 2^-133
  const int drop = max(bl - 8, -133 - kb);
  unsigned long long q;
  int qe;
  if (drop <= 0) {
    q = mag.lo;  // bl <= 8: fits
    qe = kb;
  } else {
    q = u128_shr_low(mag, drop);
    const bool half = u128_bit(mag, drop - 1);
    const bool sticky = u128_low_bits_nonzero(mag, drop - 1);
    if (half && (sticky || (q & 1ull))) ++q;
    qe = kb + drop;
  }
  const float r = ldexpf(float(q), qe);  // q <= 256: exact
  return negative ? -r : r;
}

// |pos - neg| rounded to bf16 with its sign (units 2^kb).
__device__ __forceinline__ float round_u128_bf16(const U128& pos, const U128& neg, int kb) {
  const bool pos_ge = pos.hi > neg.hi || (pos.hi == neg.hi && pos.lo >= neg.lo);
  const U128& big = pos_ge ? pos : neg;
  const U128& sml = pos_ge ? neg : pos;
  U128 mag;
  mag.lo = big.lo - sml.lo;
  mag.hi = big.hi - sml.hi - (big.lo < sml.lo ? 1ull : 0ull);
  return round_mag_bf16(mag, !pos_ge, kb);
}

// v * 2^sh as a 128-bit two's-complement number (0 <= sh < 128).
__device__ __forceinline__ U128 s128_shl(long long v, int sh) {
  unsigned long long lo = (unsigned long long)v, hi = v < 0 ? ~0ull : 0ull;
  if (sh >= 64) {
    hi = lo << (sh - 64);
    lo = 0ull;
  } else if (sh > 0) {
    hi = (hi << sh) | (lo >> (64 - sh));
    lo <<= sh;
  }
  return U128{hi, lo};
}

// One product of the general path: integer significands and exponents from
// the bf16 fields, added to pos / neg in units of 2^kb (dropped below it).
__device__ __forceinline__ void exact_add_general(uint32_t xb, uint32_t wb, int kb, U128& pos,
                                                  U128& neg) {
  uint32_t mx, mw;
  int kx, kw;
  bool nx, nw;
  bf16_parts(xb, mx, kx, nx);
  bf16_parts(wb, mw, kw, nw);
  const uint32_t m = mx * mw;
  const int sh = kx + kw - kb;
  if (m == 0u || sh < 0) return;
  if (nx != nw)
    u128_add_shifted(neg, m, sh);
  else
    u128_add_shifted(pos, m, sh);
}

// The fast path's products of one 32-bit word pair (two bf16 each): fp32
// multiplies (exact: 16 significant bits, normal numbers by the caller's
// check), |p| = m16 * 2^(e - 142) from the bits, with sh = e - eb, added as
// a signed integer to window sh / W of the lane's accumulators (window w
// holds units of 2^(kb + w W); each term is below 2^(16 + W), so 2^lg of
// them stay below 2^62).  Even and odd products use separate accumulators.
__device__ __forceinline__ void exact_word_fast(uint32_t xw, uint32_t ww, int eb, int W,
                                                long long (&acc)[2][3]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t xb = h ? xw & 0xFFFF0000u : xw << 16;
    const uint32_t wb = h ? ww & 0xFFFF0000u : ww << 16;
    const uint32_t pb = __float_as_uint(__fmul_rn(__uint_as_float(xb), __uint_as_float(wb)));
    const int e = int((pb >> 23) & 0xFFu);
    long long m = e ? (long long)(((pb >> 8) & 0x7FFFu) | 0x8000u) : 0ll;
    if (pb >> 31) m = -m;
    const int sh = e ? e - eb : 0;
    const int wi = (sh >= W) + (sh >= 2 * W);
    const long long v = (long long)((unsigned long long)m << (sh - wi * W));
    acc[h][0] += wi == 0 ? v : 0ll;
    acc[h][1] += wi == 1 ? v : 0ll;
    acc[h][2] += wi == 2 ? v : 0ll;
  }
}

// The general path's sums of this lane's products (rare: bf16 subnormals,
// extreme exponents or a spread beyond the fast path's window).
static __device__ __noinline__ void exact_sums_general(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       int n, int kb, U128& pos, U128& neg) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int i = lane * 8; i < n; i += 256) {
    uint4 xv = __ldcg(reinterpret_cast<const uint4*>(x + i));
    uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + i));
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      exact_add_general(xv.x & 0xFFFFu, wv.x & 0xFFFFu, kb, pos, neg);
      exact_add_general(xv.x >> 16, wv.x >> 16, kb, pos, neg);
      xv = make_uint4(xv.y, xv.z, xv.w, 0u);
      wv = make_uint4(wv.y, wv.z, wv.w, 0u);
    }
  }
}

// Exact x . w (bf16 rows of length n, n % 256 == 0, 16-byte aligned), rounded
// to bf16 (ties to even); all lanes of the warp return the same value.
// A product of two bf16 values is a 16-bit integer times a power of two;
// relative to the smallest exponent the rows allow (kb), every product is an
// integer, summed exactly in 128 bits (positive and negative parts), then
// rounded once.  Exact while the exponent spread of the two rows leaves the
// room: 16 + span + 2 + log2(n) < 127 (the smallest non-zero entries within
// about 2^90 of the largest); a wider spread drops the products below the
// window and reports ok = false.  Fast path: when every product is a normal
// fp32 number (no bf16 subnormals, no huge exponents) the products are formed
// with one fp32 multiply each and their bits give the integer significand
// and exponent.  The loops are kept rolled: this code runs a few times per
// call, so a compact body (instruction-cache resident) matters more than
// unrolling.
static __device__ __noinline__ float warp_exact_dot(const __nv_bfloat16* __restrict__ x,
                                                    const __nv_bfloat16* __restrict__ w, int n,
                                                    bool& ok) {
  constexpr int kChunk = 8;  // 16-byte pieces per lane per chunk (2048 elements)
  const int lane = threadIdx.x & 31;
  int kb = 0;
  U128 pos{0ull, 0ull}, neg{0ull, 0ull};
  ok = true;
  // One chunk of up to 2048 elements per pass, all of its loads issued before
  // any is used (the rows are read from L2 or HBM: a load per loop iteration
  // would serialise that latency).
  auto load_chunk = [&](int c0, uint4 (&xv)[kChunk], uint4 (&wv)[kChunk]) {
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      const int o = c0 + (i * 32 + lane) * 8;
      xv[i] = o < n ? __ldcg(reinterpret_cast<const uint4*>(x + o)) : make_uint4(0u, 0u, 0u, 0u);
      wv[i] = o < n ? __ldg(reinterpret_cast<const uint4*>(w + o)) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // pass 1: largest and smallest non-zero magnitude patterns (16-bit SIMD)
  uint32_t xmx = 0u, xmn = 0x7FFF7FFFu, wmx = 0u, wmn = 0x7FFF7FFFu;
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 256 * kChunk) {
    uint4 xv[kChunk], wv[kChunk];
    load_chunk(c0, xv, wv);
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      const uint32_t xs[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
      const uint32_t ws[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t ax = xs[j] & 0x7FFF7FFFu, aw = ws[j] & 0x7FFF7FFFu;
        xmx = __vmaxu2(xmx, ax);
        wmx = __vmaxu2(wmx, aw);
        xmn = __vminu2(xmn, ax | (__vcmpeq2(ax, 0u) & 0x7FFF7FFFu));
        wmn = __vminu2(wmn, aw | (__vcmpeq2(aw, 0u) & 0x7FFF7FFFu));
      }
    }
  }
  const uint32_t xmax = __reduce_max_sync(0xffffffffu, max(xmx & 0xFFFFu, xmx >> 16));
  const uint32_t wmax = __reduce_max_sync(0xffffffffu, max(wmx & 0xFFFFu, wmx >> 16));
  const uint32_t xmin = __reduce_min_sync(0xffffffffu, min(xmn & 0xFFFFu, xmn >> 16));
  const uint32_t wmin = __reduce_min_sync(0xffffffffu, min(wmn & 0xFFFFu, wmn >> 16));
  ok = xmax < 0x7F80u && wmax < 0x7F80u;  // finite
  if (xmax == 0u || wmax == 0u) return 0.0f;  // a row of zeros
  const int kmax = bf16_k(xmax) + bf16_k(wmax), kmin = bf16_k(xmin) + bf16_k(wmin);
  const int lg = 32 - __clz(n + 63);
  const int room = 127 - 16 - 2 - lg;  // largest shift that keeps the sums in 128 bits
  const bool normal = (xmin >> 7) != 0u && (wmin >> 7) != 0u;  // no bf16 subnormals
  const bool fast = normal && kmin >= -140 && kmax <= 110 && kmax + 2 - kmin <= room;
  if (fast) {
    kb = kmin - 1;  // the smallest product's exponent field is kmin + 141
    const int eb = kmin + 141;
    const int W = 62 - 16 - lg;  // bits per accumulator window
    long long acc[2][3] = {{0ll, 0ll, 0ll}, {0ll, 0ll, 0ll}};
#pragma unroll 1
    for (int c0 = 0; c0 < n; c0 += 256 * kChunk) {
      uint4 xv[kChunk], wv[kChunk];
      load_chunk(c0, xv, wv);
      // rolled over the chunk's pieces: piece 0 is consumed, the rest moves up
#pragma unroll 1
      for (int i = 0; i < kChunk; ++i) {
        const uint4 xa = xv[0], wa = wv[0];
#pragma unroll
        for (int q = 0; q < kChunk - 1; ++q) {
          xv[q] = xv[q + 1];
          wv[q] = wv[q + 1];
        }
        exact_word_fast(xa.x, wa.x, eb, W, acc);
        exact_word_fast(xa.y, wa.y, eb, W, acc);
        exact_word_fast(xa.z, wa.z, eb, W, acc);
        exact_word_fast(xa.w, wa.w, eb, W, acc);
      }
    }
    // the windows as one 128-bit two's-complement sum; the warp's sums
    // (|total| < 2^(16 + span + 2 + lg) < 2^127)
    U128 tot = s128_shl(acc[0][0] + acc[1][0], 0);
    u128_add(tot, s128_shl(acc[0][1] + acc[1][1], W));
    u128_add(tot, s128_shl(acc[0][2] + acc[1][2], 2 * W));
#pragma unroll 1
    for (int o = 16; o > 0; o >>= 1) u128_add(tot, u128_shfl_xor(tot, o));
    const bool negative = tot.hi >> 63;
    if (negative) {  // two's-complement negate
      tot.lo = ~tot.lo + 1ull;
      tot.hi = ~tot.hi + (tot.lo == 0ull ? 1ull : 0ull);
    }
    return round_mag_bf16(tot, negative, kb);
  } else {
    kb = kmin;
    if (kmax + 2 - kb > room) {
      kb = kmax + 2 - room;
      ok = false;
    }
    exact_sums_general(x, w, n, kb, pos, neg);
  }
#pragma unroll 1
  for (int o = 16; o > 0; o >>= 1) {
    u128_add(pos, u128_shfl_xor(pos, o));
    u128_add(neg, u128_shfl_xor(neg, o));
  }
  return round_u128_bf16(pos, neg, kb);
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

// The interval selection in full (see the file comment), for a token whose
// order the fast check of warp_select_exact could not settle.
template <typename LogitFn>
__device__ __noinline__ void warp_select_intervals(LogitFn lg, const float* __restrict__ wn,
                                                      float gx, int E, int K,
                                                      const __nv_bfloat16* __restrict__ x_row,
                                                      const __nv_bfloat16* __restrict__ w_router,
                                                      int H, ExactStats stats, int& e_out,
                                                      float& v_out) {
  const int lane = threadIdx.x & 31;
  uint32_t klo[8], khi[8];
  float val[8];
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
  // the K-th largest lower end
  uint32_t Lk = 0u;
  {
    uint32_t tmp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) tmp[j] = klo[j];
    for (int k = 0; k < K; ++k) {
      uint32_t m = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) m = max(m, tmp[j]);
      Lk = __reduce_max_sync(0xffffffffu, m);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (tmp[j] == Lk) tmp[j] = 0u;
    }
  }
  // Candidates: upper end at least Lk (no other expert can be among the K
  // largest).  An uncertain candidate (interval wider than one value) is
  // evaluated exactly when its interval overlaps another candidate's;
  // afterwards all candidate intervals are disjoint (keys are unique by
  // expert), so their order is the order of the lower ends.
  uint32_t cand = 0u, ov = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j * 32 + lane < E && khi[j] >= Lk) cand |= 1u << j;
#pragma unroll
  for (int j2 = 0; j2 < 8; ++j2) {
    unsigned cm = __ballot_sync(0xffffffffu, cand >> j2 & 1u);
    while (cm) {
      const int l = __ffs(cm) - 1;
      cm &= cm - 1;
      const uint32_t c_lo = __shfl_sync(0xffffffffu, klo[j2], l);
      const uint32_t c_hi = __shfl_sync(0xffffffffu, khi[j2], l);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if ((cand >> j & 1u) && !(j == j2 && lane == l) && klo[j] <= c_hi && khi[j] >= c_lo)
          ov |= 1u << j;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool unc = (ov >> j & 1u) && (khi[j] >> 16) != (klo[j] >> 16);
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
  uint32_t mine = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (!(cand >> j & 1u)) klo[j] = 0u;  // cannot be among the K largest
  for (int k = 0; k < K; ++k) {
    uint32_t m = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) m = max(m, klo[j]);
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, m);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (klo[j] == wmax) klo[j] = 0u;
    if (lane == k) mine = wmax;
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

// The fast check: top K of the rounded approximations RN(a), with the
// intervals of only those K and the largest upper end of all other experts.
// When these intervals are ordered and apart, that selection is the exact
// one: certain[i] is true with lane k < K holding the k-th expert and its
// value.  NT tokens at once (lg(i, e): token i's approximation of expert e),
// their steps interleaved so that the warp reductions of different tokens
// overlap.
template <int NT, typename LogitFn>
__device__ __forceinline__ void warp_fast_check_n(LogitFn lg, const float* __restrict__ wn,
                                                  const float (&gx)[NT], int E, int K,
                                                  int (&e_out)[NT], float (&v_out)[NT],
                                                  bool (&certain)[NT]) {
  const int lane = threadIdx.x & 31;
  float av[NT][8];
  uint32_t key[NT][8];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = j * 32 + lane;
      av[i][j] = e < E ? lg(i, e) : 0.f;
      key[i][j] = e < E ? logit_key(bf16_round(av[i][j]), e) : 0u;
    }
  // top K of the rounded approximations (selected keys are zeroed in key[])
  uint32_t mine[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) mine[i] = 0u;
  for (int k = 0; k < K; ++k) {
    uint32_t wmax[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const uint32_t m = max(max(max(key[i][0], key[i][1]), max(key[i][2], key[i][3])),
                             max(max(key[i][4], key[i][5]), max(key[i][6], key[i][7])));
      wmax[i] = __reduce_max_sync(0xffffffffu, m);
    }
#pragma unroll
    for (int i = 0; i < NT; ++i) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (key[i][j] == wmax[i]) key[i][j] = 0u;
      if (lane == k) mine[i] = wmax[i];
    }
  }
  uint32_t mo[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    // largest upper end among the other experts
    uint32_t m = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (key[i][j]) {
        const int e = j * 32 + lane;
        m = max(m, logit_key(bf16_round(__fadd_ru(av[i][j], gx[i] * wn[e])), e));
      }
    }
    mo[i] = __reduce_max_sync(0xffffffffu, m);
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    // the K selected experts' intervals, lane k holding the k-th
    const int ek = lane < K ? 0xFFFF - int(mine[i] & 0xFFFFu) : 0;
    float ak = 0.f;
    uint32_t lo = 0u, hi = 0u;
    if (lane < K) {
      ak = lg(i, ek);
      const float d = gx[i] * wn[ek];
      lo = logit_key(bf16_round(__fsub_rd(ak, d)), ek);
      hi = logit_key(bf16_round(__fadd_ru(ak, d)), ek);
    }
    const uint32_t prev_lo = __shfl_up_sync(0xffffffffu, lo, 1);
    const uint32_t Lk = __shfl_sync(0xffffffffu, lo, K - 1);
    const bool bad = lane >= 1 && lane < K && !(prev_lo > hi);
    e_out[i] = ek;
    v_out[i] = bf16_round(ak);
    certain[i] = mo[i] < Lk && !__any_sync(0xffffffffu, bad);
  }
}

template <typename LogitFn>
__device__ __forceinline__ bool warp_fast_check(LogitFn lg, const float* __restrict__ wn,
                                                float gx, int E, int K, int& e_out,
                                                float& v_out) {
  const float g[1] = {gx};
  int e[1];
  float v[1];
  bool c[1];
  warp_fast_check_n<1>([&](int, int ee) { return lg(ee); }, wn, g, E, K, e, v, c);
  e_out = e[0];
  v_out = v[0];
  return c[0];
}

// Per-warp top-K of one token from its approximate logits (see the file
// comment).  `lg(e)` returns the fp32 approximation of expert e's logit,
// `wn` the experts' row norms, `nx` the token's norm, `gamma` the path's
// bound factor; x_row / w_router (row stride H) feed the exact evaluations.
// Lane k < K receives the k-th expert (descending) in `e_out` and its bf16
// logit in `v_out`; the weights follow from those (caller).  The warp does
// any exact evaluation itself (CTAs that can share the work use ExactCta).
template <typename LogitFn>
__device__ __forceinline__ void warp_select_exact(LogitFn lg, const float* __restrict__ wn,
                                                  float nx, float gamma, int E, int K,
                                                  const __nv_bfloat16* __restrict__ x_row,
                                                  const __nv_bfloat16* __restrict__ w_router,
                                                  int H, ExactStats stats, int& e_out,
                                                  float& v_out) {
  const float gx = gamma * kBoundSlack * nx;
  if (warp_fast_check(lg, wn, gx, E, K, e_out, v_out)) return;
  warp_select_intervals(lg, wn, gx, E, K, x_row, w_router, H, stats, e_out, v_out);
}

// Renormalised top-K weights (router :765-768): softmax over all experts,
// top K, divided by their sum == exp(l_k - l_0) / sum_j exp(l_j - l_0) over
// the K selected.  Lanes >= K return 0.
__device__ __forceinline__ float warp_topk_weight(float v, int K) {
  const int lane = threadIdx.x & 31;
  const float l0 = __shfl_sync(0xffffffffu, v, 0);
  const float ex = lane < K ? expf(v - l0) : 0.f;
  float den = ex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  return ex / den;
}

// Sum of squares of a bf16 row (n % 256 == 0) by one warp; all lanes get it.
// The loads of up to 2048 elements are all issued before any is used.
__device__ __forceinline__ float warp_row_sumsq(const __nv_bfloat16* __restrict__ r, int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += 2048) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int o = c0 + (i * 32 + lane) * 8;
      v[i] = o < n ? __ldg(reinterpret_cast<const uint4*>(r + o)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(u[j] << 16), hi = __uint_as_float(u[j] & 0xFFFF0000u);
        s = fmaf(lo, lo, s);
        s = fmaf(hi, hi, s);
      }
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
// CTA-cooperative exact top-k.  One evaluation by one warp is a long serial
// stream (2048 products, 64 per lane); here the warps of a CTA first settle
// every token they can with the fast check, queue the remaining tokens'
// candidate intervals and the exact evaluations those need, and then all
// warps evaluate each queued logit together (H / NW elements per warp), in
// three barrier-separated steps: exponent ranges, partial exact sums,
// rounding.  A token whose candidates or evaluations exceed the queue takes
// the warp-level path instead.
// ---------------------------------------------------------------------------
constexpr int kXMaxCand = 32;  // candidates per queued token
constexpr int kXMaxReq = 32;   // queued evaluations per CTA round

template <int NW, int MAXPEND>
struct ExactCta {
  struct Pend {
    int t, nc;
    uint32_t klo[kXMaxCand], khi[kXMaxCand];
    float val[kXMaxCand];
  };
  struct Req {
    int slot, ci, e, t;
    unsigned int xmax, wmax, xmin, wmin;
    U128 part[NW];
  };
  Pend pend[MAXPEND];
  Req req[kXMaxReq];
  int n_pend, n_req;
};

// Writes token t's routing from lane k's (expert, bf16 logit); cnt: the
// expert counts this token is added to.
__device__ __forceinline__ void warp_write_route(int t, int K, int e, float v,
                                                 int32_t* __restrict__ topk_idx,
                                                 float* __restrict__ topk_w, int* cnt) {
  const int lane = threadIdx.x & 31;
  const float wk = warp_topk_weight(v, K);
  if (lane < K) {
    topk_idx[size_t(t) * K + lane] = e;
    topk_w[size_t(t) * K + lane] = wk;
    atomicAdd(&cnt[e], 1);
  }
}

// Queue token t, which the fast check could not settle (gx = gamma * slack
// * ||x_t||): its candidates' intervals and the exact evaluations they need;
// a token that does not fit the queue is settled here by warp_select_intervals.
template <int NW, int MAXPEND, typename LogitFn, typename CntFn>
__device__ __forceinline__ void warp_topk_queue(
    ExactCta<NW, MAXPEND>& sm, LogitFn lg, const float* __restrict__ wn, float gx, int t, int E,
    int K, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_router,
    int H, ExactStats stats, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    CntFn cnt_of) {
  const int lane = threadIdx.x & 31;
  int e;
  float v;
  // the intervals of all experts (as warp_select_intervals)
  uint32_t klo[8], khi[8];
  float val[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int ee = j * 32 + lane;
    klo[j] = khi[j] = 0u;
    val[j] = 0.f;
    if (ee < E) {
      const float a = lg(ee);
      const float d = gx * wn[ee];
      klo[j] = logit_key(bf16_round(__fsub_rd(a, d)), ee);
      khi[j] = logit_key(bf16_round(__fadd_ru(a, d)), ee);
      val[j] = bf16_round(a);
    }
  }
  uint32_t Lk = 0u;
  {
    uint32_t tmp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) tmp[j] = klo[j];
    for (int k = 0; k < K; ++k) {
      const uint32_t m = max(max(max(tmp[0], tmp[1]), max(tmp[2], tmp[3])),
                             max(max(tmp[4], tmp[5]), max(tmp[6], tmp[7])));
      Lk = __reduce_max_sync(0xffffffffu, m);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (tmp[j] == Lk) tmp[j] = 0u;
    }
  }
  uint32_t cand = 0u, ov = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j * 32 + lane < E && khi[j] >= Lk) cand |= 1u << j;
#pragma unroll
  for (int j2 = 0; j2 < 8; ++j2) {
    unsigned cm = __ballot_sync(0xffffffffu, cand >> j2 & 1u);
    while (cm) {
      const int l = __ffs(cm) - 1;
      cm &= cm - 1;
      const uint32_t c_lo = __shfl_sync(0xffffffffu, klo[j2], l);
      const uint32_t c_hi = __shfl_sync(0xffffffffu, khi[j2], l);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if ((cand >> j & 1u) && !(j == j2 && lane == l) && klo[j] <= c_hi && khi[j] >= c_lo)
          ov |= 1u << j;
    }
  }
  uint32_t unc = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if ((ov >> j & 1u) && (khi[j] >> 16) != (klo[j] >> 16)) unc |= 1u << j;
  int nc = 0, nr = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    nc += __popc(__ballot_sync(0xffffffffu, cand >> j & 1u));
    nr += __popc(__ballot_sync(0xffffffffu, unc >> j & 1u));
  }
  int slot = -1, rbase = 0;
  if (lane == 0 && nc <= kXMaxCand) {
    slot = atomicAdd(&sm.n_pend, 1);
    rbase = nr ? atomicAdd(&sm.n_req, nr) : 0;
    if (slot >= MAXPEND || rbase + nr > kXMaxReq) {
      // no room: invalidate what was reserved, evaluate in this warp
      for (int i = rbase; i < min(rbase + nr, kXMaxReq); ++i) sm.req[i].slot = -1;
      if (slot < MAXPEND) sm.pend[slot].nc = -1;
      slot = -1;
    }
  }
  slot = __shfl_sync(0xffffffffu, slot, 0);
  rbase = __shfl_sync(0xffffffffu, rbase, 0);
  if (slot < 0) {
    warp_select_intervals(lg, wn, gx, E, K, x + size_t(t) * H, w_router, H, stats, e, v);
    warp_write_route(t, K, e, v, topk_idx, topk_w, cnt_of(t));
    return;
  }
  auto& P = sm.pend[slot];
  const unsigned lt = (1u << lane) - 1u;
  int ci = 0, ri = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const unsigned cm = __ballot_sync(0xffffffffu, cand >> j & 1u);
    const unsigned um = __ballot_sync(0xffffffffu, unc >> j & 1u);
    if (cand >> j & 1u) {
      const int c = ci + __popc(cm & lt);
      P.klo[c] = klo[j];
      P.khi[c] = khi[j];
      P.val[c] = val[j];
      if (unc >> j & 1u) {
        auto& q = sm.req[rbase + ri + __popc(um & lt)];
        q.slot = slot;
        q.ci = c;
        q.e = j * 32 + lane;
        q.t = t;
        q.xmax = q.wmax = 0u;
        q.xmin = q.wmin = 0x7FFFu;
      }
    }
    ci += __popc(cm);
    ri += __popc(um);
  }
  if (lane == 0) {
    P.t = t;
    P.nc = nc;
  }
}

// Step A (one warp, token t): settle it, or queue it.  `sm.n_pend` and
// `sm.n_req` must be zero (and visible) before the CTA's first call.
template <int NW, int MAXPEND, typename LogitFn, typename CntFn>
__device__ __forceinline__ void warp_topk_stage(
    ExactCta<NW, MAXPEND>& sm, LogitFn lg, const float* __restrict__ wn, float nx, float gamma,
    int t, int E, int K, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w_router, int H, ExactStats stats,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, CntFn cnt_of) {
  const float gx = gamma * kBoundSlack * nx;
  int e;
  float v;
  if (warp_fast_check(lg, wn, gx, E, K, e, v)) {
    warp_write_route(t, K, e, v, topk_idx, topk_w, cnt_of(t));
    return;
  }
  warp_topk_queue(sm, lg, wn, gx, t, E, K, x, w_router, H, stats, topk_idx, topk_w, cnt_of);
}

// Step A for two tokens of one warp, their fast checks interleaved
// (valid1 false: only t0).
template <int NW, int MAXPEND, typename LogitFn2, typename CntFn>
__device__ __forceinline__ void warp_topk_stage2(
    ExactCta<NW, MAXPEND>& sm, LogitFn2 lg, const float* __restrict__ wn, float nx0, float nx1,
    float gamma, int t0, int t1, bool valid1, int E, int K, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w_router, int H, ExactStats stats,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, CntFn cnt_of) {
  if (!valid1) {
    warp_topk_stage(sm, [&](int ee) { return lg(0, ee); }, wn, nx0, gamma, t0, E, K, x, w_router,
                    H, stats, topk_idx, topk_w, cnt_of);
    return;
  }
  const float gx[2] = {gamma * kBoundSlack * nx0, gamma * kBoundSlack * nx1};
  int e[2];
  float v[2];
  bool ok[2];
  warp_fast_check_n<2>(lg, wn, gx, E, K, e, v, ok);
  const int ts[2] = {t0, t1};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if (ok[i])
      warp_write_route(ts[i], K, e[i], v[i], topk_idx, topk_w, cnt_of(ts[i]));
    else
      warp_topk_queue(sm, [&](int ee) { return lg(i, ee); }, wn, gx[i], ts[i], E, K, x, w_router,
                      H, stats, topk_idx, topk_w, cnt_of);
  }
}

// Steps B and C, by every thread of the CTA (contains __syncthreads).
template <int NW, int MAXPEND, typename CntFn>
__device__ __forceinline__ void cta_topk_finish(ExactCta<NW, MAXPEND>& sm,
                                                const __nv_bfloat16* __restrict__ x,
                                                const __nv_bfloat16* __restrict__ w_router,
                                                int H, int K, ExactStats stats,
                                                int32_t* __restrict__ topk_idx,
                                                float* __restrict__ topk_w, CntFn cnt_of) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __syncthreads();
  const int nreq = min(sm.n_req, kXMaxReq);
  const int npend = min(sm.n_pend, MAXPEND);
  const int chunk = H / NW;  // elements per warp (a multiple of 16)
  const int lg = 32 - __clz(H + 63);
  const int room = 127 - 16 - 2 - lg;
  if (nreq > NW / 4) {
    // Many evaluations: one warp per evaluation (warp_exact_dot, the same
    // exactly rounded value), so their row loads are independent instead of
    // one dependent round trip per evaluation in every warp.
    for (int r = warp; r < nreq; r += NW) {
      const auto& q = sm.req[r];
      if (q.slot < 0) continue;
      bool ok;
      const float rv = warp_exact_dot(x + size_t(q.t) * H, w_router + size_t(q.e) * H, H, ok);
      if (lane == 0) {
        auto& P = sm.pend[q.slot];
        P.klo[q.ci] = P.khi[q.ci] = logit_key(rv, q.e);
        P.val[q.ci] = rv;
        atomicAdd(stats.n_exact, 1);
        if (!ok) atomicAdd(stats.n_inexact, 1);
      }
    }
    __syncthreads();
  } else if (nreq > 0) {
    // Few evaluations (decode): each is split over the warps.
    // B1: exponent ranges of the queued rows (the loads of every request of
    // this warp's pass are issued before any is used: up to 4 at a time)
    for (int r0 = 0; r0 < nreq; r0 += 4) {
      uint2 xv[4], wv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r0 + j;
        const bool live = r < nreq && sm.req[r].slot >= 0 && lane < chunk / 4;
        xv[j] = wv[j] = make_uint2(0u, 0u);
        if (live) {
          const auto& q = sm.req[r];
          xv[j] = __ldcg(reinterpret_cast<const uint2*>(x + size_t(q.t) * H + warp * chunk) + lane);
          wv[j] = __ldg(reinterpret_cast<const uint2*>(w_router + size_t(q.e) * H + warp * chunk) +
                        lane);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r0 + j;
        if (r >= nreq || sm.req[r].slot < 0) continue;
        auto& q = sm.req[r];
        uint32_t xmx = 0u, xmn = 0x7FFF7FFFu, wmx = 0u, wmn = 0x7FFF7FFFu;
        for (int u = lane; u < chunk / 4; u += 32) {
          const uint2 xa = u == lane ? xv[j] : __ldcg(reinterpret_cast<const uint2*>(
                                                   x + size_t(q.t) * H + warp * chunk) + u);
          const uint2 wa = u == lane ? wv[j] : __ldg(reinterpret_cast<const uint2*>(
                                                   w_router + size_t(q.e) * H + warp * chunk) + u);
          const uint32_t xs[2] = {xa.x, xa.y}, ws[2] = {wa.x, wa.y};
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const uint32_t ax = xs[k] & 0x7FFF7FFFu, aw = ws[k] & 0x7FFF7FFFu;
            xmx = __vmaxu2(xmx, ax);
            wmx = __vmaxu2(wmx, aw);
            xmn = __vminu2(xmn, ax | (__vcmpeq2(ax, 0u) & 0x7FFF7FFFu));
            wmn = __vminu2(wmn, aw | (__vcmpeq2(aw, 0u) & 0x7FFF7FFFu));
          }
        }
        const uint32_t a = __reduce_max_sync(0xffffffffu, max(xmx & 0xFFFFu, xmx >> 16));
        const uint32_t b = __reduce_max_sync(0xffffffffu, max(wmx & 0xFFFFu, wmx >> 16));
        const uint32_t c = __reduce_min_sync(0xffffffffu, min(xmn & 0xFFFFu, xmn >> 16));
        const uint32_t d = __reduce_min_sync(0xffffffffu, min(wmn & 0xFFFFu, wmn >> 16));
        if (lane == 0) {
          atomicMax(&q.xmax, a);
          atomicMax(&q.wmax, b);
          atomicMin(&q.xmin, c);
          atomicMin(&q.wmin, d);
        }
      }
    }
    __syncthreads();
    // B2: each warp's exact partial sum of its elements (two's complement,
    // units 2^kb of the whole row)
    for (int r = 0; r < nreq; ++r) {
      auto& q = sm.req[r];
      if (q.slot < 0) continue;
      const unsigned xmax = q.xmax, wmax = q.wmax, xmin = q.xmin, wmin = q.wmin;
      U128 tot{0ull, 0ull};
      if (xmax != 0u && wmax != 0u) {
        const int kmax = bf16_k(xmax) + bf16_k(wmax), kmin = bf16_k(xmin) + bf16_k(wmin);
        const bool normal = (xmin >> 7) != 0u && (wmin >> 7) != 0u;
        const bool fast = normal && kmin >= -140 && kmax <= 110 && kmax + 2 - kmin <= room;
        const uint2* xr = reinterpret_cast<const uint2*>(x + size_t(q.t) * H + warp * chunk);
        const uint2* wr =
            reinterpret_cast<const uint2*>(w_router + size_t(q.e) * H + warp * chunk);
        if (fast) {
          const int eb = kmin + 141, W = 62 - 16 - lg;
          long long acc[2][3] = {{0ll, 0ll, 0ll}, {0ll, 0ll, 0ll}};
          for (int u = lane; u < chunk / 4; u += 32) {
            const uint2 xv = __ldcg(xr + u), wv = __ldg(wr + u);
            exact_word_fast(xv.x, wv.x, eb, W, acc);
            exact_word_fast(xv.y, wv.y, eb, W, acc);
          }
          tot = s128_shl(acc[0][0] + acc[1][0], 0);
          u128_add(tot, s128_shl(acc[0][1] + acc[1][1], W));
          u128_add(tot, s128_shl(acc[0][2] + acc[1][2], 2 * W));
        } else {
          int kb = kmin;
          if (kmax + 2 - kb > room) kb = kmax + 2 - room;
          U128 pos{0ull, 0ull}, neg{0ull, 0ull};
          for (int u = lane; u < chunk / 4; u += 32) {
            const uint2 xv = __ldcg(xr + u), wv = __ldg(wr + u);
            exact_add_general(xv.x & 0xFFFFu, wv.x & 0xFFFFu, kb, pos, neg);
            exact_add_general(xv.x >> 16, wv.x >> 16, kb, pos, neg);
            exact_add_general(xv.y & 0xFFFFu, wv.y & 0xFFFFu, kb, pos, neg);
            exact_add_general(xv.y >> 16, wv.y >> 16, kb, pos, neg);
          }
          tot.lo = pos.lo - neg.lo;
          tot.hi = pos.hi - neg.hi - (pos.lo < neg.lo ? 1ull : 0ull);
        }
      }
#pragma unroll 1
      for (int o = 16; o > 0; o >>= 1) u128_add(tot, u128_shfl_xor(tot, o));
      if (lane == 0) q.part[warp] = tot;
    }
    __syncthreads();
    // B3: one thread per queued evaluation: the warps' sums, rounded once
    if (tid < nreq) {
      auto& q = sm.req[tid];
      if (q.slot >= 0) {
        const unsigned xmax = q.xmax, wmax = q.wmax, xmin = q.xmin, wmin = q.wmin;
        bool ok = xmax < 0x7F80u && wmax < 0x7F80u;
        float rv = 0.f;
        if (xmax != 0u && wmax != 0u) {
          const int kmax = bf16_k(xmax) + bf16_k(wmax), kmin = bf16_k(xmin) + bf16_k(wmin);
          const bool normal = (xmin >> 7) != 0u && (wmin >> 7) != 0u;
          const bool fast = normal && kmin >= -140 && kmax <= 110 && kmax + 2 - kmin <= room;
          int kb = fast ? kmin - 1 : kmin;
          if (!fast && kmax + 2 - kb > room) {
            kb = kmax + 2 - room;
            ok = false;
          }
          U128 tot = q.part[0];
          for (int w = 1; w < NW; ++w) u128_add(tot, q.part[w]);
          const bool negative = tot.hi >> 63;
          if (negative) {
            tot.lo = ~tot.lo + 1ull;
            tot.hi = ~tot.hi + (tot.lo == 0ull ? 1ull : 0ull);
          }
          rv = round_mag_bf16(tot, negative, kb);
        }
        auto& P = sm.pend[q.slot];
        P.klo[q.ci] = P.khi[q.ci] = logit_key(rv, q.e);
        P.val[q.ci] = rv;
        atomicAdd(stats.n_exact, 1);
        if (!ok) atomicAdd(stats.n_inexact, 1);
      }
    }
    __syncthreads();
  }
  // C: the queued tokens' selection; their candidates' intervals are now
  // disjoint, so the K largest lower ends are the answer
  for (int p = warp; p < npend; p += NW) {
    const auto& P = sm.pend[p];
    const int nc = P.nc;
    if (nc < 0) continue;
    uint32_t key = lane < nc ? P.klo[lane] : 0u;
    const float vl = lane < nc ? P.val[lane] : 0.f;
    int e = 0;
    float v = 0.f;
    for (int k = 0; k < K; ++k) {
      const uint32_t wmax = __reduce_max_sync(0xffffffffu, key);
      const int owner = __ffs(__ballot_sync(0xffffffffu, key == wmax && key != 0u)) - 1;
      const float vo = __shfl_sync(0xffffffffu, vl, owner < 0 ? 0 : owner);
      if (lane == k) {
        e = 0xFFFF - int(wmax & 0xFFFFu);
        v = vo;
      }
      if (key == wmax) key = 0u;
    }
    warp_write_route(P.t, K, e, v, topk_idx, topk_w, cnt_of(P.t));
  }
}

}  // namespace pmoe
