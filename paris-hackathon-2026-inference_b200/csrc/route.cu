// Router, top-k and CSR dispatch kernels.
//
// Reference arithmetic: Qwen3_5MoeTopKRouter.forward
// (transformers models/qwen3_5_moe/modeling_qwen3_5_moe.py:762-770) and the
// stable-sort dispatch of engine/kernels/moe_dispatch.py:119-137.
//
// Two paths:
//  * T <= kFusedRouteMaxT (decode): ONE launch.  Each CTA computes a
//    16-expert x 32-token tile of partial logits over one of KS K-ranges,
//    split over its 16 warps and reduced in shared memory in a fixed order;
//    the last CTA of each 32-token group (threadfence + atomic ticket) sums
//    the KS partials in a fixed order, rounds to bf16 and selects the
//    group's top-k; the last group does the histogram, the CSR offsets and
//    the stable permutation for all tokens.
//  * larger T: router GEMM tiles -> warp-per-token top-k -> one-CTA dispatch.
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tma.cuh"
#include "pmoe_exact.cuh"

namespace pmoe {

// Sum of squares of 8 packed bf16 (squares are exact in fp32).
__device__ __forceinline__ float sumsq8(const uint4& v) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __uint_as_float(u[j] << 16), hi = __uint_as_float(u[j] & 0xFFFF0000u);
    s = fmaf(lo, lo, s);
    s = fmaf(hi, hi, s);
  }
  return s;
}

// ---------------------------------------------------------------------------
// Router tile: 16 router rows (row E = shared gate vector, rows > E zero) x
// 32 tokens over k in [k_begin, k_begin + k_len), mma.sync with the permuted
// 128-bit operand layout of mma_k32.  acc[q][*] holds tokens q*8 + 2c (+1)
// of rows g (+8).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void router_tile(const __nv_bfloat16* __restrict__ x,
                                           const __nv_bfloat16* __restrict__ w_router,
                                           const __nv_bfloat16* __restrict__ w_gvec, int T,
                                           int H, int E, int rg, int tt, int k_begin, int k_len,
                                           float (&acc)[4][4], float (&wss)[2], float (&xss)[4],
                                           const __nv_bfloat16* __restrict__ w_norm = nullptr,
                                           const float* s_rs = nullptr,
                                           __nv_bfloat16* __restrict__ xn_out = nullptr) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int r0 = rg * 16 + g, r1 = r0 + 8;
  auto row_ptr = [&](int r) -> const __nv_bfloat16* {
    if (r < E) return w_router + size_t(r) * H;
    if (r == E) return w_gvec;
    return nullptr;
  };
  const __nv_bfloat16* wa_p = row_ptr(r0);
  const __nv_bfloat16* wb_p = row_ptr(r1);
  const __nv_bfloat16* xp[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t = tt * 32 + q * 8 + g;
    xp[q] = t < T ? x + size_t(t) * H : nullptr;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    xss[q] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;
  }
  wss[0] = wss[1] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 4
  for (int k0 = k_begin; k0 < k_begin + k_len; k0 += 32) {
    const int kk = k0 + 8 * c;
    const uint4 wa = wa_p ? ldg_stream(wa_p + kk) : zero;
    const uint4 wb = wb_p ? ldg_stream(wb_p + kk) : zero;
    wss[0] += sumsq8(wa);
    wss[1] += sumsq8(wb);
    // decoder layer: x is normalised on the way in (s_rs: the group's row
    // scales), and xn_out, when given, receives the normalised rows
    const uint4 wn = w_norm ? ldg_keep(w_norm + kk) : zero;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (tt * 32 + q * 8 < T) {  // warp-uniform
        uint4 xv = xp[q] ? ldg_keep(xp[q] + kk) : zero;
        if (w_norm && xp[q]) {
          xv = rms_apply8(xv, wn, s_rs[q * 8 + g]);
          if (xn_out) *reinterpret_cast<uint4*>(xn_out + (xp[q] - x) + kk) = xv;
        }
        mma_k32(acc[q], wa, wb, xv);
        xss[q] += sumsq8(xv);
      }
    }
  }
}

// Row norms (sqrt of the fp32 sum of squares, rounded up) of a bf16 matrix
// [rows][H], one warp per row.
__global__ void __launch_bounds__(256) row_norms_kernel(const __nv_bfloat16* __restrict__ a,
                                                        int rows, int H, float* __restrict__ out) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float ss = warp_row_sumsq(a + size_t(r) * H, H);
  if ((threadIdx.x & 31) == 0) out[r] = norm_from_sumsq(ss);
}

// Exactly rounded logits of every (token, expert) pair, one warp per pair
// (test and diagnostic use: the full evaluation the top-k avoids).
__global__ void __launch_bounds__(256) exact_logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           int T, int H, int E,
                                                           float* __restrict__ out,
                                                           int* __restrict__ n_inexact) {
  const long p = long(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (p >= long(T) * E) return;
  const int t = int(p / E), e = int(p % E);
  bool ok = true;
  const float r = warp_exact_dot(x + size_t(t) * H, w + size_t(e) * H, H, ok);
  if ((threadIdx.x & 31) == 0) {
    out[p] = r;
    if (!ok) atomicAdd(n_inexact, 1);
  }
}

cudaError_t launch_exact_logits(const __nv_bfloat16* x, const __nv_bfloat16* w, int T, int H,
                                int E, float* out, int* n_inexact, cudaStream_t st) {
  const long pairs = long(T) * E;
  if (pairs == 0) return cudaSuccess;
  exact_logits_kernel<<<unsigned((pairs + 7) / 8), 256, 0, st>>>(x, w, T, H, E, out, n_inexact);
  return cudaGetLastError();
}

cudaError_t launch_row_norms(const __nv_bfloat16* a, int rows, int H, float* out,
                             cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  row_norms_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, rows, H, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Block-level CSR dispatch (any blockDim that is a multiple of 32, >= E).
//  1. exclusive scan of counts -> offsets[0..E]; offsets[E+1] = P + T
//     (rows P..P+T-1 are the shared expert's, one per token);
//  2. active list: experts in [lo,hi) with count > 0, ascending, then the
//     shared expert (index E) when requested;
//  3. stable counting sort of the P = T*K pairs by expert: pair order is
//     kept within an expert, as torch.sort(stable=True) in
//     moe_dispatch.py:129; ranks inside a warp come from __match_any_sync.
// s_wcnt must hold (blockDim/32) * E ints.
// ---------------------------------------------------------------------------
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int s = lane < nw ? warp_sums[lane] : 0;
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += n;
    }
    if (lane < nw) warp_sums[lane] = si - s;
    if (lane == 31) *total = si;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

struct DispatchOut {
  int32_t* offsets;
  int32_t* active;
  int32_t* n_active;
  int32_t* sorted_tok;
  int32_t* sorted_slot;
  int32_t* pair_dst;
  float* pair_w;
  int sh_lo, sh_hi;  // shared-expert rows P+sh_lo .. P+sh_hi are computed
};

__device__ void block_dispatch(const int* cnt_src, const int32_t* __restrict__ topk_idx,
                               const float* __restrict__ topk_w,
                               const float* __restrict__ shared_gate, int T, int E, int K, int lo,
                               int hi, int with_shared, int with_routed, DispatchOut o,
                               int* s_off, int* s_cur, int* s_wsum, int* s_tot, int* s_wcnt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int P = T * K;
  const int cnt = tid < E ? cnt_src[tid] : 0;
  const int ex = block_exclusive_scan(cnt, s_wsum, s_tot);
  if (tid < E) {
    s_off[tid] = ex;
    s_cur[tid] = 0;
    o.offsets[tid] = ex;
  }
  if (tid == 0) {
    o.offsets[E] = P;  // routed rows end here; the shared block is compacted
    o.offsets[E + 1] = P + (o.sh_hi - o.sh_lo);
  }
  const int act = (with_routed && tid < E && tid >= lo && tid < hi && cnt > 0) ? 1 : 0;
  const int apos = block_exclusive_scan(act, s_wsum, s_tot);
  if (act) o.active[apos] = tid;
  if (tid == 0) {
    int na = *s_tot;
    if (with_shared && o.sh_hi > o.sh_lo) o.active[na++] = E;
    o.n_active[0] = na;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  const int nw = nthr >> 5;
  for (int base = 0; base < P; base += nthr) {
    for (int i = tid; i < nw * E; i += nthr) s_wcnt[i] = 0;
    __syncthreads();
    const int p = base + tid;
    const int e = p < P ? topk_idx[p] : -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(m & lt_mask);
    if (e >= 0 && rank == 0) s_wcnt[warp * E + e] = __popc(m);
    __syncthreads();
    if (e >= 0) {
      int pre = 0;
      for (int w = 0; w < warp; ++w) pre += s_wcnt[w * E + e];
      const int pos = s_off[e] + s_cur[e] + pre + rank;
      o.sorted_tok[pos] = p / K;
      o.sorted_slot[pos] = p % K;
      o.pair_dst[pos] = p;
      o.pair_w[pos] = topk_w[p];
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += nthr) {
      int s = 0;
      for (int w = 0; w < nw; ++w) s += s_wcnt[w * E + ee];
      s_cur[ee] += s;
    }
    __syncthreads();
  }
  // shared-expert rows: dispatched row P+i is token sh_lo+i (output row P+t)
  for (int i = tid; i < o.sh_hi - o.sh_lo; i += nthr) {
    const int t = o.sh_lo + i;
    o.sorted_tok[P + i] = t;
    o.pair_dst[P + i] = P + t;
    o.pair_w[P + i] = shared_gate[t];
  }
}

// ---------------------------------------------------------------------------
// Fused decode routing (T <= kFusedRouteMaxT), grid = (Rpad/16) * ceil(T/32)
// * KS CTAs of 512 threads (KS K-ranges per logit tile: 136 CTAs at T=64, so
// each warp's loads are one 32-column step).  Tickets in sync[4 + group] and
// sync[0] (cleared by the launcher's memset and by the winners) pick the
// last CTA of each 32-token group for the top-k and the last group for the
// dispatch, so the serial tail runs on two CTAs and then one.
// ---------------------------------------------------------------------------
constexpr int kFusedRouteThreads = 512;
constexpr int kMaxRouteKS = 4;  // split-K factor of the decode router (Dims::KS)
constexpr int kFusedRouteWarps = kFusedRouteThreads / 32;

using FusedExact = ExactCta<kFusedRouteWarps, 32>;

// Dynamic shared memory: the group's logits, the dispatch staging, and (at
// a 16-byte aligned offset) the exact top-k queue.
__host__ __device__ inline size_t fused_route_exact_offset(int T, int E, int K, int Rpad) {
  const size_t b = sizeof(float) * size_t(T) * Rpad + sizeof(int) * size_t(T) * K +
                   sizeof(float) * size_t(T) * K + sizeof(float) * T +
                   sizeof(int) * size_t(kFusedRouteWarps) * E;
  return (b + 15) / 16 * 16;
}
size_t fused_route_smem_bytes(int T, int E, int K, int Rpad) {
  return fused_route_exact_offset(T, E, K, Rpad) + sizeof(FusedExact);
}

__global__ void __launch_bounds__(kFusedRouteThreads, 1) route_fused_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_router,
    const __nv_bfloat16* __restrict__ w_gvec, int T, int H, int E, int K, int Rpad, int KS,
    int lo, int hi, int with_shared, int with_routed, float* __restrict__ logit_part,
    float* __restrict__ xn_part, float* __restrict__ wn_part, float* __restrict__ diag,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* __restrict__ shared_gate,
    DispatchOut o, int32_t* __restrict__ sync, int* __restrict__ epoch_bump,
    const __nv_bfloat16* __restrict__ w_norm, float eps, __nv_bfloat16* __restrict__ xn) {
  __shared__ float s_part[kFusedRouteWarps][32][17];
  __shared__ float s_rs[32];
  __shared__ float s_wss[kFusedRouteWarps][16], s_xss[kFusedRouteWarps][32];
  __shared__ float s_wn[256], s_xn[32];
  __shared__ int s_cnt[256], s_off[256], s_cur[256], s_wsum[32], s_tot[2], s_last;
  extern __shared__ float s_dyn[];
  float* s_lg = s_dyn;                                       // [32][Rpad] (one token group)
  int* s_idx = reinterpret_cast<int*>(s_lg + size_t(T) * Rpad);  // [T*K]
  float* s_w = reinterpret_cast<float*>(s_idx + T * K);      // [T*K]
  float* s_sg = s_w + T * K;                                  // [T]
  int* s_wcnt = reinterpret_cast<int*>(s_sg + T);             // [warps][E]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int RG = Rpad / 16, TT = (T + 31) / 32;
  pdl_trigger();  // the gate_up kernel's CTAs may start their set-up as SMs free up
  if (epoch_bump && blockIdx.x == 0 && threadIdx.x == 0) *epoch_bump += 1;
  const int kg = blockIdx.x % KS, rest = blockIdx.x / KS;
  const int rg = rest % RG, tt = rest / RG;
  // This CTA's K range [kb, kb + Hk), split over the warps in whole 32-column
  // steps; with small H the trailing warps get an empty slice.
  const int Hk = H / KS, kb = kg * Hk;
  const int slice = (Hk / kFusedRouteWarps + 31) / 32 * 32;
  const int k_off = min(Hk, warp * slice);
  // Decoder layer (w_norm given): the RMSNorm of the group's tokens is fused
  // here -- every CTA computes the row scales (the standalone kernel's
  // arithmetic), normalises its x tiles as it loads them, and the CTAs of
  // router row group 0 write their k range of xn for the expert kernels and
  // for the exact evaluations below (which read it through L2 after the
  // group's counter); the exact top-k then works on xn.
  if (w_norm) {
    for (int tl = warp; tl < 32; tl += kFusedRouteWarps) {
      const int t = tt * 32 + tl;
      const float r = t < T ? rms_row_scale(x + size_t(t) * H, H, eps) : 0.f;
      if (lane == 0) s_rs[tl] = r;
    }
    __syncthreads();
  }
  float acc[4][4], wss[2], xss[4];
  router_tile(x, w_router, w_gvec, T, H, E, rg, tt, kb + k_off, min(slice, Hk - k_off), acc, wss,
              xss, w_norm, s_rs, (w_norm && rg == 0) ? xn : nullptr);
  // from here on the token rows are the normalised ones
  const __nv_bfloat16* xr = w_norm ? xn : x;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    s_part[warp][q * 8 + 2 * c][g] = acc[q][0];
    s_part[warp][q * 8 + 2 * c + 1][g] = acc[q][1];
    s_part[warp][q * 8 + 2 * c][g + 8] = acc[q][2];
    s_part[warp][q * 8 + 2 * c + 1][g + 8] = acc[q][3];
  }
  // sums of squares of this warp's k slice: the 4 lanes of a row group hold
  // disjoint k ranges
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    wss[0] += __shfl_xor_sync(0xffffffffu, wss[0], o);
    wss[1] += __shfl_xor_sync(0xffffffffu, wss[1], o);
#pragma unroll
    for (int q = 0; q < 4; ++q) xss[q] += __shfl_xor_sync(0xffffffffu, xss[q], o);
  }
  if (c == 0) {
    s_wss[warp][g] = wss[0];
    s_wss[warp][g + 8] = wss[1];
#pragma unroll
    for (int q = 0; q < 4; ++q) s_xss[warp][q * 8 + g] = xss[q];
  }
  __syncthreads();
  float* part = logit_part + size_t(kg) * T * Rpad;
  for (int i = tid; i < 32 * 16; i += kFusedRouteThreads) {
    const int tl = i >> 4, rl = i & 15;
    const int t = tt * 32 + tl, r = rg * 16 + rl;
    if (t < T && r <= E) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kFusedRouteWarps; ++w) s += s_part[w][tl][rl];
      part[size_t(t) * Rpad + r] = s;
    }
  }
  if (tid < 16) {  // this CTA's k range of its 16 router rows (every group keeps its own copy)
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kFusedRouteWarps; ++w) s += s_wss[w][tid];
    wn_part[(size_t(tt) * KS + kg) * Rpad + rg * 16 + tid] = s;
  } else if (tid < 48 && rg == 0) {  // and of the group's tokens
    const int tl = tid - 16, t = tt * 32 + tl;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kFusedRouteWarps; ++w) s += s_xss[w][tl];
    if (t < T) xn_part[size_t(kg) * T + t] = s;
  }
  __threadfence();
  __syncthreads();
  // Level 1: the last CTA of this 32-token group sums the KS partials in a
  // fixed order and selects the group's top-k on exactly rounded logits.
  if (tid == 0) s_last = (atomicAdd(&sync[4 + tt], 1) == RG * KS - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int t0 = tt * 32, nt = min(32, T - t0);
  // The norms' partial sums first (one round trip, overlapping the logits'),
  // then the logits: Rpad is a multiple of 16, so whole float4s; two items
  // per thread and iteration, all 2 * KS partial loads in flight.
  float wss_r = 0.f, xss_t = 0.f;
  {
    float wv[kMaxRouteKS], xv[kMaxRouteKS];
#pragma unroll
    for (int k = 0; k < kMaxRouteKS; ++k) {
      wv[k] = (k < KS && tid < E) ? __ldcg(wn_part + (size_t(tt) * KS + k) * Rpad + tid) : 0.f;
      xv[k] = (k < KS && tid < nt) ? __ldcg(xn_part + size_t(k) * T + t0 + tid) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kMaxRouteKS; ++k) {
      wss_r += wv[k];
      xss_t += xv[k];
    }
  }
  static_assert(kFusedRouteThreads >= 256, "one thread per router row");
  const int n4 = nt * Rpad / 4;
  for (int i0 = tid; i0 < n4; i0 += 2 * kFusedRouteThreads) {
    float4 v[2][kMaxRouteKS];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + u * kFusedRouteThreads;
      const size_t gi = size_t(t0) * Rpad / 4 + (i < n4 ? i : 0);
#pragma unroll
      for (int k = 0; k < kMaxRouteKS; ++k)
        if (k < KS)
          v[u][k] = __ldcg(reinterpret_cast<const float4*>(logit_part + size_t(k) * T * Rpad) + gi);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + u * kFusedRouteThreads;
      if (i >= n4) break;
      float4 sum = v[u][0];
#pragma unroll
      for (int k = 1; k < kMaxRouteKS; ++k)
        if (k < KS) {
          sum.x += v[u][k].x; sum.y += v[u][k].y; sum.z += v[u][k].z; sum.w += v[u][k].w;
        }
      reinterpret_cast<float4*>(s_lg)[i] = sum;
      if (diag) reinterpret_cast<float4*>(diag)[size_t(t0) * Rpad / 4 + i] = sum;
    }
  }
  if (tid < E) s_wn[tid] = norm_from_sumsq(wss_r);
  if (tid < nt) s_xn[tid] = norm_from_sumsq(xss_t);
  for (int e = tid; e < 256; e += kFusedRouteThreads) s_cnt[e] = 0;
  __syncthreads();
  // accumulation depth: the MMA steps of one warp's slice, the sum over the
  // CTA's warps and the sum over the KS partials
  const float gamma = accumulation_gamma(2 * (slice / 32), kFusedRouteWarps + KS);
  const ExactStats stats{sync + 8, sync + 9};
  FusedExact& xq = *reinterpret_cast<FusedExact*>(
      reinterpret_cast<char*>(s_dyn) + fused_route_exact_offset(T, E, K, Rpad));
  if (tid == 0) {
    xq.n_pend = 0;
    xq.n_req = 0;
  }
  __syncthreads();
  // two tokens per warp (tl, tl + 16), their fast checks interleaved
  static_assert(2 * kFusedRouteWarps >= 32, "a 32-token group in one pass");
  if (warp < nt) {
    const int tl0 = warp, tl1 = warp + kFusedRouteWarps;
    const bool v1 = tl1 < nt;
    const float* r0 = s_lg + size_t(tl0) * Rpad;
    const float* r1 = s_lg + size_t(v1 ? tl1 : tl0) * Rpad;
    warp_topk_stage2(xq, [&](int i, int e) { return (i ? r1 : r0)[e]; }, s_wn, s_xn[tl0],
                     s_xn[v1 ? tl1 : tl0], gamma, t0 + tl0, t0 + tl1, v1, E, K, xr, w_router, H,
                     stats, topk_idx, topk_w, [&](int) { return s_cnt; });
    if (lane == 0) {
      shared_gate[t0 + tl0] = 1.0f / (1.0f + expf(-r0[E]));
      if (v1) shared_gate[t0 + tl1] = 1.0f / (1.0f + expf(-r1[E]));
    }
  }
  cta_topk_finish(xq, xr, w_router, H, K, stats, topk_idx, topk_w, [&](int) { return s_cnt; });
  __threadfence();
  __syncthreads();
  // Level 2: the last group to finish builds the dispatch for all tokens.
  if (tid == 0) {
    sync[4 + tt] = 0;
    s_last = (atomicAdd(&sync[0], 1) == TT - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = tid; e < 256; e += kFusedRouteThreads) s_cnt[e] = 0;
  __syncthreads();
  for (int p = tid; p < T * K; p += kFusedRouteThreads) {
    const int e = __ldcg(topk_idx + p);
    s_idx[p] = e;
    s_w[p] = __ldcg(topk_w + p);
    atomicAdd(&s_cnt[e], 1);
  }
  for (int t = tid; t < T; t += kFusedRouteThreads) s_sg[t] = __ldcg(shared_gate + t);
  __syncthreads();
  block_dispatch(s_cnt, s_idx, s_w, s_sg, T, E, K, lo, hi, with_shared, with_routed, o, s_off,
                 s_cur, s_wsum, s_tot, s_wcnt);
  if (tid == 0) sync[0] = 0;
}

// ---------------------------------------------------------------------------
// Large-T path.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) router_logits_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_router,
    const __nv_bfloat16* __restrict__ w_gvec, int T, int H, int E, int Rpad,
    float* __restrict__ logits, int32_t* __restrict__ counts) {
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < E; i += blockDim.x) counts[i] = 0;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int RG = Rpad / 16, TT = (T + 31) / 32;
  const long item = long(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (item >= long(RG) * TT) return;
  const int rg = int(item % RG), tt = int(item / RG);
  float acc[4][4], wss[2], xss[4];
  router_tile(x, w_router, w_gvec, T, H, E, rg, tt, 0, H, acc, wss, xss);
  const int r0 = rg * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t0 = tt * 32 + q * 8 + 2 * c;
    if (t0 < T) {
      logits[size_t(t0) * Rpad + r0] = acc[q][0];
      logits[size_t(t0) * Rpad + r1] = acc[q][2];
    }
    if (t0 + 1 < T) {
      logits[size_t(t0 + 1) * Rpad + r0] = acc[q][1];
      logits[size_t(t0 + 1) * Rpad + r1] = acc[q][3];
    }
  }
}

// Warp per token over the logits of router_logits_kernel (one MMA chain of
// H/16 steps per logit); wn: the router rows' norms (row_norms_kernel).
__global__ void __launch_bounds__(256, 2) topk_kernel(
    const float* __restrict__ logits, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w_router, const float* __restrict__ wn, int T, int H,
    int E, int K, int Rpad, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
    float* __restrict__ shared_gate, int32_t* __restrict__ counts, ExactStats stats) {
  __shared__ ExactCta<8, 8> xq;
  if (threadIdx.x == 0) {
    xq.n_pend = 0;
    xq.n_req = 0;
  }
  __syncthreads();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < T) {
    const float nx = norm_from_sumsq(warp_row_sumsq(x + size_t(t) * H, H));
    const float gamma = accumulation_gamma(H / 16, 1);
    const float* row = logits + size_t(t) * Rpad;
    warp_topk_stage(xq, [&](int e) { return row[e]; }, wn, nx, gamma, t, E, K, x, w_router, H,
                    stats, topk_idx, topk_w, [&](int) { return counts; });
    if ((threadIdx.x & 31) == 0) shared_gate[t] = 1.0f / (1.0f + expf(-row[E]));
  }
  cta_topk_finish(xq, x, w_router, H, K, stats, topk_idx, topk_w,
                  [&](int) { return counts; });
}

constexpr int kDispatchThreads = 1024;

__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(
    const int32_t* __restrict__ counts, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, const float* __restrict__ shared_gate, int T, int E, int K,
    int lo, int hi, int with_shared, int with_routed, DispatchOut o) {
  extern __shared__ int smem[];
  int* s_off = smem;
  int* s_cur = s_off + E;
  int* s_wsum = s_cur + E;
  int* s_tot = s_wsum + 32;
  int* s_wcnt = s_tot + 2;
  block_dispatch(counts, topk_idx, topk_w, shared_gate, T, E, K, lo, hi, with_shared,
                 with_routed, o, s_off, s_cur, s_wsum, s_tot, s_wcnt);
}

size_t dispatch_smem_bytes(int E) {
  return sizeof(int) * (2 * E + 34 + (kDispatchThreads / 32) * E);
}

cudaError_t launch_route(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                         const __nv_bfloat16* w_gvec, int lo, int hi, int with_shared,
                         int with_routed, const Workspace& ws, cudaStream_t st,
                         int* epoch_bump, const __nv_bfloat16* w_norm, float eps,
                         __nv_bfloat16* xn) {
  DispatchOut o{ws.offsets, ws.active, ws.n_active, ws.sorted_tok, ws.sorted_slot, ws.pair_dst,
                ws.pair_w, d.sh_lo, d.sh_hi};
  const int RG = d.Rpad / 16, TT = (d.T + 31) / 32;
  cudaError_t err = cudaMemsetAsync(ws.status, 0, kStatusWords * sizeof(int32_t), st);
  if (err != cudaSuccess) return err;
  if (d.T <= kFusedRouteMaxT) {
    route_fused_kernel<<<RG * TT * d.KS, kFusedRouteThreads,
                         fused_route_smem_bytes(d.T, d.E, d.K, d.Rpad), st>>>(
        x, w_router, w_gvec, d.T, d.H, d.E, d.K, d.Rpad, d.KS, lo, hi, with_shared,
        with_routed, ws.logit_part, ws.xnorm, ws.wnorm, ws.diag, ws.topk_idx, ws.topk_w,
        ws.shared_gate, o, ws.status, epoch_bump, w_norm, eps, xn);
    return cudaGetLastError();
  }
  const long items = long(RG) * TT;
  router_logits_kernel<<<unsigned((items + 3) / 4), 128, 0, st>>>(
      x, w_router, w_gvec, d.T, d.H, d.E, d.Rpad, ws.logit_part, ws.counts);
  err = launch_row_norms(w_router, d.E, d.H, ws.wnorm, st);
  if (err != cudaSuccess) return err;
  if (ws.diag)
    cudaMemcpyAsync(ws.diag, ws.logit_part, sizeof(float) * size_t(d.T) * d.Rpad,
                    cudaMemcpyDeviceToDevice, st);
  topk_kernel<<<(d.T + 7) / 8, 256, 0, st>>>(ws.logit_part, x, w_router, ws.wnorm, d.T, d.H, d.E,
                                             d.K, d.Rpad, ws.topk_idx, ws.topk_w, ws.shared_gate,
                                             ws.counts, ExactStats{ws.status + 8, ws.status + 9});
  dispatch_kernel<<<1, kDispatchThreads, dispatch_smem_bytes(d.E), st>>>(
      ws.counts, ws.topk_idx, ws.topk_w, ws.shared_gate, d.T, d.E, d.K, lo, hi, with_shared,
      with_routed, o);
  return cudaGetLastError();
}

bool route_bumps_epoch(const Dims& d) { return d.T <= kFusedRouteMaxT; }
bool route_fuses_norm(const Dims& d) { return d.T <= kFusedRouteMaxT && d.H % 8 == 0; }

float route_gamma(const Dims& d) {
  if (d.T <= kFusedRouteMaxT) {
    const int slice = (d.H / d.KS / kFusedRouteWarps + 31) / 32 * 32;
    return accumulation_gamma(2 * (slice / 32), kFusedRouteWarps + d.KS);
  }
  return accumulation_gamma(d.H / 16, 1);
}

cudaError_t route_init() {
  cudaError_t e = cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(dispatch_smem_bytes(256)));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(fused_route_smem_bytes(kFusedRouteMaxT, 256, 32, 272)));
}

}  // namespace pmoe
