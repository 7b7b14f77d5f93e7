// Router, top-k and CSR dispatch kernels.
//
// Reference arithmetic: Qwen3_5MoeTopKRouter.forward
// (transformers models/qwen3_5_moe/modeling_qwen3_5_moe.py:762-770) and the
// stable-sort dispatch of engine/kernels/moe_dispatch.py:119-137.
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"

namespace pmoe {

// ---------------------------------------------------------------------------
// router_partial: logit_part[ks][t][r] = sum_{k in slice ks} x[t,k] * Wr[r,k]
// for r < E (router rows) and r == E (shared-expert gate vector).
// One warp = 16 router rows x 32 tokens x one K slice, on mma.sync with the
// 128-bit permuted-k operand layout of mma_k32.  Block 0 also zeroes the
// per-expert counters that route_topk increments (stream order makes this
// safe: route_topk starts after this kernel has finished).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) router_partial_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_router,
    const __nv_bfloat16* __restrict__ w_gvec, int T, int H, int E, int Rpad, int KS,
    float* __restrict__ part, int32_t* __restrict__ counts) {
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < E; i += blockDim.x) counts[i] = 0;
  }
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int RG = Rpad / 16, TT = (T + 31) / 32;
  const long item = long(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (item >= long(RG) * TT * KS) return;
  const int ks = int(item % KS);
  const int rg = int((item / KS) % RG);
  const int tt = int(item / (long(KS) * RG));
  const int slice = H / KS, k_begin = ks * slice;

  // Weight rows g and g+8 of this row group (row E is the shared gate vector).
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
    int t = tt * 32 + q * 8 + g;
    xp[q] = t < T ? x + size_t(t) * H : nullptr;
  }
  float acc[4][4] = {};
  const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 2
  for (int k0 = k_begin; k0 < k_begin + slice; k0 += 32) {
    const int kk = k0 + 8 * c;
    uint4 wa = wa_p ? ldg_stream(wa_p + kk) : zero;
    uint4 wb = wb_p ? ldg_stream(wb_p + kk) : zero;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (tt * 32 + q * 8 < T) {  // warp-uniform
        uint4 xv = xp[q] ? ldg_keep(xp[q] + kk) : zero;
        mma_k32(acc[q], wa, wb, xv);
      }
    }
  }
  float* out = part + size_t(ks) * T * Rpad;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int t0 = tt * 32 + q * 8 + 2 * c;
    if (t0 < T) {
      out[size_t(t0) * Rpad + r0] = acc[q][0];
      out[size_t(t0) * Rpad + r1] = acc[q][2];
    }
    if (t0 + 1 < T) {
      out[size_t(t0 + 1) * Rpad + r0] = acc[q][1];
      out[size_t(t0 + 1) * Rpad + r1] = acc[q][3];
    }
  }
}

// ---------------------------------------------------------------------------
// route_topk: one warp per token.  Sums the KS router partials in a fixed
// order, rounds each logit once to bf16 (F.linear's bf16 output), picks the
// top K by (logit desc, index asc), and renormalises:
//   w_i = exp(l_i - l_max) / sum_{j in top-K} exp(l_j - l_max)
// which equals softmax-then-topk-then-divide-by-sum (router :765-768).
// Also writes sigmoid(shared gate) and bumps the per-expert counters.
// Supports E <= 256 (8 logits per lane).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) route_topk_kernel(
    const float* __restrict__ part, int T, int E, int K, int Rpad, int KS,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* __restrict__ shared_gate,
    int32_t* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  constexpr int NJ = 8;
  float v[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int e = j * 32 + lane;
    float s = 0.f;
    if (e < E) {
      for (int ks = 0; ks < KS; ++ks) s += part[(size_t(ks) * T + t) * Rpad + e];
      v[j] = bf16_round(s);
    } else {
      v[j] = -INFINITY;
    }
  }
  if (lane == 0) {
    float s = 0.f;
    for (int ks = 0; ks < KS; ++ks) s += part[(size_t(ks) * T + t) * Rpad + E];
    shared_gate[t] = 1.0f / (1.0f + __expf(-s));
  }
  unsigned taken = 0;  // bit j set: v[j] already selected
  float sel_v[32];
  int sel_e[32];
  // K <= 32 is enforced by the launcher.
  for (int k = 0; k < K; ++k) {
    // Lane-local best among untaken entries; ties -> lower expert (lower j).
    float bv = -INFINITY;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      if (!(taken >> j & 1u) && j * 32 + lane < E && (bj < 0 || v[j] > bv)) {
        bv = v[j];
        bj = j;
      }
    }
    int be = bj < 0 ? 0x7fffffff : bj * 32 + lane;
    // Warp argmax on (value desc, expert asc).
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if (be != 0x7fffffff && (be & 31) == lane) taken |= 1u << (be >> 5);
    sel_v[k] = bv;
    sel_e[k] = be;
  }
  if (lane == 0) {
    const float m = sel_v[0];
    float den = 0.f;
    for (int k = 0; k < K; ++k) den += __expf(sel_v[k] - m);
    const float inv = 1.0f / den;
    for (int k = 0; k < K; ++k) {
      topk_idx[size_t(t) * K + k] = sel_e[k];
      topk_w[size_t(t) * K + k] = __expf(sel_v[k] - m) * inv;
      atomicAdd(&counts[sel_e[k]], 1);
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch: single CTA of 1024 threads.
//  1. exclusive scan of counts -> offsets[0..E]; offsets[E+1] = P + T
//     (rows P..P+T-1 are the shared expert's, one per token);
//  2. active list: experts in [lo,hi) with count > 0, ascending, then the
//     shared expert (index E) when requested;
//  3. stable counting sort of the P = T*K pairs by expert (pair order kept
//     within an expert, as torch.sort(stable=True) in moe_dispatch.py:129),
//     chunk by chunk with __match_any_sync for intra-warp ranks.
// ---------------------------------------------------------------------------
constexpr int kDispatchThreads = 1024;

__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int s = warp_sums[lane];
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += n;
    }
    warp_sums[lane] = si - s;
    if (lane == 31) *total = si;
  }
  __syncthreads();
  int r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(
    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const float* __restrict__ shared_gate, const int32_t* __restrict__ counts, int T, int E, int K,
    int lo, int hi, int with_shared, int with_routed, int32_t* __restrict__ offsets,
    int32_t* __restrict__ active, int32_t* __restrict__ n_active,
    int32_t* __restrict__ sorted_tok, int32_t* __restrict__ sorted_slot,
    int32_t* __restrict__ pair_dst, float* __restrict__ pair_w) {
  extern __shared__ int smem[];
  int* s_off = smem;                   // [E]
  int* s_cur = s_off + E;              // [E]
  int* s_wsum = s_cur + E;             // [32]
  int* s_tot = s_wsum + 32;            // [2]
  int* s_wcnt = s_tot + 2;             // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P = T * K;

  // 1. offsets
  const int cnt = tid < E ? counts[tid] : 0;
  const int ex = block_exclusive_scan(cnt, s_wsum, s_tot);
  if (tid < E) {
    s_off[tid] = ex;
    s_cur[tid] = 0;
    offsets[tid] = ex;
  }
  if (tid == 0) {
    offsets[E] = P;
    offsets[E + 1] = P + T;
  }
  // 2. active list
  const int act = (with_routed && tid < E && tid >= lo && tid < hi && cnt > 0) ? 1 : 0;
  const int apos = block_exclusive_scan(act, s_wsum, s_tot);
  if (act) active[apos] = tid;
  if (tid == 0) {
    int na = *s_tot;
    if (with_shared) active[na++] = E;
    n_active[0] = na;
  }
  __syncthreads();

  // 3. stable scatter
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = 0; base < P; base += kDispatchThreads) {
    for (int i = tid; i < 32 * E; i += kDispatchThreads) s_wcnt[i] = 0;
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
      sorted_tok[pos] = p / K;
      sorted_slot[pos] = p % K;
      pair_dst[pos] = p;
      pair_w[pos] = topk_w[p];
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += kDispatchThreads) {
      int s = 0;
      for (int w = 0; w < 32; ++w) s += s_wcnt[w * E + ee];
      s_cur[ee] += s;
    }
    __syncthreads();
  }
  // shared-expert rows: one per token, in token order
  for (int t = tid; t < T; t += kDispatchThreads) {
    sorted_tok[P + t] = t;
    pair_dst[P + t] = P + t;
    pair_w[P + t] = shared_gate[t];
  }
}

size_t dispatch_smem_bytes(int E) { return sizeof(int) * (2 * E + 34 + 32 * E); }

cudaError_t launch_route(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                         const __nv_bfloat16* w_gvec, int lo, int hi, int with_shared,
                         int with_routed, const Workspace& ws, cudaStream_t st) {
  const int RG = d.Rpad / 16, TT = (d.T + 31) / 32;
  const long items = long(RG) * TT * d.KS;
  const int warps_per_block = 4;
  const long blocks = (items + warps_per_block - 1) / warps_per_block;
  router_partial_kernel<<<unsigned(blocks), 32 * warps_per_block, 0, st>>>(
      x, w_router, w_gvec, d.T, d.H, d.E, d.Rpad, d.KS, ws.logit_part, ws.counts);
  route_topk_kernel<<<(d.T + 7) / 8, 256, 0, st>>>(ws.logit_part, d.T, d.E, d.K, d.Rpad, d.KS,
                                                  ws.topk_idx, ws.topk_w, ws.shared_gate,
                                                  ws.counts);
  const size_t sm = dispatch_smem_bytes(d.E);
  dispatch_kernel<<<1, kDispatchThreads, sm, st>>>(
      ws.topk_idx, ws.topk_w, ws.shared_gate, ws.counts, d.T, d.E, d.K, lo, hi, with_shared,
      with_routed, ws.offsets, ws.active, ws.n_active, ws.sorted_tok, ws.sorted_slot,
      ws.pair_dst, ws.pair_w);
  return cudaGetLastError();
}

cudaError_t route_init() {
  return cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(dispatch_smem_bytes(256)));
}

}  // namespace pmoe
