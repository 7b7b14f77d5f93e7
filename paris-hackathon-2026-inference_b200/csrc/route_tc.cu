// Prefill routing (large T): tcgen05 router GEMM with top-k in the epilogue,
// then a parallel stable CSR dispatch.
//
//   router_tc_kernel   a cluster of two CTAs per 128-token tile, CTA h on
//                      experts [128h, 128h+128): logits = x . W_r^T on the
//                      tensor cores (M=128 tokens, N=128 experts; CTA 0 also
//                      the shared-expert gate as an N=16 MMA whose B tile is
//                      w_sh_gvec with TMA zero-filling rows 1..15).  Each
//                      epilogue thread (one token) rounds its logits to bf16
//                      and keeps its top K keys in registers (ties -> lower
//                      expert); CTA 0 merges the peer's keys through
//                      distributed shared memory, renormalises, and writes the
//                      tile's per-expert histogram.  (One CTA per tile on all
//                      256 experts left 84 SMs idle at T=8192 and ran 64 %
//                      tensor-busy on the rest.)
//   route_scan_kernel  one CTA: per-expert counts, CSR offsets, active list
//                      and, per (tile, expert), the first output slot.
//   route_scatter_kernel  one CTA per tile: stable ranks of the tile's pairs
//                      within their expert (pair order kept, as the stable
//                      torch.sort of engine/kernels/moe_dispatch.py:129), the
//                      permuted rows and the shared-expert rows.
// Reference: Qwen3_5MoeTopKRouter.forward (modeling_qwen3_5_moe.py:762-770).
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tc.cuh"
#include "pmoe_exact.cuh"

namespace pmoe {

constexpr int kRtM = 128, kRtN = 256, kRtN2 = 16, kRtK = 64;
constexpr int kRtNH = kRtN / 2;            // experts per CTA of the pair
constexpr int kRtStages = 6;
constexpr int kRtA = kRtM * kRtK * 2;      // 16 KiB
constexpr int kRtB = kRtNH * kRtK * 2;     // 16 KiB
constexpr int kRtB2 = kRtN2 * kRtK * 2;    // 2 KiB
constexpr int kRtStageBytes = kRtA + kRtB + kRtB2;
constexpr int kRtSmem = kRtStages * kRtStageBytes + 1024 + 256;
static_assert(kRtSmem <= 227 * 1024, "router shared memory");
constexpr int kRtThreads = 6 * 32;
constexpr int kRtMaxK = 8;
// The expert logits accumulate in kRtChains TMEM accumulators (k chunk kc
// goes to chain kc % kRtChains), summed in fp32 in the epilogue: shorter MMA
// chains tighten the accumulation bound of the exact top-k (pmoe_exact.cuh).
constexpr int kRtChains = 3;
constexpr int kRtGateCol = kRtChains * kRtNH;  // gate accumulator (CTA 0)
constexpr int kRtTmemCols = 512;
static_assert(kRtGateCol + kRtN2 <= kRtTmemCols, "TMEM columns");
static_assert(kRtStageBytes % 1024 == 0, "stage alignment");

// Accumulation bound of one logit: the MMA steps of the longest chain and
// the fp32 additions of the chains.
__host__ __device__ inline float router_tc_gamma(int H) {
  const int nk = H / kRtK;
  return accumulation_gamma(((nk + kRtChains - 1) / kRtChains) * (kRtK / 16), kRtChains - 1);
}

__global__ void __launch_bounds__(kRtThreads, 1) router_tc_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
    const __grid_constant__ CUtensorMap tm_g, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w_router, int T, int H, int E, int Rpad,
    float* __restrict__ logits, float* __restrict__ xnorm, float* __restrict__ wnorm,
    int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRtStages * kRtStageBytes);
  uint64_t* empty = full + kRtStages;
  uint64_t* tfull = empty + kRtStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t h = cluster_ctarank();  // expert half
  const int tile = blockIdx.x >> 1;
  const int t0 = tile * kRtM;
  const int e0 = int(h) * kRtNH;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);  // the MMA commit and the four epilogue warps
    }
    mbar_init(tfull, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kRtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nk = H / kRtK;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = h == 0 ? kRtStageBytes : kRtA + kRtB;
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % kRtStages;
        if (kc >= kRtStages && !mbar_wait(&empty[s], ((kc / kRtStages) & 1) ^ 1)) {
          atomicCAS(status, 0, kStatusTimeoutEmpty);
          break;
        }
        uint8_t* sa = smem + s * kRtStageBytes;
        mbar_arrive_expect_tx(&full[s], tx);
        tma_load_2d(sa, &tm_x, kc * kRtK, t0, &full[s]);
        tma_load_2d(sa + kRtA, &tm_w, kc * kRtK, e0, &full[s]);  // rows >= E read as zero
        if (h == 0) tma_load_2d(sa + kRtA + kRtB, &tm_g, kc * kRtK, 0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id1 = idesc_bf16_f32(kRtM, kRtNH), id2 = idesc_bf16_f32(kRtM, kRtN2);
      const uint32_t sb0 = smem_u32(smem);
      bool ok = true;
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % kRtStages;
        if (!mbar_wait(&full[s], (kc / kRtStages) & 1)) {
          atomicCAS(status, 0, kStatusTimeoutFull);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = sb0 + s * kRtStageBytes;
        const uint64_t ad = sdesc_k_sw128(sa), bd = sdesc_k_sw128(sa + kRtA),
                       gd = sdesc_k_sw128(sa + kRtA + kRtB);
        const uint32_t chain = tmem_base + uint32_t(kc % kRtChains) * kRtNH;
#pragma unroll
        for (int kk = 0; kk < kRtK / 16; ++kk) {
          const uint32_t acc = (kc >= kRtChains || kk != 0) ? 1u : 0u;
          umma_bf16(chain, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), id1, acc);
          if (h == 0)
            umma_bf16(tmem_base + kRtGateCol, ad + uint64_t(kk * 2), gd + uint64_t(kk * 2), id2,
                      (kc | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
    }
  } else {
    // Epilogue warps 2..5.  While the MMAs run they read every stage too and
    // keep the sums of squares the exact top-k needs: thread r sums row r of
    // the x tile (tokens t0 + r) and of this half's router rows (experts
    // e0 + r); a stage is released once the MMAs and these four warps are
    // done with it.  Within a swizzled 128-byte row the 16-byte chunks are
    // permuted, which a sum over the whole row does not see.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    float ssx = 0.f, ssw = 0.f;
    const uint32_t sb0 = smem_u32(smem);
    bool fed = true;
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % kRtStages;
      if (!mbar_wait(&full[s], (kc / kRtStages) & 1)) {
        atomicCAS(status, 0, kStatusTimeoutFull);
        fed = false;
        break;
      }
      const uint32_t ra = sb0 + s * kRtStageBytes + r * 128, rb = ra + kRtA;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t o = uint32_t(((c ^ (r & 7)) * 16));
        const uint4 xv = lds128(ra + o), wv = lds128(rb + o);
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float x0 = __uint_as_float(xs[j] << 16), x1 = __uint_as_float(xs[j] & 0xFFFF0000u);
          const float w0 = __uint_as_float(ws[j] << 16), w1 = __uint_as_float(ws[j] & 0xFFFF0000u);
          ssx = fmaf(x0, x0, fmaf(x1, x1, ssx));
          ssw = fmaf(w0, w0, fmaf(w1, w1, ssw));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (fed) {
      if (h == 0 && t0 + r < T) xnorm[t0 + r] = norm_from_sumsq(ssx);
      if (tile == 0 && e0 + r < E) wnorm[e0 + r] = norm_from_sumsq(ssw);
    }
    // One token row per thread: the chains' sum, in a fixed order, to global.
    const int t = t0 + r;
    if (mbar_wait(tfull, 0)) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16);
#pragma unroll 1
      for (int cc = 0; cc < kRtNH / 32; ++cc) {
        uint32_t v0[32], v1[32], v2[32];
        tmem_ld32(taddr + cc * 32, v0);
        tmem_ld32(taddr + kRtNH + cc * 32, v1);
        tmem_ld32(taddr + 2 * kRtNH + cc * 32, v2);
        tmem_ld_wait();
        // the row holds Rpad floats: columns past E (< 256 experts) are not stored
        const int col0 = e0 + cc * 32;
        if (t < T && col0 < E) {
          float* dst = logits + size_t(t) * Rpad + col0;
          if (col0 + 32 <= E) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 o;
              o.x = (__uint_as_float(v0[i]) + __uint_as_float(v1[i])) + __uint_as_float(v2[i]);
              o.y = (__uint_as_float(v0[i + 1]) + __uint_as_float(v1[i + 1])) +
                    __uint_as_float(v2[i + 1]);
              o.z = (__uint_as_float(v0[i + 2]) + __uint_as_float(v1[i + 2])) +
                    __uint_as_float(v2[i + 2]);
              o.w = (__uint_as_float(v0[i + 3]) + __uint_as_float(v1[i + 3])) +
                    __uint_as_float(v2[i + 3]);
              reinterpret_cast<float4*>(dst)[i / 4] = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < E)
                dst[i] = (__uint_as_float(v0[i]) + __uint_as_float(v1[i])) +
                         __uint_as_float(v2[i]);
          }
        }
      }
      if (h == 0) {
        uint32_t gv[32];
        tmem_ld32(taddr + kRtGateCol, gv);
        tmem_ld_wait();
        if (t < T) logits[size_t(t) * Rpad + E] = __uint_as_float(gv[0]);
      }
    } else {
      atomicCAS(status, 0, kStatusTimeoutTmem);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kRtTmemCols);
  }
}

// Exact top-k over the router GEMM's logits (pmoe_exact.cuh), in two kernels
// so that the common case runs at high occupancy:
//   route_fast_kernel   one token per warp: the fast check; a settled token
//                       gets its routing and is counted in its 128-token
//                       tile's histogram (zeroed by the launcher), an open one
//                       is appended to a queue;
//   route_fixup_kernel  the queued tokens, kRtFixTokens per CTA round: the
//                       interval selection with the exact evaluations shared
//                       by the CTA's warps.
constexpr int kRtFastThreads = 256;
constexpr int kRtFixThreads = 256;
// 4 queued tokens per CTA (fix-up of the Zipf T = 8192 case: 8 per CTA 39-43
// us, 4: 31-35, 2: 41-42, 1: 56-58 -- fewer tokens per CTA spread the exact
// evaluations over more SMs until the extra CTA rounds cost more)
constexpr int kRtFixTokens = 4;

__global__ void __launch_bounds__(kRtFastThreads) route_fast_kernel(
    const float* __restrict__ logits, const float* __restrict__ xnorm,
    const float* __restrict__ wnorm, int T, int E, int K, int Rpad, float gamma,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* __restrict__ shared_gate,
    int32_t* __restrict__ hist, int32_t* __restrict__ queue, int* __restrict__ queue_count) {
  __shared__ float s_wn[kRtN];
  for (int e = threadIdx.x; e < kRtN; e += blockDim.x) s_wn[e] = e < E ? wnorm[e] : 0.f;
  __syncthreads();
  const int t = blockIdx.x * (kRtFastThreads / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const float* row = logits + size_t(t) * Rpad;
  if (lane == 0) shared_gate[t] = 1.0f / (1.0f + expf(-row[E]));
  int e;
  float v;
  if (warp_fast_check([&](int ee) { return row[ee]; }, s_wn, gamma * kBoundSlack * xnorm[t], E,
                      K, e, v))
    warp_write_route(t, K, e, v, topk_idx, topk_w, hist + size_t(t / kRtM) * E);
  else if (lane == 0)
    queue[atomicAdd(queue_count, 1)] = t;
}

__global__ void __launch_bounds__(kRtFixThreads, 2) route_fixup_kernel(
    const float* __restrict__ logits, const float* __restrict__ xnorm,
    const float* __restrict__ wnorm, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w_router, int H, int E, int K, int Rpad, float gamma,
    const int32_t* __restrict__ queue, const int* __restrict__ queue_count,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int32_t* __restrict__ hist,
    ExactStats stats) {
  constexpr int kWarps = kRtFixThreads / 32;
  __shared__ float s_wn[kRtN];
  __shared__ ExactCta<kWarps, kRtFixTokens> xq;
  __shared__ int s_n;
  for (int e = threadIdx.x; e < kRtN; e += blockDim.x) s_wn[e] = e < E ? wnorm[e] : 0.f;
  if (threadIdx.x == 0) s_n = *queue_count;
  __syncthreads();
  const int n = s_n, warp = threadIdx.x >> 5;
  auto cnt_of = [&](int t) { return hist + size_t(t / kRtM) * E; };
  for (int base = blockIdx.x * kRtFixTokens; base < n; base += gridDim.x * kRtFixTokens) {
    if (threadIdx.x == 0) {
      xq.n_pend = 0;
      xq.n_req = 0;
    }
    __syncthreads();
    for (int i = warp; i < kRtFixTokens; i += kWarps) {
      if (base + i >= n) break;
      const int t = queue[base + i];
      const float* row = logits + size_t(t) * Rpad;
      warp_topk_queue(xq, [&](int ee) { return row[ee]; }, s_wn, gamma * kBoundSlack * xnorm[t],
                      t, E, K, x, w_router, H, stats, topk_idx, topk_w, cnt_of);
    }
    cta_topk_finish(xq, x, w_router, H, K, stats, topk_idx, topk_w, cnt_of);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// One CTA of 1024 threads.  Thread (e, part) sums its quarter of the tile
// histograms; counts -> CSR offsets and active list (as block_dispatch), and
// base[b][e] = offsets[e] + sum_{b' < b} hist[b'][e].
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 1024;

__device__ int scan_block_excl(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int s = warp_sums[lane];
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += n;
    }
    warp_sums[lane] = si - s;
    if (lane == 31) *total = si;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) route_scan_kernel(
    const int32_t* __restrict__ hist, int nb, int T, int E, int K, int lo, int hi,
    int with_shared, int with_routed, int sh_lo, int sh_hi, int32_t* __restrict__ base,
    int32_t* __restrict__ offsets,
    int32_t* __restrict__ active, int32_t* __restrict__ n_active) {
  __shared__ int s_part[4][256];
  __shared__ int s_cnt[256], s_off[256], s_wsum[32], s_tot;
  const int tid = threadIdx.x;
  const int e = tid & 255, part = tid >> 8;  // 4 parts of the tile range
  const int b0 = part * nb / 4, b1 = (part + 1) * nb / 4;
  int sum = 0;
  if (e < E)
    for (int b = b0; b < b1; ++b) sum += hist[size_t(b) * E + e];
  s_part[part][e] = sum;
  __syncthreads();
  if (tid < 256)
    s_cnt[tid] = tid < E ? s_part[0][tid] + s_part[1][tid] + s_part[2][tid] + s_part[3][tid] : 0;
  __syncthreads();
  const int cnt = tid < E ? s_cnt[tid] : 0;
  const int ex = scan_block_excl(cnt, s_wsum, &s_tot);
  if (tid < E) {
    s_off[tid] = ex;
    offsets[tid] = ex;
  }
  if (tid == 0) {
    offsets[E] = T * K;  // routed rows end here; the shared block is compacted
    offsets[E + 1] = T * K + (sh_hi - sh_lo);
  }
  const int act = (with_routed && tid < E && tid >= lo && tid < hi && cnt > 0) ? 1 : 0;
  const int apos = scan_block_excl(act, s_wsum, &s_tot);
  if (act) active[apos] = tid;
  if (tid == 0) {
    int na = s_tot;
    if (with_shared && sh_hi > sh_lo) active[na++] = E;
    n_active[0] = na;
  }
  __syncthreads();
  if (e < E) {
    int run = s_off[e];
    for (int p = 0; p < part; ++p) run += s_part[p][e];
    for (int b = b0; b < b1; ++b) {
      base[size_t(b) * E + e] = run;
      run += hist[size_t(b) * E + e];
    }
  }
}

// ---------------------------------------------------------------------------
// One CTA per 128-token tile, 128*K threads (one pair each).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) route_scatter_kernel(
    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const float* __restrict__ shared_gate, const int32_t* __restrict__ base, int T, int H, int E,
    int K, int sh_lo, int sh_hi, int32_t* __restrict__ sorted_tok,
    int32_t* __restrict__ sorted_slot, int32_t* __restrict__ pair_dst,
    int32_t* __restrict__ pair_pos, float* __restrict__ pair_w) {
  __shared__ int s_wcnt[32 * 256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int P = T * K;
  for (int i = tid; i < nw * E; i += blockDim.x) s_wcnt[i] = 0;
  __syncthreads();
  const int p = blockIdx.x * kRtM * K + tid;
  const int e = p < P ? topk_idx[p] : -1;
  const unsigned m = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(m & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) s_wcnt[warp * E + e] = __popc(m);
  __syncthreads();
  if (e >= 0) {
    int pre = 0;
    for (int w = 0; w < warp; ++w) pre += s_wcnt[w * E + e];
    const int pos = base[size_t(blockIdx.x) * E + e] + pre + rank;
    sorted_tok[pos] = p / K;
    sorted_slot[pos] = p % K;
    pair_dst[pos] = p;
    pair_pos[p] = pos;
    pair_w[pos] = topk_w[p];
  }
  const int tb = blockIdx.x * kRtM;
  for (int i = tid; i < kRtM; i += blockDim.x) {
    const int t = tb + i;
    if (t >= sh_lo && t < sh_hi) {  // dispatched row P+(t-sh_lo) is token t
      sorted_tok[P + t - sh_lo] = t;
      pair_dst[P + t - sh_lo] = P + t;
      pair_pos[P + t] = P + t - sh_lo;
      pair_w[P + t - sh_lo] = shared_gate[t];
    }
  }
}

cudaError_t route_tc_init() {
  return cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kRtSmem);
}

float route_tc_gamma(const Dims& d) { return router_tc_gamma(d.H); }

bool route_tc_supported(const Dims& d) {
  return d.E <= kRtN && d.K <= kRtMaxK && d.H % kRtK == 0;
}

// Per-tile expert histogram of given routing (the router kernel produces it
// in its epilogue; this is for routing computed elsewhere): one CTA per
// 128-token tile.
__global__ void __launch_bounds__(256) route_hist_kernel(const int32_t* __restrict__ topk_idx,
                                                         int T, int E, int K,
                                                         int32_t* __restrict__ hist) {
  __shared__ int s_hist[kRtN];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * kRtM * K, p1 = min(T, (blockIdx.x + 1) * kRtM) * K;
  for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) atomicAdd(&s_hist[topk_idx[p]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[size_t(blockIdx.x) * E + e] = s_hist[e];
}

cudaError_t launch_router_tc(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                             const __nv_bfloat16* w_gvec, int32_t* topk_idx, float* topk_w,
                             float* shared_gate, int32_t* hist, int* status, float* logits,
                             float* xnorm, float* wnorm, int32_t* queue, float* diag,
                             cudaStream_t st) {
  CUtensorMap tm_x, tm_w, tm_g;
  const uint64_t H = d.H;
  if (!make_tmap_bf16_2d(&tm_x, x, H, d.T, H * 2, kRtK, kRtM) ||
      !make_tmap_bf16_2d(&tm_w, w_router, H, d.E, H * 2, kRtK, kRtNH) ||
      !make_tmap_bf16_2d(&tm_g, w_gvec, H, 1, H * 2, kRtK, kRtN2))
    return cudaErrorInvalidValue;
  const int nb = (d.T + kRtM - 1) / kRtM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * nb);
  cfg.blockDim = dim3(kRtThreads);
  cfg.dynamicSmemBytes = kRtSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, router_tc_kernel, tm_x, tm_w, tm_g, x, w_router,
                                       int(d.T), int(d.H), int(d.E), int(d.Rpad), logits, xnorm,
                                       wnorm, status + 1);
  if (err != cudaSuccess) return err;
  if (diag) {
    err = cudaMemcpyAsync(diag, logits, sizeof(float) * size_t(d.T) * d.Rpad,
                          cudaMemcpyDeviceToDevice, st);
    if (err != cudaSuccess) return err;
  }
  const float gamma = router_tc_gamma(d.H);
  err = cudaMemsetAsync(hist, 0, sizeof(int32_t) * size_t(nb) * d.E, st);
  if (err != cudaSuccess) return err;
  int* queue_count = status + 10;  // zeroed with the status words
  route_fast_kernel<<<(d.T + kRtFastThreads / 32 - 1) / (kRtFastThreads / 32), kRtFastThreads, 0,
                      st>>>(logits, xnorm, wnorm, d.T, d.E, d.K, d.Rpad, gamma, topk_idx, topk_w,
                            shared_gate, hist, queue, queue_count);
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  route_fixup_kernel<<<4 * sms, kRtFixThreads, 0, st>>>(
      logits, xnorm, wnorm, x, w_router, d.H, d.E, d.K, d.Rpad, gamma, queue, queue_count,
      topk_idx, topk_w, hist, ExactStats{status + 8, status + 9});
  return cudaGetLastError();
}

// Scan + scatter from the routing in ws.topk_idx / topk_w / shared_gate and
// the tile histograms in ws.hist.
static cudaError_t launch_dispatch(const Dims& d, int lo, int hi, int with_shared,
                                   int with_routed, const Workspace& ws, cudaStream_t st) {
  const int nb = (d.T + kRtM - 1) / kRtM;
  route_scan_kernel<<<1, kScanThreads, 0, st>>>(ws.hist, nb, d.T, d.E, d.K, lo, hi, with_shared,
                                                with_routed, d.sh_lo, d.sh_hi, ws.hist_base,
                                                ws.offsets, ws.active, ws.n_active);
  route_scatter_kernel<<<nb, kRtM * d.K, 0, st>>>(ws.topk_idx, ws.topk_w, ws.shared_gate,
                                                  ws.hist_base, d.T, d.H, d.E, d.K, d.sh_lo,
                                                  d.sh_hi, ws.sorted_tok, ws.sorted_slot,
                                                  ws.pair_dst, ws.pair_pos, ws.pair_w);
  return cudaGetLastError();
}

cudaError_t launch_route_tc(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                            const __nv_bfloat16* w_gvec, int lo, int hi, int with_shared,
                            int with_routed, const Workspace& ws, cudaStream_t st) {
  cudaError_t err = cudaMemsetAsync(ws.status, 0, kStatusWords * sizeof(int32_t), st);
  if (err != cudaSuccess) return err;
  err = launch_router_tc(d, x, w_router, w_gvec, ws.topk_idx, ws.topk_w, ws.shared_gate, ws.hist,
                         ws.status, ws.logit_part, ws.xnorm, ws.wnorm, ws.route_queue, ws.diag,
                         st);
  if (err != cudaSuccess) return err;
  return launch_dispatch(d, lo, hi, with_shared, with_routed, ws, st);
}

cudaError_t launch_dispatch_given(const Dims& d, const int32_t* topk_idx, const float* topk_w,
                                  const float* shared_gate, int lo, int hi, int with_shared,
                                  int with_routed, const Workspace& ws, cudaStream_t st) {
  cudaError_t err = cudaMemsetAsync(ws.status, 0, kStatusWords * sizeof(int32_t), st);
  const size_t P = size_t(d.T) * d.K;
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(ws.topk_idx, topk_idx, P * 4, cudaMemcpyDeviceToDevice, st);
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(ws.topk_w, topk_w, P * 4, cudaMemcpyDeviceToDevice, st);
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(ws.shared_gate, shared_gate, size_t(d.T) * 4, cudaMemcpyDeviceToDevice,
                          st);
  if (err != cudaSuccess) return err;
  const int nb = (d.T + kRtM - 1) / kRtM;
  route_hist_kernel<<<nb, 256, 0, st>>>(ws.topk_idx, d.T, d.E, d.K, ws.hist);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  return launch_dispatch(d, lo, hi, with_shared, with_routed, ws, st);
}

}  // namespace pmoe
