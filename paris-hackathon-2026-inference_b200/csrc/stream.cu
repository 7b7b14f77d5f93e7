// Weight-streaming expert kernels for the HBM-bound decode regime (small T).
//
// At T <= 64 each active expert sees a handful of tokens, so the block is a
// stream over ~1.4 GB of expert weights with arithmetic intensity of a few
// FLOP/B.  Every weight byte is loaded exactly once with a 128-bit
// L1-bypassing load straight into mma.sync fragments (see mma_k32); the
// activations (tiny, re-read by the warps of a CTA) come through L1.
//
// Reference arithmetic: the per-expert body of Qwen3_5MoeExperts.forward
// (modeling_qwen3_5_moe.py:743-749), the shared expert Qwen3_5MoeMLP
// (:709-711) with its sigmoid gate (:788), and the routed combine of
// engine/kernels/moe_grouped_mlp.py:152-163 (done here in fp32).
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"

namespace pmoe {

struct ExpertTables {
  const int32_t* active;
  const int32_t* n_active;
  const int32_t* offsets;  // [E+2]
  const int32_t* sorted_tok;
  const int32_t* pair_dst;
  const float* pair_w;
};

// Units of work per expert and their weight rows.
// gate_up: unit = 16 intermediate columns j (gate rows j.., up rows I+j..).
// down:    unit = 16 output rows of down_proj.

__global__ void __launch_bounds__(256) gate_up_stream_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate_up,
    const __nv_bfloat16* __restrict__ w_sh_gate, const __nv_bfloat16* __restrict__ w_sh_up,
    ExpertTables tb, int H, int E, int I, int Is, int ldh, __nv_bfloat16* __restrict__ h) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int U = (I > Is ? I : Is) / 16;
  const long n_units = long(tb.n_active[0]) * U;
  const long nwarps = long(gridDim.x) * (blockDim.x / 32);
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (long u = long(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); u < n_units;
       u += nwarps) {
    const int e = tb.active[u / U];
    const int jg = int(u % U);
    const bool sh = (e == E);
    const int Ie = sh ? Is : I;
    if (jg * 16 >= Ie) continue;
    const __nv_bfloat16* wg =
        sh ? w_sh_gate + size_t(jg * 16) * H : w_gate_up + (size_t(e) * 2 * I + jg * 16) * H;
    const __nv_bfloat16* wu =
        sh ? w_sh_up + size_t(jg * 16) * H : w_gate_up + (size_t(e) * 2 * I + I + jg * 16) * H;
    const __nv_bfloat16* wg0 = wg + size_t(g) * H + 8 * c;
    const __nv_bfloat16* wg1 = wg0 + size_t(8) * H;
    const __nv_bfloat16* wu0 = wu + size_t(g) * H + 8 * c;
    const __nv_bfloat16* wu1 = wu0 + size_t(8) * H;
    const int p0 = tb.offsets[e];
    const int n = tb.offsets[e + 1] - p0;
    for (int nb = 0; nb < n; nb += 32) {
      const __nv_bfloat16* xp[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = nb + q * 8 + g;
        xp[q] = i < n ? x + size_t(tb.sorted_tok[p0 + i]) * H + 8 * c : nullptr;
      }
      const int ng = min(4, (n - nb + 7) / 8);  // warp-uniform
      float ag[4][4] = {}, au[4][4] = {};
#pragma unroll 4
      for (int k0 = 0; k0 < H; k0 += 32) {
        const uint4 a0 = ldg_stream(wg0 + k0), a1 = ldg_stream(wg1 + k0);
        const uint4 b0 = ldg_stream(wu0 + k0), b1 = ldg_stream(wu1 + k0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q < ng) {
            const uint4 xv = xp[q] ? ldg_keep(xp[q] + k0) : zero;
            mma_k32(ag[q], a0, a1, xv);
            mma_k32(au[q], b0, b1, xv);
          }
        }
      }
      // Epilogue: rows j = jg*16 + g (+8), columns = dispatched rows p0+nb+q*8+2c (+1).
      const int j0 = jg * 16 + g;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < ng) {
          const int i = nb + q * 8 + 2 * c;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (i + hh < n) {
              __nv_bfloat16* hrow = h + size_t(p0 + i + hh) * ldh;
              hrow[j0] = __float2bfloat16_rn(silu_f(ag[q][hh]) * au[q][hh]);
              hrow[j0 + 8] = __float2bfloat16_rn(silu_f(ag[q][2 + hh]) * au[q][2 + hh]);
            }
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(256) down_stream_kernel(
    const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ w_down,
    const __nv_bfloat16* __restrict__ w_sh_down, ExpertTables tb, int H, int E, int I, int Is,
    int ldh, float* __restrict__ rows) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int U = H / 16;
  const long n_units = long(tb.n_active[0]) * U;
  const long nwarps = long(gridDim.x) * (blockDim.x / 32);
  for (long u = long(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); u < n_units;
       u += nwarps) {
    const int e = tb.active[u / U];
    const int rg = int(u % U);
    const bool sh = (e == E);
    const int Ke = sh ? Is : I;
    const __nv_bfloat16* w =
        sh ? w_sh_down + size_t(rg * 16) * Is : w_down + (size_t(e) * H + rg * 16) * I;
    const __nv_bfloat16* w0 = w + size_t(g) * Ke + 8 * c;
    const __nv_bfloat16* w1 = w0 + size_t(8) * Ke;
    const int p0 = tb.offsets[e];
    const int n = tb.offsets[e + 1] - p0;
    for (int nb = 0; nb < n; nb += 32) {
      const __nv_bfloat16* hp[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = nb + q * 8 + g;
        hp[q] = i < n ? h + size_t(p0 + i) * ldh + 8 * c : nullptr;
      }
      const int ng = min(4, (n - nb + 7) / 8);
      float acc[4][4] = {};
      const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll 4
      for (int k0 = 0; k0 < Ke; k0 += 32) {
        const uint4 a0 = ldg_stream(w0 + k0), a1 = ldg_stream(w1 + k0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q < ng) {
            const uint4 hv = hp[q] ? ldg_keep(hp[q] + k0) : zero;
            mma_k32(acc[q], a0, a1, hv);
          }
        }
      }
      const int r0 = rg * 16 + g;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < ng) {
          const int i = nb + q * 8 + 2 * c;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (i + hh < n) {
              const int p = p0 + i + hh;
              const float wt = tb.pair_w[p];
              float* orow = rows + size_t(tb.pair_dst[p]) * H;
              orow[r0] = acc[q][hh] * wt;
              orow[r0 + 8] = acc[q][2 + hh] * wt;
            }
          }
        }
      }
    }
  }
}

// y[t, :] = bf16( sum_{s<K, expert in [lo,hi)} rows[t*K+s, :] + rows[T*K+t, :] )
// fp32, fixed summation order.  One thread per 4 columns.
__global__ void __launch_bounds__(256) combine_kernel(
    const float* __restrict__ rows, const int32_t* __restrict__ topk_idx, int T, int H, int K,
    int lo, int hi, int with_shared, int with_routed, __nv_bfloat16* __restrict__ y) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const int cols4 = H / 4;
  if (i >= long(T) * cols4) return;
  const int t = int(i / cols4), c4 = int(i % cols4);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (with_routed) {
    for (int k = 0; k < K; ++k) {
      const int e = topk_idx[size_t(t) * K + k];
      if (e < lo || e >= hi) continue;
      const float4 v = reinterpret_cast<const float4*>(rows + (size_t(t) * K + k) * H)[c4];
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
  }
  if (with_shared) {
    const float4 v = reinterpret_cast<const float4*>(rows + (size_t(T) * K + t) * H)[c4];
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
  }
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(s.x, s.y);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(s.z, s.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo2);
  packed.y = *reinterpret_cast<uint32_t*>(&hi2);
  reinterpret_cast<uint2*>(y + size_t(t) * H)[c4] = packed;
}

static int g_stream_blocks = 0;

cudaError_t stream_init(int num_sms) {
  int per_sm_gu = 0, per_sm_dn = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_gu, gate_up_stream_kernel, 256, 0);
  if (err != cudaSuccess) return err;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_dn, down_stream_kernel, 256, 0);
  if (err != cudaSuccess) return err;
  int per_sm = per_sm_gu < per_sm_dn ? per_sm_gu : per_sm_dn;
  if (per_sm < 1) per_sm = 1;
  g_stream_blocks = num_sms * per_sm;
  return cudaSuccess;
}

cudaError_t launch_stream_experts(const Dims& d, const __nv_bfloat16* x,
                                  const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                                  const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                                  const __nv_bfloat16* w_sh_down, const Workspace& ws,
                                  cudaStream_t st, void* mid_event) {
  ExpertTables tb{ws.active, ws.n_active, ws.offsets, ws.sorted_tok, ws.pair_dst, ws.pair_w};
  const int blocks = g_stream_blocks > 0 ? g_stream_blocks : 148 * 4;
  gate_up_stream_kernel<<<blocks, 256, 0, st>>>(x, w_gate_up, w_sh_gate, w_sh_up, tb, d.H, d.E,
                                                d.I, d.Is, d.ldh, ws.h);
  if (mid_event) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(mid_event), st);
    if (e != cudaSuccess) return e;
  }
  down_stream_kernel<<<blocks, 256, 0, st>>>(ws.h, w_down, w_sh_down, tb, d.H, d.E, d.I, d.Is,
                                             d.ldh, ws.rows);
  return cudaGetLastError();
}

cudaError_t launch_combine(const Dims& d, const Workspace& ws, int lo, int hi, int with_shared,
                           int with_routed, __nv_bfloat16* y, cudaStream_t st) {
  const long n = long(d.T) * (d.H / 4);
  if (n == 0) return cudaSuccess;
  combine_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(ws.rows, ws.topk_idx, d.T, d.H, d.K,
                                                           lo, hi, with_shared, with_routed, y);
  return cudaGetLastError();
}

}  // namespace pmoe
