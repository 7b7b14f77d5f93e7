// Decoder-layer pieces around the MoE block for the MoE-only stack:
//   xn = Qwen3_5MoeRMSNorm(x) = bf16( x * rsqrt(mean(x^2) + eps) * (1 + w) )
// computed in fp32 (modeling_qwen3_5_moe.py:795-812); the residual add
// (:867-868) is folded into the combine kernels.
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"

namespace pmoe {

constexpr int kNormThreads = 256;

// One CTA per token row; 16-byte loads, fp32 sum of squares, block reduce.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, float eps, int H,
    __nv_bfloat16* __restrict__ out) {
  __shared__ float s_part[kNormThreads / 32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint4* xr = reinterpret_cast<const uint4*>(x + size_t(t) * H);
  const int n8 = H / 8;
  float ss = 0.f;
  for (int i = tid; i < n8; i += kNormThreads) {
    const uint4 v = xr[i];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b[j]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) s_part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += s_part[k];
  const float r = rsqrtf(tot / float(H) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + size_t(t) * H);
  for (int i = tid; i < n8; i += kNormThreads) {
    const uint4 v = xr[i], wv = wr[i];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* c = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b[j]), g = __bfloat1622float2(c[j]);
      __nv_bfloat162 r2 = __floats2bfloat162_rn(f.x * r * (1.f + g.x), f.y * r * (1.f + g.y));
      op[j] = *reinterpret_cast<uint32_t*>(&r2);
    }
    orow[i] = o;
  }
}

cudaError_t launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, float eps, int T,
                           int H, __nv_bfloat16* out, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  rmsnorm_kernel<<<T, kNormThreads, 0, st>>>(x, w, eps, H, out);
  return cudaGetLastError();
}

}  // namespace pmoe
