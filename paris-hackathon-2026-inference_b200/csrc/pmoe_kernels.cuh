// Host-side launchers shared between the translation units of libparis_moe.
#pragma once
#include "pmoe_common.cuh"

namespace pmoe {

cudaError_t route_init();
cudaError_t stream_init(int num_sms);

// epoch_bump (may be null): a device counter the routing kernel increments
// once (the expert-parallel exchange's epoch); false when it could not, i.e.
// the caller must bump it separately (only the T <= kFusedRouteMaxT path does).
cudaError_t launch_route(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                         const __nv_bfloat16* w_gvec, int lo, int hi, int with_shared,
                         int with_routed, const Workspace& ws, cudaStream_t st,
                         int* epoch_bump = nullptr, const __nv_bfloat16* w_norm = nullptr,
                         float eps = 0.f, __nv_bfloat16* xn = nullptr);
// The decode routing kernel can fuse a decoder layer's RMSNorm (w_norm, eps:
// x is normalised as it is read and written to xn, bit-identical to
// launch_rmsnorm) when this holds for d.
bool route_fuses_norm(const Dims& d);
bool route_bumps_epoch(const Dims& d);
// Accumulation-bound factor gamma of the exact top-k for the routing path
// that launch_route / launch_route_tc take for d (pmoe_exact.cuh).
float route_gamma(const Dims& d);
float route_tc_gamma(const Dims& d);

cudaError_t launch_stream_experts(const Dims& d, const __nv_bfloat16* x,
                                  const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                                  const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                                  const __nv_bfloat16* w_sh_down, const Workspace& ws,
                                  cudaStream_t st, void* mid_event, const EpPeers& ep);

cudaError_t tc_init(int num_sms);
bool tc_supported(const Dims& d);
cudaError_t launch_tc_experts(const Dims& d, const __nv_bfloat16* x,
                              const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                              const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                              const __nv_bfloat16* w_sh_down, const Workspace& ws,
                              const __nv_bfloat16* resid, __nv_bfloat16* y, int lo, int hi,
                              int with_shared, int with_routed, int rank, int world,
                              cudaStream_t st, void* const events[3],
                              const RowsOut* rows_out = nullptr);
cudaError_t launch_combine_slice(const __nv_bfloat16* rows, const int32_t* topk_idx,
                                 const float* topk_w, const float* shared_gate, int T, int H,
                                 int E, int K, int t_lo, int t_hi, __nv_bfloat16* y,
                                 const RowsOut* ydst, const int* abort_if, cudaStream_t st);

// Prefill routing on the tensor cores (router GEMM + top-k epilogue, parallel
// stable dispatch).
cudaError_t route_tc_init();
bool route_tc_supported(const Dims& d);
cudaError_t launch_route_tc(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                            const __nv_bfloat16* w_gvec, int lo, int hi, int with_shared,
                            int with_routed, const Workspace& ws, cudaStream_t st);
// The router GEMM + exact top-k alone, for d.T tokens starting at x, into the
// given arrays (hist: per-128-token-tile expert counts; status: the status
// words (zeroed by the caller), error at [1], exact-evaluation counts at
// [8]/[9], queue length at [10]; logits [d.T][Rpad], xnorm [d.T], wnorm [E],
// queue [d.T]: scratch; diag: optional copy of the fp32 logits).
cudaError_t launch_router_tc(const Dims& d, const __nv_bfloat16* x, const __nv_bfloat16* w_router,
                             const __nv_bfloat16* w_gvec, int32_t* topk_idx, float* topk_w,
                             float* shared_gate, int32_t* hist, int* status, float* logits,
                             float* xnorm, float* wnorm, int32_t* queue, float* diag,
                             cudaStream_t st);
// Exactly rounded logits of all T x E pairs (one warp each); n_inexact (a
// device counter) counts pairs outside the exactness condition.
cudaError_t launch_exact_logits(const __nv_bfloat16* x, const __nv_bfloat16* w, int T, int H,
                                int E, float* out, int* n_inexact, cudaStream_t st);
// Router-row norms for the exact top-k (one warp per row).
cudaError_t launch_row_norms(const __nv_bfloat16* a, int rows, int H, float* out,
                             cudaStream_t st);
// Dispatch (histogram, scan, scatter) from routing computed elsewhere.
cudaError_t launch_dispatch_given(const Dims& d, const int32_t* topk_idx, const float* topk_w,
                                  const float* shared_gate, int lo, int hi, int with_shared,
                                  int with_routed, const Workspace& ws, cudaStream_t st);

// resid (may be null): y = bf16(resid + bf16(sum)), the decoder layer's residual.
cudaError_t launch_combine(const Dims& d, const Workspace& ws, int lo, int hi, int with_shared,
                           int with_routed, const __nv_bfloat16* resid, __nv_bfloat16* y,
                           cudaStream_t st, const EpPeers& ep);
cudaError_t launch_epoch_bump(int* epoch, cudaStream_t st);

// NVLink all-reduce of row-split partials (rows_exchange.cu).
size_t rx_buffer_bytes(int T_max, int H);
size_t rx_region_offset(int T_max, int H, int epoch);
size_t rx_status_offset();
cudaError_t launch_rows_allreduce(void* const* bufs, int T_max, int world, int rank, int epoch,
                                  int T, int H, __nv_bfloat16* y, int num_sms, cudaStream_t st);
// Fused row exchange: the down GEMM stores rows at their token owner, which
// combines its slice locally; then the gather (rows_exchange.cu).
size_t rx_fused_buffer_bytes(int T_max, int H, int K);
size_t rx_fused_rows_offset(int T_max, int H, int K, int epoch);
size_t rx_fused_route_offset(int T_max, int H, int K, int epoch);
// Routing slices of the fused row exchange: this rank's slice [r*T/N,
// (r+1)*T/N) of topk_idx / topk_w / shared_gate goes to every rank's routing
// region (peer stores), flags R are raised and awaited (bounded); *all_* then
// point at the complete routing in this rank's own buffer.
cudaError_t launch_route_exchange(void* const* bufs, int T_max, int world, int rank, int epoch,
                                  int T, int H, int K, const int32_t* topk_idx,
                                  const float* topk_w, const float* shared_gate, int num_sms,
                                  cudaStream_t st, const int32_t** all_idx, const float** all_w,
                                  const float** all_sg);
cudaError_t launch_rows_fused_tail(void* const* bufs, int T_max, int world, int rank, int epoch,
                                   int T, int H, int E, int K, const int32_t* topk_idx,
                                   const float* topk_w, const float* shared_gate,
                                   __nv_bfloat16* y, int num_sms, cudaStream_t st);

// out = Qwen3_5MoeRMSNorm(x; w, eps), bf16 [T][H].
cudaError_t launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, float eps, int T,
                           int H, __nv_bfloat16* out, cudaStream_t st);

}  // namespace pmoe
