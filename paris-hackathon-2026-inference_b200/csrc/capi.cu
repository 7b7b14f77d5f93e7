// extern "C" entry points of libparis_moe (declared in include/paris_moe.h).
#include <cstring>
#include <mutex>

#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"

using namespace pmoe;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_init_mu;
bool g_dev_ready[kMaxDevices] = {};
int g_dev_sms[kMaxDevices] = {};

// Per-device one-time set-up on the current device: checks for sm_100 and
// sets kernel attributes.  Cheap after the first call.
int ensure_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PMOE_ERR_CUDA;
  if (g_dev_ready[dev]) return PMOE_OK;
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_dev_ready[dev]) return PMOE_OK;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return PMOE_ERR_CUDA;
  if (prop.major != 10) return PMOE_ERR_DEVICE;
  if (route_init() != cudaSuccess) return PMOE_ERR_CUDA;
  if (stream_init(prop.multiProcessorCount) != cudaSuccess) return PMOE_ERR_CUDA;
  if (tc_init(prop.multiProcessorCount) != cudaSuccess) return PMOE_ERR_CUDA;
  if (route_tc_init() != cudaSuccess) return PMOE_ERR_CUDA;
  g_dev_sms[dev] = prop.multiProcessorCount;
  g_dev_ready[dev] = true;
  return PMOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int T, int H, int E, int K, int I, int Is) {
  if (T < 0 || H <= 0 || E <= 0 || K <= 0 || I <= 0 || Is <= 0) return PMOE_ERR_ARG;
  if (K > E || K > 32) return PMOE_ERR_UNSUPPORTED;
  if (E > 256) return PMOE_ERR_UNSUPPORTED;
  if (H % 256 != 0 || I % 64 != 0 || Is % 64 != 0) return PMOE_ERR_UNSUPPORTED;
  if (long(T) * K > (1L << 30)) return PMOE_ERR_UNSUPPORTED;
  return PMOE_OK;
}

inline const __nv_bfloat16* bf(const uint16_t* p) {
  return reinterpret_cast<const __nv_bfloat16*>(p);
}

}  // namespace

extern "C" {

const char* pmoe_status_string(int s) {
  switch (s) {
    case PMOE_OK: return "ok";
    case PMOE_ERR_ARG: return "invalid argument";
    case PMOE_ERR_ALIGN: return "tensor not 16-byte aligned";
    case PMOE_ERR_WORKSPACE: return "workspace too small";
    case PMOE_ERR_CUDA: return "CUDA runtime error";
    case PMOE_ERR_UNSUPPORTED: return "unsupported shape";
    case PMOE_ERR_PEER_TIMEOUT: return "timed out waiting for a peer GPU";
    case PMOE_ERR_DEVICE: return "device is not sm_100 (B200)";
    case PMOE_ERR_NOALLOC_TOO_LARGE:
      return "shape needs more scratch than pmoe_block_forward_noalloc's fixed array";
    case PMOE_ERR_COMM_CAPACITY:
      return "batch larger than the communicator's exchange buffers (grow them first)";
    default: return "unknown status";
  }
}

const char* pmoe_version(void) { return "paris_moe 0.1.0 sm_100a"; }

int pmoe_workspace_size(int T, int H, int E, int K, int I, int Is, size_t* bytes) {
  if (!bytes) return PMOE_ERR_ARG;
  int s = check_shape(T, H, E, K, I, Is);
  if (s != PMOE_OK) return s;
  *bytes = carve(nullptr, make_dims(T, H, E, K, I, Is)).bytes;
  return PMOE_OK;
}

int pmoe_route(const uint16_t* x, int T, int H, int E, int K, const uint16_t* w_router,
               const uint16_t* w_sh_gvec, int32_t* topk_idx, float* topk_w, int32_t* offsets,
               int32_t* sorted_tok, int32_t* sorted_slot, float* shared_gate, void* workspace,
               size_t workspace_bytes, void* stream) {
  int s = check_shape(T, H, E, K, 64, 64);
  if (s != PMOE_OK) return s;
  if (T == 0) return PMOE_OK;
  if (!x || !w_router || !w_sh_gvec || !workspace) return PMOE_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_router) || !aligned16(w_sh_gvec)) return PMOE_ERR_ALIGN;
  if ((s = ensure_device()) != PMOE_OK) return s;
  Dims d = make_dims(T, H, E, K, 64, 64);
  Workspace ws = carve(workspace, d);
  if (ws.bytes > workspace_bytes) return PMOE_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool route_tc = T > kFusedRouteMaxT && route_tc_supported(d);
  const cudaError_t rerr =
      route_tc ? launch_route_tc(d, bf(x), bf(w_router), bf(w_sh_gvec), 0, E, 1, 1, ws, st)
               : launch_route(d, bf(x), bf(w_router), bf(w_sh_gvec), 0, E, 1, 1, ws, st);
  if (rerr != cudaSuccess) return PMOE_ERR_CUDA;
  const size_t P = size_t(T) * K;
  auto cp = [&](void* dst, const void* src, size_t n) {
    return dst ? cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, st) : cudaSuccess;
  };
  if (cp(topk_idx, ws.topk_idx, P * 4) != cudaSuccess ||
      cp(topk_w, ws.topk_w, P * 4) != cudaSuccess ||
      cp(offsets, ws.offsets, size_t(E + 1) * 4) != cudaSuccess ||
      cp(sorted_tok, ws.sorted_tok, P * 4) != cudaSuccess ||
      cp(sorted_slot, ws.sorted_slot, P * 4) != cudaSuccess ||
      cp(shared_gate, ws.shared_gate, size_t(T) * 4) != cudaSuccess)
    return PMOE_ERR_CUDA;
  return PMOE_OK;
}

int pmoe_route_diag(const uint16_t* x, int T, int H, int E, int K, const uint16_t* w_router,
                    const uint16_t* w_sh_gvec, int32_t* topk_idx, float* topk_w, float* logits,
                    float* gamma, int32_t* stats, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int s = check_shape(T, H, E, K, 64, 64);
  if (s != PMOE_OK) return s;
  if (!x || !w_router || !w_sh_gvec || !workspace || !topk_idx || !topk_w || !logits || !gamma ||
      !stats || T == 0)
    return PMOE_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_router) || !aligned16(w_sh_gvec)) return PMOE_ERR_ALIGN;
  if ((s = ensure_device()) != PMOE_OK) return s;
  Dims d = make_dims(T, H, E, K, 64, 64);
  Workspace ws = carve(workspace, d);
  if (ws.bytes > workspace_bytes) return PMOE_ERR_WORKSPACE;
  ws.diag = logits;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool route_tc = T > kFusedRouteMaxT && route_tc_supported(d);
  const cudaError_t rerr =
      route_tc ? launch_route_tc(d, bf(x), bf(w_router), bf(w_sh_gvec), 0, E, 1, 1, ws, st)
               : launch_route(d, bf(x), bf(w_router), bf(w_sh_gvec), 0, E, 1, 1, ws, st);
  if (rerr != cudaSuccess) return PMOE_ERR_CUDA;
  *gamma = route_tc ? route_tc_gamma(d) : route_gamma(d);
  const size_t P = size_t(T) * K;
  if (cudaMemcpyAsync(topk_idx, ws.topk_idx, P * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(topk_w, ws.topk_w, P * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(stats, ws.status + 8, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return PMOE_ERR_CUDA;
  return PMOE_OK;
}

int pmoe_exact_logits(const uint16_t* x, int T, int H, int E, const uint16_t* w_router,
                      float* logits, int32_t* n_inexact, void* stream) {
  if (T < 0 || H <= 0 || E <= 0 || H % 256 != 0) return PMOE_ERR_ARG;
  if (T == 0) return PMOE_OK;
  if (!x || !w_router || !logits || !n_inexact) return PMOE_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_router)) return PMOE_ERR_ALIGN;
  int s = ensure_device();
  if (s != PMOE_OK) return s;
  return launch_exact_logits(bf(x), bf(w_router), T, H, E, logits, n_inexact,
                             static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

// Decoder-layer extras: y = x + block(RMSNorm(x; w_norm, eps)).
struct LayerArgs {
  const uint16_t* w_norm;
  float eps;
};

// Row-split expert parallelism: routing given (every rank holds all of it)
// and this rank computes its share of the dispatched rows.
struct RowSplit {
  const int32_t* topk_idx;
  const float* topk_w;
  const float* shared_gate;
  int rank, world;
  // Fused exchange (bufs non-null): the down GEMM stores rows at their token
  // owner's buffer and the call ends with the full y on every rank.
  void* const* bufs = nullptr;
  int T_max = 0, epoch = 0;
  // With bufs: route only this rank's token slice and exchange the routing
  // (PMOE_F_ROUTE_SLICE) instead of routing every token on every rank.
  bool route_slice = false;
};

// Shared implementation of the forward entry points.  `ep` (world > 0)
// selects the expert-parallel NVLink exchange; sh_lo/sh_hi is the token range
// whose shared-expert rows this call computes; `layer` (may be null) adds the
// RMSNorm before and the residual after the block.
static int forward_impl(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                        const uint16_t* w_router, const uint16_t* w_gate_up,
                        const uint16_t* w_down, const uint16_t* w_sh_gate,
                        const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                        const uint16_t* w_sh_gvec, int expert_lo, int expert_hi, int sh_lo,
                        int sh_hi, int flags, uint16_t* y, void* workspace,
                        size_t workspace_bytes, void* stream, void* const* events, int n_events,
                        const EpPeers& ep, const LayerArgs* layer = nullptr,
                        const RowSplit* rs = nullptr) {
  int s = check_shape(T, H, E, K, I, Is);
  if (s != PMOE_OK) return s;
  if (expert_lo < 0 || expert_hi > E || expert_lo > expert_hi) return PMOE_ERR_ARG;
  if (sh_lo < 0 || sh_hi > T || sh_lo > sh_hi) return PMOE_ERR_ARG;
  if (flags & ~(PMOE_F_SHARED | PMOE_F_ROUTED | PMOE_F_FORCE_STREAM | PMOE_F_FORCE_TC |
                PMOE_F_ROUTE_SLICE))
    return PMOE_ERR_ARG;
  if ((flags & PMOE_F_ROUTE_SLICE) && !(rs && rs->bufs)) return PMOE_ERR_ARG;
  if (T == 0) return PMOE_OK;
  const void* ptrs[] = {x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec,
                        y, workspace};
  for (const void* p : ptrs) {
    if (!p) return PMOE_ERR_ARG;
    if (!aligned16(p)) return PMOE_ERR_ALIGN;
  }
  if (layer) {
    if (!layer->w_norm || !(layer->eps >= 0.f)) return PMOE_ERR_ARG;
    if (!aligned16(layer->w_norm)) return PMOE_ERR_ALIGN;
  }
  if ((s = ensure_device()) != PMOE_OK) return s;
  Dims d = make_dims(T, H, E, K, I, Is);
  d.sh_lo = sh_lo;
  d.sh_hi = sh_hi;
  Workspace ws = carve(workspace, d);
  if (ws.bytes > workspace_bytes) return PMOE_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int with_shared = (flags & PMOE_F_SHARED) ? 1 : 0;
  const int with_routed = (flags & PMOE_F_ROUTED) ? 1 : 0;
  if ((flags & PMOE_F_FORCE_TC) && (flags & PMOE_F_FORCE_STREAM)) return PMOE_ERR_ARG;
  if ((flags & PMOE_F_FORCE_TC) && !tc_supported(d)) return PMOE_ERR_UNSUPPORTED;
  // Weight streaming while the layer is HBM-bound (decode), tcgen05 grouped
  // GEMMs beyond.  The NVLink exchange rides on the streaming kernels.
  bool use_tc = ep.world == 0 &&
                ((flags & PMOE_F_FORCE_TC) ||
                 (!(flags & PMOE_F_FORCE_STREAM) && T > kFusedRouteMaxT && tc_supported(d)));
  if (rs) {
    const bool given = rs->topk_idx || rs->topk_w || rs->shared_gate;
    if (rs->world < 1 || rs->rank < 0 || rs->rank >= rs->world ||
        (given && (!rs->topk_idx || !rs->topk_w || !rs->shared_gate)) || ep.world > 0 ||
        (flags & PMOE_F_FORCE_STREAM))
      return PMOE_ERR_ARG;
    if (!tc_supported(d) || !route_tc_supported(d)) return PMOE_ERR_UNSUPPORTED;
    if (rs->bufs && (K > 8 || H > 2048 || given)) return PMOE_ERR_UNSUPPORTED;
    use_tc = true;
  }
  if (ep.world > 0 && (flags & PMOE_F_FORCE_TC)) return PMOE_ERR_UNSUPPORTED;
  auto mark = [&](int i) {
    if (events && i < n_events && events[i])
      return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
    return cudaSuccess;
  };
  if (mark(0) != cudaSuccess) return PMOE_ERR_CUDA;
  // The exchange's device epoch: bumped by the decode router kernel itself, or
  // by a one-thread kernel when another routing path runs.
  int* epoch_bump = ep.world > 0 ? const_cast<int*>(ep.epoch_dev) : nullptr;
  if (epoch_bump && !route_bumps_epoch(d)) {
    if (launch_epoch_bump(epoch_bump, st) != cudaSuccess) return PMOE_ERR_CUDA;
    epoch_bump = nullptr;
  }
  // The block reads xin; a decoder layer normalises x first and adds it back
  // in the combine (in place, y == x, is allowed: each combine thread reads
  // its residual chunk before writing the same chunk).
  // Prefill-sized batches route on the tensor cores.
  const bool route_tc = use_tc && T > kFusedRouteMaxT && route_tc_supported(d);
  const __nv_bfloat16* xin = bf(x);
  const __nv_bfloat16* resid = nullptr;
  // The decode routing kernel normalises x itself (writing xn, bit-identical
  // to the standalone RMSNorm kernel); other paths run that kernel first.
  const bool norm_in_route = layer && !rs && !route_tc && route_fuses_norm(d);
  if (layer) {
    if (!norm_in_route &&
        launch_rmsnorm(bf(x), bf(layer->w_norm), layer->eps, T, H, ws.xn, st) != cudaSuccess)
      return PMOE_ERR_CUDA;
    xin = ws.xn;
    resid = bf(x);
  }
  cudaError_t rerr = cudaSuccess;
  if (rs && rs->bufs && rs->route_slice) {
    // This rank's token slice on the tensor-core router (the exact top-k
    // makes each token's routing independent of the batch it is routed in),
    // the slices exchanged by peer stores, then the dispatch of all T tokens.
    const int t0 = int(long(rs->rank) * T / rs->world);
    const int t1 = int(long(rs->rank + 1) * T / rs->world);
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int32_t* ai = nullptr;
    const float *aw = nullptr, *asg = nullptr;
    rerr = cudaMemsetAsync(ws.status, 0, kStatusWords * sizeof(int32_t), st);
    if (rerr == cudaSuccess && t1 > t0)
      rerr = launch_router_tc(make_dims(t1 - t0, H, E, K, I, Is), xin + size_t(t0) * H,
                              bf(w_router), bf(w_sh_gvec), ws.topk_idx + size_t(t0) * K,
                              ws.topk_w + size_t(t0) * K, ws.shared_gate + t0, ws.hist,
                              ws.status, ws.logit_part, ws.xnorm, ws.wnorm, ws.route_queue,
                              nullptr, st);
    if (rerr == cudaSuccess)
      rerr = launch_route_exchange(rs->bufs, rs->T_max, rs->world, rs->rank, rs->epoch, T, H, K,
                                   ws.topk_idx, ws.topk_w, ws.shared_gate, sms, st, &ai, &aw,
                                   &asg);
    if (rerr == cudaSuccess)
      rerr = launch_dispatch_given(d, ai, aw, asg, expert_lo, expert_hi, with_shared,
                                   with_routed, ws, st);
  } else {
  rerr =
      rs && rs->topk_idx
          ? launch_dispatch_given(d, rs->topk_idx, rs->topk_w, rs->shared_gate, expert_lo,
                                  expert_hi, with_shared, with_routed, ws, st)
      : rs ? launch_route_tc(d, xin, bf(w_router), bf(w_sh_gvec), expert_lo, expert_hi,
                             with_shared, with_routed, ws, st)
      : route_tc ? launch_route_tc(d, xin, bf(w_router), bf(w_sh_gvec), expert_lo, expert_hi,
                                   with_shared, with_routed, ws, st)
      : norm_in_route
          ? launch_route(d, bf(x), bf(w_router), bf(w_sh_gvec), expert_lo, expert_hi, with_shared,
                         with_routed, ws, st, epoch_bump, bf(layer->w_norm), layer->eps, ws.xn)
          : launch_route(d, xin, bf(w_router), bf(w_sh_gvec), expert_lo, expert_hi, with_shared,
                         with_routed, ws, st, epoch_bump);
  }
  if (rerr != cudaSuccess) return PMOE_ERR_CUDA;
  if (use_tc) {
    void* ev[3] = {nullptr, nullptr, nullptr};  // before gate_up, after gate_up, after down
    for (int i = 0; i < 3; ++i)
      if (events && i + 1 < n_events) ev[i] = events[i + 1];
    RowsOut ro{};
    const bool fused = rs && rs->bufs;
    if (fused) {
      ro.world = rs->world;
      for (int q = 0; q < rs->world; ++q)
        ro.base[q] = reinterpret_cast<__nv_bfloat16*>(
            static_cast<char*>(rs->bufs[q]) + rx_fused_rows_offset(rs->T_max, H, K, rs->epoch));
    }
    if (launch_tc_experts(d, xin, bf(w_gate_up), bf(w_down), bf(w_sh_gate), bf(w_sh_up),
                          bf(w_sh_down), ws, resid, reinterpret_cast<__nv_bfloat16*>(y),
                          expert_lo, expert_hi, with_shared, with_routed, rs ? rs->rank : 0,
                          rs ? rs->world : 1, st, ev, fused ? &ro : nullptr) != cudaSuccess)
      return PMOE_ERR_CUDA;
    if (fused) {
      int sms = 148;
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (launch_rows_fused_tail(rs->bufs, rs->T_max, rs->world, rs->rank, rs->epoch, T, H, E, K,
                                 ws.topk_idx, ws.topk_w, ws.shared_gate,
                                 reinterpret_cast<__nv_bfloat16*>(y), sms, st) != cudaSuccess)
        return PMOE_ERR_CUDA;
    }
    if (mark(4) != cudaSuccess) return PMOE_ERR_CUDA;
    return PMOE_OK;
  }
  if (mark(1) != cudaSuccess) return PMOE_ERR_CUDA;
  if (launch_stream_experts(d, xin, bf(w_gate_up), bf(w_down), bf(w_sh_gate), bf(w_sh_up),
                            bf(w_sh_down), ws, st, events && n_events > 2 ? events[2] : nullptr,
                            ep) != cudaSuccess)
    return PMOE_ERR_CUDA;
  if (mark(3) != cudaSuccess) return PMOE_ERR_CUDA;
  // After the exchange every rank holds all routed rows and all shared rows.
  Dims dc = d;
  if (ep.world > 0) {
    dc.sh_lo = 0;
    dc.sh_hi = T;
  }
  if (launch_combine(dc, ws, ep.world > 0 ? 0 : expert_lo, ep.world > 0 ? E : expert_hi,
                     ep.world > 0 ? 1 : with_shared, ep.world > 0 ? 1 : with_routed, resid,
                     reinterpret_cast<__nv_bfloat16*>(y), st, ep) != cudaSuccess)
    return PMOE_ERR_CUDA;
  if (mark(4) != cudaSuccess) return PMOE_ERR_CUDA;
  return PMOE_OK;
}

int pmoe_block_forward_profiled(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                                const uint16_t* w_router, const uint16_t* w_gate_up,
                                const uint16_t* w_down, const uint16_t* w_sh_gate,
                                const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                                const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                                int flags, uint16_t* y, void* workspace, size_t workspace_bytes,
                                void* stream, void* const* events, int n_events) {
  const EpPeers none{};
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, expert_lo, expert_hi, 0, T, flags, y, workspace,
                      workspace_bytes, stream, events, n_events, none);
}

int pmoe_block_forward(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                       const uint16_t* w_router, const uint16_t* w_gate_up,
                       const uint16_t* w_down, const uint16_t* w_sh_gate,
                       const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                       const uint16_t* w_sh_gvec, int expert_lo, int expert_hi, int flags,
                       uint16_t* y, void* workspace, size_t workspace_bytes, void* stream) {
  return pmoe_block_forward_profiled(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down,
                                     w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec, expert_lo,
                                     expert_hi, flags, y, workspace, workspace_bytes, stream,
                                     nullptr, 0);
}

// ---- expert parallelism ------------------------------------------------------

// Exchange buffer header: flags [0,256), CTA ticket at 256, device epoch at 384,
// sticky status word at 448 (set by a combine whose peer wait gave up; only
// a fresh, zeroed buffer clears it).
static const size_t kEpHeader = 512;
static const size_t kEpTicket = 256;
static const size_t kEpEpoch = 384;
static const size_t kEpSticky = 448;

int pmoe_ep_buffer_bytes(int T_max, int H, int K, size_t* bytes) {
  if (!bytes || T_max <= 0 || H <= 0 || K <= 0) return PMOE_ERR_ARG;
  const size_t rows = (size_t(T_max) * K + T_max) * H * sizeof(float);
  *bytes = kEpHeader + 2 * ((rows + 255) / 256 * 256);
  return PMOE_OK;
}

// Fills `ep` for an exchange over peer_bufs (null peer_bufs: no exchange).
// epoch > 0: host epoch; epoch == 0: the device counter in this rank's buffer
// header (bumped by every call; CUDA-graph capturable).
static int setup_ep(int T, int H, int K, int flags, void* const* peer_bufs,
                    size_t peer_buf_bytes, int rank, int world, int epoch, EpPeers& ep) {
  ep = EpPeers{};
  if (!peer_bufs) return PMOE_OK;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || epoch < 0)
    return PMOE_ERR_ARG;
  if (T > kFusedRouteMaxT && !(flags & PMOE_F_FORCE_STREAM)) return PMOE_ERR_UNSUPPORTED;
  const size_t half = (peer_buf_bytes - kEpHeader) / 2;
  const size_t need = (size_t(T) * K + T) * H * sizeof(float);
  if (peer_buf_bytes < kEpHeader || need > half) return PMOE_ERR_WORKSPACE;
  for (int r = 0; r < world; ++r) {
    if (!peer_bufs[r] || !aligned16(peer_bufs[r])) return PMOE_ERR_ARG;
    char* b = static_cast<char*>(peer_bufs[r]);
    ep.rows[r] = reinterpret_cast<float*>(b + kEpHeader);
    ep.flags[r] = reinterpret_cast<int*>(b);
  }
  ep.par_stride = (half / 256 * 256) / sizeof(float);
  char* own = static_cast<char*>(peer_bufs[rank]);
  ep.ticket = reinterpret_cast<int*>(own + kEpTicket);
  ep.sticky = reinterpret_cast<int*>(own + kEpSticky);
  ep.epoch_dev = epoch == 0 ? reinterpret_cast<const int*>(own + kEpEpoch) : nullptr;
  ep.world = world;
  ep.rank = rank;
  ep.epoch = epoch;
  return PMOE_OK;
}

int pmoe_block_forward_ep(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                          const uint16_t* w_router, const uint16_t* w_gate_up,
                          const uint16_t* w_down, const uint16_t* w_sh_gate,
                          const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                          const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                          int shared_lo, int shared_hi, int flags, void* const* peer_bufs,
                          size_t peer_buf_bytes, int rank, int world, int epoch, uint16_t* y,
                          void* workspace, size_t workspace_bytes, void* stream) {
  EpPeers ep;
  const int s = setup_ep(T, H, K, flags, peer_bufs, peer_buf_bytes, rank, world, epoch, ep);
  if (s != PMOE_OK) return s;
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, expert_lo, expert_hi, shared_lo, shared_hi, flags, y,
                      workspace, workspace_bytes, stream, nullptr, 0, ep);
}

int pmoe_layer_forward(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                       const uint16_t* w_norm, float eps, const uint16_t* w_router,
                       const uint16_t* w_gate_up, const uint16_t* w_down,
                       const uint16_t* w_sh_gate, const uint16_t* w_sh_up,
                       const uint16_t* w_sh_down, const uint16_t* w_sh_gvec, int expert_lo,
                       int expert_hi, int shared_lo, int shared_hi, int flags,
                       void* const* peer_bufs, size_t peer_buf_bytes, int rank, int world,
                       int epoch, uint16_t* y, void* workspace, size_t workspace_bytes,
                       void* stream) {
  EpPeers ep;
  const int s = setup_ep(T, H, K, flags, peer_bufs, peer_buf_bytes, rank, world, epoch, ep);
  if (s != PMOE_OK) return s;
  const LayerArgs layer{w_norm, eps};
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, expert_lo, expert_hi, shared_lo, shared_hi, flags, y,
                      workspace, workspace_bytes, stream, nullptr, 0, ep, &layer);
}

int pmoe_route_slice(const uint16_t* x, int T, int H, int E, int K, int I, int Is, int t0,
                     int t1, const uint16_t* w_router, const uint16_t* w_sh_gvec,
                     int32_t* topk_idx, float* topk_w, float* shared_gate, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int s = check_shape(T, H, E, K, I, Is);
  if (s != PMOE_OK) return s;
  if (t0 < 0 || t1 > T || t0 > t1) return PMOE_ERR_ARG;
  if (t0 == t1) return PMOE_OK;
  const void* ptrs[] = {x, w_router, w_sh_gvec, topk_idx, topk_w, shared_gate, workspace};
  for (const void* p : ptrs)
    if (!p) return PMOE_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_router) || !aligned16(w_sh_gvec) || !aligned16(workspace))
    return PMOE_ERR_ALIGN;
  if ((s = ensure_device()) != PMOE_OK) return s;
  Dims d = make_dims(T, H, E, K, I, Is);
  if (!route_tc_supported(d)) return PMOE_ERR_UNSUPPORTED;
  Workspace ws = carve(workspace, d);
  if (ws.bytes > workspace_bytes) return PMOE_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Dims ds = make_dims(t1 - t0, H, E, K, I, Is);
  if (cudaMemsetAsync(ws.status, 0, kStatusWords * sizeof(int32_t), st) != cudaSuccess ||
      launch_router_tc(ds, bf(x) + size_t(t0) * H, bf(w_router), bf(w_sh_gvec),
                       topk_idx + size_t(t0) * K, topk_w + size_t(t0) * K, shared_gate + t0,
                       ws.hist, ws.status, ws.logit_part, ws.xnorm, ws.wnorm, ws.route_queue,
                       nullptr, st) != cudaSuccess)
    return PMOE_ERR_CUDA;
  return PMOE_OK;
}

int pmoe_block_forward_rows(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                            const uint16_t* w_router, const uint16_t* w_gate_up,
                            const uint16_t* w_down, const uint16_t* w_sh_gate,
                            const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                            const uint16_t* w_sh_gvec, const int32_t* topk_idx,
                            const float* topk_w, const float* shared_gate, int expert_lo,
                            int expert_hi, int rank, int world, int flags, uint16_t* y,
                            void* workspace, size_t workspace_bytes, void* stream) {
  const EpPeers none{};
  const RowSplit rs{topk_idx, topk_w, shared_gate, rank, world};
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, expert_lo, expert_hi, 0, T, flags, y, workspace,
                      workspace_bytes, stream, nullptr, 0, none, nullptr, &rs);
}

int pmoe_block_forward_rows_profiled(
    const uint16_t* x, int T, int H, int E, int K, int I, int Is, const uint16_t* w_router,
    const uint16_t* w_gate_up, const uint16_t* w_down, const uint16_t* w_sh_gate,
    const uint16_t* w_sh_up, const uint16_t* w_sh_down, const uint16_t* w_sh_gvec,
    const int32_t* topk_idx, const float* topk_w, const float* shared_gate, int expert_lo,
    int expert_hi, int rank, int world, int flags, uint16_t* y, void* workspace,
    size_t workspace_bytes, void* stream, void* const* events, int n_events) {
  const EpPeers none{};
  const RowSplit rs{topk_idx, topk_w, shared_gate, rank, world};
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, expert_lo, expert_hi, 0, T, flags, y, workspace,
                      workspace_bytes, stream, events, n_events, none, nullptr, &rs);
}

int pmoe_rows_fused_buffer_bytes(int T_max, int H, int K, size_t* bytes) {
  if (!bytes || T_max <= 0 || H <= 0 || H % 8 != 0 || K <= 0) return PMOE_ERR_ARG;
  *bytes = rx_fused_buffer_bytes(T_max, H, K);
  return PMOE_OK;
}

int pmoe_block_forward_rows_fused(
    const uint16_t* x, int T, int H, int E, int K, int I, int Is, const uint16_t* w_router,
    const uint16_t* w_gate_up, const uint16_t* w_down, const uint16_t* w_sh_gate,
    const uint16_t* w_sh_up, const uint16_t* w_sh_down, const uint16_t* w_sh_gvec, int rank,
    int world, void* const* bufs, int T_max, int epoch, int flags, uint16_t* y,
    void* workspace, size_t workspace_bytes, void* stream, void* const* events, int n_events) {
  if (!bufs || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || epoch <= 0 ||
      T > T_max || (flags & (PMOE_F_SHARED | PMOE_F_ROUTED)) != (PMOE_F_SHARED | PMOE_F_ROUTED))
    return PMOE_ERR_ARG;
  for (int q = 0; q < world; ++q)
    if (!bufs[q] || !aligned16(bufs[q])) return PMOE_ERR_ARG;
  const EpPeers none{};
  RowSplit rs{nullptr, nullptr, nullptr, rank, world};
  rs.bufs = bufs;
  rs.T_max = T_max;
  rs.epoch = epoch;
  rs.route_slice = (flags & PMOE_F_ROUTE_SLICE) != 0;
  return forward_impl(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, 0, E, 0, T, flags, y, workspace, workspace_bytes,
                      stream, events, n_events, none, nullptr, &rs);
}

int pmoe_rows_buffer_bytes(int T_max, int H, size_t* bytes) {
  if (!bytes || T_max <= 0 || H <= 0 || H % 8 != 0) return PMOE_ERR_ARG;
  *bytes = rx_buffer_bytes(T_max, H);
  return PMOE_OK;
}

int pmoe_rows_partial(void* own_buf, int T_max, int H, int epoch, void** partial) {
  if (!own_buf || !partial || T_max <= 0 || H <= 0 || epoch <= 0) return PMOE_ERR_ARG;
  *partial = static_cast<char*>(own_buf) + rx_region_offset(T_max, H, epoch);
  return PMOE_OK;
}

int pmoe_rows_allreduce(void* const* bufs, int T_max, int T, int H, int rank, int world,
                        int epoch, uint16_t* y, void* stream) {
  if (!bufs || !y || world < 1 || world > kMaxRanks || rank < 0 || rank >= world ||
      epoch <= 0 || T < 0 || T > T_max || H <= 0 || H % 8 != 0)
    return PMOE_ERR_ARG;
  for (int q = 0; q < world; ++q)
    if (!bufs[q] || !aligned16(bufs[q])) return PMOE_ERR_ARG;
  if (!aligned16(y)) return PMOE_ERR_ALIGN;
  if (T == 0) return PMOE_OK;
  int s = ensure_device();
  if (s != PMOE_OK) return s;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  return launch_rows_allreduce(bufs, T_max, world, rank, epoch, T, H,
                               reinterpret_cast<__nv_bfloat16*>(y), sms,
                               static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_rows_status(const void* own_buf, int* status) {
  if (!own_buf || !status) return PMOE_ERR_ARG;
  return cudaMemcpy(status, static_cast<const char*>(own_buf) + rx_status_offset(), sizeof(int),
                    cudaMemcpyDeviceToHost) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_ep_status_async(const void* own_buf, int* dst, void* stream) {
  if (!own_buf || !dst) return PMOE_ERR_ARG;
  return cudaMemcpyAsync(dst, static_cast<const char*>(own_buf) + kEpSticky, sizeof(int),
                         cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_rows_status_async(const void* own_buf, int* dst, void* stream) {
  if (!own_buf || !dst) return PMOE_ERR_ARG;
  return cudaMemcpyAsync(dst, static_cast<const char*>(own_buf) + rx_status_offset(),
                         sizeof(int), cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_rmsnorm(const uint16_t* x, int T, int H, const uint16_t* w_norm, float eps,
                 uint16_t* out, void* stream) {
  if (T < 0 || H <= 0 || H % 8 != 0 || !(eps >= 0.f)) return PMOE_ERR_ARG;
  if (T == 0) return PMOE_OK;
  if (!x || !w_norm || !out) return PMOE_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_norm) || !aligned16(out)) return PMOE_ERR_ALIGN;
  int s = ensure_device();
  if (s != PMOE_OK) return s;
  return launch_rmsnorm(bf(x), bf(w_norm), eps, T, H, reinterpret_cast<__nv_bfloat16*>(out),
                        static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_read_status(const void* workspace, int T, int H, int E, int K, int I, int Is,
                     int* status) {
  if (!workspace || !status) return PMOE_ERR_ARG;
  int s = check_shape(T, H, E, K, I, Is);
  if (s != PMOE_OK) return s;
  Workspace ws = carve(const_cast<void*>(workspace), make_dims(T, H, E, K, I, Is));
  return cudaMemcpy(status, ws.status + 1, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return PMOE_ERR_ARG;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return PMOE_ERR_CUDA;
  return cudaMemset(*ptr, 0, bytes) == cudaSuccess ? PMOE_OK : PMOE_ERR_CUDA;
}

int pmoe_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? PMOE_OK : PMOE_ERR_CUDA; }

int pmoe_ipc_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return PMOE_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return PMOE_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return PMOE_OK;
}

int pmoe_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return PMOE_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? PMOE_OK
             : PMOE_ERR_CUDA;
}

int pmoe_ipc_close(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? PMOE_OK : PMOE_ERR_CUDA;
}

}  // extern "C"
