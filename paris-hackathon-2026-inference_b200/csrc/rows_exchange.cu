// All-reduce of the per-rank partial outputs of row-split expert parallelism
// (prefill) over NVLink, replacing the NCCL all_reduce of ep.py:140.
//
// Buffer of each rank (CUDA-IPC mapped on every rank):
//   [0, 256)     flags A: flagsA[q] = epoch when rank q's partial is complete
//   [256, 512)   flags B: flagsB[q] = epoch when rank q's token slice is reduced
//   [512, 520)   ticket (CTA completion counter), status word
//   [768, 800)   flags R: flagsR[q] = epoch when rank q's routing slice is
//                delivered (fused exchange with routing slices)
//   [1024, ...)  two parity regions of T_max x H bf16
// Per call (epoch e > 0, parity e & 1), after this rank wrote its partial into
// its own region:
//   publish      raise flagsA[rank] = e on every rank
//   reduce       wait (bounded) for every rank's flagsA; rank r sums its token
//                slice [r*T/N, (r+1)*T/N) over ranks 0..N-1 in that order (fp32,
//                peer loads), stores the bf16 result into its own region, and
//                its last CTA raises flagsB[r] = e on every rank
//   gather       wait (bounded) for every rank's flagsB; y[t] = region of the
//                slice owner of t (peer loads)
// A rank one call ahead writes the other parity; it cannot be two calls ahead
// (its reduce of call e+1 waits for every rank's partial of e+1, written after
// that rank's gather of e).
#include <algorithm>

#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tma.cuh"

namespace pmoe {

constexpr size_t kRxHeader = 1024;
constexpr int kRxFlagsA = 0, kRxFlagsB = 256, kRxTicket = 512, kRxStatus = 516, kRxFlagsR = 768;
static_assert(kRxFlagsR + 4 * kMaxRanks <= 1024, "header");
constexpr int kRxThreads = 256;

struct RxPeers {
  char* base[kMaxRanks];
  int world, rank, epoch;
  size_t region;  // bytes per parity region
};

__device__ __forceinline__ __nv_bfloat16* rx_rows(const RxPeers& p, int q) {
  return reinterpret_cast<__nv_bfloat16*>(p.base[q] + kRxHeader + size_t(p.epoch & 1) * p.region);
}
__device__ __forceinline__ int* rx_flags(const RxPeers& p, int q, int off) {
  return reinterpret_cast<int*>(p.base[q] + off);
}

// Bounded wait of one thread for flags[0..world) >= epoch; false on timeout.
// Returns at once when an earlier wait of this rank already gave up.
__device__ bool rx_wait(const RxPeers& p, int off) {
  const long long t0 = clock64();
  const int* f = rx_flags(p, p.rank, off);
  const int* status = rx_flags(p, p.rank, kRxStatus);
  for (int q = 0; q < p.world; ++q) {
    while (ld_acquire_sys(f + q) < p.epoch) {
      if (__ldcg(status) != 0) return false;
      if (clock64() - t0 > kWaitBudgetCycles) {
        atomicCAS(rx_flags(p, p.rank, kRxStatus), 0, kStatusTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Raise flags[rank] = epoch (flag set at `off`) on every rank, after all of
// this rank's earlier work on the stream -- unless a wait of this rank gave
// up (status word set): its data are then incomplete and peers must not
// read them (they time out in turn and report it).
__global__ void rx_publish_kernel(RxPeers p, int off) {
  __threadfence_system();
  if (__ldcg(rx_flags(p, p.rank, kRxStatus)) != 0) return;
  for (int q = 0; q < p.world; ++q) st_release_sys(rx_flags(p, q, off) + p.rank, p.epoch);
}

// y = this rank's slice region (all T rows after the second flag round),
// unless a wait gave up.
__global__ void __launch_bounds__(kRxThreads) rx_copy_kernel(RxPeers p,
                                                             const uint4* __restrict__ src,
                                                             uint4* __restrict__ dst, long n16) {
  if (__ldcg(rx_flags(p, p.rank, kRxStatus)) != 0) return;
  for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
       i += long(gridDim.x) * blockDim.x)
    dst[i] = __ldcg(src + i);
}

// Bounded wait for every rank's flag at `off` (the kernels after it on the
// stream run once it returns; a timeout leaves status 4).
__global__ void rx_wait_kernel(RxPeers p, int off) { rx_wait(p, off); }

// The CTA-completion ticket: the last CTA to arrive resets it and, unless a
// wait of this call gave up (status word set), raises flagsB[rank] = epoch on
// every rank.  Every CTA takes the ticket, the ones that timed out included,
// so it is back at 0 for the next call.
__device__ void rx_ticket_and_publish(const RxPeers& p) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ticket = rx_flags(p, p.rank, kRxTicket);
    if (atomicAdd(ticket, 1) == int(gridDim.x) - 1) {
      __threadfence_system();
      *ticket = 0;
      if (__ldcg(rx_flags(p, p.rank, kRxStatus)) == 0)
        for (int q = 0; q < p.world; ++q)
          st_release_sys(rx_flags(p, q, kRxFlagsB) + p.rank, p.epoch);
    }
  }
}

__global__ void __launch_bounds__(kRxThreads) rx_reduce_kernel(RxPeers p, int T, int H) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = rx_wait(p, kRxFlagsA) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    rx_ticket_and_publish(p);
    return;
  }
  const int t0 = int(long(p.rank) * T / p.world), t1 = int(long(p.rank + 1) * T / p.world);
  const int h8 = H / 8;
  const long n = long(t1 - t0) * h8;
  __nv_bfloat16* own = rx_rows(p, p.rank);
  for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += long(gridDim.x) * blockDim.x) {
    const size_t off = size_t(t0) * H + size_t(i) * 8;  // row-major: slice rows are contiguous
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 v[kMaxRanks];  // all ranks' loads in flight at once
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < p.world) v[q] = *reinterpret_cast<const uint4*>(rx_rows(p, q) + off);
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {  // fixed order: deterministic
      if (q >= p.world) break;
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v[q]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        s[2 * j] += f.x;
        s[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(s[2 * j], s[2 * j + 1]);
      op[j] = *reinterpret_cast<uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(own + off) = o;
  }
  rx_ticket_and_publish(p);
}

__global__ void __launch_bounds__(kRxThreads) rx_gather_kernel(RxPeers p, int T, int H,
                                                               __nv_bfloat16* __restrict__ y) {
  __shared__ int s_ok;
  if (threadIdx.x == 0)
    s_ok = (__ldcg(rx_flags(p, p.rank, kRxStatus)) == 0 && rx_wait(p, kRxFlagsB)) ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int h8 = H / 8;
  const long n = long(T) * h8;
  const long stride = long(gridDim.x) * blockDim.x;
  // owner of token t: the rank r with r*T/N <= t < (r+1)*T/N
  auto owner = [&](int t) {
    int r = int(long(t) * p.world / T);
    while (r > 0 && long(r) * T / p.world > t) --r;
    while (r + 1 < p.world && long(r + 1) * T / p.world <= t) ++r;
    return r;
  };
  // four independent copies per thread per iteration (peer loads in flight)
  for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long j = i + u * stride;
      if (j < n)
        v[u] = *reinterpret_cast<const uint4*>(rx_rows(p, owner(int(j / h8))) + size_t(j) * 8);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long j = i + u * stride;
      if (j < n) *reinterpret_cast<uint4*>(y + size_t(j) * 8) = v[u];
    }
  }
}

size_t rx_buffer_bytes(int T_max, int H) {
  return kRxHeader + 2 * ((size_t(T_max) * H * 2 + 255) / 256 * 256);
}

size_t rx_status_offset() { return kRxStatus; }

size_t rx_region_offset(int T_max, int H, int epoch) {
  return kRxHeader + size_t(epoch & 1) * ((size_t(T_max) * H * 2 + 255) / 256 * 256);
}

cudaError_t launch_rows_allreduce(void* const* bufs, int T_max, int world, int rank, int epoch,
                                  int T, int H, __nv_bfloat16* y, int num_sms, cudaStream_t st) {
  RxPeers p{};
  for (int q = 0; q < world; ++q) p.base[q] = static_cast<char*>(bufs[q]);
  p.world = world;
  p.rank = rank;
  p.epoch = epoch;
  p.region = (size_t(T_max) * H * 2 + 255) / 256 * 256;
  rx_publish_kernel<<<1, 1, 0, st>>>(p, kRxFlagsA);
  rx_reduce_kernel<<<num_sms * 2, kRxThreads, 0, st>>>(p, T, H);
  rx_gather_kernel<<<num_sms * 4, kRxThreads, 0, st>>>(p, T, H, y);
  return cudaGetLastError();
}

// ---- fused row exchange ------------------------------------------------------
// Buffer: the layout above, then two parity regions of T_max*(K+1) rows x H
// bf16 that receive, from every rank's down GEMM (peer stores), the
// unweighted rows of the tokens this rank owns (token-major, row q at q*H).
// Per call, after the down GEMM on this rank's stream:
//   publish  flagsA[rank] = e on every rank (this rank's rows are delivered)
//   wait     (bounded) for every rank's flagsA
//   combine  this rank's token slice from its own rows region, in the
//            single-GPU order (routed k = 0..K-1, then shared), stored into
//            the slice region of every rank (peer stores)
//   publish  flagsB[rank] = e on every rank
//   wait     (bounded) for every rank's flagsB
//   copy     this rank's slice region (now all T rows) into y.
// Parity safety: a rank writes rows or slices of call e+2 into a region of
// call e only after its wait for flagsA of e+2, which every rank raises after
// its copy of e+1, which follows its own reads of call e.
static size_t rx_rows_region(int T_max, int H, int K) {
  return (size_t(T_max) * (K + 1) * H * 2 + 255) / 256 * 256;
}

// Routing region (fused exchange with routing slices), per parity after the
// rows regions: topk_idx [T_max][K] i32, topk_w [T_max][K] f32,
// shared_gate [T_max] f32.
static size_t rx_route_region(int T_max, int K) {
  return (size_t(T_max) * (2 * K + 1) * 4 + 255) / 256 * 256;
}

size_t rx_fused_buffer_bytes(int T_max, int H, int K) {
  return rx_buffer_bytes(T_max, H) + 2 * rx_rows_region(T_max, H, K) +
         2 * rx_route_region(T_max, K);
}

size_t rx_fused_route_offset(int T_max, int H, int K, int epoch) {
  return rx_buffer_bytes(T_max, H) + 2 * rx_rows_region(T_max, H, K) +
         size_t(epoch & 1) * rx_route_region(T_max, K);
}

// This rank's routing slice [t0, t1) into the routing region (parity of the
// epoch) of every rank, peer stores; made visible system-wide before the
// flag that follows on the stream.
__global__ void __launch_bounds__(kRxThreads) rx_route_push_kernel(
    RxPeers p, size_t route_off, int T_max, int K, int t0, int t1,
    const int32_t* __restrict__ idx, const float* __restrict__ w,
    const float* __restrict__ sg) {
  if (__ldcg(rx_flags(p, p.rank, kRxStatus)) != 0) return;
  const long nk = long(t1 - t0) * K, n = nk + (t1 - t0);
  for (long i = long(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += long(gridDim.x) * blockDim.x) {
    const bool gate = i >= nk;           // the shared-expert gates follow the K-wide arrays
    const long j = gate ? (i - nk) : i;  // element of the slice
    for (int q = 0; q < p.world; ++q) {
      char* r = p.base[q] + route_off;
      if (gate) {
        reinterpret_cast<float*>(r + size_t(T_max) * 2 * K * 4)[t0 + j] = sg[t0 + j];
      } else {
        const size_t o = size_t(t0) * K + j;
        reinterpret_cast<int32_t*>(r)[o] = idx[o];
        reinterpret_cast<float*>(r + size_t(T_max) * K * 4)[o] = w[o];
      }
    }
  }
  __threadfence_system();
}

cudaError_t launch_route_exchange(void* const* bufs, int T_max, int world, int rank, int epoch,
                                  int T, int H, int K, const int32_t* topk_idx,
                                  const float* topk_w, const float* shared_gate, int num_sms,
                                  cudaStream_t st, const int32_t** all_idx, const float** all_w,
                                  const float** all_sg) {
  RxPeers p{};
  for (int q = 0; q < world; ++q) p.base[q] = static_cast<char*>(bufs[q]);
  p.world = world;
  p.rank = rank;
  p.epoch = epoch;
  p.region = (size_t(T_max) * H * 2 + 255) / 256 * 256;
  const size_t off = rx_fused_route_offset(T_max, H, K, epoch);
  const int t0 = int(long(rank) * T / world), t1 = int(long(rank + 1) * T / world);
  const long n = long(t1 - t0) * (K + 1);
  const unsigned blocks =
      unsigned(std::max<long>(1, std::min<long>((n + kRxThreads - 1) / kRxThreads, num_sms)));
  rx_route_push_kernel<<<blocks, kRxThreads, 0, st>>>(p, off, T_max, K, t0, t1, topk_idx,
                                                      topk_w, shared_gate);
  rx_publish_kernel<<<1, 1, 0, st>>>(p, kRxFlagsR);
  rx_wait_kernel<<<1, 1, 0, st>>>(p, kRxFlagsR);
  const char* own = static_cast<const char*>(bufs[rank]) + off;
  *all_idx = reinterpret_cast<const int32_t*>(own);
  *all_w = reinterpret_cast<const float*>(own + size_t(T_max) * K * 4);
  *all_sg = reinterpret_cast<const float*>(own + size_t(T_max) * 2 * K * 4);
  return cudaGetLastError();
}

size_t rx_fused_rows_offset(int T_max, int H, int K, int epoch) {
  return rx_buffer_bytes(T_max, H) + size_t(epoch & 1) * rx_rows_region(T_max, H, K);
}

cudaError_t launch_rows_fused_tail(void* const* bufs, int T_max, int world, int rank, int epoch,
                                   int T, int H, int E, int K, const int32_t* topk_idx,
                                   const float* topk_w, const float* shared_gate,
                                   __nv_bfloat16* y, int num_sms, cudaStream_t st) {
  RxPeers p{};
  for (int q = 0; q < world; ++q) p.base[q] = static_cast<char*>(bufs[q]);
  p.world = world;
  p.rank = rank;
  p.epoch = epoch;
  p.region = (size_t(T_max) * H * 2 + 255) / 256 * 256;
  char* own = static_cast<char*>(bufs[rank]);
  const auto* rows = reinterpret_cast<const __nv_bfloat16*>(
      own + rx_fused_rows_offset(T_max, H, K, epoch));
  auto* reduced = reinterpret_cast<__nv_bfloat16*>(own + rx_region_offset(T_max, H, epoch));
  const int t0 = int(long(rank) * T / world), t1 = int(long(rank + 1) * T / world);
  RowsOut ydst{};
  ydst.world = world;
  for (int q = 0; q < world; ++q)
    ydst.base[q] = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(bufs[q]) +
                                                     rx_region_offset(T_max, H, epoch));
  rx_publish_kernel<<<1, 1, 0, st>>>(p, kRxFlagsA);
  rx_wait_kernel<<<1, 1, 0, st>>>(p, kRxFlagsA);
  const int* status = reinterpret_cast<const int*>(own + kRxStatus);
  cudaError_t e = launch_combine_slice(rows, topk_idx, topk_w, shared_gate, T, H, E, K, t0, t1,
                                       reduced, &ydst, status, st);
  if (e != cudaSuccess) return e;
  rx_publish_kernel<<<1, 1, 0, st>>>(p, kRxFlagsB);
  rx_wait_kernel<<<1, 1, 0, st>>>(p, kRxFlagsB);
  const long n16 = long(T) * H * 2 / 16;  // H % 8 == 0
  const unsigned blocks = unsigned(std::min<long>((n16 + kRxThreads - 1) / kRxThreads,
                                                  long(num_sms) * 4));
  rx_copy_kernel<<<blocks, kRxThreads, 0, st>>>(p, reinterpret_cast<const uint4*>(reduced),
                                                reinterpret_cast<uint4*>(y), n16);
  return cudaGetLastError();
}

}  // namespace pmoe
