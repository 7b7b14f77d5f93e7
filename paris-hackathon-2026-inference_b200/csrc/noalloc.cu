// pmoe_block_forward_noalloc: the MoE block for callers that cannot allocate
// device memory.
//
// Some callers of this library have no way to hand it a workspace: a serving
// engine that reserves all of HBM up front for its KV cache and weights and
// forbids allocations on the decode path (cudaMalloc there can also stall the
// whole device), or a host program in another language that reaches the
// library through a bare FFI and owns no device allocator.  For them this
// entry point takes only the inputs and the output; its scratch lives in one
// fixed-size array in device memory, declared below.
//
// The array occupies kNoallocScratchBytes on every GPU that loads the
// library, from load until the process exits.  All calls on a device share
// it and it keeps the last call's contents, so calls that overlap on the GPU
// (different streams, or different host threads, without ordering between
// them) race on it and must be serialised by the caller.  Nothing in it has
// to start at zero: the only accumulator, the per-expert counter block, is
// cleared by the first kernel of every call.
#include <mutex>

#include "pmoe_common.cuh"

namespace {

// 8 MiB: the workspace of a decode batch of up to 64 tokens at the
// Qwen3.5-35B-A3B shape (6.1 MiB at T = 64).
constexpr size_t kNoallocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// The array's name in host code is only a host-side handle for the symbol;
// the device address has to be looked up, once per device, with that device
// current.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PMOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    // The library holds sm_100a code only: on another device the symbol has no
    // device copy, so report the device, not the failed lookup.
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return PMOE_ERR_CUDA;
    if (major != 10) return PMOE_ERR_DEVICE;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();  // do not leave the failure for a later error check
      return PMOE_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PMOE_OK;
}

}  // namespace

extern "C" {

size_t pmoe_noalloc_scratch_bytes(void) { return kNoallocScratchBytes; }

int pmoe_block_forward_noalloc(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                               const uint16_t* w_router, const uint16_t* w_gate_up,
                               const uint16_t* w_down, const uint16_t* w_sh_gate,
                               const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                               const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                               int flags, uint16_t* y, void* stream) {
  size_t need = 0;
  int s = pmoe_workspace_size(T, H, E, K, I, Is, &need);
  if (s != PMOE_OK) return s;
  if (need > kNoallocScratchBytes) return PMOE_ERR_NOALLOC_TOO_LARGE;
  if (T == 0) return pmoe_block_forward(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down,
                                        w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec, expert_lo,
                                        expert_hi, flags, y, nullptr, 0, stream);
  void* scratch = nullptr;
  if ((s = scratch_address(&scratch)) != PMOE_OK) return s;
  return pmoe_block_forward(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate,
                            w_sh_up, w_sh_down, w_sh_gvec, expert_lo, expert_hi, flags, y,
                            scratch, kNoallocScratchBytes, stream);
}

}  // extern "C"
