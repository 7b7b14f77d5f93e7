// Expert-parallel communicator: the `comm_handle` of the paris_moe::moe_block
// operator.  It holds the peer pointers of the two NVLink exchanges (the
// decode-sized buffers of pmoe_block_forward_ep and the row-split buffers of
// pmoe_block_forward_rows_fused) and the host epoch of the row exchange, and
// picks the path by batch size the same way on every rank.  It owns no
// memory: the buffers are allocated, IPC-mapped and freed by the caller (the
// Python EPGroup), which re-registers them here when it grows them.
//
// Replaces the process-group handle of the reference's ep_forward
// (engine/runtime/ep.py:97-143: expert_range at :78-86, all_reduce at :140).
#include <cstdint>
#include <mutex>
#include <new>
#include <vector>

#include "paris_moe.h"
#include "pmoe_common.cuh"

using pmoe::kMaxRanks;

namespace {

constexpr uint32_t kCommMagic = 0x504d4f43u;  // "PMOC"

struct Comm {
  uint32_t magic = kCommMagic;
  int rank = 0, world = 1;
  std::vector<void*> ep_bufs;  // decode exchange, empty when not registered
  size_t ep_bytes = 0;
  int ep_tmax = 0;
  std::vector<void*> rows_bufs;  // row-split exchange
  int rows_tmax = 0;
  int rows_epoch = 0;  // last epoch used on the row buffers (they start zeroed)
  std::mutex mu;
};

Comm* as_comm(void* p) {
  Comm* c = static_cast<Comm*>(p);
  return (c && c->magic == kCommMagic) ? c : nullptr;
}

bool valid_bufs(void* const* bufs, int world) {
  if (!bufs) return false;
  for (int q = 0; q < world; ++q)
    if (!bufs[q] || (reinterpret_cast<uintptr_t>(bufs[q]) & 15u) != 0) return false;
  return true;
}

}  // namespace

extern "C" {

int pmoe_comm_create(int rank, int world, void** comm) {
  if (!comm || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return PMOE_ERR_ARG;
  Comm* c = new (std::nothrow) Comm;
  if (!c) return PMOE_ERR_ARG;
  c->rank = rank;
  c->world = world;
  *comm = c;
  return PMOE_OK;
}

int pmoe_comm_destroy(void* comm) {
  Comm* c = as_comm(comm);
  if (!c) return PMOE_ERR_ARG;
  c->magic = 0;
  delete c;
  return PMOE_OK;
}

int pmoe_comm_set_ep(void* comm, void* const* bufs, size_t buf_bytes, int t_max) {
  Comm* c = as_comm(comm);
  if (!c || t_max < 0) return PMOE_ERR_ARG;
  std::lock_guard<std::mutex> g(c->mu);
  if (!bufs) {
    c->ep_bufs.clear();
    c->ep_bytes = 0;
    c->ep_tmax = 0;
    return PMOE_OK;
  }
  if (!valid_bufs(bufs, c->world)) return PMOE_ERR_ARG;
  c->ep_bufs.assign(bufs, bufs + c->world);
  c->ep_bytes = buf_bytes;
  c->ep_tmax = t_max;
  return PMOE_OK;
}

int pmoe_comm_set_rows(void* comm, void* const* bufs, int t_max) {
  Comm* c = as_comm(comm);
  if (!c || t_max < 0) return PMOE_ERR_ARG;
  std::lock_guard<std::mutex> g(c->mu);
  c->rows_epoch = 0;  // fresh buffers are zeroed
  if (!bufs) {
    c->rows_bufs.clear();
    c->rows_tmax = 0;
    return PMOE_OK;
  }
  if (!valid_bufs(bufs, c->world)) return PMOE_ERR_ARG;
  c->rows_bufs.assign(bufs, bufs + c->world);
  c->rows_tmax = t_max;
  return PMOE_OK;
}

int pmoe_comm_next_rows_epoch(void* comm, int* epoch) {
  Comm* c = as_comm(comm);
  if (!c || !epoch) return PMOE_ERR_ARG;
  std::lock_guard<std::mutex> g(c->mu);
  *epoch = ++c->rows_epoch;
  return PMOE_OK;
}

int pmoe_comm_info(void* comm, int* rank, int* world, int* ep_tmax, int* rows_tmax) {
  Comm* c = as_comm(comm);
  if (!c) return PMOE_ERR_ARG;
  std::lock_guard<std::mutex> g(c->mu);
  if (rank) *rank = c->rank;
  if (world) *world = c->world;
  if (ep_tmax) *ep_tmax = c->ep_bufs.empty() ? 0 : c->ep_tmax;
  if (rows_tmax) *rows_tmax = c->rows_bufs.empty() ? 0 : c->rows_tmax;
  return PMOE_OK;
}

int pmoe_block_forward_comm(void* comm, const uint16_t* x, int T, int H, int E, int K, int I,
                            int Is, const uint16_t* w_router, const uint16_t* w_gate_up,
                            const uint16_t* w_down, const uint16_t* w_sh_gate,
                            const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                            const uint16_t* w_sh_gvec, int flags, uint16_t* y, void* workspace,
                            size_t workspace_bytes, void* stream, void* const* events,
                            int n_events) {
  if (!comm)
    return pmoe_block_forward(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate,
                              w_sh_up, w_sh_down, w_sh_gvec, 0, E, flags, y, workspace,
                              workspace_bytes, stream);
  Comm* c = as_comm(comm);
  if (!c) return PMOE_ERR_ARG;
  if (c->world == 1)
    return pmoe_block_forward(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate,
                              w_sh_up, w_sh_down, w_sh_gvec, 0, E, flags, y, workspace,
                              workspace_bytes, stream);
  // ranges of engine/runtime/ep.py:78-86 (contiguous experts) and the shared
  // expert's tokens split the same way
  const int r = c->rank, n = c->world;
  const int elo = int(int64_t(r) * E / n), ehi = int(int64_t(r + 1) * E / n);
  const int slo = int(int64_t(r) * T / n), shi = int(int64_t(r + 1) * T / n);
  std::unique_lock<std::mutex> g(c->mu);
  if (!c->ep_bufs.empty() && T <= c->ep_tmax) {
    // epoch 0: the device-side counter of the buffer, so a captured CUDA
    // graph of this call replays correctly
    std::vector<void*> bufs = c->ep_bufs;
    const size_t nb = c->ep_bytes;
    g.unlock();
    return pmoe_block_forward_ep(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down, w_sh_gate,
                                 w_sh_up, w_sh_down, w_sh_gvec, elo, ehi, slo, shi, flags,
                                 bufs.data(), nb, r, n, 0, y, workspace, workspace_bytes, stream);
  }
  if (!c->rows_bufs.empty() && T <= c->rows_tmax &&
      (flags & (PMOE_F_SHARED | PMOE_F_ROUTED)) == (PMOE_F_SHARED | PMOE_F_ROUTED)) {
    std::vector<void*> bufs = c->rows_bufs;
    const int tmax = c->rows_tmax;
    const int epoch = ++c->rows_epoch;
    g.unlock();
    return pmoe_block_forward_rows_fused(x, T, H, E, K, I, Is, w_router, w_gate_up, w_down,
                                         w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec, r, n,
                                         bufs.data(), tmax, epoch, flags, y, workspace,
                                         workspace_bytes, stream, events, n_events);
  }
  return PMOE_ERR_COMM_CAPACITY;
}

}  // extern "C"
