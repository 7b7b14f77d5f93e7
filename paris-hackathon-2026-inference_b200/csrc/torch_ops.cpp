// torch.ops.paris_moe.*: the PyTorch operators over the C ABI of paris_moe.h.
//
// The drop-in surface for the reference's patched MoE forward
// (engine/kernels/moe_grouped_mlp.py:166-186, installed by
// engine/kernels/patch.py:43-84): moe_block takes the HF module's own bf16
// tensors, allocates its output and workspace with PyTorch's caching
// allocator, launches on the current CUDA stream and never synchronises the
// host, so it can be captured in a CUDA graph at the engine's decode buckets
// (engine/runtime/cuda_graphs.py:142).  A non-zero status from the library
// becomes a c10::Error (RuntimeError in Python) carrying the status code and
// its name; the CPU kernels only raise (no CPU fallback).  Meta
// kernels give the output shapes for tracing.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <tuple>

#include "paris_moe.h"

namespace {

using at::Tensor;

#define PMOE_CALL(fn, ...)                                                             \
  do {                                                                                 \
    const int st_ = fn(__VA_ARGS__);                                                   \
    TORCH_CHECK(st_ == PMOE_OK, #fn " failed: status ", st_, " (",                      \
                pmoe_status_string(st_), ")");                                         \
  } while (0)

const uint16_t* bf(const Tensor& t) {
  return reinterpret_cast<const uint16_t*>(t.data_ptr());
}
uint16_t* bf_mut(Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); }

void check_bf16(const char* op, const char* name, const Tensor& t, const Tensor& x, int dim) {
  TORCH_CHECK(t.is_cuda(), "paris_moe.", op, ": ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == x.device(), "paris_moe.", op, ": ", name, " is on ", t.device(),
              ", x on ", x.device());
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "paris_moe.", op, ": ", name,
              " must be bf16, got ", t.scalar_type());
  TORCH_CHECK(t.is_contiguous(), "paris_moe.", op, ": ", name, " must be contiguous");
  TORCH_CHECK(t.dim() == dim, "paris_moe.", op, ": ", name, " must have ", dim,
              " dimensions, got ", t.dim());
}

struct Shapes {
  int T, H, E, I, Is;
};

// The HF module's layouts (modeling_qwen3_5_moe.py:713-792): gate.weight
// [E,H], experts.gate_up_proj [E,2I,H], experts.down_proj [E,H,I],
// shared_expert.{gate,up}_proj.weight [Is,H], down_proj.weight [H,Is],
// shared_expert_gate.weight [1,H].
Shapes check_block(const char* op, const Tensor& x, const Tensor& w_router,
                   const Tensor& w_gate_up, const Tensor& w_down, const Tensor& w_sh_gate,
                   const Tensor& w_sh_up, const Tensor& w_sh_down, const Tensor& w_sh_gvec) {
  check_bf16(op, "x", x, x, 2);
  check_bf16(op, "w_router", w_router, x, 2);
  check_bf16(op, "w_gate_up", w_gate_up, x, 3);
  check_bf16(op, "w_down", w_down, x, 3);
  check_bf16(op, "w_sh_gate", w_sh_gate, x, 2);
  check_bf16(op, "w_sh_up", w_sh_up, x, 2);
  check_bf16(op, "w_sh_down", w_sh_down, x, 2);
  check_bf16(op, "w_sh_gvec", w_sh_gvec, x, 2);
  Shapes s{int(x.size(0)), int(x.size(1)), int(w_router.size(0)), int(w_gate_up.size(1) / 2),
           int(w_sh_gate.size(0))};
  TORCH_CHECK(w_router.size(1) == s.H && w_gate_up.size(0) == s.E &&
                  w_gate_up.size(1) == 2 * s.I && w_gate_up.size(2) == s.H &&
                  w_down.size(0) == s.E && w_down.size(1) == s.H && w_down.size(2) == s.I &&
                  w_sh_up.size(0) == s.Is && w_sh_gate.size(1) == s.H &&
                  w_sh_up.size(1) == s.H && w_sh_down.size(0) == s.H &&
                  w_sh_down.size(1) == s.Is && w_sh_gvec.numel() == s.H,
              "paris_moe.", op, ": weight shapes do not match x [", s.T, ",", s.H,
              "] (E=", s.E, ", I=", s.I, ", Is=", s.Is, ")");
  return s;
}

void* stream_of(const Tensor& x) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(x.device().index()).stream());
}

Tensor workspace(const Tensor& x, int T, int H, int E, int K, int I, int Is) {
  size_t nbytes = 0;
  PMOE_CALL(pmoe_workspace_size, T, H, E, K, I, Is, &nbytes);
  return at::empty({int64_t(nbytes)}, x.options().dtype(at::kByte));
}

// y[T,H] of the block.
//   top_k, flags             as pmoe_block_forward (flags: bit 0 shared expert,
//                            bit 1 routed experts)
//   expert_lo/hi             routed experts computed (hi < 0: E); ep_size 1 only
//   comm_handle != 0         a pmoe_comm_create handle: the full output on every
//                            rank via the NVLink exchanges (pmoe_block_forward_comm);
//                            ep_rank / ep_size must match the communicator
//   comm_handle 0, ep_size>1 this rank's partial: experts
//                            [ep_rank*E/ep_size, (ep_rank+1)*E/ep_size) and the
//                            shared expert of its token slice, for the caller to
//                            sum over ranks (the all_reduce of ep.py:140)
Tensor moe_block_cuda(const Tensor& x, const Tensor& w_router, const Tensor& w_gate_up,
                      const Tensor& w_down, const Tensor& w_sh_gate, const Tensor& w_sh_up,
                      const Tensor& w_sh_down, const Tensor& w_sh_gvec, int64_t top_k,
                      int64_t expert_lo, int64_t expert_hi, int64_t flags, int64_t ep_rank,
                      int64_t ep_size, int64_t comm_handle) {
  const Shapes s = check_block("moe_block", x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                               w_sh_down, w_sh_gvec);
  TORCH_CHECK(ep_size >= 1 && ep_rank >= 0 && ep_rank < ep_size,
              "paris_moe.moe_block: bad ep_rank ", ep_rank, " / ep_size ", ep_size);
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty({s.T, s.H}, x.options());
  if (s.T == 0) return y;
  const int K = int(top_k);
  Tensor ws = workspace(x, s.T, s.H, s.E, K, s.I, s.Is);
  void* st = stream_of(x);
  if (comm_handle != 0) {
    void* comm = reinterpret_cast<void*>(comm_handle);
    int rank = -1, world = 0;
    PMOE_CALL(pmoe_comm_info, comm, &rank, &world, nullptr, nullptr);
    TORCH_CHECK(rank == ep_rank && world == ep_size, "paris_moe.moe_block: ep_rank/ep_size ",
                ep_rank, "/", ep_size, " differ from the communicator's ", rank, "/", world);
    TORCH_CHECK(expert_lo == 0 && (expert_hi < 0 || expert_hi == s.E),
                "paris_moe.moe_block: an expert range cannot be combined with comm_handle");
    PMOE_CALL(pmoe_block_forward_comm, comm, bf(x), s.T, s.H, s.E, K, s.I, s.Is, bf(w_router),
              bf(w_gate_up), bf(w_down), bf(w_sh_gate), bf(w_sh_up), bf(w_sh_down),
              bf(w_sh_gvec), int(flags), bf_mut(y), ws.data_ptr(), size_t(ws.numel()), st,
              nullptr, 0);
    return y;
  }
  if (ep_size > 1) {
    TORCH_CHECK(expert_lo == 0 && (expert_hi < 0 || expert_hi == s.E),
                "paris_moe.moe_block: an expert range cannot be combined with ep_size > 1");
    const int r = int(ep_rank), n = int(ep_size);
    PMOE_CALL(pmoe_block_forward_ep, bf(x), s.T, s.H, s.E, K, s.I, s.Is, bf(w_router),
              bf(w_gate_up), bf(w_down), bf(w_sh_gate), bf(w_sh_up), bf(w_sh_down),
              bf(w_sh_gvec), int(int64_t(r) * s.E / n), int(int64_t(r + 1) * s.E / n),
              int(int64_t(r) * s.T / n), int(int64_t(r + 1) * s.T / n), int(flags), nullptr, 0,
              r, n, 0, bf_mut(y), ws.data_ptr(), size_t(ws.numel()), st);
    return y;
  }
  const int hi = expert_hi < 0 ? s.E : int(expert_hi);
  PMOE_CALL(pmoe_block_forward, bf(x), s.T, s.H, s.E, K, s.I, s.Is, bf(w_router), bf(w_gate_up),
            bf(w_down), bf(w_sh_gate), bf(w_sh_up), bf(w_sh_down), bf(w_sh_gvec),
            int(expert_lo), hi, int(flags), bf_mut(y), ws.data_ptr(), size_t(ws.numel()), st);
  return y;
}

Tensor moe_block_meta(const Tensor& x, const Tensor&, const Tensor&, const Tensor&,
                      const Tensor&, const Tensor&, const Tensor&, const Tensor&, int64_t,
                      int64_t, int64_t, int64_t, int64_t, int64_t, int64_t) {
  return at::empty_like(x);
}

// One MoE-only decoder layer x + block(RMSNorm(x)) (pmoe_layer_forward), on one
// GPU.
Tensor moe_layer_cuda(const Tensor& x, const Tensor& w_norm, double eps, const Tensor& w_router,
                      const Tensor& w_gate_up, const Tensor& w_down, const Tensor& w_sh_gate,
                      const Tensor& w_sh_up, const Tensor& w_sh_down, const Tensor& w_sh_gvec,
                      int64_t top_k, int64_t flags) {
  const Shapes s = check_block("moe_layer", x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                               w_sh_down, w_sh_gvec);
  check_bf16("moe_layer", "w_norm", w_norm, x, 1);
  TORCH_CHECK(w_norm.size(0) == s.H, "paris_moe.moe_layer: w_norm must be [", s.H, "]");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty({s.T, s.H}, x.options());
  if (s.T == 0) return y;
  const int K = int(top_k);
  Tensor ws = workspace(x, s.T, s.H, s.E, K, s.I, s.Is);
  PMOE_CALL(pmoe_layer_forward, bf(x), s.T, s.H, s.E, K, s.I, s.Is, bf(w_norm), float(eps),
            bf(w_router), bf(w_gate_up), bf(w_down), bf(w_sh_gate), bf(w_sh_up), bf(w_sh_down),
            bf(w_sh_gvec), 0, s.E, 0, s.T, int(flags), nullptr, 0, 0, 1, 0, bf_mut(y),
            ws.data_ptr(), size_t(ws.numel()), stream_of(x));
  return y;
}

Tensor moe_layer_meta(const Tensor& x, const Tensor&, double, const Tensor&, const Tensor&,
                      const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                      int64_t, int64_t) {
  return at::empty_like(x);
}

// Qwen3_5MoeRMSNorm (modeling_qwen3_5_moe.py:795-812).
Tensor rmsnorm_cuda(const Tensor& x, const Tensor& w_norm, double eps) {
  check_bf16("rmsnorm", "x", x, x, 2);
  check_bf16("rmsnorm", "w_norm", w_norm, x, 1);
  TORCH_CHECK(w_norm.size(0) == x.size(1), "paris_moe.rmsnorm: w_norm must be [H]");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty_like(x);
  PMOE_CALL(pmoe_rmsnorm, bf(x), int(x.size(0)), int(x.size(1)), bf(w_norm), float(eps),
            bf_mut(y), stream_of(x));
  return y;
}

Tensor rmsnorm_meta(const Tensor& x, const Tensor&, double) { return at::empty_like(x); }

using RouteOut = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

// Router + top-k + CSR dispatch (pmoe_route): (topk_idx i32 [T,k], topk_w f32
// [T,k], offsets i32 [E+1], sorted_tok i32 [T*k], sorted_slot i32 [T*k],
// shared_gate f32 [T]).
RouteOut moe_route_cuda(const Tensor& x, const Tensor& w_router, const Tensor& w_sh_gvec,
                        int64_t k) {
  check_bf16("moe_route", "x", x, x, 2);
  check_bf16("moe_route", "w_router", w_router, x, 2);
  check_bf16("moe_route", "w_sh_gvec", w_sh_gvec, x, 2);
  const int T = int(x.size(0)), H = int(x.size(1)), E = int(w_router.size(0)), K = int(k);
  TORCH_CHECK(w_router.size(1) == H && w_sh_gvec.numel() == H,
              "paris_moe.moe_route: weight shapes do not match x");
  const c10::cuda::CUDAGuard guard(x.device());
  const auto i32 = x.options().dtype(at::kInt), f32 = x.options().dtype(at::kFloat);
  Tensor idx = at::empty({T, K}, i32), w = at::empty({T, K}, f32);
  Tensor offs = at::zeros({E + 1}, i32), stok = at::empty({int64_t(T) * K}, i32);
  Tensor sslot = at::empty({int64_t(T) * K}, i32), sg = at::empty({T}, f32);
  if (T == 0) return {idx, w, offs, stok, sslot, sg};
  Tensor ws = workspace(x, T, H, E, K, 64, 64);
  PMOE_CALL(pmoe_route, bf(x), T, H, E, K, bf(w_router), bf(w_sh_gvec), idx.data_ptr<int32_t>(),
            w.data_ptr<float>(), offs.data_ptr<int32_t>(), stok.data_ptr<int32_t>(),
            sslot.data_ptr<int32_t>(), sg.data_ptr<float>(), ws.data_ptr(), size_t(ws.numel()),
            stream_of(x));
  return {idx, w, offs, stok, sslot, sg};
}

RouteOut moe_route_meta(const Tensor& x, const Tensor& w_router, const Tensor&, int64_t k) {
  const int64_t T = x.size(0), E = w_router.size(0);
  const auto i32 = x.options().dtype(at::kInt), f32 = x.options().dtype(at::kFloat);
  return {at::empty({T, k}, i32),     at::empty({T, k}, f32),     at::empty({E + 1}, i32),
          at::empty({T * k}, i32), at::empty({T * k}, i32), at::empty({T}, f32)};
}

// CPU tensors: a clear error instead of a computation (there is no CPU path).
[[noreturn]] void no_cpu(const char* op) {
  TORCH_CHECK(false, "paris_moe.", op, ": tensors must be CUDA (no CPU fallback)");
}
Tensor moe_block_cpu(const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                     const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, int64_t,
                     int64_t, int64_t, int64_t, int64_t) {
  no_cpu("moe_block");
}
Tensor moe_layer_cpu(const Tensor&, const Tensor&, double, const Tensor&, const Tensor&,
                     const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                     int64_t, int64_t) {
  no_cpu("moe_layer");
}
Tensor rmsnorm_cpu(const Tensor&, const Tensor&, double) { no_cpu("rmsnorm"); }
RouteOut moe_route_cpu(const Tensor&, const Tensor&, const Tensor&, int64_t) {
  no_cpu("moe_route");
}

}  // namespace

TORCH_LIBRARY(paris_moe, m) {
  m.def(
      "moe_block(Tensor x, Tensor w_router, Tensor w_gate_up, Tensor w_down, Tensor w_sh_gate, "
      "Tensor w_sh_up, Tensor w_sh_down, Tensor w_sh_gvec, int top_k=8, int expert_lo=0, "
      "int expert_hi=-1, int flags=3, *, int ep_rank=0, int ep_size=1, int comm_handle=0) "
      "-> Tensor");
  m.def(
      "moe_layer(Tensor x, Tensor w_norm, float eps, Tensor w_router, Tensor w_gate_up, "
      "Tensor w_down, Tensor w_sh_gate, Tensor w_sh_up, Tensor w_sh_down, Tensor w_sh_gvec, "
      "int top_k=8, int flags=3) -> Tensor");
  m.def("rmsnorm(Tensor x, Tensor w_norm, float eps) -> Tensor");
  m.def(
      "moe_route(Tensor x, Tensor w_router, Tensor w_sh_gvec, int k) -> "
      "(Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(paris_moe, CUDA, m) {
  m.impl("moe_block", &moe_block_cuda);
  m.impl("moe_layer", &moe_layer_cuda);
  m.impl("rmsnorm", &rmsnorm_cuda);
  m.impl("moe_route", &moe_route_cuda);
}

TORCH_LIBRARY_IMPL(paris_moe, CPU, m) {
  m.impl("moe_block", &moe_block_cpu);
  m.impl("moe_layer", &moe_layer_cpu);
  m.impl("rmsnorm", &rmsnorm_cpu);
  m.impl("moe_route", &moe_route_cpu);
}

TORCH_LIBRARY_IMPL(paris_moe, Meta, m) {
  m.impl("moe_block", &moe_block_meta);
  m.impl("moe_layer", &moe_layer_meta);
  m.impl("rmsnorm", &rmsnorm_meta);
  m.impl("moe_route", &moe_route_meta);
}
