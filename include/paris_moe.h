/*
 * paris_moe.h -- C ABI of the B200 (sm_100a) Qwen3.5-35B-A3B sparse-MoE block.
 *
 * Plain pointers and sizes only: bf16 tensors are `uint16_t` bit patterns in
 * device memory, row-major; streams are `cudaStream_t` passed as `void*`.
 * Every entry point is asynchronous on the given stream, never synchronises
 * the host, allocates nothing, and returns a status (`PMOE_OK` = 0, negative
 * on error; see `pmoe_status_string`).
 *
 * Shapes (Qwen3.5-35B-A3B: H=2048, E=256, K=8, I=512, Is=512):
 *   x          [T, H]       hidden states
 *   w_router   [E, H]       gate.weight
 *   w_gate_up  [E, 2I, H]   experts.gate_up_proj (rows [0,I) gate, [I,2I) up)
 *   w_down     [E, H, I]    experts.down_proj
 *   w_sh_gate  [Is, H]      shared_expert.gate_proj.weight
 *   w_sh_up    [Is, H]      shared_expert.up_proj.weight
 *   w_sh_down  [H, Is]      shared_expert.down_proj.weight
 *   w_sh_gvec  [1, H]       shared_expert_gate.weight
 * These are the HF module's own tensors (transformers
 * models/qwen3_5_moe/modeling_qwen3_5_moe.py:713-792), used in place.
 */
#ifndef PARIS_MOE_H_
#define PARIS_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  PMOE_OK = 0,
  PMOE_ERR_ARG = -1,        /* bad shape, pointer or flag */
  PMOE_ERR_ALIGN = -2,      /* a tensor is not 16-byte aligned */
  PMOE_ERR_WORKSPACE = -3,  /* workspace too small */
  PMOE_ERR_CUDA = -4,       /* a CUDA runtime call failed (launch, copy) */
  PMOE_ERR_UNSUPPORTED = -5,/* shape outside what the kernels implement */
  PMOE_ERR_PEER_TIMEOUT = -6,/* a bounded wait on a peer GPU ran out */
  PMOE_ERR_DEVICE = -7,     /* not an sm_100 device */
  PMOE_ERR_NOALLOC_TOO_LARGE = -8, /* shape needs more scratch than the no-alloc entry has */
  PMOE_ERR_COMM_CAPACITY = -9 /* batch larger than the communicator's exchange buffers */
};

/* Flags of pmoe_block_forward. */
enum {
  PMOE_F_SHARED = 1,        /* add sigmoid(x.w_sh_gvec) * shared_expert(x) */
  PMOE_F_ROUTED = 2,        /* add the routed experts in [expert_lo, expert_hi) */
  PMOE_F_FORCE_STREAM = 4,  /* weight-streaming kernels at any T (testing) */
  PMOE_F_FORCE_TC = 8,      /* tcgen05 grouped GEMMs at any T (testing) */
  PMOE_F_ROUTE_SLICE = 16   /* pmoe_block_forward_rows_fused only: each rank routes its
                               token slice [r*T/N, (r+1)*T/N) and the routing slices are
                               exchanged over NVLink (peer stores) instead of every rank
                               routing all T tokens; same output bits */
};

/* Human-readable name of a status code. */
const char* pmoe_status_string(int status);

/* Library version string ("paris_moe <semver> sm_100a"). */
const char* pmoe_version(void);

/* Bytes of device workspace pmoe_route / pmoe_block_forward need for this
 * shape.  The workspace holds the router partials, routing, CSR dispatch,
 * the SiLU*up intermediate and the weighted expert rows.  Replaces the
 * per-call temporaries of engine/kernels/moe_grouped_mlp.py:115-163 and
 * engine/kernels/moe_dispatch.py:119-137. */
int pmoe_workspace_size(int T, int H, int E, int K, int I, int Is, size_t* bytes);

/* Router + top-k + dispatch only.
 * Replaces Qwen3_5MoeTopKRouter.forward (modeling_qwen3_5_moe.py:762-770)
 * followed by moe_dispatch_indices (engine/kernels/moe_dispatch.py:178-209).
 * The bf16 logit of (token, expert) is the bf16 value nearest (ties to even)
 * to the exact dot product of the bf16 operands; the selection is exact on
 * those values (approximate tensor-core logits with a stated error bound,
 * exact re-evaluation of the experts whose rounding the bound leaves open):
 *   topk_idx    [T, K] int32  experts by descending bf16 logit, ties -> lower index
 *   topk_w      [T, K] fp32   renormalised softmax weights
 *   offsets     [E+1]  int32  CSR offsets of the (token, slot) pairs by expert
 *   sorted_tok  [T*K]  int32  token of each pair, stable by pair index
 *   sorted_slot [T*K]  int32  slot of each pair
 *   shared_gate [T]    fp32   sigmoid(x . w_sh_gvec)
 * Any output pointer may be NULL (not copied out). */
int pmoe_route(const uint16_t* x, int T, int H, int E, int K,
               const uint16_t* w_router, const uint16_t* w_sh_gvec,
               int32_t* topk_idx, float* topk_w, int32_t* offsets,
               int32_t* sorted_tok, int32_t* sorted_slot, float* shared_gate,
               void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostics of the exact top-k (testing): runs the routing of pmoe_route
 * and returns, besides topk_idx / topk_w, the router GEMM's fp32
 * approximate logits logits[T][Rpad] (Rpad = E + 1 rounded up to 16; column
 * E is the shared-expert gate sum), the bound factor *gamma of that path (the
 * top-k treats |approx - exact| <= gamma * ||x_t|| * ||w_e|| as given) and
 * stats[0] = experts evaluated exactly, stats[1] = of which outside the
 * exactness condition of the double-double sum (expected 0).  stats is host
 * memory; the call synchronises the stream.  No counterpart in the reference
 * (test infrastructure for the exact selection). */
int pmoe_route_diag(const uint16_t* x, int T, int H, int E, int K, const uint16_t* w_router,
                    const uint16_t* w_sh_gvec, int32_t* topk_idx, float* topk_w, float* logits,
                    float* gamma, int32_t* stats, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Exactly rounded router logits of all T x E (token, expert) pairs: logits[t*E + e]
 * = the bf16 value (as fp32) nearest, ties to even, to the exact dot product
 * of x[t] and w_router[e] (H % 256 == 0), by integer arithmetic on the
 * GPU, one warp per pair.  *n_inexact (device int, incremented) counts pairs
 * whose operands' exponent spread exceeds the exact window (expected 0).
 * The top-k of pmoe_route evaluates only the few logits its error bound
 * leaves open; this computes them all (tests, diagnostics).  No counterpart
 * in the reference. */
int pmoe_exact_logits(const uint16_t* x, int T, int H, int E, const uint16_t* w_router,
                      float* logits, int32_t* n_inexact, void* stream);

/* The whole MoE block, y[T,H] (bf16) =
 *     sum_k w_tk * down_e(SiLU(gate_e x) * up_e x)          (PMOE_F_ROUTED, e in [lo,hi))
 *   + sigmoid(x . w_sh_gvec) * shared_expert(x)             (PMOE_F_SHARED)
 * Replaces Qwen3_5MoeSparseMoeBlock.forward (modeling_qwen3_5_moe.py:781-792)
 * and its patched twin fused_moe_forward (engine/kernels/moe_grouped_mlp.py:166-186).
 * With expert_lo/hi a strict sub-range it is one rank's routed partial of
 * ep_forward (engine/runtime/ep.py:97-143) before the all-reduce.
 * The combine accumulates in fp32 in a fixed order (deterministic). */
int pmoe_block_forward(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                       const uint16_t* w_router, const uint16_t* w_gate_up,
                       const uint16_t* w_down, const uint16_t* w_sh_gate,
                       const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                       const uint16_t* w_sh_gvec, int expert_lo, int expert_hi, int flags,
                       uint16_t* y, void* workspace, size_t workspace_bytes, void* stream);

/* pmoe_block_forward that also records CUDA events on `stream` between its
 * phases, for per-kernel timing by a benchmark: events[0] before routing,
 * [1] after routing (router, top-k, dispatch; on the tensor-core path also
 * the tile plan and the row copy, i.e. right before the gate_up GEMM), [2]
 * after gate_up+SiLU*mul, [3] after down, [4] after the combine.  NULL
 * entries and n_events < 5 skip the corresponding records.  No reference
 * counterpart (instrumentation of pmoe_block_forward). */
int pmoe_block_forward_profiled(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                                const uint16_t* w_router, const uint16_t* w_gate_up,
                                const uint16_t* w_down, const uint16_t* w_sh_gate,
                                const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                                const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                                int flags, uint16_t* y, void* workspace, size_t workspace_bytes,
                                void* stream, void* const* events, int n_events);

/* ---- expert parallelism over NVLink ------------------------------------------
 * One process per GPU; every rank calls with the same x (replicated tokens)
 * and the same weights, as ep_forward does (engine/runtime/ep.py:97-143).
 *
 * Size of each rank's exchange buffer for batches of up to T_max tokens:
 * flags + two parity copies of the weighted expert rows. */
int pmoe_ep_buffer_bytes(int T_max, int H, int K, size_t* bytes);

/* The block on one rank of an expert-parallel group.
 *   expert_lo/hi      routed experts this rank computes (engine/runtime/ep.py:78-86
 *                     contiguous ranges, replacing its per-expert loop :124-136)
 *   shared_lo/hi      tokens whose shared-expert rows this rank computes
 *   peer_bufs         NULL: y is this rank's partial (routed range + shared token
 *                     range), to be summed across ranks by the caller (the NCCL
 *                     all_reduce of ep.py:140).  Otherwise `world` pointers to
 *                     every rank's exchange buffer (IPC-mapped, this rank's own at
 *                     [rank]): each computed row is stored straight into every
 *                     rank's buffer over NVLink from the down-projection epilogue,
 *                     completion flags are raised with release stores, and the
 *                     combine waits (bounded; PMOE status kStatusTimeoutPeer via
 *                     pmoe_read_status) and sums -- y is the full block output on
 *                     every rank, no separate collective.  Streaming path only
 *                     (T <= 64 unless PMOE_F_FORCE_STREAM).
 *   epoch             > 0: increasing by one per call on every rank (host
 *                     counter); 0: a counter in this rank's exchange buffer that
 *                     every call bumps on the device, so a captured CUDA graph
 *                     replays correctly.  One group uses one of the two modes. */
int pmoe_block_forward_ep(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                          const uint16_t* w_router, const uint16_t* w_gate_up,
                          const uint16_t* w_down, const uint16_t* w_sh_gate,
                          const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                          const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                          int shared_lo, int shared_hi, int flags, void* const* peer_bufs,
                          size_t peer_buf_bytes, int rank, int world, int epoch, uint16_t* y,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Row-split expert parallelism for prefill-sized batches (the tensor-core
 * path), in two steps per rank:
 *  1. pmoe_route_slice routes tokens [t0, t1) (router GEMM, softmax, top-k,
 *     renormalisation, shared-expert gate) into rows t0.. of the caller's
 *     full-size arrays topk_idx [T][K] i32, topk_w [T][K] f32,
 *     shared_gate [T] f32; each rank routes its own slice and the caller
 *     all-gathers the arrays (a few hundred KiB).
 *  2. pmoe_block_forward_rows takes the complete routing, dispatches all
 *     T*K + T rows exactly as a single GPU would, and computes only this
 *     rank's share: the 256-row blocks of the experts (shared expert
 *     included) whose middle row falls in [rank*R/world, (rank+1)*R/world) of
 *     the R dispatched rows -- one contiguous range, so heavy experts are
 *     split across ranks instead of loading one rank.  y is this rank's
 *     partial, to be summed across ranks by the caller (as ep.py:140 sums the
 *     expert-range partials of engine/runtime/ep.py:97-143).  expert_lo/hi
 *     restrict the routed experts computed and summed (0, E: all); with
 *     world = 1 and an expert range this is the expert side of a
 *     token-dispatch (all-to-all) exchange.  topk_idx, topk_w and shared_gate
 *     all NULL: the call routes all T tokens itself (identically on every
 *     rank) instead of taking the routing.
 * Workspace as pmoe_workspace_size(T, ...). */
int pmoe_route_slice(const uint16_t* x, int T, int H, int E, int K, int I, int Is, int t0,
                     int t1, const uint16_t* w_router, const uint16_t* w_sh_gvec,
                     int32_t* topk_idx, float* topk_w, float* shared_gate, void* workspace,
                     size_t workspace_bytes, void* stream);
int pmoe_block_forward_rows(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                            const uint16_t* w_router, const uint16_t* w_gate_up,
                            const uint16_t* w_down, const uint16_t* w_sh_gate,
                            const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                            const uint16_t* w_sh_gvec, const int32_t* topk_idx,
                            const float* topk_w, const float* shared_gate, int expert_lo,
                            int expert_hi, int rank, int world, int flags, uint16_t* y,
                            void* workspace, size_t workspace_bytes, void* stream);
/* pmoe_block_forward_rows with the phase events of
 * pmoe_block_forward_profiled (events[0..4], same meaning and NULL rule). */
int pmoe_block_forward_rows_profiled(
    const uint16_t* x, int T, int H, int E, int K, int I, int Is, const uint16_t* w_router,
    const uint16_t* w_gate_up, const uint16_t* w_down, const uint16_t* w_sh_gate,
    const uint16_t* w_sh_up, const uint16_t* w_sh_down, const uint16_t* w_sh_gvec,
    const int32_t* topk_idx, const float* topk_w, const float* shared_gate, int expert_lo,
    int expert_hi, int rank, int world, int flags, uint16_t* y, void* workspace,
    size_t workspace_bytes, void* stream, void* const* events, int n_events);

/* Sum of the row-split partials over NVLink, in place of the caller's NCCL
 * all_reduce (ep.py:140): each rank owns a buffer of pmoe_rows_buffer_bytes
 * (pmoe_ipc_alloc'ed, zeroed, IPC-mapped on every rank; bufs[q] = rank q's
 * buffer as mapped here).  Per call with epoch e (> 0, +1 per call, same on
 * every rank): write this rank's partial [T][H] bf16 into the region that
 * pmoe_rows_partial(own buffer, T_max, H, e) returns (e.g. as the y of
 * pmoe_block_forward_rows), then pmoe_rows_allreduce: every rank's flags say
 * its partial is complete; rank r sums token slice [r*T/N, (r+1)*T/N) over
 * ranks 0..N-1 in that order in fp32 (deterministic), raises a second set of
 * flags, and y = the reduced slices of all ranks.  Waits are bounded
 * (status 4 via pmoe_rows_status on timeout).  No collective kernel. */
int pmoe_rows_buffer_bytes(int T_max, int H, size_t* bytes);
int pmoe_rows_partial(void* own_buf, int T_max, int H, int epoch, void** partial);
int pmoe_rows_allreduce(void* const* bufs, int T_max, int T, int H, int rank, int world,
                        int epoch, uint16_t* y, void* stream);
int pmoe_rows_status(const void* own_buf, int* status);

/* Asynchronous reads of the sticky status words of the exchange buffers, for
 * an engine that checks a peer loss at its next call instead of blocking: the
 * word (0 ok, 4 a wait on a peer gave up in some earlier call; only a fresh,
 * zeroed buffer clears it) is copied to dst (pinned host or device memory) in
 * stream order.  own_buf: this rank's buffer of pmoe_block_forward_ep /
 * pmoe_layer_forward (pmoe_ep_status_async) or of the row exchanges
 * (pmoe_rows_status_async).  Replace nothing in the reference, whose
 * ep_forward (engine/runtime/ep.py:120-143) relies on NCCL's own error path. */
int pmoe_ep_status_async(const void* own_buf, int* dst, void* stream);
int pmoe_rows_status_async(const void* own_buf, int* dst, void* stream);

/* Row-split prefill with the exchange fused into the expert GEMMs, replacing
 * the pmoe_block_forward_rows + all_reduce pair of ep.py:97-143/140 for
 * prefill-sized batches.  Every rank routes all T tokens (identically) and
 * computes its row-balanced share of the dispatched rows, as in
 * pmoe_block_forward_rows; the down GEMM stores each unweighted output row
 * straight into the buffer of the rank that owns its token (token slice
 * [r*T/world, (r+1)*T/world)) with NVLink peer stores; each rank then combines
 * its slice locally, in the single-GPU order, storing the result into every
 * rank's buffer, and copies the completed output into y.  y is the full output on every rank, bit-identical to the
 * single-GPU pmoe_block_forward.  bufs[q]: rank q's buffer of
 * pmoe_rows_fused_buffer_bytes(T_max, H, K) (pmoe_ipc_alloc'ed, zeroed,
 * mapped on every rank); epoch > 0, +1 per call, the same on every rank.
 * flags must include PMOE_F_SHARED | PMOE_F_ROUTED; K <= 8, H <= 2048.
 * events: as pmoe_block_forward_profiled ([4] after the gather; may be NULL).
 * Waits are bounded (status 4 via pmoe_rows_status). */
int pmoe_rows_fused_buffer_bytes(int T_max, int H, int K, size_t* bytes);
/* (flags may add PMOE_F_ROUTE_SLICE: routing by token slice, the token-dispatch
 * form of the exchange -- the routing of engine/runtime/ep.py's replicated
 * tokens is split by token owner, and only the routing crosses NVLink, since
 * every rank holds the tokens themselves.) */
int pmoe_block_forward_rows_fused(
    const uint16_t* x, int T, int H, int E, int K, int I, int Is, const uint16_t* w_router,
    const uint16_t* w_gate_up, const uint16_t* w_down, const uint16_t* w_sh_gate,
    const uint16_t* w_sh_up, const uint16_t* w_sh_down, const uint16_t* w_sh_gvec, int rank,
    int world, void* const* bufs, int T_max, int epoch, int flags, uint16_t* y,
    void* workspace, size_t workspace_bytes, void* stream, void* const* events, int n_events);

/* ---- communicator: the comm_handle of the paris_moe::moe_block operator -----
 * An opaque handle holding one rank's view of the two NVLink exchanges above
 * (peer pointers of the pmoe_block_forward_ep buffers and of the
 * pmoe_block_forward_rows_fused buffers) plus the host epoch of the row
 * exchange.  It owns no device memory: the caller allocates, IPC-maps and
 * frees the buffers and registers them here (again after growing them; the
 * row epoch restarts, the new buffers being zeroed).  Not thread-safe across
 * ranks' host threads beyond its internal lock.  Replaces the process-group
 * handle that engine/runtime/ep.py:97-143 hands to all_reduce (:140). */
int pmoe_comm_create(int rank, int world, void** comm);
int pmoe_comm_destroy(void* comm);
/* bufs NULL: unregister.  t_max: the batch size the buffers were sized for. */
int pmoe_comm_set_ep(void* comm, void* const* bufs, size_t buf_bytes, int t_max);
int pmoe_comm_set_rows(void* comm, void* const* bufs, int t_max);
/* Take the next row-exchange epoch (for pmoe_rows_partial / pmoe_rows_allreduce
 * calls that share the row buffers with pmoe_block_forward_comm). */
int pmoe_comm_next_rows_epoch(void* comm, int* epoch);
/* rank, world, and the largest T each registered exchange takes (0: none). */
int pmoe_comm_info(void* comm, int* rank, int* world, int* ep_tmax, int* rows_tmax);
/* The full block output on every rank of the communicator (all ranks call with
 * the same x, T and weights, in the same order).  Rank r computes the experts
 * [r*E/world, (r+1)*E/world) (engine/runtime/ep.py:78-86) and the shared expert
 * of tokens [r*T/world, (r+1)*T/world).  T <= the decode exchange's t_max:
 * pmoe_block_forward_ep with the device-side epoch (CUDA-graph capturable);
 * else, with PMOE_F_SHARED|PMOE_F_ROUTED and T <= the row exchange's t_max:
 * pmoe_block_forward_rows_fused with the next host epoch (not capturable:
 * the epoch is baked into the launch); else PMOE_ERR_COMM_CAPACITY.
 * comm NULL or world 1: pmoe_block_forward over all experts.  events /
 * n_events: as pmoe_block_forward_rows_fused (may be NULL / 0). */
int pmoe_block_forward_comm(void* comm, const uint16_t* x, int T, int H, int E, int K, int I,
                            int Is, const uint16_t* w_router, const uint16_t* w_gate_up,
                            const uint16_t* w_down, const uint16_t* w_sh_gate,
                            const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                            const uint16_t* w_sh_gvec, int flags, uint16_t* y, void* workspace,
                            size_t workspace_bytes, void* stream, void* const* events,
                            int n_events);

/* One decoder layer of the MoE-only stack: y = x + block(RMSNorm(x)), with
 * RMSNorm(x) = bf16(x * rsqrt(mean(x^2) + eps) * (1 + w_norm)) in fp32 and the
 * residual added as bf16(x + bf16(block)) -- Qwen3_5MoeDecoderLayer's
 * post_attention_layernorm, mlp and residual add
 * (modeling_qwen3_5_moe.py:795-812, 862-868), attention omitted.  The norm is
 * one kernel ahead of the router; the residual is folded into the combine.
 * y may alias x (in-place update of the residual stream).  Other arguments as
 * pmoe_block_forward_ep (peer_bufs NULL: one GPU, or a partial for the caller
 * to sum -- then the residual is added on every rank, so only one rank should
 * pass x as residual: use pmoe_block_forward for the other partials). */
int pmoe_layer_forward(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                       const uint16_t* w_norm, float eps, const uint16_t* w_router,
                       const uint16_t* w_gate_up, const uint16_t* w_down,
                       const uint16_t* w_sh_gate, const uint16_t* w_sh_up,
                       const uint16_t* w_sh_down, const uint16_t* w_sh_gvec, int expert_lo,
                       int expert_hi, int shared_lo, int shared_hi, int flags,
                       void* const* peer_bufs, size_t peer_buf_bytes, int rank, int world,
                       int epoch, uint16_t* y, void* workspace, size_t workspace_bytes,
                       void* stream);

/* out[T][H] = Qwen3_5MoeRMSNorm(x; w_norm, eps) in fp32, cast to bf16
 * (modeling_qwen3_5_moe.py:795-812): the first step of pmoe_layer_forward,
 * exported for tests and for callers that normalise separately. */
int pmoe_rmsnorm(const uint16_t* x, int T, int H, const uint16_t* w_norm, float eps,
                 uint16_t* out, void* stream);

/* Synchronously read the kernel status word of the last call that used this
 * workspace (0 ok, 1/2/3 a bounded pipeline wait ran out, 4 a peer's flag never
 * arrived).  Diagnostic; synchronises the device.  No reference counterpart. */
int pmoe_read_status(const void* workspace, int T, int H, int E, int K, int I, int Is,
                     int* status);

/* Exchange-buffer plumbing (one-time set-up, not on the hot path):
 * allocate/zero a device buffer, export it as a 64-byte CUDA IPC handle, map a
 * peer's handle into this process, unmap it.  No reference counterpart (the
 * reference only uses NCCL collectives). */
int pmoe_ipc_alloc(size_t bytes, void** ptr);
int pmoe_ipc_free(void* ptr);
int pmoe_ipc_handle(void* ptr, void* handle);
int pmoe_ipc_open(const void* handle, void** ptr);
int pmoe_ipc_close(void* ptr);

/* pmoe_block_forward for callers that cannot allocate device memory: it takes
 * no workspace.  Meant for hosts such as a serving engine that reserves all
 * of HBM up front (KV cache, weights) and allows no allocation on its decode
 * path, or a program in another language calling through a bare FFI with no
 * device allocator of its own.  No counterpart in the reference (whose torch
 * code allocates its temporaries through PyTorch on every call).
 *
 * Scratch is one fixed array of pmoe_noalloc_scratch_bytes() (8 MiB) in
 * device memory, held by every GPU that loads the library until the process
 * exits.  Shapes whose workspace (pmoe_workspace_size) exceeds it -- at the
 * Qwen3.5 shape, more than 64 tokens -- return PMOE_ERR_NOALLOC_TOO_LARGE
 * without launching anything.  The first call on a device looks up the
 * array's device address (set-up, once per device); make that first call
 * before any stream capture.  All calls on a device share the array and it
 * keeps the previous call's contents, so calls that may overlap on the GPU
 * race and must be ordered by the caller.  Allocates nothing: no cudaMalloc,
 * no cudaFree, no allocating library routine.  Same arguments, results and
 * status codes as pmoe_block_forward otherwise. */
int pmoe_block_forward_noalloc(const uint16_t* x, int T, int H, int E, int K, int I, int Is,
                               const uint16_t* w_router, const uint16_t* w_gate_up,
                               const uint16_t* w_down, const uint16_t* w_sh_gate,
                               const uint16_t* w_sh_up, const uint16_t* w_sh_down,
                               const uint16_t* w_sh_gvec, int expert_lo, int expert_hi,
                               int flags, uint16_t* y, void* stream);

/* Size in bytes of the fixed scratch array of pmoe_block_forward_noalloc. */
size_t pmoe_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
#endif /* PARIS_MOE_H_ */
