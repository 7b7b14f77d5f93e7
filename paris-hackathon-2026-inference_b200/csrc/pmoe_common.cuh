// Shared device helpers for the B200 MoE-block kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/paris_moe.h"

namespace pmoe {

// ---- workspace layout --------------------------------------------------------
// One flat caller-provided buffer; every region 256-byte aligned.  The same
// function is used by the size query and by the launchers so they can never
// disagree.
struct Workspace {
  int32_t* counts;      // [E]        per-expert pair counts (zeroed by the router kernel)
  int32_t* offsets;     // [E+2]      CSR offsets; [E]..[E+1] is the shared expert's rows
  int32_t* active;      // [E+1]      experts this rank computes (hit, in range) + shared
  int32_t* n_active;    // [4]        [0] = entries in `active`
  int32_t* topk_idx;    // [T*K]
  float* topk_w;        // [T*K]
  float* shared_gate;   // [T]        sigmoid(x . w_sh_gvec)
  int32_t* sorted_tok;  // [T*K+T]    source token of each dispatched row
  int32_t* sorted_slot; // [T*K]
  int32_t* pair_dst;    // [T*K+T]    destination row in `rows` (t*K+s, or T*K+t)
  int32_t* pair_pos;    // [T*K+T]    inverse: dispatched row of destination row q (prefill path)
  float* pair_w;        // [T*K+T]    routing weight (or shared gate) of each row
  float* logit_part;    // [KS][T][Rpad] fp32 router logits (decode: KS split-K partials) + raw
                        //            shared-gate sum in column E
  float* xnorm;         // [KS][T]    token norms (decode: partial sums of squares per k range)
  float* wnorm;         // [TT][KS][Rpad] router-row norms (decode: partial sums of squares per
                        //            token group and k range; other paths: [E] norms)
  float* diag;          // not carved: when set, the routing copies its fp32 logits [T][Rpad] here
  int32_t* status;      // [kStatusWords] [0] route ticket, [1] error code (kStatus*), [2]/[3]
                        //            stream queues, [4..7] decode group tickets, [8] exact logit
                        //            evaluations, [9] of which outside the exactness condition,
                        //            [10] entries of route_queue; cleared per call
  __nv_bfloat16* h;     // [T*K+T][ldh] SiLU(gate)*up, dispatched order
  __nv_bfloat16* xn;    // [T][H]     RMSNorm(x) (decoder-layer entry points)
  float* rows;          // [T*K+T][H] weighted expert outputs, token-major (streaming path)
  __nv_bfloat16* x_perm; // [T*K+T][H] x rows in dispatch order (tensor-core path; aliases
                         //            `rows`, which only the streaming path uses)
  __nv_bfloat16* rows_bf16; // [T*K+T][H] expert outputs (unweighted), token-major (tensor-core
                            //  path, written by down after gate_up has consumed x_perm)
  int4* gu_tiles;       // tensor-core path tile lists: (expert, row0, nrows, n_block)
  int4* dn_tiles;
  int4* m_tiles;        // (expert, row0, nrows, 0): one per 128-row block of a computed expert
  int32_t* tile_counts; // [8] tiles: [0] gate_up [1] down [2] M blocks; [4]/[5] the dispatched
                        //     rows [lo, hi) this call computes (row-split expert parallelism)
  int32_t* route_queue; // [T]       tokens the prefill top-k's fast check left open
  int32_t* hist;        // [ceil(T/128)][E] per-tile expert histogram (prefill routing)
  int32_t* hist_base;   // [ceil(T/128)][E] first output slot per (tile, expert)
  size_t bytes;
};

constexpr int kStatusWords = 16;

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Dims {
  int T, H, E, K, I, Is;
  int Rpad;   // router rows (E experts + shared gate) padded to 16
  int KS;     // decode router split-K factor (CTAs per logit tile)
  int ldh;    // row stride of h
  int sh_lo, sh_hi;  // token range this call computes the shared expert for
};

// Expert-parallel exchange of the weighted expert rows over NVLink (decode).
// Every rank routes all tokens identically; rank r computes the experts in
// its range and writes each weighted row into EVERY rank's `rows` buffer
// (peer stores), then the last of its CTAs to finish raises flags[q][r] =
// epoch on every rank q.  The combine on rank q waits (bounded) for
// flags[q][0..world) >= epoch and sums locally: no separate collective.
// The epoch is either passed per call (host counter) or read from a counter
// in this rank's exchange buffer that a one-thread kernel bumps at the start
// of every call, so that a captured CUDA graph replays correctly.  Rows go to
// one of two copies by epoch parity (a rank one call ahead never overwrites
// rows still being combined).
constexpr int kMaxRanks = 8;
struct EpPeers {
  float* rows[kMaxRanks];  // each rank's rows buffer, parity-0 copy (peer-mapped)
  size_t par_stride;       // floats from the parity-0 to the parity-1 copy
  int* flags[kMaxRanks];   // each rank's flag array, indexed by the writing rank
  int* ticket;             // this rank's CTA-completion counter (starts and ends at 0)
  int* sticky;             // this rank's sticky status word: a peer timeout of any call
  const int* epoch_dev;    // device epoch counter, or null: use `epoch`
  int world;               // 0: no exchange
  int rank;
  int epoch;               // host epoch (> 0) when epoch_dev is null
};

// Destination of the down GEMM's unweighted rows in row-split prefill with a
// fused exchange: row q (token-major, q = t*K + k, shared row T*K + t) goes to
// base[owner(t)] + q*H, owner(t) = the rank r with r*T/world <= t < (r+1)*T/world
// (peer stores over NVLink).  world == 0: this rank's workspace rows.
struct RowsOut {
  __nv_bfloat16* base[kMaxRanks];
  int world;
};

// The rank whose token slice [r*T/world, (r+1)*T/world) holds token t.
__host__ __device__ __forceinline__ int slice_owner(int t, int T, int world) {
  int r = int(long(t) * world / T);
  while (r > 0 && long(r) * T / world > t) --r;
  while (r + 1 < world && long(r + 1) * T / world <= t) ++r;
  return r;
}

__device__ __forceinline__ int ep_epoch(const EpPeers& ep) {
  return ep.epoch_dev ? *ep.epoch_dev : ep.epoch;
}
__device__ __forceinline__ float* ep_rows(const EpPeers& ep, int r, int epoch) {
  return ep.rows[r] + size_t(epoch & 1) * ep.par_stride;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Token counts up to this use the single-launch routing kernel.
constexpr int kFusedRouteMaxT = 64;

inline Dims make_dims(int T, int H, int E, int K, int I, int Is) {
  Dims d{T, H, E, K, I, Is, 0, 0, 0, 0, T};
  d.Rpad = ((E + 1) + 15) / 16 * 16;
  d.KS = (T <= kFusedRouteMaxT && H % (4 * 32) == 0) ? 4 : 1;
  d.ldh = I > Is ? I : Is;
  return d;
}

inline Workspace carve(void* base, const Dims& d) {
  Workspace w{};
  size_t off = 0;
  char* b = static_cast<char*>(base);
  auto take = [&](size_t n) { char* p = b ? b + off : nullptr; off = align256(off + n); return p; };
  size_t P = size_t(d.T) * d.K, R = P + d.T;
  w.counts = (int32_t*)take(sizeof(int32_t) * d.E);
  w.offsets = (int32_t*)take(sizeof(int32_t) * (d.E + 2));
  w.active = (int32_t*)take(sizeof(int32_t) * (d.E + 1));
  w.n_active = (int32_t*)take(sizeof(int32_t) * 4);
  w.topk_idx = (int32_t*)take(sizeof(int32_t) * P);
  w.topk_w = (float*)take(sizeof(float) * P);
  w.shared_gate = (float*)take(sizeof(float) * d.T);
  w.sorted_tok = (int32_t*)take(sizeof(int32_t) * R);
  w.sorted_slot = (int32_t*)take(sizeof(int32_t) * P);
  w.pair_dst = (int32_t*)take(sizeof(int32_t) * R);
  w.pair_pos = (int32_t*)take(sizeof(int32_t) * R);
  w.pair_w = (float*)take(sizeof(float) * R);
  w.logit_part = (float*)take(sizeof(float) * size_t(d.KS) * d.T * d.Rpad);
  w.xnorm = (float*)take(sizeof(float) * size_t(d.KS) * d.T);
  w.wnorm = (float*)take(sizeof(float) * size_t((d.T + 31) / 32) * d.KS * d.Rpad);
  w.status = (int32_t*)take(sizeof(int32_t) * kStatusWords);
  w.h = (__nv_bfloat16*)take(sizeof(__nv_bfloat16) * R * d.ldh);
  w.xn = (__nv_bfloat16*)take(sizeof(__nv_bfloat16) * size_t(d.T) * d.H);
  w.rows = (float*)take(sizeof(float) * R * d.H);
  w.x_perm = reinterpret_cast<__nv_bfloat16*>(w.rows);
  w.rows_bf16 = reinterpret_cast<__nv_bfloat16*>(w.rows);
  const size_t mt_max = R / 128 + d.E + 2;  // M tiles over all experts, partial ones included
  const int imax = d.I > d.Is ? d.I : d.Is;
  w.gu_tiles = (int4*)take(sizeof(int4) * mt_max * size_t(imax / 64 + 1));
  w.dn_tiles = (int4*)take(sizeof(int4) * mt_max * size_t(d.H / 128 + 1));
  w.m_tiles = (int4*)take(sizeof(int4) * mt_max);
  w.tile_counts = (int32_t*)take(sizeof(int32_t) * 8);
  w.route_queue = (int32_t*)take(sizeof(int32_t) * size_t(d.T));
  const size_t ntile = (size_t(d.T) + 127) / 128;
  w.hist = (int32_t*)take(sizeof(int32_t) * ntile * d.E);
  w.hist_base = (int32_t*)take(sizeof(int32_t) * ntile * d.E);
  w.bytes = off;
  return w;
}

// ---- device helpers ------------------------------------------------------------

// 128-bit streaming load for weights: each byte is read once per call, so keep
// it out of L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 128-bit load for activations that several warps of a CTA re-read.
__device__ __forceinline__ uint4 ldg_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 32-wide k step of a 16-row weight tile against 8 columns.
//
// Lane (g = lane/4, c = lane%4) holds, from one 16-byte load each, global
// k in [k0+8c, k0+8c+8) of weight rows g and g+8 (wa, wb) and of column g of
// the activation tile (xv).  The two MMAs see a fixed permutation of the 32
// k indices, identical for A and B, so the dot product is unchanged while
// every operand comes from one coalesced 128-bit load.
__device__ __forceinline__ void mma_k32(float (&d)[4], const uint4& wa, const uint4& wb,
                                        const uint4& xv) {
  mma16816(d, wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
  mma16816(d, wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
}

// silu(g) = g * sigmoid(g); fast division (for g << 0 the denominator
// overflows to +inf and the quotient is 0, the limit).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Qwen3_5MoeRMSNorm (modeling_qwen3_5_moe.py:795-812) in pieces, for kernels
// that normalise rows as they load them.  rms_row_scale is rsqrt(mean(x^2) +
// eps) of one row computed by one warp in exactly the order of
// rmsnorm_kernel's 256 threads: thread i (warp v = i / 32) sums its 16-byte
// pieces i, i + 256, ... with fmaf, each warp's sum is lane 0's result of the
// xor-shuffle tree, and the eight warp sums are added in order -- so the
// value, and every output below, equals the standalone kernel's bit for bit.
// H % 8 == 0.
__device__ __forceinline__ float rms_row_scale(const __nv_bfloat16* __restrict__ row, int H,
                                               float eps) {
  const int lane = threadIdx.x & 31, n8 = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(row);
  // the first piece of each of the eight warps, all loads in flight at once
  // (a missing piece adds fmaf(0, 0, s) = s: exact)
  uint4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = k * 32 + lane;
    v[k] = i < n8 ? __ldg(xr + i) : make_uint4(0u, 0u, 0u, 0u);
  }
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float ss = 0.f;
    uint4 p = v[k];
    for (int i = k * 32 + lane;; i += 256) {
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&p);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b[j]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
      if (i + 256 >= n8) break;  // rows longer than 2048: the thread's next piece
      p = __ldg(xr + i + 256);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    tot += __shfl_sync(0xffffffffu, ss, 0);
  }
  return rsqrtf(tot / float(H) + eps);
}
// bf16(x * r * (1 + w)) of eight elements (the standalone kernel's expression).
__device__ __forceinline__ uint4 rms_apply8(const uint4& xv, const uint4& wv, float r) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&xv);
  const __nv_bfloat162* c = reinterpret_cast<const __nv_bfloat162*>(&wv);
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(b[j]), g = __bfloat1622float2(c[j]);
    __nv_bfloat162 r2 = __floats2bfloat162_rn(f.x * r * (1.f + g.x), f.y * r * (1.f + g.y));
    op[j] = *reinterpret_cast<uint32_t*>(&r2);
  }
  return o;
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

}  // namespace pmoe
