// tcgen05 grouped GEMMs for the compute-bound prefill regime (large T).
//
// gather_rows_kernel: x_perm[p] = x[sorted_tok[p]] for every dispatched row
// of a planned gate_up tile, written once so that the GEMM loads A with
// whole-tile TMA copies.  (Row gathers inside the GEMM, by cp.async or by
// 4-row TMA gathers, cost more than this copy: each 128-row A tile is read
// once per N block.)
// tc_grouped_kernel: persistent, warp-specialised, over a tile list
// (expert, first dispatched row, rows, N block) built on the device:
//     warp 0        TMA producer: A (x_perm for gate_up, h for down) and B
//                   (expert weights), 128-byte swizzle, one mbarrier per stage
//     warp 1        TMEM owner + single-thread tcgen05.mma issuer
//     warps 2..9    epilogue: TMEM -> registers -> global; two warps per TMEM
//                   lane quadrant, each owning half of the tile's columns
// Tiles are 128 (dispatched rows) x 256 (output columns), K staged 64 at a
// time through a 4-deep ring of 48 KiB stages; the fp32 accumulator is
// double-buffered in TMEM (2 x 256 columns) so the epilogue of one tile
// overlaps the main loop of the next.  Tiles are ordered (expert, M block,
// N block), so the N blocks of one M block run side by side and share A in L2.
//
//   gate_up: N block = 128 gate rows + the 128 matching up rows of the
//            expert; epilogue h = bf16(silu(gate) * up)   (Qwen3_5MoeExperts
//            :743-746, SiLU per configuration_qwen3_5_moe.py:84)
//   down:    N block = 256 output columns; epilogue adds w * row to the
//            token's fp32 accumulator with red.global.add.v4.f32 (the
//            routed combine of moe_grouped_mlp.py:152-163 / the index_add_ of
//            modeling_qwen3_5_moe.py:748-749, summed in fp32).
// The shared expert is expert index E: rows P.. of the dispatch, one per
// token of its range, weight = its sigmoid gate.
#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tc.cuh"

namespace pmoe {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kTcStages = 4;
constexpr int kABytes = kBM * kBK * 2;   // 16 KiB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KiB
constexpr int kTcStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each owning half the columns
constexpr int kEpiStage = kEpiWarps * 32 * 33 * 4;  // down epilogue: one 32x33 fp32 tile per warp
constexpr int kTcSmem = kTcStages * kTcStageBytes + 1024 + 256 + kEpiStage;
constexpr int kTcThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;      // two 256-column fp32 accumulators
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN);

enum TcMode { kGateUp = 0, kDown = 1 };

struct TileTables {
  const int4* tiles;     // (expert, row0, nrows, n_block)
  const int32_t* count;  // number of tiles
  const int32_t* sorted_tok;
  const float* pair_w;
};

__device__ __forceinline__ uint8_t* tc_align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void tc_status(int* status, int code) { atomicCAS(status, 0, code); }

// tm_b: routed weights, tm_b_sh0/1: shared-expert weights, tm_a: A (x_perm
// for gate_up, h for down).
template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_grouped_kernel(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b_sh0,
    const __grid_constant__ CUtensorMap tm_b_sh1, const __grid_constant__ CUtensorMap tm_a,
    TileTables tt, int H, int E, int I, int Is,
    int ldh, __nv_bfloat16* __restrict__ h, float* __restrict__ y_acc, int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc_align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* tfull = empty + kTcStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = tt.count[0];
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_b);
      prefetch_tmap(&tm_a);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int4 tl = tt.tiles[t];
        const int e = tl.x, row0 = tl.y, nb = tl.w;
        const bool sh = (e == E);
        const int Ke = MODE == kGateUp ? H : (sh ? Is : I);
        const int nk = Ke / kBK;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kTcStages;
          if (it >= uint32_t(kTcStages) && !mbar_wait(&empty[s], ((it / kTcStages) & 1) ^ 1)) {
            tc_status(status, kStatusTimeoutEmpty);
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kTcStageBytes;
          uint8_t* sb = sa + kABytes;
          mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
          tma_load_2d(sa, &tm_a, kc * kBK, row0, &full[s]);
          if (MODE == kGateUp) {
            const int j0 = nb * (kBN / 2);
            if (sh) {
              tma_load_2d(sb, &tm_b_sh0, kc * kBK, j0, &full[s]);
              tma_load_2d(sb + kBBytes / 2, &tm_b_sh1, kc * kBK, j0, &full[s]);
            } else {
              tma_load_2d(sb, &tm_b, kc * kBK, e * 2 * I + j0, &full[s]);
              tma_load_2d(sb + kBBytes / 2, &tm_b, kc * kBK, e * 2 * I + I + j0, &full[s]);
            }
          } else {
            const int n0 = nb * kBN;
            if (sh)
              tma_load_2d(sb, &tm_b_sh0, kc * kBK, n0, &full[s]);
            else
              tma_load_2d(sb, &tm_b, kc * kBK, e * H + n0, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, lt = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
        const int4 tl = tt.tiles[t];
        const bool sh = (tl.x == E);
        const int Ke = MODE == kGateUp ? H : (sh ? Is : I);
        const int nk = Ke / kBK;
        const uint32_t b = lt & 1, use = lt >> 1;
        if (lt >= 2 && !mbar_wait(&tempty[b], (use - 1) & 1)) {
          tc_status(status, kStatusTimeoutTmem);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * kBN;
        bool ok = true;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kTcStages;
          if (!mbar_wait(&full[s], (it / kTcStages) & 1)) {
            tc_status(status, kStatusTimeoutFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + s * kTcStageBytes, sb = sa + kABytes;
          const uint64_t ad = sdesc_k_sw128(sa), bd = sdesc_k_sw128(sb);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(d_tmem, ad + uint64_t(kk * 2), bd + uint64_t(kk * 2), kIdesc,
                      (kc | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                // TMEM lane quadrant of this warp
    const int half = (warp - 2) / 4;      // which half of the tile columns
    const int r = q * 32 + lane;           // tile row of this thread
    uint32_t lt = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
      const int4 tl = tt.tiles[t];
      const int row0 = tl.y, nrows = tl.z, nb = tl.w;
      const uint32_t b = lt & 1, use = lt >> 1;
      if (!mbar_wait(&tfull[b], use & 1)) {
        tc_status(status, kStatusTimeoutTmem);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16) + b * kBN;
      const bool valid = r < nrows;
      if (MODE == kGateUp) {
        const int j0 = nb * (kBN / 2);
        __nv_bfloat16* hrow = h + size_t(row0 + r) * ldh + j0;
#pragma unroll 1
        for (int cc = 2 * half; cc < 2 * half + 2; ++cc) {
          uint32_t gv[32], uv[32];
          tmem_ld32(taddr + cc * 32, gv);
          tmem_ld32(taddr + 128 + cc * 32, uv);
          tmem_ld_wait();
          if (valid) {
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 = silu_f(__uint_as_float(gv[2 * i])) * __uint_as_float(uv[2 * i]);
              const float a1 =
                  silu_f(__uint_as_float(gv[2 * i + 1])) * __uint_as_float(uv[2 * i + 1]);
              __nv_bfloat162 v2 = __floats2bfloat162_rn(a0, a1);
              packed[i] = *reinterpret_cast<uint32_t*>(&v2);
            }
            uint4* dst = reinterpret_cast<uint4*>(hrow + cc * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                  packed[4 * i + 3]);
          }
        }
      } else {
        const int n0 = nb * kBN;
        int tok = 0;
        float w = 0.f;
        if (valid) {
          tok = tt.sorted_tok[row0 + r];
          w = tt.pair_w[row0 + r];
        }
        float* dst = y_acc + size_t(tok) * H + n0;
        // Per-warp 32x32 staging tile: each reduction instruction then covers
        // 4 rows x 128 contiguous bytes instead of 32 scattered 16-byte pieces.
        float* stg = reinterpret_cast<float*>(smem + kTcStages * kTcStageBytes + 256) +
                     (warp - 2) * 32 * 33;
#pragma unroll 1
        for (int cc = 4 * half; cc < 4 * half + 4; ++cc) {
          uint32_t v[32];
          tmem_ld32(taddr + cc * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) stg[lane * 33 + i] = w * __uint_as_float(v[i]);
          __syncwarp();
          const int c4 = (lane & 7) * 4;
#pragma unroll
          for (int pass = 0; pass < 8; ++pass) {
            const int rr = pass * 4 + (lane >> 3);
            float* rdst = reinterpret_cast<float*>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), rr));
            const int rvalid = __shfl_sync(0xffffffffu, valid ? 1 : 0, rr);
            if (rvalid) {
              const float* sp = stg + rr * 33 + c4;
              red_add_v4(rdst + cc * 32 + c4, sp[0], sp[1], sp[2], sp[3]);
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }

  __syncwarp();  // reconverge warps whose work ran on one elected lane
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// x_perm[p, :] = x[sorted_tok[p], :] for the rows of every M tile (each
// dispatched row of a computed expert once).  Work item = 16 rows of one M
// tile, one warp each, 16-byte copies with four in flight per lane.
// ---------------------------------------------------------------------------
constexpr int kGatherThreads = 256;

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(
    const __nv_bfloat16* __restrict__ x, const int4* __restrict__ m_tiles,
    const int32_t* __restrict__ count, const int32_t* __restrict__ sorted_tok, int H,
    __nv_bfloat16* __restrict__ x_perm) {
  const int lane = threadIdx.x & 31;
  const int nw = count[0] * (kBM / 16);
  const int h8 = H / 8;
  for (int w = blockIdx.x * (kGatherThreads / 32) + (threadIdx.x >> 5); w < nw;
       w += gridDim.x * (kGatherThreads / 32)) {
    const int4 tl = m_tiles[w / (kBM / 16)];
    const int r_end = min(tl.z, (w % (kBM / 16) + 1) * 16);
    for (int r = (w % (kBM / 16)) * 16; r < r_end; ++r) {
      const int p = tl.y + r;
      const uint4* src = reinterpret_cast<const uint4*>(x + size_t(sorted_tok[p]) * H);
      uint4* dst = reinterpret_cast<uint4*>(x_perm + size_t(p) * H);
      int i = lane;
      for (; i + 96 < h8; i += 128) {
        const uint4 a = __ldg(src + i), b = __ldg(src + i + 32), c = __ldg(src + i + 64),
                    d = __ldg(src + i + 96);
        dst[i] = a;
        dst[i + 32] = b;
        dst[i + 64] = c;
        dst[i + 96] = d;
      }
      for (; i < h8; i += 32) dst[i] = __ldg(src + i);
    }
  }
}

// ---------------------------------------------------------------------------
// Tile planning (one CTA): for every active expert (in the active-list order,
// the shared expert last) emit its (M block, N block) tiles for both GEMMs.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 512;

__global__ void __launch_bounds__(kPlanThreads) plan_tiles_kernel(
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
    const int32_t* __restrict__ n_active, int E, int H, int I, int Is, int4* __restrict__ gu_tiles,
    int4* __restrict__ dn_tiles, int4* __restrict__ m_tiles, int32_t* __restrict__ counts) {
  __shared__ int s_wsum[3][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int na = n_active[0];
  int e = -1, n = 0, p0 = 0, mt = 0, nb_gu = 0, nb_dn = H / kBN;
  if (tid < na) {
    e = active[tid];
    p0 = offsets[e];
    n = offsets[e + 1] - p0;
    mt = (n + kBM - 1) / kBM;
    nb_gu = (e == E ? Is : I) / (kBN / 2);
  }
  int v[3] = {mt * nb_gu, mt * nb_dn, mt};
  int ex[3];
  // block exclusive scan of the three tile counts
  for (int k = 0; k < 3; ++k) {
    int incl = v[k];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[k][warp] = incl;
    ex[k] = incl - v[k];
  }
  __syncthreads();
  if (warp == 0) {
    for (int k = 0; k < 3; ++k) {
      const int s = lane < kPlanThreads / 32 ? s_wsum[k][lane] : 0;
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < kPlanThreads / 32) s_wsum[k][lane] = incl - s;
      if (lane == 31) counts[k] = incl;
    }
  }
  __syncthreads();
  if (tid < na) {
    int base = s_wsum[0][warp] + ex[0];
    for (int m = 0; m < mt; ++m)
      for (int nb = 0; nb < nb_gu; ++nb)
        gu_tiles[base++] = make_int4(e, p0 + m * kBM, min(kBM, n - m * kBM), nb);
    base = s_wsum[1][warp] + ex[1];
    for (int m = 0; m < mt; ++m)
      for (int nb = 0; nb < nb_dn; ++nb)
        dn_tiles[base++] = make_int4(e, p0 + m * kBM, min(kBM, n - m * kBM), nb);
    base = s_wsum[2][warp] + ex[2];
    for (int m = 0; m < mt; ++m)
      m_tiles[base++] = make_int4(e, p0 + m * kBM, min(kBM, n - m * kBM), 0);
  }
}

// y = bf16(y_acc)
__global__ void __launch_bounds__(256) finalize_kernel(const float* __restrict__ y_acc, long n4,
                                                       __nv_bfloat16* __restrict__ y) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 v = reinterpret_cast<const float4*>(y_acc)[i];
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(v.z, v.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo2);
  packed.y = *reinterpret_cast<uint32_t*>(&hi2);
  reinterpret_cast<uint2*>(y)[i] = packed;
}

namespace {
int g_tc_sms = 148;
}

cudaError_t tc_init(int num_sms) {
  g_tc_sms = num_sms;
  cudaError_t e = cudaFuncSetAttribute(tc_grouped_kernel<kGateUp>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tc_grouped_kernel<kDown>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
}

bool tc_supported(const Dims& d) {
  return d.H % kBN == 0 && d.I % (kBN / 2) == 0 && d.Is % (kBN / 2) == 0 && d.E <= 511;
}

cudaError_t launch_tc_experts(const Dims& d, const __nv_bfloat16* x,
                              const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                              const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                              const __nv_bfloat16* w_sh_down, const Workspace& ws,
                              __nv_bfloat16* y, bool zero_acc, cudaStream_t st,
                              void* mid_event) {
  const uint64_t H = d.H, I = d.I, Is = d.Is, E = d.E, T = d.T;
  const uint64_t P = T * d.K, R = P + T, ldh = d.ldh;
  CUtensorMap tm_gu, tm_sg, tm_su, tm_dn, tm_sd, tm_h, tm_xp;
  if (!make_tmap_bf16_2d(&tm_gu, w_gate_up, H, E * 2 * I, H * 2, kBK, kBN / 2) ||
      !make_tmap_bf16_2d(&tm_sg, w_sh_gate, H, Is, H * 2, kBK, kBN / 2) ||
      !make_tmap_bf16_2d(&tm_su, w_sh_up, H, Is, H * 2, kBK, kBN / 2) ||
      !make_tmap_bf16_2d(&tm_dn, w_down, I, E * H, I * 2, kBK, kBN) ||
      !make_tmap_bf16_2d(&tm_sd, w_sh_down, Is, H, Is * 2, kBK, kBN) ||
      !make_tmap_bf16_2d(&tm_h, ws.h, ldh, R, ldh * 2, kBK, kBM) ||
      !make_tmap_bf16_2d(&tm_xp, ws.x_perm, H, R, H * 2, kBK, kBM))
    return cudaErrorInvalidValue;
  plan_tiles_kernel<<<1, kPlanThreads, 0, st>>>(ws.offsets, ws.active, ws.n_active, d.E, d.H,
                                                d.I, d.Is, ws.gu_tiles, ws.dn_tiles,
                                                ws.m_tiles, ws.tile_counts);
  gather_rows_kernel<<<g_tc_sms * 4, kGatherThreads, 0, st>>>(x, ws.m_tiles, ws.tile_counts + 2,
                                                                ws.sorted_tok, d.H, ws.x_perm);
  cudaError_t err = cudaSuccess;
  if (zero_acc) {
    err = cudaMemsetAsync(ws.y_acc, 0, sizeof(float) * size_t(T) * H, st);
    if (err != cudaSuccess) return err;
  }
  int* status = ws.status + 1;
  TileTables gu{ws.gu_tiles, ws.tile_counts, ws.sorted_tok, ws.pair_w};
  TileTables dn{ws.dn_tiles, ws.tile_counts + 1, ws.sorted_tok, ws.pair_w};
  tc_grouped_kernel<kGateUp><<<g_tc_sms, kTcThreads, kTcSmem, st>>>(
      tm_gu, tm_sg, tm_su, tm_xp, gu, d.H, d.E, d.I, d.Is, d.ldh, ws.h, ws.y_acc, status);
  if (mid_event) {
    err = cudaEventRecord(static_cast<cudaEvent_t>(mid_event), st);
    if (err != cudaSuccess) return err;
  }
  tc_grouped_kernel<kDown><<<g_tc_sms, kTcThreads, kTcSmem, st>>>(
      tm_dn, tm_sd, tm_sd, tm_h, dn, d.H, d.E, d.I, d.Is, d.ldh, ws.h, ws.y_acc, status);
  const long n4 = long(T) * d.H / 4;
  finalize_kernel<<<unsigned((n4 + 255) / 256), 256, 0, st>>>(ws.y_acc, n4, y);
  return cudaGetLastError();
}

}  // namespace pmoe
