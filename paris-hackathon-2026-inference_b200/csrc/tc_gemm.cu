// tcgen05 grouped GEMMs for the compute-bound prefill regime (large T).
//
//   plan_tiles_kernel   tile lists for both GEMMs from the dispatch offsets
//   gather_rows_kernel  x_perm[p] = x[sorted_tok[p]] for every dispatched row
//                       of a computed expert, once, so that the GEMM loads its
//                       B operand with tiled TMA copies (row gathers inside the
//                       GEMM, by cp.async or 4-row TMA gathers, cost more:
//                       every row block is read once per feature block)
//   tc_pair_kernel      the expert GEMM, persistent, warp-specialised, on CTA
//                       pairs (cta_group::2):
//     warp 0        TMA producer, 128-byte swizzle, a 6-deep ring of 32 KiB
//                   stages per CTA
//     warp 1        TMEM owner (both CTAs) + single-thread MMA issuer (even CTA)
//     warps 2..17   epilogue: TMEM -> registers -> global; four warps per
//                   TMEM lane quadrant, each owning 64 of the tile's columns
//   combine_rows_kernel y = bf16(sum of each token's expert rows)
// The fp32 accumulator is double-buffered in TMEM (2 x 256 columns) so the
// epilogue of one tile overlaps the main loop of the next.
//
//   gate_up: epilogue h = bf16(silu(gate) * up)   (Qwen3_5MoeExperts
//            :743-746, SiLU per configuration_qwen3_5_moe.py:84)
//   down:    epilogue writes bf16(w * row) to the pair's token-major row;
//            the combine then sums each token's rows in fp32 (the routed
//            combine of moe_grouped_mlp.py:152-163 / the index_add_ of
//            modeling_qwen3_5_moe.py:748-749).  Plain stores: fp32 atomic
//            adds of every output row into L2 were the down GEMM's limit.
// The shared expert is expert index E: rows P.. of the dispatch, one per
// token of its range, weight = its sigmoid gate.

#include <algorithm>
#include <cstdlib>

#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tc.cuh"

namespace pmoe {

constexpr int kBM = 128;                  // weight rows per CTA (the pair MMA has M = 256)
constexpr int kBK = 64;                   // K per stage (one 128-byte swizzle atom)
constexpr int kTok = 256;                 // dispatched rows per tile (UMMA N <= 256)
constexpr int kHalfTok = kTok / 2;        // rows of B staged by each CTA of the pair
constexpr int kGatherRows = 128;          // rows per x_perm copy block
constexpr int kTcStages = 6;
constexpr int kWBytes = kBM * kBK * 2;    // 16 KiB: this CTA's half of A (weights)
constexpr int kRowBytes = kHalfTok * kBK * 2;  // 16 KiB: this CTA's half of B (rows)
constexpr int kRowChunk = 32;             // rows per small B copy
constexpr int kTcStageBytes = kWBytes + kRowBytes;  // 32 KiB
constexpr int kEpiWarps = 16;  // four per TMEM lane quadrant, each owning 64 columns
constexpr int kEpiWarpBytes = 32 * 16 * 2;  // per-warp gate_up staging tile (bf16 32 x 16)
constexpr int kBarBytes = 256;            // mbarriers + TMEM slot
constexpr int kTcSmem = kTcStages * kTcStageBytes + 1024 + kBarBytes + kEpiWarps * kEpiWarpBytes;
constexpr int kTcThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;       // two 256-column fp32 accumulators
static_assert(kTcSmem <= 227 * 1024, "shared memory");
// barrier area: 16 mbarriers (128 B), the TMEM slot at 128, four abort flags at 192
static_assert(192 + 4 * 4 <= kBarBytes, "barrier area");

enum TcMode { kGateUp = 0, kDown = 1 };

struct TileTables {
  const int4* tiles;     // (expert, row0, nrows, feature block)
  const int32_t* count;  // number of tiles
  const int32_t* pair_dst;  // token-major output row of each dispatched row
  const float* pair_w;
  RowsOut out;              // down: peer destinations (out.world > 0) of the rows
  int T, K;                 // for the token of a token-major row
  int sh_lo;                // first token of the shared expert's rows
  int sh5;                  // gate_up: shared gate|up in one 5-D map (tm_b_sh0)
  int sh_swap;              // ... whose first half is the up rows (w_sh_up < w_sh_gate)
};

__device__ __forceinline__ uint8_t* tc_align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void tc_status(int* status, int code) { atomicCAS(status, 0, code); }

// Tile t of the list, or an empty tile past its end (used to fetch the next
// tile's descriptor one tile ahead).
__device__ __forceinline__ int4 tile_at(const TileTables& tt, int t, int ntiles) {
  return t < ntiles ? tt.tiles[t] : make_int4(0, 0, 0, 0);
}

// One persistent kernel per GEMM, launched as CTA pairs (clusters of 2).  A
// pair computes a 256 (weight rows) x N (dispatched rows) tile with
// cta_group::2 MMAs issued by the even CTA: each CTA stages 128 weight rows
// (A) and N/2 dispatched rows (B) per K step, and holds its 128 accumulator
// rows x N columns in its own TMEM.  N is the tile's rows rounded up to 16,
// so an expert's last tile wastes at most 15 rows of MMA work, and only the
// 32-row chunks of B holding its rows are loaded.
//   gate_up: a pair tile covers 128 features; each CTA's A is 64 features as
//            four groups of 16 gate rows each followed by the matching 16 up
//            rows (a 5-D tensor-map box over the [E][2I][H] weights), so TMEM
//            lane l < 16 of a quadrant holds the gate and lane l + 16 the up
//            value of the same feature.  B = x_perm rows.
//   down:    a pair tile covers 256 output features; B = h rows.
// Every CTA's producer signals the even CTA's stage barrier; the MMA commit
// releases the stage in both CTAs; both CTAs' epilogue warps release the
// accumulator on the even CTA's barrier.
// tm_b: routed weights (5-D for gate_up), tm_b_sh0/1: shared-expert weights
// (16-row boxes for gate_up), tm_a / tm_a32: the dispatched rows (x_perm for
// gate_up, h for down) in 128- and 32-row boxes; tm_x / tm_x32: gate_up's
// shared-expert rows, which are the tokens sh_lo.. in order, read from x
// itself (x_perm holds no copy of them).
template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_pair_kernel(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b_sh0,
    const __grid_constant__ CUtensorMap tm_b_sh1, const __grid_constant__ CUtensorMap tm_a,
    const __grid_constant__ CUtensorMap tm_a32, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_x32, const __grid_constant__ TileTables tt, int H,
    int E, int I, int Is,
    int ldh, __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ out_rows,
    int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc_align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* tfull = empty + kTcStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  // down epilogue: per column quarter, set when one of its warps gave up
  // waiting for an accumulator, so that its four warps leave together
  volatile int* quarter_abort = reinterpret_cast<volatile int*>(tmem_slot + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    for (int i = 0; i < 4; ++i) quarter_abort[i] = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ntiles = tt.count[0];
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_b);
      prefetch_tmap(&tm_a);
      if (MODE == kGateUp) prefetch_tmap(&tm_x);
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // even CTA's stage barriers
      uint32_t it = 0;
      bool ok = true;
      int4 tl_next = tile_at(tt, pair, ntiles);
      for (int t = pair; t < ntiles && ok; t += npairs) {
        const int4 tl = tl_next;
        tl_next = tile_at(tt, t + npairs, ntiles);
        const int e = tl.x;
        const int nh = ((tl.z + 15) & ~15) / 2;        // rows of B in this CTA
        const int r0 = tl.y + int(rank) * nh;
        const bool sh = (e == E);
        const int Ke = MODE == kGateUp ? H : (sh ? Is : I);
        const int nk = Ke / kBK;
        const int nchunks = (nh + kRowChunk - 1) / kRowChunk;
        const bool whole = nh > kHalfTok / 2;  // one 128-row box, else 32-row boxes
        const uint32_t tx = kWBytes + (whole ? kHalfTok : nchunks * kRowChunk) * kBK * 2;
        const int f0 = MODE == kGateUp ? tl.w * 128 + 64 * int(rank) : tl.w * 256 + 128 * int(rank);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kTcStages;
          if (it >= uint32_t(kTcStages) && !mbar_wait(&empty[s], ((it / kTcStages) & 1) ^ 1)) {
            tc_status(status, kStatusTimeoutEmpty);
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kTcStageBytes;
          const uint32_t fb = full0 + s * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * tx);
          if (MODE == kGateUp) {
            if (sh && tt.sh5) {
              tma_load_5d_pair(st, &tm_b_sh0, kc * kBK, 0, 0, f0 / 16, 0, fb);
            } else if (sh) {
              for (int g = 0; g < 4; ++g) {
                tma_load_2d_pair(st + g * 4096, &tm_b_sh0, kc * kBK, f0 + 16 * g, fb);
                tma_load_2d_pair(st + g * 4096 + 2048, &tm_b_sh1, kc * kBK, f0 + 16 * g, fb);
              }
            } else {
              tma_load_5d_pair(st, &tm_b, kc * kBK, 0, 0, f0 / 16, e, fb);
            }
          } else {
            if (sh)
              tma_load_2d_pair(st, &tm_b_sh0, kc * kBK, f0, fb);
            else
              tma_load_2d_pair(st, &tm_b, kc * kBK, e * H + f0, fb);
          }
          // gate_up's shared rows P + i are token sh_lo + i: straight from x
          const bool from_x = MODE == kGateUp && sh;
          const int ra = from_x ? r0 - tt.T * tt.K + tt.sh_lo : r0;
          const CUtensorMap* ma = from_x ? &tm_x : &tm_a;
          const CUtensorMap* ma32 = from_x ? &tm_x32 : &tm_a32;
          if (whole) {
            tma_load_2d_pair(st + kWBytes, ma, kc * kBK, ra, fb);
          } else {
            for (int j = 0; j < nchunks; ++j)
              tma_load_2d_pair(st + kWBytes + j * kRowChunk * kBK * 2, ma32, kc * kBK,
                               ra + j * kRowChunk, fb);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      uint32_t it = 0, lt = 0;
      int4 tl_next = tile_at(tt, pair, ntiles);
      for (int t = pair; t < ntiles; t += npairs, ++lt) {
        const int4 tl = tl_next;
        tl_next = tile_at(tt, t + npairs, ntiles);
        const bool sh = (tl.x == E);
        const int Ke = MODE == kGateUp ? H : (sh ? Is : I);
        const int nk = Ke / kBK;
        const uint32_t idesc = idesc_bf16_f32(2 * kBM, (tl.z + 15) & ~15);
        const uint32_t b = lt & 1, use = lt >> 1;
        if (lt >= 2 && !mbar_wait_cluster(&tempty[b], (use - 1) & 1)) {
          tc_status(status, kStatusTimeoutTmem);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * 256;
        bool ok = true;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kTcStages;
          if (!mbar_wait(&full[s], (it / kTcStages) & 1)) {
            tc_status(status, kStatusTimeoutFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * kTcStageBytes;
          const uint64_t wd = sdesc_k_sw128(st), rd = sdesc_k_sw128(st + kWBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16_pair(d_tmem, wd + uint64_t(kk * 2), rd + uint64_t(kk * 2), idesc,
                           (kc | kk) != 0 ? 1u : 0u);
          umma_commit_pair_both(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair_both(&tfull[b]);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs) ----------------
    // Warp (q, quarter): this CTA's weight rows q*32 .. q*32+31 (its TMEM
    // lane quadrant), tile columns quarter*64 .. +63.
    const int q = warp & 3;
    const int quarter = (warp - 2) / 4;
    const int cw = quarter * 64;
    uint8_t* stg_raw = smem + kTcStages * kTcStageBytes + kBarBytes + (warp - 2) * kEpiWarpBytes;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    uint32_t lt = 0;
    int4 tl_next = tile_at(tt, pair, ntiles);
    for (int t = pair; t < ntiles; t += npairs, ++lt) {
      const int4 tl = tl_next;
      tl_next = tile_at(tt, t + npairs, ntiles);
      const int row0 = tl.y, nrows = tl.z;
      const uint32_t b = lt & 1, use = lt >> 1;
      // down: this lane's output rows of the two 32-row chunks, loaded
      // before the accumulator wait so their latency overlaps it.
      int ldst[2] = {0, 0}, lown[2] = {0, 0};
      if (MODE == kDown) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int r = cw + 32 * k + lane;
          if (r < nrows) ldst[k] = tt.pair_dst[row0 + r];
          if (tt.out.world > 0) {
            const int tk = tt.T * tt.K;
            lown[k] = slice_owner(ldst[k] < tk ? ldst[k] / tt.K : ldst[k] - tk, tt.T,
                                  tt.out.world);
          }
        }
      }
      const bool got = mbar_wait(&tfull[b], use & 1);
      if (MODE == kDown) {
        // the quarter's warps meet at named barriers below: decide together
        if (!got && lane == 0) quarter_abort[quarter] = 1;
        named_bar_sync(1 + quarter, 128);
        if (quarter_abort[quarter]) {
          tc_status(status, kStatusTimeoutTmem);
          break;
        }
      } else if (!got) {
        tc_status(status, kStatusTimeoutTmem);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16) + b * 256;
      if (MODE == kGateUp) {
        // Quadrant q holds features f0 .. f0+15: lanes 0-15 their gate rows,
        // lanes 16-31 their up rows.  Per 32-row chunk, lane l < 16 forms
        // h for rows 0-15 and lane l + 16 for rows 16-31 (one shuffle per
        // value), then a 32 x 16 transpose in shared memory gives each row's
        // 32 bytes of h to one lane.
        const int f0 = tl.w * 128 + 64 * int(rank) + q * 16;
        const int fl = lane & 15, hi = lane >> 4;
        const bool swap_gu = tt.sh_swap && tl.x == E;
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(stg_raw);  // [32 rows][16]
        if (cw < nrows) {
          uint32_t v[2][32];  // 64 columns: two loads, one wait
          tmem_ld32(taddr + cw, v[0]);
          tmem_ld32(taddr + cw + 32, v[1]);
          tmem_ld_wait();
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const int c = cw + 32 * sub;
            if (c >= nrows) break;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float mine = __uint_as_float(hi ? v[sub][i] : v[sub][16 + i]);
              const float other = __shfl_xor_sync(0xffffffffu, mine, 16);
              float g = hi ? other : __uint_as_float(v[sub][i]);
              float u = hi ? __uint_as_float(v[sub][16 + i]) : other;
              if (swap_gu) {  // lanes 0-15 hold the up rows
                const float tmp = g;
                g = u;
                u = tmp;
              }
              stg[(hi * 16 + i) * 16 + fl] = __float2bfloat16_rn(silu_f(g) * u);
            }
            __syncwarp();
            if (c + lane < nrows) {
              const uint4* sp = reinterpret_cast<const uint4*>(stg + lane * 16);
              uint4* dp = reinterpret_cast<uint4*>(h + size_t(row0 + c + lane) * ldh + f0);
              dp[0] = sp[0];
              dp[1] = sp[1];
            }
            __syncwarp();
          }
        }
      } else {
        // Lane = output feature f0 + lane of each TMEM column (dispatched
        // row).  The four warps of a column quarter (one per lane quadrant)
        // stage 16 columns x their 128 features in shared memory, then each
        // warp stores whole 256-byte row segments (16 lanes x 16 bytes per
        // row): to this rank's rows, or to the token owner's buffer over
        // NVLink.  The routing weight is applied by the combine.
        const int fq = tl.w * 256 + 128 * int(rank);  // the quarter's first feature
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(
            smem + kTcStages * kTcStageBytes + kBarBytes + quarter * 4 * kEpiWarpBytes);
        const int bar_id = 1 + quarter;
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
          const int c = cw + 32 * sub;
          if (c >= nrows) break;  // uniform over the quarter's four warps
          uint32_t v[32];
          tmem_ld32(taddr + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int cc = c + 16 * hh;
            if (cc >= nrows) break;
            named_bar_sync(bar_id, 128);  // the previous segment's reads are done
#pragma unroll
            for (int i = 0; i < 16; ++i)
              stg[i * 128 + q * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[16 * hh + i]));
            named_bar_sync(bar_id, 128);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int ci = 4 * q + 2 * j + (lane >> 4);  // column within the 16
              const int dst = __shfl_sync(0xffffffffu, ldst[sub], 16 * hh + ci);
              const int own = __shfl_sync(0xffffffffu, lown[sub], 16 * hh + ci);
              if (cc + ci < nrows) {
                const uint4 val = reinterpret_cast<const uint4*>(stg + ci * 128)[lane & 15];
                __nv_bfloat16* base = tt.out.world > 0 ? tt.out.base[own] : out_rows;
                reinterpret_cast<uint4*>(base + size_t(dst) * H + fq)[lane & 15] = val;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + b * 8);
    }
  }

  __syncwarp();  // reconverge warps whose work ran on one elected lane
  if (MODE == kDown && tt.out.world > 0) __threadfence_system();  // peer rows visible
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// x_perm[p, :] = x[sorted_tok[p], :] for the rows of every M block (each
// dispatched row of a computed expert once).  Work item = 4 rows of one M
// block; a warp copies two rows at a time with all of their 16-byte loads in
// flight before the stores (H/256 loads per lane per row).
// ---------------------------------------------------------------------------
constexpr int kGatherThreads = 256;
constexpr int kGatherItemRows = 4;
constexpr int kGatherMaxH8 = 8;  // H <= 2048 for the unrolled row copy

__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(
    const __nv_bfloat16* __restrict__ x, const int4* __restrict__ m_tiles,
    const int32_t* __restrict__ count, const int32_t* __restrict__ sorted_tok, int H, int E,
    __nv_bfloat16* __restrict__ x_perm) {
  const int lane = threadIdx.x & 31;
  constexpr int kItems = kGatherRows / kGatherItemRows;
  const int nw = count[0] * kItems;
  const int per_lane = H / 256;  // 16-byte pieces per lane per row
  for (int w = blockIdx.x * (kGatherThreads / 32) + (threadIdx.x >> 5); w < nw;
       w += gridDim.x * (kGatherThreads / 32)) {
    const int4 tl = m_tiles[w / kItems];
    if (tl.x == E) continue;  // the shared expert's rows are read from x itself
    const int r_beg = (w % kItems) * kGatherItemRows;
    const int r_end = min(tl.z, r_beg + kGatherItemRows);
    for (int r = r_beg; r < r_end; r += 2) {
      const bool two = r + 1 < r_end;
      const int p0 = tl.y + r, p1 = two ? p0 + 1 : p0;
      const uint4* s0 = reinterpret_cast<const uint4*>(x + size_t(sorted_tok[p0]) * H);
      const uint4* s1 = reinterpret_cast<const uint4*>(x + size_t(sorted_tok[p1]) * H);
      uint4 a[kGatherMaxH8], b[kGatherMaxH8];
#pragma unroll
      for (int i = 0; i < kGatherMaxH8; ++i) {
        if (i < per_lane) {
          a[i] = __ldg(s0 + lane + 32 * i);
          b[i] = __ldg(s1 + lane + 32 * i);
        }
      }
      uint4* d0 = reinterpret_cast<uint4*>(x_perm + size_t(p0) * H);
      uint4* d1 = reinterpret_cast<uint4*>(x_perm + size_t(p1) * H);
#pragma unroll
      for (int i = 0; i < kGatherMaxH8; ++i) {
        if (i < per_lane) {
          d0[lane + 32 * i] = a[i];
          if (two) d1[lane + 32 * i] = b[i];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tile planning (one CTA, one thread per active expert; the shared expert is
// one of them): the gate_up and down tile lists (pair tiles of up to 256
// dispatched rows x 128 features for gate_up, x 256 features for down) and
// the 128-row blocks for the x_perm copy.
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 512;

// Exclusive block-wide scan of NV values per thread; totals[k] = sum.
template <int NV>
__device__ __forceinline__ void plan_scan(int (&v)[NV], int (&ex)[NV], int (*s_wsum)[32],
                                          int* totals) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
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
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int s = lane < kPlanThreads / 32 ? s_wsum[k][lane] : 0;
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < kPlanThreads / 32) s_wsum[k][lane] = incl - s;
      if (lane == 31) totals[k] = incl;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NV; ++k) ex[k] += s_wsum[k][warp];
  __syncthreads();
}

__global__ void __launch_bounds__(kPlanThreads) plan_tiles_kernel(
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
    const int32_t* __restrict__ n_active, int E, int H, int I, int Is, int rank, int world,
    int c0, int4* __restrict__ gu_tiles, int4* __restrict__ dn_tiles, int4* __restrict__ m_tiles,
    int32_t* __restrict__ counts) {
  __shared__ int s_wsum[3][32];
  __shared__ int s_tot[3];
  __shared__ int4 s_ex[kPlanThreads];       // (expert, first owned row, owned rows, nb_gu)
  __shared__ int4 s_base[kPlanThreads];     // first gate_up / down tile, first M block
  __shared__ int s_lo, s_hi;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int na = n_active[0];
  const int nb_dn = H / 256;
  if (tid == 0) {
    s_lo = 0x7fffffff;
    s_hi = 0;
  }
  __syncthreads();
  // Row split across `world` ranks: the 256-row blocks of every expert, in
  // dispatch order, each costing c0 + its rows, go to the rank whose share of
  // the total cost holds the block's middle, so each rank owns one contiguous
  // row range (c0 = 0: an even split of the rows; larger c0 evens out the
  // number of blocks, hence of GEMM tiles, per rank).
  int e = -1, r0 = 0, nrow = 0, nbg = 0, p0 = 0, n = 0, mt = 0;
  if (tid < na) {
    e = active[tid];
    p0 = offsets[e];
    n = offsets[e + 1] - p0;
    nbg = (e == E ? Is : I) / 128;
    mt = (n + kTok - 1) / kTok;
  }
  int cv[1] = {mt * c0 + n}, cx[1];
  plan_scan<1>(cv, cx, s_wsum, s_tot);
  const long total = s_tot[0];
  __syncthreads();
  if (tid < na) {
    int ma = mt, mb = mt;
    for (int m = 0; m < mt; ++m) {
      const long mid = cx[0] + long(m) * (c0 + kTok) + (c0 + min(kTok, n - m * kTok)) / 2;
      const bool own = mid * world >= long(rank) * total && mid * world < long(rank + 1) * total;
      if (own && ma == mt) ma = m;
      if (own) mb = m + 1;
    }
    if (ma < mb) {
      r0 = p0 + ma * kTok;
      nrow = min(n, mb * kTok) - ma * kTok;
      atomicMin(&s_lo, r0);
      atomicMax(&s_hi, r0 + nrow);
    }
  }
  const int mto = (nrow + kTok - 1) / kTok;
  int v[3] = {mto * nbg, mto * nb_dn, (nrow + kGatherRows - 1) / kGatherRows};
  int ex[3];
  plan_scan<3>(v, ex, s_wsum, s_tot);
  s_ex[tid] = make_int4(e, r0, nrow, nbg);
  s_base[tid] = make_int4(ex[0], ex[1], ex[2], 0);
  if (tid == 0) {
    counts[0] = s_tot[0];
    counts[1] = s_tot[1];
    counts[2] = s_tot[2];
    counts[4] = s_lo <= s_hi ? s_lo : 0;
    counts[5] = s_lo <= s_hi ? s_hi : 0;
  }
  __syncthreads();
  // Write-out: one warp per active expert, lanes striding over its tiles.
  for (int a = warp; a < na; a += kPlanThreads / 32) {
    const int4 x = s_ex[a], bs = s_base[a];
    const int mts = (x.z + kTok - 1) / kTok;
    for (int i = lane; i < mts * x.w; i += 32) {
      const int m = i / x.w;
      gu_tiles[bs.x + i] = make_int4(x.x, x.y + m * kTok, min(kTok, x.z - m * kTok), i % x.w);
    }
    for (int i = lane; i < mts * nb_dn; i += 32) {
      const int m = i / nb_dn;
      dn_tiles[bs.y + i] = make_int4(x.x, x.y + m * kTok, min(kTok, x.z - m * kTok), i % nb_dn);
    }
    const int mgs = (x.z + kGatherRows - 1) / kGatherRows;
    for (int m = lane; m < mgs; m += 32)
      m_tiles[bs.z + m] = make_int4(x.x, x.y + m * kGatherRows,
                                    min(kGatherRows, x.z - m * kGatherRows), 0);
  }
}

// y[t, :] = bf16( sum_{s<K, expert in [lo,hi)} w[t,s] * rows[t*K+s, :]
//                  + g[t] * rows[T*K+t, :] )      (+ resid: see below)
// over the bf16 expert rows the down GEMM wrote (routing weights w, shared
// gate g), in fp32 in a fixed order (the shared row for tokens in
// [sh_lo, sh_hi)).  One thread per 8 columns.
constexpr int kCombineMaxK = 8;  // top-k sizes up to this take the all-loads-in-flight path

__global__ void __launch_bounds__(256) combine_rows_kernel(
    const __nv_bfloat16* __restrict__ rows, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, const float* __restrict__ shared_gate, int T, int H,
    int K, int lo, int hi, int with_shared, int with_routed, int sh_lo, int sh_hi,
    const int32_t* __restrict__ pair_pos, const int32_t* __restrict__ row_range,
    const __nv_bfloat16* __restrict__ resid, __nv_bfloat16* __restrict__ y) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const int cols8 = H / 8;
  if (i >= long(T) * cols8) return;
  const int t = int(i / cols8), c8 = int(i % cols8);
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto add = [&](size_t row, float w) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(rows + row * H) + c8);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(b2[j]);
      s[2 * j] = fmaf(w, f.x, s[2 * j]);
      s[2 * j + 1] = fmaf(w, f.y, s[2 * j + 1]);
    }
  };
  // Row split: only rows this rank computed (dispatched position in range).
  const int p_lo = pair_pos ? row_range[0] : 0, p_hi = pair_pos ? row_range[1] : 0;
  auto mine = [&](size_t q) {
    if (!pair_pos) return true;
    const int p = pair_pos[q];
    return p >= p_lo && p < p_hi;
  };
  if (K <= kCombineMaxK) {
    // Select first, then issue every selected row's load before summing, so
    // the (up to) 9 row reads are in flight together.
    bool sel[kCombineMaxK + 1];
    float w[kCombineMaxK + 1];
    size_t q[kCombineMaxK + 1];
#pragma unroll
    for (int k = 0; k < kCombineMaxK; ++k) {
      q[k] = size_t(t) * K + k;
      sel[k] = false;
      w[k] = 0.f;
      if (k < K && with_routed) {
        const int e = topk_idx[q[k]];
        sel[k] = e >= lo && e < hi && mine(q[k]);
        if (sel[k]) w[k] = topk_w[q[k]];
      }
    }
    q[kCombineMaxK] = size_t(T) * K + t;
    sel[kCombineMaxK] = with_shared && t >= sh_lo && t < sh_hi && mine(q[kCombineMaxK]);
    w[kCombineMaxK] = sel[kCombineMaxK] ? shared_gate[t] : 0.f;
    uint4 v[kCombineMaxK + 1];
#pragma unroll
    for (int k = 0; k <= kCombineMaxK; ++k)
      if (sel[k]) v[k] = __ldg(reinterpret_cast<const uint4*>(rows + q[k] * H) + c8);
#pragma unroll
    for (int k = 0; k <= kCombineMaxK; ++k) {
      if (!sel[k]) continue;
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        s[2 * j] = fmaf(w[k], f.x, s[2 * j]);
        s[2 * j + 1] = fmaf(w[k], f.y, s[2 * j + 1]);
      }
    }
  } else {
    if (with_routed) {
      for (int k = 0; k < K; ++k) {
        const size_t qk = size_t(t) * K + k;
        const int e = topk_idx[qk];
        if (e >= lo && e < hi && mine(qk)) add(qk, topk_w[qk]);
      }
    }
    if (with_shared && t >= sh_lo && t < sh_hi && mine(size_t(T) * K + t))
      add(size_t(T) * K + t, shared_gate[t]);
  }
  if (resid) {  // decoder layer: y = bf16(resid + bf16(sum)), as residual + mlp(x) in bf16
    const uint4 rv = reinterpret_cast<const uint4*>(resid + size_t(t) * H)[c8];
    const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(r2[j]);
      s[2 * j] = f.x + bf16_round(s[2 * j]);
      s[2 * j + 1] = f.y + bf16_round(s[2 * j + 1]);
    }
  }
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 b2 = __floats2bfloat162_rn(s[2 * j], s[2 * j + 1]);
    op[j] = *reinterpret_cast<uint32_t*>(&b2);
  }
  reinterpret_cast<uint4*>(y + size_t(t) * H)[c8] = o;
}

// The same combine for K <= kCombineMaxK and H/8 <= 1024, as a persistent
// grid: a block takes one token at a time (thread = 8 columns), issues that
// token's row loads and meanwhile fetches the next token's selection (expert
// ids, weights, row positions), so the two dependent round trips overlap.
__device__ __forceinline__ void combine_select(
    int t, int T, int K, int lo, int hi, int with_shared, int with_routed, int sh_lo, int sh_hi,
    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
    const float* __restrict__ shared_gate, const int32_t* __restrict__ pair_pos, int p_lo,
    int p_hi, unsigned& mask, float (&w)[kCombineMaxK + 1]) {
  mask = 0u;
#pragma unroll
  for (int k = 0; k <= kCombineMaxK; ++k) w[k] = 0.f;
#pragma unroll
  for (int k = 0; k < kCombineMaxK; ++k) {
    if (k < K && with_routed) {
      const size_t q = size_t(t) * K + k;
      const int e = topk_idx[q];
      bool sel = e >= lo && e < hi;
      if (sel && pair_pos) {
        const int p = pair_pos[q];
        sel = p >= p_lo && p < p_hi;
      }
      if (sel) {
        mask |= 1u << k;
        w[k] = topk_w[q];
      }
    }
  }
  if (with_shared && t >= sh_lo && t < sh_hi) {
    bool sel = true;
    if (pair_pos) {
      const int p = pair_pos[size_t(T) * K + t];
      sel = p >= p_lo && p < p_hi;
    }
    if (sel) {
      mask |= 1u << kCombineMaxK;
      w[kCombineMaxK] = shared_gate[t];
    }
  }
}

__global__ void __launch_bounds__(256) combine_rows_tok_kernel(
    const __nv_bfloat16* __restrict__ rows, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, const float* __restrict__ shared_gate, int T, int H,
    int K, int lo, int hi, int with_shared, int with_routed, int sh_lo, int sh_hi,
    const int32_t* __restrict__ pair_pos, const int32_t* __restrict__ row_range,
    const __nv_bfloat16* __restrict__ resid, __nv_bfloat16* __restrict__ y, int t_lo,
    int t_hi, const __grid_constant__ RowsOut ydst, const int* __restrict__ abort_if) {
  // ydst.world > 0: each output row goes to row t of every rank's buffer
  // ydst.base[0..world) (peer stores) instead of y.
  // abort_if (may be null): a status word; non-zero (an earlier wait of the
  // exchange gave up) -> do nothing, in particular no peer stores.
  if (abort_if && __ldcg(abort_if) != 0) return;
  const int cols8 = H / 8, c8 = threadIdx.x;
  const bool act = c8 < cols8;
  const int p_lo = pair_pos ? row_range[0] : 0, p_hi = pair_pos ? row_range[1] : 0;
  unsigned mask = 0u;
  float w[kCombineMaxK + 1];
  int t = t_lo + blockIdx.x;
  if (t < t_hi)
    combine_select(t, T, K, lo, hi, with_shared, with_routed, sh_lo, sh_hi, topk_idx, topk_w,
                   shared_gate, pair_pos, p_lo, p_hi, mask, w);
  for (; t < t_hi; t += gridDim.x) {
    uint4 v[kCombineMaxK + 1];
#pragma unroll
    for (int k = 0; k <= kCombineMaxK; ++k) {
      const size_t q = k < kCombineMaxK ? size_t(t) * K + k : size_t(T) * K + t;
      if (act && (mask >> k & 1u)) v[k] = __ldg(reinterpret_cast<const uint4*>(rows + q * H) + c8);
    }
    const int tn = t + gridDim.x;  // next token's selection while the rows are in flight
    unsigned mask_n = 0u;
    float wn[kCombineMaxK + 1];
    if (tn < t_hi)
      combine_select(tn, T, K, lo, hi, with_shared, with_routed, sh_lo, sh_hi, topk_idx, topk_w,
                     shared_gate, pair_pos, p_lo, p_hi, mask_n, wn);
    if (act) {
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k <= kCombineMaxK; ++k) {
        if (!(mask >> k & 1u)) continue;
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v[k]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(b2[j]);
          s[2 * j] = fmaf(w[k], f.x, s[2 * j]);
          s[2 * j + 1] = fmaf(w[k], f.y, s[2 * j + 1]);
        }
      }
      if (resid) {  // decoder layer: y = bf16(resid + bf16(sum))
        const uint4 rv = reinterpret_cast<const uint4*>(resid + size_t(t) * H)[c8];
        const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(r2[j]);
          s[2 * j] = f.x + bf16_round(s[2 * j]);
          s[2 * j + 1] = f.y + bf16_round(s[2 * j + 1]);
        }
      }
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 b2 = __floats2bfloat162_rn(s[2 * j], s[2 * j + 1]);
        op[j] = *reinterpret_cast<uint32_t*>(&b2);
      }
      if (ydst.world > 0) {
        for (int q = 0; q < ydst.world; ++q)
          reinterpret_cast<uint4*>(ydst.base[q] + size_t(t) * H)[c8] = o;
      } else {
        reinterpret_cast<uint4*>(y + size_t(t) * H)[c8] = o;
      }
    }
    mask = mask_n;
#pragma unroll
    for (int k = 0; k <= kCombineMaxK; ++k) w[k] = wn[k];
  }
}

namespace {
int g_pairs = 74;  // co-resident CTA pairs of the GEMM kernels

// Per-block cost constant of the row split, in rows: 512 (two full blocks'
// rows) evens out the GEMM tile count per rank where few tiles per rank make
// the last round of the persistent grid decide the time, and keeps rows even
// where there are many (PMOE_SPLIT_C0 overrides).
int split_c0() {
  static const int c0 = [] {
    const char* v = std::getenv("PMOE_SPLIT_C0");
    const int n = v ? std::atoi(v) : 512;
    return n >= 0 && n <= 1 << 16 ? n : 512;
  }();
  return c0;
}

template <int MODE, typename... Args>
cudaError_t launch_pairs(cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * g_pairs);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tc_pair_kernel<MODE>, args...);
}
}  // namespace

cudaError_t tc_init(int num_sms) {
  cudaError_t e = cudaFuncSetAttribute(tc_pair_kernel<kGateUp>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(tc_pair_kernel<kDown>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTcSmem);
  if (e != cudaSuccess) return e;
  // Persistent grid: as many pairs as can be co-resident (at most one CTA per SM).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (num_sms / 2));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, tc_pair_kernel<kGateUp>, &cfg);
  if (e != cudaSuccess) return e;
  g_pairs = n > 0 ? n : 1;
  return cudaSuccess;
}

bool tc_supported(const Dims& d) {
  return d.H % 256 == 0 && d.H <= 256 * kGatherMaxH8 && d.I % 128 == 0 && d.Is % 128 == 0 &&
         d.E <= 511;
}

cudaError_t launch_tc_experts(const Dims& d, const __nv_bfloat16* x,
                              const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                              const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                              const __nv_bfloat16* w_sh_down, const Workspace& ws,
                              const __nv_bfloat16* resid, __nv_bfloat16* y, int lo, int hi,
                              int with_shared, int with_routed, int rank, int world,
                              cudaStream_t st, void* const events[3],
                              const RowsOut* rows_out) {
  // events (each may be null): before gate_up, after gate_up, after down
  auto mark = [&](int i) {
    return events[i] ? cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st) : cudaSuccess;
  };
  const uint64_t H = d.H, I = d.I, Is = d.Is, E = d.E, T = d.T;
  const uint64_t P = T * d.K, R = P + T, ldh = d.ldh;
  CUtensorMap tm_gu, tm_sg, tm_su, tm_dn, tm_sd, tm_h, tm_h32, tm_xp, tm_xp32, tm_x, tm_x32;
  // gate_up weights [E][2I][H] seen as (k, row in group, gate|up, group, expert):
  // one box = 4 groups of 16 gate rows, each followed by its 16 up rows.
  const uint64_t gu_dims[5] = {H, 16, 2, I / 16, E};
  const uint64_t gu_strides[4] = {H * 2, I * H * 2, 16 * H * 2, 2 * I * H * 2};
  const uint32_t gu_box[5] = {kBK, 16, 2, 4, 1};
  if (!make_tmap_bf16_nd(&tm_gu, w_gate_up, 5, gu_dims, gu_strides, gu_box) ||
      !make_tmap_bf16_2d(&tm_sg, w_sh_gate, H, Is, H * 2, kBK, 16) ||
      !make_tmap_bf16_2d(&tm_su, w_sh_up, H, Is, H * 2, kBK, 16) ||
      !make_tmap_bf16_2d(&tm_dn, w_down, I, E * H, I * 2, kBK, kBM) ||
      !make_tmap_bf16_2d(&tm_sd, w_sh_down, Is, H, Is * 2, kBK, kBM) ||
      !make_tmap_bf16_2d(&tm_h, ws.h, ldh, R, ldh * 2, kBK, kHalfTok) ||
      !make_tmap_bf16_2d(&tm_h32, ws.h, ldh, R, ldh * 2, kBK, kRowChunk) ||
      !make_tmap_bf16_2d(&tm_xp, ws.x_perm, H, R, H * 2, kBK, kHalfTok) ||
      !make_tmap_bf16_2d(&tm_xp32, ws.x_perm, H, R, H * 2, kBK, kRowChunk) ||
      !make_tmap_bf16_2d(&tm_x, x, H, T, H * 2, kBK, kHalfTok) ||
      !make_tmap_bf16_2d(&tm_x32, x, H, T, H * 2, kBK, kRowChunk))
    return cudaErrorInvalidValue;
  plan_tiles_kernel<<<1, kPlanThreads, 0, st>>>(ws.offsets, ws.active, ws.n_active, d.E, d.H,
                                                d.I, d.Is, rank, world, split_c0(),
                                                ws.gu_tiles,
                                                ws.dn_tiles, ws.m_tiles, ws.tile_counts);
  gather_rows_kernel<<<2 * g_pairs * 16, kGatherThreads, 0, st>>>(
      x, ws.m_tiles, ws.tile_counts + 2, ws.sorted_tok, d.H, d.E, ws.x_perm);
  cudaError_t err = mark(0);
  if (err != cudaSuccess) return err;
  int* status = ws.status + 1;
  // Shared gate and up rows as one 5-D map like the routed experts' (one
  // 16 KiB box per stage instead of eight 2 KiB ones) when the two tensors'
  // distance is a legal stride; the half at the lower address comes first.
  int sh5 = 0, sh_swap = 0;
  {
    const char* g = reinterpret_cast<const char*>(w_sh_gate);
    const char* u = reinterpret_cast<const char*>(w_sh_up);
    const uint64_t dist = uint64_t(u > g ? u - g : g - u);
    if (dist != 0 && dist % 16 == 0 && dist < (uint64_t(1) << 40) && Is % 64 == 0) {
      const uint64_t sh_dims[5] = {H, 16, 2, Is / 16, 1};
      const uint64_t sh_strides[4] = {H * 2, dist, 16 * H * 2, Is * H * 2};
      CUtensorMap m;
      if (make_tmap_bf16_nd(&m, u > g ? g : u, 5, sh_dims, sh_strides, gu_box)) {
        tm_sg = m;
        sh5 = 1;
        sh_swap = u < g ? 1 : 0;
      }
    }
  }
  TileTables gu{ws.gu_tiles, ws.tile_counts, ws.pair_dst, ws.pair_w, RowsOut{}, d.T, d.K,
                d.sh_lo, sh5, sh_swap};
  TileTables dn{ws.dn_tiles, ws.tile_counts + 1, ws.pair_dst, ws.pair_w,
                rows_out ? *rows_out : RowsOut{}, d.T, d.K, d.sh_lo, 0, 0};
  err = launch_pairs<kGateUp>(st, tm_gu, tm_sg, tm_su, tm_xp, tm_xp32, tm_x, tm_x32, gu, d.H, d.E,
                              d.I, d.Is, d.ldh, ws.h, ws.rows_bf16, status);
  if (err != cudaSuccess) return err;
  err = mark(1);
  if (err != cudaSuccess) return err;
  err = launch_pairs<kDown>(st, tm_dn, tm_sd, tm_sd, tm_h, tm_h32, tm_h, tm_h32, dn, d.H, d.E,
                            d.I, d.Is, d.ldh, ws.h, ws.rows_bf16, status);
  if (err != cudaSuccess) return err;
  err = mark(2);
  if (err != cudaSuccess) return err;
  if (rows_out && rows_out->world > 0) return cudaSuccess;  // the token owners combine
  const long n8 = long(T) * d.H / 8;
  const int* pp = world > 1 ? ws.pair_pos : nullptr;
  if (d.K <= kCombineMaxK && d.H / 8 <= 256) {
    const unsigned threads = unsigned((d.H / 8 + 31) / 32 * 32);
    const unsigned blocks = unsigned(std::min<long>(T, long(2 * g_pairs) * 4));  // one wave
    combine_rows_tok_kernel<<<blocks, threads, 0, st>>>(
        ws.rows_bf16, ws.topk_idx, ws.topk_w, ws.shared_gate, d.T, d.H, d.K, lo, hi, with_shared,
        with_routed, d.sh_lo, d.sh_hi, pp, ws.tile_counts + 4, resid, y, 0, d.T, RowsOut{},
        nullptr);
    return cudaGetLastError();
  }
  combine_rows_kernel<<<unsigned((n8 + 255) / 256), 256, 0, st>>>(
      ws.rows_bf16, ws.topk_idx, ws.topk_w, ws.shared_gate, d.T, d.H, d.K, lo, hi, with_shared,
      with_routed, d.sh_lo, d.sh_hi, world > 1 ? ws.pair_pos : nullptr, ws.tile_counts + 4,
      resid, y);
  return cudaGetLastError();
}

// Combine of tokens [t_lo, t_hi) from a complete token-major rows buffer
// (every routed expert and the shared expert), y indexed by token.
cudaError_t launch_combine_slice(const __nv_bfloat16* rows, const int32_t* topk_idx,
                                 const float* topk_w, const float* shared_gate, int T, int H,
                                 int E, int K, int t_lo, int t_hi, __nv_bfloat16* y,
                                 const RowsOut* ydst, const int* abort_if, cudaStream_t st) {
  if (K > kCombineMaxK || H / 8 > 256) return cudaErrorInvalidValue;
  if (t_hi <= t_lo) return cudaSuccess;
  const unsigned threads = unsigned((H / 8 + 31) / 32 * 32);
  const unsigned blocks = unsigned(std::min<long>(t_hi - t_lo, long(2 * g_pairs) * 4));
  combine_rows_tok_kernel<<<blocks, threads, 0, st>>>(rows, topk_idx, topk_w, shared_gate, T, H,
                                                      K, 0, E, 1, 1, 0, T, nullptr, nullptr,
                                                      nullptr, y, t_lo, t_hi,
                                                      ydst ? *ydst : RowsOut{}, abort_if);
  return cudaGetLastError();
}

}  // namespace pmoe
