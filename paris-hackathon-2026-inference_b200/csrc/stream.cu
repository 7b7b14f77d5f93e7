// TMA-staged weight-streaming expert kernels for the HBM-bound decode regime.
//
// At T <= 64 each active expert sees a handful of tokens: the block is a
// stream over ~1.4 GB of expert weights at a few FLOP/B.  Each persistent
// CTA (one per SM) runs a warp-specialised pipeline:
//   * warp 0, one lane: producer.  Takes work units from a global atomic
//     queue (heaviest first: the shared expert sees every token), publishes
//     each to the consumers through a small mbarrier ring, and issues 2D TMA
//     loads (128-byte swizzle, L2 evict-first) of the unit's weight tiles --
//     KCH k-chunks of 64 columns per stage, so each weight row contributes
//     KCH*128 contiguous bytes per stage -- plus the matching slice of the
//     activation rows, into a ~200 KiB mbarrier ring;
//   * warps 1..4: consumers.  Each owns 16 weight rows of the tile, reads
//     its mma.sync A and B fragments from shared memory with 128-bit loads,
//     and releases the stage.
// That is gate_up (96-97 % of the HBM copy rate).  The down projection, whose
// per-stage work left the mma.sync consumers the limit, runs on the tcgen05
// tensor cores instead (down_tc_kernel: single-thread MMA issue from the
// staged tiles, accumulators in TMEM); down_tma_kernel is kept for shapes it
// does not take.
// Every weight byte is loaded from HBM exactly once per call.
//
// Reference arithmetic: the per-expert body of Qwen3_5MoeExperts.forward
// (modeling_qwen3_5_moe.py:743-749), the shared expert Qwen3_5MoeMLP
// (:709-711) with its sigmoid gate (:788), and the routed combine of
// engine/kernels/moe_grouped_mlp.py:152-163 (done here in fp32).
#include <cstdlib>

#include "pmoe_common.cuh"
#include "pmoe_kernels.cuh"
#include "pmoe_tma.cuh"
#include "pmoe_tc.cuh"

namespace pmoe {

struct ExpertTables {
  const int32_t* active;
  const int32_t* n_active;
  const int32_t* offsets;  // [E+2]
  const int32_t* sorted_tok;
  const int32_t* pair_dst;
  const float* pair_w;
};

constexpr int kConsumers = 4;
constexpr int kStreamThreads = 32 * (kConsumers + 1);
constexpr int kUnitRows = 16 * kConsumers;      // 64 weight rows per tile
constexpr int kKC = 64;                         // k per tile chunk (128-byte rows)
constexpr int kBoxBytes = kUnitRows * kKC * 2;  // 8 KiB weight tile chunk
constexpr int kActRows = 32;                    // dispatched rows per pass
constexpr int kActChunkBytes = kActRows * kKC * 2;  // 4 KiB activation chunk
constexpr int kRingBudget = 200 * 1024;
constexpr int kUnitSlots = 4;
constexpr int kDnRowBlocks = 8;  // down unit = 8 x 64 output rows (4: 99.9 us, 8: 98.4, 16: 117.8)
// down: eight consumer warps, two per 16-row slice, each on half of a
// stage's k-chunks (shorter dependent MMA chains), partial sums added
// through shared memory
constexpr int kDnConsumers = 8;
constexpr int kDnThreads = 32 * (kDnConsumers + 1);

template <int KCH>
struct GuCfg {
  static constexpr int kStageBytes = KCH * (2 * kBoxBytes + kActChunkBytes);
  static constexpr int kStages = kRingBudget / kStageBytes > 16 ? 16 : kRingBudget / kStageBytes;
  static constexpr int kSmem = kStages * kStageBytes + 2 * kStages * 8 + 1024;
};
template <int KCH>
struct DnCfg {
  static constexpr int kActBytes = kActChunkBytes;
  static constexpr int kStageBytes = KCH * (kBoxBytes + kActBytes);
  static constexpr int kStages = kRingBudget / kStageBytes > 16 ? 16 : kRingBudget / kStageBytes;
  static constexpr int kSmem = kStages * kStageBytes + 2 * kStages * 8 + 1024;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void set_status(int* status, int code) { atomicCAS(status, 0, code); }

// Producer drain after an abort: wait (bounded) for every issued, not yet
// consumed stage so no bulk copy is still writing this CTA's shared memory.
__device__ __forceinline__ void drain(uint64_t* full, uint32_t issued, int stages) {
  const uint32_t first = issued > uint32_t(stages) ? issued - stages : 0;
  for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % stages], (j / stages) & 1);
}

// Work-unit hand-off from the producer lane to the consumer warps.
struct UnitRing {
  uint64_t full[kUnitSlots];
  uint64_t empty[kUnitSlots];
  int unit[kUnitSlots];
  int4 info[kUnitSlots];  // optional per-unit facts the producer already loaded

  __device__ void init(int consumers = kConsumers) {
    for (int i = 0; i < kUnitSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], consumers);
    }
  }
  // Next unit from the global queue, heaviest (last) first; -1 = done.
  __device__ static int ticket(int* queue, int n_units) {
    const int q = atomicAdd(queue, 1);
    return q < n_units ? n_units - 1 - q : -1;
  }
  // Producer: hand unit `u` to the consumers in hand-off `ui`.
  __device__ bool publish_unit(uint32_t ui, int u, int4 inf = make_int4(0, 0, 0, 0)) {
    const int slot = ui % kUnitSlots;
    if (ui >= uint32_t(kUnitSlots) && !mbar_wait(&empty[slot], ((ui / kUnitSlots) & 1) ^ 1))
      return false;
    unit[slot] = u;
    info[slot] = inf;
    mbar_arrive(&full[slot]);
    return true;
  }
  __device__ bool publish(uint32_t ui, int* queue, int n_units, int* out_unit) {
    *out_unit = ticket(queue, n_units);
    return publish_unit(ui, *out_unit);
  }
  // Consumer warp: unit published in hand-off `ui`.
  __device__ bool take(uint32_t ui, int lane, int* out_unit, int4* out_info = nullptr) {
    const int slot = ui % kUnitSlots;
    if (!mbar_wait(&full[slot], (ui / kUnitSlots) & 1)) return false;
    const int u = unit[slot];
    const int4 inf = info[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    *out_unit = u;
    if (out_info) *out_info = inf;
    return true;
  }
};

// ---------------------------------------------------------------------------
// gate_up + SiLU*mul.  Unit = (expert, 64 intermediate columns j): the gate
// rows j.. and the up rows I+j.. of that expert (shared expert: its own two
// weight matrices).  A stage holds KCH 64x64 gate and up tile chunks
// (swizzled) and the same KCH*64 k of the pass's (up to 32) gathered token
// rows of x (one unswizzled TMA row each), all landed on one mbarrier.
// h[row, j] = bf16(silu(x.Wg_j) * (x.Wu_j)).
// ---------------------------------------------------------------------------
template <int KCH>
__global__ void __launch_bounds__(kStreamThreads, 1) gate_up_tma_kernel(
    const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_sg,
    const __grid_constant__ CUtensorMap tm_su, const __grid_constant__ CUtensorMap tm_x,
    ExpertTables tb, int H, int E, int I, int Is, int ldh, __nv_bfloat16* __restrict__ h,
    int* __restrict__ status, int* __restrict__ queue) {
  using C = GuCfg<KCH>;
  constexpr int kStages = C::kStages;
  constexpr int kXRow = KCH * kKC * 2;  // bytes of one staged x row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::kStageBytes);
  uint64_t* empty = full + kStages;
  __shared__ int s_tok[kActRows];
  __shared__ UnitRing ur;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    ur.init();
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the routing tables
  const int UJ = (I > Is ? I : Is) / kUnitRows;
  const int n_units = tb.n_active[0] * UJ;
  const int nkc = H / (kKC * KCH);

  if (warp == 0) {
    if (lane != 0) return;
    prefetch_tmap(&tm_gu);
    prefetch_tmap(&tm_sg);
    prefetch_tmap(&tm_su);
    prefetch_tmap(&tm_x);
    const uint64_t pol = l2_policy_evict_first();
    uint32_t it = 0;
    int u_next = ur.ticket(queue, n_units);  // prefetched queue ticket
    for (uint32_t ui = 0;; ++ui) {
      const int u = u_next;
      if (!ur.publish_unit(ui, u)) {
        set_status(status, kStatusTimeoutEmpty);
        drain(full, it, kStages);
        return;
      }
      if (u < 0) break;
      u_next = ur.ticket(queue, n_units);
      const int e = tb.active[u / UJ], jb = u % UJ;
      const bool sh = (e == E);
      if (jb * kUnitRows >= (sh ? Is : I)) continue;
      const int p0 = tb.offsets[e];
      const int n = tb.offsets[e + 1] - p0;
      const CUtensorMap* mg = sh ? &tm_sg : &tm_gu;
      const CUtensorMap* mu = sh ? &tm_su : &tm_gu;
      const int rg = sh ? jb * kUnitRows : e * 2 * I + jb * kUnitRows;
      const int ru = sh ? jb * kUnitRows : e * 2 * I + I + jb * kUnitRows;
      for (int nb = 0; nb < n; nb += kActRows) {
        const int nr = min(kActRows, n - nb);
        for (int i = 0; i < nr; ++i) s_tok[i] = tb.sorted_tok[p0 + nb + i];
        for (int kc = 0; kc < nkc; ++kc, ++it) {
          const int s = it % kStages;
          if (it >= uint32_t(kStages) && !mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1)) {
            set_status(status, kStatusTimeoutEmpty);
            drain(full, it, kStages);
            return;
          }
          mbar_arrive_expect_tx(&full[s], KCH * 2 * kBoxBytes + nr * kXRow);
          uint8_t* dst = smem + s * C::kStageBytes;
#pragma unroll
          for (int j = 0; j < KCH; ++j) {
            const int k = (kc * KCH + j) * kKC;
            tma_load_2d_hint(dst + j * kBoxBytes, mg, k, rg, &full[s], pol);
            tma_load_2d_hint(dst + (KCH + j) * kBoxBytes, mu, k, ru, &full[s], pol);
          }
          uint8_t* xd = dst + 2 * KCH * kBoxBytes;
          for (int i = 0; i < nr; ++i)
            tma_load_2d(xd + i * kXRow, &tm_x, kc * KCH * kKC, s_tok[i], &full[s]);
        }
      }
    }
    return;
  }

  // consumers
  const int cw = warp - 1, g = lane >> 2, c = lane & 3;
  const int r0 = cw * 16 + g, r1 = r0 + 8;
  const uint32_t sbase = smem_u32(smem);
  uint32_t it = 0;
  for (uint32_t ui = 0;; ++ui) {
    int u;
    if (!ur.take(ui, lane, &u)) {
      set_status(status, kStatusTimeoutFull);
      return;
    }
    if (u < 0) break;
    const int e = tb.active[u / UJ], jb = u % UJ;
    const bool sh = (e == E);
    if (jb * kUnitRows >= (sh ? Is : I)) continue;
    const int p0 = tb.offsets[e];
    const int n = tb.offsets[e + 1] - p0;
    for (int nb = 0; nb < n; nb += kActRows) {
      const int ng = min(4, (n - nb + 7) / 8);  // warp-uniform
      float ag[4][4] = {}, au[4][4] = {};
      for (int kc = 0; kc < nkc; ++kc, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1)) {
          set_status(status, kStatusTimeoutFull);
          return;
        }
        const uint32_t st0 = sbase + s * C::kStageBytes;
        const uint32_t tx = st0 + 2 * KCH * kBoxBytes;
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
          const uint32_t tg = st0 + j * kBoxBytes, tu = st0 + (KCH + j) * kBoxBytes;
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const int ch = ks * 4 + c;
            const uint4 a0 = lds128(tg + swz128(r0, ch)), a1 = lds128(tg + swz128(r1, ch));
            const uint4 b0 = lds128(tu + swz128(r0, ch)), b1 = lds128(tu + swz128(r1, ch));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (q < ng) {
                const uint4 xv = lds128(tx + uint32_t((q * 8 + g) * kXRow + j * 128 + ch * 16));
                mma_k32(ag[q], a0, a1, xv);
                mma_k32(au[q], b0, b1, xv);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // rows j = jb*64 + r0 (+8), columns = dispatched rows p0+nb+q*8+2c (+1)
      const int j0 = jb * kUnitRows + r0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < ng) {
          const int i = nb + q * 8 + 2 * c;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (i + hh < n) {
              __nv_bfloat16* hrow = h + size_t(p0 + i + hh) * ldh;
              hrow[j0] = __float2bfloat16_rn(silu_f(ag[q][hh]) * au[q][hh]);
              hrow[j0 + 8] = __float2bfloat16_rn(silu_f(ag[q][2 + hh]) * au[q][2 + hh]);
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// down + routing weight.  Unit = (expert, 64 output rows of down_proj).  A
// stage holds KCH 64x64 weight tile chunks and the same k of the pass's 32
// dispatched rows of h (one swizzled box per chunk; rows past the end of h
// read as zero).  rows[pair_dst[p], r] = pair_w[p] * (h[p] . Wd_r).
// ---------------------------------------------------------------------------
template <int KCH>
__global__ void __launch_bounds__(kDnThreads, 1) down_tma_kernel(
    const __grid_constant__ CUtensorMap tm_dn, const __grid_constant__ CUtensorMap tm_sd,
    const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_h8,
    ExpertTables tb, int H, int E, int I, int Is,
    float* __restrict__ rows, int* __restrict__ status, int* __restrict__ queue, EpPeers ep,
    int row_blocks) {
  using C = DnCfg<KCH>;
  constexpr int AR = kActRows;
  constexpr int kGroups = AR / 8;
  const int epoch = ep.world > 0 ? ep_epoch(ep) : 0;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::kStageBytes);
  uint64_t* empty = full + kStages;
  __shared__ UnitRing ur;
  __shared__ float s_part[2][4][32][16];  // partial accumulators of the upper-k warps, by parity
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDnConsumers);
    }
    ur.init(kDnConsumers);
    mbar_fence_init();
  }
  __syncthreads();
  const int UR = H / (kUnitRows * row_blocks);
  const int n_units = tb.n_active[0] * UR;

  if (warp == 0) {
    if (lane != 0) return;
    prefetch_tmap(&tm_dn);
    prefetch_tmap(&tm_sd);
    prefetch_tmap(&tm_h);
    prefetch_tmap(&tm_h8);
    const uint64_t pol = l2_policy_evict_first();
    uint32_t it = 0;
    // The next unit's ticket is taken while this unit's stages are issued, so
    // the queue's atomic round trip is off the producer's critical path.
    int u_next = ur.ticket(queue, n_units);
    for (uint32_t ui = 0;; ++ui) {
      const int u = u_next;
      // the unit's expert and rows go to the consumers with the unit, so they
      // do not repeat these dependent global loads
      int e = 0, p0 = 0, n = 0;
      if (u >= 0) {
        e = tb.active[u / UR];
        p0 = tb.offsets[e];
        n = tb.offsets[e + 1] - p0;
      }
      if (!ur.publish_unit(ui, u, make_int4(e, p0, n, 0))) {
        set_status(status, kStatusTimeoutEmpty);
        drain(full, it, kStages);
        return;
      }
      if (u < 0) break;
      u_next = ur.ticket(queue, n_units);
      const int rbg = u % UR;
      const bool sh = (e == E);
      const int nkc = (sh ? Is : I) / (kKC * KCH);
      const CUtensorMap* m = sh ? &tm_sd : &tm_dn;
      // passes of up to 32 dispatched rows, each over the unit's row blocks
      for (int nb = 0; nb < n; nb += AR) {
      for (int sub = 0; sub < row_blocks; ++sub) {
        const int rb = rbg * row_blocks + sub;
        const int row = sh ? rb * kUnitRows : e * H + rb * kUnitRows;
        // passes of at most 8 rows load an 8-row activation box (1 KiB/chunk)
        const bool small = n - nb <= 8;
        const CUtensorMap* mh = small ? &tm_h8 : &tm_h;
        const uint32_t hbytes = small ? 8 * kKC * 2 : C::kActBytes;
        for (int kc = 0; kc < nkc; ++kc, ++it) {
          const int s = it % kStages;
          if (it >= uint32_t(kStages) && !mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1)) {
            set_status(status, kStatusTimeoutEmpty);
            drain(full, it, kStages);
            return;
          }
          mbar_arrive_expect_tx(&full[s], KCH * (kBoxBytes + hbytes));
          uint8_t* dst = smem + s * C::kStageBytes;
#pragma unroll
          for (int j = 0; j < KCH; ++j) {
            const int k = (kc * KCH + j) * kKC;
            tma_load_2d_hint(dst + j * kBoxBytes, m, k, row, &full[s], pol);
            tma_load_2d(dst + KCH * kBoxBytes + j * C::kActBytes, mh, k, p0 + nb, &full[s]);
          }
        }
      }
      }  // nb
    }
    return;
  }

  // consumer warp cw: rows slice rq (16 rows), k half kh of every stage
  const int cw = warp - 1, rq = cw & 3, kh = cw >> 2, g = lane >> 2, c = lane & 3;
  // Fragment row / token g of the MMA is weight row (and token) gp = pi(g),
  // pi = 0,4,1,5,2,6,3,7: the two rows a quarter-warp reads then differ in
  // bit 2, so their four 16-byte chunks land in opposite halves of the
  // 128-byte swizzle pattern (no bank conflict; adjacent rows collide).
  const int gp = (g >> 1) | ((g & 1) << 2);
  const int r0 = rq * 16 + gp, r1 = r0 + 8;
  const uint32_t sbase = smem_u32(smem);
  uint32_t it = 0, blk = 0;
  for (uint32_t ui = 0;; ++ui) {
    int u;
    int4 inf;
    if (!ur.take(ui, lane, &u, &inf)) {
      set_status(status, kStatusTimeoutFull);
      return;
    }
    if (u < 0) break;
    const int e = inf.x, p0 = inf.y, n = inf.z, rbg = u % UR;
    const bool sh = (e == E);
    const int nkc = (sh ? Is : I) / (kKC * KCH);
    for (int nb = 0; nb < n; nb += AR) {
    const int ng = min(kGroups, (n - nb + 7) / 8);
    // this lane's output rows of the pass (weight, destination), loaded once
    // for all of the unit's row blocks, before the first stage wait
    float wt[4][2];
    int dsti[4][2];
#pragma unroll
    for (int q = 0; q < kGroups; ++q)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = nb + q * 8 + c + 4 * hh;  // token of accumulator column 2c + hh
        const bool ok = kh == 0 && q < ng && i < n;
        wt[q][hh] = ok ? tb.pair_w[p0 + i] : 0.f;
        dsti[q][hh] = ok ? tb.pair_dst[p0 + i] : -1;
      }
    for (int sub = 0; sub < row_blocks; ++sub, ++blk) {
      const int rb = rbg * row_blocks + sub;
      float acc[4][4] = {};
      for (int kc = 0; kc < nkc; ++kc, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1)) {
          set_status(status, kStatusTimeoutFull);
          return;
        }
        const uint32_t st0 = sbase + s * C::kStageBytes;
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
          if (KCH > 1 && (2 * j) / KCH != kh) continue;  // the other warp's half
          if (KCH == 1 && kh != 0) continue;
          const uint32_t tw = st0 + j * kBoxBytes;
          const uint32_t th = st0 + KCH * kBoxBytes + j * C::kActBytes;
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const int ch = ks * 4 + c;
            const uint4 a0 = lds128(tw + swz128(r0, ch)), a1 = lds128(tw + swz128(r1, ch));
#pragma unroll
            for (int q = 0; q < kGroups; ++q) {
              if (q < ng) {
                const uint4 hv = lds128(th + swz128(q * 8 + gp, ch));
                mma_k32(acc[q], a0, a1, hv);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // the upper-k warp hands its partial sums to its partner through
      // shared memory (two parities: the partner reads slot p before it
      // arrives at the next row block's barrier)
      float* slot = &s_part[blk & 1][rq][lane][0];
      if (kh == 1) {
#pragma unroll
        for (int q = 0; q < kGroups; ++q)
#pragma unroll
          for (int i = 0; i < 4; ++i) slot[q * 4 + i] = acc[q][i];
      }
      named_bar_sync(1 + rq, 64);
      if (kh == 1) continue;
#pragma unroll
      for (int q = 0; q < kGroups; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[q][i] += slot[q * 4 + i];
      const int orow = rb * kUnitRows + r0;
#pragma unroll
      for (int q = 0; q < kGroups; ++q) {
        if (q < ng) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (dsti[q][hh] >= 0) {
              const float wk = wt[q][hh];
              const size_t off = size_t(dsti[q][hh]) * H;
              const float v0 = acc[q][hh] * wk, v1 = acc[q][2 + hh] * wk;
              if (ep.world > 0) {
                // every computed row goes to every rank (peer stores over NVLink)
                for (int rr = 0; rr < ep.world; ++rr) {
                  float* out = ep_rows(ep, rr, epoch) + off;
                  out[orow] = v0;
                  out[orow + 8] = v1;
                }
              } else {
                float* out = rows + off;
                out[orow] = v0;
                out[orow + 8] = v1;
              }
            }
          }
        }
      }
    }
    }  // nb
  }
  if (ep.world > 0) {
    // All of this warp's peer stores are made visible system-wide before it
    // takes a ticket; the last consumer warp of the grid releases the flags.
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
      const int prev = atomicAdd(ep.ticket, 1);
      if (prev == int(gridDim.x) * kDnConsumers - 1) {
        __threadfence_system();
        *ep.ticket = 0;
        for (int rr = 0; rr < ep.world; ++rr) st_release_sys(ep.flags[rr] + ep.rank, epoch);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// down + routing weight on the tcgen05 tensor cores (the decode default).
// Unit = (expert, row_blocks x 128 output rows of down_proj).  A stage holds
// one 128-row x 64-k weight box and the same k of the pass's 16 dispatched
// rows of h (128-byte swizzle; rows past the end of h read as zero), so one
// stage is four M128 x N16 x K16 MMAs issued by a single thread; the fp32
// accumulator of a row block (128 TMEM lanes x 16 columns) has four TMEM
// buffers, so remote stores in the epilogue do not hold up the MMAs.  Roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-9 epilogue (TMEM lane quadrant warp % 4, token columns 0-7 or 8-15
// by warp / 6): each lane owns one output row, so every store of a token's 32
// rows is one 128-byte segment.
// The mma.sync version (down_tma_kernel) was bound by the legacy MMA
// instruction rate, not by HBM.
// rows[pair_dst[p], r] = pair_w[p] * (h[p] . Wd_r).
// ---------------------------------------------------------------------------
constexpr int kDtRows = 128;                          // weight rows per MMA (TMEM lanes)
constexpr int kDtTok = 16;                            // dispatched rows per pass (MMA N)
constexpr int kDtWBytes = kDtRows * kKC * 2;          // 16 KiB weight box
constexpr int kDtHBytes = kDtTok * kKC * 2;           // 2 KiB activation box
constexpr int kDtStageBytes = kDtWBytes + kDtHBytes;  // 18 KiB, a multiple of 1 KiB
constexpr int kDtStages = 12;                         // 216 KiB ring
constexpr int kDtEpiWarps = 8;   // two per TMEM lane quadrant, each on half the tokens
constexpr int kDtAcc = 4;        // accumulators in flight (TMEM, 16 columns each)
constexpr int kDtThreads = 32 * (2 + kDtEpiWarps);
constexpr int kDtBarBytes = 512;
constexpr int kDtSmem = kDtStages * kDtStageBytes + kDtBarBytes + 1024;
constexpr uint32_t kDtTmemCols = kDtAcc * kDtTok;    // 64 columns
static_assert(kDtStageBytes % 1024 == 0, "stages keep the 1 KiB swizzle alignment");
static_assert((2 * kDtStages + 2 * kDtAcc + 1) * 8 + 4 <= kDtBarBytes, "barrier area");
static_assert(kDtSmem <= 227 * 1024, "shared memory");

__global__ void __launch_bounds__(kDtThreads, 1) down_tc_kernel(
    const __grid_constant__ CUtensorMap tm_dn, const __grid_constant__ CUtensorMap tm_sd,
    const __grid_constant__ CUtensorMap tm_h, ExpertTables tb, int H, int E, int I, int Is,
    float* __restrict__ rows, int* __restrict__ status, int* __restrict__ queue, EpPeers ep,
    int row_blocks) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDtStages * kDtStageBytes);
  uint64_t* empty = full + kDtStages;
  uint64_t* tfull = empty + kDtStages;
  uint64_t* tempty = tfull + kDtAcc;
  uint64_t* done = tempty + kDtAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ UnitRing ur;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kDtAcc; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kDtEpiWarps);
    }
    mbar_init(done, 1);
    ur.init(1 + kDtEpiWarps);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kDtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // h and the routing tables of the kernels before
  const int epoch = ep.world > 0 ? ep_epoch(ep) : 0;
  const uint32_t tmem_base = *tmem_slot;
  const int UR = H / (kDtRows * row_blocks);
  const int n_units = tb.n_active[0] * UR;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_dn);
      prefetch_tmap(&tm_sd);
      prefetch_tmap(&tm_h);
      const uint64_t pol = l2_policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      int u_next = ur.ticket(queue, n_units);
      for (uint32_t ui = 0; ok; ++ui) {
        const int u = u_next;
        int e = 0, p0 = 0, n = 0;
        if (u >= 0) {
          e = tb.active[u / UR];
          p0 = tb.offsets[e];
          n = tb.offsets[e + 1] - p0;
        }
        if (!ur.publish_unit(ui, u, make_int4(e, p0, n, 0))) {
          set_status(status, kStatusTimeoutEmpty);
          break;
        }
        if (u < 0) break;
        u_next = ur.ticket(queue, n_units);
        const bool sh = (e == E);
        const int nkc = (sh ? Is : I) / kKC;
        const CUtensorMap* m = sh ? &tm_sd : &tm_dn;
        // a unit read in several passes keeps its weights in L2 for the next
        const bool reread = n > kDtTok;
        for (int nb = 0; nb < n && ok; nb += kDtTok) {
          for (int sub = 0; sub < row_blocks && ok; ++sub) {
            const int rb = (u % UR) * row_blocks + sub;
            const int row = sh ? rb * kDtRows : e * H + rb * kDtRows;
            for (int kc = 0; kc < nkc; ++kc, ++it) {
              const int s = it % kDtStages;
              if (it >= uint32_t(kDtStages) &&
                  !mbar_wait(&empty[s], ((it / kDtStages) & 1) ^ 1)) {
                set_status(status, kStatusTimeoutEmpty);
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full[s], kDtStageBytes);
              uint8_t* dst = smem + s * kDtStageBytes;
              if (reread)
                tma_load_2d(dst, m, kc * kKC, row, &full[s]);
              else
                tma_load_2d_hint(dst, m, kc * kKC, row, &full[s], pol);
              tma_load_2d(dst + kDtWBytes, &tm_h, kc * kKC, p0 + nb, &full[s]);
            }
          }
        }
      }
      if (!ok) drain(full, it, kDtStages);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_bf16_f32(kDtRows, kDtTok);
    const uint32_t sbase = smem_u32(smem);
    uint32_t it = 0, acc = 0;
    bool ok = true;
    for (uint32_t ui = 0; ok; ++ui) {
      int u;
      int4 inf;
      if (!ur.take(ui, lane, &u, &inf)) {
        set_status(status, kStatusTimeoutFull);
        break;
      }
      if (u < 0) break;
      const int n = inf.z;
      const int nkc = (inf.x == E ? Is : I) / kKC;
      for (int nb = 0; nb < n && ok; nb += kDtTok) {
        for (int sub = 0; sub < row_blocks && ok; ++sub, ++acc) {
          const uint32_t b = acc % kDtAcc, use = acc / kDtAcc;
          if (acc >= uint32_t(kDtAcc) && !mbar_wait(&tempty[b], (use - 1) & 1)) {
            set_status(status, kStatusTimeoutTmem);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + b * kDtTok;
          for (int kc = 0; kc < nkc; ++kc, ++it) {
            const int s = it % kDtStages;
            if (!mbar_wait(&full[s], (it / kDtStages) & 1)) {
              set_status(status, kStatusTimeoutFull);
              ok = false;
              break;
            }
            tc_fence_after();
            if (lane == 0) {
              const uint32_t st = sbase + s * kDtStageBytes;
              const uint64_t wd = sdesc_k_sw128(st), hd = sdesc_k_sw128(st + kDtWBytes);
#pragma unroll
              for (int kk = 0; kk < kKC / 16; ++kk)
                umma_bf16(d, wd + uint64_t(kk * 2), hd + uint64_t(kk * 2), idesc,
                          (kc | kk) != 0 ? 1u : 0u);
              umma_commit(&empty[s]);
            }
            __syncwarp();
          }
          if (!ok) break;
          if (lane == 0) umma_commit(&tfull[b]);
          __syncwarp();
        }
      }
    }
    // every MMA has completed before the TMEM is freed
    if (lane == 0) umma_commit(done);
    __syncwarp();
    mbar_wait(done, 0);
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;            // TMEM lanes 32q .. 32q+31
    const int th = (warp - 2) >> 2;    // token columns th*8 .. th*8+7
    uint32_t acc = 0;
    bool ok = true;
    for (uint32_t ui = 0; ok; ++ui) {
      int u;
      int4 inf;
      if (!ur.take(ui, lane, &u, &inf)) {
        set_status(status, kStatusTimeoutFull);
        ok = false;
        break;
      }
      if (u < 0) break;
      const int p0 = inf.y, n = inf.z;
      for (int nb = 0; nb < n && ok; nb += kDtTok) {
        // lane t < 16: destination row and weight of the pass's token t
        const int nt = min(kDtTok, n - nb);
        int my_dst = -1;
        float my_w = 0.f;
        if (lane < nt) {
          my_dst = tb.pair_dst[p0 + nb + lane];
          my_w = tb.pair_w[p0 + nb + lane];
        }
        for (int sub = 0; sub < row_blocks; ++sub, ++acc) {
          const uint32_t b = acc % kDtAcc, use = acc / kDtAcc;
          if (!mbar_wait(&tfull[b], use & 1)) {
            set_status(status, kStatusTimeoutTmem);
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t v[8];
          tmem_ld8(tmem_base + (uint32_t(q * 32) << 16) + b * kDtTok + th * 8, v);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[b]);
          const int row = ((u % UR) * row_blocks + sub) * kDtRows + q * 32 + lane;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int t = th * 8 + i;
            if (t < nt) {
              const int dst = __shfl_sync(0xffffffffu, my_dst, t);
              const float val = __uint_as_float(v[i]) * __shfl_sync(0xffffffffu, my_w, t);
              const size_t off = size_t(dst) * H + row;
              if (ep.world > 0) {
                // every computed row goes to every rank (peer stores over NVLink)
                for (int rr = 0; rr < ep.world; ++rr) ep_rows(ep, rr, epoch)[off] = val;
              } else {
                rows[off] = val;
              }
            }
          }
        }
      }
    }
    if (ok && ep.world > 0) {
      // All of this warp's peer stores are made visible system-wide before it
      // takes a ticket; the last epilogue warp of the grid releases the flags.
      __threadfence_system();
      __syncwarp();
      if (lane == 0) {
        const int prev = atomicAdd(ep.ticket, 1);
        if (prev == int(gridDim.x) * kDtEpiWarps - 1) {
          __threadfence_system();
          *ep.ticket = 0;
          for (int rr = 0; rr < ep.world; ++rr) st_release_sys(ep.flags[rr] + ep.rank, epoch);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kDtTmemCols);
  }
}

// y[t, :] = bf16( sum_{s<K, expert in [lo,hi)} rows[t*K+s, :] + rows[T*K+t, :] )
// fp32, fixed summation order.  One thread per 4 columns.  The shared row is
// added for tokens in [sh_lo, sh_hi).  With a residual (decoder layer),
// y = bf16(resid + bf16(sum)), the two roundings of `residual + mlp(x)` in
// bf16 (modeling_qwen3_5_moe.py:867-868).  With an expert-parallel exchange
// (world > 0) the rows are this call's parity copy of the exchange buffer and
// every block first waits, bounded, until all ranks' completion flags for
// this epoch are up.
constexpr int kCombMaxK = 8;  // top-k sizes up to this take the all-loads-in-flight path

__global__ void __launch_bounds__(256) combine_kernel(
    const float* __restrict__ rows, size_t par_stride, const int32_t* __restrict__ topk_idx,
    int T, int H, int K, int lo, int hi, int with_shared, int with_routed, int sh_lo, int sh_hi,
    const int* __restrict__ wait_flags, int world, const int* __restrict__ epoch_dev,
    int epoch_host, int* __restrict__ status, int* __restrict__ sticky,
    const __nv_bfloat16* __restrict__ resid, __nv_bfloat16* __restrict__ y) {
  pdl_wait();  // the expert rows
  const int epoch = epoch_dev ? *epoch_dev : epoch_host;
  if (world > 0) rows += size_t(epoch & 1) * par_stride;
  if (world > 0) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
      int ok = 1;
      const long long t0 = clock64();
      for (int r = 0; r < world && ok; ++r) {
        while (ld_acquire_sys(wait_flags + r) < epoch) {
          if (clock64() - t0 > kWaitBudgetCycles) {
            ok = 0;
            atomicCAS(status, 0, kStatusTimeoutPeer);
            if (sticky) atomicCAS(sticky, 0, kStatusTimeoutPeer);  // survives the next call
            break;
          }
        }
      }
      s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
  }
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const int cols4 = H / 4;
  if (i >= long(T) * cols4) return;
  const int t = int(i / cols4), c4 = int(i % cols4);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool sh_sel = with_shared && t >= sh_lo && t < sh_hi;
  if (K <= kCombMaxK) {
    // select, then issue all selected row loads before the fixed-order sum
    bool sel[kCombMaxK];
    float4 v[kCombMaxK + 1];
#pragma unroll
    for (int k = 0; k < kCombMaxK; ++k) {
      sel[k] = false;
      if (k < K && with_routed) {
        const int e = topk_idx[size_t(t) * K + k];
        sel[k] = e >= lo && e < hi;
      }
    }
#pragma unroll
    for (int k = 0; k < kCombMaxK; ++k)
      if (sel[k]) v[k] = reinterpret_cast<const float4*>(rows + (size_t(t) * K + k) * H)[c4];
    if (sh_sel) v[kCombMaxK] = reinterpret_cast<const float4*>(rows + (size_t(T) * K + t) * H)[c4];
#pragma unroll
    for (int k = 0; k < kCombMaxK; ++k)
      if (sel[k]) {
        s.x += v[k].x; s.y += v[k].y; s.z += v[k].z; s.w += v[k].w;
      }
    if (sh_sel) {
      s.x += v[kCombMaxK].x; s.y += v[kCombMaxK].y; s.z += v[kCombMaxK].z; s.w += v[kCombMaxK].w;
    }
  } else {
    if (with_routed) {
      for (int k = 0; k < K; ++k) {
        const int e = topk_idx[size_t(t) * K + k];
        if (e < lo || e >= hi) continue;
        const float4 v = reinterpret_cast<const float4*>(rows + (size_t(t) * K + k) * H)[c4];
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
    }
    if (sh_sel) {
      const float4 v = reinterpret_cast<const float4*>(rows + (size_t(T) * K + t) * H)[c4];
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
  }
  if (resid) {
    const uint2 rb = reinterpret_cast<const uint2*>(resid + size_t(t) * H)[c4];
    const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rb.x));
    const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rb.y));
    s.x = r0.x + bf16_round(s.x);
    s.y = r0.y + bf16_round(s.y);
    s.z = r1.x + bf16_round(s.z);
    s.w = r1.y + bf16_round(s.w);
  }
  __nv_bfloat162 lo2 = __floats2bfloat162_rn(s.x, s.y);
  __nv_bfloat162 hi2 = __floats2bfloat162_rn(s.z, s.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo2);
  packed.y = *reinterpret_cast<uint32_t*>(&hi2);
  reinterpret_cast<uint2*>(y + size_t(t) * H)[c4] = packed;
}

namespace {
// Programmatic dependent launch of the decode chain (PMOE_PDL=0: plain launches).
const bool g_pdl = [] {
  const char* v = std::getenv("PMOE_PDL");
  return !(v && std::atoi(v) == 0);
}();

template <typename... KArgs, typename... Args>
cudaError_t launch_dep(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int g_num_sms = 148;
int g_kch_gu = 4;  // k-chunks per gate_up stage (512 B per weight row)
int g_dn_row_blocks = kDnRowBlocks;
int g_kch_dn = 8;  // k-chunks per stage of the mma.sync down kernel (two 96 KiB stages)
bool g_down_sync = false;  // force the mma.sync down kernel (comparison)

template <int KCH>
cudaError_t set_attrs() {
  cudaError_t e = cudaFuncSetAttribute(gate_up_tma_kernel<KCH>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GuCfg<KCH>::kSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(down_tma_kernel<KCH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              DnCfg<KCH>::kSmem);
}

int env_kch(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (!v) return dflt;
  const int k = std::atoi(v);
  return (k == 1 || k == 2 || k == 4 || k == 8) ? k : dflt;
}

// Largest supported chunk count <= want that divides every k extent.
int fit_kch(int want, int k1, int k2) {
  for (int k = want; k > 1; k >>= 1)
    if (k1 % (kKC * k) == 0 && k2 % (kKC * k) == 0) return k;
  return 1;
}
}  // namespace

cudaError_t stream_init(int num_sms) {
  g_num_sms = num_sms;
  g_kch_gu = env_kch("PMOE_STREAM_KCH_GU", g_kch_gu);
  g_kch_dn = env_kch("PMOE_STREAM_KCH_DN", g_kch_dn);
  if (const char* v = std::getenv("PMOE_DOWN_SYNC")) g_down_sync = std::atoi(v) != 0;
  if (const char* v = std::getenv("PMOE_DN_ROWBLOCKS")) {
    const int r = std::atoi(v);
    if (r == 1 || r == 2 || r == 4 || r == 8 || r == 16) g_dn_row_blocks = r;
  }
  cudaError_t e = set_attrs<1>();
  if (e == cudaSuccess) e = set_attrs<2>();
  if (e == cudaSuccess) e = set_attrs<4>();
  if (e == cudaSuccess)  // down only: 8 k-chunks per stage
    e = cudaFuncSetAttribute(down_tma_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DnCfg<8>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kDtSmem);
  return e;
}

cudaError_t launch_stream_experts(const Dims& d, const __nv_bfloat16* x,
                                  const __nv_bfloat16* w_gate_up, const __nv_bfloat16* w_down,
                                  const __nv_bfloat16* w_sh_gate, const __nv_bfloat16* w_sh_up,
                                  const __nv_bfloat16* w_sh_down, const Workspace& ws,
                                  cudaStream_t st, void* mid_event, const EpPeers& ep) {
  float* rows = ep.world > 0 ? ep.rows[ep.rank] : ws.rows;
  const int kg = fit_kch(g_kch_gu, d.H, d.H);
  const int kd = fit_kch(g_kch_dn, d.I, d.Is);
  int rbk = g_dn_row_blocks;  // 64-row blocks per down unit, dividing H / 64
  while (rbk > 1 && (d.H / kUnitRows) % rbk != 0) rbk >>= 1;
  CUtensorMap tm_gu, tm_sg, tm_su, tm_dn, tm_sd, tm_x, tm_h, tm_h8;
  const uint64_t H = d.H, I = d.I, Is = d.Is, E = d.E, T = d.T;
  const uint64_t R = T * d.K + T, ldh = d.ldh;
  if (!make_tmap_bf16_2d(&tm_gu, w_gate_up, H, E * 2 * I, H * 2, kKC, kUnitRows) ||
      !make_tmap_bf16_2d(&tm_sg, w_sh_gate, H, Is, H * 2, kKC, kUnitRows) ||
      !make_tmap_bf16_2d(&tm_su, w_sh_up, H, Is, H * 2, kKC, kUnitRows) ||
      !make_tmap_bf16_2d(&tm_dn, w_down, I, E * H, I * 2, kKC, kUnitRows) ||
      !make_tmap_bf16_2d(&tm_sd, w_sh_down, Is, H, Is * 2, kKC, kUnitRows) ||
      !make_tmap_bf16_2d(&tm_x, x, H, T, H * 2, kKC * kg, 1, /*swizzle128=*/false) ||
      !make_tmap_bf16_2d(&tm_h, ws.h, ldh, R, ldh * 2, kKC, kActRows) ||
      !make_tmap_bf16_2d(&tm_h8, ws.h, ldh, R, ldh * 2, kKC, 8))
    return cudaErrorInvalidValue;
  ExpertTables tb{ws.active, ws.n_active, ws.offsets, ws.sorted_tok, ws.pair_dst, ws.pair_w};
  int* status = ws.status + 1;
#define PMOE_GU(KCH)                                                                        \
  launch_dep(gate_up_tma_kernel<KCH>, g_num_sms, kStreamThreads, GuCfg<KCH>::kSmem, st, tm_gu, \
             tm_sg, tm_su, tm_x, tb, d.H, d.E, d.I, d.Is, d.ldh, ws.h, status, ws.status + 2)
#define PMOE_DN(KCH)                                                                  \
  down_tma_kernel<KCH><<<g_num_sms, kDnThreads, DnCfg<KCH>::kSmem, st>>>(             \
      tm_dn, tm_sd, tm_h, tm_h8, tb, d.H, d.E, d.I, d.Is, rows, status, ws.status + 3, ep, rbk)
  const cudaError_t eg = kg == 4 ? PMOE_GU(4) : kg == 2 ? PMOE_GU(2) : PMOE_GU(1);
  if (eg != cudaSuccess) return eg;
  if (mid_event) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(mid_event), st);
    if (e != cudaSuccess) return e;
  }
  // tcgen05 down: 128-row weight boxes, 16-row activation boxes
  const bool down_tc = !g_down_sync && d.H % kDtRows == 0 && d.I % kKC == 0 && d.Is % kKC == 0;
  if (down_tc) {
    CUtensorMap tm_dn128, tm_sd128, tm_h16;
    if (!make_tmap_bf16_2d(&tm_dn128, w_down, I, E * H, I * 2, kKC, kDtRows) ||
        !make_tmap_bf16_2d(&tm_sd128, w_sh_down, Is, H, Is * 2, kKC, kDtRows) ||
        !make_tmap_bf16_2d(&tm_h16, ws.h, ldh, R, ldh * 2, kKC, kDtTok))
      return cudaErrorInvalidValue;
    int rbt = 4;  // 128-row blocks per unit, dividing H / 128
    while (rbt > 1 && (d.H / kDtRows) % rbt != 0) rbt >>= 1;
    const cudaError_t e = launch_dep(down_tc_kernel, g_num_sms, kDtThreads, kDtSmem, st, tm_dn128,
                                     tm_sd128, tm_h16, tb, d.H, d.E, d.I, d.Is, rows, status,
                                     ws.status + 3, ep, rbt);
    if (e != cudaSuccess) return e;
  } else {
    if (kd == 8) PMOE_DN(8); else if (kd == 4) PMOE_DN(4); else if (kd == 2) PMOE_DN(2);
    else PMOE_DN(1);
  }
#undef PMOE_GU
#undef PMOE_DN
  return cudaGetLastError();
}

cudaError_t launch_combine(const Dims& d, const Workspace& ws, int lo, int hi, int with_shared,
                           int with_routed, const __nv_bfloat16* resid, __nv_bfloat16* y,
                           cudaStream_t st, const EpPeers& ep) {
  const long n = long(d.T) * (d.H / 4);
  if (n == 0) return cudaSuccess;
  const float* rows = ep.world > 0 ? ep.rows[ep.rank] : ws.rows;
  const int* flags = ep.world > 0 ? ep.flags[ep.rank] : nullptr;
  return launch_dep(combine_kernel, unsigned((n + 255) / 256), 256u, size_t(0), st, rows,
                    ep.par_stride, static_cast<const int32_t*>(ws.topk_idx), d.T, d.H, d.K, lo,
                    hi, with_shared, with_routed, d.sh_lo, d.sh_hi, flags, ep.world,
                    static_cast<const int*>(ep.epoch_dev), ep.epoch, ws.status + 1, ep.sticky,
                    resid, y);
}

// One thread: the device epoch counter of an exchange buffer, bumped at the
// start of every call that uses it.
__global__ void ep_epoch_bump_kernel(int* epoch) { *epoch += 1; }

cudaError_t launch_epoch_bump(int* epoch, cudaStream_t st) {
  ep_epoch_bump_kernel<<<1, 1, 0, st>>>(epoch);
  return cudaGetLastError();
}

}  // namespace pmoe
