// Grouped SwiGLU experts for mid-size row groups (a few to 64 routed rows per
// expert: batched decode, expert-parallel owners, the stacked decode step) on
// tcgen05, with the weights kept exact.
//
// ExpertFFN.forward (moe_forward.py:129-133) for expert e and its routed rows:
//   h = act(x Wg^T) * (x Wu^T),   y = h Wd^T,
// where every 32-wide GGUF block of a weight row is 32 quants q and one fp16
// scale d (w = d * q, dequant_fast.py:44-100).  Here the tensor core multiplies
// the quants themselves -- exact fp16 integers -- with the activations split
// into fp16 hi + lo (two MMA columns per routed row).  Each block gets a fresh
// accumulator in tensor memory and promoter warps fold it into f32 registers
// with round-to-nearest:
//   acc[f][r] += d[f][b] * (D_b[f][hi r] + D_b[f][lo r])
// so no weight is rounded and the tensor core's truncating accumulation never
// runs over more than one block (the numerics of the mma.sync decode GEMVs).
//
// Work unit = (chunk of up to RB sorted rows of one expert, 128 weight rows):
//   gate/up (MODE 0): 64 F-rows of W_gate (A rows 0-63) and the same 64 of W_up
//                     (A rows 64-127); the epilogue writes act(gate) * up to the
//                     hidden planes;
//   down (MODE 1):    128 output columns of W_down; the epilogue writes y rows.
// MMA: M = 128 weight rows (A: dequantised by producer warps into 128-byte-
// swizzled K-major shared memory), N = 2 RB (B: the chunk's hi rows then its lo
// rows, 2-D TMA from the fp16 planes), K = 16, two per block.  A persistent CTA
// per SM walks units c, c + grid, ...; a ring of 128-deep stages (two 64-wide
// tiles of A and of B) holds the operands.  One thread issues every tcgen05
// instruction and each costs it tens of cycles whatever N is, so the
// synchronisation is coarse: one barrier per stage (TMA bytes + producer
// arrivals), one commit per accumulator group of up to four blocks, and the
// promoter that sees a stage's last group complete releases the stage.
// Warps: 0 TMA (lane 0), 1 MMA issue (lane 0), 2-9 weight producers (one 16-row
// strip each), 10-17 promoters (tensor-memory lane quarter w % 4; half of the
// chunk's rows each).  Every wait is bounded and reports MOE_STATUS_TIMEOUT.
#include <cuda.h>
#include <math.h>

#include <algorithm>

#include "tc_common.cuh"

namespace moe {

constexpr int kBsM = 128;                       // weight rows per unit
constexpr int kBsTileK = 64;                    // k of one swizzled tile: two blocks
constexpr int kBsProducers = 8;
constexpr int kBsProm0 = 2 + kBsProducers;
constexpr int kBsPromoters = 8;
constexpr int kBsThreads = (kBsProm0 + kBsPromoters) * 32;
constexpr int kBsASub = kBsM * kBsTileK * 2;    // one 128 x 64 tile of fp16 quants: 16 KB
constexpr float kBsHScale = 1.0f / 256.0f;      // hidden planes are stored / 256
// Weight tiles are prefetched into L2 this many 64-wide tiles ahead of their
// register load; producers hold the packed tiles of the next kBsRegRing stages
// in registers; promoters load block scales kBsScaleAhead tiles ahead.
#ifndef MOE_BS_L2_AHEAD
#define MOE_BS_L2_AHEAD 16
#endif
#ifndef MOE_BS_REG_RING
#define MOE_BS_REG_RING 2
#endif
#ifndef MOE_BS_SCALE_AHEAD
#define MOE_BS_SCALE_AHEAD 4
#endif
constexpr int kBsL2Ahead = MOE_BS_L2_AHEAD;
constexpr int kBsRegRing = MOE_BS_REG_RING;
constexpr int kBsScaleAhead = MOE_BS_SCALE_AHEAD;
static_assert(kBsScaleAhead >= 2 && kBsScaleAhead % 2 == 0, "scale ring");

template <int RB, int MODE>
struct BsCfg {
  static constexpr int N = 2 * RB;                               // MMA columns
  static constexpr int kBSub = N * 128;                          // hi + lo rows of one tile
  // stage: A tiles 0, 1 then B tiles 0, 1 (all 1024-byte aligned)
  static constexpr int kStageBytes = 2 * (kBsASub + kBSub);
  static constexpr int kG = N <= 64 ? 4 : 2;                     // blocks per accumulator group
  static constexpr int kGroupCols = kG * N;
  static constexpr int kSlots = kTmemCols / kGroupCols;          // accumulator groups in flight
  // gate/up: the up sums handed to the gate warps, RB x 64 floats
  static constexpr int kXchBytes = MODE == 0 ? RB * 64 * 4 : 0;
  static constexpr int kStagesFit = (220 * 1024 - kXchBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit < 5 ? kStagesFit : 5;
  static constexpr int kUsed = kStages * kStageBytes + kXchBytes + 2048;
  // at least 120 KB, so one CTA holds an SM (and its tensor memory) at a time
  static constexpr int kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
  static_assert(kStages >= 3, "stage ring");
  static_assert(kSlots >= 2 && (kSlots & (kSlots - 1)) == 0, "accumulator slots");
  static_assert(RB % 8 == 0, "the lo rows start on a 1024-byte swizzle atom");
};

struct BsArgs {
  const uint8_t* w0;         // MODE 0: W_gate stack; MODE 1: W_down stack
  const uint8_t* w1;         // MODE 0: W_up stack
  size_t mat_bytes;          // bytes per expert of the stacks
  int act;                   // MODE 0: MOE_ACT_*
  const float* down_scale;   // MODE 1: per-expert factor, or null
  int K;                     // reduction length: d (MODE 0) or F (MODE 1)
  int n_units_n;             // units per chunk: F / 64 (MODE 0), ceil(d / 128) (MODE 1)
  int P, F, d;
  const int32_t* offsets;
  const int* chunk_e;
  const int* chunk_r0;
  const int* n_chunks;
  const float* row_scale;    // MODE 0: inverse power-of-two factor of each row
  __half* h_planes;          // MODE 0 output: [2][P][F]
  float* y;                  // MODE 1 output
  const int32_t* y_rows;
  int* status;
};

struct BsUnit {
  int e, r0;   // chunk: sorted rows from r0 of expert e
  int n0;      // MODE 0: first F-row; MODE 1: first output column
};

template <int MODE>
__device__ __forceinline__ BsUnit bs_unit(const BsArgs& a, int u) {
  const int c = u / a.n_units_n;
  BsUnit r;
  r.e = a.chunk_e[c];
  r.r0 = a.chunk_r0[c];
  r.n0 = (u - c * a.n_units_n) * (MODE == 0 ? 64 : 128);
  return r;
}

// Packed tiles of A-tile strip `strip` (rows 16 strip .. + 15) of a unit, k
// tile 0 (the next k tiles follow), or null past the matrix's last row.
template <int QT, int MODE>
__device__ __forceinline__ const uint8_t* bs_strip_tiles(const BsArgs& a, const BsUnit& u,
                                                         int strip, int ktiles) {
  using Tr = QTraits<QT>;
  const uint8_t* mat;
  int wrow;
  if (MODE == 0) {
    mat = (strip < 4 ? a.w0 : a.w1) + (size_t)u.e * a.mat_bytes;
    wrow = u.n0 + 16 * (strip & 3);
  } else {
    mat = a.w0 + (size_t)u.e * a.mat_bytes;
    wrow = u.n0 + 16 * strip;
    if (wrow >= a.d) return nullptr;
  }
  return mat + (size_t)(wrow / 16) * ktiles * Tr::kTileBytes;
}

// One packed half tile (registers) -> rows r0 + g + 8 * half of the swizzled A
// tile as exact fp16 integers (the quants, unscaled).  Element placement and
// the bank-conflict-free block order follow store_packed_half.
template <int QT>
__device__ __forceinline__ void store_packed_int(const PackedHalf<QT>& p, int lane, int half,
                                                 uint8_t* a, int r0) {
  const int g = lane >> 2, t = lane & 3;
  const int row = r0 + g + 8 * half;
  uint8_t* ar = a + row * 128;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int b = it ^ (g & 1);
    if constexpr (QT == MOE_Q8_0) {
      const uint32_t w0 = b ? p.q.z : p.q.x, w1 = b ? p.q.w : p.q.y;
      uint32_t q[4];
      dequant_q8(w0, q[0], q[1]);
      dequant_q8(w1, q[2], q[3]);
      const int ch = (4 * b + t) ^ (row & 7);
      *reinterpret_cast<uint4*>(ar + ch * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    } else {
      const uint32_t word = b ? p.q.y : p.q.x;
      // bytes i = 0..3 hold element 4t + i (low nibble) and 16 + 4t + i (high)
      const uint32_t p01 = prmt(word, 0u, 0x4140u), p23 = prmt(word, 0u, 0x4342u);
      const uint32_t kMagic = 0x64006400u, kSubLo = 0xE408E408u;   // 1024, -1032
      const uint32_t kMulHi = 0x2C002C00u, kSubHi = 0xD480D480u;   // 1/16, -72
      const uint32_t lq01 = hadd2_u(lop3_and_or(p01, 0x000F000Fu, kMagic), kSubLo);
      const uint32_t lq23 = hadd2_u(lop3_and_or(p23, 0x000F000Fu, kMagic), kSubLo);
      const uint32_t hq01 = hfma2_u(lop3_and_or(p01, 0x00F000F0u, kMagic), kMulHi, kSubHi);
      const uint32_t hq23 = hfma2_u(lop3_and_or(p23, 0x00F000F0u, kMagic), kMulHi, kSubHi);
      const int ch_lo = (4 * b + (t >> 1)) ^ (row & 7);
      const int ch_hi = (4 * b + 2 + (t >> 1)) ^ (row & 7);
      const int off = (t & 1) * 8;
      *reinterpret_cast<uint2*>(ar + ch_lo * 16 + off) = make_uint2(lq01, lq23);
      *reinterpret_cast<uint2*>(ar + ch_hi * 16 + off) = make_uint2(hq01, hq23);
    }
  }
}

// 4 columns of this warp's 32 tensor-memory lanes (no wait)
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t& a, uint32_t& b, uint32_t& c,
                                         uint32_t& d) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(taddr));
}

// NC hi columns at taddr and NC lo columns at taddr + lo_off, after the wait;
// the values pass through the wait so no use is scheduled before it.
template <int NC>
__device__ __forceinline__ void tmem_ld_hilo(uint32_t taddr, uint32_t lo_off, float (&hi)[NC],
                                             float (&lo)[NC]) {
  uint32_t h[NC], l[NC];
#pragma unroll
  for (int c = 0; c < NC; c += 4) {
    tmem_ld4(taddr + c, h[c], h[c + 1], h[c + 2], h[c + 3]);
    tmem_ld4(taddr + lo_off + c, l[c], l[c + 1], l[c + 2], l[c + 3]);
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    asm volatile("" : "+r"(h[c]), "+r"(l[c]));
    hi[c] = __uint_as_float(h[c]);
    lo[c] = __uint_as_float(l[c]);
  }
}

// ---------------------------------------------------------------------------
// roles
// ---------------------------------------------------------------------------
// k tiles (64 wide) of stage kk: two, or one for the last stage when the
// reduction is an odd number of tiles
__device__ __forceinline__ int bs_stage_tiles(int ktiles, int kk) {
  return min(2, ktiles - 2 * kk);
}

// Activation producer (one thread): the chunk's RB hi rows and RB lo rows of
// every tile of every stage by TMA, arriving on the stage's barrier with its
// byte count.  Before returning it waits (bounded) for its last stages.
template <int RB, int MODE, int STAGES, int SB>
__device__ __forceinline__ void bs_tma_role(const CUtensorMap* map, const BsArgs& a, int my_units,
                                            int ktiles, int nst, uint8_t* stage_base,
                                            uint64_t* full, uint64_t* empty, volatile int* flag) {
  using Cfg = BsCfg<RB, MODE>;
  int it = 0;
  bool ok = true;
  for (int i = 0; i < my_units && ok; ++i) {
    const int r0 = a.chunk_r0[((int)blockIdx.x + i * (int)gridDim.x) / a.n_units_n];
    for (int kk = 0; kk < nst; ++kk) {
      const int s = it % STAGES, round = it / STAGES;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
        tc_fail(flag, a.status);
        ok = false;
        break;
      }
      if (*flag) {
        ok = false;
        break;
      }
      const int nt = bs_stage_tiles(ktiles, kk);
      uint8_t* b = stage_base + s * SB + 2 * kBsASub;
      mbar_expect_tx(&full[s], (uint32_t)(nt * 2 * RB * 128));
      for (int h = 0; h < nt; ++h) {
        const int x = (2 * kk + h) * kBsTileK;
        tma_load_2d(b + h * Cfg::kBSub, map, x, r0, &full[s]);
        tma_load_2d(b + h * Cfg::kBSub + RB * 128, map, x, a.P + r0, &full[s]);
      }
      ++it;
    }
  }
  for (int s = 0; s < STAGES; ++s)
    if (it > s) mbar_wait(&full[s], ((it - 1 - s) / STAGES) & 1);
}

// One producer's registers for one stage: both halves of its packed tile for
// each of the stage's two k tiles.
template <int QT>
struct StripStageInt {
  PackedHalf<QT> h[2][2];
  bool act[2];
};

// Weight producer (one warp): dequantises A rows 16 strip .. + 15 of every
// tile of every stage.  A register ring holds the packed tiles of the next
// kBsRegRing stages; an L2 prefetch cursor runs kBsL2Ahead tiles ahead of it.
template <int QT, int MODE, int STAGES, int SB>
__device__ __forceinline__ void bs_producer_role(const BsArgs& a, int strip, int lane,
                                                 int my_units, int ktiles, int nst,
                                                 uint8_t* stage_base, uint64_t* full,
                                                 uint64_t* empty, volatile int* flag) {
  using Tr = QTraits<QT>;
  const int total = my_units * nst;
  auto strip_of = [&](int i) {
    return bs_strip_tiles<QT, MODE>(
        a, bs_unit<MODE>(a, (int)blockIdx.x + i * (int)gridDim.x), strip, ktiles);
  };
  int li = 0, lk = 0;   // register cursor: unit, stage
  const uint8_t* lp = strip_of(0);
  int qn = 0, qi = 0, qk = 0;   // L2 cursor: tiles issued, unit, tile
  const uint8_t* qp = lp;
  const int qtotal = my_units * ktiles;
  constexpr int kLines = (Tr::kTileBytes + 127) / 128;
  auto l2_step = [&]() {
    if (qp) {
      const uint8_t* t = qp + (size_t)qk * Tr::kTileBytes;
      if (lane < kLines) prefetch_l2(t + lane * 128);
      else if (lane == kLines) prefetch_l2(t + Tr::kTileBytes - 1);
    }
    ++qn;
    if (++qk == ktiles) {
      qk = 0;
      if (++qi < my_units) qp = strip_of(qi);
    }
  };
  auto load_next = [&](StripStageInt<QT>& p) {
    const int nt = bs_stage_tiles(ktiles, lk);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      p.act[h] = lp != nullptr && h < nt;
      if (p.act[h]) {
        const uint8_t* t = lp + (size_t)(2 * lk + h) * Tr::kTileBytes;
        load_packed_half<QT>(p.h[h][0], t, lane, 0);
        load_packed_half<QT>(p.h[h][1], t, lane, 1);
      }
    }
    if (++lk == nst) {
      lk = 0;
      if (++li < my_units) lp = strip_of(li);
    }
  };
  StripStageInt<QT> p[kBsRegRing];
#pragma unroll
  for (int i = 0; i < kBsRegRing; ++i)
    if (i < total) load_next(p[i]);
  while (qn < qtotal && qn < 2 * kBsRegRing + kBsL2Ahead) l2_step();
  bool ok = true;
  for (int it0 = 0; it0 < total && ok; it0 += kBsRegRing) {
#pragma unroll
    for (int j = 0; j < kBsRegRing; ++j) {
      const int it = it0 + j;
      if (it < total && ok) {
        const int s = it % STAGES, round = it / STAGES;
        if (round > 0 && !warp_mbar_wait(&empty[s], (round - 1) & 1, lane)) {
          if (lane == 0) tc_fail(flag, a.status);
          ok = false;
        } else if ((it & 7) == 0 && __shfl_sync(0xffffffffu, *flag, 0)) {
          ok = false;   // another role gave up
        } else {
          uint8_t* at = stage_base + s * SB;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (p[j].act[h]) {
              store_packed_int<QT>(p[j].h[h][0], lane, 0, at + h * kBsASub, strip * 16);
              store_packed_int<QT>(p[j].h[h][1], lane, 1, at + h * kBsASub, strip * 16);
            }
          fence_proxy_async_smem();   // generic stores -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
          if (it + kBsRegRing < total) {
            load_next(p[j]);
            if (qn < qtotal) l2_step();
            if (qn < qtotal) l2_step();
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int QT, int RB, int MODE>
__global__ void __launch_bounds__(kBsThreads, 1)
bs_kernel(const __grid_constant__ CUtensorMap bmap, const BsArgs args) {
  using Cfg = BsCfg<RB, MODE>;
  constexpr int N = Cfg::N, S = Cfg::kStages, SB = Cfg::kStageBytes, NS = Cfg::kSlots;
  constexpr int G = Cfg::kG, GC = Cfg::kGroupCols;
  constexpr int RH = RB / 2;                 // rows per promoter warp
  constexpr int CH = RH < 16 ? RH : 16;      // rows per tensor-memory read
  extern __shared__ __align__(1024) uint8_t bs_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(bs_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  float* xch = reinterpret_cast<float*>(smem + S * SB);   // MODE 0: [RB][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * SB + Cfg::kXchBytes);
  uint64_t* empty = full + S;
  uint64_t* accfull = empty + S;
  uint64_t* accempty = accfull + NS;
  uint64_t* xfull = accempty + NS;   // up sums written
  uint64_t* xempty = xfull + 1;      // up sums read
  uint64_t* drain = xempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (MODE == 0) pdl_wait();   // the chunk plan and the activation planes
  pdl_trigger();
  // MODE 1 reads the chunk plan at once (complete: gate/up triggers only after
  // its own wait) and waits for the hidden planes only in its TMA thread.
  const int n_units = *args.n_chunks * args.n_units_n;
  if ((int)blockIdx.x >= n_units) return;
  const int my_units = (n_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1;
  const int ktiles = args.K / kBsTileK;
  const int nst = (ktiles + 1) / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], kBsProducers + 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], kBsPromoters);
    }
    mbar_init(xfull, 4);
    mbar_init(xempty, 4);
    mbar_init(drain, 1);
    *flag = 0;
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&bmap) : "memory");
  }
  const uint32_t tmem = tc_alloc_all(tmem_slot, warp);

  if (warp == 0) {
    if (lane == 0) {
      if (MODE == 1) pdl_wait();   // gate/up's hidden planes
      bs_tma_role<RB, MODE, S, SB>(&bmap, args, my_units, ktiles, nst, stage_base, full, empty,
                                   flag);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc_idesc(kBsM, N);
      const uint64_t d0 = sw128_desc(stage_base);
      const uint32_t d0_lo = (uint32_t)d0, d_hi = (uint32_t)(d0 >> 32);
      int s = 0, g = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < my_units && ok; ++i) {
        for (int kk = 0; kk < nst && ok; ++kk) {
          if (!mbar_wait(&full[s], phase)) {
            tc_fail(flag, args.status);
            ok = false;
            break;
          }
          const int nb = 2 * bs_stage_tiles(ktiles, kk);   // blocks in this stage
          const uint32_t a_lo = d0_lo + (uint32_t)(s * (SB >> 4));
          const uint32_t b_lo = a_lo + (uint32_t)((2 * kBsASub) >> 4);
          for (int b0 = 0; b0 < nb && ok; b0 += G) {
            const int slot = g & (NS - 1), use = g / NS;
            if (use > 0 && !mbar_wait(&accempty[slot], (use - 1) & 1)) {
              tc_fail(flag, args.status);
              ok = false;
              break;
            }
            // the promoters' reads of this slot precede the MMAs that overwrite it
            tc_fence_after();
#pragma unroll
            for (int bi = 0; bi < G; ++bi) {
              const int blk = b0 + bi;
              if (blk < nb) {
                // tile blk / 2, block blk % 2 of it: +64 bytes, +32 per k16
                const uint32_t ao =
                    a_lo + (uint32_t)((blk >> 1) * (kBsASub >> 4) + (blk & 1) * 4);
                const uint32_t bo =
                    b_lo + (uint32_t)((blk >> 1) * (Cfg::kBSub >> 4) + (blk & 1) * 4);
                const uint32_t dt = tmem + (uint32_t)(slot * GC + bi * N);
                tc_mma_lo(dt, ao, bo, d_hi, idesc, 0u);
                tc_mma_lo(dt, ao + 2, bo + 2, d_hi, idesc, 1u);
              }
            }
            tc_commit(&accfull[slot]);
            ++g;
          }
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
      }
      // every MMA issued here completes before the tensor memory is released
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp < kBsProm0) {
    bs_producer_role<QT, MODE, S, SB>(args, warp - 2, lane, my_units, ktiles, nst, stage_base,
                                      full, empty, flag);
  } else {
    using Tr = QTraits<QT>;
    const int q = warp & 3, hh = (warp - kBsProm0) >> 2;
    const int rho = 32 * q + lane;   // A row of this lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const bool releaser = warp == kBsProm0 && lane == 0;   // frees each finished stage
    int s = 0, g = 0;
    bool ok = true;
    for (int i = 0; i < my_units && ok; ++i) {
      const BsUnit u = bs_unit<MODE>(args, (int)blockIdx.x + i * (int)gridDim.x);
      const int rend = min(u.r0 + RB, args.offsets[u.e + 1]);   // the chunk's last row + 1
      // this lane's weight row and the fp16 scales of its blocks
      const uint8_t* mat;
      int wrow;
      if (MODE == 0) {
        mat = (q < 2 ? args.w0 : args.w1) + (size_t)u.e * args.mat_bytes;
        wrow = u.n0 + 32 * (q & 1) + lane;
      } else {
        mat = args.w0 + (size_t)u.e * args.mat_bytes;
        wrow = u.n0 + rho;
      }
      const bool wvalid = MODE == 0 || wrow < args.d;
      const uint8_t* sp = mat + (size_t)(wrow / 16) * ktiles * Tr::kTileBytes + Tr::kTileQuant +
                          (wrow & 7) * 8 + ((wrow >> 3) & 1) * 4;
      auto scales = [&](int t) -> uint32_t {   // both block scales of k tile t
        return (wvalid && t < ktiles)
                   ? __ldg(reinterpret_cast<const uint32_t*>(sp + (size_t)t * Tr::kTileBytes))
                   : 0u;
      };
      uint32_t scq[kBsScaleAhead];   // scales of k tiles 2 kk .. 2 kk + kBsScaleAhead - 1
#pragma unroll
      for (int t = 0; t < kBsScaleAhead; ++t) scq[t] = scales(t);
      float acc[RH];
#pragma unroll
      for (int t = 0; t < RH; ++t) acc[t] = 0.f;
      for (int kk = 0; kk < nst && ok; ++kk) {
        const uint32_t sc_t0 = scq[0], sc_t1 = scq[1];
#pragma unroll
        for (int t = 0; t + 2 < kBsScaleAhead; ++t) scq[t] = scq[t + 2];
        scq[kBsScaleAhead - 2] = scales(2 * kk + kBsScaleAhead);
        scq[kBsScaleAhead - 1] = scales(2 * kk + kBsScaleAhead + 1);
        const int nb = 2 * bs_stage_tiles(ktiles, kk);
        for (int b0 = 0; b0 < nb; b0 += G) {
          const int slot = g & (NS - 1), use = g / NS;
          if (!warp_mbar_wait(&accfull[slot], use & 1, lane)) {
            if (lane == 0) tc_fail(flag, args.status);
            ok = false;
            break;
          }
          tc_fence_after();
          // the stage's last group is complete, so are all of its MMAs
          if (releaser && b0 + G >= nb) mbar_arrive(&empty[s]);
#pragma unroll
          for (int bi = 0; bi < G; ++bi) {
            const int blk = b0 + bi;
            if (blk < nb) {
              const uint32_t sw = (blk >> 1) ? sc_t1 : sc_t0;
              const float dsc = __half2float(
                  __ushort_as_half((unsigned short)((blk & 1) ? (sw >> 16) : (sw & 0xFFFFu))));
              const uint32_t col = lane_base + (uint32_t)(slot * GC + bi * N + hh * RH);
#pragma unroll
              for (int c0 = 0; c0 < RH; c0 += CH) {
                float hi[CH], lo[CH];
                tmem_ld_hilo<CH>(col + c0, (uint32_t)RB, hi, lo);
#pragma unroll
                for (int t = 0; t < CH; ++t)
                  acc[c0 + t] = fmaf(dsc, hi[t] + lo[t], acc[c0 + t]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[slot]);
          ++g;
        }
        if (++s == S) s = 0;
      }
      if (!ok) break;
      const int rbase = u.r0 + hh * RH;
      if (MODE == 0) {
        // up warps (quarters 2, 3) hand their sums to the gate warps of the same rows
        const int fl = 32 * (q & 1) + lane;   // F-row within the unit
        if (q >= 2) {
          if (i > 0 && !warp_mbar_wait(xempty, (i - 1) & 1, lane)) {
            if (lane == 0) tc_fail(flag, args.status);
            break;
          }
#pragma unroll
          for (int t = 0; t < RH; ++t) xch[(hh * RH + t) * 64 + fl] = acc[t];
          __syncwarp();
          if (lane == 0) mbar_arrive(xfull);
        } else {
          if (!warp_mbar_wait(xfull, i & 1, lane)) {
            if (lane == 0) tc_fail(flag, args.status);
            break;
          }
          const int f = u.n0 + fl;
#pragma unroll
          for (int t = 0; t < RH; ++t) {
            const int r = rbase + t;
            const float up = xch[(hh * RH + t) * 64 + fl];
            if (r < rend) {
              const float rs = args.row_scale[r];
              const float h = expert_act(args.act, acc[t] * rs) * (up * rs) * kBsHScale;
              if (!(fabsf(h) <= 65504.f)) set_status(args.status, MOE_STATUS_ROW_OVERFLOW);
              const __half hh16 = __float2half_rn(h);
              const __half ll16 = __float2half_rn(h - __half2float(hh16));
              args.h_planes[(size_t)r * args.F + f] = hh16;
              args.h_planes[((size_t)args.P + r) * args.F + f] = ll16;
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(xempty);
        }
      } else if (wvalid) {
        const float osc = (1.f / kBsHScale) * (args.down_scale ? args.down_scale[u.e] : 1.f);
#pragma unroll
        for (int t = 0; t < RH; ++t) {
          const int r = rbase + t;
          if (r < rend) {
            const int orow = args.y_rows ? args.y_rows[r] : r;
            args.y[(size_t)orow * args.d + wrow] = acc[t] * osc;
          }
        }
      }
    }
  }
  tc_dealloc_all(tmem, warp);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct BsWs {
  int* n_chunks;
  int* chunk_e;
  int* chunk_r0;
  float* row_scale;
  __half* x_planes;   // [2][P][d]
  __half* h_planes;   // [2][P][F]
  size_t bytes;
};

static int bs_max_chunks(int rows, int E, int rb) { return (rows + rb - 1) / rb + E; }

static BsWs carve_bs(void* ws, int rows, int E, int d, int F, int rb) {
  Carve c{static_cast<uint8_t*>(ws), 0, 0};
  BsWs w;
  const int mc = bs_max_chunks(rows, E, rb);
  c.take<int>(64);  // status word
  w.n_chunks = c.take<int>(64);
  w.chunk_e = c.take<int>(mc);
  w.chunk_r0 = c.take<int>(mc);
  w.row_scale = c.take<float>(rows);
  w.x_planes = c.take<__half>((size_t)2 * rows * d);
  w.h_planes = c.take<__half>((size_t)2 * rows * F);
  w.bytes = align_up(c.used, 256);
  return w;
}

// the smallest chunk gives the most chunks
size_t bs_workspace(int rows, int E, int d, int F) {
  return carve_bs(nullptr, rows, E, d, F, 8).bytes;
}

bool bs_supported(int rows, int E, int d, int F) {
  return rows > 0 && E <= 1024 && d % 64 == 0 && F % 64 == 0;
}

template <int QT, int RB>
static int launch_bs(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down,
                     const int32_t* offsets, int E, int rows, const float* x,
                     const int32_t* x_rows, int x_div, const float* x_row_max, int d, int F,
                     float* y, const int32_t* y_rows, const BsWs& w, int* status,
                     const moe_expert_opts* opts, cudaStream_t s) {
  using Tr = QTraits<QT>;
  using C0 = BsCfg<RB, 0>;
  using C1 = BsCfg<RB, 1>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev));
  if (!((attr_set >> (dev & 63)) & 1ull)) {
    MOE_CUDA(cudaFuncSetAttribute(bs_kernel<QT, RB, 0>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, C0::kSmem));
    MOE_CUDA(cudaFuncSetAttribute(bs_kernel<QT, RB, 1>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, C1::kSmem));
    attr_set |= 1ull << (dev & 63);
  }
  const int sms = sm_count();
  const int max_chunks = bs_max_chunks(rows, E, RB);
  {
    ::moe::ProfScope _prof(MOE_K_PLAN, s);
    MOE_CHECK(launch_tile_plan(offsets, E, RB, max_chunks, w.chunk_e, w.chunk_r0, w.n_chunks, s));
  }
  {
    ::moe::ProfScope _prof(MOE_K_XPREP, s);
    MOE_CHECK(launch_act_planes(x, x_rows, x_div, x_row_max, rows, offsets, E, d, w.row_scale,
                                w.x_planes, s));
  }
  CUtensorMap xmap, hmap;
  MOE_CHECK(make_plane_map(&xmap, w.x_planes, 2 * rows, d, RB));
  MOE_CHECK(make_plane_map(&hmap, w.h_planes, 2 * rows, F, RB));
  const size_t mat_bytes = (size_t)F * (d / 32) * Tr::kBlockBytes;
  BsArgs a1 = {};
  a1.w0 = w_gate;
  a1.w1 = w_up;
  a1.mat_bytes = (opts && opts->gate_up_stride) ? opts->gate_up_stride : mat_bytes;
  a1.act = opts ? opts->act : MOE_ACT_SWIGLU;
  a1.K = d;
  a1.n_units_n = F / 64;
  a1.P = rows;
  a1.F = F;
  a1.d = d;
  a1.offsets = offsets;
  a1.chunk_e = w.chunk_e;
  a1.chunk_r0 = w.chunk_r0;
  a1.n_chunks = w.n_chunks;
  a1.row_scale = w.row_scale;
  a1.h_planes = w.h_planes;
  a1.status = status;
  {
    ::moe::ProfScope _prof(MOE_K_GATEUP, s);
    const int grid = (int)std::min<long long>((long long)max_chunks * a1.n_units_n, sms);
    MOE_CUDA(launch_pdl(bs_kernel<QT, RB, 0>, dim3(grid), dim3(kBsThreads), C0::kSmem, s, xmap,
                        a1));
  }
  MOE_CHECK(check_launch("blockscale gate/up"));
  BsArgs a2 = a1;
  a2.w0 = w_down;
  a2.w1 = nullptr;
  a2.mat_bytes = mat_bytes;
  a2.down_scale = opts ? opts->down_scale : nullptr;
  a2.K = F;
  a2.n_units_n = (d + 127) / 128;
  a2.y = y;
  a2.y_rows = y_rows;
  {
    ::moe::ProfScope _prof(MOE_K_DOWN, s);
    const int grid = (int)std::min<long long>((long long)max_chunks * a2.n_units_n, sms);
    MOE_CUDA(launch_pdl(bs_kernel<QT, RB, 1>, dim3(grid), dim3(kBsThreads), C1::kSmem, s, hmap,
                        a2));
  }
  return check_launch("blockscale down");
}

template <int QT>
static int launch_bs_rb(int rb, const uint8_t* wg, const uint8_t* wu, const uint8_t* wd,
                        const int32_t* offsets, int E, int rows, const float* x,
                        const int32_t* x_rows, int x_div, const float* x_row_max, int d, int F,
                        float* y, const int32_t* y_rows, const BsWs& w, int* status,
                        const moe_expert_opts* opts, cudaStream_t s) {
  switch (rb) {
    case 8:
      return launch_bs<QT, 8>(wg, wu, wd, offsets, E, rows, x, x_rows, x_div, x_row_max, d, F, y,
                              y_rows, w, status, opts, s);
    case 16:
      return launch_bs<QT, 16>(wg, wu, wd, offsets, E, rows, x, x_rows, x_div, x_row_max, d, F,
                               y, y_rows, w, status, opts, s);
    case 32:
      return launch_bs<QT, 32>(wg, wu, wd, offsets, E, rows, x, x_rows, x_div, x_row_max, d, F,
                               y, y_rows, w, status, opts, s);
    default:
      return launch_bs<QT, 64>(wg, wu, wd, offsets, E, rows, x, x_rows, x_div, x_row_max, d, F,
                               y, y_rows, w, status, opts, s);
  }
}

int run_experts_bs(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                   int x_div, const float* x_row_max, int d, int F, float* y,
                   const int32_t* y_rows, void* ws, size_t ws_bytes, int* status,
                   const moe_expert_opts* opts, int rb, cudaStream_t s) {
  MOE_REQUIRE(bs_supported(rows, E, d, F), MOE_ERR_UNSUPPORTED, "block-scale path shape");
  MOE_REQUIRE(rb == 8 || rb == 16 || rb == 32 || rb == 64, MOE_ERR_INVALID, "chunk rows %d", rb);
  BsWs w = carve_bs(ws, rows, E, d, F, rb);
  MOE_REQUIRE(ws_bytes >= w.bytes, MOE_ERR_WORKSPACE, "block-scale workspace %zu < %zu",
              ws_bytes, w.bytes);
  if (!status) status = static_cast<int*>(ws);
  if (qtype == MOE_Q4_0)
    return launch_bs_rb<MOE_Q4_0>(rb, w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div,
                                  x_row_max, d, F, y, y_rows, w, status, opts, s);
  return launch_bs_rb<MOE_Q8_0>(rb, w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div,
                                x_row_max, d, F, y, y_rows, w, status, opts, s);
}

}  // namespace moe
