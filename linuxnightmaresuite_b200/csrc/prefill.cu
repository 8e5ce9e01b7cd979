// Grouped SwiGLU experts for large row groups (prefill): tcgen05 / TMEM GEMMs.
//
// For every expert with many routed rows the two products of ExpertFFN.forward
// (moe_forward.py:129-133) are dense GEMMs:
//   GEMM1  [rows x d] x [d x 2F]  -> h = silu(gate) * up      (rows x F)
//   GEMM2  [rows x F] x [F x d]   -> y                        (rows x d)
// The output is cut into 128-row x 128-column tiles (rows of one expert); a
// persistent CTA per SM walks its share of the tiles with tcgen05.mma
// (kind::f16, fp32 accumulators in tensor memory):
//   * the activation tile (fp16 hi and lo planes, see below) arrives by 2-D TMA
//     with 128-byte swizzle, and is prefetched into L2 several stages ahead;
//   * eight producer warps dequantise the packed Q4_0 / Q8_0 weight tiles into
//     the same swizzled layout as fp16 hi + lo (w = d * q exactly, w_hi =
//     fp16(w), w_lo = fp16(w - w_hi));
//   * one thread issues three MMAs per 16-wide k step -- x_hi*w_hi + x_hi*w_lo
//     + x_lo*w_hi -- so operands keep ~22 bits (outputs reach ~1e3 and the
//     reference's f32 tolerance is absolute);
//   * the stage ring runs on across tiles; stage reuse is ordered by mbarriers
//     (TMA transaction counts, producer arrivals, tcgen05.commit), and every
//     wait is bounded;
//   * gate/up keeps two partial accumulators and two correction accumulators in
//     tensor memory; eight promoter warps fold the partials into f32 registers
//     and run the SiLU(gate) * up epilogue into the hidden hi/lo planes while
//     the MMAs of the next period / tile run.  Down keeps one big and one small
//     accumulator (all 512 columns) that four epilogue warps read into f32 rows.
// Rows of a 128-row tile past the expert's range are computed and discarded.
#include <cuda.h>
#include <math.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "tc_common.cuh"

namespace moe {

constexpr int kTcM = 128;        // rows (tokens) per tile
constexpr int kTcNMax = 256;     // output columns per tile (a last, narrower tile has 128)
constexpr int kTcK = 64;         // k per stage (one packed tile column, 128 B of fp16)
constexpr int kTcStages = 2;
// Warps: 0 TMA (lane 0), 1 MMA (lane 0), 2-17 weight producers (one per
// 16-row strip of the B tile), 18-21 epilogue.
constexpr int kTcProd0 = 2;
constexpr int kTcProducers = kTcNMax / 16;
constexpr int kTcEpi0 = kTcProd0 + kTcProducers;
constexpr int kTcEpiWarps = 4;
constexpr int kTcThreads = (kTcEpi0 + kTcEpiWarps) * 32;
constexpr int kATile = kTcM * kTcK * 2;               // one 128 x 64 fp16 plane tile: 16 KB
constexpr int kBTile = kTcNMax * kTcK * 2;            // one 256 x 64 fp16 plane tile: 32 KB
constexpr int kStageBytes = 2 * kATile + 2 * kBTile;  // A hi, A lo, B hi, B lo: 96 KB
constexpr int kTcSmem = kTcStages * kStageBytes + 1024 + 1024;  // + barriers, + alignment
constexpr float kTcHScale = 1.0f / 256.0f;            // hidden planes are stored / 256
// Tensor memory: a "big" accumulator for x_hi*w_hi in columns [0, 256) and a
// "small" one for the two correction products in [256, 512), added with
// round-to-nearest in the epilogue.  The tensor core's fp32 accumulation
// truncates; keeping the corrections apart leaves the big accumulator one
// addition per 16-wide k step.
constexpr int kTcSmallCol = kTcNMax;
static_assert(2 * kTcNMax == kTmemCols, "big + small accumulators fill the tensor memory");
// activation tiles are prefetched into L2 this many stages ahead of their TMA load,
// weight tiles this many stages ahead of their register load
#ifndef MOE_TC_L2_AHEAD
#define MOE_TC_L2_AHEAD 6
#endif
constexpr int kTcL2Ahead = MOE_TC_L2_AHEAD;

// big + small accumulator, 16 columns from taddr
__device__ __forceinline__ void tmem_ld_pair(uint32_t taddr, float (&v)[16]) {
  float w[16];
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + (uint32_t)kTcSmallCol, w);
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __fadd_rn(v[i], w[i]);
}

// ---------------------------------------------------------------------------
// activation planes: sorted row r -> hi plane row r, lo plane row P + r (fp16),
// scaled by a power of two so the row's max |x| sits in [2^14, 2^15)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
tc_prep_kernel(const float* __restrict__ x, const int32_t* __restrict__ x_rows, int x_div,
               const float* __restrict__ x_row_max, int P, const int32_t* __restrict__ offsets,
               int E, int d, float* __restrict__ row_scale, __half* __restrict__ planes) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  // P bounds the planes; the routed rows are offsets[E] <= P of them
  if (r >= P || r >= offsets[E]) return;
  const int src = x_rows ? x_rows[r] / x_div : r;
  const float4* s4 = reinterpret_cast<const float4*>(x + (size_t)src * d);
  float m = 0.f;
  if (x_row_max) {
    m = x_row_max[src];
  } else {
    for (int i = lane; i < d / 4; i += 32) {
      const float4 v = __ldg(s4 + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  float scale = 1.f, inv = 1.f;
  if (m > 0.f && isfinite(m)) {
    const int ex = ilogbf(m);
    scale = ldexpf(1.f, 14 - ex);
    inv = ldexpf(1.f, ex - 14);
  }
  if (lane == 0) row_scale[r] = inv;
  __half* hi = planes + (size_t)r * d;
  __half* lo = planes + ((size_t)P + r) * d;
  for (int i = lane; i < d / 4; i += 32) {
    const float4 v = __ldg(s4 + i);
    const float a[4] = {v.x * scale, v.y * scale, v.z * scale, v.w * scale};
    const __half2 h0 = __floats2half2_rn(a[0], a[1]), h1 = __floats2half2_rn(a[2], a[3]);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    const __half2 l0 = __floats2half2_rn(a[0] - f0.x, a[1] - f0.y);
    const __half2 l1 = __floats2half2_rn(a[2] - f1.x, a[3] - f1.y);
    reinterpret_cast<__half2*>(hi)[2 * i] = h0;
    reinterpret_cast<__half2*>(hi)[2 * i + 1] = h1;
    reinterpret_cast<__half2*>(lo)[2 * i] = l0;
    reinterpret_cast<__half2*>(lo)[2 * i + 1] = l1;
  }
}

// m-tiles of tm rows per active expert: tile_e[i], tile_r0[i] (sorted row),
// *n_tiles.  One CTA, E <= 1024.
__global__ void __launch_bounds__(1024)
tc_tile_plan_kernel(const int32_t* __restrict__ offsets, int E, int tm, int max_tiles,
                    int* __restrict__ tile_e, int* __restrict__ tile_r0, int* __restrict__ n_tiles) {
  __shared__ int sh[33];
  const int e = threadIdx.x;
  const int n = e < E ? offsets[e + 1] - offsets[e] : 0;
  const int nt = n > 0 ? (n + tm - 1) / tm : 0;
  int tot;
  const int t0 = block_excl_scan(nt, sh, tot);
  if (e < E)
    for (int i = 0; i < nt && t0 + i < max_tiles; ++i) {
      tile_e[t0 + i] = e;
      tile_r0[t0 + i] = offsets[e] + i * tm;
    }
  if (e == 0) *n_tiles = min(tot, max_tiles);
}

// ---------------------------------------------------------------------------
// the GEMMs.  MODE 0 (gate/up): an n-tile covers 64 F-rows -- B rows 0-63 from
// W_gate, 64-127 from W_up -- and the epilogue writes SiLU(gate) * up to the
// hidden planes.  MODE 1 (down): an n-tile covers min(256, d - 256 nt) output
// columns.
// ---------------------------------------------------------------------------
struct TcArgs {
  const uint8_t* w0;       // MODE 0: W_gate stack; MODE 1: W_down stack
  const uint8_t* w1;       // MODE 0: W_up stack
  size_t mat_bytes;        // bytes per expert of the MODE's stacks
  int act;                 // MODE 0: MOE_ACT_*
  const float* down_scale; // MODE 1: per-expert factor, or null
  int K;                   // reduction length (d or F)
  int n_tiles_n;           // output column tiles
  int P;                   // sorted rows (plane height)
  int F, d;
  const int32_t* offsets;
  const int* tile_e;
  const int* tile_r0;
  const int* n_mtiles;
  const float* row_scale;  // MODE 0
  __half* h_planes;        // MODE 0 output: [2][P][F]
  float* y;                // MODE 1 output
  const int32_t* y_rows;
  int* status;
};

constexpr int kGuFRows = 64;   // F-rows per gate/up tile

// Tile t of a launch: m-tile t / n_tiles_n (128 sorted rows of one expert) and
// n-tile t % n_tiles_n.  CTA c of the persistent grid takes tiles c, c + grid, ...
struct TcTile {
  int e, row0;
  int n0;   // MODE 0: first F-row; MODE 1: first output column
  int nr;   // MODE 0: F-rows (64); MODE 1: output columns (128 or 256)
};

template <int MODE>
__device__ __forceinline__ TcTile tc_tile(const TcArgs& a, int t) {
  const int mt = t / a.n_tiles_n;
  const int nt = t - mt * a.n_tiles_n;
  TcTile r;
  r.e = a.tile_e[mt];
  r.row0 = a.tile_r0[mt];
  if (MODE == 0) {
    r.n0 = nt * kGuFRows;
    r.nr = kGuFRows;
  } else {
    r.n0 = nt * kTcNMax;
    r.nr = min(kTcNMax, a.d - r.n0);
  }
  return r;
}

// First packed weight tile of B strip `strip` (rows 16 strip .. + 15) of a
// tile, or null if the tile is narrower; the tiles of consecutive k stages
// follow it.
template <int QT, int MODE>
__device__ __forceinline__ const uint8_t* tc_strip_tiles(const TcArgs& a, const TcTile& tt,
                                                         int strip, int ksteps) {
  using Tr = QTraits<QT>;
  const int row = 16 * strip;
  const uint8_t* mat;
  int wstrip;
  if (MODE == 0) {
    if (row >= 2 * tt.nr) return nullptr;
    const bool up = row >= tt.nr;
    mat = (up ? a.w1 : a.w0) + (size_t)tt.e * a.mat_bytes;
    wstrip = (tt.n0 + row - (up ? tt.nr : 0)) / 16;
  } else {
    if (row >= tt.nr) return nullptr;
    mat = a.w0 + (size_t)tt.e * a.mat_bytes;
    wstrip = (tt.n0 + row) / 16;
  }
  return mat + (size_t)wstrip * ksteps * Tr::kTileBytes;
}

// Activation producer (one thread): hi and lo planes of each stage's 128 x 64
// A tile by TMA; an L2 prefetch cursor runs kTcL2Ahead stages ahead of the
// loads.  Before returning it waits (bounded) for the copies it issued.
template <int MODE, int STAGES, int STAGE_BYTES>
__device__ __forceinline__ void tc_tma_role(const CUtensorMap* amap, const TcArgs& args,
                                            int my_tiles, int ksteps, uint8_t* stage_base,
                                            uint64_t* full_a, uint64_t* empty,
                                            volatile int* flag) {
  const int total = my_tiles * ksteps;
  int pf = 0, pf_i = 0, pf_k = 0;
  int pf_row = tc_tile<MODE>(args, blockIdx.x).row0;
  auto l2_step = [&]() {
    tma_prefetch_2d(amap, pf_k * kTcK, pf_row);
    tma_prefetch_2d(amap, pf_k * kTcK, args.P + pf_row);
    ++pf;
    if (++pf_k == ksteps) {
      pf_k = 0;
      if (++pf_i < my_tiles) pf_row = tc_tile<MODE>(args, blockIdx.x + pf_i * gridDim.x).row0;
    }
  };
  while (pf < total && pf < kTcL2Ahead) l2_step();
  int it = 0;
  bool ok = true;
  for (int i = 0; i < my_tiles && ok; ++i) {
    const int row0 = tc_tile<MODE>(args, blockIdx.x + i * gridDim.x).row0;
    for (int kk = 0; kk < ksteps; ++kk) {
      const int s = it % STAGES, round = it / STAGES;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
        tc_fail(flag, args.status);
        ok = false;
        break;
      }
      if (*flag) {
        ok = false;
        break;
      }
      if (pf < total) l2_step();
      uint8_t* st = stage_base + s * STAGE_BYTES;
      mbar_expect_tx(&full_a[s], 2 * kATile);
      tma_load_2d(st, amap, kk * kTcK, row0, &full_a[s]);
      tma_load_2d(st + kATile, amap, kk * kTcK, args.P + row0, &full_a[s]);
      ++it;
    }
  }
  for (int s = 0; s < STAGES; ++s)
    if (it > s) mbar_wait(&full_a[s], ((it - 1 - s) / STAGES) & 1);
}

// One producer's registers for one stage: both halves of its packed tile, or
// nothing (tile narrower than the producer's strip).
template <int QT>
struct StripStage {
  PackedHalf<QT> h[2];
  bool active;
};

// Weight producer (one warp): dequantises B rows 16 strip .. + 15 of every
// stage (both halves of one packed tile) into the hi / lo planes at B_OFF and
// B_OFF + B_PLANE.  The register ring loads stage it + STAGES as soon as stage
// it is stored; the L2 cursor runs kTcL2Ahead stages ahead of it.
template <int QT, int MODE, int STAGES, int STAGE_BYTES, int B_OFF, int B_PLANE>
__device__ __forceinline__ void tc_producer_role(const TcArgs& args, int strip, int lane,
                                                 int my_tiles, int ksteps, uint8_t* stage_base,
                                                 uint64_t* full, uint64_t* empty,
                                                 volatile int* flag) {
  using Tr = QTraits<QT>;
  const int total = my_tiles * ksteps;
  auto strip_of = [&](int i) {
    return tc_strip_tiles<QT, MODE>(args, tc_tile<MODE>(args, blockIdx.x + i * gridDim.x), strip,
                                    ksteps);
  };
  int li = 0, lk = 0;
  const uint8_t* lp = strip_of(0);
  int qn = 0, qi = 0, qk = 0;
  const uint8_t* qp = lp;
  constexpr int kLines = (Tr::kTileBytes + 127) / 128;
  auto l2_step = [&]() {
    if (qp) {
      const uint8_t* t = qp + (size_t)qk * Tr::kTileBytes;
      if (lane < kLines) prefetch_l2(t + lane * 128);
      else if (lane == kLines) prefetch_l2(t + Tr::kTileBytes - 1);
    }
    ++qn;
    if (++qk == ksteps) {
      qk = 0;
      if (++qi < my_tiles) qp = strip_of(qi);
    }
  };
  auto load_next = [&](StripStage<QT>& p) {
    p.active = lp != nullptr;
    if (p.active) {
      const uint8_t* t = lp + (size_t)lk * Tr::kTileBytes;
      load_packed_half<QT>(p.h[0], t, lane, 0);
      load_packed_half<QT>(p.h[1], t, lane, 1);
    }
    if (++lk == ksteps) {
      lk = 0;
      if (++li < my_tiles) lp = strip_of(li);
    }
  };
  StripStage<QT> p[STAGES];
#pragma unroll
  for (int i = 0; i < STAGES; ++i)
    if (i < total) load_next(p[i]);
  while (qn < total && qn < STAGES + kTcL2Ahead) l2_step();
  bool ok = true;
  for (int it0 = 0; it0 < total && ok; it0 += STAGES) {
#pragma unroll
    for (int j = 0; j < STAGES; ++j) {
      const int it = it0 + j;
      if (it < total && ok) {
        const int round = it / STAGES;   // slot = j
        if (round > 0 && !warp_mbar_wait(&empty[j], (round - 1) & 1, lane)) {
          if (lane == 0) tc_fail(flag, args.status);
          ok = false;
        } else if ((it & 15) == 0 && __shfl_sync(0xffffffffu, *flag, 0)) {
          ok = false;   // another role gave up
        } else {
          if (p[j].active) {
            uint8_t* bt = stage_base + j * STAGE_BYTES + B_OFF;
            store_packed_half<QT>(p[j].h[0], lane, 0, bt, bt + B_PLANE, strip * 16);
            store_packed_half<QT>(p[j].h[1], lane, 1, bt, bt + B_PLANE, strip * 16);
            fence_proxy_async_smem();   // generic stores -> visible to the tensor core
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[j]);
          // the next loads go out after the fence, which would otherwise wait for them
          if (it + STAGES < total) {
            load_next(p[j]);
            if (qn < total) l2_step();
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// gate/up: 128 x 128 tiles, 3 stages of 64 KB.  The x_hi * w_hi products of
// each kGuPeriod-stage period go to a fresh partial accumulator (P0 / P1 in
// tensor memory, alternating); eight promoter warps add each finished partial
// into fp32 registers with round-to-nearest, so the tensor core's truncating
// accumulation never runs over more than 4 * kGuPeriod k16 steps.  The
// correction products accumulate over the whole tile in S0 / S1 (alternating
// per tile; they are ~2^-11 of the result).  Warps: 0 TMA, 1 MMA, 2-9 weight
// producers, 10-17 promoters + epilogue (two per tensor-memory lane quarter,
// each owning 32 gate and the matching 32 up columns).
// ---------------------------------------------------------------------------
constexpr int kGuN = 2 * kGuFRows;                        // 128 B rows
constexpr int kGuStages = 3;
constexpr int kGuBTile = kGuN * kTcK * 2;                 // 16 KB
constexpr int kGuStageBytes = 2 * kATile + 2 * kGuBTile;  // 64 KB
constexpr int kGuProducers = kGuN / 16;                   // 8
constexpr int kGuProm0 = 2 + kGuProducers;
constexpr int kGuPromoters = 8;
constexpr int kGuThreads = (kGuProm0 + kGuPromoters) * 32;
constexpr int kGuSmem = kGuStages * kGuStageBytes + 1024 + 1024;
constexpr int kGuPeriod = 2;                              // stages per partial
constexpr int kGuSCol = 2 * kGuN;                         // S0 at 256, S1 at 384

template <int QT>
__global__ void __launch_bounds__(kGuThreads, 1)
tc_gateup_kernel(const __grid_constant__ CUtensorMap amap, const TcArgs args) {
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + kGuStages * kGuStageBytes);
  uint64_t* empty = full_a + kGuStages;
  uint64_t* pfull = empty + kGuStages;    // [2] partial written
  uint64_t* pempty = pfull + 2;           // [2] partial added to the registers
  uint64_t* sfull = pempty + 2;           // [2] corrections of a tile written
  uint64_t* sempty = sfull + 2;           // [2] corrections read
  uint64_t* drain = sempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();       // the tile plan and activation planes
  pdl_trigger();
  const int n_tiles = *args.n_mtiles * args.n_tiles_n;
  if ((int)blockIdx.x >= n_tiles) return;
  const int my_tiles = (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1;
  const int ksteps = args.K / kTcK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGuStages; ++s) {
      // one barrier per stage: the TMA thread's byte count and every producer
      mbar_init(&full_a[s], 1 + kGuProducers);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], kGuPromoters);
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], kGuPromoters);
    }
    mbar_init(drain, 1);
    *flag = 0;
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&amap) : "memory");
  }
  const uint32_t tmem = tc_alloc_all(tmem_slot, warp);

  if (warp == 0) {
    if (lane == 0)
      tc_tma_role<0, kGuStages, kGuStageBytes>(&amap, args, my_tiles, ksteps, stage_base, full_a,
                                               empty, flag);
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc_idesc(kTcM, kGuN);
      const uint64_t d0 = sw128_desc(stage_base);
      const uint32_t d0_lo = (uint32_t)d0, d_hi = (uint32_t)(d0 >> 32);
      constexpr uint32_t kA16 = kATile >> 4, kB16 = kGuBTile >> 4, kStage16 = kGuStageBytes >> 4;
      int s = 0, pc = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int b = i & 1, use = i >> 1;
        if (use > 0 && !mbar_wait(&sempty[b], (use - 1) & 1)) {
          tc_fail(flag, args.status);
          ok = false;
        }
        const uint32_t dsmall = tmem + (uint32_t)(kGuSCol + b * kGuN);
        uint32_t dpart = tmem;
        int c = 0;
        for (int kk = 0; kk < ksteps && ok; ++kk) {
          if (kk % kGuPeriod == 0) {
            c = pc & 1;
            const int n = pc >> 1;
            if (n > 0 && !mbar_wait(&pempty[c], (n - 1) & 1)) {
              tc_fail(flag, args.status);
              ok = false;
              break;
            }
            dpart = tmem + (uint32_t)(c * kGuN);
            // the promoters' reads of this partial (and of S) precede the MMAs
            tc_fence_after();
          }
          if (!mbar_wait(&full_a[s], phase)) {
            tc_fail(flag, args.status);
            ok = false;
            break;
          }
          const uint32_t ahi = d0_lo + (uint32_t)s * kStage16, alo = ahi + kA16;
          const uint32_t bhi = ahi + 2 * kA16, blo = bhi + kB16;
          const bool first_p = kk % kGuPeriod == 0;
#pragma unroll
          for (int k16 = 0; k16 < kTcK / 16; ++k16) {
            const uint32_t adv = (uint32_t)((k16 * 32) >> 4);   // +32 bytes per k16
            tc_mma_lo(dpart, ahi + adv, bhi + adv, d_hi, idesc, (!first_p || k16 > 0) ? 1u : 0u);
            tc_mma_lo(dsmall, ahi + adv, blo + adv, d_hi, idesc, (kk > 0 || k16 > 0) ? 1u : 0u);
            tc_mma_lo(dsmall, alo + adv, bhi + adv, d_hi, idesc, 1u);
          }
          tc_commit(&empty[s]);   // stage s free once these MMAs complete
          if (++s == kGuStages) {
            s = 0;
            phase ^= 1u;
          }
          if (kk % kGuPeriod == kGuPeriod - 1 || kk == ksteps - 1) {
            tc_commit(&pfull[c]);
            ++pc;
          }
        }
        if (!ok) tc_commit(&pfull[c]);   // wake the promoters; they see the flag
        tc_commit(&sfull[b]);
      }
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp < kGuProm0) {
    tc_producer_role<QT, 0, kGuStages, kGuStageBytes, 2 * kATile, kGuBTile>(
        args, warp - 2, lane, my_tiles, ksteps, stage_base, full_a, empty, flag);
  } else {
    // promoters: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (tile rows)
    // and owns gate columns [32 hh, 32 hh + 32) and the matching up columns
    const int q = warp & 3, hh = (warp - kGuProm0) >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const int nper = (ksteps + kGuPeriod - 1) / kGuPeriod;
    int pc = 0;
    bool ok = true;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const TcTile tt = tc_tile<0>(args, blockIdx.x + i * gridDim.x);
      const int row = tt.row0 + r;
      const bool valid = row < args.offsets[tt.e + 1];
      const float rs = valid ? args.row_scale[row] : 0.f;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      // adds 64 columns of tensor memory at `base` (32 gate, 32 up) into acc
      auto gather = [&](uint32_t base) {
#pragma unroll
        for (int part = 0; part < 4; ++part) {
          const uint32_t col = (part < 2 ? 0u : (uint32_t)kGuFRows) + 32u * hh + 16u * (part & 1);
          float v[16];
          tmem_ld16(base + col, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[16 * part + j] = __fadd_rn(acc[16 * part + j], v[j]);
        }
      };
      for (int per = 0; per < nper; ++per) {
        const int c = pc & 1, n = pc >> 1;
        if (!warp_mbar_wait(&pfull[c], n & 1, lane)) {
          if (lane == 0) tc_fail(flag, args.status);
          ok = false;
          break;
        }
        tc_fence_after();
        if (__shfl_sync(0xffffffffu, *flag, 0)) {
          ok = false;
          break;
        }
        gather(lane_base + (uint32_t)(c * kGuN));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[c]);
        ++pc;
      }
      if (!ok) break;
      const int b = i & 1, use = i >> 1;
      if (!warp_mbar_wait(&sfull[b], use & 1, lane)) {
        if (lane == 0) tc_fail(flag, args.status);
        break;
      }
      tc_fence_after();
      if (__shfl_sync(0xffffffffu, *flag, 0)) break;
      gather(lane_base + (uint32_t)(kGuSCol + b * kGuN));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[b]);
      if (valid) {
        __half* hi = args.h_planes + (size_t)row * args.F + tt.n0 + 32 * hh;
        __half* lo = args.h_planes + ((size_t)args.P + row) * args.F + tt.n0 + 32 * hh;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            float hv[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int col = 8 * c8 + j + k;
              const float h = expert_act(args.act, acc[col] * rs) * (acc[32 + col] * rs);
              hv[k] = h * kTcHScale;
              if (!(fabsf(hv[k]) <= 65504.f)) set_status(args.status, MOE_STATUS_ROW_OVERFLOW);
            }
            const __half2 hh2 = __floats2half2_rn(hv[0], hv[1]);
            const float2 hf = __half22float2(hh2);
            const __half2 ll = __floats2half2_rn(hv[0] - hf.x, hv[1] - hf.y);
            hw[j / 2] = *reinterpret_cast<const uint32_t*>(&hh2);
            lw[j / 2] = *reinterpret_cast<const uint32_t*>(&ll);
          }
          reinterpret_cast<uint4*>(hi)[c8] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          reinterpret_cast<uint4*>(lo)[c8] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    }
  }
  tc_dealloc_all(tmem, warp);
}

// ---------------------------------------------------------------------------
// down: 128 x 256 tiles (128 x 128 for a last, narrower one), 2 stages of
// 96 KB, a "big" accumulator for x_hi * w_hi in tensor-memory columns
// [0, 256) and a "small" one for the corrections in [256, 512), added with
// round-to-nearest in the epilogue.  Warps: 0 TMA, 1 MMA, 2-17 weight
// producers (one per 16-row strip), 18-21 epilogue.
// ---------------------------------------------------------------------------
template <int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_down_kernel(const __grid_constant__ CUtensorMap amap, const TcArgs args) {
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + kTcStages * kStageBytes);
  uint64_t* empty = full_a + kTcStages;
  uint64_t* tfull = empty + kTcStages;    // accumulators written
  uint64_t* tempty = tfull + 1;           // accumulators read out
  uint64_t* drain = tempty + 1;           // the issuer's last MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Down reads the tile plan at once (complete, because gate/up triggers only
  // after its own wait) and waits for gate/up's hidden planes only in its
  // activation producer, so its weight producers start early.
  pdl_trigger();
  const int n_tiles = *args.n_mtiles * args.n_tiles_n;
  if ((int)blockIdx.x >= n_tiles) return;
  const int my_tiles = (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1;
  const int ksteps = args.K / kTcK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full_a[s], 1 + kTcProducers);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kTcEpiWarps);
    mbar_init(drain, 1);
    *flag = 0;
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&amap) : "memory");
  }
  const uint32_t tmem = tc_alloc_all(tmem_slot, warp);

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      tc_tma_role<1, kTcStages, kStageBytes>(&amap, args, my_tiles, ksteps, stage_base, full_a,
                                             empty, flag);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // descriptor of stage 0's A-hi tile; every other operand tile of every
      // stage differs from it only in the start-address field (addr >> 4 < 2^14)
      const uint64_t d0 = sw128_desc(stage_base);
      const uint32_t d0_lo = (uint32_t)d0, d_hi = (uint32_t)(d0 >> 32);
      constexpr uint32_t kA16 = kATile >> 4, kStage16 = kStageBytes >> 4;
      const uint32_t dbig = tmem, dsmall = tmem + (uint32_t)kTcSmallCol;
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const uint32_t idesc = tc_idesc(kTcM, tc_tile<1>(args, blockIdx.x + i * gridDim.x).nr);
        if (i > 0 && !mbar_wait(tempty, (i - 1) & 1)) {
          tc_fail(flag, args.status);
          ok = false;
        }
        // the epilogue's tensor-memory reads of the previous tile precede these MMAs
        tc_fence_after();
        for (int kk = 0; kk < ksteps && ok; ++kk) {
          // the stage's one barrier (the TMA bytes and every weight producer)
          // orders the producers' proxy-fenced stores and the TMA bytes before
          // the MMAs' shared-memory reads
          if (!mbar_wait(&full_a[s], phase)) {
            tc_fail(flag, args.status);
            ok = false;
            break;
          }
          const uint32_t ahi = d0_lo + (uint32_t)s * kStage16, alo = ahi + kA16;
          const uint32_t bhi = ahi + 2 * kA16, blo = bhi + (kBTile >> 4);
#pragma unroll
          for (int k16 = 0; k16 < kTcK / 16; ++k16) {
            const uint32_t adv = (uint32_t)((k16 * 32) >> 4);   // +32 bytes per k16
            const uint32_t acc = (kk > 0 || k16 > 0) ? 1u : 0u;
            tc_mma_lo(dbig, ahi + adv, bhi + adv, d_hi, idesc, acc);
            tc_mma_lo(dsmall, ahi + adv, blo + adv, d_hi, idesc, acc);
            tc_mma_lo(dsmall, alo + adv, bhi + adv, d_hi, idesc, 1u);
          }
          tc_commit(&empty[s]);   // stage s free once these MMAs complete
          if (++s == kTcStages) {
            s = 0;
            phase ^= 1u;
          }
        }
        tc_commit(tfull);         // accumulators complete (or abandoned: the flag is set)
      }
      // every MMA issued here completes before the tensor memory is released
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp < kTcEpi0) {
    tc_producer_role<QT, 1, kTcStages, kStageBytes, 2 * kATile, kBTile>(
        args, warp - kTcProd0, lane, my_tiles, ksteps, stage_base, full_a, empty, flag);
  } else {
    // epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (= tile rows)
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
    for (int i = 0; i < my_tiles; ++i) {
      const TcTile tt = tc_tile<1>(args, blockIdx.x + i * gridDim.x);
      const int row = tt.row0 + r;
      const bool valid = row < args.offsets[tt.e + 1];
      const int orow = valid ? (args.y_rows ? args.y_rows[row] : row) : 0;
      const bool got = warp_mbar_wait(tfull, i & 1, lane);
      tc_fence_after();
      if (!got) {
        if (lane == 0) tc_fail(flag, args.status);
        break;
      }
      if (__shfl_sync(0xffffffffu, *flag, 0)) break;
      const float osc = (1.f / kTcHScale) * (args.down_scale ? args.down_scale[tt.e] : 1.f);
#pragma unroll 1
      for (int c = 0; c < tt.nr; c += 16) {
        float v[16];
        tmem_ld_pair(taddr + c, v);
        if (valid) {
          float4* dst = reinterpret_cast<float4*>(args.y + (size_t)orow * args.d + tt.n0 + c);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_float4(v[4 * j] * osc, v[4 * j + 1] * osc, v[4 * j + 2] * osc,
                                 v[4 * j + 3] * osc);
        }
      }
      // the next tile may overwrite the accumulators once every epilogue warp has read them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
    }
  }
  tc_dealloc_all(tmem, warp);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D map over [rows][cols] fp16, box box_rows x 64 cols, 128-byte swizzle.
int make_plane_map(CUtensorMap* map, const __half* base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  MOE_REQUIRE(fn, MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  MOE_REQUIRE(((uintptr_t)base & 15) == 0 && (cols * 2) % 16 == 0, MOE_ERR_INVALID,
              "plane not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTcK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MOE_REQUIRE(r == CUDA_SUCCESS, MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MOE_OK;
}

int launch_tile_plan(const int32_t* offsets, int E, int tm, int max_tiles, int* tile_e,
                     int* tile_r0, int* n_tiles, cudaStream_t s) {
  tc_tile_plan_kernel<<<1, 1024, 0, s>>>(offsets, E, tm, max_tiles, tile_e, tile_r0, n_tiles);
  return check_launch("tile plan");
}

int launch_act_planes(const float* x, const int32_t* x_rows, int x_div, const float* x_row_max,
                      int P, const int32_t* offsets, int E, int d, float* row_scale,
                      __half* planes, cudaStream_t s) {
  tc_prep_kernel<<<(P + 7) / 8, 256, 0, s>>>(x, x_rows, x_div, x_row_max, P, offsets, E, d,
                                             row_scale, planes);
  return check_launch("activation planes");
}

struct TcWs {
  int* n_mtiles;
  int* tile_e;
  int* tile_r0;
  float* row_scale;
  __half* x_planes;   // [2][P][d]
  __half* h_planes;   // [2][P][F]
  size_t bytes;
};

static int tc_max_tiles(int rows, int E) { return (rows + kTcM - 1) / kTcM + E; }

static TcWs carve_tc(void* ws, int rows, int E, int d, int F) {
  Carve c{static_cast<uint8_t*>(ws), 0, 0};
  TcWs w;
  const int mt = tc_max_tiles(rows, E);
  c.take<int>(64);  // status word
  w.n_mtiles = c.take<int>(64);
  w.tile_e = c.take<int>(mt);
  w.tile_r0 = c.take<int>(mt);
  w.row_scale = c.take<float>(rows);
  w.x_planes = c.take<__half>((size_t)2 * rows * d);
  w.h_planes = c.take<__half>((size_t)2 * rows * F);
  w.bytes = align_up(c.used, 256);
  return w;
}

size_t tc_workspace(int rows, int E, int d, int F) { return carve_tc(nullptr, rows, E, d, F).bytes; }

bool tc_supported(int rows, int E, int d, int F) {
  return rows > 0 && E <= 1024 && d % 128 == 0 && F % 64 == 0;
}

template <int QT>
static int launch_tc(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down,
                     const int32_t* offsets, int E, int rows, const float* x,
                     const int32_t* x_rows, int x_div, const float* x_row_max, int d, int F,
                     float* y, const int32_t* y_rows, const TcWs& w, int* status,
                     const moe_expert_opts* opts, cudaStream_t s) {
  using Tr = QTraits<QT>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev));
  if (!((attr_set >> (dev & 63)) & 1ull)) {
    MOE_CUDA(cudaFuncSetAttribute(tc_gateup_kernel<QT>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kGuSmem));
    MOE_CUDA(cudaFuncSetAttribute(tc_down_kernel<QT>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
    attr_set |= 1ull << (dev & 63);
  }
  static int sm_count[64] = {};
  if (!sm_count[dev & 63])
    MOE_CUDA(cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev));
  const int sms = sm_count[dev & 63];
  const int max_tiles = tc_max_tiles(rows, E);
  {
    ::moe::ProfScope _prof(MOE_K_PLAN, s);
    MOE_CHECK(launch_tile_plan(offsets, E, kTcM, max_tiles, w.tile_e, w.tile_r0, w.n_mtiles, s));
  }
  {
    ::moe::ProfScope _prof(MOE_K_XPREP, s);
    MOE_CHECK(launch_act_planes(x, x_rows, x_div, x_row_max, rows, offsets, E, d, w.row_scale,
                                w.x_planes, s));
  }
  CUtensorMap xmap, hmap;
  MOE_CHECK(make_plane_map(&xmap, w.x_planes, 2 * rows, d, kTcM));
  MOE_CHECK(make_plane_map(&hmap, w.h_planes, 2 * rows, F, kTcM));
  const size_t mat_bytes = (size_t)F * (d / 32) * Tr::kBlockBytes;
  TcArgs a1 = {};
  a1.w0 = w_gate;
  a1.w1 = w_up;
  a1.mat_bytes = (opts && opts->gate_up_stride) ? opts->gate_up_stride : mat_bytes;
  a1.act = opts ? opts->act : MOE_ACT_SWIGLU;
  a1.K = d;
  a1.n_tiles_n = F / kGuFRows;
  a1.P = rows;
  a1.F = F;
  a1.d = d;
  a1.offsets = offsets;
  a1.tile_e = w.tile_e;
  a1.tile_r0 = w.tile_r0;
  a1.n_mtiles = w.n_mtiles;
  a1.row_scale = w.row_scale;
  a1.h_planes = w.h_planes;
  a1.status = status;
  {
    ::moe::ProfScope _prof(MOE_K_GATEUP, s);
    // persistent: one CTA per SM at most, each walking its share of the tiles
    const int grid = std::min(max_tiles * a1.n_tiles_n, sms);
    MOE_CUDA(launch_pdl(tc_gateup_kernel<QT>, dim3(grid), dim3(kGuThreads), kGuSmem, s, xmap, a1));
  }
  MOE_CHECK(check_launch("tc_gemm gate/up"));
  TcArgs a2 = a1;
  a2.w0 = w_down;
  a2.w1 = nullptr;
  a2.mat_bytes = mat_bytes;
  a2.down_scale = opts ? opts->down_scale : nullptr;
  a2.K = F;
  a2.n_tiles_n = (d + kTcNMax - 1) / kTcNMax;
  a2.y = y;
  a2.y_rows = y_rows;
  {
    ::moe::ProfScope _prof(MOE_K_DOWN, s);
    const int grid = std::min(max_tiles * a2.n_tiles_n, sms);
    MOE_CUDA(launch_pdl(tc_down_kernel<QT>, dim3(grid), dim3(kTcThreads), kTcSmem, s, hmap, a2));
  }
  return check_launch("tc_gemm down");
}

int run_experts_tc(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                   int x_div, const float* x_row_max, int d, int F, float* y,
                   const int32_t* y_rows, void* ws, size_t ws_bytes, int* status,
                   const moe_expert_opts* opts, cudaStream_t s) {
  MOE_REQUIRE(tc_supported(rows, E, d, F), MOE_ERR_UNSUPPORTED, "tensor-core path shape");
  TcWs w = carve_tc(ws, rows, E, d, F);
  MOE_REQUIRE(ws_bytes >= w.bytes, MOE_ERR_WORKSPACE, "tensor-core workspace %zu < %zu",
              ws_bytes, w.bytes);
  if (!status) status = static_cast<int*>(ws);
  if (qtype == MOE_Q4_0)
    return launch_tc<MOE_Q4_0>(w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div,
                               x_row_max, d, F, y, y_rows, w, status, opts, s);
  return launch_tc<MOE_Q8_0>(w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div, x_row_max,
                             d, F, y, y_rows, w, status, opts, s);
}

}  // namespace moe
