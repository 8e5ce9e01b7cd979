// tcgen05 / TMA building blocks shared by the tensor-core expert kernels
// (prefill.cu: split-operand GEMMs for large row groups; blockscale.cu:
// integer-weight GEMMs with per-block scaling for mid-size groups).
#pragma once
#include <cuda.h>

#include <type_traits>

#include "moe_common.cuh"

namespace moe {

constexpr int kTmemCols = 512;   // a CTA holds all of its SM's tensor memory

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major, 128-byte-swizzled operand tile: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint32_t a = smem_u32(tile);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFF);           // start address
  d |= (uint64_t)1 << 16;                       // leading byte offset (unused when swizzled)
  d |= (uint64_t)(1024 >> 4) << 32;             // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                       // swizzle: 128 B
  return d;
}

// kind::f16 instruction descriptor: f16 A/B, f32 accumulate, K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same MMA with both descriptors given as (low word, shared high word): the
// stage and k offsets only ever change the 14-bit start-address field.
__device__ __forceinline__ void tc_mma_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                          uint32_t desc_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b64 da, db;\n setp.ne.b32 p, %5, 0;\n"
      " mov.b64 da, {%1, %3};\n mov.b64 db, {%2, %3};\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// L2 prefetch of one 128 x 64 box of a tensor map (no shared-memory write)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// ---------------------------------------------------------------------------
// weight dequantisation into the swizzled B tile
// ---------------------------------------------------------------------------
// Registers of one half of a packed 16-row x 64-column weight tile for one
// lane: half 0 holds the lane's row g, half 1 its row g + 8 (lane = 4g + t).
template <int QT>
struct PackedHalf {
  typename std::conditional<QT == MOE_Q8_0, uint4, uint2>::type q;
  uint32_t sc;   // the two fp16 block scales of that row
};

template <int QT>
__device__ __forceinline__ void load_packed_half(PackedHalf<QT>& p, const uint8_t* tile, int lane,
                                                 int half) {
  using Tr = QTraits<QT>;
  const uint8_t* qp = tile + lane * Tr::kLaneBytes;
  if constexpr (QT == MOE_Q8_0) p.q = __ldg(reinterpret_cast<const uint4*>(qp + 16 * half));
  else p.q = __ldg(reinterpret_cast<const uint2*>(qp + 8 * half));
  p.sc = __ldg(reinterpret_cast<const uint32_t*>(tile + Tr::kTileQuant + (lane >> 2) * 8 +
                                                 4 * half));
}

// w = d * q split into fp16 hi = rn(w) and lo = rn(w - hi), two at a time:
// the f16x2 multiply rounds the exact product, and the fused multiply-add
// rounds the exact residual d*q - hi (d: fp16, q: small integer, so both are
// what an f32 detour would give).
__device__ __forceinline__ void split_mul2(uint32_t q2, uint32_t d2, uint32_t& hi, uint32_t& lo) {
  asm("{\n .reg .b32 nh;\n mul.rn.f16x2 %0, %2, %3;\n neg.f16x2 nh, %0;\n"
      " fma.rn.f16x2 %1, %2, %3, nh;\n}"
      : "=r"(hi), "=r"(lo)
      : "r"(q2), "r"(d2));
}

// One packed half tile (registers) -> row r0 + g + 8 * half of the swizzled hi
// / lo B tiles.  Lane (g, t) owns, per 32-wide block, the elements its fragment
// layout assigns to t.  Quants become exact fp16 integers (magic-number adds),
// then d * q is split in packed fp16 math.  Odd rows write their blocks in the
// opposite order so the lanes of a store phase hit distinct 16-byte chunks (no
// bank conflicts).
template <int QT>
__device__ __forceinline__ void store_packed_half(const PackedHalf<QT>& p, int lane, int half,
                                                  uint8_t* bhi, uint8_t* blo, int r0) {
  const int g = lane >> 2, t = lane & 3;
  const int row = r0 + g + 8 * half;
  uint8_t* hr = bhi + row * 128;
  uint8_t* lr = blo + row * 128;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int b = it ^ (g & 1);
    const uint32_t d2 = prmt(p.sc, p.sc, b ? 0x3232u : 0x1010u);   // {d, d}
    if constexpr (QT == MOE_Q8_0) {
      const uint32_t w0 = b ? p.q.z : p.q.x, w1 = b ? p.q.w : p.q.y;
      uint32_t q[4], h[4], l[4];
      dequant_q8(w0, q[0], q[1]);
      dequant_q8(w1, q[2], q[3]);
#pragma unroll
      for (int i = 0; i < 4; ++i) split_mul2(q[i], d2, h[i], l[i]);
      // elements 32b + 8t .. +7 -> 16-byte chunk 4b + t, swizzled by row
      const int ch = (4 * b + t) ^ (row & 7);
      *reinterpret_cast<uint4*>(hr + ch * 16) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4*>(lr + ch * 16) = make_uint4(l[0], l[1], l[2], l[3]);
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
      uint32_t h0, h1, l0, l1;
      const int ch_lo = (4 * b + (t >> 1)) ^ (row & 7);
      const int ch_hi = (4 * b + 2 + (t >> 1)) ^ (row & 7);
      const int off = (t & 1) * 8;
      split_mul2(lq01, d2, h0, l0);
      split_mul2(lq23, d2, h1, l1);
      *reinterpret_cast<uint2*>(hr + ch_lo * 16 + off) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(lr + ch_lo * 16 + off) = make_uint2(l0, l1);
      split_mul2(hq01, d2, h0, l0);
      split_mul2(hq23, d2, h1, l1);
      *reinterpret_cast<uint2*>(hr + ch_hi * 16 + off) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(lr + ch_hi * 16 + off) = make_uint2(l0, l1);
    }
  }
}

// Every lane polls (the phase, once complete, stays complete until the next
// one can start) and the warp follows the vote; measured faster on B200 than
// lane 0 polling while the other lanes wait on a shuffle (prefill gate/up
// 1.08 -> 1.03 ms).
__device__ __forceinline__ bool warp_mbar_wait(uint64_t* bar, uint32_t parity, int lane) {
  (void)lane;
  return __all_sync(0xffffffffu, mbar_wait(bar, parity) ? 1 : 0) != 0;
}

__device__ __forceinline__ void tc_fail(volatile int* flag, int* status) {
  *flag = 1;
  set_status(status, MOE_STATUS_TIMEOUT);
}

__device__ __forceinline__ void tc_dealloc_all(uint32_t tmem, int warp) {
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols)
                 : "memory");
  }
}

__device__ __forceinline__ uint32_t tc_alloc_all(uint32_t* slot, int warp) {
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "n"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *slot;
}

// host side (prefill.cu)
// 2-D TMA map over [rows][cols] fp16, box box_rows x 64 columns, 128-byte swizzle.
int make_plane_map(CUtensorMap* map, const __half* base, int rows, int cols, int box_rows);
// tiles of tm sorted rows per active expert: tile_e[i], tile_r0[i], *n_tiles
int launch_tile_plan(const int32_t* offsets, int E, int tm, int max_tiles, int* tile_e,
                     int* tile_r0, int* n_tiles, cudaStream_t s);
// routed rows -> fp16 hi / lo planes [2][P][d], scaled per row by a power of two
// (row_scale[r] = the inverse factor)
int launch_act_planes(const float* x, const int32_t* x_rows, int x_div, const float* x_row_max,
                      int P, const int32_t* offsets, int E, int d, float* row_scale,
                      __half* planes, cudaStream_t s);

}  // namespace moe
