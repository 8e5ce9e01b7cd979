// Grouped SwiGLU experts over expert-sorted rows (decode / small-group path).
//
// ExpertFFN.forward (moe_forward.py:129-133) for every routed row at once:
//   h = silu(W_gate x) * (W_up x),  y = W_down h.
//
// Kernels, per call:
//   plan_kernel    active-expert list and 4-row group offsets from expert_offsets
//   gateup_kernel  gathers its expert's rows into shared memory, scales each by
//                  a power of two and splits it into fp16 hi + lo parts laid out
//                  as m16n8k16 B fragments (4 rows x {hi, lo} = the 8 MMA
//                  columns) plus one offset correction per block and column
//                  (below), while the first weight stages are already in
//                  flight; then streams packed W_gate / W_up tiles with 128-bit
//                  loads and
//                  turns each quant into an fp16 subnormal with a bare mask
//                  (Q4_0 nibble n -> n * 2^-24, Q8_0 byte q + 128 -> (q+128) *
//                  2^-24): the tensor core multiplies those exactly, and the
//                  missing "- 8" / "- 128" offset enters as the accumulator's
//                  initial value, -offset * 2^-24 * (sum of the block's
//                  activations).  One pair of MMAs per 32-weight block, then the
//                  block, times its fp16 scale, is added to the fp32 running
//                  sum; the 2^24 comes back with the row scale.  SiLU(gate) * up
//                  in the epilogue, written as fragments for the next GEMV
//   down_kernel    the same for W_down, writing f32 rows of y
// The fp16 hi/lo split keeps ~22 bits of each activation, which is what the
// reference's f32 tolerance needs; a single fp16 rounding does not.
#include <math.h>

#include <algorithm>

#include "moe_common.cuh"

namespace moe {

int raw_rows_per_chunk(int d, int F);   // experts_raw.cu
bool experts_packed(int qtype, int dn_qtype);

constexpr int kMaxCG = 4;                 // column groups (4 rows each) per pass
constexpr float kHScale = 1.0f / 256.0f;  // hidden activations are stored / 256
constexpr float kSubUnit = 16777216.0f;   // 2^24: one fp16 subnormal step
// Activation block record in shared memory: 512 B of fragments, then the
// offset corrections as one f32x4 accumulator quad per lane column t
// ({C[2t], C[2t+1], C[2t], C[2t+1]}), then 16 B of padding so that records of
// consecutive blocks start on different banks.
constexpr int kXRec = 592;

// quant offset removed by the subnormal dequantisation
template <int QT>
__host__ __device__ constexpr float quant_offset() { return QT == MOE_Q4_0 ? 8.f : 128.f; }
constexpr int kPlanThreads = 1024;

__device__ __forceinline__ float half_lo(uint32_t v) {
  return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu)));
}
__device__ __forceinline__ float half_hi(uint32_t v) {
  return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
}

// element of a 32-block held at register slot i (0..7) of lane-column t
template <int QT>
__device__ __forceinline__ constexpr int frag_elem_c(int t, int i) {
  return QT == MOE_Q4_0 ? ((i < 4 ? 0 : 16) + 4 * t + ((i & 3) == 1 ? 2 : ((i & 3) == 2 ? 1 : (i & 3))))
                        : 8 * t + i;
}
// inverse: element e -> (t, i)
template <int QT>
__device__ __forceinline__ void frag_pos(int e, int& t, int& i) {
  if (QT == MOE_Q4_0) {
    int hi = e >= 16;
    int r = e & 15;
    t = r >> 2;
    int m = r & 3;                       // 0,1,2,3 -> slot 0,2,1,3
    i = (hi ? 4 : 0) + (m == 1 ? 2 : (m == 2 ? 1 : m));
  } else {
    t = e >> 3;
    i = e & 7;
  }
}

// ---------------------------------------------------------------------------
// plan: active experts, group offsets, group -> expert map
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kPlanThreads)
plan_kernel(const int32_t* __restrict__ offsets, int E, int rows, int max_groups, int rpc,
            int* __restrict__ n_active, int* __restrict__ active, int* __restrict__ goff,
            int* __restrict__ coff, int* __restrict__ done, int* __restrict__ status) {
  __shared__ int sh[33];
  const int e = threadIdx.x;
  int n = 0;
  if (e < E) {
    n = offsets[e + 1] - offsets[e];
    if (n < 0 || offsets[e] < 0 || offsets[e + 1] > rows) {
      set_status(status, MOE_STATUS_ROW_OVERFLOW);
      n = 0;
    }
  }
  write_expert_plan(n, e, E, rpc, max_groups, sh, n_active, active, goff, coff, done, status);
}

// ---------------------------------------------------------------------------
// tile fragments
// ---------------------------------------------------------------------------
template <int QT>
struct TileRegs {
  uint4 q[QT == MOE_Q4_0 ? 1 : 2];
  uint2 sc;
};

// fragment registers of one staged tile (shared memory, lane-contiguous)
template <int QT>
__device__ __forceinline__ void lds_tile(TileRegs<QT>& r, const uint8_t* tile, int lane) {
  using Tr = QTraits<QT>;
  const uint8_t* qp = tile + lane * Tr::kLaneBytes;
  r.q[0] = *reinterpret_cast<const uint4*>(qp);
  if (QT == MOE_Q8_0) r.q[QT == MOE_Q4_0 ? 0 : 1] = *reinterpret_cast<const uint4*>(qp + 16);
  r.sc = *reinterpret_cast<const uint2*>(tile + Tr::kTileQuant + (lane >> 2) * 8);
}

// Q4_0 quant word -> four fp16x2 subnormals: low nibbles n * 2^-24, high
// nibbles 16 n * 2^-24 (paired with activations stored / 16).
__device__ __forceinline__ void dequant_q4_sub(uint32_t w, uint32_t& lo01, uint32_t& lo23,
                                               uint32_t& hi01, uint32_t& hi23) {
  const uint32_t w8 = w >> 8;
  lo01 = w & 0x000F000Fu;
  lo23 = w8 & 0x000F000Fu;
  hi01 = w & 0x00F000F0u;
  hi23 = w8 & 0x00F000F0u;
}

// Q8_0 quant word -> two fp16x2 subnormals (q + 128) * 2^-24.
__device__ __forceinline__ void dequant_q8_sub(uint32_t w, uint32_t& h01, uint32_t& h23) {
  const uint32_t u = w ^ 0x80808080u;
  h01 = prmt(u, 0u, 0x4140u);
  h23 = prmt(u, 0u, 0x4342u);
}

// A fragments of both k16 steps for block b (rows g and g+8), block scales.
// SUB: subnormal quants (offset handled by the accumulator's initial value);
// otherwise exact signed fp16 integers.
template <int QT, bool SUB>
__device__ __forceinline__ void tile_afrags(const TileRegs<QT>& r, int b, uint32_t (&a0)[4],
                                            uint32_t (&a1)[4], float2& dg, float2& dg8) {
  if (QT == MOE_Q4_0) {
    uint32_t wg = b ? r.q[0].y : r.q[0].x;
    uint32_t w8 = b ? r.q[0].w : r.q[0].z;
    uint32_t l01, l23, h01, h23, m01, m23, n01, n23;
    if (SUB) {
      dequant_q4_sub(wg, l01, l23, h01, h23);
      dequant_q4_sub(w8, m01, m23, n01, n23);
    } else {
      dequant_q4(wg, l01, l23, h01, h23);
      dequant_q4(w8, m01, m23, n01, n23);
    }
    a0[0] = l01; a0[1] = m01; a0[2] = l23; a0[3] = m23;
    a1[0] = h01; a1[1] = n01; a1[2] = h23; a1[3] = n23;
  } else {
    const uint4& qa = r.q[0];
    const uint4& qb = r.q[QT == MOE_Q4_0 ? 0 : 1];
    uint32_t g0 = b ? qa.z : qa.x, g1 = b ? qa.w : qa.y;
    uint32_t e0 = b ? qb.z : qb.x, e1 = b ? qb.w : qb.y;
    uint32_t x01, x23, y01, y23;
    if (SUB) {
      dequant_q8_sub(g0, x01, x23);
      dequant_q8_sub(e0, y01, y23);
    } else {
      dequant_q8(g0, x01, x23);
      dequant_q8(e0, y01, y23);
    }
    a0[0] = x01; a0[1] = y01; a0[2] = x23; a0[3] = y23;
    if (SUB) {
      dequant_q8_sub(g1, x01, x23);
      dequant_q8_sub(e1, y01, y23);
    } else {
      dequant_q8(g1, x01, x23);
      dequant_q8(e1, y01, y23);
    }
    a1[0] = x01; a1[1] = y01; a1[2] = x23; a1[3] = y23;
  }
  const float s0 = b ? half_hi(r.sc.x) : half_lo(r.sc.x);
  const float s8 = b ? half_hi(r.sc.y) : half_lo(r.sc.y);
  dg = make_float2(s0, s0);
  dg8 = make_float2(s8, s8);
}

// One 32-weight block: two k16 MMAs into an accumulator that starts at c0
// (zero, or the offset corrections of the lane's two columns for rows g and
// g+8), then acc += scale * block (packed f32x2 FMA).  acc[0]: row g,
// acc[1]: row g+8.
__device__ __forceinline__ void block_mma(float2 (&acc)[2], const uint32_t (&a0)[4],
                                          const uint32_t (&a1)[4], uint4 xf, float4 c0, float2 dg,
                                          float2 dg8) {
  const float init[4] = {c0.x, c0.y, c0.z, c0.w};
  float tmp[4];
  mma_16816(tmp, a0[0], a0[1], a0[2], a0[3], xf.x, xf.y, init);
  mma_16816(tmp, a1[0], a1[1], a1[2], a1[3], xf.z, xf.w, tmp);
  acc[0] = __ffma2_rn(dg, make_float2(tmp[0], tmp[1]), acc[0]);
  acc[1] = __ffma2_rn(dg8, make_float2(tmp[2], tmp[3]), acc[1]);
}

// Bulk-copy ring geometry: U tiles (of each matrix) per stage, stages per warp.
// The split-K reduction buffer (NCG KB per warp) aliases a gate/up ring.
template <int QT> struct Ring;
template <> struct Ring<MOE_Q4_0> {
  static constexpr int kGuU = 3, kGuStages = 2, kDnU = 4, kDnStages = 3;
};
template <> struct Ring<MOE_Q8_0> {
  static constexpr int kGuU = 2, kGuStages = 2, kDnU = 2, kDnStages = 3;
};

constexpr int kGuWarps = 16;            // warps per gate/up CTA
constexpr int kGuMaxCG = 4;             // column groups per pass of either GEMV (registers)
constexpr int kDnWarps = 8;             // warps per down CTA
constexpr int kBarArea = 1024;          // mbarriers: 1 + warps x stages, 8 B each
constexpr int kMaxSmem = 227 * 1024;    // dynamic shared memory per CTA on sm_100
__host__ __device__ inline int x_stage_bytes(int K, int cgp) { return cgp * (K / 32) * 512; }
__host__ __device__ inline int gu_x_stage_bytes(int K, int cgp) { return cgp * (K / 32) * kXRec; }

template <int QT>
__host__ __device__ constexpr int gu_stage_bytes() {
  return 2 * Ring<QT>::kGuU * QTraits<QT>::kTileBytes;
}
template <int QT>
__host__ __device__ constexpr int dn_stage_bytes() {
  return Ring<QT>::kDnU * QTraits<QT>::kTileBytes;
}

// Bounded wait (thread-level) until *p >= target, with acquire semantics at
// GPU scope: gives up after ~0.2 s of wall time or 2^22 polls.
__device__ __forceinline__ bool wait_count(const int* p, int target) {
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if ((it & 63u) == 0u) {
      const uint64_t now = globaltimer_ns();
      if (it == 0u) t0 = now;
      else if (now - t0 > 200000000ull) return false;
    }
    __nanosleep(128);
  }
  return false;
}

// Per-CTA state of a gate/up work item.
struct GuCtx {
  const uint8_t* gbase;   // this warp's strip of W_gate (tile 0)
  const uint8_t* ubase;   // ... of W_up
  uint8_t* ring;          // this warp's stages
  uint64_t* bars;         // this warp's stage barriers
  const uint8_t* xs;      // activation fragments (shared)
  const float* rs;        // row scales of the chunk's rows (shared)
  uint8_t* hfrag;
  int* status;
  uint64_t pol;
  int nst, jb, ntile, nbx, nbF, ks, kp, s, row0, n, G0, lane, act;
  int xt0;          // first tile (of the warp's K slice) whose activations are staged
  bool strip_ok;
};

// Stage q of this warp's (gate, up) tiles into ring slot `slot` (lane 0).
template <int QT>
__device__ __forceinline__ void gu_issue(const GuCtx& c, int q, int slot) {
  using Tr = QTraits<QT>;
  constexpr int U = Ring<QT>::kGuU;
  constexpr int TB = Tr::kTileBytes;
  constexpr int SB = U * TB;
  const int t0 = q * U;
  const uint32_t bytes = (uint32_t)(min(U, c.ntile - t0) * TB);
  uint8_t* st = c.ring + slot * 2 * SB;
  mbar_expect_tx(&c.bars[slot], 2 * bytes);
  bulk_g2s(st, c.gbase + (size_t)(c.jb + t0) * TB, bytes, &c.bars[slot], c.pol);
  bulk_g2s(st + SB, c.ubase + (size_t)(c.jb + t0) * TB, bytes, &c.bars[slot], c.pol);
}

// First stages of a chunk, issued before the activations are built.
template <int QT>
__device__ __forceinline__ void gu_prefetch(const GuCtx& c) {
  constexpr int U = Ring<QT>::kGuU;
  const int nstage = (c.ntile + U - 1) / U;
  if (c.lane == 0 && c.strip_ok) {
    fence_proxy_async_smem();
    for (int q = 0; q < min(c.nst, nstage); ++q) gu_issue<QT>(c, q, q);
  }
}

// Streams this warp's tiles through its ring for one chunk of NCG column
// groups.  Lane 0 keeps up to nst stages of U (gate, up) tile pairs in flight
// with bulk copies (the first ones from gu_prefetch); every lane reads its
// fragments of a whole stage from shared memory, releases the stage, then
// computes.  False if a wait timed out.
template <int QT, int NCG>
__device__ __forceinline__ bool gu_stream(float2 (&accg)[NCG][2], float2 (&accu)[NCG][2],
                                          const GuCtx& c, uint32_t& parity, int q0, int q1) {
  using Tr = QTraits<QT>;
  constexpr int U = Ring<QT>::kGuU;
  constexpr int TB = Tr::kTileBytes;
  constexpr int SB = U * TB;
  constexpr int STAGE = 2 * SB;
  const int nstage = (c.ntile + U - 1) / U;
  const int cs = c.nbx * kXRec;
  // activation records of the staged blocks: tile t of the warp's K slice is
  // at records 2 (jb + t - xt0) and + 1 of each column group
  const int rec0 = 2 * (c.jb + q0 * U - c.xt0);
  const uint8_t* xq = c.xs + c.lane * 16 + rec0 * kXRec;
  const uint8_t* cq = c.xs + 512 + (c.lane & 3) * 16 + rec0 * kXRec;
  int slot = q0 % c.nst;
  for (int q = q0; q < q1; ++q) {
    if (!mbar_wait(&c.bars[slot], (parity >> slot) & 1u)) return false;
    parity ^= 1u << slot;
    const int nt = min(U, c.ntile - q * U);
    const uint8_t* st = c.ring + slot * STAGE;
    TileRegs<QT> tg[U], tu[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < nt) {
        lds_tile<QT>(tg[u], st + u * TB, c.lane);
        lds_tile<QT>(tu[u], st + SB + u * TB, c.lane);
      }
    }
    __syncwarp();
    if (c.lane == 0 && q + c.nst < nstage) {
      fence_proxy_async_smem();
      gu_issue<QT>(c, q + c.nst, slot);
    }
    slot = (slot + 1 == c.nst) ? 0 : slot + 1;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < nt) {
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t ga0[4], ga1[4], ua0[4], ua1[4];
          float2 dg, dg8, du, du8;
          tile_afrags<QT, true>(tg[u], b, ga0, ga1, dg, dg8);
          tile_afrags<QT, true>(tu[u], b, ua0, ua1, du, du8);
#pragma unroll
          for (int cg = 0; cg < NCG; ++cg) {
            const int off = cg * cs + (2 * u + b) * kXRec;
            const uint4 xf = *reinterpret_cast<const uint4*>(xq + off);
            const float4 c0 = *reinterpret_cast<const float4*>(cq + off);
            block_mma(accg[cg], ga0, ga1, xf, c0, dg, dg8);
            block_mma(accu[cg], ua0, ua1, xf, c0, du, du8);
          }
        }
      }
    }
    xq += U * 2 * kXRec;
    cq += U * 2 * kXRec;
  }
  return true;
}

// One chunk of NCG column groups: stream, split-K reduction across the
// warps of a strip (rank order), SiLU(gate) * up epilogue into hidden
// fragments.  Called uniformly by every warp of the CTA.
// What a chunk needs to (re)build its activation records: with pt < the
// tiles of K, the records are staged one K phase of pt tiles at a time (more
// column groups than the whole of K would leave room for), the CTA meeting at
// a barrier between phases; the weight rings stream on across the barrier.
struct GuBuild {
  const float* x;
  const int32_t* x_rows;
  const float* x_row_max;
  float* rs;
  float* rmax;
  int x_div, ncg, d, pt;
};

template <int QT>
__device__ __forceinline__ void build_x_stage(uint8_t* xs, float* rs, float* rmax,
                                              const float* __restrict__ x,
                                              const int32_t* __restrict__ x_rows, int x_div,
                                              const float* __restrict__ x_row_max, int row0,
                                              int c0, int n, int ncg, int d, int b0, int nbp,
                                              int cgs);

template <int QT, int NCG>
__device__ __forceinline__ bool gu_chunk(GuCtx c, uint32_t& parity, int c0, bool ok,
                                         const GuBuild& bd) {
  constexpr int U = Ring<QT>::kGuU;
  float2 accg[NCG][2], accu[NCG][2];
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
    for (int i = 0; i < 2; ++i) accg[cg][i] = accu[cg][i] = make_float2(0.f, 0.f);
  const int JT = bd.d / 64;
  const int nstage = (c.ntile + U - 1) / U;
  for (int t0 = 0; t0 < JT; t0 += bd.pt) {
    const int t1 = min(JT, t0 + bd.pt);
    if (t0 > 0) __syncthreads();   // every warp is done with the previous phase's records
    build_x_stage<QT>(const_cast<uint8_t*>(c.xs), bd.rs, bd.rmax, bd.x, bd.x_rows, bd.x_div,
                      bd.x_row_max, c.row0, c0, c.n, bd.ncg, bd.d, 2 * t0, 2 * (t1 - t0),
                      c.nbx);
    __syncthreads();
    c.xt0 = t0;
    // one phase covers all of K (any K split), or phases of whole stages (no split)
    const int q0 = t0 == 0 && t1 == JT ? 0 : t0 / U;
    const int q1 = t0 == 0 && t1 == JT ? nstage : (t1 + U - 1) / U;
    if (c.strip_ok && ok) {
      if (!gu_stream<QT, NCG>(accg, accu, c, parity, q0, q1)) {
        set_status(c.status, MOE_STATUS_TIMEOUT);
        ok = false;
      }
    }
  }
  const int lane = c.lane;
  if (c.ks > 1) {
    // partial sums of the K-slices meet in the (now idle) rings
    float* red = reinterpret_cast<float*>(c.ring);
    constexpr int RING = Ring<QT>::kGuStages * gu_stage_bytes<QT>();
    (void)RING;
    __syncthreads();
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        red[(cg * 8 + 2 * i) * 32 + lane] = accg[cg][i].x;
        red[(cg * 8 + 2 * i + 1) * 32 + lane] = accg[cg][i].y;
        red[(cg * 8 + 4 + 2 * i) * 32 + lane] = accu[cg][i].x;
        red[(cg * 8 + 5 + 2 * i) * 32 + lane] = accu[cg][i].y;
      }
    __syncthreads();
    if (c.kp == 0) {
      for (int q = 1; q < c.ks; ++q) {
        const float* rq = reinterpret_cast<const float*>(c.ring + q * c.nst * gu_stage_bytes<QT>());
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            accg[cg][i].x += rq[(cg * 8 + 2 * i) * 32 + lane];
            accg[cg][i].y += rq[(cg * 8 + 2 * i + 1) * 32 + lane];
            accu[cg][i].x += rq[(cg * 8 + 4 + 2 * i) * 32 + lane];
            accu[cg][i].y += rq[(cg * 8 + 5 + 2 * i) * 32 + lane];
          }
      }
    }
  }
  if (c.kp == 0 && c.strip_ok) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        accg[cg][i].x += __shfl_xor_sync(0xffffffffu, accg[cg][i].x, 2);
        accg[cg][i].y += __shfl_xor_sync(0xffffffffu, accg[cg][i].y, 2);
        accu[cg][i].x += __shfl_xor_sync(0xffffffffu, accu[cg][i].x, 2);
        accu[cg][i].y += __shfl_xor_sync(0xffffffffu, accu[cg][i].y, 2);
      }
    if (t < 2) {
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) {
        const int G = c.G0 + c0 / 4 + cg;
#pragma unroll
        for (int ci = 0; ci < 2; ++ci) {
          const int rig = 2 * t + ci;              // row inside the group
          const int tok = c0 + 4 * cg + rig;
          if (tok >= c.n) continue;
          const float rs = c.rs[4 * cg + rig] * kSubUnit;
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const float gacc = ci ? accg[cg][rr].y : accg[cg][rr].x;
            const float uacc = ci ? accu[cg][rr].y : accu[cg][rr].x;
            const float h = expert_act(c.act, gacc * rs) * (uacc * rs);
            const float hsc = h * kHScale;
            if (!(fabsf(hsc) <= 65504.f)) set_status(c.status, MOE_STATUS_ROW_OVERFLOW);
            const __half hh = __float2half_rn(hsc);
            const __half hl = __float2half_rn(hsc - __half2float(hh));
            const int f = c.s * 16 + g + 8 * rr;
            int tf, fi;
            frag_pos<QT>(f & 31, tf, fi);
            uint8_t* dst =
                c.hfrag + ((size_t)G * c.nbF + (f >> 5)) * 512 + rig * 64 + tf * 16 + fi * 2;
            *reinterpret_cast<__half*>(dst) = hh;
            *reinterpret_cast<__half*>(dst + 256) = hl;
          }
        }
      }
    }
  }
  return ok;
}

// ---------------------------------------------------------------------------
// Activations of one chunk (ncg groups of 4 rows, from row c0 of the expert)
// -> shared fragment records, plus each row's scale.  Rows past the expert's
// end are zero.  Each row is scaled by a power of two so that its max |x|
// lands in [2^14, 2^15), then split into fp16 hi + lo; for Q4_0 the high-nibble
// half of every block is stored / 16 (exact: it meets nibbles that a bare mask
// leaves 16x too large).  The correction of column n (hi or lo part of a row)
// is -offset * 2^-24 * the block's sum of that part as the MMA sees it.
template <int QT>
__device__ __forceinline__ void build_x_stage(uint8_t* xs, float* rs, float* rmax,
                                              const float* __restrict__ x,
                                              const int32_t* __restrict__ x_rows, int x_div,
                                              const float* __restrict__ x_row_max, int row0,
                                              int c0, int n, int ncg, int d, int b0, int nbp,
                                              int cgs) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NT = kGuWarps * 32;
  const int nb = nbp;      // blocks b0 .. b0 + nbp - 1 of the rows (a K phase),
                           // record (cg * cgs + b - b0) for column group cg
  const int nrows = 4 * ncg;
  auto src_of = [&](int rr) -> const float* {
    const int r = row0 + c0 + rr;
    const int sr = x_rows ? x_rows[r] / x_div : r;
    return x + (size_t)sr * d;
  };
  if (b0 > 0) {
    // a later K phase: the rows' maxima and scales are in shared memory already
  } else if (x_row_max) {
    if (tid < nrows) {
      const int r = row0 + c0 + tid;
      rmax[tid] = c0 + tid < n ? x_row_max[x_rows ? x_rows[r] / x_div : r] : 0.f;
    }
  } else {
    for (int rr = warp; rr < nrows; rr += kGuWarps) {
      float m = 0.f;
      if (c0 + rr < n) {
        const float4* src = reinterpret_cast<const float4*>(src_of(rr));
        for (int i = lane; i < d / 4; i += 32) {
          const float4 v = __ldg(src + i);
          m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) rmax[rr] = m;
    }
  }
  __syncthreads();
  if (tid < nrows && b0 == 0) {
    const float m = rmax[tid];
    float inv = 1.f;
    if (m > 0.f && isfinite(m)) inv = ldexpf(1.f, ilogbf(m) - 14);
    rs[tid] = inv;
  }
  const float k = -quant_offset<QT>() / kSubUnit;
  for (int it = tid; it < nrows * nb; it += NT) {
    const int rr = it / nb, b = it - rr * nb;
    const int cg = rr >> 2, w = rr & 3;
    uint8_t* rec = xs + (size_t)(cg * cgs + b) * kXRec;
    float* cor = reinterpret_cast<float*>(rec + 512);
    if (c0 + rr >= n) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(rec + (q >> 2) * 256 + w * 64 + (q & 3) * 16) =
            make_uint4(0, 0, 0, 0);
      cor[4 * (w >> 1) + (w & 1)] = 0.f;
      cor[4 * (w >> 1) + (w & 1) + 2] = 0.f;
      cor[4 * (2 + (w >> 1)) + (w & 1)] = 0.f;
      cor[4 * (2 + (w >> 1)) + (w & 1) + 2] = 0.f;
      continue;
    }
    const float m = rmax[rr];
    float scale = 1.f;
    if (m > 0.f && isfinite(m)) scale = ldexpf(1.f, 14 - ilogbf(m));
    const float4* src = reinterpret_cast<const float4*>(src_of(rr)) + (b0 + b) * 8;
    float v[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 f = __ldg(src + q);
      v[4 * q + 0] = f.x * scale;
      v[4 * q + 1] = f.y * scale;
      v[4 * q + 2] = f.z * scale;
      v[4 * q + 3] = f.w * scale;
    }
    float sum_hi = 0.f, sum_lo = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float div = (QT == MOE_Q4_0 && i >= 4) ? 0.0625f : 1.0f;
        const float mul = (QT == MOE_Q4_0 && i >= 4) ? 16.0f : 1.0f;
        const float a = v[frag_elem_c<QT>(t, i)] * div;
        const float c = v[frag_elem_c<QT>(t, i + 1)] * div;
        const __half ha = __float2half_rn(a), hc = __float2half_rn(c);
        const __half la = __float2half_rn(a - __half2float(ha));
        const __half lc = __float2half_rn(c - __half2float(hc));
        sum_hi += mul * (__half2float(ha) + __half2float(hc));
        sum_lo += mul * (__half2float(la) + __half2float(lc));
        hi[i / 2] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hc) << 16);
        lo[i / 2] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lc) << 16);
      }
      uint8_t* dst = rec + w * 64 + t * 16;
      *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(dst + 256) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    // column w (hi part) sits in lane column t = w / 2, column 4 + w (lo part)
    // in t = 2 + w / 2; each appears for rows g and g + 8 of the quad
    cor[4 * (w >> 1) + (w & 1)] = k * sum_hi;
    cor[4 * (w >> 1) + (w & 1) + 2] = k * sum_hi;
    cor[4 * (2 + (w >> 1)) + (w & 1)] = k * sum_lo;
    cor[4 * (2 + (w >> 1)) + (w & 1) + 2] = k * sum_lo;
  }
}

// gate / up: CTA = 16 warps = (16 / ks) strips of 16 F-rows x ks K-slices of
// one expert.  Per chunk of up to cgp groups of 4 rows, every warp first starts
// its weight ring, then the CTA builds the chunk's activation fragments.
// ---------------------------------------------------------------------------
template <int QT, int NCGM>
__global__ void __launch_bounds__(kGuWarps * 32, 1)
gateup_kernel(const uint8_t* __restrict__ wg, const uint8_t* __restrict__ wu, size_t gu_stride,
              int act, int d, int F, const int32_t* __restrict__ offsets, const int* __restrict__ n_active,
              const int* __restrict__ active, const int* __restrict__ goff,
              const int* __restrict__ citem, const float* __restrict__ x,
              const int32_t* __restrict__ x_rows, int x_div, const float* __restrict__ x_row_max,
              uint8_t* __restrict__ hfrag, int ks, int cgp, int nst, int pt,
              int* __restrict__ done, int* __restrict__ status) {
  using Tr = QTraits<QT>;
  constexpr int TB = Tr::kTileBytes;
  constexpr int SMAX = Ring<QT>::kGuStages;
  static_assert(kGuWarps * SMAX * 8 + 2 * 4 * kGuMaxCG * 4 <= kBarArea, "barrier area");
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Wait for the plan of the previous kernels, then let the down kernel be
  // scheduled on SMs this grid leaves idle (it reads the plan at once, but the
  // hidden fragments only after this grid has completed).  Triggering only
  // after the wait keeps the plan complete for it.
  pdl_wait();
  pdl_trigger();
  const int xbytes = cgp * 2 * pt * kXRec;
  GuCtx c;
  c.xs = smem;
  c.bars = reinterpret_cast<uint64_t*>(smem + xbytes) + warp * SMAX;
  float* rs_s = reinterpret_cast<float*>(smem + xbytes + kGuWarps * SMAX * 8);
  float* rmax_s = rs_s + 4 * kGuMaxCG;
  c.rs = rs_s;
  c.ring = smem + xbytes + kBarArea + warp * nst * gu_stage_bytes<QT>();
  const int spc = kGuWarps / ks;
  const int strips = F / 16;
  const int cpe = (strips + spc - 1) / spc;
  const int item = blockIdx.x / cpe;      // one chunk of 4 * cgp rows of one expert
  int e, c0;
  if (!chunk_of(item, citem, 4 * cgp, e, c0)) return;
  c.ks = ks;
  c.kp = warp % ks;
  c.s = (blockIdx.x % cpe) * spc + warp / ks;
  c.strip_ok = c.s < strips;
  const int JT = d / 64;
  c.jb = c.kp * JT / ks;
  c.ntile = (c.kp + 1) * JT / ks - c.jb;
  c.row0 = offsets[e];
  c.n = offsets[e + 1] - c.row0;
  c.G0 = goff[e];
  c.nbx = 2 * pt;      // staged blocks per column group
  c.xt0 = 0;
  c.nbF = F / 32;
  c.nst = nst;
  c.lane = lane;
  c.hfrag = hfrag;
  c.status = status;
  c.gbase = wg + (size_t)e * gu_stride + (size_t)(c.strip_ok ? c.s : 0) * JT * TB;
  c.ubase = wu + (size_t)e * gu_stride + (size_t)(c.strip_ok ? c.s : 0) * JT * TB;
  c.act = act;
  c.pol = evict_first_policy();
  if (lane == 0) {
    for (int i = 0; i < nst; ++i) mbar_init(&c.bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t parity = 0u;
  const int ncg = min(cgp, (c.n - c0 + 3) / 4);
  gu_prefetch<QT>(c);
  const GuBuild bd = {x, x_rows, x_row_max, rs_s, rmax_s, x_div, ncg, d, pt};
  // NCGM: the most column groups this instance handles (2 or 4; the
  // 4-group accumulators need registers the smaller instance keeps free)
  if (ncg == 1) gu_chunk<QT, 1>(c, parity, c0, true, bd);
  else if constexpr (NCGM <= 2) gu_chunk<QT, 2>(c, parity, c0, true, bd);
  else if (ncg == 2) gu_chunk<QT, 2>(c, parity, c0, true, bd);
  else if (ncg == 3) gu_chunk<QT, 3>(c, parity, c0, true, bd);
  else gu_chunk<QT, 4>(c, parity, c0, true, bd);
  // this CTA's hidden fragments of the chunk are complete: count it (the down
  // kernel's CTAs of the chunk start once all of its gate/up CTAs have)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0)
    asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(done + item) : "memory");
}

// ---------------------------------------------------------------------------
// down: CTA = 8 warps of one expert chunk; warp w streams strips
// s0 + w, s0 + w + 8, ... (spw of them, 16 d-rows each) back to back through
// one continuous ring, so a CTA's prologue, its wait for the gate/up CTAs and
// its first-copy latency are paid once for spw strips.  K = F is short (11
// tiles at F = 704), which is why one strip per warp left the kernel
// latency-bound.
// ---------------------------------------------------------------------------
struct DnCtx {
  const uint8_t* mat;    // this expert's W_down
  uint8_t* ring;
  uint64_t* bars;
  const uint8_t* hs;
  float* y;
  const int32_t* y_rows;
  int* status;
  uint64_t pol;
  float scale;   // per-expert factor on the down projection (1 if none)
  int nst, JT, nbF, d, row0, n, lane;
  int s0, sstep, ns;     // strips s0 + i * sstep, i < ns
};

// Stage q of the warp's flattened stage sequence (stage j of strip i, with
// nsps stages per strip) into ring slot `slot` (lane 0).
template <int QT>
__device__ __forceinline__ void dn_issue(const DnCtx& c, int q, int slot) {
  using Tr = QTraits<QT>;
  constexpr int U = Ring<QT>::kDnU;
  constexpr int TB = Tr::kTileBytes;
  const int nsps = (c.JT + U - 1) / U;
  const int i = q / nsps, j = q - i * nsps;
  const int t0 = j * U;
  const uint32_t bytes = (uint32_t)(min(U, c.JT - t0) * TB);
  const uint8_t* src = c.mat + ((size_t)(c.s0 + i * c.sstep) * c.JT + t0) * TB;
  mbar_expect_tx(&c.bars[slot], bytes);
  bulk_g2s(c.ring + slot * U * TB, src, bytes, &c.bars[slot], c.pol);
}

// First stages; the weights do not depend on the gate/up kernel, so they are
// issued before waiting for it.
template <int QT>
__device__ __forceinline__ void dn_prefetch(const DnCtx& c) {
  constexpr int U = Ring<QT>::kDnU;
  const int total = c.ns * ((c.JT + U - 1) / U);
  if (c.lane == 0 && total > 0) {
    fence_proxy_async_smem();
    for (int q = 0; q < min(c.nst, total); ++q) dn_issue<QT>(c, q, q);
  }
}

// Epilogue of strip s: quad reduction, y rows of the chunk's tokens.
template <int NCG>
__device__ __forceinline__ void dn_store(const DnCtx& c, float2 (&acc)[NCG][2], int s, int c0) {
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      acc[cg][i].x += __shfl_xor_sync(0xffffffffu, acc[cg][i].x, 2);
      acc[cg][i].y += __shfl_xor_sync(0xffffffffu, acc[cg][i].y, 2);
    }
  const int g = c.lane >> 2, t = c.lane & 3;
  if (t < 2 && c.y != nullptr) {
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg) {
#pragma unroll
      for (int ci = 0; ci < 2; ++ci) {
        const int tok = c0 + 4 * cg + 2 * t + ci;
        if (tok >= c.n) continue;
        const int r = c.row0 + tok;
        const int orow = c.y_rows ? c.y_rows[r] : r;
        float* yr = c.y + (size_t)orow * c.d + s * 16 + g;
        yr[0] = (ci ? acc[cg][0].y : acc[cg][0].x) * (1.0f / kHScale) * c.scale;
        yr[8] = (ci ? acc[cg][1].y : acc[cg][1].x) * (1.0f / kHScale) * c.scale;
      }
    }
  }
}

// Streams the warp's ns strips; after each strip's last stage its rows are
// stored and the accumulators restart.  After a timed-out wait no further
// copy is issued, but every copy already issued is still waited for (each
// wait bounded), so none is left in flight when the kernel returns.
template <int QT, int NCG>
__device__ __forceinline__ bool dn_stream(const DnCtx& c, uint32_t& parity, int c0) {
  using Tr = QTraits<QT>;
  constexpr int U = Ring<QT>::kDnU;
  constexpr int TB = Tr::kTileBytes;
  constexpr int STAGE = U * TB;
  const int nsps = (c.JT + U - 1) / U;
  const int total = c.ns * nsps;
  const int cs = c.nbF * 512;
  float2 acc[NCG][2];
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg) acc[cg][0] = acc[cg][1] = make_float2(0.f, 0.f);
  bool ok = true;
  int slot = 0, j = 0, i = 0;
  int issued = min(c.nst, total);          // stages issued so far (dn_prefetch)
  const uint8_t* xq = c.hs + c.lane * 16;
  for (int q = 0; q < issued; ++q) {
    ok = __all_sync(0xffffffffu, mbar_wait(&c.bars[slot], (parity >> slot) & 1u)) && ok;
    parity ^= 1u << slot;
    const int nt = min(U, c.JT - j * U);
    const uint8_t* st = c.ring + slot * STAGE;
    TileRegs<QT> tw[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (u < nt) lds_tile<QT>(tw[u], st + u * TB, c.lane);
    __syncwarp();
    if (ok && q + c.nst < total) {
      if (c.lane == 0) {
        fence_proxy_async_smem();
        dn_issue<QT>(c, q + c.nst, slot);
      }
      issued = q + c.nst + 1;
    }
    slot = (slot + 1 == c.nst) ? 0 : slot + 1;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < nt) {
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t a0[4], a1[4];
          float2 dw, dw8;
          tile_afrags<QT, false>(tw[u], b, a0, a1, dw, dw8);
#pragma unroll
          for (int cg = 0; cg < NCG; ++cg) {
            const uint4 xf = *reinterpret_cast<const uint4*>(xq + cg * cs + u * 1024 + b * 512);
            block_mma(acc[cg], a0, a1, xf, make_float4(0.f, 0.f, 0.f, 0.f), dw, dw8);
          }
        }
      }
    }
    xq += U * 1024;
    if (++j == nsps) {
      if (ok) dn_store<NCG>(c, acc, c.s0 + i * c.sstep, c0);
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) acc[cg][0] = acc[cg][1] = make_float2(0.f, 0.f);
      j = 0;
      ++i;
      xq = c.hs + c.lane * 16;
    }
  }
  return ok;
}

template <int QT, int NCGM>
__global__ void __launch_bounds__(kDnWarps * 32, 2)
down_kernel(const uint8_t* __restrict__ wd, size_t mat_bytes, int d, int F,
            const int32_t* __restrict__ offsets, const int* __restrict__ n_active,
            const int* __restrict__ active, const int* __restrict__ goff,
            const int* __restrict__ citem, const uint8_t* __restrict__ hfrag, float* __restrict__ y,
            const int32_t* __restrict__ y_rows, const float* __restrict__ down_scale, int cgp,
            int nst, int spw, const int* __restrict__ done, int gu_cpe,
            int* __restrict__ status) {
  constexpr int SMAX = Ring<QT>::kDnStages;
  static_assert(kDnWarps * SMAX * 8 + 16 <= kBarArea, "barrier area");
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int xbytes = x_stage_bytes(F, cgp);
  DnCtx c;
  c.hs = smem;
  c.bars = reinterpret_cast<uint64_t*>(smem + xbytes) + warp * SMAX;
  int* ok_s = reinterpret_cast<int*>(smem + xbytes + kDnWarps * SMAX * 8);
  c.ring = smem + xbytes + kBarArea + warp * nst * dn_stage_bytes<QT>();
  const int strips = d / 16;
  const int per_cta = kDnWarps * spw;
  const int cpe = (strips + per_cta - 1) / per_cta;
  const int item = blockIdx.x / cpe;      // the same chunk as the gate/up CTAs that wrote it
  int e, c0;
  if (!chunk_of(item, citem, 4 * cgp, e, c0)) return;
  c.s0 = (blockIdx.x % cpe) * per_cta + warp;
  c.sstep = kDnWarps;
  c.ns = c.s0 < strips ? min(spw, (strips - c.s0 + kDnWarps - 1) / kDnWarps) : 0;
  c.JT = F / 64;
  c.row0 = offsets[e];
  c.n = offsets[e + 1] - c.row0;
  const int G0 = goff[e];
  c.nbF = F / 32;
  c.d = d;
  c.nst = nst;
  c.lane = lane;
  c.y = y;
  c.y_rows = y_rows;
  c.status = status;
  c.mat = wd + (size_t)e * mat_bytes;
  c.scale = down_scale ? down_scale[e] : 1.0f;
  c.pol = evict_first_policy();
  if (lane == 0) {
    for (int i = 0; i < nst; ++i) mbar_init(&c.bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t parity = 0u;
  dn_prefetch<QT>(c);
  // Launched as a programmatic dependent of the gate/up kernel, which may still
  // be running: wait (bounded) until every gate/up CTA of this chunk has
  // counted its hidden fragments as written.  The plan read above is complete
  // (gate/up lets this grid start only after its own wait for the plan).
  if (threadIdx.x == 0) *ok_s = wait_count(done + item, gu_cpe) ? 1 : 0;
  __syncthreads();
  const bool ok = *ok_s != 0;
  if (!ok && threadIdx.x == 0) set_status(status, MOE_STATUS_TIMEOUT);
  pdl_trigger();
  const int ncg = min(cgp, (c.n - c0 + 3) / 4);
  // hidden fragments of the chunk's groups: plain loads (they were written by
  // other CTAs' plain stores, ordered by the counter's release / acquire)
  const uint4* src = reinterpret_cast<const uint4*>(hfrag + (size_t)(G0 + c0 / 4) * c.nbF * 512);
  uint4* dst = reinterpret_cast<uint4*>(smem);
  for (int i = threadIdx.x; i < ncg * c.nbF * 32; i += kDnWarps * 32) dst[i] = src[i];
  __syncthreads();
  // the rings are streamed regardless of a timeout so every issued copy is
  // consumed; rows are stored only when both the wait and the stream succeeded
  bool st;
  if (!ok) c.y = nullptr;
  if (ncg == 1) st = dn_stream<QT, 1>(c, parity, c0);
  else if constexpr (NCGM <= 2) st = dn_stream<QT, 2>(c, parity, c0);
  else if (ncg == 2) st = dn_stream<QT, 2>(c, parity, c0);
  else if (ncg == 3) st = dn_stream<QT, 3>(c, parity, c0);
  else st = dn_stream<QT, 4>(c, parity, c0);
  if (!st) set_status(status, MOE_STATUS_TIMEOUT);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct ExpertsWs {
  int* status;
  int* n_active;
  int* active;
  int* goff;
  int* coff;    // work items: (expert << 16) | chunk, -1 past the last
  int* done;    // per chunk: gate/up CTAs finished
  uint8_t* hfrag;
  size_t bytes;
};

static int max_groups(int rows, int E) { return (rows + 3) / 4 + E; }

static ExpertsWs carve_experts(void* ws, int rows, int E, int d, int F) {
  Carve c{static_cast<uint8_t*>(ws), 0, 0};
  ExpertsWs w;
  const int mg = max_groups(rows, E);
  w.status = c.take<int>(64);
  w.n_active = c.take<int>(64);
  w.active = c.take<int>(E);
  w.goff = c.take<int>(E + 1);
  w.coff = c.take<int>(mg);
  w.done = c.take<int>(mg);
  w.hfrag = c.take<uint8_t>((size_t)mg * F * 16);
  w.bytes = align_up(c.used, 256);
  return w;
}

size_t tc_workspace(int rows, int E, int d, int F);
bool tc_supported(int rows, int E, int d, int F);
int run_experts_tc(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                   int x_div, const float* x_row_max, int d, int F, float* y,
                   const int32_t* y_rows, void* ws, size_t ws_bytes, int* status,
                   const moe_expert_opts* opts, cudaStream_t s);

size_t bs_workspace(int rows, int E, int d, int F);
bool bs_supported(int rows, int E, int d, int F);
int run_experts_bs(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                   int x_div, const float* x_row_max, int d, int F, float* y,
                   const int32_t* y_rows, void* ws, size_t ws_bytes, int* status,
                   const moe_expert_opts* opts, int rb, cudaStream_t s);

// Routed rows per active expert from which the split-operand tcgen05 GEMMs
// are used, and from which the block-scale tcgen05 GEMMs would be (below
// that).  The block-scale threshold defaults to the split one, so automatic
// selection never picks them: measured on B200 they trail the GEMVs at every
// group size tried (4-32 rows per expert); options can still pin them.
#ifndef MOE_TC_MIN_MEAN_ROWS
#define MOE_TC_MIN_MEAN_ROWS 64
#endif
#ifndef MOE_BS_MIN_MEAN_ROWS
#define MOE_BS_MIN_MEAN_ROWS MOE_TC_MIN_MEAN_ROWS
#endif
constexpr int kTcMinMeanRows = MOE_TC_MIN_MEAN_ROWS;
constexpr int kBsMinMeanRows = MOE_BS_MIN_MEAN_ROWS;

static int mean_rows_per_expert(int rows, int E) {
  const int active = rows < E ? rows : E;
  return active > 0 ? rows / active : 0;
}

static bool use_tc(int rows, int E, int d, int F) {
  return mean_rows_per_expert(rows, E) >= kTcMinMeanRows && tc_supported(rows, E, d, F);
}

// The kernel family of a call with `hint` expected rows (opts may pin it).
static int expert_family(int rows, int hint, int E, int d, int F, const moe_expert_opts* opts) {
  if (opts && opts->kernels != MOE_KERNELS_AUTO) return opts->kernels;
  if (use_tc(hint, E, d, F)) return MOE_KERNELS_SPLIT_GEMM;
  if (mean_rows_per_expert(hint, E) >= kBsMinMeanRows && bs_supported(rows, E, d, F))
    return MOE_KERNELS_BLOCKSCALE;
  return MOE_KERNELS_GEMV;
}

// Block-scale chunk rows: about the busiest expert's rows at this mean, so
// most experts take one chunk (each chunk streams its expert's weights once).
static int bs_chunk_rows(int hint, int E, const moe_expert_opts* opts) {
  if (opts && opts->chunk_rows) return opts->chunk_rows;
  const int m = mean_rows_per_expert(hint, E);
  return m <= 5 ? 8 : m <= 10 ? 16 : m <= 22 ? 32 : 64;
}

// rows: the most rows a call may see (buffers); rows_hint: the rows it is
// expected to see, which picks the kernel family.  Every family's buffers are
// included, so options may pin any of them.
int experts_workspace_hint(int rows, int rows_hint, int E, int d, int F, size_t* bytes) {
  size_t a = carve_experts(nullptr, rows, E, d, F).bytes;
  if (bs_supported(rows, E, d, F)) a = std::max(a, bs_workspace(rows, E, d, F));
  if (tc_supported(rows, E, d, F)) a = std::max(a, tc_workspace(rows, E, d, F));
  (void)rows_hint;
  *bytes = a;
  return MOE_OK;
}

int experts_workspace(int rows, int E, int d, int F, size_t* bytes) {
  return experts_workspace_hint(rows, rows, E, d, F, bytes);
}

// Launch shape of the two GEMV kernels for a call.
struct ExpertsPlan {
  int ks, cgp_gu, nst_gu, smem_gu, grid_gu, cpe_gu, pt_gu;
  int cgp_dn, nst_dn, smem_dn, grid_dn, spw_dn;
};

// Strips per warp of the down kernel.  A strip is short (F / 64 tiles), so a
// CTA's fixed cost (prologue, wait for gate/up, first-copy latency, about one
// strip's streaming time) is amortised over spw strips; spw is chosen to
// minimise rounds * (spw + 1) for the expected work items on two CTAs per SM.
#ifndef MOE_DN_SPW
#define MOE_DN_SPW 0
#endif
static int down_strips_per_warp(int rows, int est_active, int strips_d, int cgp) {
  if (MOE_DN_SPW > 0) return MOE_DN_SPW;
  // measured on B200: with fewer than about four CTAs per SM the down grid
  // stops overlapping the gate/up tail (decode T=64: 4 strips per warp,
  // 786 CTAs, 151 us per layer; 11 strips, 262 CTAs, 169 us; 1 strip, 159 us)
  const long long items = std::max(est_active, (rows + 4 * cgp - 1) / (4 * cgp));
  const long long min_ctas = 4LL * sm_count();
  int best = 1;
  for (int spw = 2; spw <= 8; ++spw) {
    const long long cpe = (strips_d + kDnWarps * spw - 1) / (kDnWarps * spw);
    if (items * cpe >= min_ctas) best = spw;
  }
  return best;
}

// rows bounds the call (grids, buffers); hint (when below it) is the rows it
// is expected to see, which picks column groups and the K split -- an
// expert-parallel owner is planned for up to every rank's rows but usually
// receives its own share.
template <int QT>
static bool plan_experts(int rows, int E, int d, int F, ExpertsPlan& p, int hint = 0) {
  // K-phased activation staging (items wider than all of K leaves room for,
  // at a CTA barrier per phase) only from this many expected rows per expert;
  // below, narrower single-phase items
#ifndef MOE_GU_PHASE_MIN_ROWS
#define MOE_GU_PHASE_MIN_ROWS 12
#endif
  constexpr int kGuPhaseMinRows = MOE_GU_PHASE_MIN_ROWS;
  const int bound_active = rows < E ? rows : E;
  const int hrows = hint > 0 && hint < rows ? hint : rows;
  const int est_active = hrows < E ? hrows : E;
  const int strips_f = F / 16, strips_d = d / 16;
  const int JT = d / 64;
  const int target = sm_count() * kGuWarps;  // one full CTA per SM
  // column groups per pass: about twice the mean rows of an expert
  const int mean_rows = (hrows + est_active - 1) / est_active;
  const int want_cg = std::max(1, std::min(kMaxCG, (2 * mean_rows + 3) / 4));
  // split K over 2, 4 or 8 warps of a strip until the chunks' strips fill the
  // GPU with one CTA per SM (every CTA builds its chunk's activations for all
  // of K, so fewer, longer CTAs are preferred)
#ifndef MOE_KS_BY_ITEMS
#define MOE_KS_BY_ITEMS 1
#endif
  const int cg_est = std::min(want_cg, kGuMaxCG);
  const int items_est = MOE_KS_BY_ITEMS ? std::max(est_active, (hrows + 4 * cg_est - 1) / (4 * cg_est))
                                        : est_active;
  p.ks = 1;
  while (p.ks < 8 && (long long)items_est * strips_f * p.ks < target && JT / (2 * p.ks) >= 2)
    p.ks *= 2;
  const int spc = kGuWarps / p.ks;
  p.cpe_gu = (strips_f + spc - 1) / spc;
  // gate/up: stages for the tiles a warp streams (clamped), then the largest
  // column-group count whose activation records fit beside the rings -- for
  // all of K, or (without a K split) for one K phase of pt tiles, a whole
  // number of stages, staged phase by phase
  const int gu_u = Ring<QT>::kGuU;
  p.nst_gu = std::max(1, std::min(Ring<QT>::kGuStages, ((JT + p.ks - 1) / p.ks + gu_u - 1) / gu_u));
  const int ring = kGuWarps * p.nst_gu * gu_stage_bytes<QT>();
  const int avail = kMaxSmem - kBarArea - ring;
  const int want = std::min(want_cg, kGuMaxCG);
  p.cgp_gu = 0;
  p.pt_gu = JT;
  for (int cg = want; cg >= 1 && p.cgp_gu == 0; --cg) {
    // the split-K reduction (cg KB per warp) lives in the rings
    if (p.ks > 1 && p.nst_gu * gu_stage_bytes<QT>() < cg * 1024) continue;
    if (cg * 2 * JT * kXRec <= avail) {
      p.cgp_gu = cg;
      p.pt_gu = JT;
    } else if (p.ks == 1 && mean_rows >= kGuPhaseMinRows) {
      const int pt = avail / (cg * 2 * kXRec) / gu_u * gu_u;   // tiles per phase
      if (pt >= gu_u && cg > 2) {
        p.cgp_gu = cg;
        p.pt_gu = pt;
      }
    }
  }
  if (p.cgp_gu < 1) return false;
  p.smem_gu = p.cgp_gu * 2 * p.pt_gu * kXRec + kBarArea + ring;
  const int dn_u = Ring<QT>::kDnU;
  p.nst_dn = std::max(1, std::min(Ring<QT>::kDnStages, (F / 64 + dn_u - 1) / dn_u));
  const int ring_dn = kDnWarps * p.nst_dn * dn_stage_bytes<QT>();
  // both kernels work on the same chunks of 4 * cgp rows
  p.cgp_dn = p.cgp_gu;
  if ((kMaxSmem - kBarArea - ring_dn) / x_stage_bytes(F, 1) < p.cgp_dn) return false;
  p.smem_dn = x_stage_bytes(F, p.cgp_dn) + kBarArea + ring_dn;
  // work items: chunks of 4 * cgp rows, at most rows / (4 cgp) + one per expert
  const int items = std::min(max_groups(rows, E), rows / (4 * p.cgp_gu) + bound_active);
  p.grid_gu = items * p.cpe_gu;
  p.spw_dn = down_strips_per_warp(hrows, est_active, strips_d, p.cgp_gu);
  p.grid_dn = items * ((strips_d + kDnWarps * p.spw_dn - 1) / (kDnWarps * p.spw_dn));
  return true;
}

// Launches the grouped experts with an already-carved workspace.
template <int QT>
static int launch_experts(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down,
                          const int32_t* offsets, int E, int rows, const float* x,
                          const int32_t* x_rows, int x_div, const float* x_row_max, bool planned,
                          int d, int F, float* y, const int32_t* y_rows, const ExpertsWs& w,
                          const moe_expert_opts* opts, int rows_hint, cudaStream_t s) {
  using Tr = QTraits<QT>;
  ExpertsPlan p;
  MOE_REQUIRE(plan_experts<QT>(rows, E, d, F, p, rows_hint), MOE_ERR_UNSUPPORTED,
              "d=%d / F=%d too large for the staged activation buffers", d, F);
  static unsigned long long attr_set = 0;  // per template instance, bit per device
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev));
  if (!((attr_set >> (dev & 63)) & 1ull)) {
    MOE_CUDA(cudaFuncSetAttribute(gateup_kernel<QT, 2>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    MOE_CUDA(cudaFuncSetAttribute(gateup_kernel<QT, 4>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    MOE_CUDA(cudaFuncSetAttribute(down_kernel<QT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kMaxSmem));
    MOE_CUDA(cudaFuncSetAttribute(down_kernel<QT, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kMaxSmem));
    attr_set |= 1ull << (dev & 63);
  }
  const bool wide = p.cgp_gu > 2;
  const int mg = max_groups(rows, E);
  if (!planned) {
    ::moe::ProfScope _prof(MOE_K_PLAN, s);
    plan_kernel<<<1, kPlanThreads, 0, s>>>(offsets, E, rows, mg, 4 * p.cgp_gu, w.n_active,
                                           w.active, w.goff, w.coff, w.done, w.status);
  }
  MOE_CHECK(check_launch("plan"));
  const size_t mat_bytes = (size_t)F * (d / 32) * Tr::kBlockBytes;
  const size_t gu_stride = (opts && opts->gate_up_stride) ? opts->gate_up_stride : mat_bytes;
  const int act = opts ? opts->act : MOE_ACT_SWIGLU;
  const float* down_scale = opts ? opts->down_scale : nullptr;
  {
    ::moe::ProfScope _prof(MOE_K_GATEUP, s);
    MOE_CUDA(launch_pdl(wide ? gateup_kernel<QT, 4> : gateup_kernel<QT, 2>, dim3(p.grid_gu),
                        dim3(kGuWarps * 32), p.smem_gu, s,
                        w_gate, w_up, gu_stride, act, d, F, offsets, (const int*)w.n_active,
                        (const int*)w.active, (const int*)w.goff, (const int*)w.coff, x, x_rows,
                        x_div, x_row_max, w.hfrag, p.ks, p.cgp_gu, p.nst_gu, p.pt_gu, w.done,
                        w.status));
  }
  MOE_CHECK(check_launch("gateup"));
  {
    ::moe::ProfScope _prof(MOE_K_DOWN, s);
    MOE_CUDA(launch_pdl(wide ? down_kernel<QT, 4> : down_kernel<QT, 2>, dim3(p.grid_dn),
                        dim3(kDnWarps * 32), p.smem_dn, s,
                        w_down, mat_bytes, d, F, offsets, (const int*)w.n_active,
                        (const int*)w.active, (const int*)w.goff, (const int*)w.coff,
                        (const uint8_t*)w.hfrag, y, y_rows, down_scale, p.cgp_dn, p.nst_dn,
                        p.spw_dn,
                        (const int*)w.done, p.cpe_gu, w.status));
  }
  return check_launch("down");
}

// Plan arrays inside an experts workspace, for a dispatch that writes them.
// Rows per work item (chunk) of the GEMV kernels for a call's shape.
int experts_rows_per_chunk(int qtype, int dn_qtype, int rows, int E, int d, int F,
                           int rows_hint) {
  if (!experts_packed(qtype, dn_qtype)) return raw_rows_per_chunk(d, F);
  ExpertsPlan p;
  const bool ok = qtype == MOE_Q4_0 ? plan_experts<MOE_Q4_0>(rows, E, d, F, p, rows_hint)
                                    : plan_experts<MOE_Q8_0>(rows, E, d, F, p, rows_hint);
  return ok ? 4 * p.cgp_gu : 4;
}

void experts_plan_arrays(void* ws, int rows, int E, int d, int F, int** n_active, int** active,
                         int** goff, int** coff, int** done, int* mg) {
  ExpertsWs w = carve_experts(ws, rows, E, d, F);
  *n_active = w.n_active;
  *active = w.active;
  *goff = w.goff;
  *coff = w.coff;
  *done = w.done;
  *mg = max_groups(rows, E);
}

void experts_hidden(void* ws, int rows, int E, int d, int F, uint8_t** hidden, int** status) {
  ExpertsWs w = carve_experts(ws, rows, E, d, F);
  *hidden = w.hfrag;
  *status = w.status;
}

// The expert plan (work items of rpc rows) from expert_offsets, in ws.
int launch_expert_plan(const int32_t* offsets, int E, int rows, int rpc, void* ws, int d, int F,
                       cudaStream_t s) {
  ExpertsWs w = carve_experts(ws, rows, E, d, F);
  {
    ::moe::ProfScope _prof(MOE_K_PLAN, s);
    plan_kernel<<<1, kPlanThreads, 0, s>>>(offsets, E, rows, max_groups(rows, E), rpc, w.n_active,
                                           w.active, w.goff, w.coff, w.done, w.status);
  }
  return check_launch("plan");
}

int raw_rows_per_chunk(int d, int F);
int run_experts_raw(const uint8_t* wg, const uint8_t* wu, const uint8_t* wd, int gu_fmt,
                    int dn_fmt, const moe_expert_opts* opts, const int32_t* offsets, int E,
                    int rows, const float* x, const int32_t* x_rows, int x_div, int d, int F,
                    float* y, const int32_t* y_rows, void* ws, bool planned, cudaStream_t s);

// quant type of the down matrices under opts
int experts_down_qtype(int qtype, const moe_expert_opts* opts) {
  return (opts && opts->down_qtype != 0) ? opts->down_qtype : qtype;
}

// Whether a layer's weights run on the packed-tile kernels (Q4_0 / Q8_0 for
// all three matrices) rather than the raw-block path.
bool experts_packed(int qtype, int dn_qtype) {
  return qtype_ok(qtype) && dn_qtype == qtype;
}

int run_experts(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                int x_div, int d, int F, float* y, const int32_t* y_rows, void* ws,
                size_t ws_bytes, cudaStream_t s, int* status, const float* x_row_max,
                bool planned, int rows_hint, const moe_expert_opts* opts) {
  const int dn_qtype = experts_down_qtype(qtype, opts);
  if (!experts_packed(qtype, dn_qtype)) {
    MOE_REQUIRE(E > 0 && E <= kPlanThreads, MOE_ERR_UNSUPPORTED, "local expert count %d", E);
    MOE_REQUIRE(rows >= 0, MOE_ERR_INVALID, "rows must be >= 0");
    if (rows == 0) return MOE_OK;
    MOE_REQUIRE(w_gate && w_up && w_down && offsets && x && y && ws, MOE_ERR_INVALID,
                "null pointer");
    MOE_REQUIRE(x_div > 0, MOE_ERR_INVALID, "x_rows_div must be positive");
    const size_t need = carve_experts(nullptr, rows, E, d, F).bytes;
    MOE_REQUIRE(ws_bytes >= need, MOE_ERR_WORKSPACE, "experts workspace %zu < %zu", ws_bytes,
                need);
    return run_experts_raw(w_gate, w_up, w_down, qtype, dn_qtype, opts, offsets, E, rows, x,
                           x_rows, x_div, d, F, y, y_rows, ws, planned, s);
  }
  MOE_REQUIRE(E > 0 && E <= kPlanThreads, MOE_ERR_UNSUPPORTED, "local expert count %d", E);
  MOE_REQUIRE(d > 0 && F > 0 && d % 64 == 0 && F % 64 == 0, MOE_ERR_UNSUPPORTED,
              "d=%d and F=%d must be multiples of 64", d, F);
  MOE_REQUIRE(rows >= 0, MOE_ERR_INVALID, "rows must be >= 0");
  if (rows == 0) return MOE_OK;
  MOE_REQUIRE(w_gate && w_up && w_down && offsets && x && y && ws, MOE_ERR_INVALID,
              "null pointer");
  MOE_REQUIRE(x_div > 0, MOE_ERR_INVALID, "x_rows_div must be positive");
  MOE_REQUIRE(((uintptr_t)w_gate | (uintptr_t)w_up | (uintptr_t)w_down | (uintptr_t)x) % 16 == 0,
              MOE_ERR_INVALID, "weights and activations must be 16-byte aligned");
  const int hint = rows_hint > 0 ? rows_hint : rows;
  const int family = expert_family(rows, hint, E, d, F, opts);
  if (family == MOE_KERNELS_SPLIT_GEMM)
    return run_experts_tc(w_gate, w_up, w_down, qtype, offsets, E, rows, x, x_rows, x_div,
                          x_row_max, d, F, y, y_rows, ws, ws_bytes, status, opts, s);
  if (family == MOE_KERNELS_BLOCKSCALE)
    return run_experts_bs(w_gate, w_up, w_down, qtype, offsets, E, rows, x, x_rows, x_div,
                          x_row_max, d, F, y, y_rows, ws, ws_bytes, status, opts,
                          bs_chunk_rows(hint, E, opts), s);
  MOE_REQUIRE(family == MOE_KERNELS_GEMV, MOE_ERR_INVALID, "unknown kernel family %d", family);
  ExpertsWs w = carve_experts(ws, rows, E, d, F);
  if (status) w.status = status;
  MOE_REQUIRE(ws_bytes >= w.bytes, MOE_ERR_WORKSPACE, "experts workspace %zu < %zu", ws_bytes,
              w.bytes);
  if (qtype == MOE_Q4_0)
    return launch_experts<MOE_Q4_0>(w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div,
                                    x_row_max, planned, d, F, y, y_rows, w, opts, rows_hint, s);
  return launch_experts<MOE_Q8_0>(w_gate, w_up, w_down, offsets, E, rows, x, x_rows, x_div,
                                  x_row_max, planned, d, F, y, y_rows, w, opts, rows_hint, s);
}

}  // namespace moe

extern "C" {

int moe_experts_workspace_bytes(int rows, int E_local, int d, int F, size_t* bytes) {
  MOE_REQUIRE(bytes, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(rows >= 0 && E_local > 0 && d > 0 && F > 0, MOE_ERR_INVALID, "bad shape");
  return moe::experts_workspace(rows, E_local, d, F, bytes);
}

int moe_experts(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                const int32_t* expert_offsets, int E_local, int rows, const float* x,
                const int32_t* x_rows, int x_rows_div, int d, int F, float* y,
                const int32_t* y_rows, void* workspace, size_t workspace_bytes,
                moe_stream_t stream) {
  return moe_experts_ex(w_gate, w_up, w_down, qtype, nullptr, expert_offsets, E_local, rows, x,
                        x_rows, x_rows_div, d, F, y, y_rows, workspace, workspace_bytes, stream);
}

int moe_experts_ex(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const moe_expert_opts* opts, const int32_t* expert_offsets, int E_local,
                   int rows, const float* x, const int32_t* x_rows, int x_rows_div, int d, int F,
                   float* y, const int32_t* y_rows, void* workspace, size_t workspace_bytes,
                   moe_stream_t stream) {
  MOE_REQUIRE(!opts || opts->act == MOE_ACT_SWIGLU || opts->act == MOE_ACT_GEGLU_TANH,
              MOE_ERR_INVALID, "unknown activation %d", opts ? opts->act : 0);
  return moe::run_experts(w_gate, w_up, w_down, qtype, expert_offsets, E_local, rows, x, x_rows,
                          x_rows_div, d, F, y, y_rows, workspace, workspace_bytes,
                          reinterpret_cast<cudaStream_t>(stream), nullptr, nullptr, false, 0,
                          opts);
}

}  // extern "C"
