// Router: logits = x @ G (+ bias), top-k selection and softmax weights.
//
// moe_forward.py:91-109 (MoERouter.route: top-k of the logits, descending, then
// softmax over the k selected logits) and nightmare_stream.py:3227-3238
// (softmax over all experts, top-k of the probabilities, ascending, renormalised).
//
// Pass 1 (router_gemv_kernel): a grid of (d-slice, token tile) CTAs; each
// stages its tokens' slice of x in shared memory, streams the matching rows of
// the router matrix straight from global memory (one 128-bit load per lane and
// row, eight rows in flight per warp) and reduces the per-warp partial logits
// in warp order.  It also records each token's max |x| over the slice.
// For 128 tokens or more pass 1 is router_gemm_kernel instead: (d-slice, 64-token
// tile, 128-expert tile) CTAs, both operands staged in shared memory (double
// buffered), each thread holding a 4 x 8 register tile of logits; every logit
// is still one fused multiply-add chain over its slice, in row order.
// Pass 2 (router_select_kernel, a programmatic dependent launch of pass 1): one
// warp per token sums the slice partials in slice order, adds the bias, and
// selects with warp max-reductions on order-preserving integer keys.  Softmax
// denominators use numpy's float32 summation order (sequential below 8 terms,
// 8-way pairwise at and above) so the weights follow the reference.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "internal.cuh"

namespace moe {

constexpr int kRouterThreads = 256;   // pass 1: 8 warps
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kRouterChunk = 64;      // x columns staged per chunk
constexpr int kMaxE = 512;
constexpr int kMaxK = 32;
constexpr int kSelMaxThreads = 512;   // pass 2: up to 4 threads per expert

// Grid of pass 1: token tiles of TT tokens and d-slices of `rows` rows (a
// multiple of 4), about two CTAs per SM.  gemm: the tiled kernel (TT = 64,
// 128-expert tiles, rows a multiple of 32).  max_parts caps nds * T * E.
constexpr int kRgTT = 64, kRgTE = 128, kRgK = 16, kRgThreads = 256;
constexpr int kRgMinT = 128;

struct RouterPlan {
  int tt, tiles, nds, rows;
  bool gemm;
};

static RouterPlan router_plan(int T, int d, int E,
                              size_t max_parts = ~(size_t)0) {
  RouterPlan p;
  p.gemm = T >= kRgMinT && d % 4 == 0;
  int want;
  if (p.gemm) {
    p.tt = kRgTT;
    p.tiles = (T + kRgTT - 1) / kRgTT;
    const int ez = (E + kRgTE - 1) / kRgTE;
    want = std::max(1, std::min(d / 128, (2 * sm_count() + p.tiles * ez - 1) / (p.tiles * ez)));
  } else {
    p.tt = T >= 16 ? 16 : (T >= 8 ? 8 : (T >= 4 ? 4 : 1));
    p.tiles = (T + p.tt - 1) / p.tt;
    want = std::max(1, (2 * sm_count() + p.tiles - 1) / p.tiles);
  }
  for (;; --want) {
    int rows = (d + want - 1) / want;
    rows = std::max(32, (rows + 31) / 32 * 32);
    p.rows = std::min(rows, p.gemm ? (d + 31) / 32 * 32 : (d + 3) / 4 * 4);
    p.nds = (d + p.rows - 1) / p.rows;
    if (want <= 1 || (size_t)p.nds * T * E <= max_parts) break;
  }
  return p;
}

static size_t router_part_floats(const RouterPlan& p, int T, int E) {
  return (size_t)p.nds * T * E;
}

// Router matrix entries (row i, experts e0 .. e0+3) in either layout.
__device__ __forceinline__ float4 load_g4(const float* __restrict__ G, int layout, int d, int E,
                                          int i, int e0) {
  if (layout == MOE_ROUTER_D_E) return __ldg(reinterpret_cast<const float4*>(G + (size_t)i * E + e0));
  return make_float4(__ldg(G + (size_t)e0 * d + i), __ldg(G + (size_t)(e0 + 1) * d + i),
                     __ldg(G + (size_t)(e0 + 2) * d + i), __ldg(G + (size_t)(e0 + 3) * d + i));
}

template <int TT>
__global__ void __launch_bounds__(kRouterThreads)
router_gemv_kernel(const float* __restrict__ x, const float* __restrict__ G, int T, int d, int E,
                   int layout, int rows_per_slice, float* __restrict__ part,
                   float* __restrict__ pmax, float* __restrict__ xcopy) {
  // pass 2 may start (and wait) while this grid runs
  pdl_trigger();
  __shared__ __align__(16) float xs[kRouterChunk][TT];   // x chunk, token-minor
  __shared__ float pm[TT];
  extern __shared__ __align__(16) float red[];           // [warps][TT][128]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slice = blockIdx.x, t0 = blockIdx.y * TT;
  const int r0 = slice * rows_per_slice, r1 = min(d, r0 + rows_per_slice);
  const int nt = min(TT, T - t0);
  if (tid < TT) pm[tid] = 0.f;
  for (int eg = 0; eg < E; eg += 128) {
    const int e0 = eg + 4 * lane;
    const bool ev = e0 < E;
    float acc[TT][4];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[t][c] = 0.f;
    for (int i0 = r0; i0 < r1; i0 += kRouterChunk) {
      const int rows = min(kRouterChunk, r1 - i0);
      __syncthreads();   // previous chunk fully read
      for (int v = tid; v < TT * (kRouterChunk / 4); v += kRouterThreads) {
        const int tl = v % TT, q = v / TT;
        float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tl < nt && 4 * q < rows) {
          f = __ldg(reinterpret_cast<const float4*>(x + (size_t)(t0 + tl) * d + i0) + q);
          // x in host memory: this pass's reads are the layer's only ones,
          // and it leaves the device copy the later kernels read
          if (xcopy && eg == 0)
            reinterpret_cast<float4*>(xcopy + (size_t)(t0 + tl) * d + i0)[q] = f;
        }
        xs[4 * q + 0][tl] = f.x;
        xs[4 * q + 1][tl] = f.y;
        xs[4 * q + 2][tl] = f.z;
        xs[4 * q + 3][tl] = f.w;
      }
      __syncthreads();
      if (pmax && eg == 0) {
        for (int tl = warp; tl < TT; tl += kRouterWarps) {
          float m = fmaxf(fabsf(xs[lane][tl]), fabsf(xs[lane + 32][tl]));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) pm[tl] = fmaxf(pm[tl], m);
        }
      }
      if (ev) {
        constexpr int RPW = kRouterChunk / kRouterWarps;   // rows per warp and chunk
        float4 g[RPW];
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
          const int i = warp + kRouterWarps * q;
          g[q] = i < rows ? load_g4(G, layout, d, E, i0 + i, e0) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
          const int i = warp + kRouterWarps * q;
          if (TT % 4 == 0) {
#pragma unroll
            for (int tq = 0; tq < TT / 4; ++tq) {
              const float4 xv = *reinterpret_cast<const float4*>(&xs[i][4 * tq]);
              const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                acc[4 * tq + u][0] = fmaf(xa[u], g[q].x, acc[4 * tq + u][0]);
                acc[4 * tq + u][1] = fmaf(xa[u], g[q].y, acc[4 * tq + u][1]);
                acc[4 * tq + u][2] = fmaf(xa[u], g[q].z, acc[4 * tq + u][2]);
                acc[4 * tq + u][3] = fmaf(xa[u], g[q].w, acc[4 * tq + u][3]);
              }
            }
          } else {
#pragma unroll
            for (int t = 0; t < TT; ++t) {
              const float xv = xs[i][t];
              acc[t][0] = fmaf(xv, g[q].x, acc[t][0]);
              acc[t][1] = fmaf(xv, g[q].y, acc[t][1]);
              acc[t][2] = fmaf(xv, g[q].z, acc[t][2]);
              acc[t][3] = fmaf(xv, g[q].w, acc[t][3]);
            }
          }
        }
      }
    }
    // per-warp partials meet in shared memory and are summed in warp order
    __syncthreads();
#pragma unroll
    for (int t = 0; t < TT; ++t)
      *reinterpret_cast<float4*>(red + ((size_t)warp * TT + t) * 128 + 4 * lane) =
          make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
    __syncthreads();
    for (int v = tid; v < TT * 128; v += kRouterThreads) {
      const int t = v >> 7, e = v & 127;
      if (t < nt && eg + e < E) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kRouterWarps; ++w) sum += red[((size_t)w * TT + t) * 128 + e];
        part[((size_t)slice * T + t0 + t) * E + eg + e] = sum;
      }
    }
  }
  if (pmax) {
    __syncthreads();
    if (tid < nt) pmax[(size_t)slice * T + t0 + tid] = pm[tid];
  }
}

// Order-preserving key of a logit: larger value -> larger key, NaN above every
// number, -0 equal to +0 (so equal values tie and the index decides).  0 is
// never the key of a value and marks an empty slot.
__device__ __forceinline__ unsigned order_key(float v) {
  if (isnan(v)) return 0xFFFFFFFFu;
  const unsigned u = __float_as_uint(v + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Selection and weights for one token; executed by one warp whose lanes hold
// the logits e = lane + 32 j (bias included) in v.  Rules: larger value first,
// NaN above every number, equal values -> higher expert index first.
template <int NJ>
__device__ __forceinline__ void select_warp(float (&v)[NJ], int E, int k, int mode,
                                            float* __restrict__ buf,
                                            int32_t* __restrict__ ids_t, float* __restrict__ w_t) {
  const int lane = threadIdx.x & 31;
  if (mode == MOE_ROUTE_SOFTMAX_TOPK_RENORM) {
    float m = -INFINITY;
    bool any_nan = false;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      if (lane + 32 * j < E) {
        any_nan |= isnan(v[j]);
        m = fmaxf(m, v[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (__any_sync(0xffffffffu, any_nan)) m = NAN;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      if (e < E) {
        v[j] = expf(v[j] - m);
        buf[e] = v[j];
      }
    }
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, E);
    s = __shfl_sync(0xffffffffu, s, 0);
#pragma unroll
    for (int j = 0; j < NJ; ++j) v[j] = v[j] / s;
    __syncwarp();
  }
  unsigned key[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) key[j] = lane + 32 * j < E ? order_key(v[j]) : 0u;
  int sel_id = -1;
  float sel_val = 0.f;
  for (int r = 0; r < k; ++r) {
    unsigned bk = 0u;
    int bj = 0;
    float bv = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      if (key[j] != 0u && key[j] >= bk) {   // >=: equal keys -> higher index
        bk = key[j];
        bj = j;
        bv = v[j];
      }
    const unsigned m = __reduce_max_sync(0xffffffffu, bk);
    const unsigned cand = (bk != 0u && bk == m) ? (unsigned)(lane + 32 * bj + 1) : 0u;
    const int win = (int)__reduce_max_sync(0xffffffffu, cand) - 1;
    const float wv = __shfl_sync(0xffffffffu, bv, win & 31);
    if (lane == (win & 31)) {
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        if (j == (win >> 5)) key[j] = 0u;
    }
    if (lane == r) {
      sel_id = win;
      sel_val = wv;
    }
  }
  if (mode == MOE_ROUTE_TOPK_SOFTMAX) {
    // softmax over the k selected logits, in selection (descending) order
    float mx = lane < k ? sel_val : NAN;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane < k) buf[lane] = expf(sel_val - mx);
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, k);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (lane < k) {
      ids_t[lane] = sel_id;
      w_t[lane] = buf[lane] / s;
    }
  } else {
    // renormalised probabilities, written in ascending order
    const int pos = k - 1 - lane;
    if (lane < k) buf[pos] = sel_val;
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, k);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (lane < k) {
      ids_t[pos] = sel_id;
      w_t[pos] = sel_val / s;
    }
  }
  __syncwarp();
}

// One CTA per token.  Q = blockDim / 128 thread groups split the slices into
// Q contiguous ranges; thread (q, e) sums its range in slice order with eight
// loads in flight, and the Q range sums are added in range order (a fixed
// order for a given plan).  Then the bias, the optional row max over the
// slices' maxima, and the selection by warp 0.
// Pass 1 for many tokens: logits of 64 tokens x 128 experts over one d-slice.
// Thread (ty, tx) keeps tokens 4 ty .. 4 ty + 3 and experts 4 tx .. 4 tx + 3,
// 64 + 4 tx .. 64 + 4 tx + 3 of the tile; chunks of 16 rows are staged
// k-major in shared memory, the next chunk's loads in flight during the FMAs.
__global__ void __launch_bounds__(kRgThreads)
router_gemm_kernel(const float* __restrict__ x, const float* __restrict__ G, int T, int d, int E,
                   int layout, int rows_per_slice, float* __restrict__ part,
                   float* __restrict__ pmax, float* __restrict__ xcopy) {
  pdl_trigger();
  __shared__ __align__(16) float xs[2][kRgK][kRgTT + 8];
  __shared__ __align__(16) float gs[2][kRgK][kRgTE];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int slice = blockIdx.x, t0 = blockIdx.y * kRgTT, e0 = blockIdx.z * kRgTE;
  const int r0 = slice * rows_per_slice, r1 = min(d, r0 + rows_per_slice);
  // x loader: token tid >> 2, four rows at 4 (tid & 3)
  const int xt = tid >> 2, xk = 4 * (tid & 3);
  float xm = 0.f;
  float4 xr, gr[2];
  auto gload = [&](int i0) {
    {
      const int t = t0 + xt, i = i0 + xk;
      xr = (t < T && i < r1) ? __ldg(reinterpret_cast<const float4*>(x + (size_t)t * d + i))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      if (xcopy && blockIdx.z == 0 && t < T && i < r1)   // device copy of host x
        *reinterpret_cast<float4*>(xcopy + (size_t)t * d + i) = xr;
      xm = fmaxf(xm, fmaxf(fmaxf(fabsf(xr.x), fabsf(xr.y)), fmaxf(fabsf(xr.z), fabsf(xr.w))));
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int idx = tid + kRgThreads * j;
      if (layout == MOE_ROUTER_D_E) {
        const int k = idx >> 5, e = e0 + 4 * (idx & 31), i = i0 + k;
        gr[j] = (i < r1 && e < E) ? __ldg(reinterpret_cast<const float4*>(G + (size_t)i * E + e))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        const int e = e0 + (idx >> 2), i = i0 + 4 * (idx & 3);
        gr[j] = (i < r1 && e < E) ? __ldg(reinterpret_cast<const float4*>(G + (size_t)e * d + i))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  auto sstore = [&](int b) {
    xs[b][xk + 0][xt] = xr.x;
    xs[b][xk + 1][xt] = xr.y;
    xs[b][xk + 2][xt] = xr.z;
    xs[b][xk + 3][xt] = xr.w;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int idx = tid + kRgThreads * j;
      if (layout == MOE_ROUTER_D_E) {
        *reinterpret_cast<float4*>(&gs[b][idx >> 5][4 * (idx & 31)]) = gr[j];
      } else {
        const int e = idx >> 2, k = 4 * (idx & 3);
        gs[b][k + 0][e] = gr[j].x;
        gs[b][k + 1][e] = gr[j].y;
        gs[b][k + 2][e] = gr[j].z;
        gs[b][k + 3][e] = gr[j].w;
      }
    }
  };
  float acc[4][8];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[u][v] = 0.f;
  gload(r0);
  sstore(0);
  __syncthreads();
  int b = 0;
  for (int i0 = r0; i0 < r1; i0 += kRgK) {
    const bool more = i0 + kRgK < r1;
    if (more) gload(i0 + kRgK);
#pragma unroll
    for (int k = 0; k < kRgK; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[b][k][4 * ty]);
      const float4 g0 = *reinterpret_cast<const float4*>(&gs[b][k][4 * tx]);
      const float4 g1 = *reinterpret_cast<const float4*>(&gs[b][k][64 + 4 * tx]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 8; ++v) acc[u][v] = fmaf(av[u], gv[v], acc[u][v]);
    }
    if (more) sstore(b ^ 1);
    __syncthreads();
    b ^= 1;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int t = t0 + 4 * ty + u;
    if (t >= T) continue;
    float* dst = part + ((size_t)slice * T + t) * E;
    const int ea = e0 + 4 * tx, eb = e0 + 64 + 4 * tx;
    if (ea < E)
      *reinterpret_cast<float4*>(dst + ea) = make_float4(acc[u][0], acc[u][1], acc[u][2], acc[u][3]);
    if (eb < E)
      *reinterpret_cast<float4*>(dst + eb) = make_float4(acc[u][4], acc[u][5], acc[u][6], acc[u][7]);
  }
  if (pmax && blockIdx.z == 0) {
    float m = xm;
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int t = t0 + xt;
    if ((tid & 3) == 0 && t < T) pmax[(size_t)slice * T + t] = m;
  }
}

template <int NJ>
__global__ void __launch_bounds__(kSelMaxThreads)
router_select_kernel(const float* __restrict__ part, const float* __restrict__ pmax, int nds,
                     const float* __restrict__ bias, int T, int E, int k, int mode,
                     int32_t* __restrict__ ids, float* __restrict__ weights,
                     float* __restrict__ row_max) {
  __shared__ float red[kSelMaxThreads / 128][kMaxE];
  __shared__ float lg[kMaxE];
  // launched as a programmatic dependent of the partial-logit pass; the
  // dispatch after it may start early too
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int Q = blockDim.x / 128;
  const int q = tid / 128;
  const int s0 = q * nds / Q, s1 = (q + 1) * nds / Q;
  const size_t stride = (size_t)T * E;
  for (int e = tid % 128; e < E; e += 128) {
    const float* p = part + (size_t)t * E + e;
    float acc = 0.f;
    int s = s0;
    for (; s + 8 <= s1; s += 8) {
      float v8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v8[u] = p[(size_t)(s + u) * stride];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += v8[u];
    }
    for (; s < s1; ++s) acc += p[(size_t)s * stride];
    red[q][e] = acc;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    float acc = red[0][e];
    for (int qq = 1; qq < Q; ++qq) acc += red[qq][e];
    if (bias) acc += bias[e];
    lg[e] = acc;
  }
  if (row_max && tid >= 128 * (Q - 1) && tid < 128 * (Q - 1) + 32) {
    float m = 0.f;
    for (int s = lane; s < nds; s += 32) m = fmaxf(m, pmax[(size_t)s * T + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) row_max[t] = m;
  }
  __syncthreads();
  if (tid < 32) {
    float v[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? lg[e] : 0.f;
    }
    select_warp<NJ>(v, E, k, mode, red[0], ids + (size_t)t * k, weights + (size_t)t * k);
  }
}

// One token (decode at T = 1): the selection as router_select_kernel, then the
// dispatch of its k pairs in the same CTA -- a stable sort by expert of k
// values, the offsets and the grouped experts' plan -- which saves the
// dispatch kernel's launch and dependency on the layer's critical path.  The
// result equals dispatch_kernel's for the same ids.
template <int NJ>
__global__ void __launch_bounds__(kSelMaxThreads)
router_select_dispatch_kernel(const float* __restrict__ part, const float* __restrict__ pmax,
                              int nds, const float* __restrict__ bias, int E, int k, int mode,
                              int32_t* __restrict__ ids, float* __restrict__ weights,
                              float* __restrict__ row_max, SmallDispatch sd) {
  __shared__ float red[kSelMaxThreads / 128][kMaxE];
  __shared__ float lg[kMaxE];
  __shared__ int sel[kMaxK];
  __shared__ int sh[33];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31;
  const int Q = blockDim.x / 128;
  const int q = tid / 128;
  const int s0 = q * nds / Q, s1 = (q + 1) * nds / Q;
  const size_t stride = (size_t)E;
  for (int e = tid % 128; e < E; e += 128) {
    const float* p = part + e;
    float acc = 0.f;
    int s = s0;
    for (; s + 8 <= s1; s += 8) {
      float v8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v8[u] = p[(size_t)(s + u) * stride];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += v8[u];
    }
    for (; s < s1; ++s) acc += p[(size_t)s * stride];
    red[q][e] = acc;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    float acc = red[0][e];
    for (int qq = 1; qq < Q; ++qq) acc += red[qq][e];
    if (bias) acc += bias[e];
    lg[e] = acc;
  }
  if (row_max && tid >= 128 * (Q - 1) && tid < 128 * (Q - 1) + 32) {
    float m = 0.f;
    for (int s = lane; s < nds; s += 32) m = fmaxf(m, pmax[s]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) row_max[0] = m;
  }
  __syncthreads();
  if (tid < 32) {
    float v[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      v[j] = e < E ? lg[e] : 0.f;
    }
    select_warp<NJ>(v, E, k, mode, red[0], ids, weights);
    __syncwarp();
    if (lane < k) sel[lane] = ids[lane];
  }
  __syncthreads();
  // stable counting sort of the k pairs by expert
  if (tid < k) {
    const int ej = sel[tid];
    int rank = 0;
    for (int i = 0; i < k; ++i) rank += (sel[i] < ej || (sel[i] == ej && i < tid)) ? 1 : 0;
    sd.perm[rank] = tid;
    sd.inv[tid] = rank;
  }
  int n = 0, below = 0;
  if (tid < E) {
    for (int i = 0; i < k; ++i) {
      n += sel[i] == tid ? 1 : 0;
      below += sel[i] < tid ? 1 : 0;
    }
    sd.offsets[tid] = below;
  }
  if (tid == 0) sd.offsets[E] = k;
  if (sd.n_active)
    write_expert_plan(n, tid, E, sd.rpc, sd.max_groups, sh, sd.n_active, sd.active, sd.goff,
                      sd.coff, sd.done, sd.status);
}

// Workspace of moe_router: the status word, the partial logits and the
// partial row maxima.
static size_t router_ws(int T, int d, int E) {
  const RouterPlan p = router_plan(T, d, E);
  return 256 + align_up(router_part_floats(p, T, E) * sizeof(float), 256) +
         align_up((size_t)p.nds * T * sizeof(float), 256);
}

// Both passes; part / pmax hold the plan's partials (pmax only when row_max).
static int launch_router_passes(const float* x, const float* gate_w, const float* bias, int T,
                                int d, int E, int k, int layout, int mode, int32_t* ids,
                                float* weights, float* part, float* pmax, float* row_max,
                                cudaStream_t s, size_t max_parts = ~(size_t)0,
                                const SmallDispatch* sd = nullptr, float* xcopy = nullptr) {
  const RouterPlan p = router_plan(T, d, E, max_parts);
  const size_t red = (size_t)kRouterWarps * p.tt * 128 * sizeof(float);
  {
    static std::mutex mu;
    static bool attr_done[64] = {false};
    int dev = 0;
    MOE_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
      MOE_CUDA(cudaFuncSetAttribute(router_gemv_kernel<16>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
      MOE_CUDA(cudaFuncSetAttribute(router_gemv_kernel<8>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
      if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
  }
  const dim3 grid(p.nds, p.tiles);
  float* pm = row_max ? pmax : nullptr;
  if (p.gemm) {
    ::moe::ProfScope _prof(MOE_K_ROUTER, s);
    const dim3 g3(p.nds, p.tiles, (E + kRgTE - 1) / kRgTE);
    router_gemm_kernel<<<g3, kRgThreads, 0, s>>>(x, gate_w, T, d, E, layout, p.rows, part, pm,
                                                  xcopy);
  } else {
    ::moe::ProfScope _prof(MOE_K_ROUTER, s);
    switch (p.tt) {
      case 16:
        router_gemv_kernel<16><<<grid, kRouterThreads, red, s>>>(x, gate_w, T, d, E, layout,
                                                                 p.rows, part, pm, xcopy);
        break;
      case 8:
        router_gemv_kernel<8><<<grid, kRouterThreads, red, s>>>(x, gate_w, T, d, E, layout,
                                                                p.rows, part, pm, xcopy);
        break;
      case 4:
        router_gemv_kernel<4><<<grid, kRouterThreads, red, s>>>(x, gate_w, T, d, E, layout,
                                                                p.rows, part, pm, xcopy);
        break;
      default:
        router_gemv_kernel<1><<<grid, kRouterThreads, red, s>>>(x, gate_w, T, d, E, layout,
                                                                p.rows, part, pm, xcopy);
    }
  }
  MOE_CHECK(check_launch("router_gemv"));
  {
    ::moe::ProfScope _prof(MOE_K_ROUTER_SELECT, s);
    // thread groups per token: about 8 slices each, at most 4
    const int Q = std::max(1, std::min(kSelMaxThreads / 128, p.nds / 8));
    const dim3 grid2(T), block2(128 * Q);
    const float* pc = part;
    const float* pmc = pm;
    if (sd) {
      // one token: selection and dispatch in one CTA of at least E threads
      const dim3 b1(128 * std::max(Q, (E + 127) / 128));
      if (E <= 32)
        MOE_CUDA(launch_pdl(router_select_dispatch_kernel<1>, dim3(1), b1, 0, s, pc, pmc, p.nds,
                            bias, E, k, mode, ids, weights, row_max, *sd));
      else if (E <= 128)
        MOE_CUDA(launch_pdl(router_select_dispatch_kernel<4>, dim3(1), b1, 0, s, pc, pmc, p.nds,
                            bias, E, k, mode, ids, weights, row_max, *sd));
      else
        MOE_CUDA(launch_pdl(router_select_dispatch_kernel<kMaxE / 32>, dim3(1), b1, 0, s, pc,
                            pmc, p.nds, bias, E, k, mode, ids, weights, row_max, *sd));
      return check_launch("router_select_dispatch");
    }
    if (E <= 32)
      MOE_CUDA(launch_pdl(router_select_kernel<1>, grid2, block2, 0, s, pc, pmc, p.nds, bias, T,
                          E, k, mode, ids, weights, row_max));
    else if (E <= 128)
      MOE_CUDA(launch_pdl(router_select_kernel<4>, grid2, block2, 0, s, pc, pmc, p.nds, bias, T,
                          E, k, mode, ids, weights, row_max));
    else
      MOE_CUDA(launch_pdl(router_select_kernel<kMaxE / 32>, grid2, block2, 0, s, pc, pmc, p.nds,
                          bias, T, E, k, mode, ids, weights, row_max));
  }
  return check_launch("router_select");
}

static int check_router_args(const float* x, const float* gate_w, int T, int d, int E, int k,
                             int layout, int mode, const int32_t* ids, const float* weights) {
  MOE_REQUIRE(x && gate_w && ids && weights, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(d > 0 && E > 0 && k > 0, MOE_ERR_INVALID, "d, E and k must be positive");
  MOE_REQUIRE(k <= E, MOE_ERR_INVALID, "top_k %d exceeds the expert count %d", k, E);
  MOE_REQUIRE(k <= kMaxK, MOE_ERR_UNSUPPORTED, "top_k %d above %d", k, kMaxK);
  MOE_REQUIRE(E % 4 == 0 && E <= kMaxE, MOE_ERR_UNSUPPORTED,
              "expert count %d must be a multiple of 4 and <= %d", E, kMaxE);
  MOE_REQUIRE(layout == MOE_ROUTER_D_E || layout == MOE_ROUTER_E_D, MOE_ERR_INVALID,
              "bad router layout %d", layout);
  MOE_REQUIRE(mode == MOE_ROUTE_TOPK_SOFTMAX || mode == MOE_ROUTE_SOFTMAX_TOPK_RENORM,
              MOE_ERR_INVALID, "bad routing mode %d", mode);
  MOE_REQUIRE(d % 4 == 0, MOE_ERR_UNSUPPORTED, "d=%d must be a multiple of 4", d);
  MOE_REQUIRE(((uintptr_t)x & 15) == 0, MOE_ERR_INVALID, "x not 16B aligned");
  MOE_REQUIRE(((uintptr_t)gate_w & 15) == 0, MOE_ERR_INVALID, "router weight not 16B aligned");
  return MOE_OK;
}

// moe_router plus, when row_max is given, each token's max |x| (used by the
// activation prep of the grouped experts).
int launch_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
                  int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream, float* row_max,
                  const SmallDispatch* sd, float* xcopy) {
  MOE_REQUIRE(T >= 0, MOE_ERR_INVALID, "T must be >= 0");
  MOE_REQUIRE(!sd || router_fuses_dispatch(T, E, k), MOE_ERR_INVALID,
              "the fused dispatch serves one token");
  if (T == 0) return MOE_OK;
  MOE_CHECK(check_router_args(x, gate_w, T, d, E, k, layout, mode, ids, weights));
  MOE_REQUIRE(workspace, MOE_ERR_INVALID, "null workspace");
  MOE_REQUIRE(workspace_bytes >= router_ws(T, d, E), MOE_ERR_WORKSPACE,
              "router workspace %zu < %zu", workspace_bytes, router_ws(T, d, E));
  const RouterPlan p = router_plan(T, d, E);
  uint8_t* base = static_cast<uint8_t*>(workspace) + 256;
  float* part = reinterpret_cast<float*>(base);
  float* pmax = reinterpret_cast<float*>(
      base + align_up(router_part_floats(p, T, E) * sizeof(float), 256));
  return launch_router_passes(x, gate_w, bias, T, d, E, k, layout, mode, ids, weights, part,
                              pmax, row_max, stream, ~(size_t)0, sd, xcopy);
}

bool router_fuses_dispatch(int T, int E, int k) {
  return T == 1 && E <= kSelMaxThreads && k <= kMaxK;
}

}  // namespace moe

extern "C" {

int moe_router_workspace_bytes(int T, int d, int E, size_t* bytes) {
  MOE_REQUIRE(bytes, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(T >= 0 && d > 0 && E > 0, MOE_ERR_INVALID, "bad shape");
  *bytes = moe::router_ws(T, d, E);
  return MOE_OK;
}

int moe_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
               int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
               size_t workspace_bytes, moe_stream_t stream) {
  return moe::launch_router(x, gate_w, bias, T, d, E, k, layout, mode, ids, weights, workspace,
                            workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr,
                            nullptr, nullptr);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free router.
//
// Some callers cannot give this library a workspace: they run where no device
// allocation may happen at all -- a host program that has already handed every
// byte of device memory to its own pool, or a serving loop that must keep a
// fixed memory footprint -- so neither the caller nor the library may call
// cudaMalloc.  moe_router_noalloc serves them: it takes the same inputs and
// outputs as moe_router, and keeps its only scratch (the per-slice partial
// logits, slices x T x E floats) in the fixed array below, which is part of the
// library image.  Every GPU that loads the library holds these 4 MiB until the
// process exits.
//
// Host code cannot use the array's name as a device address (on the host it
// names a host-side stand-in), so the address is looked up with
// cudaGetSymbolAddress once per device, with that device current, on the first
// call made on that device; make that first call before any stream capture.
// The looked-up address is kept for the rest of the process: after a
// cudaDeviceReset the device's module is loaded again and may sit elsewhere,
// so a process that resets a device must not call this entry point again.
// All calls share the array and it keeps the last call's contents.  Nothing
// needs clearing: a call writes every partial logit it later reads.  Calls
// whose kernels overlap on the GPU (different streams, or different host
// threads) race on the array and must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace moe {

constexpr size_t kNoAllocScratchFloats = (size_t)1 << 20;  // 4 MiB of partial logits
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {nullptr};

static int noalloc_scratch(float** out) {
  int dev = -1;
  MOE_CUDA(cudaGetDevice(&dev));
  MOE_REQUIRE(dev >= 0 && dev < 64, MOE_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    MOE_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    MOE_REQUIRE(p != nullptr, MOE_ERR_CUDA, "no device address for the fixed router scratch");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MOE_OK;
}

}  // namespace moe

extern "C" int moe_router_noalloc(const float* x, const float* gate_w, const float* bias, int T,
                                  int d, int E, int k, int layout, int mode, int32_t* ids,
                                  float* weights, moe_stream_t stream) {
  using namespace moe;
  MOE_REQUIRE(T >= 0, MOE_ERR_INVALID, "T must be >= 0");
  if (T == 0) return MOE_OK;
  MOE_CHECK(check_router_args(x, gate_w, T, d, E, k, layout, mode, ids, weights));
  const RouterPlan p = router_plan(T, d, E, kNoAllocScratchFloats);
  const size_t need = router_part_floats(p, T, E);
  MOE_REQUIRE(need <= kNoAllocScratchFloats, MOE_ERR_WORKSPACE,
              "moe_router_noalloc: T=%d E=%d needs %zu partial logits (%d slices), above the "
              "fixed scratch of %zu floats; call moe_router with a workspace instead",
              T, E, need, p.nds, kNoAllocScratchFloats);
  float* part = nullptr;
  MOE_CHECK(noalloc_scratch(&part));
  return launch_router_passes(x, gate_w, bias, T, d, E, k, layout, mode, ids, weights, part,
                              nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream),
                              kNoAllocScratchFloats);
}
