// Router: logits = x @ G (+ bias), top-k selection and softmax weights.
//
// moe_forward.py:91-109 (MoERouter.route: top-k of the logits, descending, then
// softmax over the k selected logits) and nightmare_stream.py:3227-3238
// (softmax over all experts, top-k of the probabilities, ascending, renormalised).
//
// Pass 1 (router_partial_kernel): a grid of (token tile, d-slice) CTAs; each
// stages its slice of the router matrix in shared memory and accumulates
// partial logits for its tokens in registers.  Pass 2 (router_select_kernel):
// one warp per token sums the d-slice partials in a fixed order, then selects
// and weighs the experts.  Sums use numpy's float32 order (sequential below 8
// terms, 8-way pairwise at and above) so the denominators follow the reference.
#include <math.h>

#include <cooperative_groups.h>

#include <mutex>

#include "moe_common.cuh"

namespace moe {

constexpr int kRouterThreads = 256;
constexpr int kRouterDC = 64;        // rows of G per staged chunk
constexpr int kRouterTPT = 4;        // tokens per thread
constexpr int kMaxE = 512;
constexpr int kMaxK = 32;

struct RouterPlan {
  int ct;        // column threads (E / 4)
  int tg;        // token groups per CTA
  int tt;        // tokens per CTA
  int tiles;     // token tiles
  int nds;       // d-slices
  int chunks;    // d-chunks per slice
};

static RouterPlan router_plan(int T, int d, int E) {
  RouterPlan p;
  p.ct = E / 4;
  p.tg = kRouterThreads / p.ct;
  if (p.tg > 8) p.tg = 8;
  p.tt = p.tg * kRouterTPT;
  p.tiles = (T + p.tt - 1) / p.tt;
  int total_chunks = (d + kRouterDC - 1) / kRouterDC;
  int want = (2 * sm_count() + p.tiles - 1) / p.tiles;
  p.nds = want < 1 ? 1 : (want > total_chunks ? total_chunks : want);
  p.chunks = (total_chunks + p.nds - 1) / p.nds;
  p.nds = (total_chunks + p.chunks - 1) / p.chunks;
  return p;
}

__global__ void __launch_bounds__(kRouterThreads)
router_partial_kernel(const float* __restrict__ x, const float* __restrict__ G, int T, int d,
                      int E, int layout, int tt, int chunks, float* __restrict__ part) {
  extern __shared__ float smem[];
  float* gs = smem;                                  // [kRouterDC][E]
  float* xs = smem + kRouterDC * E;                  // [tt][kRouterDC + 1]
  const int ct = E / 4;
  const int tid = threadIdx.x;
  const int col = tid % ct;                          // experts 4*col .. 4*col+3
  const int tgrp = tid / ct;
  const int tg = blockDim.x / ct;
  const int t0 = blockIdx.x * tt;
  const int slice = blockIdx.y;
  float acc[kRouterTPT][4];
#pragma unroll
  for (int a = 0; a < kRouterTPT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;

  for (int c = 0; c < chunks; ++c) {
    const int i0 = (slice * chunks + c) * kRouterDC;
    if (i0 >= d) break;
    const int rows = min(kRouterDC, d - i0);
    __syncthreads();
    // stage G[i0 : i0+rows, :] as [row][E]
    if (layout == MOE_ROUTER_D_E) {
      const float4* src = reinterpret_cast<const float4*>(G + (size_t)i0 * E);
      float4* dst = reinterpret_cast<float4*>(gs);
      for (int v = tid; v < rows * E / 4; v += blockDim.x) dst[v] = __ldg(src + v);
    } else {
      for (int v = tid; v < rows * E; v += blockDim.x) {
        int e = v / rows, i = v % rows;
        gs[i * E + e] = __ldg(G + (size_t)e * d + i0 + i);
      }
    }
    // stage x[t0 : t0+tt, i0 : i0+rows]
    for (int v = tid; v < tt * kRouterDC; v += blockDim.x) {
      int tl = v / kRouterDC, i = v % kRouterDC;
      int t = t0 + tl;
      xs[tl * (kRouterDC + 1) + i] = (t < T && i < rows) ? __ldg(x + (size_t)t * d + i0 + i) : 0.f;
    }
    __syncthreads();
    for (int i = 0; i < rows; ++i) {
      float4 g4 = *reinterpret_cast<const float4*>(gs + i * E + 4 * col);
#pragma unroll
      for (int a = 0; a < kRouterTPT; ++a) {
        float xv = xs[(tgrp + a * tg) * (kRouterDC + 1) + i];
        acc[a][0] = fmaf(xv, g4.x, acc[a][0]);
        acc[a][1] = fmaf(xv, g4.y, acc[a][1]);
        acc[a][2] = fmaf(xv, g4.z, acc[a][2]);
        acc[a][3] = fmaf(xv, g4.w, acc[a][3]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < kRouterTPT; ++a) {
    int t = t0 + tgrp + a * tg;
    if (t < T) {
      float4 v = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
      *reinterpret_cast<float4*>(part + ((size_t)slice * T + t) * E + 4 * col) = v;
    }
  }
}

// a beats b: larger value, NaN above numbers, equal values -> higher index.
__device__ __forceinline__ bool beats(float a, int ia, float b, int ib) {
  bool na = isnan(a), nb = isnan(b);
  if (na != nb) return na;
  if (na) return ia > ib;
  return a > b || (a == b && ia > ib);
}

// Selection and weights for one token whose E logits (bias included) sit in
// shared memory; executed by one warp.  Same rules as router_select_kernel.
__device__ void select_token(const float* __restrict__ lg, float* __restrict__ buf,
                             float* __restrict__ sv, int E, int k, int mode,
                             int32_t* __restrict__ ids_t, float* __restrict__ w_t) {
  const int lane = threadIdx.x & 31;
  const int J = (E + 31) / 32;
  float v[kMaxE / 32];
#pragma unroll
  for (int j = 0; j < kMaxE / 32; ++j) {
    const int e = lane + 32 * j;
    v[j] = (j < J && e < E) ? lg[e] : 0.f;
  }
  if (mode == MOE_ROUTE_SOFTMAX_TOPK_RENORM) {
    float m = -INFINITY;
    bool any_nan = false;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      if (j < J && e < E) {
        any_nan |= isnan(v[j]);
        m = fmaxf(m, v[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    any_nan = __any_sync(0xffffffffu, any_nan);
    if (any_nan) m = NAN;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      if (j < J && e < E) {
        v[j] = expf(v[j] - m);
        buf[e] = v[j];
      }
    }
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, E);
    s = __shfl_sync(0xffffffffu, s, 0);
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) v[j] = v[j] / s;
  }
  unsigned taken = 0u;
  int sel_id = -1;
  float sel_val = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = -1;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      const int e = lane + 32 * j;
      if (j < J && e < E && !((taken >> j) & 1u)) {
        if (bi < 0 || beats(v[j], e, bv, bi)) {
          bv = v[j];
          bi = e;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || beats(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == 0) sv[r] = bv;
    if (lane == r) {
      sel_id = bi;
      sel_val = bv;
    }
  }
  __syncwarp();
  if (mode == MOE_ROUTE_TOPK_SOFTMAX) {
    float mx = sv[0];
    for (int r = 1; r < k; ++r) mx = fmaxf(mx, sv[r]);
    __syncwarp();
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
    const int pos = k - 1 - lane;
    __syncwarp();
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

// Router in one launch: a cluster of kRouterCluster CTAs per token tile.  CTA
// rank r accumulates partial logits of the tile's tokens over its d-range:
// 32-row chunks of the router matrix and the matching slice of the tokens
// stream through a ring of up to kFusedMaxStages shared-memory stages filled
// by bulk copies (TMA) -- for decode-sized d every chunk of the CTA's range is
// in flight at once -- and each thread
// keeps TPT tokens x 4 experts of partial sums in registers.  The partials stay
// in the CTA's shared memory; after a cluster barrier CTA r sums, for its share
// of the tile's tokens, the partials of ranks 0..C-1 in rank order through
// distributed shared memory, adds the bias and selects with one warp per token.
// The same pass records each token's max |x| when row_max is given.
constexpr int kRouterCluster = 8;
constexpr int kFusedDC = 32;            // router rows per chunk
constexpr int kFusedXP = kFusedDC + 4;  // padded x row (16-byte aligned)
constexpr int kFusedMaxStages = 16;

struct FusedShape {
  int ct, tg, tt, per, tiles;
};

// Thread shape of router_fused_kernel: ct threads cover the E experts (4 each),
// tg token groups of TPT tokens fill the 256 threads; tt = tg * TPT tokens per
// cluster, a multiple of the cluster size so every rank reduces per = tt / C.
static FusedShape fused_shape(int T, int E, int tpt) {
  FusedShape f;
  f.ct = E / 4;
  f.tg = kRouterThreads / f.ct;
  if (f.tg >= kRouterCluster) f.tg -= f.tg % kRouterCluster;
  f.tt = f.tg * tpt;
  f.per = f.tt / kRouterCluster;
  f.tiles = (T + f.tt - 1) / f.tt;
  return f;
}

static size_t fused_smem(const FusedShape& f, int E, int nst) {
  return ((size_t)nst * kFusedDC * E + (size_t)nst * f.tt * kFusedXP + (size_t)f.tt * E +
          (size_t)f.per * E + (size_t)(kRouterThreads / 32) * (kMaxE + kMaxK) + (size_t)f.tt) *
             sizeof(float) +
         8 * (size_t)nst + 64;
}

// Ring depth.  A grid that fits in one wave keeps every chunk of a rank's
// d-range in flight (as many as shared memory holds); a larger grid keeps two
// stages so that several CTAs share an SM.
static int fused_stages(const FusedShape& f, int d, int E) {
  const int nchunks = (d + kFusedDC - 1) / kFusedDC;
  if (f.tiles * kRouterCluster > sm_count()) return 2;
  int nst = std::min(kFusedMaxStages, (nchunks + kRouterCluster - 1) / kRouterCluster);
  while (nst > 2 && fused_smem(f, E, nst) > 227 * 1024) --nst;
  return std::max(nst, 1);
}

template <int TPT>
__global__ void __launch_bounds__(kRouterThreads)
router_fused_kernel(const float* __restrict__ x, const float* __restrict__ G,
                    const float* __restrict__ bias, int T, int d, int E, int k, int layout,
                    int mode, int tg, int nst, int32_t* __restrict__ ids,
                    float* __restrict__ weights, float* __restrict__ row_max,
                    int* __restrict__ status) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) float smem[];
  constexpr int NT = kRouterThreads;
  constexpr int NW = NT / 32;
  const int ct = E / 4;
  const int tt = tg * TPT;
  const int per = tt / kRouterCluster;
  float* gbuf = smem;                                // [nst][kFusedDC][E] (E_D: [nst][E][kFusedDC])
  float* xbuf = gbuf + nst * kFusedDC * E;           // [nst][tt][kFusedXP]
  float* part = xbuf + nst * tt * kFusedXP;          // [tt][E] partial logits
  float* lg = part + tt * E;                         // [per][E] reduced logits
  float* buf = lg + per * E;                         // [NW][kMaxE]
  float* sv = buf + NW * kMaxE;                      // [NW][kMaxK]
  float* xmax = sv + NW * kMaxK;                     // [tt]
  uint64_t* bar = reinterpret_cast<uint64_t*>(xmax + tt + ((tt & 1) ? 1 : 0));  // [nst]
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int col = tid % ct;
  const int tgrp = tid / ct;                         // >= tg: idle in the compute
  const int rank = (int)cluster.block_rank();
  const int t0 = (blockIdx.x / kRouterCluster) * tt;
  const int nchunks = (d + kFusedDC - 1) / kFusedDC;
  const int cb = rank * nchunks / kRouterCluster, ce = (rank + 1) * nchunks / kRouterCluster;
  const int nvalid = max(0, min(tt, T - t0));
  if (tid == 0) {
    for (int i = 0; i < nst; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  // rows of tokens past T stay zero in every stage
  for (int v = tid; v < nst * tt * kFusedXP; v += NT) {
    const int tl = (v / kFusedXP) % tt;
    if (tl >= nvalid) xbuf[v] = 0.f;
  }
  for (int tl = tid; tl < tt; tl += NT) xmax[tl] = 0.f;
  __syncthreads();

  // warp 0 issues one chunk into a stage: the router rows and the tile's x slice
  auto issue = [&](int c, int stg) {
    if (warp != 0) return;
    const int i0 = c * kFusedDC;
    const int rows = min(kFusedDC, d - i0);
    float* gs = gbuf + stg * kFusedDC * E;
    float* xs = xbuf + stg * tt * kFusedXP;
    const uint32_t gbytes = (uint32_t)(rows * E * 4);
    const uint32_t xbytes = (uint32_t)(rows * 4);
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_expect_tx(&bar[stg], gbytes + xbytes * nvalid);
    }
    __syncwarp();
    if (layout == MOE_ROUTER_D_E) {
      if (lane == 0) bulk_g2s_plain(gs, G + (size_t)i0 * E, gbytes, &bar[stg]);
    } else {
      for (int e = lane; e < E; e += 32)
        bulk_g2s_plain(gs + e * kFusedDC, G + (size_t)e * d + i0, xbytes, &bar[stg]);
    }
    for (int tl = lane; tl < nvalid; tl += 32)
      bulk_g2s_plain(xs + tl * kFusedXP, x + (size_t)(t0 + tl) * d + i0, xbytes, &bar[stg]);
  };

  float acc[TPT][4];
#pragma unroll
  for (int a = 0; a < TPT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  for (int i = 0; i < nst && cb + i < ce; ++i) issue(cb + i, i);
  bool ok = true;
  for (int c = cb; c < ce; ++c) {
    const int stg = (c - cb) % nst;
    const uint32_t parity = ((c - cb) / nst) & 1;
    if (ok && !mbar_wait(&bar[stg], parity)) {
      set_status(status, MOE_STATUS_TIMEOUT);
      ok = false;
    }
    const int rows = min(kFusedDC, d - c * kFusedDC);
    const float* gs = gbuf + stg * kFusedDC * E;
    const float* xs = xbuf + stg * tt * kFusedXP;
    if (row_max) {  // each token row owned by one thread
      for (int tl = tid; tl < tt; tl += NT) {
        float m = xmax[tl];
        for (int i = 0; i < rows; ++i) m = fmaxf(m, fabsf(xs[tl * kFusedXP + i]));
        xmax[tl] = m;
      }
    }
    if (tgrp < tg) {
      if (layout == MOE_ROUTER_D_E) {
        for (int i = 0; i < rows; ++i) {
          const float4 g4 = *reinterpret_cast<const float4*>(gs + i * E + 4 * col);
#pragma unroll
          for (int a = 0; a < TPT; ++a) {
            const float xv = xs[(tgrp + a * tg) * kFusedXP + i];
            acc[a][0] = fmaf(xv, g4.x, acc[a][0]);
            acc[a][1] = fmaf(xv, g4.y, acc[a][1]);
            acc[a][2] = fmaf(xv, g4.z, acc[a][2]);
            acc[a][3] = fmaf(xv, g4.w, acc[a][3]);
          }
        }
      } else {
        for (int i = 0; i < rows; ++i) {
          float g[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) g[j] = gs[(4 * col + j) * kFusedDC + i];
#pragma unroll
          for (int a = 0; a < TPT; ++a) {
            const float xv = xs[(tgrp + a * tg) * kFusedXP + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[a][j] = fmaf(xv, g[j], acc[a][j]);
          }
        }
      }
    }
    if (c + nst < ce) {
      __syncthreads();  // stage fully read before it is refilled
      if (ok) issue(c + nst, stg);
    }
  }
  if (tgrp < tg) {
#pragma unroll
    for (int a = 0; a < TPT; ++a) {
      const float4 v = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
      *reinterpret_cast<float4*>(part + (tgrp + a * tg) * E + 4 * col) = v;
    }
  }
  cluster.sync();
  // reduce this rank's tokens over the cluster, in rank order
  for (int v = tid; v < per * E; v += NT) {
    const int tl = rank * per + v / E, e = v % E;
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < kRouterCluster; ++q) sum += cluster.map_shared_rank(part, q)[tl * E + e];
    if (bias) sum += __ldg(bias + e);
    lg[(v / E) * E + e] = sum;
  }
  if (row_max) {
    for (int i = tid; i < per; i += NT) {
      const int tl = rank * per + i;
      float m = 0.f;
#pragma unroll
      for (int q = 0; q < kRouterCluster; ++q) m = fmaxf(m, cluster.map_shared_rank(xmax, q)[tl]);
      if (t0 + tl < T) row_max[t0 + tl] = m;
    }
  }
  __syncthreads();
  for (int i = warp; i < per; i += NW) {
    const int t = t0 + rank * per + i;
    if (t < T)
      select_token(lg + i * E, buf + warp * kMaxE, sv + warp * kMaxK, E, k, mode,
                   ids + (size_t)t * k, weights + (size_t)t * k);
  }
  cluster.sync();  // peers may still be reading this CTA's partials
}

// One warp per token.  Lanes hold logits e = lane + 32 j.
__global__ void __launch_bounds__(128)
router_select_kernel(const float* __restrict__ part, int nds, const float* __restrict__ bias,
                     int T, int E, int k, int mode, int32_t* __restrict__ ids,
                     float* __restrict__ weights) {
  __shared__ float sbuf[4][kMaxE];
  __shared__ float ssel[4][kMaxK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= T) return;
  const int J = (E + 31) / 32;
  float v[kMaxE / 32];
#pragma unroll
  for (int j = 0; j < kMaxE / 32; ++j) {
    int e = lane + 32 * j;
    float acc = 0.f;
    if (j < J && e < E) {
      // fixed summation order; loads issued eight at a time
      int s = 0;
      for (; s + 8 <= nds; s += 8) {
        float v8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v8[u] = part[((size_t)(s + u) * T + t) * E + e];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += v8[u];
      }
      for (; s < nds; ++s) acc += part[((size_t)s * T + t) * E + e];
      if (bias) acc += bias[e];
    }
    v[j] = acc;
  }
  float* buf = sbuf[warp];
  if (mode == MOE_ROUTE_SOFTMAX_TOPK_RENORM) {
    // probs = exp(l - max) / sum(exp(l - max)) over all experts
    float m = -INFINITY;
    bool any_nan = false;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      int e = lane + 32 * j;
      if (j < J && e < E) {
        any_nan |= isnan(v[j]);
        m = fmaxf(m, v[j]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    any_nan = __any_sync(0xffffffffu, any_nan);
    if (any_nan) m = NAN;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      int e = lane + 32 * j;
      if (j < J && e < E) {
        v[j] = expf(v[j] - m);
        buf[e] = v[j];
      }
    }
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, E);
    s = __shfl_sync(0xffffffffu, s, 0);
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) v[j] = v[j] / s;
  }
  // k rounds of warp arg-max
  unsigned taken = 0u;  // bit j: lane's element j already selected
  int sel_id = -1;
  float sel_val = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = -1;
#pragma unroll
    for (int j = 0; j < kMaxE / 32; ++j) {
      int e = lane + 32 * j;
      if (j < J && e < E && !((taken >> j) & 1u)) {
        if (bi < 0 || beats(v[j], e, bv, bi)) {
          bv = v[j];
          bi = e;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || beats(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == 0) ssel[warp][r] = bv;
    if (lane == r) {
      sel_id = bi;
      sel_val = bv;
    }
  }
  __syncwarp();
  // weights, in the reference's output order
  float* sv = ssel[warp];
  if (mode == MOE_ROUTE_TOPK_SOFTMAX) {
    // descending order; softmax over the k selected logits
    float mx = sv[0];
    for (int r = 1; r < k; ++r) mx = fmaxf(mx, sv[r]);  // np.max
    __syncwarp();
    if (lane < k) buf[lane] = expf(sel_val - mx);
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, k);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (lane < k) {
      ids[(size_t)t * k + lane] = sel_id;
      weights[(size_t)t * k + lane] = buf[lane] / s;
    }
  } else {
    // ascending order (argsort(probs)[-k:]); renormalise by their sum
    int pos = k - 1 - lane;  // lane r holds the r-th largest -> output position k-1-r
    __syncwarp();
    if (lane < k) buf[pos] = sel_val;
    __syncwarp();
    float s = 0.f;
    if (lane == 0) s = np_pairwise_sum(buf, k);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (lane < k) {
      ids[(size_t)t * k + pos] = sel_id;
      weights[(size_t)t * k + pos] = sel_val / s;
    }
  }
}

// moe_router keeps its partial logits in shared memory (cluster reduction);
// the workspace only carries the status word.
static size_t router_ws(int T, int d, int E) {
  (void)T;
  (void)d;
  (void)E;
  return 256;
}

}  // namespace moe

namespace moe {
int launch_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
                  int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream, float* row_max);
}

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
                            workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"

namespace moe {

// moe_router plus, when row_max is given, each token's max |x| (used by the
// expert activation prep of the fused layer).
int launch_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
                  int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream, float* row_max) {
  MOE_REQUIRE(T >= 0, MOE_ERR_INVALID, "T must be >= 0");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(x && gate_w && ids && weights && workspace, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(d > 0 && E > 0 && k > 0, MOE_ERR_INVALID, "d, E and k must be positive");
  MOE_REQUIRE(k <= E, MOE_ERR_INVALID, "top_k %d exceeds the expert count %d", k, E);
  MOE_REQUIRE(k <= kMaxK, MOE_ERR_UNSUPPORTED, "top_k %d above %d", k, kMaxK);
  MOE_REQUIRE(E % 4 == 0 && E <= kMaxE, MOE_ERR_UNSUPPORTED,
              "expert count %d must be a multiple of 4 and <= %d", E, kMaxE);
  MOE_REQUIRE(layout == MOE_ROUTER_D_E || layout == MOE_ROUTER_E_D, MOE_ERR_INVALID,
              "bad router layout %d", layout);
  MOE_REQUIRE(mode == MOE_ROUTE_TOPK_SOFTMAX || mode == MOE_ROUTE_SOFTMAX_TOPK_RENORM,
              MOE_ERR_INVALID, "bad routing mode %d", mode);
  MOE_REQUIRE(workspace_bytes >= router_ws(T, d, E), MOE_ERR_WORKSPACE,
              "router workspace %zu < %zu", workspace_bytes, router_ws(T, d, E));
  MOE_REQUIRE(((uintptr_t)gate_w & 15) == 0, MOE_ERR_INVALID, "router weight not 16B aligned");
  cudaStream_t s = stream;
  MOE_REQUIRE(d % 4 == 0, MOE_ERR_UNSUPPORTED, "d=%d must be a multiple of 4", d);
  MOE_REQUIRE(((uintptr_t)x & 15) == 0, MOE_ERR_INVALID, "x not 16B aligned");
  // one token per thread for small batches (more clusters), four for large
  // ones or when few token groups fit beside the experts
  const int tg1 = fused_shape(T, E, 1).tg;
  const int tpt = (tg1 < kRouterCluster || (T > 256 && tg1 <= kRouterCluster)) ? 4 : 1;
  const FusedShape f = fused_shape(T, E, tpt);
  const int nst = fused_stages(f, d, E);
  const size_t smem = fused_smem(f, E, nst);
  MOE_REQUIRE(f.per >= 1 && f.tt % kRouterCluster == 0 && f.ct * f.tg <= kRouterThreads &&
                  smem <= 227 * 1024,
              MOE_ERR_UNSUPPORTED, "router shape E=%d does not fit the fused router", E);
  static std::mutex attr_mu;
  static int attr_smem[2][64] = {{0}};  // largest size set so far, per instance and device
  {
    int dev = 0;
    MOE_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(attr_mu);
    const int ti = tpt == 1 ? 0 : 1;
    if (dev < 0 || dev >= 64 || attr_smem[ti][dev] < (int)smem) {
      if (tpt == 1)
        MOE_CUDA(cudaFuncSetAttribute(router_fused_kernel<1>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      else
        MOE_CUDA(cudaFuncSetAttribute(router_fused_kernel<4>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (dev >= 0 && dev < 64) attr_smem[ti][dev] = (int)smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(f.tiles * kRouterCluster);
  cfg.blockDim = dim3(kRouterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRouterCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int* status = workspace ? static_cast<int*>(workspace) : nullptr;
  {
    ::moe::ProfScope _prof(MOE_K_ROUTER, s);
    if (tpt == 1)
      MOE_CUDA(cudaLaunchKernelEx(&cfg, router_fused_kernel<1>, x, gate_w, bias, T, d, E, k,
                                  layout, mode, f.tg, nst, ids, weights, row_max, status));
    else
      MOE_CUDA(cudaLaunchKernelEx(&cfg, router_fused_kernel<4>, x, gate_w, bias, T, d, E, k,
                                  layout, mode, f.tg, nst, ids, weights, row_max, status));
  }
  return check_launch("router_fused");
}

}  // namespace moe

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
  MOE_REQUIRE(((uintptr_t)gate_w & 15) == 0, MOE_ERR_INVALID, "router weight not 16B aligned");
  RouterPlan p = router_plan(T, d, E);
  const size_t need = (size_t)p.nds * T * E;
  MOE_REQUIRE(need <= kNoAllocScratchFloats, MOE_ERR_WORKSPACE,
              "moe_router_noalloc: T=%d E=%d needs %zu partial logits (%d slices), above the "
              "fixed scratch of %zu floats; call moe_router with a workspace instead",
              T, E, need, p.nds, kNoAllocScratchFloats);
  float* part = nullptr;
  MOE_CHECK(noalloc_scratch(&part));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  size_t smem = ((size_t)kRouterDC * E + (size_t)p.tt * (kRouterDC + 1)) * sizeof(float);
  if (smem > 48 * 1024) {
    MOE_CUDA(cudaFuncSetAttribute(router_partial_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  dim3 grid(p.tiles, p.nds);
  {
    ::moe::ProfScope _prof(MOE_K_ROUTER, s);
    router_partial_kernel<<<grid, p.ct * p.tg, smem, s>>>(x, gate_w, T, d, E, layout, p.tt,
                                                          p.chunks, part);
  }
  MOE_CHECK(check_launch("router_partial"));
  {
    ::moe::ProfScope _prof(MOE_K_ROUTER_SELECT, s);
    router_select_kernel<<<(T + 3) / 4, 128, 0, s>>>(part, p.nds, bias, T, E, k, mode, ids,
                                                     weights);
  }
  return check_launch("router_select");
}
