// Shared device/host helpers for the MoE layer kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <utility>
#include <stdint.h>

#include "moe_b200.h"

namespace moe {

// ---------------------------------------------------------------------------
// host-side error reporting: every C entry point returns a status and leaves a
// message retrievable with moe_last_error().
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);

#define MOE_REQUIRE(cond, status, ...)            \
  do {                                            \
    if (!(cond)) return ::moe::fail(status, __VA_ARGS__); \
  } while (0)

#define MOE_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t _e = (call);                                                  \
    if (_e != cudaSuccess)                                                    \
      return ::moe::fail(MOE_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
  } while (0)

#define MOE_CHECK(call)             \
  do {                              \
    int _s = (call);                \
    if (_s != MOE_OK) return _s;    \
  } while (0)

int sm_count();

// Per-kernel event profiling (see moe_profile_enable).
void prof_begin(int kernel_id, cudaStream_t s);
void prof_end(cudaStream_t s);

// Launch that may begin while the previous kernel on the stream is still
// running (programmatic dependent launch).  The kernel must execute
// pdl_wait() before it reads anything the previous kernel writes; the
// previous kernel lets it start early with pdl_trigger().
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Brackets one kernel launch with the profiler's events.
struct ProfScope {
  cudaStream_t s;
  ProfScope(int kid, cudaStream_t st) : s(st) { prof_begin(kid, st); }
  ~ProfScope() { prof_end(s); }
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Simple bump allocator over a caller-provided workspace.
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t used;
  template <typename T>
  T* take(size_t count) {
    size_t off = align_up(used, 256);
    used = off + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + off) : nullptr;
  }
  bool fits() const { return used <= cap; }
};

// ---------------------------------------------------------------------------
// packed weight tiles
//
// A (rows, cols) quantised matrix is stored as (rows/16) strips of 16 rows;
// each strip is cols/64 tiles of 16 rows x 64 columns (two 32-weight blocks
// per row).  Inside a tile, the quant bytes come first, laid out so that lane
// L = 4g + t of a warp reads one contiguous vector with the bytes of rows g and
// g+8 it needs for an m16n8k16 A fragment; the fp16 block scales follow,
// 8 bytes per group g: d(g,b0) d(g,b1) d(g+8,b0) d(g+8,b1).
//   Q4_0: lane owns bytes [4t,4t+4) of each 16-byte quant array -> 16 B/lane
//   Q8_0: lane owns bytes [8t,8t+8) of each 32-byte quant array -> 32 B/lane
// The tile holds exactly the bytes of its 32 GGUF blocks, so a packed matrix
// has the same size as the raw one.
// ---------------------------------------------------------------------------
template <int QT> struct QTraits;
template <> struct QTraits<MOE_Q4_0> {
  static constexpr int kBlockBytes = 18;
  static constexpr int kQuantBytes = 16;
  static constexpr int kLaneBytes = 16;        // quant bytes per lane per tile
  static constexpr int kTileQuant = 512;
  static constexpr int kTileBytes = 576;
};
template <> struct QTraits<MOE_Q8_0> {
  static constexpr int kBlockBytes = 34;
  static constexpr int kQuantBytes = 32;
  static constexpr int kLaneBytes = 32;
  static constexpr int kTileQuant = 1024;
  static constexpr int kTileBytes = 1088;
};

inline int tile_bytes(int qtype) { return qtype == MOE_Q4_0 ? 576 : 1088; }
inline int block_bytes(int qtype) { return qtype == MOE_Q4_0 ? 18 : 34; }
inline bool qtype_ok(int qtype) { return qtype == MOE_Q4_0 || qtype == MOE_Q8_0; }
inline size_t matrix_bytes(int qtype, int rows, int cols) {
  return (size_t)rows * (cols / 32) * block_bytes(qtype);
}

// Element order of the activation fragments (the B operand): for a 32-wide
// block, the 8 halves lane t of a column reads, in register order
// (b0.lo, b0.hi, b1.lo, b1.hi) of the first k16 step then of the second.
// They must match the A-fragment element order the dequantiser produces.
__host__ __device__ inline int frag_elem(int qtype, int t, int i) {
  if (qtype == MOE_Q4_0) {
    // first k16 step: low nibbles of bytes 4t..4t+3 -> elements 4t+{0,2,1,3}
    // second k16 step: high nibbles -> elements 16+4t+{0,2,1,3}
    const int perm[4] = {0, 2, 1, 3};
    return (i < 4 ? 0 : 16) + 4 * t + perm[i & 3];
  }
  return 8 * t + i;  // Q8_0: int8 bytes 8t..8t+7 in order
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  // (a & mask) | orv  -> LUT 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}

__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// D = A(16x16,row) * B(16x8,col) + C, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// Q4_0 quant word (nibble bytes 4t..4t+3 of one row) -> A-fragment halves
// for the two k16 steps of the block: values (q - 8) exactly in fp16.
//   lo01: elements {4t, 4t+2}, lo23: {4t+1, 4t+3}
//   hi01: {16+4t, 16+4t+2},    hi23: {16+4t+1, 16+4t+3}
__device__ __forceinline__ void dequant_q4(uint32_t w, uint32_t& lo01, uint32_t& lo23,
                                           uint32_t& hi01, uint32_t& hi23) {
  const uint32_t kMagic = 0x64006400u;      // fp16 1024 in both halves
  const uint32_t kSubLo = 0xE408E408u;      // fp16 -1032
  const uint32_t kMulHi = 0x2C002C00u;      // fp16 1/16
  const uint32_t kSubHi = 0xD480D480u;      // fp16 -72
  uint32_t w8 = w >> 8;
  lo01 = hadd2_u(lop3_and_or(w, 0x000F000Fu, kMagic), kSubLo);
  lo23 = hadd2_u(lop3_and_or(w8, 0x000F000Fu, kMagic), kSubLo);
  hi01 = hfma2_u(lop3_and_or(w, 0x00F000F0u, kMagic), kMulHi, kSubHi);
  hi23 = hfma2_u(lop3_and_or(w8, 0x00F000F0u, kMagic), kMulHi, kSubHi);
}

// Q8_0 quant word (int8 bytes i..i+3) -> two fp16x2 with the exact values.
__device__ __forceinline__ void dequant_q8(uint32_t w, uint32_t& h01, uint32_t& h23) {
  const uint32_t kSub = 0xE480E480u;        // fp16 -1152
  uint32_t u = w ^ 0x80808080u;             // q + 128 as unsigned bytes
  h01 = hadd2_u(prmt(u, 0x64646464u, 0x5140u), kSub);
  h23 = hadd2_u(prmt(u, 0x64646464u, 0x7362u), kSub);
}

__device__ __forceinline__ float silu_f(float g) {
  // moe_forward.py:43-45: x / (1 + exp(-clip(x, -88, 88)))
  float c = fminf(fmaxf(g, -88.0f), 88.0f);
  return g / (1.0f + expf(-c));
}

// GeGLU with the tanh approximation, the gemma4 expert activation
// (qwen35_gpu.py:933-939, nightmare_stream.py:3256-3271):
// 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))).
__device__ __forceinline__ float gelu_tanh_f(float g) {
  const float a = 0.7978845608028654f * (g + 0.044715f * g * g * g);
  return 0.5f * g * (1.0f + tanhf(a));
}

// Gated activation of an expert: act(gate) (times up, by the caller).
__device__ __forceinline__ float expert_act(int act, float g) {
  return act == MOE_ACT_GEGLU_TANH ? gelu_tanh_f(g) : silu_f(g);
}

// numpy's float32 add.reduce order over n contiguous values (its pairwise
// summation): sequential below 8 terms, eight running sums up to 128 terms,
// and above that a split at n/2 rounded down to a multiple of 8.
static __device__ float np_pairwise_sum(const float* a, int n) {
  if (n < 8) {
    float res = 0.f;
    for (int i = 0; i < n; ++i) res = res + a[i];
    return res;
  }
  if (n <= 128) {
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = r[j] + a[i + j];
    }
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res = res + a[i];
    return res;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  return np_pairwise_sum(a, n2) + np_pairwise_sum(a + n2, n - n2);
}

// The same sum computed by a CTA: the leaves of the pairwise tree// The same sum computed by a CTA: the leaves of the pairwise tree (runs of at
// most 128 terms) are summed by separate threads, then thread 0 adds them along
// the tree.  Bit-identical to np_pairwise_sum.  Call from every thread; scratch
// holds one float per leaf (np_pairwise_leaves(n)); the result is valid in
// thread 0 after the call returns (the call ends with a barrier).
static __device__ int np_pairwise_leaves(int n) {
  if (n <= 128) return 1;
  int n2 = n / 2;
  n2 -= n2 % 8;
  return np_pairwise_leaves(n2) + np_pairwise_leaves(n - n2);
}

static __device__ void np_pairwise_leaf(int n, int idx, int& start, int& len) {
  start = 0;
  len = n;
  while (len > 128) {
    int n2 = len / 2;
    n2 -= n2 % 8;
    const int left = np_pairwise_leaves(n2);
    if (idx < left) {
      len = n2;
    } else {
      idx -= left;
      start += n2;
      len -= n2;
    }
  }
}

static __device__ float np_pairwise_combine(const float* leaf, int n, int& next) {
  if (n <= 128) return leaf[next++];
  int n2 = n / 2;
  n2 -= n2 % 8;
  const float l = np_pairwise_combine(leaf, n2, next);
  const float r = np_pairwise_combine(leaf, n - n2, next);
  return l + r;
}

static __device__ float np_pairwise_sum_cta(const float* a, int n, float* scratch) {
  const int L = np_pairwise_leaves(n);
  for (int t = threadIdx.x; t < L; t += blockDim.x) {
    int st, len;
    np_pairwise_leaf(n, t, st, len);
    scratch[t] = np_pairwise_sum(a + st, len);
  }
  __syncthreads();
  float res = 0.f;
  if (threadIdx.x == 0) {
    int next = 0;
    res = np_pairwise_combine(scratch, n, next);
  }
  __syncthreads();
  return res;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, 1-D) helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bulk global -> shared copy completing on an mbarrier; evict-first in L2
// (weights stream through once).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for an mbarrier phase.  Gives up (returns false; the caller
// flags MOE_STATUS_TIMEOUT) after ~0.2 s of wall time or 2^24 polls.  Each
// poll may suspend the thread in hardware for up to that many ns while the
// phase is incomplete, so a waiting warp takes few issue slots
// (MOE_MBAR_SUSPEND_NS, 0 for the hardware's default).
#ifndef MOE_MBAR_SUSPEND_NS
#define MOE_MBAR_SUSPEND_NS 20000
#endif

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  {
    // fast path: the phase is often complete already
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    uint32_t done;
#if MOE_MBAR_SUSPEND_NS > 0
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity), "n"(MOE_MBAR_SUSPEND_NS)
        : "memory");
#else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
#endif
    if (done) return true;
    if ((it & 255u) == 0u) {
      const uint64_t now = globaltimer_ns();
      if (it == 0u) t0 = now;
      else if (now - t0 > 200000000ull) return false;
    }
  }
  return false;
}

__device__ __forceinline__ void set_status(int* status, int bit) {
  if (status) atomicOr(status, bit);
}

// Exclusive scan of one int per thread over the block (<= 1024 threads);
// sh needs 33 ints.
static __device__ int block_excl_scan(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) sh[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    sh[lane] = wi - w;
    if (lane == 31) sh[32] = wi;
  }
  __syncthreads();
  int res = sh[warp] + incl - v;
  total = sh[32];
  __syncthreads();
  return res;
}

// Grouped-expert plan from per-expert row counts, written by one CTA whose
// thread e (< E <= blockDim.x) holds expert e's row count n (0 for e >= E).
// Every thread calls.  Writes: active experts in ascending order and their
// count n_active; 4-row group offsets goff[E+1]; the work items of the GEMV
// kernels, one per chunk of rpc rows of an expert, citem[i] = (e << 16) | j
// (chunk j of expert e) for i < items and -1 up to max_groups; done[i] = 0.
// More groups than max_groups sets MOE_STATUS_ROW_OVERFLOW and no items.
static __device__ void write_expert_plan(int n, int e, int E, int rpc, int max_groups, int* sh,
                                         int* n_active, int* active, int* goff, int* citem,
                                         int* done, int* status) {
  const int ng = (n + 3) / 4;
  const int nch = n > 0 ? (n + rpc - 1) / rpc : 0;
  int tot_g, tot_a, tot_c;
  const int g0 = block_excl_scan(ng, sh, tot_g);
  const int a0 = block_excl_scan(n > 0 ? 1 : 0, sh, tot_a);
  const int c0 = block_excl_scan(nch, sh, tot_c);
  const bool overflow = tot_g > max_groups;
  if (e < E) {
    goff[e] = g0;
    if (n > 0) active[a0] = e;
    if (!overflow)
      for (int j = 0; j < nch; ++j) citem[c0 + j] = (e << 16) | j;
  }
  if (threadIdx.x == 0) {
    goff[E] = tot_g;
    *n_active = overflow ? 0 : tot_a;
    if (overflow) set_status(status, MOE_STATUS_ROW_OVERFLOW);
  }
  const int items = overflow ? 0 : tot_c;
  for (int i = threadIdx.x; i < max_groups; i += blockDim.x) {
    if (i >= items) citem[i] = -1;
    else done[i] = 0;
  }
}


// Work item `item` (a chunk of rpc rows of one expert) -> expert e and the
// chunk's first row c0 inside the expert; false past the last item.
__device__ __forceinline__ bool chunk_of(int item, const int* __restrict__ citem, int rpc,
                                         int& e, int& c0) {
  const int v = citem[item];
  if (v < 0) return false;
  e = v >> 16;
  c0 = (v & 0xFFFF) * rpc;
  return true;
}

// Programmatic dependent launch: wait for the previous kernel's completion
// (no-op when launched normally) / allow the next kernel to start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}


}  // namespace moe
