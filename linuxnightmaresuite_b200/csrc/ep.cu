// Expert-parallel helpers: row gather for the send buffer and the owner-side
// expert order of received rows.
#include <string.h>

#include "internal.cuh"

namespace moe {

// out[r] = x[rows[r] / div]  (float4 copies; one CTA row-block per row)
__global__ void __launch_bounds__(256)
gather_rows_kernel(const float* __restrict__ x, const int32_t* __restrict__ rows, int div, int n,
                   int d, float* __restrict__ out) {
  const int r = blockIdx.x;
  if (r >= n) return;
  const float4* src = reinterpret_cast<const float4*>(x + (size_t)(rows[r] / div) * d);
  float4* dst = reinterpret_cast<float4*>(out + (size_t)r * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// recv_counts[src][e] -> local_offsets[e] (E_local+1) and row_map: expert-sorted
// local row r reads receive-buffer row row_map[r]; the receive buffer is
// source-major, expert-minor.  One CTA; W * E_local <= 1024.
__global__ void __launch_bounds__(1024)
ep_local_order_kernel(const int32_t* __restrict__ rc, int W, int El, int max_rows,
                      int32_t* __restrict__ loff, int32_t* __restrict__ row_map,
                      int* __restrict__ status) {
  __shared__ int sh[33];
  __shared__ int start[1024];   // receive-buffer start of block (src, e)
  __shared__ int dest[1024];    // local sorted start of block (src, e)
  const int i = threadIdx.x;    // i = src * El + e
  const int n = i < W * El ? rc[i] : 0;
  int tot;
  const int st = block_excl_scan(n, sh, tot);   // source-major scan = receive positions
  if (i < W * El) start[i] = st;
  // expert-major order: j = e * W + src
  const int e = i / W, src = i % W;
  const int nj = (i < W * El) ? rc[src * El + e] : 0;
  int tot2;
  const int dj = block_excl_scan(nj, sh, tot2);
  if (i < W * El) dest[src * El + e] = dj;
  __syncthreads();
  if (i < El) loff[i] = dest[i];   // src 0, expert i
  if (i == 0) loff[El] = tot;
  if (tot > max_rows) {
    if (i == 0) set_status(status, MOE_STATUS_ROW_OVERFLOW);
    return;
  }
  __syncthreads();
  // scatter: each block (src, e) maps its rows
  for (int b = 0; b < W * El; ++b) {
    const int cnt = rc[b];
    for (int q = i; q < cnt; q += blockDim.x) row_map[dest[b] + q] = start[b] + q;
  }
}

}  // namespace moe

extern "C" {

int moe_gather_rows(const float* x, const int32_t* rows, int div, int n, int d, float* out,
                    moe_stream_t stream) {
  MOE_REQUIRE(n >= 0 && d > 0 && div > 0, MOE_ERR_INVALID, "bad shape");
  if (n == 0) return MOE_OK;
  MOE_REQUIRE(x && rows && out, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(d % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0,
              MOE_ERR_UNSUPPORTED, "rows must be 16-byte aligned (d %% 4 == 0)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  {
    ::moe::ProfScope _prof(MOE_K_AUX, s);
    moe::gather_rows_kernel<<<n, 256, 0, s>>>(x, rows, div, n, d, out);
  }
  return moe::check_launch("gather_rows");
}

int moe_ep_local_order(const int32_t* recv_counts, int W, int E_local, int max_rows,
                       int32_t* local_offsets, int32_t* row_map, void* workspace,
                       moe_stream_t stream) {
  MOE_REQUIRE(W > 0 && E_local > 0 && W * E_local <= 1024, MOE_ERR_UNSUPPORTED,
              "W * E_local must be in [1, 1024]");
  MOE_REQUIRE(recv_counts && local_offsets && row_map && workspace, MOE_ERR_INVALID,
              "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  {
    ::moe::ProfScope _prof(MOE_K_AUX, s);
    moe::ep_local_order_kernel<<<1, 1024, 0, s>>>(recv_counts, W, E_local, max_rows,
                                                 local_offsets, row_map,
                                                 static_cast<int*>(workspace));
  }
  return moe::check_launch("ep_local_order");
}

}  // extern "C"

// ===========================================================================
// Expert parallelism over NVLink peer memory.
//
// Every rank owns one exchange window (cudaMalloc, shared with the other ranks
// of the node through CUDA IPC).  Window layout (bytes):
//   0      recv_flag[32]  int  rank s writes the step's epoch after its rows
//   128    counters[2]    int  this rank's last-CTA counters (send, return)
//   256    ret_flag[32]   int  owner o writes the epoch after returning results
//   512    meta[W][El+1]  int  from source s: rows per local expert, then the
//                              sorted position of its first row for this rank
//   recv_x [W][cap][d]    f32  rows from source s at s * cap (cap = T * k); the
//                              expert outputs overwrite them in place
//   ret_y  [cap][d]       f32  this rank's expert outputs, in its sorted order
// One step, with no host synchronisation and no collective library:
//   router -> dispatch -> ep_send (rows and counts straight into the owners'
//   windows, then a release flag per owner) -> ep_recv_plan (acquire all
//   sources' flags, expert order of the received rows, expert plan) ->
//   grouped experts on the window's rows -> ep_return (outputs straight into
//   the sources' windows, then a release flag per source) -> ep_wait (acquire
//   all owners' flags) -> combine.
// Waits on other ranks are bounded (1 s); a timeout sets MOE_STATUS_TIMEOUT.
// A source's next send cannot overtake an owner still reading its rows: the
// source's next step starts after its combine, which waited for every
// owner's return, which each owner issued after its experts had read them.
// ===========================================================================
namespace moe {

constexpr int kEpMaxW = 32;

struct EpWin {
  size_t recv_flag, counters, ret_flag, meta, recv_x, ret_y, bytes;
};

static EpWin ep_win(int W, int El, int T, int k, int d) {
  EpWin w;
  const size_t cap = (size_t)T * k;
  w.recv_flag = 0;
  w.counters = 128;
  w.ret_flag = 256;
  w.meta = 512;
  w.recv_x = 512 + align_up((size_t)W * (El + 1) * sizeof(int), 256);
  w.ret_y = w.recv_x + align_up((size_t)W * cap * d * sizeof(float), 256);
  w.bytes = w.ret_y + align_up(cap * d * sizeof(float), 256);
  return w;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait for a flag written by another GPU: *p >= target (acquire, system
// scope); gives up after ~1 s.
__device__ __forceinline__ bool wait_flag_sys(const int* p, int target) {
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < (1u << 26); ++it) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if ((it & 63u) == 0u) {
      const uint64_t now = globaltimer_ns();
      if (it == 0u) t0 = now;
      else if (now - t0 > 1000000000ull) return false;
    }
    __nanosleep(256);
  }
  return false;
}

// One row of n4 float4s copied by one warp with 8 loads in flight per lane
// (the destination may be another GPU's window: posted stores over NVLink).
__device__ __forceinline__ void copy_row_warp(float4* dst, const float4* src, int n4, int lane) {
  for (int v = lane; v < n4; v += 32 * 8) {
    float4 t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (v + 32 * u < n4) t[u] = src[v + 32 * u];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (v + 32 * u < n4) dst[v + 32 * u] = t[u];
  }
}

struct EpArgs {
  uint8_t* const* peers;   // W window bases (device array; own window included)
  uint8_t* win;            // this rank's window
  EpWin off;
  int W, El, rank, cap, d, epoch;
};

// Completion of a multi-CTA send: the last CTA to finish raises every peer's
// flag (slot `rank` of the flag array at `flag_off`) to the epoch.  Each CTA's
// rows are visible system-wide (its system fence) before it counts itself,
// so the last CTA needs only a GPU-scope fence to order the flags after the
// other CTAs' counts (whose rows are then already visible to the peers).
__device__ __forceinline__ void ep_finish(const EpArgs& a, int* ctr, size_t flag_off) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(ctr, 1);
    if (prev == (int)(gridDim.x * gridDim.y) - 1) {
      *ctr = 0;
      __threadfence();
      for (int o = 0; o < a.W; ++o)
        st_release_sys(reinterpret_cast<int*>(a.peers[o] + flag_off) + a.rank, a.epoch);
    }
  }
}

// Rows in this rank's expert-sorted order -> the owners' windows; counts and
// base positions -> the owners' meta.  One warp per row.
__global__ void __launch_bounds__(256)
ep_send_kernel(const float* __restrict__ x, const int32_t* __restrict__ perm, int k,
               const int32_t* __restrict__ offsets, int P, EpArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + warp;
  if (i < P) {
    int o = 0;   // owner: last rank whose first row is <= i
    for (int q = 1; q < a.W; ++q)
      if (offsets[q * a.El] <= i) o = q;
    const int j = i - offsets[o * a.El];
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)(perm[i] / k) * a.d);
    float4* dst = reinterpret_cast<float4*>(
        reinterpret_cast<float*>(a.peers[o] + a.off.recv_x) + ((size_t)a.rank * a.cap + j) * a.d);
    copy_row_warp(dst, src, a.d / 4, lane);
  }
  if (blockIdx.x == 0) {
    for (int v = threadIdx.x; v < a.W * (a.El + 1); v += blockDim.x) {
      const int o = v / (a.El + 1), q = v - o * (a.El + 1);
      const int val = q < a.El ? offsets[o * a.El + q + 1] - offsets[o * a.El + q]
                               : offsets[o * a.El];
      reinterpret_cast<int*>(a.peers[o] + a.off.meta)[a.rank * (a.El + 1) + q] = val;
    }
  }
  ep_finish(a, reinterpret_cast<int*>(a.win + a.off.counters), a.off.recv_flag);
}

// Waits for every source, then: local_offsets / row_map of the received rows
// in (local expert, source, source order) order, and the grouped experts' plan.
__global__ void __launch_bounds__(1024)
ep_recv_plan_kernel(EpArgs a, int32_t* __restrict__ loff, int32_t* __restrict__ row_map,
                    int* __restrict__ n_active, int* __restrict__ active, int* __restrict__ goff,
                    int* __restrict__ coff, int* __restrict__ done, int max_groups, int rpc,
                    int* __restrict__ status) {
  __shared__ int sh[33];
  __shared__ int rc[1024];             // clamped counts [src][e]
  __shared__ int start[1024];
  __shared__ int dest[1024];
  __shared__ int ok_s;
  const int i = threadIdx.x;
  if (i == 0) ok_s = 1;
  __syncthreads();
  if (i < a.W) {
    if (!wait_flag_sys(reinterpret_cast<const int*>(a.win + a.off.recv_flag) + i, a.epoch))
      ok_s = 0;
  }
  __syncthreads();
  if (!ok_s && i == 0) set_status(status, MOE_STATUS_TIMEOUT);
  const int* meta = reinterpret_cast<const int*>(a.win + a.off.meta);
  const int WE = a.W * a.El;
  // counts, clamped so that no source overruns its cap rows
  int n = 0;
  if (i < WE) {
    const int src = i / a.El;
    n = ok_s ? meta[src * (a.El + 1) + (i - src * a.El)] : 0;
    n = n < 0 ? 0 : (n > a.cap ? a.cap : n);
  }
  // source-major prefix; minus the source's first entry = prefix within the
  // source, so the receive position is s * cap + that
  int tot;
  const int st = block_excl_scan(n, sh, tot);
  if (i < WE) {
    start[i] = st;
    rc[i] = n;
  }
  __syncthreads();
  int within = 0;
  if (i < WE) {
    const int src = i / a.El;
    within = st - start[src * a.El];
    if (within + n > a.cap) within = a.cap - n;   // overrun guard (corrupt counts)
  }
  __syncthreads();
  if (i < WE) start[i] = (i / a.El) * a.cap + within;
  __syncthreads();
  // expert-major order j = e * W + src
  const int e = i / a.W, src = i - (i / a.W) * a.W;
  const int nj = i < WE ? rc[src * a.El + e] : 0;
  int tot2;
  const int dj = block_excl_scan(nj, sh, tot2);
  if (i < WE) dest[src * a.El + e] = dj;
  __syncthreads();
  const bool over = tot2 > a.W * a.cap;   // only with corrupt counts
  if (over && i == 0) set_status(status, MOE_STATUS_ROW_OVERFLOW);
  if (i < a.El) loff[i] = over ? 0 : dest[i];
  if (i == 0) loff[a.El] = over ? 0 : tot2;
  if (!over) {
    for (int b = 0; b < WE; ++b) {
      const int cnt = rc[b];
      for (int q = i; q < cnt; q += blockDim.x) row_map[dest[b] + q] = start[b] + q;
    }
  }
  // plan of the grouped experts (as the dispatch kernel writes it)
  int ne = 0;
  if (i < a.El && !over) {
    for (int s2 = 0; s2 < a.W; ++s2) ne += rc[s2 * a.El + i];
  }
  write_expert_plan(ne, i, a.El, rpc, max_groups, sh, n_active, active, goff, coff, done, status);
}

// Expert outputs of the rows received from source s (in place in recv_x) ->
// source s's ret_y at its sorted positions.  Grid (row chunks of 8, W).
__global__ void __launch_bounds__(256)
ep_return_kernel(EpArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.y;
  const int i = blockIdx.x * 8 + warp;
  const int* meta = reinterpret_cast<const int*>(a.win + a.off.meta) + s * (a.El + 1);
  int rows = 0;
  for (int e = 0; e < a.El; ++e) {
    const int c = meta[e];
    rows += c < 0 ? 0 : c;
  }
  rows = rows > a.cap ? a.cap : rows;
  int base = meta[a.El];
  base = base < 0 ? 0 : (base > a.cap - rows ? a.cap - rows : base);
  if (i < rows) {
    const float4* src = reinterpret_cast<const float4*>(
        reinterpret_cast<const float*>(a.win + a.off.recv_x) + ((size_t)s * a.cap + i) * a.d);
    float4* dst = reinterpret_cast<float4*>(
        reinterpret_cast<float*>(a.peers[s] + a.off.ret_y) + (size_t)(base + i) * a.d);
    copy_row_warp(dst, src, a.d / 4, lane);
  }
  ep_finish(a, reinterpret_cast<int*>(a.win + a.off.counters) + 1, a.off.ret_flag);
}

// Waits until every owner has returned this step's outputs.
__global__ void ep_wait_kernel(EpArgs a, int* __restrict__ status) {
  if ((int)threadIdx.x < a.W &&
      !wait_flag_sys(reinterpret_cast<const int*>(a.win + a.off.ret_flag) + threadIdx.x, a.epoch))
    set_status(status, MOE_STATUS_TIMEOUT);
}

__global__ void ep_fill_two(int32_t* off, int n) {
  if (threadIdx.x == 0) {
    off[0] = 0;
    off[1] = n;
  }
}

struct EpWs {
  int* status;
  uint8_t* router_ws;
  size_t router_bytes;
  int32_t* ids;
  float* wts;
  int32_t* offsets;
  int32_t* perm;
  int32_t* inv;
  int32_t* disp_scratch;
  int32_t* loff;
  int32_t* row_map;
  uint8_t* exp_ws;
  size_t exp_bytes;
  float* xdev;         // device copy of x when the caller's x is in host memory
  int32_t* s_off;      // shared expert: [0, T]
  float* s_y;          // shared expert output (T, d)
  uint8_t* s_ws;       // shared expert workspace (its own plan and buffers)
  size_t s_bytes;
  size_t bytes;
};

static EpWs carve_ep(void* ws, const moe_layer_weights* w, int W, int T) {
  Carve c{static_cast<uint8_t*>(ws), 0, 0};
  EpWs L;
  const int El = w->E / W;
  const size_t P = (size_t)T * w->k;
  const int R = (int)(P * W);
  L.status = c.take<int>(64);
  moe_router_workspace_bytes(T, w->d, w->E, &L.router_bytes);
  L.router_ws = c.take<uint8_t>(L.router_bytes);
  L.ids = c.take<int32_t>(P);
  L.wts = c.take<float>(P);
  L.offsets = c.take<int32_t>(w->E + 1);
  L.perm = c.take<int32_t>(P);
  L.inv = c.take<int32_t>(P);
  L.disp_scratch = c.take<int32_t>(dispatch_scratch_bytes((int)P, w->E) / 4 + 1);
  L.loff = c.take<int32_t>(El + 1);
  L.row_map = c.take<int32_t>(R);
  experts_workspace_hint(R, (int)P, El, w->d, w->F, &L.exp_bytes);
  L.exp_ws = c.take<uint8_t>(L.exp_bytes);
  L.xdev = c.take<float>((size_t)T * w->d);
  L.s_off = c.take<int32_t>(2);
  L.s_y = w->s_gate ? c.take<float>((size_t)T * w->d) : nullptr;
  L.s_bytes = 0;
  if (w->s_gate) experts_workspace_hint(T, T, 1, w->d, w->Fs, &L.s_bytes);
  L.s_ws = c.take<uint8_t>(L.s_bytes > 0 ? L.s_bytes : 256);
  L.bytes = align_up(c.used, 256);
  return L;
}

}  // namespace moe

extern "C" {

int moe_ipc_alloc(size_t bytes, void** ptr) {
  MOE_REQUIRE(ptr && bytes > 0, MOE_ERR_INVALID, "bad allocation request");
  void* p = nullptr;
  MOE_CUDA(cudaMalloc(&p, bytes));
  MOE_CUDA(cudaMemset(p, 0, bytes));
  MOE_CUDA(cudaDeviceSynchronize());
  *ptr = p;
  return MOE_OK;
}

int moe_ipc_free(void* ptr) {
  if (ptr) MOE_CUDA(cudaFree(ptr));
  return MOE_OK;
}

int moe_ipc_handle(void* ptr, void* handle) {
  MOE_REQUIRE(ptr && handle, MOE_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  MOE_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, sizeof(h));
  return MOE_OK;
}

int moe_ipc_open(const void* handle, void** ptr) {
  MOE_REQUIRE(ptr && handle, MOE_ERR_INVALID, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  MOE_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return MOE_OK;
}

int moe_ipc_close(void* ptr) {
  if (ptr) MOE_CUDA(cudaIpcCloseMemHandle(ptr));
  return MOE_OK;
}

int moe_ep_window_bytes(int W, int E, int T, int k, int d, size_t* bytes) {
  MOE_REQUIRE(bytes, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(W > 0 && W <= moe::kEpMaxW && E % W == 0 && T > 0 && k > 0 && d > 0,
              MOE_ERR_INVALID, "bad expert-parallel shape");
  *bytes = moe::ep_win(W, E / W, T, k, d).bytes;
  return MOE_OK;
}

int moe_ep_workspace_bytes(const moe_layer_weights* w, int W, int T, size_t* bytes) {
  MOE_REQUIRE(w && bytes, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(W > 0 && w->E % W == 0 && T > 0, MOE_ERR_INVALID, "bad expert-parallel shape");
  *bytes = moe::carve_ep(nullptr, w, W, T).bytes;
  return MOE_OK;
}

int moe_ep_forward_phases(const moe_layer_weights* w, int W, int rank, void* const* peers,
                          void* window, const float* x, int T, float* out, const float* residual,
                          int epoch, int phases, void* workspace, size_t workspace_bytes,
                          moe_stream_t stream) {
  using namespace moe;
  MOE_REQUIRE(w && peers && window && x && out && workspace, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(W > 0 && W <= kEpMaxW && rank >= 0 && rank < W && w->E % W == 0,
              MOE_ERR_INVALID, "bad expert-parallel shape (W=%d rank=%d E=%d)", W, rank, w->E);
  MOE_REQUIRE(T > 0 && epoch > 0, MOE_ERR_INVALID, "T and epoch must be positive");
  MOE_REQUIRE(phases > 0 && (phases & ~MOE_EP_PHASE_ALL) == 0, MOE_ERR_INVALID,
              "phases must be a non-empty mask of MOE_EP_PHASE_* bits");
  MOE_REQUIRE(!w->s_gate || (w->s_up && w->s_down && w->Fs > 0), MOE_ERR_INVALID,
              "incomplete shared expert");
  const int El = w->E / W;
  MOE_REQUIRE(W * El <= 1024, MOE_ERR_UNSUPPORTED, "W * E_local must be <= 1024");
  MOE_REQUIRE(w->d % 4 == 0, MOE_ERR_UNSUPPORTED, "d must be a multiple of 4");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  EpWs L = carve_ep(workspace, w, W, T);
  MOE_REQUIRE(workspace_bytes >= L.bytes, MOE_ERR_WORKSPACE, "ep workspace %zu < %zu",
              workspace_bytes, L.bytes);
  const int P = T * w->k;
  EpArgs a;
  a.peers = reinterpret_cast<uint8_t* const*>(peers);
  a.win = static_cast<uint8_t*>(window);
  a.off = ep_win(W, El, T, w->k, w->d);
  a.W = W;
  a.El = El;
  a.rank = rank;
  a.cap = P;
  a.d = w->d;
  a.epoch = epoch;
  // x may be pinned host memory: the router's first pass reads it over the
  // bus and leaves the device copy the send (and the shared expert) read
  const int xk = memory_kind(x);
  MOE_REQUIRE(xk != kMemPageable && memory_kind(out) != kMemPageable, MOE_ERR_INVALID,
              "x and out must be device or pinned host memory");
  const float* xe = xk == kMemPinnedHost ? L.xdev : x;
  if (phases & MOE_EP_PHASE_SEND) {
    MOE_CHECK(launch_router(x, w->gate_w, w->bias, T, w->d, w->E, w->k, w->router_layout,
                            w->mode, L.ids, L.wts, L.router_ws, L.router_bytes, s, nullptr,
                            nullptr, xk == kMemPinnedHost ? L.xdev : nullptr));
    MOE_CHECK(launch_dispatch_planned(L.ids, T, w->k, w->E, L.offsets, L.perm, L.inv, L.status,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, 0, 1,
                                      L.disp_scratch, s));
    {
      ::moe::ProfScope _prof(MOE_K_EP_SEND, s);
      ep_send_kernel<<<(P + 7) / 8, 256, 0, s>>>(xe, L.perm, w->k, L.offsets, P, a);
    }
    MOE_CHECK(check_launch("ep_send"));
  }
  if (phases & MOE_EP_PHASE_SERVE) {
    const int R = P * W;
    int *n_active, *active, *goff, *coff, *done, mg;
    experts_plan_arrays(L.exp_ws, R, El, w->d, w->F, &n_active, &active, &goff, &coff, &done,
                        &mg);
    const int rpc = experts_rows_per_chunk(w->qtype, experts_down_qtype(w->qtype, w->opts), R,
                                           El, w->d, w->F, P);
    {
      // a programmatic dependent of the send: it reads nothing of it before
      // the per-source flags (its own included) say the rows and counts are in
      ::moe::ProfScope _prof(MOE_K_EP_RECV, s);
      MOE_CUDA(launch_pdl(ep_recv_plan_kernel, dim3(1), dim3(1024), 0, s, a, L.loff, L.row_map,
                          n_active, active, goff, coff, done, mg, rpc, L.status));
    }
    MOE_CHECK(check_launch("ep_recv_plan"));
    float* recv = reinterpret_cast<float*>(a.win + a.off.recv_x);
    MOE_CHECK(run_experts(w->w_gate, w->w_up, w->w_down, w->qtype, L.loff, El, R, recv,
                          L.row_map, 1, w->d, w->F, recv, L.row_map, L.exp_ws, L.exp_bytes, s,
                          L.status, nullptr, true, P, w->opts));
    {
      ::moe::ProfScope _prof(MOE_K_EP_RETURN, s);
      ep_return_kernel<<<dim3((P + 7) / 8, W), 256, 0, s>>>(a);
    }
    MOE_CHECK(check_launch("ep_return"));
    if (w->s_gate) {
      // the shared expert runs on this rank's own tokens (replicated weights)
      // while the other ranks finish their experts and returns
      {
        ::moe::ProfScope _prof(MOE_K_AUX, s);
        ep_fill_two<<<1, 32, 0, s>>>(L.s_off, T);
      }
      MOE_CHECK(check_launch("ep_fill_two"));
      const moe_expert_opts so = shared_expert_opts(w->opts);
      MOE_CHECK(run_experts(w->s_gate, w->s_up, w->s_down, w->shared_qtype, L.s_off, 1, T, xe,
                            nullptr, 1, w->d, w->Fs, L.s_y, nullptr, L.s_ws, L.s_bytes, s,
                            L.status, nullptr, false, T, &so));
    }
  }
  if (phases & MOE_EP_PHASE_COMBINE) {
    {
      // likewise after the return: only the owners' flags are read
      ::moe::ProfScope _prof(MOE_K_EP_WAIT, s);
      MOE_CUDA(launch_pdl(ep_wait_kernel, dim3(1), dim3(32), 0, s, a, L.status));
    }
    MOE_CHECK(check_launch("ep_wait"));
    MOE_CHECK(launch_combine(reinterpret_cast<const float*>(a.win + a.off.ret_y), L.inv, L.wts,
                             L.s_y, residual, T, w->k, w->d, out, s));
  }
  return MOE_OK;
}

int moe_ep_forward(const moe_layer_weights* w, int W, int rank, void* const* peers, void* window,
                   const float* x, int T, float* out, const float* residual, int epoch,
                   void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  return moe_ep_forward_phases(w, W, rank, peers, window, x, T, out, residual, epoch,
                               MOE_EP_PHASE_ALL, workspace, workspace_bytes, stream);
}

}  // extern "C"
