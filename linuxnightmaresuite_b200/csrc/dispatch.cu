// Dispatch: stable counting sort of (token, slot) pairs by expert id.
//
// Replaces the per-token expert loops of moe_forward.py:166-168 and
// nightmare_stream.py:3240-3253 with one permutation of all T*k pairs.  Rows of
// expert e are contiguous and, inside an expert, pairs keep ascending
// (token, slot) order, so the result is a pure function of the ids.
//
// One CTA of 32 warps; warp w owns a contiguous range of pairs.  No atomics:
// within a 32-pair round, __match_any_sync groups lanes by expert and the
// lowest lane of each group updates the warp's private counter for that
// expert; counters are then prefix-summed over warps (in warp order) and over
// experts, and a second pass ranks each pair inside its round.
#include <algorithm>

#include "moe_common.cuh"

namespace moe {

constexpr int kDispThreads = 1024;
constexpr int kDispWarps = kDispThreads / 32;

__global__ void __launch_bounds__(kDispThreads)
dispatch_kernel(const int32_t* __restrict__ ids, int P, int E, int32_t* __restrict__ offsets,
                int32_t* __restrict__ perm_rows, int32_t* __restrict__ inv_perm,
                int* __restrict__ status, int* __restrict__ n_active, int* __restrict__ active,
                int* __restrict__ goff, int* __restrict__ coff, int* __restrict__ done,
                int max_groups, int rpc) {
  pdl_wait();   // the router's ids
  pdl_trigger();
  extern __shared__ int sm[];
  int* wcnt = sm;                          // [kDispWarps][E]
  int* etot = sm + kDispWarps * E;         // [E]
  __shared__ int sh[33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int chunk = ((P + kDispWarps - 1) / kDispWarps + 31) / 32 * 32;
  const int p0 = warp * chunk;
  const int p1 = min(P, p0 + chunk);

  for (int i = threadIdx.x; i < kDispWarps * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();

  // pass 1: per-warp counts
  for (int base = p0; base < p1; base += 32) {
    int p = base + lane;
    int e = -1;
    if (p < p1) {
      e = ids[p];
      if (e < 0 || e >= E) {
        set_status(status, MOE_STATUS_BAD_EXPERT_ID);
        inv_perm[p] = -1;
        e = -1;
      }
    }
    unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (peers & lt_mask) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // per-expert exclusive prefix over warps, then totals
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kDispWarps; ++w) {
      int c = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += c;
    }
    etot[e] = run;
  }
  __syncthreads();
  if (n_active) {
    // plan of the grouped expert kernels (E <= blockDim.x)
    const int e = threadIdx.x;
    write_expert_plan(e < E ? etot[e] : 0, e, E, rpc, max_groups, sh, n_active, active, goff, coff,
                      done, status);
    __syncthreads();
  }
  // exclusive scan of etot over experts (single warp; E is small)
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      int e = e0 + lane;
      int v = e < E ? etot[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (e < E) {
        etot[e] = carry + incl - v;
        offsets[e] = carry + incl - v;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) offsets[E] = carry;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kDispWarps * E; i += blockDim.x) wcnt[i] += etot[i % E];
  __syncthreads();

  // pass 2: stable ranks and scatter
  for (int base = p0; base < p1; base += 32) {
    int p = base + lane;
    int e = -1;
    if (p < p1) {
      e = ids[p];
      if (e < 0 || e >= E) e = -1;
    }
    unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      int pos = wcnt[warp * E + e] + __popc(peers & lt_mask);
      perm_rows[pos] = p;
      inv_perm[p] = pos;
    }
    __syncwarp();
    if (e >= 0 && (peers & lt_mask) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Chunked dispatch for many pairs (prefill): the same stable order from three
// launches, still without atomics.  Chunk c holds pairs [c * chunk,
// (c + 1) * chunk); warp w of its CTA owns the w-th of kChunkWarps equal parts.
//   count:   per-chunk expert counts: warp-private counters updated by the
//            leader lane of each __match_any_sync group, summed over the warps
//   scan:    expert offsets, each chunk's first slot per expert, the plan
//   scatter: per chunk, warp counts + in-warp ranks as in dispatch_kernel,
//            placed after the chunk's first slot
// ---------------------------------------------------------------------------
constexpr int kChunkThreads = 256;
constexpr int kChunkWarps = kChunkThreads / 32;
constexpr int kChunkedMinPairs = 4096;   // below: the one-CTA kernel

__global__ void __launch_bounds__(kChunkThreads)
dispatch_count_kernel(const int32_t* __restrict__ ids, int P, int E, int chunk,
                      int32_t* __restrict__ cta_counts, int32_t* __restrict__ inv_perm,
                      int* __restrict__ status) {
  pdl_wait();   // the router's ids
  pdl_trigger();
  extern __shared__ int wcnt[];   // [warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i = threadIdx.x; i < kChunkWarps * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int wchunk = chunk / kChunkWarps;   // chunk is a multiple of 32 * warps
  const int p0 = min(P, blockIdx.x * chunk + warp * wchunk), p1 = min(P, p0 + wchunk);
  for (int base = p0; base < p1; base += 32) {
    const int p = base + lane;
    int e = -1;
    if (p < p1) {
      e = ids[p];
      if (e < 0 || e >= E) {
        set_status(status, MOE_STATUS_BAD_EXPERT_ID);
        inv_perm[p] = -1;
        e = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (peers & lt_mask) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int n = 0;
    for (int w = 0; w < kChunkWarps; ++w) n += wcnt[w * E + e];
    cta_counts[(size_t)blockIdx.x * E + e] = n;
  }
}

__global__ void __launch_bounds__(kDispThreads)
dispatch_scan_kernel(const int32_t* __restrict__ cta_counts, int C, int E,
                     int32_t* __restrict__ offsets, int32_t* __restrict__ cta_base,
                     int* __restrict__ status, int* __restrict__ n_active,
                     int* __restrict__ active, int* __restrict__ goff, int* __restrict__ coff,
                     int* __restrict__ done, int max_groups, int rpc) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sh[33];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    for (int c = 0; c < C; ++c) {
      const int v = cta_counts[(size_t)c * E + e];
      cta_base[(size_t)c * E + e] = run;
      run += v;
    }
  }
  int total;
  const int off = block_excl_scan(e < E ? run : 0, sh, total);
  if (e < E) {
    offsets[e] = off;
    for (int c = 0; c < C; ++c) cta_base[(size_t)c * E + e] += off;
  }
  if (e == 0) offsets[E] = total;
  if (n_active)
    write_expert_plan(e < E ? run : 0, e, E, rpc, max_groups, sh, n_active, active, goff, coff,
                      done, status);
}

__global__ void __launch_bounds__(kChunkThreads)
dispatch_scatter_kernel(const int32_t* __restrict__ ids, int P, int E, int chunk,
                        const int32_t* __restrict__ cta_base, int32_t* __restrict__ perm_rows,
                        int32_t* __restrict__ inv_perm) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int wcnt[];   // [warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int c = blockIdx.x;
  const int wchunk = chunk / kChunkWarps;   // chunk is a multiple of 32 * warps
  const int p0 = min(P, c * chunk + warp * wchunk), p1 = min(P, p0 + wchunk);
  for (int i = threadIdx.x; i < kChunkWarps * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  for (int base = p0; base < p1; base += 32) {
    const int p = base + lane;
    int e = p < p1 ? ids[p] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (peers & lt_mask) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = cta_base[(size_t)c * E + e];
    for (int w = 0; w < kChunkWarps; ++w) {
      const int v = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += v;
    }
  }
  __syncthreads();
  for (int base = p0; base < p1; base += 32) {
    const int p = base + lane;
    int e = p < p1 ? ids[p] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int pos = wcnt[warp * E + e] + __popc(peers & lt_mask);
      perm_rows[pos] = p;
      inv_perm[p] = pos;
    }
    __syncwarp();
    if (e >= 0 && (peers & lt_mask) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

static int chunk_count(int P) {
  const int want = std::max(1, std::min(2 * sm_count(), (P + kChunkThreads - 1) / kChunkThreads));
  return want;
}

static int chunk_size(int P, int C) {
  const int per = (P + C - 1) / C;
  return (per + kChunkThreads - 1) / kChunkThreads * kChunkThreads;   // 32 per warp multiple
}

// Scratch of the chunked dispatch: cta_counts and cta_base, C x E each.
size_t dispatch_scratch_bytes(int P, int E) {
  if (P < kChunkedMinPairs) return 0;
  return 2 * align_up((size_t)chunk_count(P) * E * sizeof(int32_t), 256);
}

static int launch_dispatch_chunked(const int32_t* ids, int P, int E, int32_t* offsets,
                                   int32_t* perm_rows, int32_t* inv_perm, int* status,
                                   int* n_active, int* active, int* goff, int* coff, int* done,
                                   int max_groups, int rpc, int32_t* scratch, cudaStream_t s) {
  int C = chunk_count(P);
  const int chunk = chunk_size(P, C);
  C = (P + chunk - 1) / chunk;
  int32_t* cta_counts = scratch;
  int32_t* cta_base = scratch + align_up((size_t)chunk_count(P) * E * sizeof(int32_t), 256) / 4;
  const size_t smem_w = sizeof(int) * (size_t)kChunkWarps * E;
  if (smem_w > 48 * 1024)
    MOE_CUDA(cudaFuncSetAttribute(dispatch_scatter_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_w));
  ::moe::ProfScope _prof(MOE_K_DISPATCH, s);
  if (smem_w > 48 * 1024)
    MOE_CUDA(cudaFuncSetAttribute(dispatch_count_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_w));
  MOE_CUDA(launch_pdl(dispatch_count_kernel, dim3(C), dim3(kChunkThreads), smem_w, s, ids, P, E,
                      chunk, cta_counts, inv_perm, status));
  MOE_CUDA(launch_pdl(dispatch_scan_kernel, dim3(1), dim3(kDispThreads), 0, s,
                      (const int32_t*)cta_counts, C, E, offsets, cta_base, status, n_active, active,
                      goff, coff, done, max_groups, rpc));
  MOE_CUDA(launch_pdl(dispatch_scatter_kernel, dim3(C), dim3(kChunkThreads), smem_w, s, ids, P, E,
                      chunk, (const int32_t*)cta_base, perm_rows, inv_perm));
  return MOE_OK;
}

// moe_dispatch that also writes the grouped-expert plan (see plan_kernel).
int launch_dispatch_planned(const int32_t* ids, int T, int k, int E, int32_t* offsets,
                            int32_t* perm_rows, int32_t* inv_perm, int* status, int* n_active,
                            int* active, int* goff, int* coff, int* done, int max_groups,
                            int rpc, int32_t* scratch, cudaStream_t s) {
  MOE_REQUIRE(E > 0 && E <= kDispThreads, MOE_ERR_UNSUPPORTED, "expert count %d above %d", E,
              kDispThreads);
  const int P = T * k;
  MOE_REQUIRE(P > 0, MOE_ERR_INVALID, "no pairs");
  if (P >= kChunkedMinPairs && scratch) {
    MOE_CHECK(launch_dispatch_chunked(ids, P, E, offsets, perm_rows, inv_perm, status, n_active,
                                      active, goff, coff, done, max_groups, rpc, scratch, s));
    return check_launch("dispatch");
  }
  size_t smem = sizeof(int) * ((size_t)kDispWarps * E + E);
  if (smem > 48 * 1024) {
    MOE_CUDA(cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
  }
  {
    ::moe::ProfScope _prof(MOE_K_DISPATCH, s);
    MOE_CUDA(launch_pdl(dispatch_kernel, dim3(1), dim3(kDispThreads), smem, s, ids, P, E, offsets,
                        perm_rows, inv_perm, status, n_active, active, goff, coff, done,
                        max_groups, rpc));
  }
  return check_launch("dispatch");
}

}  // namespace moe

extern "C" {

int moe_dispatch_workspace_bytes(int T, int k, int E, size_t* bytes) {
  MOE_REQUIRE(bytes, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(T >= 0 && k > 0 && E > 0, MOE_ERR_INVALID, "bad shape");
  *bytes = 256 + moe::dispatch_scratch_bytes(T * k, E);  // status word + chunk scratch
  return MOE_OK;
}

int moe_dispatch(const int32_t* ids, int T, int k, int E, int32_t* expert_offsets,
                 int32_t* perm_rows, int32_t* inv_perm, void* workspace,
                 size_t workspace_bytes, moe_stream_t stream) {
  using namespace moe;
  MOE_REQUIRE(T >= 0 && k > 0 && E > 0, MOE_ERR_INVALID, "bad shape T=%d k=%d E=%d", T, k, E);
  MOE_REQUIRE(expert_offsets && workspace, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(workspace_bytes >= 256, MOE_ERR_WORKSPACE, "dispatch workspace too small");
  MOE_REQUIRE(E <= 1024, MOE_ERR_UNSUPPORTED, "expert count %d above 1024", E);
  int64_t P = (int64_t)T * k;
  MOE_REQUIRE(P < (1LL << 30), MOE_ERR_UNSUPPORTED, "too many pairs");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (P == 0) {
    MOE_CUDA(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (E + 1), s));
    return MOE_OK;
  }
  MOE_REQUIRE(ids && perm_rows && inv_perm, MOE_ERR_INVALID, "null pointer");
  const size_t scratch = dispatch_scratch_bytes((int)P, E);
  MOE_REQUIRE(workspace_bytes >= 256 + scratch, MOE_ERR_WORKSPACE,
              "dispatch workspace %zu < %zu", workspace_bytes, 256 + scratch);
  if (scratch) {
    MOE_CHECK(launch_dispatch_chunked(ids, (int)P, E, expert_offsets, perm_rows, inv_perm,
                                      static_cast<int*>(workspace), nullptr, nullptr, nullptr,
                                      nullptr, nullptr, 0, 1,
                                      reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + 256),
                                      s));
    return check_launch("dispatch");
  }
  size_t smem = sizeof(int) * ((size_t)kDispWarps * E + E);
  if (smem > 48 * 1024) {
    MOE_CUDA(cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
  }
  {
    ::moe::ProfScope _prof(MOE_K_DISPATCH, s);
    MOE_CUDA(launch_pdl(dispatch_kernel, dim3(1), dim3(kDispThreads), smem, s, ids, (int)P, E,
                        expert_offsets, perm_rows, inv_perm, static_cast<int*>(workspace),
                        (int*)nullptr, (int*)nullptr, (int*)nullptr, (int*)nullptr,
                        (int*)nullptr, 0, 1));
  }
  return check_launch("dispatch");
}

}  // extern "C"
