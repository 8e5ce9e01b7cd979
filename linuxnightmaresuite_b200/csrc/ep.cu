// Expert-parallel helpers: row gather for the send buffer and the owner-side
// expert order of received rows.
#include "moe_common.cuh"

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
