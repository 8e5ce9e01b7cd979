// Combine (weighted un-permute + shared expert + residual) and RMSNorm.
#include <math.h>

#include "moe_common.cuh"

namespace moe {

// CTA (token t, column slice blockIdx.y of kCombineThreads float4s).
// moe_forward.py:165-172: output = 0; output += w * y_e in router order;
// output += shared; then the caller's residual add (moe_forward.py:359,
// x = x + ffn_out).  Multiply and add are rounded separately, as numpy
// evaluates them.
constexpr int kCombineThreads = 128;

__global__ void __launch_bounds__(kCombineThreads)
combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ inv_perm,
               const float* __restrict__ w, const float* __restrict__ shared,
               const float* __restrict__ residual, int k, int d, float* __restrict__ out) {
  pdl_wait();   // the expert outputs
  const int t = blockIdx.x;
  __shared__ int rows[32];
  __shared__ float wts[32];
  if (threadIdx.x < k) {
    rows[threadIdx.x] = inv_perm[(size_t)t * k + threadIdx.x];
    wts[threadIdx.x] = w[(size_t)t * k + threadIdx.x];
  }
  __syncthreads();
  for (int i = blockIdx.y * kCombineThreads + threadIdx.x; i < d / 4;
       i += gridDim.y * kCombineThreads) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q0 = 0; q0 < k; q0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {   // loads first, so they overlap
        const int r = (q0 + u < k) ? rows[q0 + u] : -1;
        v[u] = r >= 0 ? __ldg(reinterpret_cast<const float4*>(y + (size_t)r * d) + i)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (q0 + u >= k || rows[q0 + u] < 0) continue;
        const float wq = wts[q0 + u];
        acc.x = __fadd_rn(acc.x, __fmul_rn(wq, v[u].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(wq, v[u].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(wq, v[u].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(wq, v[u].w));
      }
    }
    if (shared) {
      float4 v = __ldg(reinterpret_cast<const float4*>(shared + (size_t)t * d) + i);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (residual) {
      float4 v = __ldg(reinterpret_cast<const float4*>(residual + (size_t)t * d) + i);
      acc.x = v.x + acc.x; acc.y = v.y + acc.y; acc.z = v.z + acc.z; acc.w = v.w + acc.w;
    }
    reinterpret_cast<float4*>(out + (size_t)t * d)[i] = acc;
  }
}

// moe_forward.py:34-40: ms = mean(x*x) + eps; x / sqrt(ms) * weight.
// The sum of squares follows numpy's pairwise order (one thread), the rest is
// elementwise.
__global__ void __launch_bounds__(256)
rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ weight, float eps, int d,
                float* __restrict__ out) {
  extern __shared__ float sq[];       // [d] squares, then the pairwise leaves
  __shared__ float s_den;
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float v = xr[i];
    sq[i] = __fmul_rn(v, v);
  }
  __syncthreads();
  const float sum = np_pairwise_sum_cta(sq, d, sq + d);
  if (threadIdx.x == 0) {
    float ms = sum / (float)d;
    ms = ms + eps;
    s_den = sqrtf(ms);
  }
  __syncthreads();
  const float den = s_den;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    out[(size_t)t * d + i] = __fmul_rn(__fdiv_rn(xr[i], den), weight[i]);
}

int launch_combine(const float* y, const int32_t* inv_perm, const float* w, const float* shared,
                   const float* residual, int T, int k, int d, float* out, cudaStream_t s) {
  if (T == 0) return MOE_OK;
  {
    ::moe::ProfScope _prof(MOE_K_COMBINE, s);
    const int slices = (d / 4 + kCombineThreads - 1) / kCombineThreads;
    MOE_CUDA(launch_pdl(combine_kernel, dim3(T, slices), dim3(kCombineThreads), 0, s, y, inv_perm,
                        w, shared, residual, k, d, out));
  }
  return check_launch("combine");
}

}  // namespace moe

extern "C" {

int moe_combine(const float* y, const int32_t* inv_perm, const float* weights,
                const float* shared, const float* residual, int T, int k, int d, float* out,
                moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && k > 0 && k <= 32 && d > 0, MOE_ERR_INVALID, "bad shape");
  MOE_REQUIRE(d % 4 == 0, MOE_ERR_UNSUPPORTED, "d must be a multiple of 4");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(y && inv_perm && weights && out, MOE_ERR_INVALID, "null pointer");
  return moe::launch_combine(y, inv_perm, weights, shared, residual, T, k, d, out,
                             reinterpret_cast<cudaStream_t>(stream));
}

int moe_rms_norm(const float* x, const float* weight, float eps, int T, int d, float* out,
                 moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && d > 0, MOE_ERR_INVALID, "bad shape");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(x && weight && out, MOE_ERR_INVALID, "null pointer");
  // squares + one float per pairwise leaf (every leaf holds more than 32 terms)
  size_t smem = ((size_t)d + d / 32 + 2) * sizeof(float);
  MOE_REQUIRE(smem <= 200 * 1024, MOE_ERR_UNSUPPORTED, "d=%d too large", d);
  if (smem > 48 * 1024)
    MOE_CUDA(cudaFuncSetAttribute(moe::rms_norm_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  {
    ::moe::ProfScope _prof(MOE_K_RMS_NORM, reinterpret_cast<cudaStream_t>(stream));
    moe::rms_norm_kernel<<<T, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(x, weight, eps,
                                                                                   d, out);
  }
  return moe::check_launch("rms_norm");
}

}  // extern "C"
