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
               const float* residual, int k, int d, float* out) {
  // out may alias residual (the stacked step keeps its residual stream in
  // place): each element is read, then written, by the same thread, so those
  // two pointers are neither restrict nor read through the read-only path
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
      float4 v = reinterpret_cast<const float4*>(residual + (size_t)t * d)[i];
      acc.x = v.x + acc.x; acc.y = v.y + acc.y; acc.z = v.z + acc.z; acc.w = v.w + acc.w;
    }
    reinterpret_cast<float4*>(out + (size_t)t * d)[i] = acc;
  }
}

// moe_forward.py:34-40: ms = mean(x*x) + eps; x / sqrt(ms) * weight, or
// * (1 + weight) with gemma_style; or gemma4's router input, x / sqrt(ms) * c
// * scale.  The sum of squares follows numpy's pairwise order, the rest is
// elementwise, each operation rounded as numpy rounds it.
enum { kNormWeight = 0, kNormGemma = 1, kNormRouterIn = 2 };

__device__ __forceinline__ float norm_out(float xn, const float* __restrict__ w, int i, int mode,
                                          float c) {
  if (mode == kNormWeight) return __fmul_rn(xn, __ldg(w + i));
  if (mode == kNormGemma) return __fmul_rn(xn, __fadd_rn(1.0f, __ldg(w + i)));
  const float v = __fmul_rn(xn, c);
  return w ? __fmul_rn(v, __ldg(w + i)) : v;
}

__global__ void __launch_bounds__(256)
rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ weight, float eps, int d,
                int mode, float c, float* __restrict__ out) {
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
    out[(size_t)t * d + i] = norm_out(__fdiv_rn(xr[i], den), weight, i, mode, c);
}

// One CTA per row, for widths whose numpy pairwise tree is perfect: 2^levels
// equal leaves of leaf_len terms (levels <= 5, leaf_len a multiple of 4).
// Lane l of warp 0 sums the squares of leaf l in numpy's leaf order (eight
// running sums, then ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))); a shuffle tree
// then adds (left + right) level by level -- the tree's own order -- so the
// sum is bit-identical to numpy's.  All threads write the scaled row.
__global__ void __launch_bounds__(256)
rms_norm_leaf_kernel(const float* __restrict__ x, const float* __restrict__ weight, float eps,
                     int d, int leaf_len, int levels, int mode, float c,
                     float* __restrict__ out) {
  __shared__ float s_den;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = x + (size_t)t * d;
  if (warp == 0) {
    const int L = 1 << levels;
    float v = 0.f;
    if (lane < L) {
      const float4* e4 = reinterpret_cast<const float4*>(xr + lane * leaf_len);
      if (leaf_len < 8) {
        for (int i = 0; i < leaf_len; ++i) v = v + __fmul_rn(xr[lane * leaf_len + i], xr[lane * leaf_len + i]);
      } else {
        float r[8];
        {
          const float4 a = __ldg(e4), b = __ldg(e4 + 1);
          r[0] = __fmul_rn(a.x, a.x); r[1] = __fmul_rn(a.y, a.y);
          r[2] = __fmul_rn(a.z, a.z); r[3] = __fmul_rn(a.w, a.w);
          r[4] = __fmul_rn(b.x, b.x); r[5] = __fmul_rn(b.y, b.y);
          r[6] = __fmul_rn(b.z, b.z); r[7] = __fmul_rn(b.w, b.w);
        }
        const int full = leaf_len - leaf_len % 8;
        for (int i = 8; i < full; i += 8) {
          const float4 a = __ldg(e4 + i / 4), b = __ldg(e4 + i / 4 + 1);
          r[0] = r[0] + __fmul_rn(a.x, a.x); r[1] = r[1] + __fmul_rn(a.y, a.y);
          r[2] = r[2] + __fmul_rn(a.z, a.z); r[3] = r[3] + __fmul_rn(a.w, a.w);
          r[4] = r[4] + __fmul_rn(b.x, b.x); r[5] = r[5] + __fmul_rn(b.y, b.y);
          r[6] = r[6] + __fmul_rn(b.z, b.z); r[7] = r[7] + __fmul_rn(b.w, b.w);
        }
        v = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (int i = full; i < leaf_len; ++i) {
          const float e = xr[lane * leaf_len + i];
          v = v + __fmul_rn(e, e);
        }
      }
    }
    for (int off = 1; off < L; off <<= 1) {
      const float o = __shfl_down_sync(0xffffffffu, v, off);
      if ((lane & (2 * off - 1)) == 0) v = v + o;
    }
    if (lane == 0) {
      float ms = v / (float)d;
      ms = ms + eps;
      s_den = sqrtf(ms);
    }
  }
  __syncthreads();
  const float den = s_den;
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  float4* o4 = reinterpret_cast<float4*>(out + (size_t)t * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
    const float4 a = __ldg(x4 + i);
    o4[i] = make_float4(norm_out(__fdiv_rn(a.x, den), weight, 4 * i, mode, c),
                        norm_out(__fdiv_rn(a.y, den), weight, 4 * i + 1, mode, c),
                        norm_out(__fdiv_rn(a.z, den), weight, 4 * i + 2, mode, c),
                        norm_out(__fdiv_rn(a.w, den), weight, 4 * i + 3, mode, c));
  }
}

// leaf length of numpy's pairwise tree over n terms when that tree is perfect
// with at most 32 leaves (levels set), else 0
static int pairwise_perfect_leaf(int n, int& levels) {
  levels = 0;
  int len = n;
  while (len > 128) {
    int n2 = len / 2;
    n2 -= n2 % 8;
    if (2 * n2 != len) return 0;
    len = n2;
    ++levels;
  }
  return levels <= 5 ? len : 0;
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

int launch_norm(const float* x, const float* weight, float eps, int mode, float c, int T, int d,
                float* out, cudaStream_t stream);

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
  return moe_rms_norm_ex(x, weight, eps, 0, T, d, out, stream);
}

int moe_rms_norm_ex(const float* x, const float* weight, float eps, int gemma_style, int T, int d,
                    float* out, moe_stream_t stream) {
  MOE_REQUIRE(weight, MOE_ERR_INVALID, "null weight");
  return moe::launch_norm(x, weight, eps, gemma_style ? moe::kNormGemma : moe::kNormWeight, 0.f,
                          T, d, out, reinterpret_cast<cudaStream_t>(stream));
}

int moe_router_input(const float* x, const float* scale, float eps, int T, int d, float* out,
                     moe_stream_t stream) {
  // nightmare_stream.py:4666: rtmp * np.float32(1.0 / np.sqrt(float(dim)))
  const float c = (float)(1.0 / sqrt((double)d));
  return moe::launch_norm(x, scale, eps, moe::kNormRouterIn, c, T, d, out,
                          reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace moe {

int launch_norm(const float* x, const float* weight, float eps, int mode, float c, int T, int d,
                float* out, cudaStream_t stream) {
  MOE_REQUIRE(T >= 0 && d > 0, MOE_ERR_INVALID, "bad shape");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(x && out, MOE_ERR_INVALID, "null pointer");
  int levels = 0;
  const int leaf = moe::pairwise_perfect_leaf(d, levels);
  if (leaf > 0 && leaf % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0) {
    ::moe::ProfScope _prof(MOE_K_RMS_NORM, stream);
    moe::rms_norm_leaf_kernel<<<T, 256, 0, stream>>>(
        x, weight, eps, d, leaf, levels, mode, c, out);
    return moe::check_launch("rms_norm");
  }
  // squares + one float per pairwise leaf (every leaf holds more than 32 terms)
  size_t smem = ((size_t)d + d / 32 + 2) * sizeof(float);
  MOE_REQUIRE(smem <= 200 * 1024, MOE_ERR_UNSUPPORTED, "d=%d too large", d);
  if (smem > 48 * 1024)
    MOE_CUDA(cudaFuncSetAttribute(moe::rms_norm_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  {
    ::moe::ProfScope _prof(MOE_K_RMS_NORM, stream);
    moe::rms_norm_kernel<<<T, 256, smem, stream>>>(x, weight, eps,
                                                                                   d, mode, c,
                                                                                   out);
  }
  return moe::check_launch("rms_norm");
}

}  // namespace moe

