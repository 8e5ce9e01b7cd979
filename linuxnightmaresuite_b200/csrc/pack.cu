// GGUF block decode and the load-time repack into MMA tiles.
#include "blockfmt.cuh"

namespace moe {

// dequant_fast.py:44-66 (Q8_0) and :69-100 (Q4_0): one thread per 32-weight block.
template <int QT>
__global__ void dequantize_kernel(const uint8_t* __restrict__ raw, float* __restrict__ out,
                                  int64_t n_blocks) {
  constexpr int BB = QTraits<QT>::kBlockBytes;
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const uint8_t* blk = raw + b * BB;
  __half_raw hr;
  hr.x = (uint16_t)(blk[0] | (blk[1] << 8));
  float d = __half2float(__half(hr));
  float* o = out + b * 32;
  if (QT == MOE_Q8_0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = d * (float)(int8_t)blk[2 + i];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint8_t q = blk[2 + i];
      o[i] = d * (float)((int)(q & 0x0F) - 8);
      o[16 + i] = d * (float)((int)(q >> 4) - 8);
    }
  }
}

// One thread per (tile, lane): moves the lane's quant slice and, for t == 0,
// the group's four scales.  dir = 0 packs raw -> tiles, dir = 1 unpacks.
template <int QT>
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              int64_t n_tiles, int rows, int cols, int dir) {
  using Tr = QTraits<QT>;
  constexpr int BB = Tr::kBlockBytes;
  constexpr int SL = Tr::kLaneBytes / 4;  // quant bytes per (row, block) slice
  int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= n_tiles * 32) return;
  int64_t tile = gid >> 5;
  int lane = (int)(gid & 31);
  int g = lane >> 2, t = lane & 3;
  const int kt = cols / 64, strips = rows / 16, nb = cols / 32;
  int64_t j = tile % kt;
  int64_t s = (tile / kt) % strips;
  int64_t m = tile / ((int64_t)kt * strips);
  int64_t tile_base = tile * Tr::kTileBytes;
#pragma unroll
  for (int half = 0; half < 2; ++half) {     // row g, row g + 8
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      int64_t row = (int64_t)s * 16 + g + 8 * half;
      int64_t raw_blk = ((m * rows + row) * nb + 2 * j + b) * BB;
      int64_t pk = tile_base + lane * Tr::kLaneBytes + (half * 2 + b) * SL;
#pragma unroll
      for (int i = 0; i < SL; ++i) {
        int64_t ro = raw_blk + 2 + SL * t + i;
        if (dir == 0) dst[pk + i] = src[ro];
        else dst[ro] = src[pk + i];
      }
      if (t == 0) {
        int64_t so = tile_base + Tr::kTileQuant + 8 * g + 2 * (half * 2 + b);
        if (dir == 0) {
          dst[so] = src[raw_blk];
          dst[so + 1] = src[raw_blk + 1];
        } else {
          dst[raw_blk] = src[so];
          dst[raw_blk + 1] = src[so + 1];
        }
      }
    }
  }
}

static int repack(const uint8_t* src, uint8_t* dst, int qtype, int n_mats, int rows, int cols,
                  cudaStream_t s, int dir) {
  MOE_REQUIRE(src && dst, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(qtype_ok(qtype), MOE_ERR_UNSUPPORTED, "quant type %d not supported", qtype);
  MOE_REQUIRE(n_mats > 0 && rows > 0 && cols > 0, MOE_ERR_INVALID, "non-positive shape");
  MOE_REQUIRE(rows % 16 == 0 && cols % 64 == 0, MOE_ERR_UNSUPPORTED,
              "packed tiles need rows %% 16 == 0 and cols %% 64 == 0 (got %d x %d)", rows, cols);
  int64_t n_tiles = (int64_t)n_mats * (rows / 16) * (cols / 64);
  int64_t threads = n_tiles * 32;
  int blk = 256;
  int64_t grid = (threads + blk - 1) / blk;
  {
    ::moe::ProfScope _prof(MOE_K_PACK, s);
    if (qtype == MOE_Q4_0)
      repack_kernel<MOE_Q4_0><<<(unsigned)grid, blk, 0, s>>>(src, dst, n_tiles, rows, cols, dir);
    else
      repack_kernel<MOE_Q8_0><<<(unsigned)grid, blk, 0, s>>>(src, dst, n_tiles, rows, cols, dir);
  }
  return check_launch("repack");
}

// Q5_1 / Q4_K / Q6_K (dequant_fast.py:169-201, :237-289, :343-378): one thread
// per eight weights, decoded by the expert kernels' own register decoder.
template <int FMT>
__global__ void dequantize8_kernel(const uint8_t* __restrict__ raw, float* __restrict__ out,
                                   int64_t n_groups) {
  constexpr int BE = BlockFmt<FMT>::kElems, BB = BlockFmt<FMT>::kBytes;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_groups) return;
  const int64_t c = 8 * g;
  float w[8];
  dq8<FMT>(raw + (c / BE) * BB, (int)(c % BE), w);
  float4* o = reinterpret_cast<float4*>(out + c);
  o[0] = make_float4(w[0], w[1], w[2], w[3]);
  o[1] = make_float4(w[4], w[5], w[6], w[7]);
}

}  // namespace moe

extern "C" {

int moe_dequantize(const uint8_t* raw, float* out, int qtype, int64_t n_elements,
                   moe_stream_t stream) {
  MOE_REQUIRE(raw && out, MOE_ERR_INVALID, "null pointer");
  if (qtype == MOE_Q5_1 || qtype == MOE_Q4_K || qtype == MOE_Q6_K) {
    const int be = moe::blockfmt_elems(qtype);
    MOE_REQUIRE(n_elements >= 0 && n_elements % be == 0, MOE_ERR_INVALID,
                "element count %lld is not a multiple of %d", (long long)n_elements, be);
    if (n_elements == 0) return MOE_OK;
    MOE_REQUIRE(((uintptr_t)out & 15) == 0, MOE_ERR_INVALID, "out must be 16-byte aligned");
    const int64_t ng = n_elements / 8;
    const unsigned grid = (unsigned)((ng + 255) / 256);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    {
      ::moe::ProfScope _prof(MOE_K_DEQUANT, s);
      if (qtype == MOE_Q5_1)
        moe::dequantize8_kernel<MOE_Q5_1><<<grid, 256, 0, s>>>(raw, out, ng);
      else if (qtype == MOE_Q4_K)
        moe::dequantize8_kernel<MOE_Q4_K><<<grid, 256, 0, s>>>(raw, out, ng);
      else
        moe::dequantize8_kernel<MOE_Q6_K><<<grid, 256, 0, s>>>(raw, out, ng);
    }
    return moe::check_launch("dequantize");
  }
  MOE_REQUIRE(moe::qtype_ok(qtype), MOE_ERR_UNSUPPORTED, "quant type %d not supported", qtype);
  MOE_REQUIRE(n_elements >= 0 && n_elements % 32 == 0, MOE_ERR_INVALID,
              "element count %lld is not a multiple of 32", (long long)n_elements);
  if (n_elements == 0) return MOE_OK;
  int64_t nb = n_elements / 32;
  int blk = 256;
  unsigned grid = (unsigned)((nb + blk - 1) / blk);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  {
    ::moe::ProfScope _prof(MOE_K_DEQUANT, s);
    if (qtype == MOE_Q4_0)
      moe::dequantize_kernel<MOE_Q4_0><<<grid, blk, 0, s>>>(raw, out, nb);
    else
      moe::dequantize_kernel<MOE_Q8_0><<<grid, blk, 0, s>>>(raw, out, nb);
  }
  return moe::check_launch("dequantize");
}

int moe_packed_bytes(int qtype, int n_mats, int rows, int cols, size_t* bytes) {
  MOE_REQUIRE(bytes, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(moe::qtype_ok(qtype), MOE_ERR_UNSUPPORTED, "quant type %d not supported", qtype);
  MOE_REQUIRE(n_mats > 0 && rows > 0 && cols > 0 && cols % 32 == 0, MOE_ERR_INVALID,
              "bad shape");
  *bytes = (size_t)n_mats * moe::matrix_bytes(qtype, rows, cols);
  return MOE_OK;
}

int moe_pack_weights(const uint8_t* raw, uint8_t* packed, int qtype, int n_mats, int rows,
                     int cols, moe_stream_t stream) {
  return moe::repack(raw, packed, qtype, n_mats, rows, cols,
                     reinterpret_cast<cudaStream_t>(stream), 0);
}

int moe_unpack_weights(const uint8_t* packed, uint8_t* raw, int qtype, int n_mats, int rows,
                       int cols, moe_stream_t stream) {
  return moe::repack(packed, raw, qtype, n_mats, rows, cols,
                     reinterpret_cast<cudaStream_t>(stream), 1);
}

}  // extern "C"
