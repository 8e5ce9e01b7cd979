// Raw GGUF block formats decoded in registers, eight consecutive weights at a
// time, to exactly the f32 values the reference's decoders produce
// (dequant_fast.py): F32, Q4_0 (:69-100), Q8_0 (:44-66), Q5_1 (:169-201),
// Q4_K (:237-289), Q6_K (:343-378).  Every product below is exact in f32 (the
// operands' significands are at most 24 bits together); the one sum (Q5_1's
// + min, Q4_K's - min) is rounded once, as numpy rounds it.
#pragma once

#include "moe_common.cuh"

namespace moe {

template <int FMT> struct BlockFmt;
template <> struct BlockFmt<MOE_F32> { static constexpr int kElems = 1, kBytes = 4; };
template <> struct BlockFmt<MOE_Q4_0> { static constexpr int kElems = 32, kBytes = 18; };
template <> struct BlockFmt<MOE_Q8_0> { static constexpr int kElems = 32, kBytes = 34; };
template <> struct BlockFmt<MOE_Q5_1> { static constexpr int kElems = 32, kBytes = 24; };
template <> struct BlockFmt<MOE_Q4_K> { static constexpr int kElems = 256, kBytes = 144; };
template <> struct BlockFmt<MOE_Q6_K> { static constexpr int kElems = 256, kBytes = 210; };

inline bool blockfmt_ok(int fmt) {
  return fmt == MOE_F32 || fmt == MOE_Q4_0 || fmt == MOE_Q8_0 || fmt == MOE_Q5_1 ||
         fmt == MOE_Q4_K || fmt == MOE_Q6_K;
}
inline int blockfmt_elems(int fmt) {
  switch (fmt) {
    case MOE_F32: return 1;
    case MOE_Q4_K: case MOE_Q6_K: return 256;
    default: return 32;
  }
}
inline int blockfmt_bytes(int fmt) {
  switch (fmt) {
    case MOE_F32: return 4;
    case MOE_Q4_0: return 18;
    case MOE_Q8_0: return 34;
    case MOE_Q5_1: return 24;
    case MOE_Q4_K: return 144;
    case MOE_Q6_K: return 210;
    default: return 0;
  }
}
// bytes of one row of `cols` weights (cols a multiple of the block length)
inline size_t blockfmt_row_bytes(int fmt, int cols) {
  return (size_t)(cols / blockfmt_elems(fmt)) * blockfmt_bytes(fmt);
}

__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(p))));
}

__device__ __forceinline__ uint32_t ld_b(const uint8_t* p) { return __ldg(p); }

// w[i] = weight c + i of a row starting at `row`; c % 8 == 0.
template <int FMT>
__device__ __forceinline__ void dq8(const uint8_t* __restrict__ row, int c, float (&w)[8]) {
  if (FMT == MOE_F32) {
    const float4* p = reinterpret_cast<const float4*>(row) + c / 4;
    const float4 a = __ldg(p), b = __ldg(p + 1);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else if (FMT == MOE_Q8_0) {
    // [fp16 d][int8 q x 32]: d * q
    const uint8_t* blk = row + (size_t)(c / 32) * 34;
    const float d = ld_half(blk);
    const uint8_t* q = blk + 2 + (c & 31);
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = d * (float)(int8_t)ld_b(q + i);
  } else if (FMT == MOE_Q4_0) {
    // [fp16 d][16 bytes]: weight j < 16 = low nibble of byte j, j >= 16 = high
    // nibble of byte j - 16; d * (nibble - 8)
    const uint8_t* blk = row + (size_t)(c / 32) * 18;
    const float d = ld_half(blk);
    const int j = c & 31;
    const uint8_t* q = blk + 2 + (j & 15);
    const int sh = j >= 16 ? 4 : 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = d * (float)((int)((ld_b(q + i) >> sh) & 15u) - 8);
  } else if (FMT == MOE_Q5_1) {
    // [fp16 d][fp16 m][u32 qh][16 bytes]: nibble as Q4_0, fifth bit = qh bit of
    // the weight's index; d * q + m
    const uint8_t* blk = row + (size_t)(c / 32) * 24;
    const float d = ld_half(blk), m = ld_half(blk + 2);
    const uint32_t qh = ld_b(blk + 4) | (ld_b(blk + 5) << 8) | (ld_b(blk + 6) << 16) |
                        (ld_b(blk + 7) << 24);
    const int j = c & 31;
    const uint8_t* q = blk + 8 + (j & 15);
    const int sh = j >= 16 ? 4 : 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t v = ((ld_b(q + i) >> sh) & 15u) | (((qh >> (j + i)) & 1u) << 4);
      w[i] = __fadd_rn(__fmul_rn(d, (float)v), m);
    }
  } else if (FMT == MOE_Q4_K) {
    // super-block of 256: [fp16 d][fp16 dmin][12 scale bytes][128 quant bytes];
    // sub-block s (32 weights) has 6-bit scale / min (llama.cpp's
    // get_scale_min_k4 packing); its weights are the low (s even) or high
    // (s odd) nibbles of quant bytes 32 (s / 2) .. + 31; (d sc) q - dmin m
    const uint8_t* sb = row + (size_t)(c / 256) * 144;
    const int p = c & 255, s = p >> 5;
    const uint8_t* sc = sb + 4;
    uint32_t scv, mnv;
    if (s < 4) {
      scv = ld_b(sc + s) & 63u;
      mnv = ld_b(sc + s + 4) & 63u;
    } else {
      scv = (ld_b(sc + s + 4) & 15u) | ((ld_b(sc + s - 4) >> 6) << 4);
      mnv = (ld_b(sc + s + 4) >> 4) | ((ld_b(sc + s) >> 6) << 4);
    }
    const float scale = __fmul_rn(ld_half(sb), (float)scv);
    const float mn = __fmul_rn(ld_half(sb + 2), (float)mnv);
    const uint8_t* q = sb + 16 + 32 * (s >> 1) + (p & 31);
    const int sh = (s & 1) ? 4 : 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i] = __fsub_rn(__fmul_rn(scale, (float)((ld_b(q + i) >> sh) & 15u)), mn);
  } else if (FMT == MOE_Q6_K) {
    // super-block of 256: [ql x 128][qh x 64][int8 scales x 16][fp16 d]; each
    // half of 128 weights is four streams of 32 (low / high nibbles of ql
    // bytes l and l + 32 with two bits of qh byte l); d * scale[p / 16] * (q - 32)
    const uint8_t* sb = row + (size_t)(c / 256) * 210;
    const int p = c & 255, half = p >> 7, ph = p & 127, st = ph >> 5, l = ph & 31;
    const uint8_t* ql = sb + 64 * half + ((st & 1) ? 32 : 0) + l;
    const uint8_t* qh = sb + 128 + 32 * half + l;
    const float dsc = __fmul_rn(ld_half(sb + 208), (float)(int8_t)ld_b(sb + 192 + 8 * half + (ph >> 4)));
    const int qsh = (st & 2) ? 4 : 0, hsh = 2 * st;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = (int)(((ld_b(ql + i) >> qsh) & 15u) | (((ld_b(qh + i) >> hsh) & 3u) << 4));
      w[i] = __fmul_rn(dsc, (float)(v - 32));
    }
  }
}

}  // namespace moe
