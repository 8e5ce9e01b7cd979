// Grouped experts on raw (unpacked) weight matrices: f32 (GGML type 0) and the
// block formats Q5_1, Q4_K, Q6_K -- plus Q4_0 / Q8_0 when they meet one of
// those in the same layer (gemma4 ships a Q4_K gate/up with a Q5_1 down).
//
// The reference's own ExpertFFN holds dequantised f32 matrices
// (moe_forward.py:119-133), and the gemma4 expert loader dequantises Q4_K /
// Q5_1 slices before its f32 matvecs (nightmare_stream.py:3361-3441).  Here the
// matrices stay as stored; every weight is decoded in registers to the same
// f32 value the reference's decoder gives (blockfmt.cuh) and multiplied in f32.
//
//   raw_gateup_kernel  CTA = (work item of NR rows of one expert, strip of 16
//                      F-rows).  The item's activation rows are staged in
//                      shared memory; each warp owns two F-rows and streams
//                      their gate and up rows together, lane l decoding eight
//                      consecutive weights per 256-column step; shuffle
//                      reduction; act(g) * u into an f32 hidden buffer
//   raw_down_kernel    the same over W_down and the hidden rows, writing y
//                      (times the expert's down scale, if any)
// Work items come from the expert plan (chunks of NR rows per expert).
#include "blockfmt.cuh"

namespace moe {

constexpr int kRawWarps = 8;
constexpr int kRawRowsPerWarp = 2;
constexpr int kRawStrip = kRawWarps * kRawRowsPerWarp;   // output features per CTA
constexpr int kRawSmemLimit = 160 * 1024;

// acc[m][r] += w_m . xs[r] for NM weight rows w_m over this lane's columns,
// then the warp sums in every lane.  xs: NR rows of K floats (shared).
template <int FMT, int NR, int NM>
__device__ __forceinline__ void raw_dot(const uint8_t* const (&w)[NM], const float* xs, int K,
                                        float (&acc)[NM][NR], int lane) {
  for (int c = 8 * lane; c < K; c += 256) {
    float v[NM][8];
#pragma unroll
    for (int m = 0; m < NM; ++m) dq8<FMT>(w[m], c, v[m]);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const float4 a = *reinterpret_cast<const float4*>(xs + (size_t)r * K + c);
      const float4 b = *reinterpret_cast<const float4*>(xs + (size_t)r * K + c + 4);
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        float s = acc[m][r];
        s = fmaf(v[m][0], a.x, s); s = fmaf(v[m][1], a.y, s);
        s = fmaf(v[m][2], a.z, s); s = fmaf(v[m][3], a.w, s);
        s = fmaf(v[m][4], b.x, s); s = fmaf(v[m][5], b.y, s);
        s = fmaf(v[m][6], b.z, s); s = fmaf(v[m][7], b.w, s);
        acc[m][r] = s;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < NM; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m][r] += __shfl_xor_sync(0xffffffffu, acc[m][r], o);
}

// Stages NR rows of K floats (row r of the item from src_row(r), zeros past
// the item's nr rows) into xs.
template <int NR, typename RowFn>
__device__ __forceinline__ void raw_stage(float* xs, int K, int nr, RowFn src_row) {
  const int k4 = K / 4;
  for (int i = threadIdx.x; i < NR * k4; i += blockDim.x) {
    const int r = i / k4, q = i - r * k4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nr) v = __ldg(reinterpret_cast<const float4*>(src_row(r)) + q);
    reinterpret_cast<float4*>(xs)[i] = v;
  }
  __syncthreads();
}

struct RawArgs {
  const uint8_t* wg;
  const uint8_t* wu;
  const uint8_t* wd;
  size_t gu_stride;    // bytes per expert in the gate / up stacks
  size_t gu_row;       // bytes per gate / up row (d weights)
  size_t dn_stride;    // bytes per expert in the down stack
  size_t dn_row;       // bytes per down row (F weights)
  int d, F, act;
  const int32_t* offsets;
  const int* citem;
  const float* x;
  const int32_t* x_rows;
  int x_div;
  float* hidden;       // [rows][F]
  float* y;
  const int32_t* y_rows;
  const float* down_scale;
  int strips;
};

template <int FMT, int NR>
__global__ void __launch_bounds__(kRawWarps * 32)
raw_gateup_kernel(RawArgs a) {
  pdl_wait();   // the plan and the activations
  extern __shared__ __align__(16) float xs[];
  const int item = blockIdx.x / a.strips, strip = blockIdx.x - item * a.strips;
  int e, c0;
  if (!chunk_of(item, a.citem, NR, e, c0)) return;
  const int row0 = a.offsets[e], n = a.offsets[e + 1] - row0;
  const int nr = min(NR, n - c0);
  const int d = a.d, F = a.F;
  raw_stage<NR>(xs, d, nr, [&](int r) {
    const int rr = row0 + c0 + r;
    return a.x + (size_t)(a.x_rows ? a.x_rows[rr] / a.x_div : rr) * d;
  });
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = strip * kRawStrip + warp * kRawRowsPerWarp;
  if (f0 >= F) return;
  const int nf = min(kRawRowsPerWarp, F - f0);
  const uint8_t* gbase = a.wg + (size_t)e * a.gu_stride;
  const uint8_t* ubase = a.wu + (size_t)e * a.gu_stride;
  // gate and up rows of both F-rows stream together (rows past F repeat the
  // last one; their sums are not stored)
  const uint8_t* w[4] = {gbase + (size_t)f0 * a.gu_row, ubase + (size_t)f0 * a.gu_row,
                         gbase + (size_t)(f0 + nf - 1) * a.gu_row,
                         ubase + (size_t)(f0 + nf - 1) * a.gu_row};
  float acc[4][NR];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[m][r] = 0.f;
  raw_dot<FMT, NR, 4>(w, xs, d, acc, lane);
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < kRawRowsPerWarp; ++j) {
      if (j >= nf) break;
#pragma unroll
      for (int r = 0; r < NR; ++r)
        if (r < nr)
          a.hidden[(size_t)(row0 + c0 + r) * F + f0 + j] =
              expert_act(a.act, acc[2 * j][r]) * acc[2 * j + 1][r];
    }
  }
}

template <int FMT, int NR>
__global__ void __launch_bounds__(kRawWarps * 32)
raw_down_kernel(RawArgs a) {
  pdl_wait();   // the hidden rows
  extern __shared__ __align__(16) float hs[];
  const int item = blockIdx.x / a.strips, strip = blockIdx.x - item * a.strips;
  int e, c0;
  if (!chunk_of(item, a.citem, NR, e, c0)) return;
  const int row0 = a.offsets[e], n = a.offsets[e + 1] - row0;
  const int nr = min(NR, n - c0);
  const int d = a.d, F = a.F;
  raw_stage<NR>(hs, F, nr, [&](int r) { return a.hidden + (size_t)(row0 + c0 + r) * F; });
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = strip * kRawStrip + warp * kRawRowsPerWarp;
  if (o0 >= d) return;
  const int no = min(kRawRowsPerWarp, d - o0);
  const uint8_t* base = a.wd + (size_t)e * a.dn_stride;
  const uint8_t* w[2] = {base + (size_t)o0 * a.dn_row, base + (size_t)(o0 + no - 1) * a.dn_row};
  float acc[2][NR];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[m][r] = 0.f;
  raw_dot<FMT, NR, 2>(w, hs, F, acc, lane);
  if (lane == 0) {
    const float sc = a.down_scale ? a.down_scale[e] : 1.0f;
#pragma unroll
    for (int j = 0; j < kRawRowsPerWarp; ++j) {
      if (j >= no) break;
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        if (r >= nr) continue;
        const int sr = row0 + c0 + r;
        a.y[(size_t)(a.y_rows ? a.y_rows[sr] : sr) * d + o0 + j] =
            a.down_scale ? acc[j][r] * sc : acc[j][r];
      }
    }
  }
}

// Rows per work item for a shape: the largest of 8, 4, 2, 1 whose staged rows
// fit the shared-memory budget.
int raw_rows_per_chunk(int d, int F) {
  const int K = d > F ? d : F;
  int nr = 8;
  while (nr > 1 && (size_t)nr * K * sizeof(float) > (size_t)kRawSmemLimit) nr /= 2;
  return nr;
}

static bool raw_fmt_cols_ok(int fmt, int cols) {
  return blockfmt_ok(fmt) && cols % blockfmt_elems(fmt) == 0 && cols % 8 == 0;
}

void experts_plan_arrays(void* ws, int rows, int E, int d, int F, int** n_active, int** active,
                         int** goff, int** coff, int** done, int* mg);
void experts_hidden(void* ws, int rows, int E, int d, int F, uint8_t** hidden, int** status);
int launch_expert_plan(const int32_t* offsets, int E, int rows, int rpc, void* ws, int d, int F,
                       cudaStream_t s);

template <int FMT, int NR>
static int raw_set_attr(bool down) {
  static unsigned long long attr_set[2] = {0, 0};
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev));
  if (!((attr_set[down] >> (dev & 63)) & 1ull)) {
    if (down)
      MOE_CUDA(cudaFuncSetAttribute(raw_down_kernel<FMT, NR>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kRawSmemLimit));
    else
      MOE_CUDA(cudaFuncSetAttribute(raw_gateup_kernel<FMT, NR>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kRawSmemLimit));
    attr_set[down] |= 1ull << (dev & 63);
  }
  return MOE_OK;
}

template <int FMT, int NR>
static int raw_launch(const RawArgs& a, int items, bool down, cudaStream_t s) {
  MOE_CHECK((raw_set_attr<FMT, NR>(down)));
  RawArgs b = a;
  if (!down) {
    b.strips = (a.F + kRawStrip - 1) / kRawStrip;
    ::moe::ProfScope _prof(MOE_K_GATEUP, s);
    MOE_CUDA(launch_pdl(raw_gateup_kernel<FMT, NR>, dim3((unsigned)items * b.strips),
                        dim3(kRawWarps * 32), (size_t)NR * a.d * sizeof(float), s, b));
  } else {
    b.strips = (a.d + kRawStrip - 1) / kRawStrip;
    ::moe::ProfScope _prof(MOE_K_DOWN, s);
    MOE_CUDA(launch_pdl(raw_down_kernel<FMT, NR>, dim3((unsigned)items * b.strips),
                        dim3(kRawWarps * 32), (size_t)NR * a.F * sizeof(float), s, b));
  }
  return check_launch(down ? "raw_down" : "raw_gateup");
}

template <int NR>
static int raw_launch_fmt(int fmt, const RawArgs& a, int items, bool down, cudaStream_t s) {
  switch (fmt) {
    case MOE_F32: return raw_launch<MOE_F32, NR>(a, items, down, s);
    case MOE_Q4_0: return raw_launch<MOE_Q4_0, NR>(a, items, down, s);
    case MOE_Q8_0: return raw_launch<MOE_Q8_0, NR>(a, items, down, s);
    case MOE_Q5_1: return raw_launch<MOE_Q5_1, NR>(a, items, down, s);
    case MOE_Q4_K: return raw_launch<MOE_Q4_K, NR>(a, items, down, s);
    case MOE_Q6_K: return raw_launch<MOE_Q6_K, NR>(a, items, down, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "weight format %d", fmt);
  }
}

static int raw_launch_nr(int nr, int fmt, const RawArgs& a, int items, bool down,
                         cudaStream_t s) {
  switch (nr) {
    case 8: return raw_launch_fmt<8>(fmt, a, items, down, s);
    case 4: return raw_launch_fmt<4>(fmt, a, items, down, s);
    case 2: return raw_launch_fmt<2>(fmt, a, items, down, s);
    default: return raw_launch_fmt<1>(fmt, a, items, down, s);
  }
}

// Grouped experts on raw matrices of formats gu_fmt (gate, up) and dn_fmt
// (down).  opts: activation, gate/up stride (0 = one matrix), down scale.
int run_experts_raw(const uint8_t* wg, const uint8_t* wu, const uint8_t* wd, int gu_fmt,
                    int dn_fmt, const moe_expert_opts* opts, const int32_t* offsets, int E,
                    int rows, const float* x, const int32_t* x_rows, int x_div, int d, int F,
                    float* y, const int32_t* y_rows, void* ws, bool planned, cudaStream_t s) {
  MOE_REQUIRE(raw_fmt_cols_ok(gu_fmt, d), MOE_ERR_UNSUPPORTED,
              "gate/up format %d with d=%d (rows must be whole blocks)", gu_fmt, d);
  MOE_REQUIRE(raw_fmt_cols_ok(dn_fmt, F), MOE_ERR_UNSUPPORTED,
              "down format %d with F=%d (rows must be whole blocks)", dn_fmt, F);
  MOE_REQUIRE((size_t)d * sizeof(float) <= (size_t)kRawSmemLimit &&
                  (size_t)F * sizeof(float) <= (size_t)kRawSmemLimit,
              MOE_ERR_UNSUPPORTED, "d=%d / F=%d above %d floats", d, F, kRawSmemLimit / 4);
  MOE_REQUIRE(((uintptr_t)x & 15) == 0, MOE_ERR_INVALID, "activations must be 16-byte aligned");
  if (gu_fmt == MOE_F32 || dn_fmt == MOE_F32)
    MOE_REQUIRE(((uintptr_t)wg | (uintptr_t)wu | (uintptr_t)wd) % 16 == 0, MOE_ERR_INVALID,
                "f32 weights must be 16-byte aligned");
  const int nr = raw_rows_per_chunk(d, F);
  if (!planned) MOE_CHECK(launch_expert_plan(offsets, E, rows, nr, ws, d, F, s));
  int *n_active, *active, *goff, *coff, *done, mg;
  experts_plan_arrays(ws, rows, E, d, F, &n_active, &active, &goff, &coff, &done, &mg);
  uint8_t* hid = nullptr;
  int* status = nullptr;
  experts_hidden(ws, rows, E, d, F, &hid, &status);
  RawArgs a = {};
  a.wg = wg;
  a.wu = wu;
  a.wd = wd;
  a.gu_row = blockfmt_row_bytes(gu_fmt, d);
  a.gu_stride = (opts && opts->gate_up_stride) ? opts->gate_up_stride : a.gu_row * F;
  a.dn_row = blockfmt_row_bytes(dn_fmt, F);
  a.dn_stride = a.dn_row * d;
  a.d = d;
  a.F = F;
  a.act = opts ? opts->act : MOE_ACT_SWIGLU;
  a.offsets = offsets;
  a.citem = coff;
  a.x = x;
  a.x_rows = x_rows;
  a.x_div = x_div;
  a.hidden = reinterpret_cast<float*>(hid);
  a.y = y;
  a.y_rows = y_rows;
  a.down_scale = opts ? opts->down_scale : nullptr;
  const int items = rows / nr + E;            // upper bound on work items
  MOE_CHECK(raw_launch_nr(nr, gu_fmt, a, items, false, s));
  return raw_launch_nr(nr, dn_fmt, a, items, true, s);
}

}  // namespace moe
