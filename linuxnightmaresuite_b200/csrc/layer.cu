// Whole MoE layer: router -> dispatch -> grouped experts -> combine.
// MoELayer.forward (moe_forward.py:154-174) for a batch of tokens.
#include "internal.cuh"

namespace moe {

__global__ void fill_two_offsets(int32_t* off, int n) {
  if (threadIdx.x == 0) {
    off[0] = 0;
    off[1] = n;
  }
}

struct LayerWs {
  int* status;
  uint8_t* router_ws;
  size_t router_bytes;
  int32_t* ids;
  float* wts;
  int32_t* offsets;
  int32_t* perm;
  int32_t* inv;
  int32_t* disp_scratch;
  uint8_t* exp_ws;
  size_t exp_bytes;
  float* y;
  int32_t* s_off;
  float* s_y;
  float* row_max;
  float* xdev;      // device copy of x when the caller's x is in host memory
  size_t bytes;
};

static LayerWs carve_layer(void* ws, const moe_layer_weights* w, int T) {
  Carve c{static_cast<uint8_t*>(ws), 0, 0};
  LayerWs L;
  const size_t P = (size_t)T * w->k;
  L.status = c.take<int>(64);
  moe_router_workspace_bytes(T, w->d, w->E, &L.router_bytes);
  L.router_ws = c.take<uint8_t>(L.router_bytes);
  L.ids = c.take<int32_t>(P);
  L.wts = c.take<float>(P);
  L.offsets = c.take<int32_t>(w->E + 1);
  L.perm = c.take<int32_t>(P);
  L.inv = c.take<int32_t>(P);
  L.disp_scratch = c.take<int32_t>(dispatch_scratch_bytes((int)P, w->E) / 4 + 1);
  size_t eb = 0, sb = 0;
  experts_workspace((int)P, w->E, w->d, w->F, &eb);
  if (w->s_gate) experts_workspace(T, 1, w->d, w->Fs, &sb);
  L.exp_bytes = eb > sb ? eb : sb;
  L.exp_ws = c.take<uint8_t>(L.exp_bytes);
  L.y = c.take<float>(P * w->d);
  L.s_off = c.take<int32_t>(2);
  L.s_y = w->s_gate ? c.take<float>((size_t)T * w->d) : nullptr;
  L.row_max = c.take<float>(T > 0 ? T : 1);
  L.xdev = c.take<float>((size_t)(T > 0 ? T : 1) * w->d);
  L.bytes = align_up(c.used, 256);
  return L;
}

}  // namespace moe

extern "C" {

int moe_layer_workspace_bytes(const moe_layer_weights* w, int T, size_t* bytes) {
  MOE_REQUIRE(w && bytes, MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(T >= 0 && w->E > 0 && w->k > 0 && w->d > 0 && w->F > 0, MOE_ERR_INVALID,
              "bad shape");
  *bytes = moe::carve_layer(nullptr, w, T).bytes;
  return MOE_OK;
}

int moe_layer_forward(const moe_layer_weights* w, const float* x, int T, float* out,
                      const float* residual, int32_t* ids_out, float* weights_out,
                      void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  return moe_layer_forward_ex(w, x, nullptr, T, out, residual, ids_out, weights_out, workspace,
                              workspace_bytes, stream);
}

int moe_layer_forward_ex(const moe_layer_weights* w, const float* x, const float* router_x, int T,
                         float* out, const float* residual, int32_t* ids_out, float* weights_out,
                         void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  using namespace moe;
  MOE_REQUIRE(w, MOE_ERR_INVALID, "null weights");
  MOE_REQUIRE(T >= 0, MOE_ERR_INVALID, "T must be >= 0");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(x && out && workspace && w->gate_w && w->w_gate && w->w_up && w->w_down,
              MOE_ERR_INVALID, "null pointer");
  MOE_REQUIRE(x != out && router_x != out, MOE_ERR_INVALID, "out must not alias the inputs");
  MOE_REQUIRE(!w->opts || w->opts->act == MOE_ACT_SWIGLU || w->opts->act == MOE_ACT_GEGLU_TANH,
              MOE_ERR_INVALID, "unknown activation %d", w->opts ? w->opts->act : 0);
  MOE_REQUIRE(w->k > 0 && w->k <= w->E, MOE_ERR_INVALID, "top_k %d vs %d experts", w->k, w->E);
  MOE_REQUIRE(!w->s_gate || (w->s_up && w->s_down && w->Fs > 0), MOE_ERR_INVALID,
              "incomplete shared expert");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LayerWs L = carve_layer(workspace, w, T);
  MOE_REQUIRE(workspace_bytes >= L.bytes, MOE_ERR_WORKSPACE, "layer workspace %zu < %zu",
              workspace_bytes, L.bytes);
  int32_t* ids = ids_out ? ids_out : L.ids;
  float* wts = weights_out ? weights_out : L.wts;
  const int P = T * w->k;
  int *n_active, *active, *goff, *coff, *done, mg;
  experts_plan_arrays(L.exp_ws, P, w->E, w->d, w->F, &n_active, &active, &goff, &coff, &done,
                      &mg);
  const int rpc = experts_rows_per_chunk(w->qtype, experts_down_qtype(w->qtype, w->opts), P,
                                         w->E, w->d, w->F);
  // one token: the router's selection CTA also sorts its k pairs and writes
  // the plan (no dispatch kernel)
  SmallDispatch sd = {L.offsets, L.perm, L.inv, L.status, n_active, active, goff, coff, done,
                      mg, rpc};
  const bool fused = router_fuses_dispatch(T, w->E, w->k);
  // x (and out) may be pinned host memory: the router's first pass then
  // reads x over the bus and leaves the device copy every later kernel reads
  // (no separate host-to-device copy); out is written in place by the combine
  const int xk = memory_kind(x);
  MOE_REQUIRE(xk != kMemPageable && memory_kind(out) != kMemPageable, MOE_ERR_INVALID,
              "x and out must be device or pinned host memory");
  const bool x_host = xk == kMemPinnedHost;
  const float* xe = x;
  float* xcopy = nullptr;
  if (x_host) {
    xe = L.xdev;
    if (router_x) MOE_CUDA(cudaMemcpyAsync(L.xdev, x, (size_t)T * w->d * sizeof(float),
                                           cudaMemcpyDefault, s));
    else xcopy = L.xdev;
  }
  // the router's per-row maxima double as the experts' activation scaling,
  // so they are only taken from the router when it reads the experts' input
  MOE_CHECK(launch_router(router_x ? router_x : x, w->gate_w, w->bias, T, w->d, w->E, w->k,
                          w->router_layout, w->mode, ids, wts, L.router_ws, L.router_bytes, s,
                          router_x ? nullptr : L.row_max, fused ? &sd : nullptr, xcopy));
  const float* row_max = router_x ? nullptr : L.row_max;
  if (!fused)
    MOE_CHECK(launch_dispatch_planned(ids, T, w->k, w->E, L.offsets, L.perm, L.inv, L.status,
                                      n_active, active, goff, coff, done, mg, rpc,
                                      L.disp_scratch, s));
  MOE_CHECK(run_experts(w->w_gate, w->w_up, w->w_down, w->qtype, L.offsets, w->E, P, xe, L.perm,
                        w->k, w->d, w->F, L.y, nullptr, L.exp_ws, L.exp_bytes, s, L.status,
                        row_max, true, 0, w->opts));
  if (w->s_gate) {
    {
      ::moe::ProfScope _prof(MOE_K_AUX, s);
      fill_two_offsets<<<1, 32, 0, s>>>(L.s_off, T);
    }
    MOE_CHECK(check_launch("fill_offsets"));
    const moe_expert_opts so = shared_expert_opts(w->opts);
    MOE_CHECK(run_experts(w->s_gate, w->s_up, w->s_down, w->shared_qtype, L.s_off, 1, T, xe,
                          nullptr, 1, w->d, w->Fs, L.s_y, nullptr, L.exp_ws, L.exp_bytes, s,
                          L.status, row_max, false, 0, &so));
  }
  return launch_combine(L.y, L.inv, wts, L.s_y, residual, T, w->k, w->d, out, s);
}

}  // extern "C"
