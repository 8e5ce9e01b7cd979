// Host-side functions shared between the library's translation units.
#pragma once

#include "moe_common.cuh"

namespace moe {

// router.cu
// The dispatch of one token's k pairs, done by the router's selection CTA
// (the outputs of launch_dispatch_planned).
struct SmallDispatch {
  int32_t* offsets;
  int32_t* perm;
  int32_t* inv;
  int* status;
  int* n_active;
  int* active;
  int* goff;
  int* coff;
  int* done;
  int max_groups, rpc;
};
bool router_fuses_dispatch(int T, int E, int k);
int launch_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
                  int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream, float* row_max,
                  const SmallDispatch* sd = nullptr, float* xcopy = nullptr);

// dispatch.cu
int launch_dispatch_planned(const int32_t* ids, int T, int k, int E, int32_t* offsets,
                            int32_t* perm_rows, int32_t* inv_perm, int* status, int* n_active,
                            int* active, int* goff, int* coff, int* done, int max_groups,
                            int rpc, int32_t* scratch, cudaStream_t s);
size_t dispatch_scratch_bytes(int P, int E);

// experts.cu
int run_experts(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                const int32_t* offsets, int E, int rows, const float* x, const int32_t* x_rows,
                int x_div, int d, int F, float* y, const int32_t* y_rows, void* ws,
                size_t ws_bytes, cudaStream_t s, int* status, const float* x_row_max,
                bool planned, int rows_hint, const moe_expert_opts* opts);
// rows per work item of the GEMV path; rows_hint as run_experts'
int experts_rows_per_chunk(int qtype, int dn_qtype, int rows, int E, int d, int F,
                           int rows_hint = 0);
int experts_down_qtype(int qtype, const moe_expert_opts* opts);
int experts_workspace(int rows, int E, int d, int F, size_t* bytes);
int experts_workspace_hint(int rows, int rows_hint, int E, int d, int F, size_t* bytes);
void experts_plan_arrays(void* ws, int rows, int E, int d, int F, int** n_active, int** active,
                         int** goff, int** coff, int** done, int* mg);

// combine.cu
int launch_combine(const float* y, const int32_t* inv_perm, const float* w, const float* shared,
                   const float* residual, int T, int k, int d, float* out, cudaStream_t s);

// Where a pointer lives: pinned (page-locked, device-mapped) host memory is
// read and written by device code through the same pointer; pageable host
// memory cannot be.
enum { kMemDevice = 0, kMemPinnedHost = 1, kMemPageable = 2 };
inline int memory_kind(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return kMemDevice;
  }
  if (a.type == cudaMemoryTypeHost) return kMemPinnedHost;
  if (a.type == cudaMemoryTypeUnregistered) return kMemPageable;
  return kMemDevice;
}

// The shared expert's options: the routed experts' activation, one matrix
// per stack, no down scale.
inline moe_expert_opts shared_expert_opts(const moe_expert_opts* routed) {
  moe_expert_opts o = {};
  o.act = routed ? routed->act : MOE_ACT_SWIGLU;
  return o;
}

}  // namespace moe
