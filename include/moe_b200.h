/*
 * moe_b200.h -- C ABI of the B200 mixture-of-experts layer forward.
 *
 * Replaces the Python/NVRTC MoE FFN path of NightmareDesigns/Linuxnightmaresuite:
 * moe_forward.py (MoERouter / ExpertFFN / MoELayer), the GGUF block decoders of
 * dequant_fast.py and the per-expert GpuMM launches of qwen35_gpu.py that the
 * streaming engines drive (nightmare_stream.py _moe_ffn_gpu / _moe_ffn_g4_gpu).
 *
 * Conventions
 *   - Every function returns an int status: MOE_OK (0) or a negative MOE_ERR_*;
 *     moe_last_error() returns the calling thread's last message.
 *   - All tensor pointers are DEVICE pointers owned by the caller.  Nothing here
 *     allocates device memory: scratch comes from a caller-provided workspace
 *     whose size the matching *_workspace_bytes() reports.
 *   - Work is enqueued asynchronously on the given stream (0 = legacy default).
 *   - Weights enter as raw GGUF block bytes (Q4_0 = GGML type 2, Q8_0 = type 8),
 *     expert-major, each matrix (rows, cols) row-major in the reference's
 *     (out, in) orientation.  moe_pack_weights() rearranges them once, at load
 *     time, into the tile order the expert kernels stream; the packed buffer
 *     has exactly the size of the raw one and moe_unpack_weights() inverts it.
 *   - Routing modes: MOE_ROUTE_TOPK_SOFTMAX follows MoERouter.route
 *     (moe_forward.py:91-109); MOE_ROUTE_SOFTMAX_TOPK_RENORM follows
 *     GPUStreamEngine._moe_ffn (nightmare_stream.py:3227-3238).  Ties between
 *     equal scores go to the higher expert index first.
 *   - Device-detected input errors (e.g. an out-of-range expert id) set bits in
 *     the status word at the start of the workspace; moe_read_status() fetches it.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* moe_stream_t; /* same object as cudaStream_t */

enum {
  MOE_OK = 0,
  MOE_ERR_INVALID = -1,     /* bad argument (null pointer, non-positive size, k > E) */
  MOE_ERR_UNSUPPORTED = -2, /* quant type or shape this build does not handle */
  MOE_ERR_WORKSPACE = -3,   /* workspace smaller than *_workspace_bytes() */
  MOE_ERR_CUDA = -4,        /* a CUDA runtime call or kernel launch failed */
  MOE_ERR_DEVICE = -5       /* moe_read_status found a device-side error bit */
};

/* GGML type ids, dequant_fast.py:689-754.  Q4_0 and Q8_0 run on the packed-tile
 * GEMV / tensor-core kernels.  MOE_F32 (type 0: f32 matrices as the reference's
 * ExpertFFN holds them, moe_forward.py:119-133) and the block formats Q5_1,
 * Q4_K and Q6_K (dequant_fast.py:169-401; the formats gemma4 experts ship in)
 * run on the raw-block path: the matrices are used as stored, each weight
 * decoded in registers exactly as the reference decodes it. */
enum { MOE_F32 = 0, MOE_Q4_0 = 2, MOE_Q5_1 = 7, MOE_Q8_0 = 8, MOE_Q4_K = 12, MOE_Q6_K = 14 };

/* Gated activation of the experts: SwiGLU silu(g) * u (moe_forward.py:129-133)
 * or gemma4's GeGLU-tanh (qwen35_gpu.py:933-939, nightmare_stream.py:3256-3271). */
enum { MOE_ACT_SWIGLU = 0, MOE_ACT_GEGLU_TANH = 1 };

/* Expert variant options (zero-initialised = the reference's MoELayer experts).
 *   act             MOE_ACT_*
 *   down_qtype      quant type of w_down; 0 with qtype != MOE_F32 means "same
 *                   as qtype" (gemma4 ships Q4_K gate/up with a Q5_1 down)
 *   gate_up_stride  bytes from one expert's gate (and up) matrix to the next;
 *                   0 = one matrix.  For a fused ffn_gate_up_exps stack
 *                   (E, 2F, d) pass w_gate = the stack, w_up = w_gate + one
 *                   (F, d) matrix, stride = two matrices
 *                   (nightmare_stream.py:3361-3441)
 *   down_scale      (E_local,) f32 per-expert factor on the down projection
 *                   (ffn_down_exps.scale, nightmare_stream.py:4307-4330), or NULL
 *   kernels         MOE_KERNELS_*: which kernel family runs packed Q4_0 / Q8_0
 *                   experts; 0 = chosen from the routed rows per active expert
 *   chunk_rows      block-scale family: rows per work unit (8, 16, 32 or 64;
 *                   0 = chosen from the routed rows per active expert) */
typedef struct moe_expert_opts {
  int act;
  int down_qtype;
  size_t gate_up_stride;
  const float* down_scale;
  int kernels;
  int chunk_rows;
} moe_expert_opts;

/* Kernel families for packed experts: mma.sync GEMVs (a few rows per expert),
 * block-scale tcgen05 GEMMs (exact integer weights, per-block scaling; mid-size
 * groups), split-operand tcgen05 GEMMs (large groups). */
enum { MOE_KERNELS_AUTO = 0, MOE_KERNELS_GEMV = 1, MOE_KERNELS_BLOCKSCALE = 2,
       MOE_KERNELS_SPLIT_GEMM = 3 };

enum { MOE_ROUTE_TOPK_SOFTMAX = 0, MOE_ROUTE_SOFTMAX_TOPK_RENORM = 1 };

enum { MOE_ROUTER_D_E = 0, MOE_ROUTER_E_D = 1 }; /* router weight layout */

/* device status bits */
enum { MOE_STATUS_BAD_EXPERT_ID = 1, MOE_STATUS_ROW_OVERFLOW = 2, MOE_STATUS_TIMEOUT = 4 };

/* ---- library ------------------------------------------------------------ */

/* Library version, major*10000 + minor*100 + patch. */
int moe_version(void);

/* Copies the calling thread's last error message (NUL-terminated). */
int moe_last_error(char* buf, size_t len);

/* Weights per block and bytes per block of a GGML type (F32 is one weight of
 * 4 bytes).  Replaces dequant_fast.BLOCK_SIZES (dequant_fast.py:723-754) for
 * the types this library takes. */
int moe_block_geometry(int qtype, int* elems_per_block, int* bytes_per_block);

/* Reads (and clears) the device status word a workspace carries. Synchronises
 * the stream.  Returns MOE_ERR_DEVICE if any bit was set. */
int moe_read_status(const void* workspace, int* status_out, moe_stream_t stream);

/* ---- profiling (no counterpart in the reference) ---------------------------------
 * When enabled, every kernel launch of the library is bracketed by a pair of
 * CUDA events on its stream; moe_profile_collect() waits for them and returns,
 * per kernel id, the summed device milliseconds and the number of launches,
 * then resets.  Do not enable while capturing a CUDA graph. */
enum {
  MOE_K_ROUTER = 0, MOE_K_ROUTER_SELECT, MOE_K_DISPATCH, MOE_K_PLAN, MOE_K_XPREP,
  MOE_K_GATEUP, MOE_K_DOWN, MOE_K_COMBINE, MOE_K_RMS_NORM, MOE_K_PACK, MOE_K_DEQUANT,
  MOE_K_AUX, MOE_K_EP_SEND, MOE_K_EP_RECV, MOE_K_EP_RETURN, MOE_K_EP_WAIT, MOE_K_COUNT
};
int moe_profile_enable(int on);
int moe_profile_collect(float* ms, int* launches, int n);

/* ---- weights ---------------------------------------------------------------- */

/* Decodes n_elements weights of raw GGUF blocks (Q4_0, Q8_0, Q5_1, Q4_K, Q6_K)
 * to f32, bit for bit as the reference.  GPU counterpart of
 * dequant_fast.dequantize_q4_0 / dequantize_q8_0 / dequantize_q5_1 /
 * dequantize_q4_k / dequantize_q6_k (dequant_fast.py:44-100, :169-201,
 * :237-289, :343-378) and of the dequant_q4_0 / dequant_q8_34 kernels
 * (qwen35_gpu.py:610-648). */
int moe_dequantize(const uint8_t* raw, float* out, int qtype, int64_t n_elements,
                   moe_stream_t stream);

/* Size in bytes of n_mats packed (rows, cols) matrices (== raw size). */
int moe_packed_bytes(int qtype, int n_mats, int rows, int cols, size_t* bytes);

/* Raw GGUF blocks of n_mats stacked (rows, cols) matrices -> packed tiles.
 * Needs rows % 16 == 0 and cols % 64 == 0.  Replaces the raw expert upload of
 * GpuMM.upload_raw (qwen35_gpu.py:1884-1924) / _load_expert_fast
 * (nightmare_stream.py:3361-3441) as the load-time step. */
int moe_pack_weights(const uint8_t* raw, uint8_t* packed, int qtype, int n_mats, int rows,
                     int cols, moe_stream_t stream);

/* Inverse of moe_pack_weights (bit-exact round trip). */
int moe_unpack_weights(const uint8_t* packed, uint8_t* raw, int qtype, int n_mats, int rows,
                       int cols, moe_stream_t stream);

/* ---- router ------------------------------------------------------------------- */

int moe_router_workspace_bytes(int T, int d, int E, size_t* bytes);

/* Router logits, selection and weights for T tokens in one pass.
 *   x        (T, d) f32
 *   gate_w   (d, E) f32 for MOE_ROUTER_D_E (MoERouter.gate_weight, moe_forward.py:83)
 *            or (E, d) for MOE_ROUTER_E_D (the production 'moe_router' tensor)
 *   bias     (E,) f32 added to the logits, or NULL
 *   ids      (T, k) int32 out, weights (T, k) f32 out, in the reference's order:
 *            descending for MOE_ROUTE_TOPK_SOFTMAX, ascending for
 *            MOE_ROUTE_SOFTMAX_TOPK_RENORM.
 * Replaces MoERouter.route (moe_forward.py:91-109), the host softmax/argsort of
 * nightmare_stream.py:3227-3238 / :3296-3306 and the router matvec_t launch
 * (qwen35_gpu.py:39-47). */
int moe_router(const float* x, const float* gate_w, const float* bias, int T, int d, int E,
               int k, int layout, int mode, int32_t* ids, float* weights, void* workspace,
               size_t workspace_bytes, moe_stream_t stream);

/* moe_router without a workspace: no counterpart in the reference.  For callers
 * that can neither allocate device memory nor let the library allocate (all
 * device memory already belongs to the caller's own pool, or a fixed memory
 * footprint is required).  Same inputs, outputs and results as moe_router; its
 * scratch is a fixed 4 MiB array inside the library (held on every GPU that
 * loads it), so it rejects with MOE_ERR_WORKSPACE any call needing more than
 * 1,048,576 partial logits (slices x T x E; it uses as few slices as fit, so up
 * to 8192 tokens at E=128).  The first call on a device looks up the array's device address;
 * make it before any stream capture.  That address is kept for the life of the
 * process: do not call this again on a device after cudaDeviceReset.  Calls share the array: calls that overlap
 * on the GPU race and must be serialised by the caller.  Allocates nothing. */
int moe_router_noalloc(const float* x, const float* gate_w, const float* bias, int T, int d,
                       int E, int k, int layout, int mode, int32_t* ids, float* weights,
                       moe_stream_t stream);

/* ---- dispatch ------------------------------------------------------------------ */

int moe_dispatch_workspace_bytes(int T, int k, int E, size_t* bytes);

/* Stable counting sort of the T*k (token, slot) pairs by expert id.
 *   expert_offsets (E+1) out: rows of expert e are [off[e], off[e+1])
 *   perm_rows (T*k) out: sorted row r holds pair perm_rows[r] = t*k + slot
 *   inv_perm  (T*k) out: pair p sits at row inv_perm[p]
 * Within an expert, pairs keep ascending (t, slot) order.  Ids outside [0,E)
 * set MOE_STATUS_BAD_EXPERT_ID and are dropped (their inv_perm entry is -1).
 * Replaces the per-token `for eid in top_idx` loops of moe_forward.py:166-168 and
 * nightmare_stream.py:3240-3253. */
int moe_dispatch(const int32_t* ids, int T, int k, int E, int32_t* expert_offsets,
                 int32_t* perm_rows, int32_t* inv_perm, void* workspace,
                 size_t workspace_bytes, moe_stream_t stream);

/* ---- experts --------------------------------------------------------------------- */

int moe_experts_workspace_bytes(int rows, int E_local, int d, int F, size_t* bytes);

/* Grouped SwiGLU experts over expert-sorted rows:
 *   y[r] = W_down[e] (silu(W_gate[e] x[r]) * (W_up[e] x[r]))   for r in expert e's rows.
 *   w_gate, w_up   packed (E_local, F, d) stacks, w_down packed (E_local, d, F)
 *   expert_offsets (E_local+1) row offsets (as moe_dispatch writes them)
 *   x              activations; sorted row r reads x row
 *                  (x_rows ? x_rows[r] / x_rows_div : r)
 *   y              (.., d) f32 out; sorted row r writes y row (y_rows ? y_rows[r] : r)
 *   rows           number of sorted rows (== expert_offsets[E_local])
 * Replaces ExpertFFN.forward (moe_forward.py:129-133) and the per-expert
 * matvec_q4_0 / matvec_q8_34 / kernel_silu_mul launches (qwen35_gpu.py:55-104,
 * :904-910) of _moe_ffn_gpu (nightmare_stream.py:3308-3331). */
int moe_experts(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                const int32_t* expert_offsets, int E_local, int rows, const float* x,
                const int32_t* x_rows, int x_rows_div, int d, int F, float* y,
                const int32_t* y_rows, void* workspace, size_t workspace_bytes,
                moe_stream_t stream);

/* moe_experts with an expert variant (activation, fused gate/up stride,
 * per-expert down scale, a down matrix of another type).  Q4_0 / Q8_0 on all
 * three matrices run on packed weights; F32 and the other block formats (and
 * mixed types) take the matrices as stored.  Replaces the gemma4 expert path
 * of _moe_ffn_g4_gpu (nightmare_stream.py:4330-4459) and its CPU counterpart
 * (_load_expert_fast + _expert_act, nightmare_stream.py:3256-3441). */
int moe_experts_ex(const uint8_t* w_gate, const uint8_t* w_up, const uint8_t* w_down, int qtype,
                   const moe_expert_opts* opts, const int32_t* expert_offsets, int E_local,
                   int rows, const float* x, const int32_t* x_rows, int x_rows_div, int d, int F,
                   float* y, const int32_t* y_rows, void* workspace, size_t workspace_bytes,
                   moe_stream_t stream);

/* ---- combine ----------------------------------------------------------------------- */

/* out[t] = sum_slot weights[t,slot] * y[inv_perm[t*k+slot]]  (+ shared[t]) (+ residual[t]),
 * summed in slot order in f32.  shared / residual may be NULL.  out may alias
 * residual.  Replaces `output += w * expert_out` and the shared-expert add
 * (moe_forward.py:165-172) and kernel_add_scaled (qwen35_gpu.py:920-924). */
int moe_combine(const float* y, const int32_t* inv_perm, const float* weights,
                const float* shared, const float* residual, int T, int k, int d, float* out,
                moe_stream_t stream);

/* ---- expert parallelism ----------------------------------------------------------- */

/* out[r] = x[rows[r] / div] for r < n: the expert-sorted send buffer of the
 * expert-parallel exchange (rows = moe_dispatch's perm_rows, div = k).  Replaces
 * the per-expert host upload of the token vector to each card
 * (nightmare_stream.py:4381-4395). */
int moe_gather_rows(const float* x, const int32_t* rows, int div, int n, int d, float* out,
                    moe_stream_t stream);

/* Owner-side order of rows received in an expert-parallel exchange.
 *   recv_counts (W, E_local) int32: rows source s sent for local expert e; the
 *   receive buffer holds them source-major, expert-minor.
 *   local_offsets (E_local+1) out; row_map (<= max_rows) out: expert-sorted local
 *   row r is receive-buffer row row_map[r] (feed it to moe_experts as x_rows and
 *   y_rows).  More than max_rows rows sets MOE_STATUS_ROW_OVERFLOW in the status
 *   word at the start of workspace (256 B) and leaves row_map unwritten.
 * Replaces the host-side per-expert bookkeeping of _moe_ffn_g4_gpu
 * (nightmare_stream.py:4400-4449). */
int moe_ep_local_order(const int32_t* recv_counts, int W, int E_local, int max_rows,
                       int32_t* local_offsets, int32_t* row_map, void* workspace,
                       moe_stream_t stream);

/* RMSNorm of moe_forward.rms_norm (moe_forward.py:34-40):
 * out[t] = x[t] / sqrt(mean(x[t]^2) + eps) * weight. */
int moe_rms_norm(const float* x, const float* weight, float eps, int T, int d, float* out,
                 moe_stream_t stream);

/* moe_rms_norm with the reference's gemma_style switch (moe_forward.py:34-40):
 * non-zero gemma_style scales by (1 + weight) instead of weight. */
int moe_rms_norm_ex(const float* x, const float* weight, float eps, int gemma_style, int T, int d,
                    float* out, moe_stream_t stream);

/* ---- whole layer ----------------------------------------------------------------------- */

typedef struct moe_layer_weights {
  const float* gate_w;   /* router weight, layout per router_layout */
  const float* bias;     /* (E,) or NULL */
  const uint8_t* w_gate; /* packed (E, F, d) */
  const uint8_t* w_up;   /* packed (E, F, d) */
  const uint8_t* w_down; /* packed (E, d, F) */
  const uint8_t* s_gate; /* packed shared expert (1, Fs, d) or NULL */
  const uint8_t* s_up;
  const uint8_t* s_down;
  int router_layout;
  int qtype;
  int shared_qtype;
  int E, k, d, F, Fs;
  int mode;
  const moe_expert_opts* opts; /* expert variant, or NULL for the reference's SwiGLU experts;
                                  the shared expert takes its activation only.  Under
                                  expert parallelism down_scale holds the rank's experts */
} moe_layer_weights;

int moe_layer_workspace_bytes(const moe_layer_weights* w, int T, size_t* bytes);

/* MoELayer.forward (moe_forward.py:154-174) for T tokens:
 * router -> dispatch -> grouped experts -> combine (+ shared expert).
 *   x (T, d) f32 in device memory or in pinned (page-locked) host memory: the
 *   router's first pass then reads it over the bus and leaves a device copy in
 *   the workspace for the later kernels (no separate host-to-device copy).
 *   Pageable host memory is rejected (MOE_ERR_INVALID).
 *   out (T, d) f32, device or pinned host memory (written in place by the
 *   combine); must not alias x.
 *   residual (T, d) or NULL: added to the output (the transformer residual,
 *   moe_forward.py:359 `x = x + ffn_out`); may alias out.
 *   ids_out / weights_out (T, k) or NULL: receive the routing decisions.
 * Replaces MoELayer.forward and the GPU engine's _moe_ffn_gpu
 * (nightmare_stream.py:3280-3334) / _moe_ffn_gpu_native
 * (nightmare_gpu_native.py:1542-1590). */
int moe_layer_forward(const moe_layer_weights* w, const float* x, int T, float* out,
                      const float* residual, int32_t* ids_out, float* weights_out,
                      void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* moe_layer_forward whose router reads router_x (T, d) instead of x: gemma4
 * routes a scaled, unweighted RMS of the attention output while its experts
 * read a differently normalised vector (nightmare_stream.py:4659-4674).
 * router_x NULL = x. */
int moe_layer_forward_ex(const moe_layer_weights* w, const float* x, const float* router_x, int T,
                         float* out, const float* residual, int32_t* ids_out, float* weights_out,
                         void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* gemma4's router input (nightmare_stream.py:4662-4667):
 * out[t] = x[t] / sqrt(mean(x[t]^2) + eps) * f32(1 / sqrt(d)) * scale, each
 * product rounded to f32 in that order; scale (d,) f32 (ffn_gate_inp.scale) or
 * NULL. */
int moe_router_input(const float* x, const float* scale, float eps, int T, int d, float* out,
                     moe_stream_t stream);

/* ---- expert parallelism over NVLink peer memory ----------------------------------
 * One process per GPU of a node.  Each rank allocates an exchange window
 * (moe_ipc_alloc, moe_ep_window_bytes), shares its IPC handle with the other
 * ranks (moe_ipc_handle; 64 bytes, exchanged by the caller, e.g. over
 * torch.distributed) and maps theirs (moe_ipc_open).  moe_ep_forward then runs
 * one expert-parallel layer step with no host synchronisation and no collective
 * library: the routed rows are stored straight into the owners' windows, the
 * owners run their experts on them and store the outputs straight back, and
 * release/acquire flags carrying `epoch` (1, 2, 3, ... the same on every rank
 * and step) order each exchange.  Replaces the multi-card MoE of
 * _moe_ffn_g4_gpu (nightmare_stream.py:4381-4449), which uploads the token to
 * every card and sums the per-expert outputs on the host. */
int moe_ipc_alloc(size_t bytes, void** ptr);          /* zeroed device memory */
int moe_ipc_free(void* ptr);
int moe_ipc_handle(void* ptr, void* handle_out);       /* 64-byte IPC handle */
int moe_ipc_open(const void* handle, void** ptr);      /* a peer's window */
int moe_ipc_close(void* ptr);
int moe_ep_window_bytes(int W, int E, int T, int k, int d, size_t* bytes);
/* w: router over all E experts; expert weights of this rank's E / W experts
 * (experts rank * E/W .. (rank+1) * E/W - 1); an optional shared expert runs
 * on this rank's own tokens (replicated weights, no exchange). */
int moe_ep_workspace_bytes(const moe_layer_weights* w, int W, int T, size_t* bytes);
/* peers: device array of the W window pointers (own window at index rank,
 * peers' as mapped by moe_ipc_open); window: this rank's window; x, out (T, d)
 * f32; residual as in moe_layer_forward.  Every rank must call it with the same
 * T and epoch.  Waits on other ranks give up after about a second and set
 * MOE_STATUS_TIMEOUT in the status word at the start of workspace. */
int moe_ep_forward(const moe_layer_weights* w, int W, int rank, void* const* peers, void* window,
                   const float* x, int T, float* out, const float* residual, int epoch,
                   void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* The same step split into its three phases, for a caller that schedules them
 * itself (no counterpart in the reference):
 *   MOE_EP_PHASE_SEND     router, dispatch, rows and counts into the owners' windows
 *   MOE_EP_PHASE_SERVE    wait for every source, experts on the received rows,
 *                         outputs back into the sources' windows (+ shared expert)
 *   MOE_EP_PHASE_COMBINE  wait for every owner, weighted combine into out
 * moe_ep_forward is all three in order.  Phases of one step run in this order
 * on each rank with the same epoch.  When all W ranks live on ONE device (one
 * process driving W windows and workspaces), running a phase for every rank
 * before any rank starts the next phase satisfies each wait from work that
 * has already completed in stream order, so no kernel waits on another that
 * is still to be scheduled. */
enum { MOE_EP_PHASE_SEND = 1, MOE_EP_PHASE_SERVE = 2, MOE_EP_PHASE_COMBINE = 4,
       MOE_EP_PHASE_ALL = 7 };
int moe_ep_forward_phases(const moe_layer_weights* w, int W, int rank, void* const* peers,
                          void* window, const float* x, int T, float* out, const float* residual,
                          int epoch, int phases, void* workspace, size_t workspace_bytes,
                          moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
