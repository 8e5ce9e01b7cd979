// Library-level C entry points: version, error strings, block geometry,
// device status word.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "blockfmt.cuh"

namespace moe {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MOE_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return MOE_OK;
}

// Device attribute cache, guarded by a mutex (the only shared mutable state).
static std::mutex g_attr_mu;
static int g_sm_count[64] = {0};

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// ---------------------------------------------------------------------------
// profiler: a pool of event pairs, one per recorded launch
// ---------------------------------------------------------------------------
struct ProfRec {
  cudaEvent_t a = nullptr, b = nullptr;
  int kid = 0;
};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static ProfRec g_prof[8192];
static int g_prof_n = 0;
static thread_local int t_prof_open = -1;

void prof_begin(int kernel_id, cudaStream_t s) {
  if (!g_prof_on) return;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (!g_prof_on || g_prof_n >= 8192) return;
  ProfRec& r = g_prof[g_prof_n];
  if (!r.a) {
    if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return;
  }
  r.kid = kernel_id;
  if (cudaEventRecord(r.a, s) != cudaSuccess) return;
  t_prof_open = g_prof_n++;
}

void prof_end(cudaStream_t s) {
  if (t_prof_open < 0) return;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  cudaEventRecord(g_prof[t_prof_open].b, s);
  t_prof_open = -1;
}

}  // namespace moe

extern "C" {

int moe_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(moe::g_prof_mu);
  moe::g_prof_on = on != 0;
  return MOE_OK;
}

int moe_profile_collect(float* ms, int* launches, int n) {
  MOE_REQUIRE(ms && launches && n > 0, MOE_ERR_INVALID, "null output");
  for (int i = 0; i < n; ++i) {
    ms[i] = 0.f;
    launches[i] = 0;
  }
  std::lock_guard<std::mutex> lock(moe::g_prof_mu);
  for (int i = 0; i < moe::g_prof_n; ++i) {
    moe::ProfRec& r = moe::g_prof[i];
    float t = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess) continue;
    if (cudaEventElapsedTime(&t, r.a, r.b) != cudaSuccess) continue;
    if (r.kid >= 0 && r.kid < n) {
      ms[r.kid] += t;
      launches[r.kid] += 1;
    }
  }
  moe::g_prof_n = 0;
  return MOE_OK;
}


int moe_version(void) { return 1 * 10000 + 0 * 100 + 0; }

int moe_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return MOE_ERR_INVALID;
  strncpy(buf, moe::g_err, len - 1);
  buf[len - 1] = '\0';
  return MOE_OK;
}

int moe_block_geometry(int qtype, int* elems_per_block, int* bytes_per_block) {
  MOE_REQUIRE(elems_per_block && bytes_per_block, MOE_ERR_INVALID, "null output pointer");
  MOE_REQUIRE(moe::blockfmt_ok(qtype), MOE_ERR_UNSUPPORTED, "quant type %d not supported", qtype);
  *elems_per_block = moe::blockfmt_elems(qtype);
  *bytes_per_block = moe::blockfmt_bytes(qtype);
  return MOE_OK;
}

int moe_read_status(const void* workspace, int* status_out, moe_stream_t stream) {
  MOE_REQUIRE(workspace && status_out, MOE_ERR_INVALID, "null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int host = 0;
  MOE_CUDA(cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
  MOE_CUDA(cudaStreamSynchronize(s));
  MOE_CUDA(cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int), s));
  *status_out = host;
  if (host != 0) return moe::fail(MOE_ERR_DEVICE, "device status 0x%x", host);
  return MOE_OK;
}

}  // extern "C"
