// Error reporting and version for the C ABI (include/laguna_b200.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace lg {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<long long> g_launches{0};
static thread_local char g_stage[32] = "";
static thread_local cudaEvent_t g_ev0 = nullptr, g_ev1 = nullptr;

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static std::atomic<int> g_pdl{0};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int device_sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return 148;
  }
  int c = cached[dev].load(std::memory_order_relaxed);
  if (c <= 0) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) {
      (void)cudaGetLastError();
      c = 148;
    }
    cached[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

// Inside a stream capture the record becomes a graph node that timestamps on every replay
// (an "external" event record); outside it is an ordinary record.
static void prof_record(cudaEvent_t ev, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, s);
}

void prof_begin(const char* stage, cudaStream_t s) {
  if (g_ev0 && std::strcmp(stage, g_stage) == 0) prof_record(g_ev0, s);
}

void prof_end(const char* stage, cudaStream_t s) {
  if (g_ev1 && std::strcmp(stage, g_stage) == 0) prof_record(g_ev1, s);
}

}  // namespace lg

extern "C" long long lg_launch_count(void) { return lg::g_launches.load(); }

extern "C" int lg_set_pdl(int on) {
  const int prev = lg::g_pdl.exchange(on ? 1 : 0);
  return prev;
}

extern "C" int lg_profile_stage(const char* stage, void* ev_start, void* ev_end) {
  if (!stage || !ev_start || !ev_end) {
    lg::g_stage[0] = 0;
    lg::g_ev0 = lg::g_ev1 = nullptr;
    return LG_OK;
  }
  std::snprintf(lg::g_stage, sizeof(lg::g_stage), "%s", stage);
  lg::g_ev0 = static_cast<cudaEvent_t>(ev_start);
  lg::g_ev1 = static_cast<cudaEvent_t>(ev_end);
  return LG_OK;
}

extern "C" int lg_event_elapsed_ms(void* ev_start, void* ev_end, float* ms) {
  if (!ev_start || !ev_end || !ms) return lg::fail(LG_ERR_INVALID, "event_elapsed: NULL");
  cudaError_t e = cudaEventSynchronize(static_cast<cudaEvent_t>(ev_end));
  if (e == cudaSuccess)
    e = cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(ev_start), static_cast<cudaEvent_t>(ev_end));
  if (e != cudaSuccess) return lg::fail(LG_ERR_CUDA, "event_elapsed: %s", cudaGetErrorString(e));
  return LG_OK;
}

extern "C" int lg_abi_version(void) { return 2; }

extern "C" const char* lg_last_error(void) { return lg::g_err; }
