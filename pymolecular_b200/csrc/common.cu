// Error plumbing, launch accounting and device queries of libegnn_b200.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>

#include "common.cuh"

namespace egnn {

namespace {
thread_local char g_err[1024] = "";
std::atomic<uint64_t> g_launches{0};

// Opt-in kernel timer: CUDA events recorded on the launching stream around
// the named kernels while enabled.
struct TimedLaunch {
  std::string name;
  cudaEvent_t start, stop;
};
std::mutex g_timer_mu;
std::atomic<int> g_timer_on{0};
std::vector<TimedLaunch> g_timed;

void clear_timed_locked() {
  for (auto& t : g_timed) {
    cudaEventDestroy(t.start);
    cudaEventDestroy(t.stop);
  }
  g_timed.clear();
}
}  // namespace

TimerScope::TimerScope(const char* name, cudaStream_t s) : active(false), stream(s) {
  if (!g_timer_on.load(std::memory_order_relaxed)) return;
  TimedLaunch t{name, nullptr, nullptr};
  if (cudaEventCreate(&t.start) != cudaSuccess) return;
  if (cudaEventCreate(&t.stop) != cudaSuccess) { cudaEventDestroy(t.start); return; }
  cudaEventRecord(t.start, s);
  std::lock_guard<std::mutex> lk(g_timer_mu);
  g_timed.push_back(t);
  index = g_timed.size() - 1;
  active = true;
}

TimerScope::~TimerScope() {
  if (!active) return;
  std::lock_guard<std::mutex> lk(g_timer_mu);
  if (index < g_timed.size()) cudaEventRecord(g_timed[index].stop, stream);
}

void set_error(int code, const char* fmt, ...) {
  char msg[900];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  snprintf(g_err, sizeof(g_err), "[egnn status %d] %s", code, msg);
}

int fail(int code, const char* fmt, ...) {
  char msg[900];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  snprintf(g_err, sizeof(g_err), "[egnn status %d] %s", code, msg);
  return code;
}

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int num_sms_current() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n > 0 ? n : 148;
}

uint64_t device_bit() {
  int dev = 0;
  cudaGetDevice(&dev);
  return uint64_t(1) << (dev & 63);
}

}  // namespace egnn

extern "C" size_t egnn_last_error(char* buf, size_t len) {
  size_t n = strlen(egnn::g_err);
  if (buf && len) {
    size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, egnn::g_err, c);
    buf[c] = 0;
  }
  return n;
}

extern "C" const char* egnn_version(void) { return "egnn_b200 0.1 sm_100a"; }

extern "C" uint64_t egnn_launch_count(void) { return egnn::g_launches.load(); }

extern "C" void egnn_launch_count_reset(void) { egnn::g_launches.store(0); }

extern "C" void egnn_kernel_timing(int enable) {
  std::lock_guard<std::mutex> lk(egnn::g_timer_mu);
  egnn::clear_timed_locked();
  egnn::g_timer_on.store(enable ? 1 : 0);
}

extern "C" int egnn_kernel_time(const char* name, double* total_ms, int64_t* launches) {
  if (!name || !total_ms || !launches)
    return egnn::fail(EGNN_ERR_INVALID_ARG, "egnn_kernel_time: null argument");
  std::lock_guard<std::mutex> lk(egnn::g_timer_mu);
  double tot = 0.0;
  int64_t n = 0;
  for (auto& t : egnn::g_timed) {
    if (t.name != name) continue;
    cudaError_t e = cudaEventSynchronize(t.stop);
    if (e != cudaSuccess) return egnn::fail(EGNN_ERR_CUDA, "event sync: %s", cudaGetErrorString(e));
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, t.start, t.stop);
    if (e != cudaSuccess) return egnn::fail(EGNN_ERR_CUDA, "elapsed time: %s", cudaGetErrorString(e));
    tot += ms;
    ++n;
  }
  *total_ms = tot;
  *launches = n;
  return EGNN_OK;
}

namespace egnn {

bool tensor_map_i32_1d(void* map, const int32_t* p, int64_t n, int box) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static std::atomic<Encode> encode{nullptr};
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode.store(reinterpret_cast<Encode>(fn));
  });
  Encode f = encode.load();
  if (!f || !p || n <= 0 || (reinterpret_cast<uintptr_t>(p) & 15u)) return false;
  const cuuint64_t dim[1] = {(cuuint64_t)n};
  const cuuint64_t stride[1] = {(cuuint64_t)n * 4};   // not read for rank 1
  const cuuint32_t boxd[1] = {(cuuint32_t)box};
  const cuuint32_t estr[1] = {1};
  return f(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_INT32, 1, const_cast<int32_t*>(p), dim, stride,
           boxd, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace egnn
