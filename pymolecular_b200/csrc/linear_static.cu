// egnn_linear_bwd_static: the embedding-layer backward for callers that
// cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they need the
// backward: a plugin whose host framework owns all device memory and offers
// it no workspace, or host code that must not add a synchronising allocation
// to a latency-critical path.  This entry point gives them the same
// computation as egnn_linear_bwd with its split-K scratch taken from a fixed
// array compiled into the library.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace egnn {
namespace {

constexpr size_t kScratchFloats = EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// One copy per device that loads the library; lives until the process exits.
static __device__ __align__(256) float g_linear_bwd_scratch[kScratchFloats];

std::mutex g_addr_mu;
// Device address of the array per CUDA context: a cudaDeviceReset, or a
// caller that makes a different (non-primary) context current, gets a fresh
// lookup instead of a stale address.
CUcontext g_scratch_ctx[kMaxDevices] = {};
float* g_scratch_addr[kMaxDevices] = {};

// Device address of g_linear_bwd_scratch on the current device.  The host
// symbol is only a stand-in for the array, so the address is looked up with
// that device (and context) current, once per context.
// The driver's cuCtxGetCurrent, found through the runtime (the library does
// not link the driver library itself).
CUresult current_context(CUcontext* ctx) {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return CUDA_ERROR_NOT_FOUND;
    fn = reinterpret_cast<Fn>(p);
  }
  return fn(ctx);
}

int scratch_address(float** out) {
  int dev = 0;
  EGNN_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_bwd_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_addr_mu);
  CUcontext ctx = nullptr;
  if (current_context(&ctx) != CUDA_SUCCESS)
    return fail(EGNN_ERR_CUDA, "egnn_linear_bwd_static: cuCtxGetCurrent unavailable");
  if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
    // the lookup itself makes the device's primary context current if no
    // context was
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_linear_bwd_scratch);
    if (e != cudaSuccess || !p)
      return fail(EGNN_ERR_CUDA, "egnn_linear_bwd_static: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    if (!ctx && (current_context(&ctx) != CUDA_SUCCESS || !ctx))
      return fail(EGNN_ERR_CUDA, "egnn_linear_bwd_static: no current CUDA context");
    g_scratch_addr[dev] = static_cast<float*>(p);
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return EGNN_OK;
}

}  // namespace
}  // namespace egnn

extern "C" int egnn_linear_bwd_static(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                                      const float* dy, float* dx, float* dw, float* db, void* stream) {
  using namespace egnn;
  if (m < 0 || k <= 0 || o <= 0) return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_bwd_static: bad shape");
  const size_t need = egnn_linear_workspace_size(m, k, o);
  if (need > EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES)
    return fail(EGNN_ERR_WORKSPACE,
                "egnn_linear_bwd_static: shape (m=%lld, k=%d, o=%d) needs %zu scratch bytes, the static "
                "array holds %zu; use egnn_linear_bwd with a workspace",
                (long long)m, k, o, need, (size_t)EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES);
  float* scratch = nullptr;
  EGNN_TRY(scratch_address(&scratch));
  return egnn_linear_bwd(m, k, o, x, w, dy, dx, dw, db, scratch, EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES,
                         stream);
}
