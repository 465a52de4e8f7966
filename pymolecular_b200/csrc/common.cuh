// Shared helpers of libegnn_b200: status/error plumbing, launch accounting,
// activations and bf16 rounding.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include <string>

#include "egnn_b200.h"

namespace egnn {

// ---- error plumbing -------------------------------------------------------
void set_error(int code, const char* fmt, ...);
int fail(int code, const char* fmt, ...);
void count_launch(int n = 1);

// While egnn_kernel_timing(1) is on, brackets the kernels launched in its
// lifetime with CUDA events on `s`, filed under `name`.
struct TimerScope {
  TimerScope(const char* name, cudaStream_t s);
  ~TimerScope();
  bool active;
  cudaStream_t stream;
  size_t index = 0;
};

#define EGNN_CHECK_CUDA(expr)                                                   \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess)                                                      \
      return ::egnn::fail(EGNN_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,        \
                          cudaGetErrorString(_e), __FILE__, __LINE__);          \
  } while (0)

#define EGNN_CHECK_LAUNCH()                                                     \
  do {                                                                          \
    ::egnn::count_launch();                                                     \
    cudaError_t _e = cudaGetLastError();                                        \
    if (_e != cudaSuccess)                                                      \
      return ::egnn::fail(EGNN_ERR_CUDA, "kernel launch failed: %s (%s:%d)",    \
                          cudaGetErrorString(_e), __FILE__, __LINE__);          \
  } while (0)

#define EGNN_TRY(expr)                                                          \
  do {                                                                          \
    int _s = (expr);                                                            \
    if (_s != EGNN_OK) return _s;                                               \
  } while (0)

int num_sms_current();
// A 1-D tensor map over n int32 elements at p with boxes of `box` elements
// (TMA loads; elements past n read as zero).  False when p is not 16-byte
// aligned or the driver cannot encode it (callers then load per thread).
bool tensor_map_i32_1d(void* map, const int32_t* p, int64_t n, int box);
// Bit of the current device (for per-device one-time setup flags).
uint64_t device_bit();

// ---- programmatic dependent launch ------------------------------------------
// Kernels on the layer's hot path are launched with launch_pdl: such a kernel
// may start while its predecessor in the stream is still finishing.  It calls
// pdl_enter() before it reads or writes any memory its predecessor writes or
// reads (griddepcontrol.wait returns once the predecessor grid has completed
// and its writes are visible), and only then lets its own successor start, so
// that anything written two or more kernels back is complete whenever a
// kernel runs at all: a prologue may read such data (weights) before its wait.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ---- workspace carving ----------------------------------------------------
// Sub-buffers are 256-byte aligned so every float4 / TMA access is aligned.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
  size_t size() const { return (off + 255) & ~size_t(255); }
};

// ---- device math ----------------------------------------------------------
__device__ __forceinline__ float sigmoidf_(float x) {
  return 1.0f / (1.0f + __expf(-x));
}

// SiLU and its derivative from the same sigmoid:
//   silu(a) = a s,  silu'(a) = s (1 + a (1 - s)),  s = sigmoid(a).
__device__ __forceinline__ float silu_f(float a) { return a * sigmoidf_(a); }

__device__ __forceinline__ void silu_and_grad(float a, float& y, float& dy) {
  float s = sigmoidf_(a);
  y = a * s;
  dy = s * (1.0f + a * (1.0f - s));
}

// Fast variants for the bf16 tensor-core path: approximate exp and divide
// (two MUFU operations, relative error ~1e-7), whose results are rounded to
// bf16 or fp16 downstream anyway.
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_fast(float a) { return a * sigmoid_fast(a); }
__device__ __forceinline__ void silu_grad_fast(float a, float& y, float& dy) {
  const float s = sigmoid_fast(a);
  y = a * s;
  dy = s * (1.0f + a * (1.0f - s));
}

// Per-edge activations of the bf16 tensor-core edge kernels: one MUFU
// operation per sigmoid, sigmoid(x) = 1/2 + tanh(x/2)/2 with the hardware's
// tanh.approx (relative error about 2^-11, a quarter of bf16's half-unit;
// these values are rounded to bf16 or fp16, or summed in fp32 over many
// edges, downstream).
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sigmoid_edge(float x) { return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f); }
__device__ __forceinline__ float silu_edge(float a) { return a * sigmoid_edge(a); }
__device__ __forceinline__ void silu_grad_edge(float a, float& y, float& dy) {
  const float s = sigmoid_edge(a);
  y = a * s;
  dy = s * (1.0f + a * (1.0f - s));
}

// Round-to-nearest-even to the bf16 grid, kept in a float register.
__device__ __forceinline__ float bf16r(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// hi + lo with hi = bf16(v), lo = bf16(v - hi): the value a weight stored as
// a pair of bf16 tiles contributes to a pair of MMAs (exact in fp32).
__device__ __forceinline__ float bf16_split(float v) {
  const float hi = bf16r(v);
  return hi + bf16r(v - hi);
}

template <bool BF>
__device__ __forceinline__ float maybe_bf(float v) {
  if constexpr (BF) return bf16r(v); else return v;
}

}  // namespace egnn
