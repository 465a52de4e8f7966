// Graph-level regression loss of the training step: per-graph sums of a node
// value (the model's h_out[:, 0]) and their mean squared error against one
// target per graph, forward and backward, deterministic (fixed association
// order everywhere, no atomics).
//
//   pred_g = sum_{i in graph g} v_i          (graphs are contiguous node ranges)
//   loss   = (1 / G) sum_g (pred_g - y_g)^2
//   dL/dv_i = dL/dloss * 2 (pred_g - y_g) / G,   g the graph of node i
//
// Forward, three launches:
//   chunk pass   one block per CHUNK consecutive nodes: a segmented scan over
//                the chunk (segments = runs of one graph) gives each segment's
//                sum in a fixed tree order; a graph that lies inside the chunk
//                gets its pred directly, the chunk's first and last segments,
//                when their graph crosses the chunk's boundary, go to head[c]
//                / tail[c];
//   span pass    one warp per graph that crosses a chunk boundary: tail of its
//                first chunk + heads of the following chunks, lane-strided and
//                tree-reduced in a fixed order;
//   loss pass    one block: the mean of (pred - y)^2 over the graphs.
// Backward: one thread per node, its graph found by binary search in graph_ptr.
//
// graph_ptr (G + 1, int64) is trusted for the results, not for memory safety:
// every offset is clamped to [0, N], so a malformed graph_ptr gives wrong
// sums but never an out-of-range access.
#include <algorithm>

#include "common.cuh"

namespace egnn {
namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 8;
constexpr int kChunk = kThreads * kPerThread;   // nodes per chunk

__device__ __forceinline__ int64_t clamp_ptr(const int64_t* __restrict__ gp, int64_t g, int64_t N) {
  return min(max(gp[g], (int64_t)0), N);
}

// Graph of node i: the g in [0, G) with gp[g] <= i < gp[g + 1] (empty graphs
// are skipped); G - 1 when i is past every offset.
__device__ __forceinline__ int64_t graph_of(const int64_t* __restrict__ gp, int64_t G, int64_t N, int64_t i) {
  int64_t lo = 0, hi = G;   // first u in [1, G] with gp[u] > i, minus one
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (clamp_ptr(gp, mid, N) <= i) lo = mid; else hi = mid - 1;
  }
  return min(lo, G - 1);
}

struct Seg {   // segmented-scan element: a head flag and a running sum
  int f;
  float a;
};
// (f1, a1) then (f2, a2): a segment head in the second part restarts the sum
__device__ __forceinline__ Seg seg_op(Seg x, Seg y) { return Seg{x.f | y.f, y.f ? y.a : x.a + y.a}; }

__global__ void __launch_bounds__(kThreads) graph_sum_chunk_kernel(int64_t N, int64_t G,
                                                                   const float* __restrict__ v, int64_t ld,
                                                                   const int64_t* __restrict__ gp,
                                                                   float* __restrict__ pred, float* __restrict__ head,
                                                                   float* __restrict__ tail) {
  pdl_enter();
  __shared__ int64_t last_key[kThreads];
  __shared__ Seg warp_tot[kThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * kChunk;
  const int64_t cend = min(N, c0 + kChunk);
  const int64_t i0 = c0 + (int64_t)t * kPerThread;

  // keys (graph ids; -1 past N) and values of the thread's nodes
  int64_t key[kPerThread];
  float val[kPerThread];
  {
    int64_t g = i0 < N ? graph_of(gp, G, N, i0) : -1;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int64_t i = i0 + k;
      if (i < N) {
        while (g + 1 < G && clamp_ptr(gp, g + 1, N) <= i) ++g;
        key[k] = g;
        val[k] = v[i * ld];
      } else {
        key[k] = -1;
        val[k] = 0.f;
      }
    }
  }
  last_key[t] = key[kPerThread - 1];
  __syncthreads();
  const int64_t prev_key = t > 0 ? last_key[t - 1] : INT64_MIN;

  // thread-local inclusive segmented scan
  int flag[kPerThread];
  float s[kPerThread];
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    flag[k] = (k == 0 ? key[0] != prev_key : key[k] != key[k - 1]) ? 1 : 0;
    s[k] = (k == 0 || flag[k]) ? val[k] : s[k - 1] + val[k];
  }
  Seg mine{0, s[kPerThread - 1]};
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) mine.f |= flag[k];

  // exclusive scan of the thread summaries: warp shuffles, then warp totals
  Seg inc = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    Seg o{__shfl_up_sync(0xffffffffu, inc.f, d), __shfl_up_sync(0xffffffffu, inc.a, d)};
    if (lane >= d) inc = seg_op(o, inc);
  }
  if (lane == 31) warp_tot[warp] = inc;
  Seg exc{__shfl_up_sync(0xffffffffu, inc.f, 1), __shfl_up_sync(0xffffffffu, inc.a, 1)};
  bool have = lane > 0;   // exc holds the lanes before this one
  __syncthreads();
  Seg wpre{0, 0.f};
  bool wpre_have = false;
  for (int w = 0; w < warp; ++w) {   // the warps before this one, in order
    wpre = wpre_have ? seg_op(wpre, warp_tot[w]) : warp_tot[w];
    wpre_have = true;
  }
  Seg pre{0, 0.f};
  bool pre_have = false;
  if (wpre_have && have) { pre = seg_op(wpre, exc); pre_have = true; }
  else if (wpre_have) { pre = wpre; pre_have = true; }
  else if (have) { pre = exc; pre_have = true; }

  // segment ends: the next node is in another graph, or the chunk ends
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int64_t i = i0 + k;
    if (i >= cend || key[k] < 0) continue;
    bool head_seen = false;   // a head at or before k inside this thread
#pragma unroll
    for (int q = 0; q <= k; ++q) head_seen |= flag[q] != 0;
    const float total = (!head_seen && pre_have) ? pre.a + s[k] : s[k];
    const int64_t next_key = (k + 1 < kPerThread) ? key[k + 1] : (i + 1 < cend ? graph_of(gp, G, N, i + 1) : -2);
    if (next_key == key[k]) continue;
    const int64_t g = key[k];
    const bool before = clamp_ptr(gp, g, N) < c0;
    const bool after = clamp_ptr(gp, g + 1, N) > cend;
    if (before) head[blockIdx.x] = total;
    else if (after) tail[blockIdx.x] = total;
    else pred[g] = total;
  }
}

__global__ void __launch_bounds__(256) graph_sum_span_kernel(int64_t N, int64_t G, const int64_t* __restrict__ gp,
                                                             const float* __restrict__ head,
                                                             const float* __restrict__ tail,
                                                             float* __restrict__ pred) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (g >= G) return;
  const int64_t s = clamp_ptr(gp, g, N), e = max(s, clamp_ptr(gp, g + 1, N));
  if (e == s) {
    if (lane == 0) pred[g] = 0.f;
    return;
  }
  const int64_t c0 = s / kChunk, c1 = (e - 1) / kChunk;
  if (c0 == c1) return;   // inside one chunk: written by the chunk pass
  float a = lane == 0 ? tail[c0] : 0.f;
  for (int64_t c = c0 + 1 + lane; c <= c1; c += 32) a += head[c];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) a += __shfl_xor_sync(0xffffffffu, a, d);
  if (lane == 0) pred[g] = a;
}

__global__ void __launch_bounds__(1024) graph_mse_loss_kernel(int64_t G, const float* __restrict__ pred,
                                                              const float* __restrict__ y, float* __restrict__ loss) {
  pdl_enter();
  __shared__ float red[1024];
  const int t = threadIdx.x;
  float a = 0.f;
  for (int64_t g = t; g < G; g += 1024) {
    const float d = pred[g] - y[g];
    a = fmaf(d, d, a);
  }
  red[t] = a;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if (t < w) red[t] += red[t + w];
    __syncthreads();
  }
  if (t == 0) *loss = red[0] / (float)G;   // G = 0: 0 / 0, as the mean of nothing
}

__global__ void __launch_bounds__(256) graph_mse_bwd_kernel(int64_t N, int64_t G, const int64_t* __restrict__ gp,
                                                            const float* __restrict__ pred,
                                                            const float* __restrict__ y,
                                                            const float* __restrict__ gloss,
                                                            float* __restrict__ grad, int64_t ld) {
  pdl_enter();
  const float sc = 2.f * gloss[0] / (float)G;
  const int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i0 >= N) return;
  int64_t g = graph_of(gp, G, N, i0);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t i = i0 + k;
    if (i >= N) break;
    while (g + 1 < G && clamp_ptr(gp, g + 1, N) <= i) ++g;
    grad[i * ld] = sc * (pred[g] - y[g]);
  }
}

int64_t n_chunks(int64_t N) { return std::max<int64_t>(1, (N + kChunk - 1) / kChunk); }

}  // namespace
}  // namespace egnn

using namespace egnn;

extern "C" size_t egnn_graph_mse_workspace_size(int64_t n_nodes) {
  Carver c(nullptr);
  c.take<float>((size_t)n_chunks(std::max<int64_t>(n_nodes, 0)));
  c.take<float>((size_t)n_chunks(std::max<int64_t>(n_nodes, 0)));
  return c.size();
}

extern "C" int egnn_graph_mse_fwd(int64_t n_nodes, int64_t n_graphs, const float* values, int64_t ld,
                                  const int64_t* graph_ptr, const float* target, float* pred, float* loss,
                                  void* ws, size_t ws_bytes, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n_nodes < 0 || n_graphs < 0 || ld < 1) return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_fwd: bad shape");
  if (!graph_ptr || !loss || (n_graphs > 0 && (!target || !pred)) || (n_nodes > 0 && !values))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_fwd: null pointer");
  if (n_nodes > 0 && n_graphs == 0)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_fwd: nodes without graphs");
  if (!ws || ws_bytes < egnn_graph_mse_workspace_size(n_nodes))
    return fail(EGNN_ERR_WORKSPACE, "egnn_graph_mse_fwd: workspace too small");
  Carver c(ws);
  float* head = c.take<float>((size_t)n_chunks(n_nodes));
  float* tail = c.take<float>((size_t)n_chunks(n_nodes));
  TimerScope ts("graph_mse", s);
  if (n_nodes > 0) {
    EGNN_CHECK_CUDA(launch_pdl(graph_sum_chunk_kernel, dim3((unsigned)n_chunks(n_nodes)), dim3(kThreads), 0, s,
                               n_nodes, n_graphs, values, ld, graph_ptr, pred, head, tail));
    EGNN_CHECK_LAUNCH();
  }
  if (n_graphs > 0) {
    EGNN_CHECK_CUDA(launch_pdl(graph_sum_span_kernel, dim3((unsigned)((n_graphs + 7) / 8)), dim3(256), 0, s, n_nodes,
                               n_graphs, graph_ptr, (const float*)head, (const float*)tail, pred));
    EGNN_CHECK_LAUNCH();
  }
  EGNN_CHECK_CUDA(launch_pdl(graph_mse_loss_kernel, dim3(1), dim3(1024), 0, s, n_graphs, (const float*)pred, target,
                             loss));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

extern "C" int egnn_graph_mse_bwd(int64_t n_nodes, int64_t n_graphs, const int64_t* graph_ptr, const float* pred,
                                  const float* target, const float* grad_loss, float* grad_values, int64_t ld,
                                  void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n_nodes < 0 || n_graphs < 0 || ld < 1) return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_bwd: bad shape");
  if (n_nodes == 0) return EGNN_OK;
  if (n_graphs == 0) return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_bwd: nodes without graphs");
  if (!graph_ptr || !pred || !target || !grad_loss || !grad_values)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_mse_bwd: null pointer");
  const int64_t threads = (n_nodes + 3) / 4;
  TimerScope ts("graph_mse", s);
  EGNN_CHECK_CUDA(launch_pdl(graph_mse_bwd_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, s, n_nodes,
                             n_graphs, graph_ptr, pred, target, grad_loss, grad_values, ld));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}
