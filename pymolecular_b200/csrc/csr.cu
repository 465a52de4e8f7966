// Graph construction: edge list -> destination-sorted CSR, its transpose,
// and validation of caller-supplied CSRs.
//
// Reference convention: edges (row, col) with aggregation over row
// (egnn_clean.py:61-62, 76-78); the reference kernels take the CSR triple
// row_ptrs / col_indices / edge_id (forward_kernel.py:18-21) built on the
// host (test_mem.py:62-65).  Here it is built on the device with a stable
// radix sort, so the CSR order equals torch.sort(row, stable=True).
#include <algorithm>
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace egnn {
namespace {

__global__ void validate_edges_kernel(int64_t E, int64_t N, const int64_t* row, const int64_t* col,
                                      int32_t* key, int32_t* val, int* err) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = row[e], c = col[e];
    bool ok = r >= 0 && r < N && c >= 0 && c < N;
    if (!ok) atomicOr(err, 1);
    key[e] = ok ? (int32_t)r : 0;
    val[e] = (int32_t)e;
  }
}

// out_ptr[r] = first position p with sorted_key[p] >= r (lower bound).
__global__ void segment_ptr_kernel(int64_t N, int64_t E, const int32_t* sorted_key, int32_t* ptr) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= N;
       r += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = E;
    while (lo < hi) {
      int64_t mid = (lo + hi) >> 1;
      if (sorted_key[mid] < r) lo = mid + 1; else hi = mid;
    }
    ptr[r] = (int32_t)lo;
  }
}

// Out-of-range sources (already flagged) become node 0, so that a CSR whose
// flag has not been read yet never sends a later kernel out of bounds.
__global__ void gather_cols_kernel(int64_t E, int64_t N, const int64_t* col, const int32_t* perm,
                                   int32_t* col_idx) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < E;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = col[perm[k]];
    col_idx[k] = (c >= 0 && c < N) ? (int32_t)c : 0;
  }
}

__global__ void iota_kernel(int64_t E, int32_t* v) {
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < E;
       k += (int64_t)gridDim.x * blockDim.x)
    v[k] = (int32_t)k;
}

__global__ void check_graph_kernel(int64_t N, int64_t E, egnn_graph g, int* err) {
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (tid == 0) {
    if (g.row_ptr[0] != 0 || g.row_ptr[N] != E) atomicOr(err, 1);
    if (g.src_ptr && (g.src_ptr[0] != 0 || g.src_ptr[N] != E)) atomicOr(err, 1);
  }
  for (int64_t r = tid; r < N; r += stride) {
    int32_t a = g.row_ptr[r], b = g.row_ptr[r + 1];
    if (a > b || a < 0 || b > E) { atomicOr(err, 2); continue; }
    if (g.src_ptr && (g.src_ptr[r] > g.src_ptr[r + 1])) atomicOr(err, 2);
  }
  for (int64_t k = tid; k < E; k += stride) {
    int32_t c = g.col_idx[k];
    if (c < 0 || c >= N) atomicOr(err, 4);
    if (g.row_idx) {
      int32_t r = g.row_idx[k];
      if (r < 0 || r >= N) { atomicOr(err, 4); }
      else if (!(g.row_ptr[r] <= k && k < g.row_ptr[r + 1])) atomicOr(err, 8);
    }
    if (g.edge_id) {
      int32_t id = g.edge_id[k];
      if (id < 0 || id >= E) atomicOr(err, 16);
    }
    if (g.src_edge) {
      int32_t p = g.src_edge[k];
      if (p < 0 || p >= E) atomicOr(err, 32);
    }
  }
}

int grid_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4096)); }

int end_bit_for(int64_t n) {
  int b = 1;
  while (b < 31 && (int64_t(1) << b) <= n) ++b;
  return b;
}

size_t cub_bytes(int64_t E, int64_t N) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs<int32_t, int32_t>(nullptr, bytes, (const int32_t*)nullptr,
                                                    (int32_t*)nullptr, (const int32_t*)nullptr,
                                                    (int32_t*)nullptr, (int)std::max<int64_t>(E, 1),
                                                    0, end_bit_for(N));
  return bytes;
}

}  // namespace
}  // namespace egnn

using namespace egnn;

extern "C" size_t egnn_csr_workspace_size(int64_t n_nodes, int64_t n_edges) {
  Carver c(nullptr);
  c.take<int>(4);
  c.take<int32_t>(n_edges);  // keys in
  c.take<int32_t>(n_edges);  // vals in
  c.take<int32_t>(n_edges);  // sorted keys
  c.take<int32_t>(n_edges);  // sorted vals
  c.take<char>(cub_bytes(n_edges, n_nodes));
  return c.size();
}

namespace egnn {
namespace {

// Shared body of egnn_csr_build (flag in the workspace, read back) and
// egnn_csr_build_async (flag in caller memory, left on the device).
int csr_build(int64_t N, int64_t E, const int64_t* row, const int64_t* col, int32_t* row_ptr,
              int32_t* col_idx, int32_t* row_idx, int32_t* edge_id, void* ws, size_t ws_bytes,
              int32_t* status, cudaStream_t s) {
  if (N < 0 || E < 0 || N >= INT32_MAX || E >= INT32_MAX)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_csr_build: sizes out of range (N=%lld, E=%lld)",
                (long long)N, (long long)E);
  if (!row_ptr || (E > 0 && (!row || !col || !col_idx || !row_idx || !edge_id)))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_csr_build: null pointer");
  if (ws_bytes < egnn_csr_workspace_size(N, E) || !ws)
    return fail(EGNN_ERR_WORKSPACE, "egnn_csr_build: workspace too small");
  Carver c(ws);
  int* ws_err = c.take<int>(4);
  int* err = status ? reinterpret_cast<int*>(status) : ws_err;
  int32_t* kin = c.take<int32_t>(E);
  int32_t* vin = c.take<int32_t>(E);
  int32_t* kout = c.take<int32_t>(E);
  int32_t* vout = c.take<int32_t>(E);
  size_t cb = cub_bytes(E, N);
  void* ctmp = c.take<char>(cb);
  EGNN_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  if (E > 0) {
    validate_edges_kernel<<<grid_for(E), 256, 0, s>>>(E, N, row, col, kin, vin, err);
    EGNN_CHECK_LAUNCH();
    EGNN_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(ctmp, cb, kin, kout, vin, vout, (int)E, 0,
                                                    end_bit_for(N), s));
    count_launch();
    gather_cols_kernel<<<grid_for(E), 256, 0, s>>>(E, N, col, vout, col_idx);
    EGNN_CHECK_LAUNCH();
    EGNN_CHECK_CUDA(cudaMemcpyAsync(row_idx, kout, E * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    EGNN_CHECK_CUDA(cudaMemcpyAsync(edge_id, vout, E * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  }
  segment_ptr_kernel<<<grid_for(N + 1), 256, 0, s>>>(N, E, kout, row_ptr);
  EGNN_CHECK_LAUNCH();
  if (status) return EGNN_OK;
  int herr = 0;
  EGNN_CHECK_CUDA(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  EGNN_CHECK_CUDA(cudaStreamSynchronize(s));
  if (herr) return fail(EGNN_ERR_INDEX, "egnn_csr_build: edge index outside [0, %lld)", (long long)N);
  return EGNN_OK;
}

}  // namespace
}  // namespace egnn

extern "C" int egnn_csr_build(int64_t N, int64_t E, const int64_t* row, const int64_t* col,
                              int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx,
                              int32_t* edge_id, void* ws, size_t ws_bytes, void* stream) {
  return csr_build(N, E, row, col, row_ptr, col_idx, row_idx, edge_id, ws, ws_bytes, nullptr,
                   (cudaStream_t)stream);
}

extern "C" int egnn_csr_build_async(int64_t N, int64_t E, const int64_t* row, const int64_t* col,
                                    int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx,
                                    int32_t* edge_id, int32_t* status, void* ws, size_t ws_bytes,
                                    void* stream) {
  if (!status) return fail(EGNN_ERR_INVALID_ARG, "egnn_csr_build_async: null status");
  return csr_build(N, E, row, col, row_ptr, col_idx, row_idx, edge_id, ws, ws_bytes, status,
                   (cudaStream_t)stream);
}

extern "C" int egnn_csr_transpose(int64_t N, int64_t E, const int32_t* row_ptr, const int32_t* col_idx,
                                  int32_t* src_ptr, int32_t* src_edge, void* ws, size_t ws_bytes,
                                  void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (N < 0 || E < 0 || N >= INT32_MAX || E >= INT32_MAX)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_csr_transpose: sizes out of range");
  if (!src_ptr || (E > 0 && (!col_idx || !src_edge)))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_csr_transpose: null pointer");
  if (ws_bytes < egnn_csr_workspace_size(N, E) || !ws)
    return fail(EGNN_ERR_WORKSPACE, "egnn_csr_transpose: workspace too small");
  (void)row_ptr;
  Carver c(ws);
  c.take<int>(4);
  c.take<int32_t>(E);
  int32_t* vin = c.take<int32_t>(E);
  int32_t* kout = c.take<int32_t>(E);
  c.take<int32_t>(E);
  size_t cb = cub_bytes(E, N);
  void* ctmp = c.take<char>(cb);
  if (E > 0) {
    iota_kernel<<<grid_for(E), 256, 0, s>>>(E, vin);
    EGNN_CHECK_LAUNCH();
    EGNN_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(ctmp, cb, col_idx, kout, vin, src_edge, (int)E,
                                                    0, end_bit_for(N), s));
    count_launch();
  }
  segment_ptr_kernel<<<grid_for(N + 1), 256, 0, s>>>(N, E, kout, src_ptr);
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

extern "C" int egnn_graph_check(int64_t N, int64_t E, const egnn_graph* g, void* ws, size_t ws_bytes,
                                void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!g || !g->row_ptr || (E > 0 && !g->col_idx))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_check: null pointer");
  if (N < 0 || E < 0 || N >= INT32_MAX || E >= INT32_MAX)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_graph_check: sizes out of range");
  if (!ws || ws_bytes < 256) return fail(EGNN_ERR_WORKSPACE, "egnn_graph_check: workspace too small");
  int* err = static_cast<int*>(ws);
  EGNN_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  check_graph_kernel<<<grid_for(std::max(N, E) + 1), 256, 0, s>>>(N, E, *g, err);
  EGNN_CHECK_LAUNCH();
  int herr = 0;
  EGNN_CHECK_CUDA(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  EGNN_CHECK_CUDA(cudaStreamSynchronize(s));
  if (herr) return fail(EGNN_ERR_INDEX, "egnn_graph_check: malformed CSR (code %d)", herr);
  return EGNN_OK;
}
