/*
 * egnn_b200.h — C ABI of libegnn_b200.so, the B200 (sm_100a) EGNN layer.
 *
 * The library replaces the E(n)-equivariant graph convolution of
 * SatxaFortuny/PyMolecular, models/EGNN/egnn_clean.py:
 *   E_GCL.forward            egnn_clean.py:95-103   -> egnn_layer_fwd
 *   autograd of E_GCL         (implied by :49-103)   -> egnn_layer_bwd
 *   unsorted_segment_sum/mean egnn_clean.py:149-164  -> fused into both
 *   edge list -> dst CSR      egnn_clean.py:167-191, forward_kernel.py:19-21
 *                                                    -> egnn_csr_build
 *   get_edges_batch           egnn_clean.py:167-191  -> egnn_fc_graph
 *   radius / kNN graphs and Morton order of the workloads
 *                                                    -> egnn_spatial_*, egnn_morton_order
 * and the reference's fused-kernel entry points, which take the same CSR
 * triple (row_ptr, col_indices, edge_id):
 *   egnn_forward_kernel_node_parallel   forward_kernel.py:13-43
 *   egnn_backward_kernel_node_parallel  backward_kernel.py:13-50
 *
 * Conventions
 *  - Every pointer except descriptors is a DEVICE pointer of the current
 *    device.  `stream` is a cudaStream_t passed as void* (NULL = legacy
 *    default stream).  All calls are asynchronous on `stream` unless noted.
 *  - The library allocates no device memory: callers pass `workspace` of at
 *    least the size the matching *_workspace_size function returns.
 *  - Edges are (row, col) = (destination i, source j), as in egnn_clean.py:85-86.
 *    Aggregation runs over rows.  CSR order = stable sort of the edges by row.
 *  - Tensors are dense row-major float32: h (N,H), x (N,3), edge_attr (E_in,d)
 *    indexed by the ORIGINAL edge id.  Parameters use nn.Linear layout
 *    W (out,in) row-major, b (out).
 *  - Return value: EGNN_OK or an egnn_status code; egnn_last_error() gives a
 *    message for the calling thread.
 */
#ifndef EGNN_B200_H
#define EGNN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EGNN_API __attribute__((visibility("default")))
#else
#define EGNN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  EGNN_OK = 0,
  EGNN_ERR_INVALID_ARG = 1,   /* null pointer, bad size, unsupported shape */
  EGNN_ERR_INDEX = 2,         /* CSR / edge index out of range, row_ptr not monotone */
  EGNN_ERR_CUDA = 3,          /* a CUDA runtime call failed */
  EGNN_ERR_UNSUPPORTED = 4,   /* flag / size combination not built */
  EGNN_ERR_WORKSPACE = 5      /* workspace too small */
} egnn_status;

/* Layer flags: the E_GCL constructor switches (egnn_clean.py:11). */
enum {
  EGNN_FLAG_RESIDUAL = 1,     /* residual=True   (egnn_clean.py:68-69) */
  EGNN_FLAG_ATTENTION = 2,    /* attention=True  (egnn_clean.py:44-47, 55-57) */
  EGNN_FLAG_NORMALIZE = 4,    /* normalize=True  (egnn_clean.py:89-91) */
  EGNN_FLAG_TANH = 8,         /* tanh=True       (egnn_clean.py:40-41) */
  EGNN_FLAG_COORDS_SUM = 16   /* coords_agg='sum' instead of 'mean' (egnn_clean.py:75-78) */
};

/* GEMM input precision. Accumulation and coordinates are always float32. */
enum { EGNN_PREC_FP32 = 0, EGNN_PREC_BF16 = 1 };

/* E_GCL(input_nf = I, output_nf = O, hidden_nf = H, edges_in_d = d)
 * (egnn_clean.py:11-47).  EGNN builds every layer with I = O = H
 * (egnn_clean.py:136); I and O may differ from H (0 means H), and the
 * residual (h' = h + ...) needs I = O. */
typedef struct {
  int64_t n_nodes;        /* N */
  int64_t n_edges;        /* E (< 2^31) */
  int32_t hidden;         /* H = hidden_nf: 32, 64, 128 or 256 */
  int32_t edge_attr_dim;  /* edges_in_d (0..16) */
  int32_t flags;          /* EGNN_FLAG_* */
  int32_t precision;      /* EGNN_PREC_* */
  int32_t in_dim;         /* I = input_nf, columns of h (1..1024; 0 = H) */
  int32_t out_dim;        /* O = output_nf, columns of h_out (1..1024; 0 = H) */
} egnn_layer_desc;

/* A destination-sorted CSR and its transpose (built by egnn_csr_build /
 * egnn_csr_transpose).  Positions k in [0,E) are CSR positions. */
typedef struct {
  const int32_t* row_ptr;   /* (N+1) edge offsets of each destination row */
  const int32_t* col_idx;   /* (E) source node of CSR edge k */
  const int32_t* row_idx;   /* (E) destination node of CSR edge k */
  const int32_t* edge_id;   /* (E) original edge index of CSR edge k (edge_attr row) */
  const int32_t* src_ptr;   /* (N+1) offsets of each source node in src order */
  const int32_t* src_edge;  /* (E) CSR position of the k-th edge in src order */
} egnn_graph;

/* Parameters of one E_GCL (nn.Linear layout, float32). */
typedef struct {
  const float* edge_w1;  const float* edge_b1;   /* edge_mlp.0: (H, 2I+1+d), (H) */
  const float* edge_w2;  const float* edge_b2;   /* edge_mlp.2: (H, H), (H)      */
  const float* node_w1;  const float* node_b1;   /* node_mlp.0: (H, I+H), (H)    */
  const float* node_w2;  const float* node_b2;   /* node_mlp.2: (O, H), (O)      */
  const float* coord_w1; const float* coord_b1;  /* coord_mlp.0: (H, H), (H)     */
  const float* coord_w2;                         /* coord_mlp.2: (1, H), no bias */
  const float* att_w;    const float* att_b;     /* att_mlp.0: (1, H), (1); attention only */
} egnn_layer_params;

/* Gradient outputs, same shapes as egnn_layer_params; overwritten (not
 * accumulated).  att_* may be NULL when attention is off. */
typedef struct {
  float* edge_w1;  float* edge_b1;
  float* edge_w2;  float* edge_b2;
  float* node_w1;  float* node_b1;
  float* node_w2;  float* node_b2;
  float* coord_w1; float* coord_b1;
  float* coord_w2;
  float* att_w;    float* att_b;
} egnn_layer_grads;

enum { EGNN_WS_FWD = 0, EGNN_WS_BWD = 1 };

/* ---- graph construction ------------------------------------------------ */

/* Scratch bytes egnn_csr_build / egnn_csr_transpose need. */
EGNN_API size_t egnn_csr_workspace_size(int64_t n_nodes, int64_t n_edges);

/* Stable sort of the edge list (row, col) (int64, length E) by row into a
 * dst CSR: row_ptr (N+1), col_idx, row_idx, edge_id (E).  Validates every
 * index; returns EGNN_ERR_INDEX on a row/col outside [0,N).  Synchronises
 * `stream` (reads back the validation flag).  Replaces the host-side CSR of
 * test_mem.py:62-65 / datasets_loaders.py:7-11. */
EGNN_API int egnn_csr_build(int64_t n_nodes, int64_t n_edges, const int64_t* row, const int64_t* col,
                   int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx, int32_t* edge_id,
                   void* workspace, size_t workspace_bytes, void* stream);

/* egnn_csr_build without the host read-back: the validation result goes to
 * `status` (device int32; 0 = every index in range, nonzero = an edge index
 * outside [0,N), in which case the CSR content is unspecified) and the call
 * stays asynchronous, so it can be captured in a CUDA graph.  The caller
 * reads `status` before trusting the CSR. */
EGNN_API int egnn_csr_build_async(int64_t n_nodes, int64_t n_edges, const int64_t* row, const int64_t* col,
                                  int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx, int32_t* edge_id,
                                  int32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/* Transpose of a dst CSR: for each source node, the CSR positions of its
 * out-edges in increasing position order.  Asynchronous. */
EGNN_API int egnn_csr_transpose(int64_t n_nodes, int64_t n_edges, const int32_t* row_ptr,
                       const int32_t* col_idx, int32_t* src_ptr, int32_t* src_edge,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Checks a caller-supplied CSR: row_ptr[0]=0, non-decreasing, row_ptr[N]=E,
 * col_idx/row_idx in range and consistent with row_ptr, edge_id in [0,E).
 * Synchronises `stream`.  EGNN_ERR_INDEX when it is malformed. */
EGNN_API int egnn_graph_check(int64_t n_nodes, int64_t n_edges, const egnn_graph* g,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- graph builders (device) -------------------------------------------- */

/* Scratch bytes of egnn_fc_graph for a batch of n_graphs graphs. */
EGNN_API size_t egnn_fc_graph_workspace_size(int64_t n_graphs);

/* Fully connected intra-graph edges of a batch, written directly as a dst CSR
 * (get_edges / get_edges_batch, egnn_clean.py:167-191, generalised to graphs
 * of different sizes): graph g owns nodes [graph_ptr[g], graph_ptr[g+1])
 * (graph_ptr: device int64, n_graphs + 1 entries, from 0 to n_nodes); row i
 * holds every other node j of its graph in increasing order.  n_edges must
 * be sum n_g (n_g - 1).  Writes row_ptr (N+1), col_idx and row_idx (E); the
 * edge ids are the CSR positions.  Synchronises `stream` (validation). */
EGNN_API int egnn_fc_graph(int64_t n_nodes, int64_t n_graphs, const int64_t* graph_ptr, int64_t n_edges,
                           int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx, void* workspace,
                           size_t workspace_bytes, void* stream);

enum { EGNN_GRAPH_RADIUS = 0, EGNN_GRAPH_KNN = 1 };

/* Spatial graph request.  Points x (N,3) float32 (device), optionally split
 * into graphs by graph_ptr (device int64, n_graphs + 1 entries, nodes of a
 * graph contiguous; NULL = one graph); edges never cross graphs.  Distances
 * are d2 = (dx*dx + dy*dy) + dz*dz in float32 with every operation rounded,
 * dx = x_i - x_j; ties in d2 go to the smaller j.
 *   EGNN_GRAPH_RADIUS: row i holds every j != i of its graph with
 *     d2 < cutoff*cutoff (float32), in increasing j; with max_nbrs > 0 only
 *     the max_nbrs nearest, nearest first (the survey's radius graphs of
 *     configs 3 and 4).
 *   EGNN_GRAPH_KNN: row i holds the k = max_nbrs (<= 256) nearest j != i of
 *     its graph (all of them in smaller graphs), nearest first (config 5);
 *     `cutoff` > 0 is a cell-size hint, 0 = chosen from the point density. */
typedef struct {
  int64_t n_nodes;
  int64_t n_graphs;
  const float* x;
  const int64_t* graph_ptr;
  int32_t mode;
  int32_t max_nbrs;
  float cutoff;
} egnn_spatial_desc;

/* Scratch bytes of egnn_spatial_count / egnn_spatial_fill for n_nodes points. */
EGNN_API size_t egnn_spatial_workspace_size(int64_t n_nodes);

/* Phase 1: builds the cell grid in `workspace` and writes row_ptr (N+1), the
 * exclusive scan of the row lengths (row_ptr[N] = E < 2^31).  The caller reads
 * row_ptr[N] to size col_idx.  Synchronises `stream` when graph_ptr is given
 * (validation) and to check that E fits int32. */
EGNN_API int egnn_spatial_count(const egnn_spatial_desc* d, int32_t* row_ptr, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Phase 2: writes col_idx and row_idx (E) for the same request, row_ptr and
 * workspace as phase 1 (unchanged in between).  Synchronises `stream`. */
EGNN_API int egnn_spatial_fill(const egnn_spatial_desc* d, const int32_t* row_ptr, int32_t* col_idx,
                               int32_t* row_idx, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes of egnn_morton_order. */
EGNN_API size_t egnn_morton_workspace_size(int64_t n_nodes);

/* Morton order of points x (N,3) float32 (the survey's config-5 node order):
 * per axis q = floor((double(x) - lo) / (hi - lo) * 2^bits) clipped to
 * [0, 2^bits), code = bits interleaved with bit b of axis a at 3b + a
 * (bits <= 21; lo, hi: HOST arrays of 3 doubles).  Writes codes (N, uint64,
 * node order) and perm (N): the nodes sorted stably by code. */
EGNN_API int egnn_morton_order(int64_t n_nodes, const float* x, const double* lo, const double* hi, int bits,
                               uint64_t* codes, int32_t* perm, void* workspace, size_t workspace_bytes,
                               void* stream);

/* ---- layer ------------------------------------------------------------- */

/* Bytes of per-layer state egnn_layer_fwd stores for egnn_layer_bwd: per
 * node, agg (H), the projections P and Q (2H) and the node-MLP hidden layer
 * before and after SiLU (2H), all float32.  No per-edge state is kept. */
EGNN_API size_t egnn_saved_size(const egnn_layer_desc* d);

/* Scratch bytes for egnn_layer_fwd (which = EGNN_WS_FWD) or egnn_layer_bwd
 * (EGNN_WS_BWD) on a device with `num_sms` SMs (0 = current device). */
EGNN_API size_t egnn_workspace_size(const egnn_layer_desc* d, int which, int num_sms);

/* E_GCL.forward (egnn_clean.py:95-103): h (N,I) -> h_out (N,O), x_out (N,3).
 * edge_attr may be NULL iff d->edge_attr_dim == 0.  `saved` (may be NULL in
 * inference) receives egnn_saved_size(d) bytes for the backward. */
EGNN_API int egnn_layer_fwd(const egnn_layer_desc* d, const egnn_graph* g, const egnn_layer_params* p,
                   const float* h, const float* x, const float* edge_attr,
                   float* h_out, float* x_out, void* saved,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Backward of E_GCL given dL/dh_out, dL/dx_out: writes dL/dh, dL/dx and every
 * parameter gradient.  Deterministic (no atomics): two calls on the same
 * inputs give bit-identical outputs. */
EGNN_API int egnn_layer_bwd(const egnn_layer_desc* d, const egnn_graph* g, const egnn_layer_params* p,
                   const float* h, const float* x, const float* edge_attr, const void* saved,
                   const float* grad_h_out, const float* grad_x_out,
                   float* grad_h, float* grad_x, const egnn_layer_grads* gp,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- graph-level loss of the training step ----------------------------- */

/* The benchmark objective around EGNN.forward (egnn_clean.py:141-146): the
 * per-graph sum of one node value (h_out[:, 0]) regressed on one target per
 * graph.  Graphs are contiguous node ranges: graph g holds nodes
 * graph_ptr[g] .. graph_ptr[g+1]-1 (graph_ptr: G+1 int64 offsets, 0 .. N).
 *   pred_g = sum_{i in g} values[i * ld],  loss = (1/G) sum_g (pred_g - target_g)^2
 * Deterministic: every sum is added in a fixed order (bit-identical reruns).
 * A malformed graph_ptr gives wrong sums, never an out-of-range access. */
EGNN_API size_t egnn_graph_mse_workspace_size(int64_t n_nodes);

/* Writes pred (G floats) and *loss (device). */
EGNN_API int egnn_graph_mse_fwd(int64_t n_nodes, int64_t n_graphs, const float* values, int64_t ld,
                                const int64_t* graph_ptr, const float* target, float* pred, float* loss,
                                void* workspace, size_t workspace_bytes, void* stream);

/* grad_values[i * ld] = grad_loss[0] * 2 (pred_g - target_g) / G for node i of
 * graph g (grad_loss: one device float). */
EGNN_API int egnn_graph_mse_bwd(int64_t n_nodes, int64_t n_graphs, const int64_t* graph_ptr, const float* pred,
                                const float* target, const float* grad_loss, float* grad_values, int64_t ld,
                                void* stream);

/* ---- node linear (embedding_in / embedding_out, egnn_clean.py:133-134) --- */

/* y (M,O) = x (M,K) W^T + b  (b may be NULL). */
EGNN_API int egnn_linear_fwd(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                    const float* b, float* y, void* stream);

/* Scratch bytes for egnn_linear_bwd. */
EGNN_API size_t egnn_linear_workspace_size(int64_t m, int32_t k, int32_t o);

/* dx = dy W (may be NULL to skip), dW = dy^T x, db = sum_rows dy (may be NULL). */
EGNN_API int egnn_linear_bwd(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                    const float* dy, float* dx, float* dw, float* db,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Size of the scratch array compiled into the library for
 * egnn_linear_bwd_static (4 MiB; each GPU that loads the library holds one
 * copy of it until the process exits). */
#define EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES ((size_t)4 << 20)

/* egnn_linear_bwd for callers that cannot allocate device memory.
 * No counterpart in the reference: it exists for host code that must not
 * call cudaMalloc, e.g. a plugin living inside a framework that owns every
 * device allocation and hands out no workspace, or a latency-critical host
 * path that must not add a synchronising allocation.  Same
 * inputs, outputs and results as egnn_linear_bwd; its scratch is a fixed
 * device array inside the library instead of a caller workspace, and it
 * calls no cudaMalloc, cudaFree or allocating library routine.
 * - Shapes whose egnn_linear_workspace_size(m, k, o) exceeds
 *   EGNN_LINEAR_BWD_STATIC_SCRATCH_BYTES are rejected with
 *   EGNN_ERR_WORKSPACE before anything is launched.
 * - The first call on each device (and on each CUDA context, so again after
 *   a cudaDeviceReset or under a caller's own context) looks up the array's
 *   device address with that device current; make that first call before
 *   any stream capture.
 * - All calls on a device share the one array and it keeps the previous
 *   call's contents (this entry point writes every scratch word before it
 *   reads it, so nothing needs clearing).  Calls whose GPU work overlaps,
 *   on different streams or threads, race on it: order them on one stream. */
EGNN_API int egnn_linear_bwd_static(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                                    const float* dy, float* dx, float* dw, float* db, void* stream);

/* ---- diagnostics ------------------------------------------------------- */

/* Copies the calling thread's last error message into buf (NUL-terminated);
 * returns the message length. */
EGNN_API size_t egnn_last_error(char* buf, size_t len);

/* Synchronises `stream` and reports whether a tensor-core edge kernel gave
 * up on a bounded wait since the last call (EGNN_ERR_CUDA, counter reset)
 * or not (EGNN_OK).  A kernel that gives up skips its remaining work, frees
 * its tensor memory and returns, so the context stays usable. */
EGNN_API int egnn_device_status(void* stream);

/* Library version, e.g. "egnn_b200 0.1 sm_100a". */
EGNN_API const char* egnn_version(void);

/* Number of kernel launches this library issued (all threads) since the
 * last call of egnn_launch_count_reset (for launch accounting). */
EGNN_API uint64_t egnn_launch_count(void);
EGNN_API void egnn_launch_count_reset(void);

/* Kernel timer for benchmarks: while enabled, the fused edge kernels
 * ("edge_fwd", "edge_bwd", "src_pass") are bracketed by CUDA events on their
 * launching stream.  Enabling or disabling clears the records.
 * egnn_kernel_time waits for the recorded events and returns the summed
 * milliseconds and launch count of one kernel name. */
EGNN_API void egnn_kernel_timing(int enable);
EGNN_API int egnn_kernel_time(const char* name, double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* EGNN_B200_H */
