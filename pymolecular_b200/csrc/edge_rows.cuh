// EGNN edge MLPs as edge-row GEMMs on the tensor cores (bf16-GEMM mode,
// H = 256): the per-edge products run as persistent tcgen05 GEMMs over
// 128-edge tiles with one weight matrix resident in shared memory and fused
// epilogues; the per-edge operands live in a workspace that every layer
// reuses (the forward keeps only per-node state for the backward, which
// recomputes the edge activations).
#pragma once

#include <cuda_fp16.h>

#include "edge_simt.cuh"

namespace egnn {

// True when the edge-row GEMM path covers this layer configuration.
bool edge_rows_supported(int H, int d, int flags, int precision);

// Number of 128-edge tiles and the persistent CTA count for E edges.
int64_t rows_tiles(int64_t E);
int rows_grid(int64_t E, int num_sms);

// Per-edge operands, tile-major bf16 ("tiles": 64 KB per 128 edges, four
// 16 KB column blocks of 128 rows x 64 features in the 128-byte swizzle) or
// row-major fp32.
struct RowsBufs {
  char* W2img = nullptr; // bf16 images of W2 hi | lo (256 KB) for the split W2 products
  char* U = nullptr;     // tiles: u1 = silu(a1)
  char* Mb = nullptr;    // tiles: m = silu(a2 + b2)
  char* Gc1 = nullptr;   // tiles: dL/dc1 (backward)
  char* Ga2 = nullptr;   // tiles: dL/da2 (backward)
  float* M32 = nullptr;  // (E, H) fp32 m (forward, for the row sums)
  __half* D2 = nullptr;  // (E, H) fp16 silu'(a2 + b2) (backward)
  __half* S1 = nullptr;  // (E, H) fp16 silu'(a1) (backward)
  float4* gtr = nullptr; // (E) backward: dL/dx'_i s_i (xyz), 1 / (|d| + eps) or 0 on a self-loop (w)
  float* phi = nullptr;  // (E) coordinate weight phi_e
  float4* geo = nullptr; // (E) x_i - x_j, |x_i - x_j|^2
  float* part = nullptr; // (G, edge_part_floats(H, 0)) per-CTA weight-gradient partials
  int G = 1;
};

// Carves the buffers from a workspace (fwd: U, Mb, M32, phi, geo; bwd: U,
// Mb, Gc1, Ga2, D2, S1, gtr, phi, geo, part).
RowsBufs carve_rows(Carver& c, int64_t E, int H, bool bwd, int num_sms);

// Forward: agg, x_out.
int edge_fwd_rows(const EdgeFwdArgs& a, const RowsBufs& b, cudaStream_t s);

// Backward up to the per-edge gradients: gstore (bf16 dL/da1 rows), gdstore,
// and the bias / w_c2 / w_r slots of the per-CTA partials.
int edge_bwd_rows(const EdgeBwdArgs& a, const RowsBufs& b, cudaStream_t s);

// dW_c1 and dW_2 slots of the per-CTA partials (after edge_bwd_rows).
int edge_wgrad_rows(int64_t E, const RowsBufs& b, cudaStream_t s);

// Number of waits in these kernels that ran out since the last call (reset).
int rows_take_timeouts();

}  // namespace egnn
