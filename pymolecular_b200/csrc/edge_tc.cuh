// Tensor-core (tcgen05) EGNN edge kernels for bf16-GEMM mode.
#pragma once

#include "edge_simt.cuh"

namespace egnn {

// True when the tensor-core kernels cover this layer configuration.
bool edge_tc_supported(int H, int d, int flags, int precision);
// The forward also runs the attention gate and edge attributes (d <= 16).
bool edge_tc_fwd_supported(int H, int d, int flags, int precision);

// CTA count and edges per CTA (a multiple of the 128-edge chunk).
EdgeGrid edge_tc_grid(int64_t E, int num_sms);

// Forward: agg, x_out (with the boundary fix-up).
int edge_fwd_tc(int H, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s);

// Backward edge kernel: per-edge dL/da1 rows (bf16) in gstore, coordinate
// gradients in gdstore, per-CTA weight-gradient partials.
int edge_bwd_tc(int H, const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s);

// Node pass after edge_bwd_tc: S_dst / S_src (sums of the bf16 gstore rows over
// each node's in- / out-edges) and gx = gx_out + (in-edge) - (out-edge)
// coordinate-gradient sums.
int edge_node_pass_tc(int H, int64_t N, const int32_t* row_ptr, const int32_t* src_ptr, const int32_t* src_edge,
                      const void* gstore, const float4* gdstore, const float* gx_out, float* S_dst, float* S_src,
                      float* gx, cudaStream_t s);

}  // namespace egnn
