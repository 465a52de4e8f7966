// Tensor-core (tcgen05) EGNN edge kernels for bf16-GEMM mode.
#pragma once

#include "edge_simt.cuh"

namespace egnn {

// True when the tensor-core kernels cover this layer configuration.
bool edge_tc_supported(int H, int d, int flags, int precision);

// CTA count and edges per CTA (a multiple of the 128-edge chunk).
EdgeGrid edge_tc_grid(int64_t E, int num_sms);

// Forward: agg, x_out (with the boundary fix-up).
int edge_fwd_tc(int H, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s);

// Backward dst pass: gstore, gdstore, per-CTA partials, then the row pass
// that fills S_dst and gxd.
int edge_bwd_tc(int H, const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s);

}  // namespace egnn
