// Node-side GEMMs on the tensor cores for bf16 mode: every fp32 operand is
// split into two bf16 parts (hi = bf16(x), lo = bf16(x - hi)) and the product
// is taken as hi*hi + hi*lo + lo*hi with fp32 accumulation in TMEM, about
// 16 bits of operand precision (relative error ~1e-5 per output).
#pragma once

#include "node_gemm.cuh"

namespace egnn {

// Whether gemm_tc() takes these operands (same GemmArgs meaning as gemm()).
bool gemm_tc_ok(const GemmArgs& a);

// C = op(A) op(B) with the gemm() epilogue; split-K partials (ksplit > 1)
// are added by the same ordered reduction as gemm().
int gemm_tc(const GemmArgs& a, cudaStream_t s);

// Split-K count of wgrad_tc() for R rows: about one wave of 128 x 128 output
// tiles, at least two 64-row chunks per slice, at most 64 slices.  The
// split-K workspace holds that many slices of M x N (+ M for the bias).
int64_t wgrad_tc_splits(int64_t R, int64_t M, int64_t N);

// Weight gradient as wgrad(), on the tensor cores; `part` holds
// max(wgrad_splits, wgrad_tc_splits) slices.
int wgrad_tc(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw, float* db, float* part,
             cudaStream_t s);

// Number of tensor-core waits in these kernels that ran out since the last
// call (the counter is reset).
int node_tc_take_timeouts();

}  // namespace egnn
