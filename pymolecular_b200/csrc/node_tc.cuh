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

// Weight gradient as wgrad() (same workspace bound), on the tensor cores.
int wgrad_tc(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw, float* db, float* part,
             cudaStream_t s);

// Number of tensor-core waits in these kernels that ran out since the last
// call (the counter is reset).
int node_tc_take_timeouts();

}  // namespace egnn
