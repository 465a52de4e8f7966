// Node-side SIMT GEMMs (fp32 FFMA, optional bf16 rounding of the inputs).
//
// 64x64 output tile per 256-thread CTA, K staged through shared memory in
// slices of 16, 4x4 outputs per thread.  Deterministic: every output is one
// thread's fixed-order sum; split-K partial slices are added in slice order.
#include <algorithm>

#include "node_gemm.cuh"

namespace egnn {

namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

struct Epi {
  const float* bias; float* pre; int64_t ldp; int act;
  const float* aux; int64_t ldaux; const float* resid; int64_t ldr;
  float* C; int64_t ldc;
  __device__ __forceinline__ void apply(int64_t m, int64_t n, float v) const {
    if (bias) v += bias[n];
    if (pre) pre[m * ldp + n] = v;
    if (act == ACT_SILU) {
      v = silu_f(v);
    } else if (act == ACT_DSILU) {
      float y, dy;
      silu_and_grad(aux[m * ldaux + n], y, dy);
      v *= dy;
    }
    if (resid) v += resid[m * ldr + n];
    C[m * ldc + n] = v;
  }
};

__global__ void __launch_bounds__(NT) gemm_kernel(GemmArgs a) {
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  int64_t kbeg = 0, kend = a.K;
  if (a.ksplit > 1) {
    int64_t kc = (a.K + a.ksplit - 1) / a.ksplit;
    kc = (kc + BK - 1) / BK * BK;
    kbeg = (int64_t)blockIdx.z * kc;
    kend = min(a.K, kbeg + kc);
  }

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int64_t k0 = kbeg; k0 < kend; k0 += BK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int idx = tid + NT * q;
      int ml, kl;
      if (a.a_t) { kl = idx / BM; ml = idx % BM; } else { ml = idx / BK; kl = idx % BK; }
      int64_t m = m0 + ml, k = k0 + kl;
      float v = 0.f;
      if (m < a.M && k < kend) v = a.a_t ? a.A.at(k, m) : a.A.at(m, k);
      if (a.round_bf16) v = bf16r(v);
      As[kl][ml] = v;
      int nl;
      if (a.b_t) { nl = idx / BK; kl = idx % BK; } else { kl = idx / BN; nl = idx % BN; }
      int64_t n = n0 + nl;
      k = k0 + kl;
      float w = 0.f;
      if (n < a.N && k < kend) w = a.b_t ? a.B.at(n, k) : a.B.at(k, n);
      if (a.round_bf16) w = bf16r(w);
      Bs[kl][nl] = w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float4 av = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      float4 bv = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
      float ar[4] = {av.x, av.y, av.z, av.w};
      float br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }

  if (a.ksplit > 1) {
    float* part = a.part + (int64_t)blockIdx.z * a.M * a.N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t m = m0 + ty * 4 + i;
      if (m >= a.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int64_t n = n0 + tx * 4 + j;
        if (n < a.N) part[m * a.N + n] = acc[i][j];
      }
    }
    return;
  }
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.C, a.ldc};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t m = m0 + ty * 4 + i;
    if (m >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t n = n0 + tx * 4 + j;
      if (n < a.N) e.apply(m, n, acc[i][j]);
    }
  }
}

__global__ void gemm_reduce_kernel(GemmArgs a) {
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.C, a.ldc};
  const int64_t total = a.M * a.N;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int z = 0; z < a.ksplit; ++z) v += a.part[(int64_t)z * total + idx];
    e.apply(idx / a.N, idx % a.N, v);
  }
}

__global__ void colsum_partial_kernel(int64_t R, int64_t C, Mat G, int64_t rows_per, float* part) {
  int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  int64_t r0 = (int64_t)blockIdx.y * rows_per, r1 = min(R, r0 + rows_per);
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += G.at(r, c);
  part[(int64_t)blockIdx.y * C + c] = s;
}

__global__ void colsum_reduce_kernel(int64_t C, int S, const float* part, float* out) {
  int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (int z = 0; z < S; ++z) s += part[(int64_t)z * C + c];
  out[c] = s;
}

}  // namespace

int gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return EGNN_OK;
  dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM),
            (unsigned)(a.ksplit > 1 ? a.ksplit : 1));
  if (a.K <= 0 && a.ksplit <= 1) {
    // empty reduction: the epilogue still runs on zeros
  }
  gemm_kernel<<<grid, NT, 0, s>>>(a);
  EGNN_CHECK_LAUNCH();
  if (a.ksplit > 1) {
    int64_t total = a.M * a.N;
    int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
    gemm_reduce_kernel<<<blocks, 256, 0, s>>>(a);
    EGNN_CHECK_LAUNCH();
  }
  return EGNN_OK;
}

int64_t wgrad_splits(int64_t K, int64_t M, int64_t N) {
  int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  int64_t want = (2 * 148 + tiles - 1) / tiles;          // about two waves of CTAs
  int64_t by_len = std::max<int64_t>(1, K / 128);         // at least 128 rows per slice
  return std::max<int64_t>(1, std::min<int64_t>({want, by_len, 64}));
}

int wgrad(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw,
          float* db, int round_bf16, float* part, cudaStream_t s) {
  GemmArgs a;
  a.M = M; a.N = N; a.K = R;
  a.A = G; a.a_t = 1;
  a.B = X; a.b_t = 0;
  a.C = dW; a.ldc = lddw;
  a.round_bf16 = round_bf16;
  a.ksplit = (int)wgrad_splits(R, M, N);
  a.part = part;
  if (a.ksplit == 1) a.part = nullptr;
  EGNN_TRY(gemm(a, s));
  if (db) EGNN_TRY(colsum(R, M, G, db, part, s));
  return EGNN_OK;
}

int64_t colsum_splits(int64_t R) {
  return std::max<int64_t>(1, std::min<int64_t>(64, R / 256));
}

int colsum(int64_t R, int64_t C, Mat G, float* db, float* part, cudaStream_t s) {
  if (C <= 0) return EGNN_OK;
  int64_t S = colsum_splits(R);
  int64_t rows_per = (R + S - 1) / S;
  if (R == 0) rows_per = 1;
  dim3 grid((unsigned)((C + 127) / 128), (unsigned)S);
  colsum_partial_kernel<<<grid, 128, 0, s>>>(R, C, G, rows_per, part);
  EGNN_CHECK_LAUNCH();
  colsum_reduce_kernel<<<(unsigned)((C + 127) / 128), 128, 0, s>>>(C, (int)S, part, db);
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

}  // namespace egnn
