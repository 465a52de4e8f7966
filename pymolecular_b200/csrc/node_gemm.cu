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
  const float* aux; int64_t ldaux; const float* resid; int64_t ldr; int64_t resid_cols;
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
    if (resid && n < resid_cols) v += resid[m * ldr + n];
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
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.resid_cols, a.C, a.ldc};
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
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.resid_cols, a.C, a.ldc};
  const int64_t total = a.M * a.N;
  if (a.db && a.db_part) {
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < a.M;
         m += (int64_t)gridDim.x * blockDim.x) {
      float v = 0.f;
      for (int z = 0; z < a.ksplit; ++z) v += a.db_part[(int64_t)z * a.M + m];
      a.db[m] = v;
    }
  }
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


// ---- register-tiled path -------------------------------------------------------
// BM x 128 output tile (BM = 128 or 64), K in slices of 8 through a double
// buffer, 256 threads each owning (BM/16) x 8 outputs.  Used when K is a
// multiple of 8 and the operands allow 16-byte loads (checked by gemm()).
template <int BM, int A_T, int B_T>
__global__ void __launch_bounds__(256) gemm_tiled_kernel(GemmArgs a) {
  constexpr int BN2 = 128, BK2 = 8, TM = BM / 16;
  __shared__ __align__(16) float As[2][BK2][BM + 4];
  __shared__ __align__(16) float Bs[2][BK2][BN2 + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN2;
  int64_t kbeg = 0, kend = a.K;
  if (a.ksplit > 1) {
    int64_t kc = (a.K + a.ksplit - 1) / a.ksplit;
    kc = (kc + BK2 - 1) / BK2 * BK2;
    kbeg = (int64_t)blockIdx.z * kc;
    kend = min(a.K, kbeg + kc);
  }
  // A slice: BM x 8 floats, B slice: 8 x 128 floats; one float4 each per
  // thread (A with BM = 64 uses half of the threads).
  float4 ra = make_float4(0.f, 0.f, 0.f, 0.f), rb = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load = [&](int64_t k0) {
    ra = make_float4(0.f, 0.f, 0.f, 0.f);
    rb = make_float4(0.f, 0.f, 0.f, 0.f);
    if (A_T == 0) {          // A(m, k) row-major: row m = tid/2, k = 4*(tid%2)
      const int64_t m = m0 + tid / 2, k = k0 + (tid % 2) * 4;
      if (tid / 2 < BM && m < a.M && k < kend) {
        const float* p = k < a.A.split ? a.A.p0 + m * a.A.ld0 + k : a.A.p1 + m * a.A.ld1 + (k - a.A.split);
        ra = *reinterpret_cast<const float4*>(p);
      }
    } else {                 // A(m, k) = G[k][m]: k = tid/32, m = 4*(tid%32)
      const int64_t k = k0 + tid / 32, m = m0 + (tid % 32) * 4;
      if ((tid % 32) * 4 < BM && m < a.M && k < kend)
        ra = *reinterpret_cast<const float4*>(a.A.p0 + k * a.A.ld0 + m);
    }
    if (B_T == 1) {          // B(k, n) = W[n][k]: row n = tid/2, k = 4*(tid%2)
      const int64_t n = n0 + tid / 2, k = k0 + (tid % 2) * 4;
      if (n < a.N && k < kend) {
        const float* p = (a.B.split_rows && n >= a.B.split) ? a.B.p1 + (n - a.B.split) * a.B.ld1 + k
                                                             : a.B.p0 + n * a.B.ld0 + k;
        rb = *reinterpret_cast<const float4*>(p);
      }
    } else {                 // B(k, n) = X[k][n] (columns may be split): k = tid/32, n = 4*(tid%32)
      const int64_t k = k0 + tid / 32, n = n0 + (tid % 32) * 4;
      if (n < a.N && k < kend) {
        const float* p = n < a.B.split ? a.B.p0 + k * a.B.ld0 + n : a.B.p1 + k * a.B.ld1 + (n - a.B.split);
        rb = *reinterpret_cast<const float4*>(p);
      }
    }
  };
  auto store = [&](int buf) {
    if (a.round_bf16) {
      ra = make_float4(bf16r(ra.x), bf16r(ra.y), bf16r(ra.z), bf16r(ra.w));
      rb = make_float4(bf16r(rb.x), bf16r(rb.y), bf16r(rb.z), bf16r(rb.w));
    }
    if (A_T == 0) {
      if (tid / 2 < BM) {
        const int ml = tid / 2, kl = (tid % 2) * 4;
        As[buf][kl + 0][ml] = ra.x; As[buf][kl + 1][ml] = ra.y;
        As[buf][kl + 2][ml] = ra.z; As[buf][kl + 3][ml] = ra.w;
      }
    } else if ((tid % 32) * 4 < BM) {
      *reinterpret_cast<float4*>(&As[buf][tid / 32][(tid % 32) * 4]) = ra;
    }
    if (B_T == 1) {
      const int nl = tid / 2, kl = (tid % 2) * 4;
      Bs[buf][kl + 0][nl] = rb.x; Bs[buf][kl + 1][nl] = rb.y;
      Bs[buf][kl + 2][nl] = rb.z; Bs[buf][kl + 3][nl] = rb.w;
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][tid / 32][(tid % 32) * 4]) = rb;
    }
  };

  float acc[TM][8];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  // db[m] = sum_k A(m, k): taken by the tx == 0 threads of the first column tile
  const bool do_db = A_T == 1 && a.db != nullptr && blockIdx.x == 0 && tx == 0;
  float dbacc[TM];
#pragma unroll
  for (int i = 0; i < TM; ++i) dbacc[i] = 0.f;

  int buf = 0;
  if (kbeg < kend) {
    load(kbeg);
    store(0);
  }
  __syncthreads();
#pragma unroll 1
  for (int64_t k0 = kbeg; k0 < kend; k0 += BK2) {
    const bool more = k0 + BK2 < kend;
    if (more) load(k0 + BK2);
#pragma unroll
    for (int k = 0; k < BK2; ++k) {
      float av[TM], bv[8];
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
      bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
      bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
      if constexpr (TM == 8) {
        const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
        av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      if (do_db) {
#pragma unroll
        for (int i = 0; i < TM; ++i) dbacc[i] += av[i];
      }
    }
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

  if (do_db) {
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
      if (m >= a.M) continue;
      if (a.ksplit > 1) a.db_part[(int64_t)blockIdx.z * a.M + m] = dbacc[i];
      else a.db[m] = dbacc[i];
    }
  }
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.resid_cols, a.C, a.ldc};
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= a.N) continue;
      if (a.ksplit > 1) a.part[(int64_t)blockIdx.z * a.M * a.N + m * a.N + n] = acc[i][j];
      else e.apply(m, n, acc[i][j]);
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the register-tiled kernel can take these operands.
bool tiled_ok(const GemmArgs& a) {
  // 16-byte loads along k need K % 8 == 0; row-wise loads (A^T, B) take any K.
  if ((a.a_t == 0 || a.b_t == 1) && a.K % 8 != 0) return false;
  const Mat& A = a.A;
  const Mat& B = a.B;
  if (a.a_t == 0) {
    if (A.split_rows || !aligned16(A.p0) || A.ld0 % 4) return false;
    if (A.p1 && (!aligned16(A.p1) || A.ld1 % 4 || A.split % 8)) return false;
  } else {
    if (A.p1 || !aligned16(A.p0) || A.ld0 % 4 || a.M % 4) return false;
  }
  if (a.b_t == 1) {
    if (!aligned16(B.p0) || B.ld0 % 4) return false;
    if (B.p1 && (!B.split_rows || !aligned16(B.p1) || B.ld1 % 4)) return false;
  } else {
    if (B.split_rows || !aligned16(B.p0) || B.ld0 % 4 || a.N % 4) return false;
    if (B.p1 && (!aligned16(B.p1) || B.ld1 % 4 || B.split % 4)) return false;
  }
  return true;
}

template <int BM>
void launch_tiled(const GemmArgs& a, dim3 grid, cudaStream_t s) {
  if (a.a_t == 0 && a.b_t == 1) gemm_tiled_kernel<BM, 0, 1><<<grid, 256, 0, s>>>(a);
  else if (a.a_t == 0 && a.b_t == 0) gemm_tiled_kernel<BM, 0, 0><<<grid, 256, 0, s>>>(a);
  else if (a.a_t == 1 && a.b_t == 0) gemm_tiled_kernel<BM, 1, 0><<<grid, 256, 0, s>>>(a);
  else gemm_tiled_kernel<BM, 1, 1><<<grid, 256, 0, s>>>(a);
}

}  // namespace

int gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return EGNN_OK;
  const unsigned z = (unsigned)(a.ksplit > 1 ? a.ksplit : 1);
  if (tiled_ok(a)) {
    const int64_t tiles128 = ((a.M + 127) / 128) * ((a.N + 127) / 128) * z;
    if (tiles128 >= 148) {
      launch_tiled<128>(a, dim3((unsigned)((a.N + 127) / 128), (unsigned)((a.M + 127) / 128), z), s);
    } else {
      launch_tiled<64>(a, dim3((unsigned)((a.N + 127) / 128), (unsigned)((a.M + 63) / 64), z), s);
    }
  } else {
    dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM), z);
    gemm_kernel<<<grid, NT, 0, s>>>(a);
  }
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
  int64_t tiles = ((M + 63) / 64) * ((N + 127) / 128);
  int64_t want = (148 + tiles - 1) / tiles;               // about one wave of CTAs
  int64_t by_len = std::max<int64_t>(1, K / 256);         // at least 256 rows per slice
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
  const bool fused_db = db && tiled_ok(a);
  if (fused_db) {
    a.db = db;
    a.db_part = a.ksplit > 1 ? part + (int64_t)a.ksplit * M * N : nullptr;
  }
  EGNN_TRY(gemm(a, s));
  if (db && !fused_db) EGNN_TRY(colsum(R, M, G, db, part, s));
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
