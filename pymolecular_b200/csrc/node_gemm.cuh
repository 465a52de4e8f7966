// Node-side dense GEMMs of the EGNN layer (embedding, phi_e layer-1
// projections, node MLP and their gradients).  These run over N rows, an
// order of magnitude fewer than the E edge rows of the fused edge kernels.
#pragma once

#include "common.cuh"

namespace egnn {

// A logical row-major matrix that may be the concatenation of two buffers,
// either side by side (split on columns, e.g. cat([h, agg], 1)) or stacked
// (split on rows).  at(r, c) is element (r, c).
struct Mat {
  const float* p0 = nullptr;
  const float* p1 = nullptr;
  int64_t ld0 = 0, ld1 = 0;
  int64_t split = INT64_MAX;   // columns (or rows) < split live in p0
  int split_rows = 0;
  __device__ __forceinline__ float at(int64_t r, int64_t c) const {
    if (split_rows) {
      return r < split ? p0[r * ld0 + c] : p1[(r - split) * ld1 + c];
    }
    return c < split ? p0[r * ld0 + c] : p1[r * ld1 + (c - split)];
  }
};

inline Mat mat(const float* p, int64_t ld) { Mat m; m.p0 = p; m.ld0 = ld; return m; }
inline Mat mat_cols(const float* a, int64_t lda, int64_t ka, const float* b, int64_t ldb) {
  Mat m; m.p0 = a; m.ld0 = lda; m.p1 = b; m.ld1 = ldb; m.split = ka; return m;
}
inline Mat mat_rows(const float* a, int64_t lda, int64_t ra, const float* b, int64_t ldb) {
  Mat m; m.p0 = a; m.ld0 = lda; m.p1 = b; m.ld1 = ldb; m.split = ra; m.split_rows = 1; return m;
}

enum { ACT_NONE = 0, ACT_SILU = 1, ACT_DSILU = 2 };

// C (M,N) = epilogue( op(A) (M,K) * op(B) (K,N) ).
//   a_t: A(m,k) = A.at(k,m) (else A.at(m,k));  b_t: B(k,n) = B.at(n,k) (nn.Linear W).
// Epilogue: v = acc + bias[n];  pre[m,n] = v (if pre);
//   act SILU: v = silu(v);  act DSILU: v = v * silu'(aux[m,n]);
//   v += resid[m,n] (if resid);  C[m,n] = v.
// Split-K (ksplit > 1): grid.z slices of the K range write raw partial sums
// to part[z][M][N]; gemm_reduce() then adds the slices in slice order.
struct GemmArgs {
  int64_t M = 0, N = 0, K = 0;
  Mat A, B;
  int a_t = 0, b_t = 0;
  float* C = nullptr; int64_t ldc = 0;
  const float* bias = nullptr;
  float* pre = nullptr; int64_t ldp = 0;
  int act = ACT_NONE;
  const float* aux = nullptr; int64_t ldaux = 0;
  const float* resid = nullptr; int64_t ldr = 0;
  int64_t resid_cols = INT64_MAX;   // the residual is added to columns n < resid_cols only
  int round_bf16 = 0;           // round A and B elements to bf16 (bf16-GEMM mode)
  int ksplit = 1;
  float* part = nullptr;
  // Weight-gradient GEMMs (a_t = 1) may also produce db[m] = sum_k A(m, k);
  // with split-K the slices go to db_part[z][M] first.
  float* db = nullptr;
  float* db_part = nullptr;
  int vec = 0;   // set by gemm(): the epilogue may move four columns at a time
  // bf16 mode: B (K x N, b_t = 0) already split into bf16 hi / lo parts laid
  // out as the GEMM's shared-memory tiles (see BImage); nullptr: split per CTA
  const char* b_img = nullptr;
  int64_t b_img_nb = 0;          // 64-column blocks per 64-row chunk of the image
  int64_t b_img_part = 0;        // bytes from the hi part to the lo part
};

// A weight operand B (K x N, element (k, n)) as bf16 hi = bf16(B) and
// lo = bf16(B - hi) images: for each 64-row chunk kc of k and each 64-column
// block nb of n an 8 KB block of 64 k-rows x 128 bytes in the 128-byte
// swizzle of an MN-major tcgen05 operand (16-byte chunk c of row r at
// c ^ (r % 8)), block (kc, nb) at byte (kc NB + nb) 8192, the lo part at
// NKC NB 8192.  Padding rows and columns are zero.  NB is a multiple of 4,
// so a 128- or 256-column tile is one contiguous 16 or 32 KB piece per part.
struct BImage {
  char* base = nullptr;
  int64_t K = 0, N = 0, nkc = 0, nb = 0;
  __host__ __device__ int64_t part_bytes() const { return nkc * nb * 8192; }
  __host__ __device__ int64_t bytes() const { return 2 * part_bytes(); }
};
inline BImage bimage_shape(int64_t K, int64_t N) {
  BImage b;
  b.K = K; b.N = N;
  b.nkc = (K + 63) / 64;
  b.nb = ((N + 63) / 64 + 3) / 4 * 4;
  return b;
}
inline void gemm_use_image(GemmArgs& g, const BImage& b) {
  if (!b.base) return;
  g.b_img = b.base; g.b_img_nb = b.nb; g.b_img_part = b.part_bytes();
}

int gemm(const GemmArgs& a, cudaStream_t s);

// y (M x N, row stride ldy) = x (M x K, row stride ldx) W^T (+ b) for the
// degenerate shapes of the embeddings: K <= 8, or N == 1.  W is (N x K)
// row-major when w_nk, else (K x N).
bool linear_small_ok(int N, int K);
int linear_small(int64_t M, int N, int K, const float* x, int64_t ldx, const float* w, int w_nk, const float* b,
                 float* y, int64_t ldy, cudaStream_t s);

// The ordered split-K reduction (and epilogue) of a GEMM whose ksplit > 1
// partial slices sit in a.part (and db slices in a.db_part).
int gemm_reduce(const GemmArgs& a, cudaStream_t s);

// Workspace floats gemm() needs for its split-K partials when used as a
// weight-gradient GEMM with reduction length K.
int64_t wgrad_splits(int64_t K, int64_t M, int64_t N);

// Weight gradient dW (M,N) = sum_r G[r, m] * X[r, n]  over r in [0,R),
// plus optional db[m] = sum_r G[r, m].  Deterministic split-K.
// `part` must hold wgrad_splits(R,M,N) * (M*N + M) floats (and at least
// colsum_splits(R) * M).
int wgrad(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw,
          float* db, int round_bf16, float* part, cudaStream_t s);

// Column sums db[c] = sum_r G[r,c] (deterministic, 2-level).  part holds
// colsum_splits(R) * C floats.
int64_t colsum_splits(int64_t R);
int colsum(int64_t R, int64_t C, Mat G, float* db, float* part, cudaStream_t s);

}  // namespace egnn
