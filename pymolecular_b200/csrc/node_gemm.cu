// Node-side SIMT GEMMs (fp32 FFMA).
//
// The tiled kernel (below) takes every operand layout the layer uses; a
// plain 64x64-tile kernel covers the rest (bf16-rounded inputs, K not a
// multiple of 4, unaligned operands).  Deterministic: every output is one thread's
// fixed-order sum; split-K partial slices are added in slice order.
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
  pdl_enter();
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

// Split-K reduction: a block takes 32 consecutive outputs (one per lane);
// its 8 warps each add a contiguous eighth of the slices (all loads of a
// warp in flight at once), and warp 0 adds the 8 partial sums in warp order:
// a fixed association, so the result is bit-reproducible.  Blocks past the
// outputs do the same for the db slices.
__global__ void __launch_bounds__(256) gemm_reduce_kernel(GemmArgs a) {
  pdl_enter();
  __shared__ float red[8][33];
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.resid_cols, a.C, a.ldc};
  const int64_t total = a.M * a.N;
  const int64_t nb_main = (total + 31) / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool main = blockIdx.x < nb_main;
  const int64_t stride = main ? total : a.M;
  const int64_t idx = (main ? (int64_t)blockIdx.x : (int64_t)blockIdx.x - nb_main) * 32 + lane;
  const float* src = main ? a.part : a.db_part;
  const int S = a.ksplit, per = (S + 7) / 8;
  const int z0 = min(S, warp * per), z1 = min(S, z0 + per);
  float v = 0.f;
  if (idx < stride) {
    for (int z = z0; z < z1; z += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = (z + u < z1) ? src[(int64_t)(z + u) * stride + idx] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) v += t[u];
    }
  }
  red[warp][lane] = v;
  __syncthreads();
  if (warp == 0 && idx < stride) {
    float s = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) s += red[w][lane];
    if (main) e.apply(idx / a.N, idx % a.N, s);
    else a.db[idx] = s;
  }
}

// Column sums in row order; rows are loaded eight at a time (independent
// loads) and added one by one, so the result equals the plain row loop's.
__global__ void colsum_partial_kernel(int64_t R, int64_t C, Mat G, int64_t rows_per, float* part) {
  pdl_enter();
  int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  int64_t r0 = (int64_t)blockIdx.y * rows_per, r1 = min(R, r0 + rows_per);
  float s = 0.f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    float t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = G.at(r + u, c);
#pragma unroll
    for (int u = 0; u < 8; ++u) s += t[u];
  }
  for (; r < r1; ++r) s += G.at(r, c);
  part[(int64_t)blockIdx.y * C + c] = s;
}

__global__ void colsum_reduce_kernel(int64_t C, int S, const float* part, float* out) {
  pdl_enter();
  int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  int z = 0;
  for (; z + 8 <= S; z += 8) {
    float t[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = part[(int64_t)(z + u) * C + c];
#pragma unroll
    for (int u = 0; u < 8; ++u) s += t[u];
  }
  for (; z < S; ++z) s += part[(int64_t)z * C + c];
  out[c] = s;
}


// ---- degenerate shapes of the embeddings ------------------------------------------
// y = x W^T (+ b) with K <= 8 (embedding_in; the input gradient of
// embedding_out, K = 1).  Thread (n, row slot): W's column n in registers,
// one output per row, k in order then the bias (as the tiled kernels do).
constexpr int kSmallK = 8;
__global__ void linear_smallk_kernel(int64_t M, int N, int K, const float* __restrict__ x, int64_t ldx,
                                     const float* __restrict__ w, int w_nk, const float* __restrict__ b,
                                     float* __restrict__ y, int64_t ldy) {
  pdl_enter();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float wk[kSmallK];
#pragma unroll
  for (int k = 0; k < kSmallK; ++k) wk[k] = k < K ? (w_nk ? w[(int64_t)n * K + k] : w[(int64_t)k * N + n]) : 0.f;
  const float bias = b ? b[n] : 0.f;
  for (int64_t m = (int64_t)blockIdx.y * blockDim.y + threadIdx.y; m < M; m += (int64_t)gridDim.y * blockDim.y) {
    const float* xr = x + m * ldx;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kSmallK; ++k)
      if (k < K) acc = fmaf(__ldg(xr + k), wk[k], acc);
    y[m * ldy + n] = b ? acc + bias : acc;
  }
}

// y = x w (+ b) with one output column (embedding_out): one warp per row,
// lanes over k, a fixed-order shuffle tree.
__global__ void linear_n1_kernel(int64_t M, int K, const float* __restrict__ x, int64_t ldx,
                                 const float* __restrict__ w, const float* __restrict__ b, float* __restrict__ y,
                                 int64_t ldy) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t m = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; m < M; m += warps) {
    const float* xr = x + m * ldx;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc = fmaf(__ldg(xr + k), __ldg(w + k), acc);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[m * ldy] = b ? acc + b[0] : acc;
  }
}

// ---- weight gradients with one narrow side (the embeddings) -----------------------
// dW (M x N) = sum_r G[r][i] X[r][j] and db (M) = sum_r G[r][i], computed as
// one product with X extended by a column of ones (db = its last column).
// The wide side (max(M, N + 1) <= 288) runs over the lanes, the narrow side
// (min(M, N + 1) <= 45) in groups of 9, one group per grid row.  Block z
// streams rows [z rows_per, ...) through a ring of shared-memory stages of 32
// rows filled by cp.async (depth small_stages); warp w takes rows w, w + 8,
// w + 16, w + 24 of every stage (each warp adds its rows in row order), a lane
// owns the wide indices lane + 32 t; warp partials are added in warp order,
// then the block slices in block order (wgrad_small_reduce_kernel).
constexpr int kNarrow = 9;            // narrow indices per group
constexpr int kNarrowMax = 45;        // narrow side incl. the ones column: 5 groups
constexpr int kWideSlots = 9;         // wide side up to 288 (with the ones column)
constexpr int kStageRows = 32;
// ring depth: six stages while two blocks of them still fit on an SM (wide
// side up to 128), three beyond
__host__ __device__ constexpr int small_stages(int slots) { return slots <= 4 ? 6 : 3; }

struct SmallShape {
  int lanes_n;     // lanes over the extended columns of X (else over the rows i of dW)
  int wide, narrow;
  int wide_data;   // staged wide values (the ones column is implied)
  int groups, slots;
};
__host__ __device__ inline SmallShape small_shape(int M, int N) {
  SmallShape s;
  const int N1 = N + 1;
  s.lanes_n = N1 >= M;
  s.wide = s.lanes_n ? N1 : M;
  s.narrow = s.lanes_n ? M : N1;
  s.wide_data = s.lanes_n ? N : M;
  s.groups = (s.narrow + kNarrow - 1) / kNarrow;
  s.slots = (s.wide + 31) / 32;
  return s;
}
size_t small_smem_bytes(int slots) {
  const size_t ring = (size_t)small_stages(slots) * kStageRows * (32 * slots + kNarrow) * 4;
  const size_t red = (size_t)8 * 32 * slots * kNarrow * 4;
  return std::max(ring, red);
}

__global__ void wgrad_small_reduce_kernel(int M, int N, int S, const float* part, float* dW, int64_t lddw,
                                          float* db) {
  pdl_enter();
  const int N1 = N + 1, O = M * N1;
  for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < O; o += gridDim.x * blockDim.x) {
    float v = 0.f;
    int z = 0;
    for (; z + 8 <= S; z += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = part[(int64_t)(z + u) * O + o];
#pragma unroll
      for (int u = 0; u < 8; ++u) v += t[u];
    }
    for (; z < S; ++z) v += part[(int64_t)z * O + o];
    const int i = o / N1, j = o % N1;
    if (j < N) dW[(int64_t)i * lddw + j] = v;
    else if (db) db[i] = v;
  }
}

// ---- tiled path ------------------------------------------------------------------
// C (M x N) = A B for every operand layout the layer uses.  Tile 64 x 128
// per 256-thread CTA; thread (tx, ty) owns rows ty*4 + {0..3} and columns
// tx*4 + {0..3}, 64 + tx*4 + {0..3}.  K runs in slices of 16 through a double
// buffer in shared memory, stored k-major: As[k][m], Bs[k][n], so every step
// of the inner product is an outer product of two register fragments read
// with 16-byte loads.
//   k-major operands in global memory (A^T of a weight gradient, B = X[k][n])
//   are copied with cp.async; row-major ones (A[m][k], B = W[n][k]) are read
//   four k at a time into registers one slice ahead and stored transposed.
// 256 threads form a 16 x 16 grid in which every half-warp is a 4 x 4 block,
// so each fragment load touches 4 distinct 16-byte words per half-warp.
__device__ __forceinline__ uint32_t sptr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Zero-filling 16-byte asynchronous copy: nothing is read when `ok` is false.
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sptr(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ const float* mat_ptr(const Mat& A, int64_t r, int64_t c) {
  if (A.split_rows) return r < A.split ? A.p0 + r * A.ld0 + c : A.p1 + (r - A.split) * A.ld1 + c;
  return c < A.split ? A.p0 + r * A.ld0 + c : A.p1 + r * A.ld1 + (c - A.split);
}

// Zero-filling 4-byte asynchronous copy (any alignment).
__device__ __forceinline__ void cp_async4z(float* dst, const float* src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sptr(dst)), "l"(src), "r"(ok ? 4 : 0)
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_n() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <int WS>
__global__ void __launch_bounds__(256) wgrad_small_partial_kernel(int64_t R, int M, int N, Mat G, Mat X,
                                                                  int64_t rows_per, int vec_w, float* part) {
  pdl_enter();
  constexpr int kStages = small_stages(WS);
  extern __shared__ __align__(16) float wsm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const SmallShape sh = small_shape(M, N);
  const int N1 = N + 1;
  const int q0 = blockIdx.y * kNarrow;                 // first narrow index of this group
  const int nq = min(kNarrow, sh.narrow - q0);
  constexpr int LDW = 32 * WS;                         // staged wide row (floats)
  float* ring_w = wsm;                                 // [kStages][kStageRows][LDW]
  float* ring_n = wsm + kStages * kStageRows * LDW;    // [kStages][kStageRows][kNarrow]
  const int64_t r0 = (int64_t)blockIdx.x * rows_per, r1 = min(R, r0 + rows_per);
  const int64_t nrows = r1 > r0 ? r1 - r0 : 0;
  const int nstage = (int)((nrows + kStageRows - 1) / kStageRows);
  const Mat& Wm = sh.lanes_n ? X : G;                  // wide operand
  const Mat& Nm = sh.lanes_n ? G : X;                  // narrow operand
  const int narrow_data = sh.lanes_n ? M : N;          // narrow index N of X is the ones column

  auto issue = [&](int st) {
    if (st < nstage) {
      float* dw = ring_w + (st % kStages) * kStageRows * LDW;
      float* dn = ring_n + (st % kStages) * kStageRows * kNarrow;
      const int64_t rs = r0 + (int64_t)st * kStageRows;
      if (vec_w) {   // aligned rows, wide_data % 4 == 0: 16-byte words
        const int words = sh.wide_data / 4;
        for (int c = threadIdx.x; c < kStageRows * words; c += 256) {
          const int rl = c / words, w4 = (c % words) * 4;
          const int64_t r = rs + rl;
          const bool ok = r < r1;
          cp_async16(dw + rl * LDW + w4, ok ? mat_ptr(Wm, r, w4) : Wm.p0, ok);
        }
      } else {
        for (int c = threadIdx.x; c < kStageRows * sh.wide_data; c += 256) {
          const int rl = c / sh.wide_data, w = c % sh.wide_data;
          const int64_t r = rs + rl;
          const bool ok = r < r1;
          cp_async4z(dw + rl * LDW + w, ok ? mat_ptr(Wm, r, w) : Wm.p0, ok);
        }
      }
      for (int c = threadIdx.x; c < kStageRows * nq; c += 256) {
        const int rl = c / nq, q = c % nq, j = q0 + q;
        const int64_t r = rs + rl;
        const bool ok = r < r1 && j < narrow_data;
        cp_async4z(dn + rl * kNarrow + q, ok ? mat_ptr(Nm, r, j) : Nm.p0, ok);
      }
    }
    cp_async_commit();   // empty groups keep the count uniform
  };

  float acc[WS][kNarrow];
#pragma unroll
  for (int t = 0; t < WS; ++t)
#pragma unroll
    for (int q = 0; q < kNarrow; ++q) acc[t][q] = 0.f;
#pragma unroll
  for (int p = 0; p < kStages - 1; ++p) issue(p);
#pragma unroll 1
  for (int st = 0; st < nstage; ++st) {
    cp_async_wait_n<kStages - 2>();   // this thread's copies of stage st have landed
    __syncthreads();                  // everyone's have; stage st - 1 is consumed
    issue(st + kStages - 1);
    const float* sw = ring_w + (st % kStages) * kStageRows * LDW;
    const float* sn = ring_n + (st % kStages) * kStageRows * kNarrow;
    const int64_t left = r1 - (r0 + (int64_t)st * kStageRows);
    const int live = left < kStageRows ? (int)left : kStageRows;
#pragma unroll 1
    for (int u = 0; u < kStageRows / 8; ++u) {
      const int rl = warp + 8 * u;
      if (rl >= live) break;
      float wv[WS], nv[kNarrow];
#pragma unroll
      for (int t = 0; t < WS; ++t) {
        const int w = lane + 32 * t;
        wv[t] = w < sh.wide_data ? sw[rl * LDW + w] : (w < sh.wide ? 1.f : 0.f);
      }
#pragma unroll
      for (int q = 0; q < kNarrow; ++q) nv[q] = q < nq ? (q0 + q < narrow_data ? sn[rl * kNarrow + q] : 1.f) : 0.f;
#pragma unroll
      for (int t = 0; t < WS; ++t)
#pragma unroll
        for (int q = 0; q < kNarrow; ++q) acc[t][q] = fmaf(wv[t], nv[q], acc[t][q]);
    }
  }
  cp_async_wait_n<0>();
  __syncthreads();   // the ring is free for the warp partials
  float* red = wsm;  // [8 warps][32 WS wide][kNarrow]
  constexpr int PER = 32 * WS * kNarrow;
#pragma unroll
  for (int t = 0; t < WS; ++t)
#pragma unroll
    for (int q = 0; q < kNarrow; ++q) red[warp * PER + (t * 32 + lane) * kNarrow + q] = acc[t][q];
  __syncthreads();
  for (int o = threadIdx.x; o < PER; o += 256) {
    const int wi = o / kNarrow, q = o % kNarrow;
    if (wi >= sh.wide || q >= nq) continue;
    float v = red[o];
#pragma unroll
    for (int w = 1; w < 8; ++w) v += red[w * PER + o];
    const int ni = q0 + q;
    const int i = sh.lanes_n ? ni : wi, j = sh.lanes_n ? wi : ni;
    part[(int64_t)blockIdx.x * M * N1 + (int64_t)i * N1 + j] = v;
  }
}

__device__ __forceinline__ void thread_grid(int& tx, int& ty) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ty = (warp >> 2) * 8 + (lane >> 2);
  tx = (warp & 3) * 4 + (lane & 3);
}

// 64 x 128 tiles (TM = 4): on B200 the 128 x 128 tile (TM = 8) measured no
// faster on these shapes (K = 128..256) and quantises worse over 148 SMs.
// 64 x 64 tiles (NBN = 1 column group) when 128-column tiles would leave
// more than half the SMs idle (small row counts, N <= 64).
constexpr int TBN = 128, TBK = 16, TTM = 4;

template <int BM, int BN>
constexpr size_t tiled_smem_bytes() {
  return (size_t)2 * TBK * ((BM + 4) + (BN + 4)) * sizeof(float);
}

// One operand slice: ROWS rows (m or n) x 16 k into s[k][row] (leading
// dimension ROWS + 4).  KMAJ: element (row, k) at X[k][row] (cp.async);
// otherwise at X[row][k] (register staging, transposed store).
template <int ROWS, int KMAJ>
struct Slice {
  static constexpr int LD = ROWS + 4;
  static constexpr int Q = ROWS * TBK / 4 / 256;   // 16-byte words per thread
  float4 r[KMAJ ? 1 : Q];
  __device__ __forceinline__ void fetch(float* s, const Mat& X, int64_t r0, int64_t rows, int64_t k0,
                                        int64_t kend) {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int c = threadIdx.x + 256 * q;
      if (KMAJ) {   // word c: k = c / (ROWS / 4), rows 4 (c % (ROWS / 4)) .. + 3
        const int kl = c / (ROWS / 4), rl = (c % (ROWS / 4)) * 4;
        const int64_t rr = r0 + rl, k = k0 + kl;
        const bool ok = rr < rows && k < kend;   // rows % 4 == 0: a word is wholly in or out
        cp_async16(s + kl * LD + rl, ok ? mat_ptr(X, k, rr) : X.p0, ok);
      } else {      // word c: row c % ROWS, k 4 (c / ROWS) .. + 3 (a warp reads 32 rows)
        const int rl = c % ROWS, kl = (c / ROWS) * 4;
        const int64_t rr = r0 + rl, k = k0 + kl;
        if (rr < rows && k + 3 < kend) {
          r[q] = *reinterpret_cast<const float4*>(mat_ptr(X, rr, k));
        } else {
          float t[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) t[u] = (rr < rows && k + u < kend) ? *mat_ptr(X, rr, k + u) : 0.f;
          r[q] = make_float4(t[0], t[1], t[2], t[3]);
        }
      }
    }
  }
  __device__ __forceinline__ void store(float* s) const {
    if constexpr (!KMAJ) {   // k-major slices went to shared memory by cp.async
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const int c = threadIdx.x + 256 * q;
        const int rl = c % ROWS, kl = (c / ROWS) * 4;
        s[(kl + 0) * LD + rl] = r[q].x;
        s[(kl + 1) * LD + rl] = r[q].y;
        s[(kl + 2) * LD + rl] = r[q].z;
        s[(kl + 3) * LD + rl] = r[q].w;
      }
    }
  }
};

__device__ __forceinline__ float4 epi_act(float4 v, int act, const float* aux) {
  if (act == ACT_SILU) {
    v = make_float4(silu_f(v.x), silu_f(v.y), silu_f(v.z), silu_f(v.w));
  } else if (act == ACT_DSILU) {
    const float4 z = *reinterpret_cast<const float4*>(aux);
    float y, d;
    silu_and_grad(z.x, y, d); v.x *= d;
    silu_and_grad(z.y, y, d); v.y *= d;
    silu_and_grad(z.z, y, d); v.z *= d;
    silu_and_grad(z.w, y, d); v.w *= d;
  }
  return v;
}

template <int TM, int A_T, int B_T, int NBN = 2>
__global__ void __launch_bounds__(256, 2) gemm_tiled_kernel(GemmArgs a) {
  static_assert(TM == 4, "fragment loads below cover 4 rows per thread");
  static_assert(NBN == 1 || NBN == 2, "one or two 64-column groups per thread");
  pdl_enter();
  constexpr int BNT = 64 * NBN;   // tile columns
  constexpr int BM = 16 * TM, LDA = BM + 4, LDB = BNT + 4;
  constexpr int SA = TBK * LDA, SB = TBK * LDB;
  extern __shared__ __align__(16) float tsm[];
  float* As = tsm;
  float* Bs = tsm + 2 * SA;
  int tx, ty;
  thread_grid(tx, ty);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BNT;
  int64_t kbeg = 0, kend = a.K;
  if (a.ksplit > 1) {
    int64_t kc = (a.K + a.ksplit - 1) / a.ksplit;
    kc = (kc + TBK - 1) / TBK * TBK;
    kbeg = min(a.K, (int64_t)blockIdx.z * kc);
    kend = min(a.K, kbeg + kc);
  }
  const int64_t nk = (kend - kbeg + TBK - 1) / TBK;
  Slice<BM, A_T> sa;
  Slice<BNT, 1 - B_T> sb;

  float acc[TM][4 * NBN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < 4 * NBN; ++j) acc[i][j] = 0.f;
  // db[m] = sum_k A(m, k): taken by the tx == 0 threads of the first column tile
  const bool do_db = A_T == 1 && a.db != nullptr && blockIdx.x == 0 && tx == 0;
  float dbacc[TM];
#pragma unroll
  for (int i = 0; i < TM; ++i) dbacc[i] = 0.f;

  if (nk > 0) {
    sa.fetch(As, a.A, m0, a.M, kbeg, kend);
    sb.fetch(Bs, a.B, n0, a.N, kbeg, kend);
    cp_async_commit();
    sa.store(As);
    sb.store(Bs);
    cp_async_wait_all();
  }
  __syncthreads();
#pragma unroll 1
  for (int64_t kt = 0; kt < nk; ++kt) {
    const int cur = (int)(kt & 1);
    const bool more = kt + 1 < nk;
    if (more) {   // next slice: copies in flight / loads in registers during the compute
      sa.fetch(As + (cur ^ 1) * SA, a.A, m0, a.M, kbeg + (kt + 1) * TBK, kend);
      sb.fetch(Bs + (cur ^ 1) * SB, a.B, n0, a.N, kbeg + (kt + 1) * TBK, kend);
      cp_async_commit();
    }
    const float* as = As + cur * SA + ty * 4;
    const float* bs = Bs + cur * SB + tx * 4;
#pragma unroll
    for (int k = 0; k < TBK; ++k) {
      float av[TM], bv[4 * NBN];
#pragma unroll
      for (int jj = 0; jj < NBN; ++jj) {
        const float4 b = *reinterpret_cast<const float4*>(bs + k * LDB + 64 * jj);
        bv[4 * jj] = b.x; bv[4 * jj + 1] = b.y; bv[4 * jj + 2] = b.z; bv[4 * jj + 3] = b.w;
      }
      const float4 a0 = *reinterpret_cast<const float4*>(as + k * LDA);
      av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 4 * NBN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      if (do_db) {
#pragma unroll
        for (int i = 0; i < TM; ++i) dbacc[i] += av[i];
      }
    }
    if (more) {
      sa.store(As + (cur ^ 1) * SA);
      sb.store(Bs + (cur ^ 1) * SB);
      cp_async_wait_all();
    }
    __syncthreads();
  }

  auto row_of = [&](int i) { return m0 + ty * 4 + i; };
  if (do_db) {
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t m = row_of(i);
      if (m >= a.M) continue;
      if (a.ksplit > 1) a.db_part[(int64_t)blockIdx.z * a.M + m] = dbacc[i];
      else a.db[m] = dbacc[i];
    }
  }
  Epi e{a.bias, a.pre, a.ldp, a.act, a.aux, a.ldaux, a.resid, a.ldr, a.resid_cols, a.C, a.ldc};
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = row_of(i);
    if (m >= a.M) continue;
#pragma unroll
    for (int jj = 0; jj < NBN; ++jj) {
      const int64_t n = n0 + jj * 64 + tx * 4;
      const float* v4 = &acc[i][jj * 4];
      if (a.ksplit > 1) {
        float* dst = a.part + (int64_t)blockIdx.z * a.M * a.N + m * a.N + n;
        if (n + 3 < a.N) {   // N % 4 == 0 on the split-K path
          *reinterpret_cast<float4*>(dst) = make_float4(v4[0], v4[1], v4[2], v4[3]);
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t)
            if (n + t < a.N) dst[t] = v4[t];
        }
      } else if (a.vec && n + 3 < a.N) {
        float4 v = make_float4(v4[0], v4[1], v4[2], v4[3]);
        if (a.bias) {
          const float4 b = *reinterpret_cast<const float4*>(a.bias + n);
          v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
        }
        if (a.pre) *reinterpret_cast<float4*>(a.pre + m * a.ldp + n) = v;
        v = epi_act(v, a.act, a.aux + m * a.ldaux + n);
        if (a.resid && n < a.resid_cols) {
          const float4 r = *reinterpret_cast<const float4*>(a.resid + m * a.ldr + n);
          v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
        }
        *reinterpret_cast<float4*>(a.C + m * a.ldc + n) = v;
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (n + t < a.N) e.apply(m, n + t, v4[t]);
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A k-major operand (copied 16 bytes at a time): aligned rows, no row split,
// a column split on a 4-element boundary, and a row count that is a multiple
// of 4.  A row-major operand (read as float4 along k): aligned rows, K % 4 == 0,
// a column split on a 4-element boundary.
bool kmajor_ok(const Mat& X, int64_t rows) {
  if (X.split_rows || rows % 4 || !aligned16(X.p0) || X.ld0 % 4) return false;
  if (X.p1 && (!aligned16(X.p1) || X.ld1 % 4 || X.split % 4)) return false;
  return true;
}
bool rowmajor_ok(const Mat& X, int64_t K) {
  if (K % 4 || !aligned16(X.p0) || X.ld0 % 4) return false;
  if (X.p1 && (!aligned16(X.p1) || X.ld1 % 4 || X.split % 4)) return false;
  return true;
}

bool tiled_ok(const GemmArgs& a) {
  if (a.round_bf16) return false;
  if (a.a_t == 1 ? !kmajor_ok(a.A, a.M) : (a.A.split_rows || !rowmajor_ok(a.A, a.K))) return false;
  if (a.b_t == 0 ? !kmajor_ok(a.B, a.N) : !rowmajor_ok(a.B, a.K)) return false;
  if (a.ksplit > 1 && a.N % 4) return false;
  return true;
}

// Whether the epilogue may move four columns at a time.
int vec_epilogue(const GemmArgs& a) {
  if (a.N % 4 || a.ldc % 4 || !aligned16(a.C)) return 0;
  if (a.bias && !aligned16(a.bias)) return 0;
  if (a.pre && (a.ldp % 4 || !aligned16(a.pre))) return 0;
  if (a.act == ACT_DSILU && (a.ldaux % 4 || !aligned16(a.aux))) return 0;
  if (a.resid && (a.ldr % 4 || !aligned16(a.resid) || (a.resid_cols != INT64_MAX && a.resid_cols % 4))) return 0;
  return 1;
}

template <int TM, int A_T, int B_T, int NBN>
int launch_tiled_t(const GemmArgs& a, cudaStream_t s) {
  static uint64_t attr_set = 0;
  constexpr int BNT = 64 * NBN;
  constexpr size_t bytes = tiled_smem_bytes<16 * TM, BNT>();
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(gemm_tiled_kernel<TM, A_T, B_T, NBN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    attr_set |= bit;
  }
  const unsigned z = (unsigned)(a.ksplit > 1 ? a.ksplit : 1);
  const dim3 grid((unsigned)((a.N + BNT - 1) / BNT), (unsigned)((a.M + 16 * TM - 1) / (16 * TM)), z);
  EGNN_CHECK_CUDA(launch_pdl(gemm_tiled_kernel<TM, A_T, B_T, NBN>, grid, dim3(256), bytes, s, a));
  return EGNN_OK;
}

template <int A_T, int B_T>
int launch_tiled_ab(const GemmArgs& a, cudaStream_t s) {
  const int64_t z = a.ksplit > 1 ? a.ksplit : 1;
  const int64_t tiles128 = (a.N + TBN - 1) / TBN * ((a.M + 16 * TTM - 1) / (16 * TTM)) * z;
  if (a.N <= 64 || 2 * tiles128 <= num_sms_current()) return launch_tiled_t<TTM, A_T, B_T, 1>(a, s);
  return launch_tiled_t<TTM, A_T, B_T, 2>(a, s);
}

int launch_tiled(const GemmArgs& a, cudaStream_t s) {
  if (a.a_t == 0 && a.b_t == 0) return launch_tiled_ab<0, 0>(a, s);
  if (a.a_t == 0 && a.b_t == 1) return launch_tiled_ab<0, 1>(a, s);
  if (a.a_t == 1 && a.b_t == 0) return launch_tiled_ab<1, 0>(a, s);
  return launch_tiled_ab<1, 1>(a, s);
}

}  // namespace

int gemm(const GemmArgs& a_in, cudaStream_t s) {
  if (a_in.M <= 0 || a_in.N <= 0) return EGNN_OK;
  GemmArgs a = a_in;
  a.vec = vec_epilogue(a);
  {
    TimerScope ts(a.a_t == 1 ? "node_wgrad" : (tiled_ok(a) ? "node_gemm" : "gemm_small"), s);
    if (tiled_ok(a)) {
      EGNN_TRY(launch_tiled(a, s));
    } else {
      const unsigned z = (unsigned)(a.ksplit > 1 ? a.ksplit : 1);
      dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM), z);
      EGNN_CHECK_CUDA(launch_pdl(gemm_kernel, grid, dim3(NT), 0, s, a));
    }
  }
  EGNN_CHECK_LAUNCH();
  if (a.ksplit > 1) EGNN_TRY(gemm_reduce(a, s));
  return EGNN_OK;
}

int linear_small(int64_t M, int N, int K, const float* x, int64_t ldx, const float* w, int w_nk, const float* b,
                 float* y, int64_t ldy, cudaStream_t s) {
  if (M <= 0 || N <= 0) return EGNN_OK;
  TimerScope ts("linear_small", s);
  if (K <= kSmallK) {
    const int tx = N >= 32 ? 32 : N;
    const int ty = 256 / tx;
    dim3 block(tx, ty);
    const int64_t rows = std::min<int64_t>((M + ty - 1) / ty, 65535);
    dim3 grid((unsigned)((N + tx - 1) / tx), (unsigned)std::max<int64_t>(1, std::min<int64_t>(rows, 4096 / ((N + tx - 1) / tx) + 1)));
    EGNN_CHECK_CUDA(launch_pdl(linear_smallk_kernel, grid, block, 0, s, M, N, K, x, ldx, w, w_nk, b, y, ldy));
  } else if (N == 1) {
    const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((M + 7) / 8, 4096));
    EGNN_CHECK_CUDA(launch_pdl(linear_n1_kernel, dim3(blocks), dim3(256), 0, s, M, K, x, ldx, w, b, y, ldy));
  } else {
    return fail(EGNN_ERR_UNSUPPORTED, "linear_small: shape not covered");
  }
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

bool linear_small_ok(int N, int K) { return K <= kSmallK || N == 1; }

int gemm_reduce(const GemmArgs& a_in, cudaStream_t s) {
  GemmArgs a = a_in;
  a.vec = 0;
  const int64_t total = a.M * a.N;
  const int64_t blocks = (total + 31) / 32 + ((a.db && a.db_part) ? (a.M + 31) / 32 : 0);
  if (blocks == 0) return EGNN_OK;
  TimerScope ts("gemm_reduce", s);
  EGNN_CHECK_CUDA(launch_pdl(gemm_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, s, a));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

bool wgrad_small_ok(int64_t M, int64_t N) {
  const int64_t n1 = N + 1;
  return M >= 1 && std::min(M, n1) <= kNarrowMax && std::max(M, n1) <= 32 * kWideSlots;
}

// Row slices of a weight gradient: for the narrow-side kernel about two
// blocks per SM over all narrow groups with at least 256 rows each, for the
// split-K GEMM about one wave of tiles with at least 128 rows each.
int64_t wgrad_splits(int64_t K, int64_t M, int64_t N) {
  if (wgrad_small_ok(M, N)) {
    const SmallShape sh = small_shape((int)M, (int)N);
    return std::max<int64_t>(1, std::min<int64_t>(K / 256, std::max(1, 296 / sh.groups)));
  }
  int64_t tiles = ((M + 63) / 64) * ((N + 127) / 128);
  int64_t want = (148 + tiles - 1) / tiles;               // about one wave of CTAs
  int64_t by_len = std::max<int64_t>(1, K / 128);         // at least 128 rows per slice
  return std::max<int64_t>(1, std::min<int64_t>({want, by_len, 64}));
}

template <int WS>
int launch_small(int64_t R, int M, int N, const Mat& G, const Mat& X, int64_t S, int64_t rows_per, int vec_w,
                 float* part, cudaStream_t s) {
  static uint64_t attr_set = 0;
  const size_t bytes = small_smem_bytes(WS);
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(wgrad_small_partial_kernel<WS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes));
    attr_set |= bit;
  }
  const dim3 grid((unsigned)S, (unsigned)small_shape(M, N).groups);
  EGNN_CHECK_CUDA(launch_pdl(wgrad_small_partial_kernel<WS>, grid, dim3(256), bytes, s, R, M, N, G, X, rows_per,
                             vec_w, part));
  return EGNN_OK;
}

int wgrad(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw,
          float* db, int round_bf16, float* part, cudaStream_t s) {
  if (!round_bf16 && wgrad_small_ok(M, N) && R > 0) {
    // S slices of the wgrad_splits count, so the caller's split-K workspace
    // (S (M N + M) floats) holds the slices
    const int64_t S = wgrad_splits(R, M, N);
    const int64_t rows_per = (R + S - 1) / S;
    const SmallShape sh = small_shape((int)M, (int)N);
    const Mat& Wm = sh.lanes_n ? X : G;
    const int vec_w = (sh.wide_data % 4 == 0 && !Wm.split_rows && !Wm.p1 && aligned16(Wm.p0) && Wm.ld0 % 4 == 0);
    TimerScope ts("wgrad_small", s);
    switch (sh.slots) {
      case 1: EGNN_TRY(launch_small<1>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 2: EGNN_TRY(launch_small<2>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 3: EGNN_TRY(launch_small<3>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 4: EGNN_TRY(launch_small<4>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 5: EGNN_TRY(launch_small<5>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 6: EGNN_TRY(launch_small<6>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 7: EGNN_TRY(launch_small<7>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      case 8: EGNN_TRY(launch_small<8>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
      default: EGNN_TRY(launch_small<9>(R, (int)M, (int)N, G, X, S, rows_per, vec_w, part, s)); break;
    }
    EGNN_CHECK_LAUNCH();
    const int O = (int)(M * (N + 1));
    EGNN_CHECK_CUDA(launch_pdl(wgrad_small_reduce_kernel, dim3((unsigned)((O + 255) / 256)), dim3(256), 0, s, (int)M,
                               (int)N, (int)S, (const float*)part, dW, lddw, db));
    EGNN_CHECK_LAUNCH();
    return EGNN_OK;
  }
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
  return std::max<int64_t>(1, std::min<int64_t>(128, R / 64));
}

int colsum(int64_t R, int64_t C, Mat G, float* db, float* part, cudaStream_t s) {
  if (C <= 0) return EGNN_OK;
  int64_t S = colsum_splits(R);
  int64_t rows_per = (R + S - 1) / S;
  if (R == 0) rows_per = 1;
  dim3 grid((unsigned)((C + 127) / 128), (unsigned)S);
  TimerScope ts("colsum", s);
  EGNN_CHECK_CUDA(launch_pdl(colsum_partial_kernel, grid, dim3(128), 0, s, R, C, G, rows_per, part));
  EGNN_CHECK_LAUNCH();
  EGNN_CHECK_CUDA(launch_pdl(colsum_reduce_kernel, dim3((unsigned)((C + 127) / 128)), dim3(128), 0, s, C, (int)S,
                             (const float*)part, db));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

}  // namespace egnn
