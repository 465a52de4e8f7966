// Fused EGNN edge kernels, SIMT FFMA path (fp32, or fp32 math on
// bf16-rounded GEMM inputs in bf16 mode).
//
// What one E_GCL does per edge e = (i <- j) (egnn_clean.py:84-103):
//   d = x_i - x_j, r = |d|^2                                   coord2radial :84-93
//   a1 = W1 [h_i, h_j, r, attr] + b1 ; u1 = silu(a1)            edge_mlp.0   :22-24
//   a2 = W2 u1 + b2 ; m = silu(a2)                              edge_mlp.2   :25-26
//   [attention] m <- m sigmoid(wa . m + ba)                     att_mlp      :44-47, :55-57
//   c1 = Wc1 m + bc1 ; phi = wc2 . silu(c1) [tanh]              coord_mlp    :36-42
//   agg_i = sum_e m_e ; x'_i = x_i + mean/sum_e d_e phi_e       :62, :74-81
// W1 [h_i, h_j] is factored into per-node projections P = h Wa^T + b1 and
// Q = h Wb^T (node GEMMs), so each edge needs a1 = P_i + Q_j + w_r r.
//
// Work split: the E CSR edges are cut into G equal contiguous ranges, one
// per CTA, processed in chunks of T edges.  A CTA walks the rows of its range
// in order and writes every row that lies wholly inside it; a row cut by a
// range boundary leaves partial sums in carry slots that edge_fixup adds in
// CTA order.  No atomics: results are bit-identical run to run.
//
// Inside a chunk all per-edge tensors live in shared memory "feature-major"
// (XT[k][e], edges contiguous), which serves both the per-chunk GEMMs
// (C[e][n] = sum_k XT[k][e] B[k][n]) and the weight-gradient products
// (dW[o][k] += sum_e GT[o][e] XT[k][e]) with 16-byte shared loads.
#include <algorithm>

#include "edge_simt.cuh"

namespace egnn {
namespace {

template <int H_>
struct Cfg {
  static constexpr int H = H_;
  static constexpr int NT = 256;
  static constexpr int T = (H >= 256) ? 32 : 64;        // edges per chunk
  static constexpr int TXN = (H / 4 < 16) ? H / 4 : 16; // threads along features
  static constexpr int TY = NT / TXN;                    // threads along edges
  static constexpr int TM = T / TY;                      // edges per thread
  static constexpr int NG = H / (4 * TXN);               // float4 feature groups per thread
  static constexpr int NC = NG * 4;                      // features per thread
  static constexpr int LDT = T + 4;                      // row stride of XT arrays
  static constexpr int KT = (H >= 256) ? 16 : 32;        // weight rows per staged tile
  static constexpr int VC = H + 3;                       // walked columns: H features + 3 coords
  static_assert(TM == 2 || TM == 4, "edges per thread");
  __device__ static int col(int g, int q) { return g * (4 * TXN) + (threadIdx.x % TXN) * 4 + q; }
};

constexpr int kMaxAttr = 16;

// ---- per-chunk GEMM: acc[e][n] += sum_k AT[k][e] * Bg[k][n] ----------------
// Bg is a (H,H) row-major global matrix, staged in KT-row tiles through a
// double buffer Bs with a register prefetch of the next tile.
template <class C>
__device__ __forceinline__ void chunk_gemm(float (&acc)[C::TM][C::NC], const float* AT,
                                           const float* __restrict__ Bg, float* Bs) {
  constexpr int H = C::H, KT = C::KT, NKT = H / KT;
  constexpr int PER = KT * H / 4 / C::NT;
  static_assert(PER >= 1 && PER * 4 * C::NT == KT * H, "tile split");
  const int tid = threadIdx.x;
  const int ty = tid / C::TXN, tx = tid % C::TXN;
  const float4* B4 = reinterpret_cast<const float4*>(Bg);
  float4 pf[PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) pf[p] = __ldg(B4 + tid + C::NT * p);
#pragma unroll
  for (int p = 0; p < PER; ++p) reinterpret_cast<float4*>(Bs)[tid + C::NT * p] = pf[p];
  __syncthreads();
#pragma unroll 1
  for (int kt = 0; kt < NKT; ++kt) {
    if (kt + 1 < NKT) {
#pragma unroll
      for (int p = 0; p < PER; ++p) pf[p] = __ldg(B4 + (kt + 1) * (KT * H / 4) + tid + C::NT * p);
    }
    const float* B = Bs + (kt & 1) * KT * H;
#pragma unroll 4
    for (int kk = 0; kk < KT; ++kk) {
      const float* arow = AT + (kt * KT + kk) * C::LDT + ty * C::TM;
      float a[C::TM];
      if constexpr (C::TM == 4) {
        float4 v = *reinterpret_cast<const float4*>(arow);
        a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
      } else {
        float2 v = *reinterpret_cast<const float2*>(arow);
        a[0] = v.x; a[1] = v.y;
      }
#pragma unroll
      for (int g = 0; g < C::NG; ++g) {
        float4 b = *reinterpret_cast<const float4*>(B + kk * H + g * 4 * C::TXN + tx * 4);
#pragma unroll
        for (int m = 0; m < C::TM; ++m) {
          acc[m][g * 4 + 0] = fmaf(a[m], b.x, acc[m][g * 4 + 0]);
          acc[m][g * 4 + 1] = fmaf(a[m], b.y, acc[m][g * 4 + 1]);
          acc[m][g * 4 + 2] = fmaf(a[m], b.z, acc[m][g * 4 + 2]);
          acc[m][g * 4 + 3] = fmaf(a[m], b.w, acc[m][g * 4 + 3]);
        }
      }
    }
    if (kt + 1 < NKT) {
#pragma unroll
      for (int p = 0; p < PER; ++p)
        reinterpret_cast<float4*>(Bs + ((kt + 1) & 1) * KT * H)[tid + C::NT * p] = pf[p];
    }
    __syncthreads();
  }
}

// Store a thread's GEMM-layout values into a feature-major array XT[col][e].
template <class C, bool ROUND>
__device__ __forceinline__ void store_T(float* XT, const float (&v)[C::TM][C::NC]) {
  const int ty = threadIdx.x / C::TXN;
#pragma unroll
  for (int g = 0; g < C::NG; ++g)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float* dst = XT + C::col(g, q) * C::LDT + ty * C::TM;
      if constexpr (C::TM == 4) {
        *reinterpret_cast<float4*>(dst) =
            make_float4(maybe_bf<ROUND>(v[0][g * 4 + q]), maybe_bf<ROUND>(v[1][g * 4 + q]),
                        maybe_bf<ROUND>(v[2][g * 4 + q]), maybe_bf<ROUND>(v[3][g * 4 + q]));
      } else {
        *reinterpret_cast<float2*>(dst) =
            make_float2(maybe_bf<ROUND>(v[0][g * 4 + q]), maybe_bf<ROUND>(v[1][g * 4 + q]));
      }
    }
}

// Load XT[col][e] for the thread's (edge, feature) slots.
template <class C>
__device__ __forceinline__ float load_T(const float* XT, int m, int g, int q) {
  const int ty = threadIdx.x / C::TXN;
  return XT[C::col(g, q) * C::LDT + ty * C::TM + m];
}

// Sum over the TXN threads that share an edge row.
template <class C>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int off = C::TXN / 2; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// ---- attention gate (egnn_clean.py:44-47, 55-57) --------------------------------
// m <- m * at with at = sigmoid(wa . m + ba) per edge; the dot runs over the
// TXN threads of an edge row, so every one of them gets at[m].
template <class C>
__device__ __forceinline__ void att_gate(float (&acc)[C::TM][C::NC], const float* __restrict__ wa, float ba,
                                         float (&at)[C::TM]) {
  float w[C::NC];
#pragma unroll
  for (int g = 0; g < C::NG; ++g)
#pragma unroll
    for (int q = 0; q < 4; ++q) w[g * 4 + q] = __ldg(wa + C::col(g, q));
#pragma unroll
  for (int m = 0; m < C::TM; ++m) {
    float p = 0.f;
#pragma unroll
    for (int c = 0; c < C::NC; ++c) p = fmaf(acc[m][c], w[c], p);
    at[m] = sigmoidf_(row_sum<C>(p) + ba);
#pragma unroll
    for (int c = 0; c < C::NC; ++c) acc[m][c] *= at[m];
  }
}

// Per-CTA attention scratch of the backward (floats): ungated messages of the
// chunk as float4 [TM][NG][NT] (each thread reads back what it wrote) | gwa
// sums [TY][H] | gba sums [TY] (one owner thread per slot, so no atomics).
template <class C>
constexpr int64_t att_scratch_floats() { return (int64_t)C::T * C::H + (int64_t)C::TY * (C::H + 1); }

// ---- per-chunk weight-gradient product ------------------------------------
// Pw[o][k] += sum_{e<T} GT[o][e] * XT[k][e].  Thread (ot, kt) owns rows
// o = ot + 16 a and columns k = kt + 16 b.
template <class C>
__device__ __forceinline__ void chunk_wgrad(float* __restrict__ Pw, const float* GT, const float* XT) {
  constexpr int H = C::H, R = H / 16, RA = (H >= 256) ? 4 : (R < 8 ? R : 8);
  const int ot = threadIdx.x / 16, kt = threadIdx.x % 16;
#pragma unroll 1
  for (int pass = 0; pass < R / RA; ++pass) {
    float acc[RA][R];
#pragma unroll
    for (int a = 0; a < RA; ++a)
#pragma unroll
      for (int b = 0; b < R; ++b) acc[a][b] = 0.f;
#pragma unroll 1
    for (int e = 0; e < C::T; e += 4) {
      float4 xv[R];
#pragma unroll
      for (int b = 0; b < R; ++b) xv[b] = *reinterpret_cast<const float4*>(XT + (kt + 16 * b) * C::LDT + e);
#pragma unroll
      for (int a = 0; a < RA; ++a) {
        float4 gv = *reinterpret_cast<const float4*>(GT + (ot + 16 * (pass * RA + a)) * C::LDT + e);
#pragma unroll
        for (int b = 0; b < R; ++b) {
          float s = acc[a][b];
          s = fmaf(gv.x, xv[b].x, s);
          s = fmaf(gv.y, xv[b].y, s);
          s = fmaf(gv.z, xv[b].z, s);
          s = fmaf(gv.w, xv[b].w, s);
          acc[a][b] = s;
        }
      }
    }
#pragma unroll
    for (int a = 0; a < RA; ++a)
#pragma unroll
      for (int b = 0; b < R; ++b) {
        int o = ot + 16 * (pass * RA + a), k = kt + 16 * b;
        Pw[o * H + k] += acc[a][b];
      }
  }
}

template <class C>
__device__ __forceinline__ void zero_wgrad(float* __restrict__ Pw) {
  constexpr int H = C::H, R = H / 16;
  const int ot = threadIdx.x / 16, kt = threadIdx.x % 16;
  for (int a = 0; a < R; ++a)
    for (int b = 0; b < R; ++b) Pw[(ot + 16 * a) * H + kt + 16 * b] = 0.f;
}

// ---- row walker --------------------------------------------------------------
// Each thread owns walked columns vc0 = tid and vc1 = tid + 256 (if < H+3).
// Rows are visited in CSR order; a finished row goes to its final place or,
// when it crosses the CTA's range boundary, to a carry slot.
struct Walker {
  int64_t eb, ee;
  int cur;
  float s0, s1;
};

// ---- shared-memory layout ---------------------------------------------------
template <class C>
struct FwdSmem {
  static constexpr size_t uT = 0;
  static constexpr size_t mT = uT + (size_t)C::H * C::LDT;
  static constexpr size_t Bs = mT + (size_t)C::H * C::LDT;
  static constexpr size_t dl = Bs + 2 * (size_t)C::KT * C::H;        // float4[T]
  static constexpr size_t phi = dl + 4 * (size_t)C::T;               // float[T]
  static constexpr size_t rowl = phi + C::T;                         // int[T]
  static constexpr size_t total_floats = rowl + C::T;
  static constexpr size_t bytes = total_floats * 4;
};

template <class C>
struct BwdSmem {
  static constexpr size_t A = (size_t)C::H * C::LDT;
  static constexpr size_t uT = 0;
  static constexpr size_t s1T = uT + A;
  static constexpr size_t mT = s1T + A;
  static constexpr size_t d2T = mT + A;
  static constexpr size_t gT = d2T + A;
  static constexpr size_t Bs = gT + A;
  static constexpr size_t dl = Bs + 2 * (size_t)C::KT * C::H;        // float4[T]: d.xyz, r
  static constexpr size_t gt = dl + 4 * (size_t)C::T;               // float4[T]: g_trans.xyz, 1/norm
  static constexpr size_t gd = gt + 4 * (size_t)C::T;               // float4[T]: dL/dd
  static constexpr size_t phi = gd + 4 * (size_t)C::T;              // float[T]
  static constexpr size_t rowl = phi + C::T;                        // int[T]
  static constexpr size_t attr = rowl + C::T;                       // float[T][kMaxAttr]
  static constexpr size_t att = attr + (size_t)C::T * kMaxAttr;     // float[T]: attention gate
  static constexpr size_t total_floats = att + C::T;
  static constexpr size_t bytes = total_floats * 4;
};

__device__ __forceinline__ float deg_scale(const int32_t* row_ptr, int r, int flags) {
  if (flags & EGNN_FLAG_COORDS_SUM) return 1.f;
  int deg = row_ptr[r + 1] - row_ptr[r];
  return 1.f / (float)max(deg, 1);
}

// ---- gather phase: per-edge geometry and layer-1 activations ---------------
// Warp w handles edge quads; lane l handles features l + 32 c.  Writes
// uT = silu(a1) (bf16-rounded in bf16 mode) and, for the backward, s1T =
// silu'(a1), g_trans and the edge attributes.
template <class C, bool BF, bool BWD>
__device__ __forceinline__ void gather_phase(const EdgeCommon& a, int64_t c0, int n, float* sm,
                                             size_t off_uT, size_t off_s1T, size_t off_dl,
                                             size_t off_gt, size_t off_rowl, size_t off_attr,
                                             const float* gx_out) {
  constexpr int H = C::H, CC = H / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* uT = sm + off_uT;
  float4* dl = reinterpret_cast<float4*>(sm + off_dl);
  int* rowl = reinterpret_cast<int*>(sm + off_rowl);
  const bool normalize = a.flags & EGNN_FLAG_NORMALIZE;
  for (int qd = warp; qd < C::T / 4; qd += C::NT / 32) {
    const int e0 = qd * 4;
    float u[CC][4];
    float s1[CC][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int e = e0 + t;
      if (e < n) {
        const int64_t k = c0 + e;
        const int i = a.row_idx[k], j = a.col_idx[k];
        const float4 xi = a.xp[i], xj = a.xp[j];
        const float dx = xi.x - xj.x, dy = xi.y - xj.y, dz = xi.z - xj.z;
        const float r = dx * dx + dy * dy + dz * dz;
        float inv = 1.f;
        if (normalize) inv = 1.f / (sqrtf(r) + 1e-8f);
        // A self-loop's d = x_i - x_i adds +g to x_i and -g to the same x_i:
        // its coordinate gradient is exactly zero, so drop it rather than let
        // the 1/(|d| + eps) factor of normalize=True blow up the cancellation.
        const float inv_g = (i == j) ? 0.f : inv;
        const float* Pi = a.PQ + (int64_t)i * 2 * H;
        const float* Qj = a.PQ + (int64_t)j * 2 * H + H;
        int eid = 0;
        if (a.d) eid = a.edge_id[k];
        if (lane == 0) {
          rowl[e] = i;
          if constexpr (BWD) {
            dl[e] = make_float4(dx, dy, dz, r);
            const float sc = deg_scale(a.row_ptr, i, a.flags);
            float4* gt = reinterpret_cast<float4*>(sm + off_gt);
            gt[e] = make_float4(gx_out[i * 3 + 0] * sc, gx_out[i * 3 + 1] * sc, gx_out[i * 3 + 2] * sc, inv_g);
          } else {
            dl[e] = make_float4(dx * inv, dy * inv, dz * inv, r);
          }
        }
        if constexpr (BWD) {
          if (lane < a.d) sm[off_attr + e * kMaxAttr + lane] = a.attr[(int64_t)eid * a.d + lane];
        }
#pragma unroll
        for (int c = 0; c < CC; ++c) {
          const int f = lane + 32 * c;
          float v = Pi[f] + Qj[f] + a.wr[f] * r;
          for (int t2 = 0; t2 < a.d; ++t2) v = fmaf(a.attr[(int64_t)eid * a.d + t2], a.We[f * a.d + t2], v);
          if constexpr (BWD) {
            float y, dy1;
            silu_and_grad(v, y, dy1);
            u[c][t] = maybe_bf<BF>(y);
            s1[c][t] = dy1;
          } else {
            u[c][t] = maybe_bf<BF>(silu_f(v));
          }
        }
      } else {
        if (lane == 0) {
          rowl[e] = 0x7fffffff;
          dl[e] = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (BWD) reinterpret_cast<float4*>(sm + off_gt)[e] = make_float4(0.f, 0.f, 0.f, 1.f);
        }
        if constexpr (BWD) {
          if (lane < a.d) sm[off_attr + e * kMaxAttr + lane] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < CC; ++c) { u[c][t] = 0.f; s1[c][t] = 0.f; }
      }
    }
#pragma unroll
    for (int c = 0; c < CC; ++c) {
      const int f = lane + 32 * c;
      *reinterpret_cast<float4*>(uT + f * C::LDT + e0) = make_float4(u[c][0], u[c][1], u[c][2], u[c][3]);
      if constexpr (BWD)
        *reinterpret_cast<float4*>(sm + off_s1T + f * C::LDT + e0) =
            make_float4(s1[c][0], s1[c][1], s1[c][2], s1[c][3]);
    }
  }
}

// ---- forward kernel -----------------------------------------------------------
template <int H, bool BF>
__global__ void __launch_bounds__(256) edge_fwd_kernel(EdgeFwdArgs a) {
  pdl_enter();
  using C = Cfg<H>;
  using S = FwdSmem<C>;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* uT = sm + S::uT;
  float* mT = sm + S::mT;
  float* Bs = sm + S::Bs;
  const float4* dl = reinterpret_cast<const float4*>(sm + S::dl);
  float* phi = sm + S::phi;
  const int* rowl = reinterpret_cast<const int*>(sm + S::rowl);

  const int tid = threadIdx.x, ty = tid / C::TXN, tx = tid % C::TXN;
  const int cta = blockIdx.x, G = gridDim.x;
  const int64_t eb = std::min<int64_t>(a.E, (int64_t)cta * a.epc);
  const int64_t ee = std::min<int64_t>(a.E, eb + a.epc);
  const int N = (int)a.N;
  int cur = (cta == 0) ? 0 : a.row_idx[eb];
  const int end_row = (cta == G - 1) ? N : a.row_idx[ee];
  if (tid == 0) { a.carry_row[cta * 2] = -1; a.carry_row[cta * 2 + 1] = -1; }
  const int vc0 = tid, vc1 = tid + 256;
  float s0 = 0.f, s1 = 0.f;
  const bool tanh_ = a.flags & EGNN_FLAG_TANH;

  auto colval = [&](int vc, int e) -> float {
    if (vc < H) return mT[vc * C::LDT + e];
    const float4 d = dl[e];
    const float c = (vc == H) ? d.x : (vc == H + 1 ? d.y : d.z);
    return c * phi[e];
  };
  auto final_write = [&](int r, int vc, float v) {
    if (vc < H) a.agg[(int64_t)r * H + vc] = v;
    else if (vc < H + 3) {
      const int dd = vc - H;
      a.x_out[(int64_t)r * 3 + dd] = a.x[(int64_t)r * 3 + dd] + v * deg_scale(a.row_ptr, r, a.flags);
    }
  };
  auto carry_write = [&](int slot, int r, int vc, float v) {
    if (vc < C::VC) a.carry[((int64_t)cta * 2 + slot) * (H + 4) + vc] = v;
    if (tid == 0) a.carry_row[cta * 2 + slot] = r;
  };
  auto flush = [&](int r) {
    const bool before = a.row_ptr[r] < eb;
    if (!before) {
      if (vc0 < C::VC) final_write(r, vc0, s0);
      if (vc1 < C::VC) final_write(r, vc1, s1);
    } else {
      carry_write(0, r, vc0, s0);
      if (vc1 < C::VC) carry_write(0, r, vc1, s1);
    }
  };

#pragma unroll 1
  for (int64_t c0 = eb; c0 < ee; c0 += C::T) {
    const int n = (int)std::min<int64_t>(C::T, ee - c0);
    gather_phase<C, BF, false>(a, c0, n, sm, S::uT, 0, S::dl, 0, S::rowl, 0, nullptr);
    __syncthreads();

    // m = silu(W2 u1 + b2)
    float acc[C::TM][C::NC];
#pragma unroll
    for (int g = 0; g < C::NG; ++g)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = a.b2[C::col(g, q)];
#pragma unroll
        for (int m = 0; m < C::TM; ++m) acc[m][g * 4 + q] = b;
      }
    chunk_gemm<C>(acc, uT, a.W2T, Bs);
#pragma unroll
    for (int m = 0; m < C::TM; ++m)
#pragma unroll
      for (int c = 0; c < C::NC; ++c) acc[m][c] = silu_f(acc[m][c]);
    if (a.flags & EGNN_FLAG_ATTENTION) {
      float at[C::TM];
      att_gate<C>(acc, a.wa, __ldg(a.ba), at);
    }
    store_T<C, false>(mT, acc);
    if constexpr (BF) store_T<C, true>(uT, acc);
    __syncthreads();

    // phi = wc2 . silu(Wc1 m + bc1)
#pragma unroll
    for (int g = 0; g < C::NG; ++g)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = a.bc1[C::col(g, q)];
#pragma unroll
        for (int m = 0; m < C::TM; ++m) acc[m][g * 4 + q] = b;
      }
    chunk_gemm<C>(acc, BF ? uT : mT, a.Wc1T, Bs);
    float ph[C::TM];
#pragma unroll
    for (int m = 0; m < C::TM; ++m) {
      float p = 0.f;
#pragma unroll
      for (int g = 0; g < C::NG; ++g)
#pragma unroll
        for (int q = 0; q < 4; ++q) p = fmaf(silu_f(acc[m][g * 4 + q]), a.wc2[C::col(g, q)], p);
      ph[m] = row_sum<C>(p);
    }
    if (tx == 0) {
#pragma unroll
      for (int m = 0; m < C::TM; ++m) phi[ty * C::TM + m] = tanh_ ? tanhf(ph[m]) : ph[m];
    }
    __syncthreads();

    // walk rows: agg (columns < H) and coordinate updates (columns H..H+2)
#pragma unroll 1
    for (int e = 0; e < n; ++e) {
      const int r = rowl[e];
      while (cur < r) { flush(cur); ++cur; s0 = 0.f; s1 = 0.f; }
      if (vc0 < C::VC) s0 += colval(vc0, e);
      if (vc1 < C::VC) s1 += colval(vc1, e);
    }
    __syncthreads();
  }
  while (cur < end_row) { flush(cur); ++cur; s0 = 0.f; s1 = 0.f; }
  if (cur == end_row && end_row < N && a.row_ptr[end_row] < ee) {
    const int slot = (a.row_ptr[cur] < eb) ? 0 : 1;
    carry_write(slot, cur, vc0, s0);
    if (vc1 < C::VC) carry_write(slot, cur, vc1, s1);
  }
}

// ---- backward kernel (dst pass) --------------------------------------------------
template <int H, bool BF>
__global__ void __launch_bounds__(256) edge_bwd_kernel(EdgeBwdArgs a) {
  pdl_enter();
  using C = Cfg<H>;
  using S = BwdSmem<C>;
  extern __shared__ float4 smem_b4[];
  float* sm = reinterpret_cast<float*>(smem_b4);
  float* uT = sm + S::uT;
  float* s1T = sm + S::s1T;
  float* mT = sm + S::mT;
  float* d2T = sm + S::d2T;
  float* gT = sm + S::gT;
  float* Bs = sm + S::Bs;
  const float4* dl = reinterpret_cast<const float4*>(sm + S::dl);
  const float4* gtr = reinterpret_cast<const float4*>(sm + S::gt);
  float4* gd = reinterpret_cast<float4*>(sm + S::gd);
  float* phi = sm + S::phi;
  const int* rowl = reinterpret_cast<const int*>(sm + S::rowl);
  const float* attr_s = sm + S::attr;
  float* att_s = sm + S::att;

  const int tid = threadIdx.x, ty = tid / C::TXN, tx = tid % C::TXN;
  const int cta = blockIdx.x, G = gridDim.x;
  const int64_t eb = std::min<int64_t>(a.E, (int64_t)cta * a.epc);
  const int64_t ee = std::min<int64_t>(a.E, eb + a.epc);
  const int N = (int)a.N;
  const int PF = (int)edge_part_floats(H, a.d);
  float* part = a.part + (int64_t)cta * PF;
  float* pWc1 = part;
  float* pW2 = part + H * H;
  zero_wgrad<C>(pWc1);
  zero_wgrad<C>(pW2);

  const bool att = a.flags & EGNN_FLAG_ATTENTION;
  float* const scr = att ? a.att_scr + (int64_t)cta * att_scratch_floats<C>() : nullptr;
  float4* const att_n = reinterpret_cast<float4*>(scr);
  float* const att_wa = att ? scr + C::T * H : nullptr;
  float* const att_ba = att ? att_wa + C::TY * H : nullptr;
  if (att) {
#pragma unroll
    for (int g = 0; g < C::NG; ++g)
#pragma unroll
      for (int q = 0; q < 4; ++q) att_wa[ty * H + C::col(g, q)] = 0.f;
    if (tx == 0) att_ba[ty] = 0.f;
  }

  int cur = (cta == 0) ? 0 : a.row_idx[eb];
  const int end_row = (cta == G - 1) ? N : a.row_idx[ee];
  if (tid == 0) { a.carry_row[cta * 2] = -1; a.carry_row[cta * 2 + 1] = -1; }
  const int vc0 = tid, vc1 = tid + 256;
  float s0 = 0.f, s1 = 0.f;
  float gwe[kMaxAttr];
#pragma unroll
  for (int t = 0; t < kMaxAttr; ++t) gwe[t] = 0.f;
  const bool tanh_ = a.flags & EGNN_FLAG_TANH;
  const bool normalize = a.flags & EGNN_FLAG_NORMALIZE;

  float v_bc1[C::NC], v_b2[C::NC], v_wc2[C::NC], v_wr[C::NC];
#pragma unroll
  for (int c = 0; c < C::NC; ++c) { v_bc1[c] = 0.f; v_b2[c] = 0.f; v_wc2[c] = 0.f; v_wr[c] = 0.f; }

  auto colval = [&](int vc, int e) -> float {
    if (vc < H) return gT[vc * C::LDT + e];
    const float4 d = gd[e];
    return (vc == H) ? d.x : (vc == H + 1 ? d.y : d.z);
  };
  auto final_write = [&](int r, int vc, float v) {
    if (vc < H) a.S_dst[(int64_t)r * H + vc] = v;
    else if (vc < H + 3) a.gxd[(int64_t)r * 3 + (vc - H)] = v;
  };
  auto carry_write = [&](int slot, int r, int vc, float v) {
    if (vc < C::VC) a.carry[((int64_t)cta * 2 + slot) * (H + 4) + vc] = v;
    if (tid == 0) a.carry_row[cta * 2 + slot] = r;
  };
  auto flush = [&](int r) {
    const bool before = a.row_ptr[r] < eb;
    if (!before) {
      if (vc0 < C::VC) final_write(r, vc0, s0);
      if (vc1 < C::VC) final_write(r, vc1, s1);
    } else {
      carry_write(0, r, vc0, s0);
      if (vc1 < C::VC) carry_write(0, r, vc1, s1);
    }
  };

#pragma unroll 1
  for (int64_t c0 = eb; c0 < ee; c0 += C::T) {
    const int n = (int)std::min<int64_t>(C::T, ee - c0);
    gather_phase<C, BF, true>(a, c0, n, sm, S::uT, S::s1T, S::dl, S::gt, S::rowl, S::attr, a.gx_out);
    __syncthreads();

    // recompute m = silu(a2), keep silu'(a2)
    float acc[C::TM][C::NC];
    float aux[C::TM][C::NC];
#pragma unroll
    for (int g = 0; g < C::NG; ++g)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = a.b2[C::col(g, q)];
#pragma unroll
        for (int m = 0; m < C::TM; ++m) acc[m][g * 4 + q] = b;
      }
    chunk_gemm<C>(acc, uT, a.W2T, Bs);
#pragma unroll
    for (int m = 0; m < C::TM; ++m)
#pragma unroll
      for (int c = 0; c < C::NC; ++c) {
        float y, dy;
        silu_and_grad(acc[m][c], y, dy);
        acc[m][c] = y;
        aux[m][c] = dy;
      }
    if (att) {
      // park the ungated messages for the gate's backward, then gate
#pragma unroll
      for (int m = 0; m < C::TM; ++m)
#pragma unroll
        for (int g = 0; g < C::NG; ++g)
          att_n[(m * C::NG + g) * C::NT + tid] =
              make_float4(acc[m][g * 4 + 0], acc[m][g * 4 + 1], acc[m][g * 4 + 2], acc[m][g * 4 + 3]);
      float at[C::TM];
      att_gate<C>(acc, a.wa, __ldg(a.ba), at);
      if (tx == 0) {
#pragma unroll
        for (int m = 0; m < C::TM; ++m) att_s[ty * C::TM + m] = at[m];
      }
    }
    store_T<C, BF>(mT, acc);
    store_T<C, false>(d2T, aux);
    __syncthreads();

    // recompute c1, phi; backward through phi_x
#pragma unroll
    for (int g = 0; g < C::NG; ++g)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float b = a.bc1[C::col(g, q)];
#pragma unroll
        for (int m = 0; m < C::TM; ++m) acc[m][g * 4 + q] = b;
      }
    chunk_gemm<C>(acc, mT, a.Wc1T, Bs);
#pragma unroll
    for (int m = 0; m < C::TM; ++m) {
      float p = 0.f;
#pragma unroll
      for (int g = 0; g < C::NG; ++g)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float y, dy;
          silu_and_grad(acc[m][g * 4 + q], y, dy);
          acc[m][g * 4 + q] = y;      // v = silu(c1)
          aux[m][g * 4 + q] = dy;     // silu'(c1)
          p = fmaf(y, a.wc2[C::col(g, q)], p);
        }
      p = row_sum<C>(p);
      const int e = ty * C::TM + m;
      const float4 d = dl[e];
      const float4 gt = gtr[e];
      float ph = p, gph;
      if (normalize) {
        gph = (gt.x * d.x + gt.y * d.y + gt.z * d.z) * gt.w;
      } else {
        gph = gt.x * d.x + gt.y * d.y + gt.z * d.z;
      }
      if (tanh_) {
        ph = tanhf(p);
        gph *= (1.f - ph * ph);
      }
      if (tx == 0) phi[e] = ph;
#pragma unroll
      for (int g = 0; g < C::NG; ++g)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = g * 4 + q;
          v_wc2[c] = fmaf(gph, acc[m][c], v_wc2[c]);
          const float gc1 = gph * a.wc2[C::col(g, q)] * aux[m][c];
          v_bc1[c] += gc1;
          acc[m][c] = gc1;
        }
    }
    store_T<C, BF>(gT, acc);   // g_c1
    __syncthreads();

    // dWc1 += g_c1^T m ;  g_m = g_c1 Wc1 + g_agg[i] ;  g_a2 = g_m * silu'(a2)
    chunk_wgrad<C>(pWc1, gT, mT);
#pragma unroll
    for (int m = 0; m < C::TM; ++m) {
      const int e = ty * C::TM + m;
#pragma unroll
      for (int g = 0; g < C::NG; ++g) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < n) v = *reinterpret_cast<const float4*>(a.g_agg + (int64_t)rowl[e] * (a.ld_gagg ? a.ld_gagg : H) + C::col(g, 0));
        acc[m][g * 4 + 0] = v.x; acc[m][g * 4 + 1] = v.y;
        acc[m][g * 4 + 2] = v.z; acc[m][g * 4 + 3] = v.w;
      }
    }
    chunk_gemm<C>(acc, gT, a.Wc1, Bs);
    if (att) {
      // g_m is dL/d(n at): dL/dn = g_m at + gs wa with gs = (g_m . n) at (1 - at);
      // gwa += gs n, gba += gs
#pragma unroll
      for (int m = 0; m < C::TM; ++m) {
        const float at = att_s[ty * C::TM + m];
        float nv[C::NC];
#pragma unroll
        for (int g = 0; g < C::NG; ++g) {
          const float4 t = att_n[(m * C::NG + g) * C::NT + tid];
          nv[g * 4 + 0] = t.x; nv[g * 4 + 1] = t.y; nv[g * 4 + 2] = t.z; nv[g * 4 + 3] = t.w;
        }
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < C::NC; ++c) dot = fmaf(acc[m][c], nv[c], dot);
        const float gs = row_sum<C>(dot) * at * (1.f - at);
#pragma unroll
        for (int g = 0; g < C::NG; ++g)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int c = g * 4 + q, f = C::col(g, q);
            att_wa[ty * H + f] = fmaf(gs, nv[c], att_wa[ty * H + f]);
            acc[m][c] = fmaf(acc[m][c], at, gs * __ldg(a.wa + f));
          }
        if (tx == 0) att_ba[ty] += gs;
      }
    }
#pragma unroll
    for (int m = 0; m < C::TM; ++m)
#pragma unroll
      for (int g = 0; g < C::NG; ++g)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = g * 4 + q;
          const float ga2 = acc[m][c] * load_T<C>(d2T, m, g, q);
          v_b2[c] += ga2;
          acc[m][c] = ga2;
        }
    store_T<C, BF>(gT, acc);   // g_a2 (chunk_gemm ended with a barrier)
    __syncthreads();

    // dW2 += g_a2^T u1 ;  g_u1 = g_a2 W2 ;  g_a1 = g_u1 * silu'(a1)
    chunk_wgrad<C>(pW2, gT, uT);
#pragma unroll
    for (int m = 0; m < C::TM; ++m)
#pragma unroll
      for (int c = 0; c < C::NC; ++c) acc[m][c] = 0.f;
    chunk_gemm<C>(acc, gT, a.W2, Bs);
#pragma unroll
    for (int m = 0; m < C::TM; ++m) {
      const int e = ty * C::TM + m;
      const float4 d = dl[e];
      float pr = 0.f;
#pragma unroll
      for (int g = 0; g < C::NG; ++g)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = g * 4 + q;
          const float ga1 = acc[m][c] * load_T<C>(s1T, m, g, q);
          acc[m][c] = ga1;
          pr = fmaf(ga1, a.wr[C::col(g, q)], pr);
          v_wr[c] = fmaf(ga1, d.w, v_wr[c]);
        }
      const float gr = row_sum<C>(pr);
      if (e < n) {
#pragma unroll
        for (int g = 0; g < C::NG; ++g)
          *reinterpret_cast<float4*>(a.gstore + (c0 + e) * H + C::col(g, 0)) =
              make_float4(acc[m][g * 4 + 0], acc[m][g * 4 + 1], acc[m][g * 4 + 2], acc[m][g * 4 + 3]);
      }
      if (tx == 0) {
        // d(loss)/d(x_i - x_j): through trans = dn * phi, dn = d / norm (norm detached),
        // and through r = |d|^2.
        const float4 gt = gtr[e];
        const float ph = phi[e];
        float4 g4;
        g4.x = gt.x * ph * gt.w + 2.f * gr * d.x;
        g4.y = gt.y * ph * gt.w + 2.f * gr * d.y;
        g4.z = gt.z * ph * gt.w + 2.f * gr * d.z;
        g4.w = 0.f;
        if (e >= n) g4 = make_float4(0.f, 0.f, 0.f, 0.f);
        gd[e] = g4;
        if (e < n) a.gdstore[c0 + e] = g4;
      }
    }
    store_T<C, false>(gT, acc);  // g_a1 in fp32 for the row sums
    __syncthreads();

    // walk rows: S_dst (columns < H), gxd (H..H+2), dWe via the attributes
#pragma unroll 1
    for (int e = 0; e < n; ++e) {
      const int r = rowl[e];
      while (cur < r) { flush(cur); ++cur; s0 = 0.f; s1 = 0.f; }
      if (vc0 < C::VC) {
        const float v = colval(vc0, e);
        s0 += v;
        if (vc0 < H) {
#pragma unroll
          for (int t = 0; t < kMaxAttr; ++t)
            if (t < a.d) gwe[t] = fmaf(v, attr_s[e * kMaxAttr + t], gwe[t]);
        }
      }
      if (vc1 < C::VC) s1 += colval(vc1, e);
    }
    __syncthreads();
  }
  while (cur < end_row) { flush(cur); ++cur; s0 = 0.f; s1 = 0.f; }
  if (cur == end_row && end_row < N && a.row_ptr[end_row] < ee) {
    const int slot = (a.row_ptr[cur] < eb) ? 0 : 1;
    carry_write(slot, cur, vc0, s0);
    if (vc1 < C::VC) carry_write(slot, cur, vc1, s1);
  }

  // reduce the per-thread vector partials over the TY edge rows, in order
  __syncthreads();
  float* red = sm;  // reuse: [4][TY][H]
#pragma unroll
  for (int g = 0; g < C::NG; ++g)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int f = C::col(g, q), c = g * 4 + q;
      red[(0 * C::TY + ty) * H + f] = v_bc1[c];
      red[(1 * C::TY + ty) * H + f] = v_b2[c];
      red[(2 * C::TY + ty) * H + f] = v_wc2[c];
      red[(3 * C::TY + ty) * H + f] = v_wr[c];
    }
  __syncthreads();
  for (int idx = tid; idx < 4 * H; idx += C::NT) {
    const int v = idx / H, f = idx % H;
    float s = 0.f;
    for (int y = 0; y < C::TY; ++y) s += red[(v * C::TY + y) * H + f];
    part[2 * H * H + v * H + f] = s;
  }
  if (tid < H) {
#pragma unroll
    for (int t = 0; t < kMaxAttr; ++t)
      if (t < a.d) part[2 * H * H + 4 * H + tid * a.d + t] = gwe[t];
  }
  if (att) {   // the barriers above order every thread's scratch updates
    const int64_t off = edge_part_att(H, a.d);
    for (int f = tid; f < H; f += C::NT) {
      float sacc = 0.f;
      for (int y = 0; y < C::TY; ++y) sacc += att_wa[y * H + f];
      part[off + f] = sacc;
    }
    if (tid == 0) {
      float sacc = 0.f;
      for (int y = 0; y < C::TY; ++y) sacc += att_ba[y];
      part[off + H] = sacc;
    }
  }
}

// ---- boundary fix-up -----------------------------------------------------------
// One block per CTA boundary c (1..G-1).  If the boundary cuts a row and it is
// the first boundary inside that row, sum the row's partials in CTA order:
// tail slot of CTA c-1, then head slots of CTAs c, c+1, ... inside the row.
template <bool BWD>
__global__ void edge_fixup_kernel(int H, int64_t E, int G, int64_t epc, const int32_t* row_ptr,
                                  const int32_t* row_idx, const float* carry, int flags,
                                  const float* x, float* out_h, float* out_x) {
  pdl_enter();
  const int c = blockIdx.x + 1;
  const int64_t b = (int64_t)c * epc;
  if (c >= G || b >= E || b == 0) return;
  const int r = row_idx[b];
  if (row_idx[b - 1] != r) return;
  const int64_t rs = row_ptr[r], re = row_ptr[r + 1];
  if ((int64_t)(c - 1) * epc > rs) return;
  for (int vc = threadIdx.x; vc < H + 3; vc += blockDim.x) {
    float s = carry[((int64_t)(c - 1) * 2 + 1) * (H + 4) + vc];
    for (int cc = c; cc < G && (int64_t)cc * epc < re; ++cc) s += carry[((int64_t)cc * 2) * (H + 4) + vc];
    if (vc < H) {
      out_h[(int64_t)r * H + vc] = s;
    } else if (BWD) {
      out_x[(int64_t)r * 3 + vc - H] = s;
    } else {
      const int dd = vc - H;
      float sc = 1.f;
      if (!(flags & EGNN_FLAG_COORDS_SUM)) sc = 1.f / (float)max((int)(re - rs), 1);
      out_x[(int64_t)r * 3 + dd] = x[(int64_t)r * 3 + dd] + s * sc;
    }
  }
}

// ---- source pass -----------------------------------------------------------------
template <int H, typename T>
__global__ void src_pass_kernel(int64_t N, const int32_t* __restrict__ src_ptr,
                                const int32_t* __restrict__ src_edge, const T* __restrict__ gstore,
                                const float4* __restrict__ gdstore, const float* __restrict__ gx_out,
                                const float* __restrict__ gxd, float* __restrict__ S_src,
                                float* __restrict__ gx) {
  pdl_enter();
  // One warp per source node; lane owns the H / 32 consecutive features
  // lane*VW .. +VW-1.  Edge rows are fetched four at a time (indices first),
  // and added in increasing CSR-position order as before.
  constexpr int VW = H / 32;
  const int lane = threadIdx.x % 32;
  const int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (j >= N) return;
  float s[VW];
#pragma unroll
  for (int c = 0; c < VW; ++c) s[c] = 0.f;
  float gs = 0.f;
  const int kb = src_ptr[j], ke = src_ptr[j + 1];
  int k = kb;
  for (; k + 4 <= ke; k += 4) {
    int64_t p[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) p[u] = src_edge[k + u];
    float v[4][VW];
#pragma unroll
    for (int u = 0; u < 4; ++u) load_row_slice<H>(gstore + p[u] * H, lane, v[u]);
    float4 g[4];
    if (lane < 3) {
#pragma unroll
      for (int u = 0; u < 4; ++u) g[u] = gdstore[p[u]];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int c = 0; c < VW; ++c) s[c] += v[u][c];
      if (lane < 3) gs += (lane == 0) ? g[u].x : (lane == 1 ? g[u].y : g[u].z);
    }
  }
  for (; k < ke; ++k) {
    const int64_t p = src_edge[k];
    float v[VW];
    load_row_slice<H>(gstore + p * H, lane, v);
#pragma unroll
    for (int c = 0; c < VW; ++c) s[c] += v[c];
    if (lane < 3) {
      const float4 g = gdstore[p];
      gs += (lane == 0) ? g.x : (lane == 1 ? g.y : g.z);
    }
  }
  store_row_slice<H>(S_src + j * H, lane, s);
  if (lane < 3) gx[j * 3 + lane] = gx_out[j * 3 + lane] + gxd[j * 3 + lane] - gs;
}

// Per-CTA weight-gradient partials -> parameter gradients.  A block takes 32
// consecutive slots (one per lane); its 8 warps each add a contiguous eighth
// of the CTA partials (eight loads in flight), and warp 0 adds the 8 sums in
// warp order (a fixed association: bit-reproducible).
__global__ void __launch_bounds__(256) part_reduce_kernel(int H, int d, int att, int G, int64_t PF,
                                                          const float* part, egnn_layer_grads gp, int64_t ld_w1,
                                                          int64_t c_r) {
  pdl_enter();
  __shared__ float red[8][33];
  const int64_t total = edge_part_att(H, d) + (att ? H + 1 : 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t idx = (int64_t)blockIdx.x * 32 + lane;
  const int per = (G + 7) / 8;
  const int c0 = min(G, warp * per), c1 = min(G, c0 + per);
  float v = 0.f;
  if (idx < total) {
    for (int c = c0; c < c1; c += 8) {
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = (c + u < c1) ? part[(int64_t)(c + u) * PF + idx] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) v += t[u];
    }
  }
  red[warp][lane] = v;
  __syncthreads();
  if (warp != 0 || idx >= total) return;
  float s = red[0][lane];
#pragma unroll
  for (int w = 1; w < 8; ++w) s += red[w][lane];
  const int64_t HH = (int64_t)H * H;
  if (idx < HH) {
    gp.coord_w1[idx] = s;
  } else if (idx < 2 * HH) {
    gp.edge_w2[idx - HH] = s;
  } else {
    const int64_t v2 = idx - 2 * HH;
    if (v2 < H) gp.coord_b1[v2] = s;
    else if (v2 < 2 * H) gp.edge_b2[v2 - H] = s;
    else if (v2 < 3 * H) gp.coord_w2[v2 - 2 * H] = s;
    else if (v2 < 4 * H) gp.edge_w1[(v2 - 3 * H) * ld_w1 + c_r] = s;
    else if (v2 < 4 * H + (int64_t)H * d) {
      const int64_t w = v2 - 4 * H;
      const int64_t f = w / d, t = w % d;
      gp.edge_w1[f * ld_w1 + c_r + 1 + t] = s;
    } else {
      const int64_t w = v2 - 4 * H - (int64_t)H * d;
      if (w < H) gp.att_w[w] = s;
      else gp.att_b[0] = s;
    }
  }
}

// ---- host-side dispatch -------------------------------------------------------------
template <int H, bool BF>
int launch_fwd(const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
  using C = Cfg<H>;
  constexpr size_t bytes = FwdSmem<C>::bytes;
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(edge_fwd_kernel<H, BF>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    attr_set |= bit;
  }
  {
    TimerScope ts("edge_fwd", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_fwd_kernel<H, BF>, dim3(g.G), dim3(C::NT), bytes, s, a));
  }
  EGNN_CHECK_LAUNCH();
  if (g.G > 1) {
    TimerScope ts_fix("edge_fixup", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_fixup_kernel<false>, dim3(g.G - 1), dim3(128), 0, s, H, a.E, g.G, g.epc,
                               a.row_ptr, a.row_idx, (const float*)a.carry, a.flags, a.x, a.agg, a.x_out));
    EGNN_CHECK_LAUNCH();
  }
  return EGNN_OK;
}

template <int H, bool BF>
int launch_bwd(const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
  using C = Cfg<H>;
  constexpr size_t bytes = BwdSmem<C>::bytes;
  static_assert(4 * C::TY * H <= BwdSmem<C>::Bs, "reduction scratch must fit");
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(edge_bwd_kernel<H, BF>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    attr_set |= bit;
  }
  {
    TimerScope ts("edge_bwd", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_bwd_kernel<H, BF>, dim3(g.G), dim3(C::NT), bytes, s, a));
  }
  EGNN_CHECK_LAUNCH();
  if (g.G > 1) {
    TimerScope ts_fix("edge_fixup", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_fixup_kernel<true>, dim3(g.G - 1), dim3(128), 0, s, H, a.E, g.G, g.epc,
                               a.row_ptr, a.row_idx, (const float*)a.carry, a.flags, (const float*)nullptr,
                               a.S_dst, a.gxd));
    EGNN_CHECK_LAUNCH();
  }
  return EGNN_OK;
}

template <int H>
size_t smem_bytes(bool bwd) {
  return bwd ? BwdSmem<Cfg<H>>::bytes : FwdSmem<Cfg<H>>::bytes;
}

template <int H, bool BF>
int occupancy(bool bwd, int* out) {
  size_t bytes = smem_bytes<H>(bwd);
  int n = 0;
  cudaError_t e;
  if (bwd) {
    e = cudaFuncSetAttribute(edge_bwd_kernel<H, BF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, edge_bwd_kernel<H, BF>, 256, bytes);
  } else {
    e = cudaFuncSetAttribute(edge_fwd_kernel<H, BF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, edge_fwd_kernel<H, BF>, 256, bytes);
  }
  if (e != cudaSuccess) return fail(EGNN_ERR_CUDA, "occupancy query failed: %s", cudaGetErrorString(e));
  *out = std::max(1, n);
  return EGNN_OK;
}

}  // namespace

int edge_chunk(int H) { return H >= 256 ? 32 : 64; }

int64_t edge_att_scratch_floats(int H) {
  switch (H) {
    case 32: return att_scratch_floats<Cfg<32>>();
    case 64: return att_scratch_floats<Cfg<64>>();
    case 128: return att_scratch_floats<Cfg<128>>();
    default: return att_scratch_floats<Cfg<256>>();
  }
}

int edge_grid(int H, bool bwd, bool bf16, int64_t E, int num_sms, EdgeGrid* out) {
  int occ = 1;
  // Occupancy is fixed by shared memory; cache per (H, bwd, bf16).
  static int cache[4][2][2] = {};
  int hi = H == 32 ? 0 : H == 64 ? 1 : H == 128 ? 2 : 3;
  int& slot = cache[hi][bwd][bf16];
  if (slot == 0) {
    int st = EGNN_OK;
#define EGNN_OCC(HH)                                                             \
    if (H == HH) st = bf16 ? occupancy<HH, true>(bwd, &slot) : occupancy<HH, false>(bwd, &slot);
    EGNN_OCC(32) EGNN_OCC(64) EGNN_OCC(128) EGNN_OCC(256)
#undef EGNN_OCC
    if (st != EGNN_OK) return st;
  }
  occ = slot;
  const int T = edge_chunk(H);
  int64_t G = (int64_t)num_sms * occ;
  int64_t chunks = (E + T - 1) / T;
  G = std::max<int64_t>(1, std::min<int64_t>(G, chunks));
  int64_t epc = (chunks + G - 1) / G * T;
  if (E == 0) epc = T;
  G = std::max<int64_t>(1, (E + epc - 1) / epc);
  out->G = (int)G;
  out->epc = epc;
  return EGNN_OK;
}

int edge_fwd(int H, bool bf16, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
#define EGNN_FWD(HH) \
  if (H == HH) return bf16 ? launch_fwd<HH, true>(a, g, s) : launch_fwd<HH, false>(a, g, s);
  EGNN_FWD(32) EGNN_FWD(64) EGNN_FWD(128) EGNN_FWD(256)
#undef EGNN_FWD
  return fail(EGNN_ERR_UNSUPPORTED, "hidden size %d not built (32, 64, 128, 256)", H);
}

int edge_fixup_fwd(int H, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
  TimerScope ts_fix("edge_fixup", s);
  EGNN_CHECK_CUDA(launch_pdl(edge_fixup_kernel<false>, dim3(g.G - 1), dim3(128), 0, s, H, a.E, g.G, g.epc,
                             a.row_ptr, a.row_idx, (const float*)a.carry, a.flags, a.x, a.agg, a.x_out));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

int edge_bwd(int H, bool bf16, const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
#define EGNN_BWD(HH) \
  if (H == HH) return bf16 ? launch_bwd<HH, true>(a, g, s) : launch_bwd<HH, false>(a, g, s);
  EGNN_BWD(32) EGNN_BWD(64) EGNN_BWD(128) EGNN_BWD(256)
#undef EGNN_BWD
  return fail(EGNN_ERR_UNSUPPORTED, "hidden size %d not built (32, 64, 128, 256)", H);
}

int edge_src_pass(int H, int64_t N, const int32_t* src_ptr, const int32_t* src_edge,
                  const void* gstore, bool bf16_rows, const float4* gdstore, const float* gx_out,
                  const float* gxd, float* S_src, float* gx, cudaStream_t s) {
  if (N <= 0) return EGNN_OK;
  const int warps = 8;
  const unsigned blocks = (unsigned)((N + warps - 1) / warps);
#define EGNN_SRC(HH)                                                                               \
  if (H == HH) {                                                                                   \
    TimerScope ts("src_pass", s);                                                                  \
    if (bf16_rows)                                                                                 \
      EGNN_CHECK_CUDA(launch_pdl(src_pass_kernel<HH, __nv_bfloat16>, dim3(blocks), dim3(warps * 32), 0, s, \
          N, src_ptr, src_edge, static_cast<const __nv_bfloat16*>(gstore), gdstore, gx_out, gxd, S_src, gx)); \
    else                                                                                           \
      EGNN_CHECK_CUDA(launch_pdl(src_pass_kernel<HH, float>, dim3(blocks), dim3(warps * 32), 0, s,  \
          N, src_ptr, src_edge, static_cast<const float*>(gstore), gdstore, gx_out, gxd, S_src, gx));       \
    EGNN_CHECK_LAUNCH();                                                                           \
    return EGNN_OK;                                                                                \
  }
  EGNN_SRC(32) EGNN_SRC(64) EGNN_SRC(128) EGNN_SRC(256)
#undef EGNN_SRC
  return fail(EGNN_ERR_UNSUPPORTED, "hidden size %d not built", H);
}

int edge_part_reduce(int H, int d, bool att, int G, const float* part, const egnn_layer_grads* gp,
                     int64_t ld_w1, int64_t c_r, cudaStream_t s) {
  const int64_t total = edge_part_att(H, d) + (att ? H + 1 : 0);
  const int blocks = (int)((total + 31) / 32);
  TimerScope ts("part_reduce", s);
  EGNN_CHECK_CUDA(launch_pdl(part_reduce_kernel, dim3(blocks), dim3(256), 0, s, H, d, att ? 1 : 0, G,
                             edge_part_floats(H, d), part, *gp, ld_w1, c_r));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

}  // namespace egnn
