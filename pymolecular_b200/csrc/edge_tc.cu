// Fused EGNN edge kernels on the 5th-generation tensor cores (tcgen05, bf16
// operands, fp32 accumulation in TMEM), for bf16-GEMM mode with H = 128.
//
// Same per-edge math and work split as the SIMT kernels (edge_simt.cu): each
// CTA owns an equal contiguous range of CSR edges, processed in chunks of 128
// edges.  Inside a chunk thread t owns edge t, which is also row t of every
// MMA tile and lane t of TMEM:
//
//   forward  u1 = silu(P_i + Q_j + w_r r)        CUDA cores -> bf16 tile U
//            a2 = U W2hi^T + U W2lo^T             tcgen05 -> TMEM
//            (edge attributes: a1 += We attr[edge_id], forward only)
//            m  = silu(a2 + b2)                   -> bf16 tile M, fp32 staging
//                 [attention: m *= sigmoid(wa . m + ba), the dot over the
//                  four column slices of the edge's row]
//            c1 = M Wc1^T                         tcgen05 -> TMEM
//            phi = wc2 . silu(c1 + bc1)           per thread
//            agg, x' : row walk over the staging (as in the SIMT kernel)
//   backward recompute a2, m, c1 as above, then
//            g_c1 = gphi wc2 silu'(c1)             -> bf16 tile G
//            dWc1 += G^T M   (TMEM, persists over the CTA's chunks)
//            g_m  = G Wc1 + g_agg[i]              tcgen05 + CUDA cores
//            g_a2 = g_m silu'(a2)                 -> tile G
//            dW2  += G^T U   (TMEM, persistent)
//            g_a1 = (G W2hi + G W2lo) silu'(a1)   -> global, one bf16 H-vector per edge
// The weight tiles live in shared memory for the whole kernel; one copy of
// each serves the forward product (K-major B) and the data-gradient product
// (MN-major B).  W2 is held as two bf16 tiles, hi = bf16(W2) and
// lo = bf16(W2 - hi), and every product with it is the pair of MMAs: a single
// bf16 W2 would be one rounding shared by every edge, a systematic error that
// the coordinate-MLP weight gradients amplify far past the bf16 tolerance.  The row sums of g_a1 and of the coordinate gradients, over
// each node's in-edges and out-edges, are taken by node_pass_kernel.
#include <algorithm>
#include <climits>
#include <cstdlib>

#include "edge_rows.cuh"
#include "edge_simt.cuh"
#include "edge_tc.cuh"
#include "node_tc.cuh"
#include "tc.cuh"

namespace egnn {

// Number of tensor-core waits that ran out (a kernel that gives up sets it,
// skips its remaining work, frees its TMEM and returns).
__device__ int g_tc_wait_timeouts = 0;

namespace {

using namespace tc;

constexpr int kM = 128;     // edges per chunk = threads per CTA = TMEM lanes

// Every MMA is M = 128 (edge rows, or output features for the weight
// gradients), which ties this path to H = 128.
template <int H>
struct TC {
  static_assert(H == 128, "tensor-core path built for H = 128");
  static constexpr int TILE = kM * H * 2;   // [128 x H] bf16 tile
  static constexpr int WT = H * H * 2;      // [H x H] bf16 weight tile
  static constexpr uint32_t IDESC_FWD = make_idesc_bf16(kM, H, 0, 0);    // A K-major, B K-major
  static constexpr uint32_t IDESC_DGRAD = make_idesc_bf16(kM, H, 0, 1);  // B = W, MN-major
  static constexpr uint32_t IDESC_WGRAD = make_idesc_bf16(H, H, 1, 1);   // A = G^T, B = X, both MN-major
};

// Load an (H x H) fp32 nn.Linear weight into an SW128 bf16 tile (rows = out).
// With `lo`, also the residual tile lo = bf16(W - bf16(W)).
template <int H>
__device__ void load_weight_tile(char* tile, const float* __restrict__ W, char* lo = nullptr) {
  for (int idx = threadIdx.x; idx < H * H / 8; idx += blockDim.x) {
    const int o = idx / (H / 8), c8 = (idx % (H / 8)) * 8;
    const float4 a = __ldg(reinterpret_cast<const float4*>(W + o * H + c8));
    const float4 b = __ldg(reinterpret_cast<const float4*>(W + o * H + c8 + 4));
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st_row8_bf16(tile, H, o, c8, v);
    if (lo) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] -= bf16r(v[k]);
      st_row8_bf16(lo, H, o, c8, v);
    }
  }
}

// K-major operand descriptor of K-step kk (16 columns) of a tile with `rows` rows.
__device__ __forceinline__ uint64_t desc_k(const char* tile, int rows, int kk) {
  return make_desc(smem_u32(tile) + (kk >> 2) * rows * 128 + (kk & 3) * 32, 16, 1024);
}
// MN-major operand descriptor of K-step kk (16 rows) of a tile with `rows` rows.
__device__ __forceinline__ uint64_t desc_mn(const char* tile, int rows, int kk) {
  return make_desc(smem_u32(tile) + kk * 2048, rows * 128, 1024);
}

// Thread-uniform bounded wait on the chunk barrier; false on timeout, after
// one more bounded wait (the built-in limit) for the MMAs still in flight.
// polls < 0: the built-in limit for the first wait too.
__device__ __forceinline__ bool wait_mma(uint64_t* bar, uint32_t& phase, int polls) {
  const bool ok = mbar_wait(bar, phase, polls < 0 ? (1u << 22) : (uint32_t)polls);
  const int bad = __syncthreads_or(!ok);
  if (bad) {
    if (threadIdx.x == 0) {
      atomicAdd(&g_tc_wait_timeouts, 1);
      mbar_wait(bar, phase);
    }
    __syncthreads();
    return false;
  }
  phase ^= 1;
  fence_after_sync();
  return true;
}

// Thread 0: the TMA loads of the index tiles of the chunk starting at CSR
// position c1 (a multiple of 128, so 512-byte aligned) into nrow / ncol.
template <class Args>
__device__ __forceinline__ void issue_idx(const Args& a, int64_t c1, int* nrow, int* ncol, uint64_t* ibar) {
  fence_proxy_async();   // this chunk's generic reads of nrow / ncol precede the async writes
  mbar_expect_tx_bytes(ibar, 2 * kM * 4);
  tma_load_1d(nrow, &a.tm_row, (int)c1, ibar);
  tma_load_1d(ncol, &a.tm_col, (int)c1, ibar);
}

// Operand writes (generic proxy) and TMEM reads done -> tensor core may go.
__device__ __forceinline__ void handoff_to_mma() {
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
}

// Sum over the warp's 32 lanes of x[c]; lane l returns the sum for c = l.
__device__ __forceinline__ float warp_colsum32(float (&x)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const bool up = lane & off;
      const float send = up ? x[i] : x[i + off];
      const float keep = up ? x[i + off] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return x[0];
}

// ---- thread geometry -------------------------------------------------------------
// 512 threads: warp w covers TMEM lanes 32*(w%4)..+31 (edge rows) and the
// 32-column slice 32*(w/4)..+31 of those rows.
struct Geo {
  int tid, warp, lane, q, cg, e, col0;
  uint32_t lane_base;
  __device__ Geo() {
    tid = threadIdx.x;
    warp = tid >> 5;
    lane = tid & 31;
    q = warp & 3;
    cg = warp >> 2;
    e = q * 32 + lane;
    col0 = cg * 32;
    lane_base = (uint32_t)(q * 32) << 16;
  }
};
constexpr int kNT = 512;

// fp32 row staging [128 edges][H features] in shared memory, in 16-byte
// words; word w of row e lives at w ^ (e & 31).  A warp then moves one whole
// row per instruction (lane = word), and a thread that owns a row reads its
// 32-column slice with each quarter-warp on 8 distinct bank groups.
__device__ __forceinline__ int stage_word(int e, int w) { return e * 32 + (w ^ (e & 31)); }

// a1 = P_i + Q_j + w_r r for the chunk's edges, one warp per edge and four
// features per lane (the P and Q rows are read whole), into the staging.
// Invalid edges (e >= n) stage zeros.  GB edges' rows are in flight at once.
template <int GB>
__device__ __forceinline__ void gather_a1(float4* stage, const float* __restrict__ PQ, const int* rows,
                                          const int* cols, const float4* geo, const float* s_wr, int n,
                                          int warp, int lane) {
  constexpr int H = 128;
  const float4 wr4 = *reinterpret_cast<const float4*>(s_wr + 4 * lane);
#pragma unroll
  for (int b = 0; b < 8; b += GB) {
    float4 p[GB], q[GB];
#pragma unroll
    for (int t = 0; t < GB; ++t) {
      const int e = warp * 8 + b + t;
      if (e < n) {
        p[t] = __ldg(reinterpret_cast<const float4*>(PQ + (int64_t)rows[e] * 2 * H) + lane);
        q[t] = __ldg(reinterpret_cast<const float4*>(PQ + (int64_t)cols[e] * 2 * H + H) + lane);
      } else {
        p[t] = q[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int t = 0; t < GB; ++t) {
      const int e = warp * 8 + b + t;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < n) {
        const float r = geo[e].w;
        a = make_float4(fmaf(wr4.x, r, p[t].x + q[t].x), fmaf(wr4.y, r, p[t].y + q[t].y),
                        fmaf(wr4.z, r, p[t].z + q[t].z), fmaf(wr4.w, r, p[t].w + q[t].w));
      }
      stage[stage_word(e, lane)] = a;
    }
  }
}

// Forward variant: u1 = silu(a1) rounded to bf16 straight into row e of the
// SW128 tile U (lane = features 4 lane .. + 3, one 8-byte store); invalid
// edges get zero rows.  Same arithmetic and rounding as staging a1 first.
// Edge attributes (d > 0): a1 += We a_e with a_e = attr[edge_id] (lane k < d
// loads feature k, broadcast by shuffles) and s_WeT[k][f] = We[f][k].
template <int GB>
__device__ __forceinline__ void gather_u(char* Ut, const float* __restrict__ PQ, const int* rows, const int* cols,
                                         const float4* geo, const float* s_wr, int n, int warp, int lane,
                                         const float* __restrict__ attr, const int* eids, const float* s_WeT,
                                         int d) {
  constexpr int H = 128;
  const float4 wr4 = *reinterpret_cast<const float4*>(s_wr + 4 * lane);
#pragma unroll
  for (int b = 0; b < 8; b += GB) {
    float4 p[GB], q[GB];
    float av[GB];
#pragma unroll
    for (int t = 0; t < GB; ++t) {
      const int e = warp * 8 + b + t;
      if (e < n) {
        p[t] = __ldg(reinterpret_cast<const float4*>(PQ + (int64_t)rows[e] * 2 * H) + lane);
        q[t] = __ldg(reinterpret_cast<const float4*>(PQ + (int64_t)cols[e] * 2 * H + H) + lane);
      } else {
        p[t] = q[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      av[t] = (d > 0 && e < n && lane < d) ? __ldg(attr + (int64_t)eids[e] * d + lane) : 0.f;
    }
#pragma unroll
    for (int t = 0; t < GB; ++t) {
      const int e = warp * 8 + b + t;
      float u0 = 0.f, u1 = 0.f, u2 = 0.f, u3 = 0.f;
      float4 x4 = make_float4(p[t].x + q[t].x, p[t].y + q[t].y, p[t].z + q[t].z, p[t].w + q[t].w);
      for (int k = 0; k < d; ++k) {   // uniform trip count: every lane takes part in the shuffles
        const float ak = __shfl_sync(0xffffffffu, av[t], k);
        const float4 w = *reinterpret_cast<const float4*>(s_WeT + k * H + 4 * lane);
        x4 = make_float4(fmaf(w.x, ak, x4.x), fmaf(w.y, ak, x4.y), fmaf(w.z, ak, x4.z), fmaf(w.w, ak, x4.w));
      }
      if (e < n) {
        const float r = geo[e].w;
        u0 = silu_edge(fmaf(wr4.x, r, x4.x));
        u1 = silu_edge(fmaf(wr4.y, r, x4.y));
        u2 = silu_edge(fmaf(wr4.z, r, x4.z));
        u3 = silu_edge(fmaf(wr4.w, r, x4.w));
      }
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(u0, u1);
      const __nv_bfloat162 h23 = __floats2bfloat162_rn(u2, u3);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&h01);
      w.y = *reinterpret_cast<const uint32_t*>(&h23);
      *reinterpret_cast<uint2*>(Ut + sw128_offset(e, 4 * lane, kM)) = w;
    }
  }
}

// The 32-column slice col0..col0+31 of staged row e.
__device__ __forceinline__ void stage_read32(const float4* stage, int e, int col0, float (&v)[32]) {
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float4 t = stage[stage_word(e, col0 / 4 + w)];
    v[4 * w] = t.x; v[4 * w + 1] = t.y; v[4 * w + 2] = t.z; v[4 * w + 3] = t.w;
  }
}
__device__ __forceinline__ void stage_write32(float4* stage, int e, int col0, const float (&v)[32]) {
#pragma unroll
  for (int w = 0; w < 8; ++w)
    stage[stage_word(e, col0 / 4 + w)] = make_float4(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3]);
}

__device__ __forceinline__ void st_row32_bf16(char* tile, int row, int col0, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 32; k += 8) st_row8_bf16(tile, kM, row, col0 + k, v + k);
}

// ---- forward ----------------------------------------------------------------------
// The U tile is free once the a2 product has completed, so the residual tile
// of m (bf16(m - bf16(m)), the second operand of the agg product) reuses it.
template <int H>
struct FwdLayout {
  static constexpr size_t W2 = 0;
  static constexpr size_t W2LO = W2 + TC<H>::WT;
  static constexpr size_t WC1 = W2LO + TC<H>::WT;
  static constexpr size_t U = WC1 + TC<H>::WT;         // u1, then bf16(m - bf16(m))
  static constexpr size_t M = U + TC<H>::TILE;
  static constexpr size_t S = M + TC<H>::TILE;         // 0/1 segment matrix [slot][edge]
  static constexpr size_t VEC = S + TC<H>::TILE;       // wr, b2, bc1, wc2, wa
  static constexpr size_t PART = VEC + 5 * H * 4;      // float[4][128]
  static constexpr size_t DL = PART + 4 * kM * 4;      // float4[128]: dn.xyz, r
  static constexpr size_t SEGX = DL + kM * 16;         // float4[128]: coordinate sums per segment
  static constexpr size_t NXI = SEGX + kM * 16;        // float4[128]: next chunk's x_i (prefetch)
  static constexpr size_t NXJ = NXI + kM * 16;         // float4[128]: next chunk's x_j
  static constexpr size_t PHI = NXJ + kM * 16;         // float[128]
  static constexpr size_t ROWL = PHI + kM * 4;         // int[128]
  static constexpr size_t COLL = ROWL + kM * 4;        // int[128]
  static constexpr size_t NROW = COLL + kM * 4;        // int[128]: next chunk's destination ids
  static constexpr size_t NCOL = NROW + kM * 4;        // int[128]: next chunk's source ids
  static constexpr size_t SEGROW = NCOL + kM * 4;      // int[129]
  static constexpr size_t SEGSTART = SEGROW + (kM + 4) * 4;
  static constexpr size_t SEGRP = SEGSTART + (kM + 4) * 4;   // int[128][2]: row_ptr[r], row_ptr[r + 1] of segment rows
  static constexpr size_t XLI = SEGRP + kM * 8;        // float4[128]: x_i of each edge
  static constexpr size_t EIDL = XLI + kM * 16;        // int[128]: edge ids (edge attributes only)
  static constexpr size_t WET = EIDL + kM * 4;         // float[16][H]: We^T (edge attributes only)
  static constexpr size_t OPEN = WET + 16 * H * 4;     // float[H + 4]
  static constexpr size_t MISC = OPEN + (H + 4) * 4;   // ints: nseg, open_row, prev_row, warp counts[4]
  static constexpr size_t BAR = MISC + 64;
  static constexpr size_t END = BAR + 32;   // MMA barrier, TMEM base, index-tile barrier
  static constexpr size_t BYTES = END + 1024;
};

template <int H>
__global__ void __launch_bounds__(kNT, 1) edge_fwd_tc_kernel(const __grid_constant__ EdgeFwdArgs a) {
  using C = TC<H>;
  using L = FwdLayout<H>;
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* W2t = sm + L::W2;
  char* W2lo = sm + L::W2LO;
  char* Wc1t = sm + L::WC1;
  char* Ut = sm + L::U;
  char* Mt = sm + L::M;
  char* Mlo = Ut;   // U is dead once the a2 product has completed
  char* St = sm + L::S;
  float* s_wr = reinterpret_cast<float*>(sm + L::VEC);
  float* s_b2 = s_wr + H;
  float* s_bc1 = s_b2 + H;
  float* s_wc2 = s_bc1 + H;
  float* s_wa = s_wc2 + H;   // att_mlp.0.weight (attention only)
  float* part = reinterpret_cast<float*>(sm + L::PART);
  float4* dl = reinterpret_cast<float4*>(sm + L::DL);
  float4* segx = reinterpret_cast<float4*>(sm + L::SEGX);
  float* phi = reinterpret_cast<float*>(sm + L::PHI);
  int* rowl = reinterpret_cast<int*>(sm + L::ROWL);
  int* coll = reinterpret_cast<int*>(sm + L::COLL);
  int* nrow = reinterpret_cast<int*>(sm + L::NROW);
  int* ncol = reinterpret_cast<int*>(sm + L::NCOL);
  float4* nxi = reinterpret_cast<float4*>(sm + L::NXI);
  float4* nxj = reinterpret_cast<float4*>(sm + L::NXJ);
  int* segrow = reinterpret_cast<int*>(sm + L::SEGROW);
  int* segstart = reinterpret_cast<int*>(sm + L::SEGSTART);
  int* segrp = reinterpret_cast<int*>(sm + L::SEGRP);
  float4* xli = reinterpret_cast<float4*>(sm + L::XLI);
  int* eidl = reinterpret_cast<int*>(sm + L::EIDL);
  float* s_WeT = reinterpret_cast<float*>(sm + L::WET);
  float* open = reinterpret_cast<float*>(sm + L::OPEN);
  int* misc = reinterpret_cast<int*>(sm + L::MISC);   // [0] nseg [1] open_row [2] prev_row [4..7] warp counts
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(sm + L::BAR + 8);
  uint64_t* ibar = reinterpret_cast<uint64_t*>(sm + L::BAR + 16);
  int* idx_abort = reinterpret_cast<int*>(sm + L::BAR + 24);   // a prefetcher gave up on the index tiles
  uint32_t iphase = 0, idx_last = 0;
  bool idx_pending = false;   // an index-tile copy issued and not yet waited for
  bool idx_drain = false;     // ... or waited for without success (drain before leaving)

  const Geo g;
  constexpr uint32_t NCOL = 2 * H;   // D0 | DAGG
  if (g.warp == 0) tmem_alloc(tmem_base_s, NCOL);
  if (g.tid == 0) {
    mbar_init(bar, 1);
    mbar_init(ibar, 1);
    *idx_abort = 0;
    fence_mbar_init();
  }
  load_weight_tile<H>(W2t, a.W2_src, W2lo);
  load_weight_tile<H>(Wc1t, a.Wc1_src);
  const bool att = a.flags & EGNN_FLAG_ATTENTION;
  for (int c = g.tid; c < H; c += kNT) {
    s_wr[c] = a.wr[c]; s_b2[c] = a.b2[c]; s_bc1[c] = a.bc1[c]; s_wc2[c] = a.wc2[c];
    s_wa[c] = att ? a.wa[c] : 0.f;
  }
  for (int c = g.tid; c < H * a.d; c += kNT) s_WeT[(c % a.d) * H + c / a.d] = a.We[c];   // We is (H, d)
  const float ba = att ? a.ba[0] : 0.f;
  pdl_enter();   // everything below reads the predecessor's output (P, Q) or writes
  const int cta = blockIdx.x, G = gridDim.x;
  const int64_t eb = std::min<int64_t>(a.E, (int64_t)cta * a.epc);
  const int64_t ee = std::min<int64_t>(a.E, eb + a.epc);
  const int N = (int)a.N;
  const int end_row = (cta == G - 1) ? N : a.row_idx[ee];
  if (g.tid == 0) {
    misc[1] = -1;                                      // open_row
    misc[2] = (cta == 0) ? -1 : a.row_idx[eb] - 1;     // last row seen
    a.carry_row[cta * 2] = -1;
    a.carry_row[cta * 2 + 1] = -1;
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_base_s;
  const uint32_t tD0 = tmem, tAGG = tmem + H;
  uint32_t phase = 0;
  const bool normalize = a.flags & EGNN_FLAG_NORMALIZE;
  const bool tanh_ = a.flags & EGNN_FLAG_TANH;
  bool ok = true;

  // Write the 32-column slice of a finished row (and its coordinates when cg == 0).
  // rp0, rp1 = row_ptr[r], row_ptr[r + 1]; xr = x_r (xyz)
  auto put_row = [&](int r, const float (&v)[32], float4 cx, bool zero, int rp0, int rp1, float4 xr) {
    const bool before = rp0 < eb;
    if (!before) {
      float* dst = a.agg + (int64_t)r * H + g.col0;
#pragma unroll
      for (int k = 0; k < 32; k += 4)
        *reinterpret_cast<float4*>(dst + k) = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                   : make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
      if (g.cg == 0) {
        const float sc = (a.flags & EGNN_FLAG_COORDS_SUM) ? 1.f : 1.f / (float)max(rp1 - rp0, 1);
        const float c3[3] = {cx.x, cx.y, cx.z}, x3[3] = {xr.x, xr.y, xr.z};
#pragma unroll
        for (int d = 0; d < 3; ++d) a.x_out[(int64_t)r * 3 + d] = x3[d] + (zero ? 0.f : c3[d] * sc);
      }
    } else {
      float* dst = a.carry + ((int64_t)cta * 2 + 0) * (H + 4);
#pragma unroll
      for (int k = 0; k < 32; ++k) dst[g.col0 + k] = v[k];
      if (g.cg == 0) {
        dst[H] = cx.x; dst[H + 1] = cx.y; dst[H + 2] = cx.z;
        a.carry_row[cta * 2] = r;
      }
    }
  };
  const float zero32[32] = {};
  // a row with no edges in this chunk: its row pointers and coordinates from memory
  auto put_empty_row = [&](int r) {
    put_row(r, zero32, make_float4(0.f, 0.f, 0.f, 0.f), true, a.row_ptr[r], a.row_ptr[r + 1], a.xp[r]);
  };

  // The next chunk's edge ids and coordinates are prefetched with cp.async by
  // the threads of column slice 1 while this chunk's MMAs and activations run
  // (ids after the first MMA is issued, coordinates once they have landed).
  bool pref = false;
#pragma unroll 1
  for (int64_t c0 = eb; c0 < ee && ok; c0 += kM) {
    const int n = (int)std::min<int64_t>(kM, ee - c0);
    const bool valid = g.e < n;
    const int64_t c1 = c0 + kM;
    const int n_next = (int)std::max<int64_t>(0, std::min<int64_t>(kM, ee - c1));
    const bool prefetcher = g.cg == 1 && g.e < n_next;
    // ---- per-edge geometry (column slice 0); zero the segment matrix
    if (g.cg == 0) {
      if (valid) {
        int i, j;
        float4 xi, xj;
        if (pref) {
          i = nrow[g.e]; j = ncol[g.e]; xi = nxi[g.e]; xj = nxj[g.e];
        } else {
          const int64_t k = c0 + g.e;
          i = a.row_idx[k]; j = a.col_idx[k]; xi = a.xp[i]; xj = a.xp[j];
        }
        const float dx = xi.x - xj.x, dy = xi.y - xj.y, dz = xi.z - xj.z;
        const float r = dx * dx + dy * dy + dz * dz;
        const float inv = normalize ? 1.f / (sqrtf(r) + 1e-8f) : 1.f;
        rowl[g.e] = i;
        coll[g.e] = j;
        dl[g.e] = make_float4(dx * inv, dy * inv, dz * inv, r);
        xli[g.e] = xi;
        if (a.d > 0) eidl[g.e] = a.edge_id[c0 + g.e];
      } else {
        rowl[g.e] = INT_MAX;
        coll[g.e] = 0;
        dl[g.e] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    {
      uint4* sz = reinterpret_cast<uint4*>(St);
#pragma unroll
      for (int k = 0; k < C::TILE / 16 / kNT; ++k) sz[g.tid + k * kNT] = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    // ---- u1 = silu(a1) rows -> tile U (coalesced P / Q rows, one warp per edge)
    gather_u<4>(Ut, a.PQ, rowl, coll, dl, s_wr, n, g.warp, g.lane, a.attr, eidl, s_WeT, a.d);
    // ---- segments of the chunk (runs of equal destination rows)
    if (g.cg == 0) {
      const int r = rowl[g.e];
      const bool flag = valid && (g.e == 0 || rowl[g.e - 1] != r);
      const unsigned mask = __ballot_sync(0xffffffffu, flag);
      if (g.lane == 0) misc[4 + g.q] = __popc(mask);
      asm volatile("bar.sync 1, 128;" ::: "memory");   // warps 0..3 only
      int before = __popc(mask & ((1u << g.lane) - 1u)) + (flag ? 1 : 0);
      for (int w = 0; w < g.q; ++w) before += misc[4 + w];
      const int seg = before - 1;   // segment of this edge
      if (flag) {
        segrow[seg] = r;
        segstart[seg] = g.e;
        cp_async4(&segrp[2 * seg], a.row_ptr + r);     // needed by the row flush
        cp_async4(&segrp[2 * seg + 1], a.row_ptr + r + 1);
        cp_async_commit_group();
      }
      if (valid) {
        const __nv_bfloat16 one = __float2bfloat16_rn(1.f);
        *reinterpret_cast<__nv_bfloat16*>(St + sw128_offset(seg, g.e, kM)) = one;
      }
      if (g.e == kM - 1) {
        const int total = misc[4] + misc[5] + misc[6] + misc[7];
        misc[0] = total;
        segstart[total] = n;
      }
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Ut, kM, kk), desc_k(W2t, H, kk), C::IDESC_FWD, kk > 0);
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Ut, kM, kk), desc_k(W2lo, H, kk), C::IDESC_FWD, 1u);
      mma_commit(bar);
      if (a.use_tma && n_next > 0) issue_idx(a, c1, nrow, ncol, ibar);
    }
    if (a.use_tma && n_next > 0) idx_pending = true;
    if (prefetcher && !a.use_tma) {
      cp_async4(&nrow[g.e], a.row_idx + c1 + g.e);
      cp_async4(&ncol[g.e], a.col_idx + c1 + g.e);
      cp_async_commit_group();
    }
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;
    // the prefetchers alone wait for the index tiles; one that gives up skips
    // its loads and raises the flag the end-of-chunk barrier publishes
    bool idx_ok = true;
    if (idx_pending) {
      idx_pending = false;
      idx_last = iphase;
      iphase ^= 1;
      if (prefetcher && !mbar_wait(ibar, idx_last)) {
        idx_ok = false;
        if (atomicExch(idx_abort, 1) == 0) atomicAdd(&g_tc_wait_timeouts, 1);
      }
    }
    if (prefetcher && idx_ok) {
      if (!a.use_tma) cp_async_wait_all_groups();
      cp_async16_ca(&nxi[g.e], a.xp + nrow[g.e]);
      cp_async16_ca(&nxj[g.e], a.xp + ncol[g.e]);
      cp_async_commit_group();
    }

    // ---- m = silu(a2 + b2) [* sigmoid(wa . m + ba)] -> tiles M (bf16) and MLO (bf16 residual)
    {
      float v[32], lo[32];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
#pragma unroll
      for (int q = 0; q < 32; ++q) v[q] = silu_edge(v[q] + s_b2[g.col0 + q]);
      if (att) {   // the gate's dot product over the edge's four column slices (uniform branch)
        float pa = 0.f;
#pragma unroll
        for (int q = 0; q < 32; ++q) pa = fmaf(v[q], s_wa[g.col0 + q], pa);
        part[g.cg * kM + g.e] = pa;
        __syncthreads();
        const float gate = sigmoidf_(part[g.e] + part[kM + g.e] + part[2 * kM + g.e] + part[3 * kM + g.e] + ba);
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] *= gate;
      }
#pragma unroll
      for (int q = 0; q < 32; ++q) lo[q] = v[q] - __bfloat162float(__float2bfloat16_rn(v[q]));
      st_row32_bf16(Mt, g.e, g.col0, v);
      st_row32_bf16(Mlo, g.e, g.col0, lo);
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Mt, kM, kk), desc_k(Wc1t, H, kk), C::IDESC_FWD, kk > 0);
      // agg rows of the chunk: S (slots x edges) times M and MLO (edges x features)
#pragma unroll
      for (int kk = 0; kk < kM / 16; ++kk)
        mma_bf16(tAGG, desc_k(St, kM, kk), desc_mn(Mt, kM, kk), C::IDESC_DGRAD, kk > 0);
#pragma unroll
      for (int kk = 0; kk < kM / 16; ++kk)
        mma_bf16(tAGG, desc_k(St, kM, kk), desc_mn(Mlo, kM, kk), C::IDESC_DGRAD, 1u);
      mma_commit(bar);
    }
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;

    // ---- phi = wc2 . silu(c1 + bc1), four column slices per edge
    {
      float v[32];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
      float p = 0.f;
#pragma unroll
      for (int q = 0; q < 32; ++q) p = fmaf(silu_edge(v[q] + s_bc1[g.col0 + q]), s_wc2[g.col0 + q], p);
      part[g.cg * kM + g.e] = p;
    }
    if (g.cg == 0) cp_async_wait_all_groups();   // segment heads: row pointers landed
    __syncthreads();
    if (g.cg == 0) {
      const float p = part[g.e] + part[kM + g.e] + part[2 * kM + g.e] + part[3 * kM + g.e];
      phi[g.e] = valid ? (tanh_ ? tanhf(p) : p) : 0.f;
    }
    __syncthreads();
    const int nseg = misc[0];
    if (g.tid < nseg) {
      const int s = g.tid;
      float sx = 0.f, sy = 0.f, sz = 0.f;
      for (int e2 = segstart[s]; e2 < segstart[s + 1]; ++e2) {
        const float4 d = dl[e2];
        const float f = phi[e2];
        sx = fmaf(d.x, f, sx); sy = fmaf(d.y, f, sy); sz = fmaf(d.z, f, sz);
      }
      segx[s] = make_float4(sx, sy, sz, 0.f);
    }
    __syncthreads();
    // ---- finish the chunk's rows: slot s = edge lane of this thread
    {
      const int s = g.e;
      const int open_row = misc[1];
      const int prev = misc[2];
      float v[32];
      tmem_ld32(tAGG + g.lane_base + g.col0, v);   // every warp takes part in the TMEM load
      if (s < nseg) {
        const int r = segrow[s];
        const int pr = (s == 0) ? prev : segrow[s - 1];
        for (int rr = pr + 1; rr < r; ++rr) put_empty_row(rr);
        float4 cx = segx[s];
        if (s == 0 && r == open_row) {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] += open[g.col0 + k];
          cx.x += open[H]; cx.y += open[H + 1]; cx.z += open[H + 2];
        }
        const int rp0 = segrp[2 * s], rp1 = segrp[2 * s + 1];
        const bool complete = (s < nseg - 1) || (rp1 <= c0 + n);
        if (complete) {
          put_row(r, v, cx, false, rp0, rp1, xli[segstart[s]]);
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) open[g.col0 + k] = v[k];
          if (g.cg == 0) { open[H] = cx.x; open[H + 1] = cx.y; open[H + 2] = cx.z; }
        }
      }
    }
    if (prefetcher) cp_async_wait_all_groups();
    fence_before_sync();
    __syncthreads();
    if (g.tid == 0) {
      const int r = segrow[nseg - 1];
      misc[2] = r;
      misc[1] = (segrp[2 * (nseg - 1) + 1] <= c0 + n) ? -1 : r;
    }
    __syncthreads();
    pref = n_next > 0;
    if (*idx_abort) {   // read after the barrier: the same value in every thread
      ok = false;
      idx_drain = true;
      break;
    }
  }
  cp_async_wait_all_groups();   // nothing in flight when the CTA leaves (also after a timeout)
  if (g.tid == 0) {   // no index-tile copy may still be landing when the CTA leaves
    if (idx_pending) mbar_wait(ibar, iphase);
    if (idx_drain) mbar_wait(ibar, idx_last);
  }
  // ---- end of the CTA range: open row -> carry slot, trailing empty rows
  if (ok) {
    const int open_row = misc[1];
    const int last = misc[2];
    if (open_row >= 0) {
      const int slot = (a.row_ptr[open_row] < eb) ? 0 : 1;
      if (g.e == 0) {
        float* dst = a.carry + ((int64_t)cta * 2 + slot) * (H + 4);
#pragma unroll
        for (int k = 0; k < 32; ++k) dst[g.col0 + k] = open[g.col0 + k];
        if (g.cg == 0) {
          dst[H] = open[H]; dst[H + 1] = open[H + 1]; dst[H + 2] = open[H + 2];
          a.carry_row[cta * 2 + slot] = open_row;
        }
      }
    }
    for (int rr = last + 1 + g.e; rr < end_row; rr += kM) put_empty_row(rr);
  }
  fence_before_sync();
  __syncthreads();
  if (g.warp == 0) tmem_dealloc(tmem, NCOL);
}

// ---- backward (dst pass) ---------------------------------------------------------------
// silu'(a1) and silu'(a2) of the chunk live in TMEM as fp16 pairs (the
// columns after the accumulator), so shared memory holds both W2 tiles.
template <int H>
struct BwdLayout {
  static constexpr size_t W2 = 0;
  static constexpr size_t W2LO = W2 + TC<H>::WT;
  static constexpr size_t WC1 = W2LO + TC<H>::WT;
  static constexpr size_t U = WC1 + TC<H>::WT;
  static constexpr size_t M = U + TC<H>::TILE;
  static constexpr size_t G = M + TC<H>::TILE;
  static constexpr size_t VEC = G + TC<H>::TILE;                      // wr, b2, bc1, wc2
  static constexpr size_t PART = VEC + 4 * H * 4;                     // float[4][128]
  static constexpr size_t DL = PART + 4 * kM * 4;                     // float4[128]: d.xyz, r
  static constexpr size_t GT = DL + kM * 16;                          // float4[128]: g_trans.xyz, inv
  static constexpr size_t PHI = GT + kM * 16;                         // float2[128]: phi, gphi'
  static constexpr size_t ROWI = PHI + kM * 8;                        // int[128]
  static constexpr size_t COLI = ROWI + kM * 4;                       // int[128]
  // next chunk's prefetched inputs: ids, row_ptr[i], row_ptr[i + 1], x_i, x_j, dL/dx'_i
  static constexpr size_t NROW = COLI + kM * 4;                       // int[128]
  static constexpr size_t NCOL = NROW + kM * 4;                       // int[128]
  static constexpr size_t NRP = NCOL + kM * 4;                        // int[128][2]
  static constexpr size_t NXI = NRP + kM * 8;                         // float4[128]
  static constexpr size_t NXJ = NXI + kM * 16;                        // float4[128]
  static constexpr size_t NGX = NXJ + kM * 16;                        // float4[128] (xyz)
  static constexpr size_t BAR = NGX + kM * 16;
  static constexpr size_t END = BAR + 32;   // MMA barrier, TMEM base, index-tile barrier
  static constexpr size_t BYTES = END + 1024;
};

template <int H>
__global__ void __launch_bounds__(kNT, 1) edge_bwd_tc_kernel(const __grid_constant__ EdgeBwdArgs a) {
  using C = TC<H>;
  using L = BwdLayout<H>;
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* W2t = sm + L::W2;
  char* W2lo = sm + L::W2LO;
  char* Wc1t = sm + L::WC1;
  char* Ut = sm + L::U;
  char* Mt = sm + L::M;
  char* Gt = sm + L::G;
  float* s_wr = reinterpret_cast<float*>(sm + L::VEC);
  float* s_b2 = s_wr + H;
  float* s_bc1 = s_b2 + H;
  float* s_wc2 = s_bc1 + H;
  float* part = reinterpret_cast<float*>(sm + L::PART);
  float4* dl = reinterpret_cast<float4*>(sm + L::DL);
  float4* gtr = reinterpret_cast<float4*>(sm + L::GT);
  float2* phis = reinterpret_cast<float2*>(sm + L::PHI);
  int* rowi = reinterpret_cast<int*>(sm + L::ROWI);
  int* coli = reinterpret_cast<int*>(sm + L::COLI);
  int* nrow = reinterpret_cast<int*>(sm + L::NROW);
  int* ncol = reinterpret_cast<int*>(sm + L::NCOL);
  int* nrp = reinterpret_cast<int*>(sm + L::NRP);
  float4* nxi = reinterpret_cast<float4*>(sm + L::NXI);
  float4* nxj = reinterpret_cast<float4*>(sm + L::NXJ);
  float4* ngx = reinterpret_cast<float4*>(sm + L::NGX);
  float4* stage = reinterpret_cast<float4*>(Mt);   // fp32 row staging over the M | G tiles (64 KB)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(sm + L::BAR + 8);
  uint64_t* ibar = reinterpret_cast<uint64_t*>(sm + L::BAR + 16);
  int* idx_abort = reinterpret_cast<int*>(sm + L::BAR + 24);   // a prefetcher gave up on the index tiles
  uint32_t iphase = 0, idx_last = 0;
  bool idx_pending = false;   // an index-tile copy issued and not yet waited for
  bool idx_drain = false;     // ... or waited for without success (drain before leaving)

  const Geo g;
  constexpr uint32_t NCOL = 4 * H;   // D0 | fp16 pairs of silu'(a1), silu'(a2) | dWc1 | dW2
  if (g.warp == 0) tmem_alloc(tmem_base_s, NCOL);
  if (g.tid == 0) {
    mbar_init(bar, 1);
    mbar_init(ibar, 1);
    *idx_abort = 0;
    fence_mbar_init();
  }
  load_weight_tile<H>(W2t, a.W2_src, W2lo);
  load_weight_tile<H>(Wc1t, a.Wc1_src);
  for (int c = g.tid; c < H; c += kNT) {
    s_wr[c] = a.wr[c]; s_b2[c] = a.b2[c]; s_bc1[c] = a.bc1[c]; s_wc2[c] = a.wc2[c];
  }
  pdl_enter();   // everything below reads the predecessor's output (dL/dagg) or writes
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_base_s;
  // tS1: silu'(a1) of feature f as the fp16 half (f & 1) of column f / 2;
  // tD2 = tS1 + H / 2: silu'(a2) likewise
  const uint32_t tD0 = tmem, tS1 = tmem + H, tD2 = tmem + H + H / 2, tWC1 = tmem + 2 * H, tW2 = tmem + 3 * H;
  uint32_t phase = 0;

  const int cta = blockIdx.x;
  const int64_t eb = std::min<int64_t>(a.E, (int64_t)cta * a.epc);
  const int64_t ee = std::min<int64_t>(a.E, eb + a.epc);
  const bool normalize = a.flags & EGNN_FLAG_NORMALIZE;
  const bool tanh_ = a.flags & EGNN_FLAG_TANH;

  // per-lane column partials over the warp's 32 rows: column col0 + lane
  float r_bc1 = 0.f, r_b2 = 0.f, r_wc2 = 0.f, r_wr = 0.f;
  bool ok = true;
  bool first = true;

  // The next chunk's per-edge inputs are prefetched with cp.async by the
  // threads of column slice 1 while this chunk's MMAs and activations run.
  bool pref = false;
#pragma unroll 1
  for (int64_t c0 = eb; c0 < ee && ok; c0 += kM) {
    const int n = (int)std::min<int64_t>(kM, ee - c0);
    const bool valid = g.e < n;
    const int64_t c1 = c0 + kM;
    const int n_next = (int)std::max<int64_t>(0, std::min<int64_t>(kM, ee - c1));
    const bool prefetcher = g.cg == 1 && g.e < n_next;
    // ---- per-edge geometry (column slice 0)
    if (g.cg == 0) {
      if (valid) {
        int i, j, rp0, rp1;
        float4 xi, xj, gxi;
        if (pref) {
          i = nrow[g.e]; j = ncol[g.e]; rp0 = nrp[2 * g.e]; rp1 = nrp[2 * g.e + 1];
          xi = nxi[g.e]; xj = nxj[g.e]; gxi = ngx[g.e];
        } else {
          const int64_t k = c0 + g.e;
          i = a.row_idx[k]; j = a.col_idx[k]; rp0 = a.row_ptr[i]; rp1 = a.row_ptr[i + 1];
          xi = a.xp[i]; xj = a.xp[j];
          gxi = make_float4(a.gx_out[(int64_t)i * 3], a.gx_out[(int64_t)i * 3 + 1], a.gx_out[(int64_t)i * 3 + 2], 0.f);
        }
        const float dx = xi.x - xj.x, dy = xi.y - xj.y, dz = xi.z - xj.z;
        const float r = dx * dx + dy * dy + dz * dz;
        const float inv = normalize ? 1.f / (sqrtf(r) + 1e-8f) : 1.f;
        const float inv_g = (i == j) ? 0.f : inv;   // self-loop: zero coordinate gradient
        const float sc = (a.flags & EGNN_FLAG_COORDS_SUM) ? 1.f : 1.f / (float)max(rp1 - rp0, 1);
        rowi[g.e] = i;
        coli[g.e] = j;
        dl[g.e] = make_float4(dx, dy, dz, r);
        gtr[g.e] = make_float4(gxi.x * sc, gxi.y * sc, gxi.z * sc, inv_g);
      } else {
        rowi[g.e] = 0;
        coli[g.e] = 0;
        dl[g.e] = make_float4(0.f, 0.f, 0.f, 0.f);
        gtr[g.e] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    __syncthreads();
    // ---- a1 rows (coalesced); u1 slice -> tile U, s1 = silu'(a1) slice -> TMEM (fp16)
    gather_a1<4>(stage, a.PQ, rowi, coli, dl, s_wr, n, g.warp, g.lane);
    __syncthreads();
    {
      float u[32], s1v[32];
      stage_read32(stage, g.e, g.col0, u);
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        silu_grad_edge(u[q], u[q], s1v[q]);
        if (!valid) { u[q] = 0.f; s1v[q] = 0.f; }
      }
      st_row32_bf16(Ut, g.e, g.col0, u);
      uint32_t w[16];
      pack_half32(s1v, w);
      tmem_st16u(tS1 + g.lane_base + g.col0 / 2, w);
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Ut, kM, kk), desc_k(W2t, H, kk), C::IDESC_FWD, kk > 0);
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Ut, kM, kk), desc_k(W2lo, H, kk), C::IDESC_FWD, 1u);
      mma_commit(bar);
      if (a.use_tma && n_next > 0) issue_idx(a, c1, nrow, ncol, ibar);
    }
    if (a.use_tma && n_next > 0) idx_pending = true;
    if (prefetcher && !a.use_tma) {
      cp_async4(&nrow[g.e], a.row_idx + c1 + g.e);
      cp_async4(&ncol[g.e], a.col_idx + c1 + g.e);
      cp_async_commit_group();
    }
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;
    // the prefetchers alone wait for the index tiles; one that gives up skips
    // its loads and raises the flag the end-of-chunk barrier publishes
    bool idx_ok = true;
    if (idx_pending) {
      idx_pending = false;
      idx_last = iphase;
      iphase ^= 1;
      if (prefetcher && !mbar_wait(ibar, idx_last)) {
        idx_ok = false;
        if (atomicExch(idx_abort, 1) == 0) atomicAdd(&g_tc_wait_timeouts, 1);
      }
    }
    if (prefetcher && idx_ok) {
      if (!a.use_tma) cp_async_wait_all_groups();
      const int i = nrow[g.e], j = ncol[g.e];
      cp_async16_ca(&nxi[g.e], a.xp + i);
      cp_async16_ca(&nxj[g.e], a.xp + j);
      cp_async4(&nrp[2 * g.e], a.row_ptr + i);
      cp_async4(&nrp[2 * g.e + 1], a.row_ptr + i + 1);
      cp_async4(reinterpret_cast<float*>(&ngx[g.e]), a.gx_out + (int64_t)i * 3);
      cp_async4(reinterpret_cast<float*>(&ngx[g.e]) + 1, a.gx_out + (int64_t)i * 3 + 1);
      cp_async4(reinterpret_cast<float*>(&ngx[g.e]) + 2, a.gx_out + (int64_t)i * 3 + 2);
      cp_async_commit_group();
    }

    // ---- m = silu(a2 + b2) -> tile M ; silu'(a2) -> TMEM (fp16)
    {
      float v[32], d2v[32];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
#pragma unroll
      for (int q = 0; q < 32; ++q) silu_grad_edge(v[q] + s_b2[g.col0 + q], v[q], d2v[q]);
      st_row32_bf16(Mt, g.e, g.col0, v);
      uint32_t w[16];
      pack_half32(d2v, w);
      tmem_st16u(tD2 + g.lane_base + g.col0 / 2, w);
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Mt, kM, kk), desc_k(Wc1t, H, kk), C::IDESC_FWD, kk > 0);
      mma_commit(bar);
    }
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;

    // ---- phi = wc2 . silu(c1 + bc1) (row sums across the four column slices)
    // and g_c1 = gphi' wc2 silu'(c1) -> tile G, with column sums.  Without
    // tanh, gphi' = (dL/dx'_i / deg_i) . d (x 1/|d| when normalising) does not
    // depend on phi: one pass over c1 gives both, and phi is summed later.
    if (!tanh_) {
      const float4 d = dl[g.e], gt = gtr[g.e];
      float gp = gt.x * d.x + gt.y * d.y + gt.z * d.z;
      if (normalize) gp *= gt.w;
      if (!valid) gp = 0.f;
      float v[32], gc[32];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
      float p = 0.f;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        float y, dy;
        silu_grad_edge(v[q] + s_bc1[g.col0 + q], y, dy);
        p = fmaf(y, s_wc2[g.col0 + q], p);
        gc[q] = gp * s_wc2[g.col0 + q] * dy;
        v[q] = gp * y;
      }
      part[g.cg * kM + g.e] = p;
      st_row32_bf16(Gt, g.e, g.col0, gc);
      r_bc1 += warp_colsum32(gc);
      r_wc2 += warp_colsum32(v);
    } else {
      {
        float v[32];
        tmem_ld32(tD0 + g.lane_base + g.col0, v);
        float p = 0.f;
#pragma unroll
        for (int q = 0; q < 32; ++q) p = fmaf(silu_edge(v[q] + s_bc1[g.col0 + q]), s_wc2[g.col0 + q], p);
        part[g.cg * kM + g.e] = p;
      }
      __syncthreads();
      if (g.cg == 0) {
        const float p = part[g.e] + part[kM + g.e] + part[2 * kM + g.e] + part[3 * kM + g.e];
        const float4 d = dl[g.e], gt = gtr[g.e];
        const float ph = tanhf(p);
        float gp = gt.x * d.x + gt.y * d.y + gt.z * d.z;
        if (normalize) gp *= gt.w;
        gp *= (1.f - ph * ph);
        phis[g.e] = valid ? make_float2(ph, gp) : make_float2(0.f, 0.f);
      }
      __syncthreads();
      const float gp = phis[g.e].y;
      float v[32], gc[32];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        float y, dy;
        silu_grad_edge(v[q] + s_bc1[g.col0 + q], y, dy);
        gc[q] = gp * s_wc2[g.col0 + q] * dy;
        v[q] = gp * y;
      }
      st_row32_bf16(Gt, g.e, g.col0, gc);
      r_bc1 += warp_colsum32(gc);
      r_wc2 += warp_colsum32(v);
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < kM / 16; ++kk)
        mma_bf16(tWC1, desc_mn(Gt, kM, kk), desc_mn(Mt, kM, kk), C::IDESC_WGRAD, (first && kk == 0) ? 0u : 1u);
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Gt, kM, kk), desc_mn(Wc1t, H, kk), C::IDESC_DGRAD, kk > 0);
      mma_commit(bar);
    }
    if (!tanh_ && g.cg == 0) {   // phi of the one-pass path (its parts are complete after the handoff)
      const float p = part[g.e] + part[kM + g.e] + part[2 * kM + g.e] + part[3 * kM + g.e];
      phis[g.e] = make_float2(valid ? p : 0.f, 0.f);
    }
    // g_agg[i] slice of edge e: loads issued before the wait, used after it
    float4 gagg[8];
    {
      const float* ga = a.g_agg + (int64_t)rowi[g.e] * (a.ld_gagg ? a.ld_gagg : H) + g.col0;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        gagg[q] = valid ? *reinterpret_cast<const float4*>(ga + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;

    // ---- g_a2 = (g_m + g_agg[i]) silu'(a2) -> tile G ; column sums
    {
      float v[32];
      uint32_t w[16];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
      tmem_ld16u(tD2 + g.lane_base + g.col0 / 2, w);
#pragma unroll
      for (int q = 0; q < 32; q += 4) {
        const float4 g4 = gagg[q / 4];
        const float2 d01 = __half22float2(*reinterpret_cast<const __half2*>(&w[q / 2]));
        const float2 d23 = __half22float2(*reinterpret_cast<const __half2*>(&w[q / 2 + 1]));
        v[q] = valid ? (v[q] + g4.x) * d01.x : 0.f;
        v[q + 1] = valid ? (v[q + 1] + g4.y) * d01.y : 0.f;
        v[q + 2] = valid ? (v[q + 2] + g4.z) * d23.x : 0.f;
        v[q + 3] = valid ? (v[q + 3] + g4.w) * d23.y : 0.f;
      }
      st_row32_bf16(Gt, g.e, g.col0, v);
      r_b2 += warp_colsum32(v);
    }
    handoff_to_mma();
    if (g.tid == 0) {
#pragma unroll
      for (int kk = 0; kk < kM / 16; ++kk)
        mma_bf16(tW2, desc_mn(Gt, kM, kk), desc_mn(Ut, kM, kk), C::IDESC_WGRAD, (first && kk == 0) ? 0u : 1u);
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Gt, kM, kk), desc_mn(W2t, H, kk), C::IDESC_DGRAD, kk > 0);
#pragma unroll
      for (int kk = 0; kk < H / 16; ++kk)
        mma_bf16(tD0, desc_k(Gt, kM, kk), desc_mn(W2lo, H, kk), C::IDESC_DGRAD, 1u);
      mma_commit(bar);
    }
    first = false;
    if (!(ok = wait_mma(bar, phase, a.wait_polls))) break;

    // ---- g_a1 = g_u1 silu'(a1) -> global ; d-gradient
    {
      const float4 d = dl[g.e];
      float v[32];
      uint32_t w[16];
      tmem_ld32(tD0 + g.lane_base + g.col0, v);
      tmem_ld16u(tS1 + g.lane_base + g.col0 / 2, w);
      float pr = 0.f;
#pragma unroll
      for (int q = 0; q < 32; q += 2) {
        const float2 sv = __half22float2(*reinterpret_cast<const __half2*>(&w[q / 2]));
        v[q] = valid ? v[q] * sv.x : 0.f;
        v[q + 1] = valid ? v[q + 1] * sv.y : 0.f;
        pr = fmaf(v[q], s_wr[g.col0 + q], pr);
        pr = fmaf(v[q + 1], s_wr[g.col0 + q + 1], pr);
      }
      stage_write32(stage, g.e, g.col0, v);   // the M and G tiles are free again here
      part[g.cg * kM + g.e] = pr;
#pragma unroll
      for (int q = 0; q < 32; ++q) v[q] *= d.w;
      r_wr += warp_colsum32(v);
    }
    fence_before_sync();
    __syncthreads();
    if (g.cg == 0 && valid) {
      const float gr = part[g.e] + part[kM + g.e] + part[2 * kM + g.e] + part[3 * kM + g.e];
      const float4 d = dl[g.e], gt = gtr[g.e];
      const float f = phis[g.e].x * gt.w;
      a.gdstore[c0 + g.e] = make_float4(gt.x * f + 2.f * gr * d.x, gt.y * f + 2.f * gr * d.y,
                                        gt.z * f + 2.f * gr * d.z, 0.f);
    }
    // g_a1 rows of the chunk to global memory as bf16 (the operand of the
    // dst / src row sums), one warp per edge row, 8 bytes per lane
    __nv_bfloat16* gst = reinterpret_cast<__nv_bfloat16*>(a.gstore);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int e = g.warp * 8 + t;
      if (e < n) {
        const float4 w = stage[stage_word(e, g.lane)];
        const __nv_bfloat162 h01 = __floats2bfloat162_rn(w.x, w.y), h23 = __floats2bfloat162_rn(w.z, w.w);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&h01);
        u.y = *reinterpret_cast<const uint32_t*>(&h23);
        reinterpret_cast<uint2*>(gst + (c0 + e) * H)[g.lane] = u;
      }
    }
    if (prefetcher) cp_async_wait_all_groups();
    __syncthreads();
    pref = n_next > 0;
    if (*idx_abort) {   // read after the barrier: the same value in every thread
      ok = false;
      idx_drain = true;
      break;
    }
  }
  cp_async_wait_all_groups();   // nothing in flight when the CTA leaves (also after a timeout)
  if (g.tid == 0) {   // no index-tile copy may still be landing when the CTA leaves
    if (idx_pending) mbar_wait(ibar, iphase);
    if (idx_drain) mbar_wait(ibar, idx_last);
  }

  // ---- per-CTA partials: dWc1, dW2 rows from TMEM; column sums over the row quarters
  const int PF = (int)edge_part_floats(H, 0);
  float* out = a.part + (int64_t)cta * PF;
  if (ok) {
    if (first) {
      for (int c = g.tid; c < 2 * H * H; c += kNT) out[c] = 0.f;
    } else {
      float v[32];
      tmem_ld32(tWC1 + g.lane_base + g.col0, v);
#pragma unroll
      for (int q = 0; q < 32; q += 4)
        *reinterpret_cast<float4*>(out + g.e * H + g.col0 + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      tmem_ld32(tW2 + g.lane_base + g.col0, v);
#pragma unroll
      for (int q = 0; q < 32; q += 4)
        *reinterpret_cast<float4*>(out + H * H + g.e * H + g.col0 + q) =
            make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
    }
  }
  fence_before_sync();
  __syncthreads();
  float* red = reinterpret_cast<float*>(Ut);   // [4 quarters][4 vectors][H]
  {
    const int c = g.col0 + g.lane;
    red[(g.q * 4 + 0) * H + c] = r_bc1;
    red[(g.q * 4 + 1) * H + c] = r_b2;
    red[(g.q * 4 + 2) * H + c] = r_wc2;
    red[(g.q * 4 + 3) * H + c] = r_wr;
  }
  __syncthreads();
  for (int idx = g.tid; idx < 4 * H; idx += kNT) {
    const int v = idx / H, c = idx % H;
    out[2 * H * H + v * H + c] = red[(0 * 4 + v) * H + c] + red[(1 * 4 + v) * H + c] +
                                 red[(2 * 4 + v) * H + c] + red[(3 * 4 + v) * H + c];
  }
  __syncthreads();
  if (g.warp == 0) tmem_dealloc(tmem, NCOL);
}

// ---- node pass: the row sums of g_a1 and of the coordinate gradients -------------
// For node v, over its in-edges (its CSR row: S_dst, gd_dst) and over its
// out-edges (transpose CSR: S_src, gd_src), then
// dL/dx_v = dL/dx'_v + gd_dst - gd_src.  SPLIT warps per node, each owning
// H / SPLIT features (lane: H / (32 SPLIT) consecutive ones); UR rows of each
// list in flight per warp, each list added in CSR-position order.
template <int H, int SPLIT, int UR>
__global__ void node_pass_kernel(int64_t N, const int32_t* __restrict__ row_ptr,
                                 const int32_t* __restrict__ src_ptr, const int32_t* __restrict__ src_edge,
                                 const __nv_bfloat16* __restrict__ gstore, const float4* __restrict__ gdstore,
                                 const float* __restrict__ gx_out, float* __restrict__ S_dst,
                                 float* __restrict__ S_src, float* __restrict__ gx) {
  constexpr int HS = H / SPLIT, VW = HS / 32;
  pdl_enter();
  const int lane = threadIdx.x % 32;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t v = gw / SPLIT;
  const int part = (int)(gw % SPLIT);
  if (v >= N) return;
  gstore += part * HS;
  float sd[VW], ss[VW];
#pragma unroll
  for (int c = 0; c < VW; ++c) { sd[c] = 0.f; ss[c] = 0.f; }
  float gdd = 0.f, gds = 0.f;
  // lanes 0..2 read component `lane` of a coordinate gradient
  const float* gdf = reinterpret_cast<const float*>(gdstore);
  auto comp = [&](int64_t k) { return (lane < 3) ? __ldg(gdf + k * 4 + lane) : 0.f; };
  int kd = row_ptr[v];
  const int ked = row_ptr[v + 1];
  int ks = src_ptr[v];
  const int kes = src_ptr[v + 1];
  // the transpose-CSR positions of the next full round are loaded while this
  // round's rows are in flight
  int64_t p[UR];
  if (ks + UR <= kes) {
#pragma unroll
    for (int u = 0; u < UR; ++u) p[u] = src_edge[ks + u];
  }
  while (kd + UR <= ked || ks + UR <= kes) {   // warp-uniform
    const bool bd = kd + UR <= ked, bs = ks + UR <= kes;
    const bool bs_next = ks + 2 * UR <= kes;
    float vd[UR][VW], vs[UR][VW], gd1[UR], gs1[UR];
    if (bd) {
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        load_row_slice<HS>(gstore + (int64_t)(kd + u) * H, lane, vd[u]);
        gd1[u] = comp(kd + u);
      }
    }
    if (bs) {
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        load_row_slice<HS>(gstore + p[u] * H, lane, vs[u]);
        gs1[u] = comp(p[u]);
      }
    }
    int64_t pn[UR];
    if (bs_next) {
#pragma unroll
      for (int u = 0; u < UR; ++u) pn[u] = src_edge[ks + UR + u];
    }
    if (bd) {
#pragma unroll
      for (int u = 0; u < UR; ++u) {
#pragma unroll
        for (int c = 0; c < VW; ++c) sd[c] += vd[u][c];
        gdd += gd1[u];
      }
      kd += UR;
    }
    if (bs) {
#pragma unroll
      for (int u = 0; u < UR; ++u) {
#pragma unroll
        for (int c = 0; c < VW; ++c) ss[c] += vs[u][c];
        gds += gs1[u];
      }
      ks += UR;
    }
    if (bs_next) {
#pragma unroll
      for (int u = 0; u < UR; ++u) p[u] = pn[u];
    }
  }
  for (; kd < ked; ++kd) {
    float t[VW];
    load_row_slice<HS>(gstore + (int64_t)kd * H, lane, t);
#pragma unroll
    for (int c = 0; c < VW; ++c) sd[c] += t[c];
    gdd += comp(kd);
  }
  for (; ks < kes; ++ks) {
    const int64_t q = src_edge[ks];
    float t[VW];
    load_row_slice<HS>(gstore + q * H, lane, t);
#pragma unroll
    for (int c = 0; c < VW; ++c) ss[c] += t[c];
    gds += comp(q);
  }
  store_row_slice<HS>(S_dst + v * H + part * HS, lane, sd);
  store_row_slice<HS>(S_src + v * H + part * HS, lane, ss);
  if (lane < 3 && part == 0) gx[v * 3 + lane] = gx_out[v * 3 + lane] + gdd - gds;
}

// EGNN_DEBUG_WAIT_POLLS (debugging aid, read at every launch): the poll
// limit of the tensor-core kernels' MMA-completion waits; 0 makes every such
// wait give up at once, which exercises the give-up path.  Unset: -1.
int debug_wait_polls() {
  const char* v = getenv("EGNN_DEBUG_WAIT_POLLS");
  if (!v || !*v) return -1;
  const long n = strtol(v, nullptr, 10);
  return n < 0 ? -1 : (int)std::min<long>(n, 1L << 22);
}

template <int H>
int launch_fwd_tc(const EdgeFwdArgs& a_in, int G, cudaStream_t s) {
  EdgeFwdArgs a = a_in;
  a.wait_polls = debug_wait_polls();
  a.use_tma = tensor_map_i32_1d(&a.tm_row, a.row_idx, a.E, kM) && tensor_map_i32_1d(&a.tm_col, a.col_idx, a.E, kM);
  constexpr size_t bytes = FwdLayout<H>::BYTES;
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(edge_fwd_tc_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes));
    attr_set |= bit;
  }
  {
    TimerScope ts("edge_fwd", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_fwd_tc_kernel<H>, dim3(G), dim3(kNT), bytes, s, a));
  }
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

template <int H>
int launch_bwd_tc(const EdgeBwdArgs& a_in, int G, cudaStream_t s) {
  EdgeBwdArgs a = a_in;
  a.wait_polls = debug_wait_polls();
  a.use_tma = tensor_map_i32_1d(&a.tm_row, a.row_idx, a.E, kM) && tensor_map_i32_1d(&a.tm_col, a.col_idx, a.E, kM);
  constexpr size_t bytes = BwdLayout<H>::BYTES;
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(edge_bwd_tc_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes));
    attr_set |= bit;
  }
  {
    TimerScope ts("edge_bwd", s);
    EGNN_CHECK_CUDA(launch_pdl(edge_bwd_tc_kernel<H>, dim3(G), dim3(kNT), bytes, s, a));
  }
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

}  // namespace

bool edge_tc_supported(int H, int d, int flags, int precision) {
  // the backward of the attention gate runs on the SIMT kernels: the ungated
  // messages it needs would take TMEM columns the backward does not have
  return precision == EGNN_PREC_BF16 && H == 128 && d == 0 && !(flags & EGNN_FLAG_ATTENTION);
}

bool edge_tc_fwd_supported(int H, int d, int flags, int precision) {
  return precision == EGNN_PREC_BF16 && H == 128 && d <= 16;
}

EdgeGrid edge_tc_grid(int64_t E, int num_sms) {
  const int64_t chunks = std::max<int64_t>(1, (E + kM - 1) / kM);
  int64_t G = std::min<int64_t>(num_sms, chunks);
  const int64_t epc = (chunks + G - 1) / G * kM;
  G = std::max<int64_t>(1, (E + epc - 1) / epc);
  return EdgeGrid{(int)G, epc};
}

int edge_fwd_tc(int H, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
  if (H != 128) return fail(EGNN_ERR_UNSUPPORTED, "tensor-core edge path built for H = 128");
  EGNN_TRY(launch_fwd_tc<128>(a, g.G, s));
  if (g.G > 1) EGNN_TRY(edge_fixup_fwd(H, a, g, s));
  return EGNN_OK;
}

int edge_bwd_tc(int H, const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s) {
  if (H != 128) return fail(EGNN_ERR_UNSUPPORTED, "tensor-core edge path built for H = 128");
  return launch_bwd_tc<128>(a, g.G, s);
}

int edge_node_pass_tc(int H, int64_t N, const int32_t* row_ptr, const int32_t* src_ptr, const int32_t* src_edge,
                      const void* gstore, const float4* gdstore, const float* gx_out, float* S_dst, float* S_src,
                      float* gx, cudaStream_t s) {
  if (H != 128 && H != 256) return fail(EGNN_ERR_UNSUPPORTED, "node pass built for H = 128, 256");
  if (N <= 0) return EGNN_OK;
  // H = 256: four warps per node (more rows in flight per node; at H = 128 a
  // second warp per node measured slower)
  const int warps = 8, split = H == 128 ? 1 : 4;
  const unsigned blocks = (unsigned)((N * split + warps - 1) / warps);
  {
    TimerScope ts("node_pass", s);
    auto kern = H == 128 ? node_pass_kernel<128, 1, 4> : node_pass_kernel<256, 4, 4>;
    EGNN_CHECK_CUDA(launch_pdl(kern, dim3(blocks), dim3(warps * 32), 0, s, N, row_ptr, src_ptr, src_edge,
                               static_cast<const __nv_bfloat16*>(gstore), gdstore, gx_out, S_dst, S_src, gx));
  }
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

}  // namespace egnn

extern "C" int egnn_device_status(void* stream) {
  using namespace egnn;
  cudaStream_t s = (cudaStream_t)stream;
  EGNN_CHECK_CUDA(cudaStreamSynchronize(s));
  int n = 0;
  EGNN_CHECK_CUDA(cudaMemcpyFromSymbol(&n, g_tc_wait_timeouts, sizeof(int)));
  if (n != 0) {
    const int zero = 0;
    EGNN_CHECK_CUDA(cudaMemcpyToSymbol(g_tc_wait_timeouts, &zero, sizeof(int)));
  }
  n += node_tc_take_timeouts();
  n += rows_take_timeouts();
  if (n != 0) {
    return fail(EGNN_ERR_CUDA, "%d tensor-core wait(s) timed out; results are invalid", n);
  }
  return EGNN_OK;
}
