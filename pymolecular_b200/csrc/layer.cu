// C ABI of the EGNN layer: argument checks, workspace layout and the
// sequence of node GEMMs and fused edge kernels for one E_GCL forward and
// backward (egnn_clean.py:95-103 and its autograd).
//
// Forward:  PQ = h [Wa; Wb]^T + [b1; 0]            node GEMM (N x 2H)
//           edge_fwd: agg, x'                      fused edge kernel + fix-up
//           n1 = silu([h, agg] Wn1^T + bn1)        node GEMM
//           h' = h + n1 Wn2^T + bn2                node GEMM
// Backward: node-MLP backward (GEMMs), edge_bwd (dst pass, recompute),
//           src pass through the transpose CSR, then the W1 gradients and
//           dL/dh by node GEMMs.
// Precision: fp32 mode runs every GEMM in fp32 FFMA.  bf16 mode rounds the
// operands of the per-edge GEMMs (phi_e layer 2, phi_x layer 1 and their
// gradients, E rows) to bf16, except edge_mlp.2.weight (W2), which enters
// as hi + lo = bf16(W2) + bf16(W2 - bf16(W2)) (two MMAs on the tensor cores):
// a plain bf16 W2 is one fixed rounding shared by every edge, and the
// coordinate-MLP weight gradients (sums with heavy cancellation) amplify that
// systematic error tenfold past 2e-2.  The node-side GEMMs (N rows) run on the
// tensor cores with each fp32 operand split into two bf16 parts (about 16
// bits of precision).  Plain bf16 node-side operands would cost far more
// accuracy than time: on graphs with high in-degree rows the node MLP input
// [h, agg] and the projections P, Q lose several percent in their weight
// gradients.
#include <algorithm>
#include <map>
#include <mutex>
#include <thread>

#include "edge_rows.cuh"
#include "edge_simt.cuh"
#include "edge_tc.cuh"
#include "node_gemm.cuh"
#include "node_tc.cuh"

namespace egnn {
namespace {

bool valid_hidden(int H) { return H == 32 || H == 64 || H == 128 || H == 256; }

// input_nf and output_nf of the layer (0 in the descriptor: hidden_nf)
int in_dim(const egnn_layer_desc* d) { return d->in_dim ? d->in_dim : d->hidden; }
int out_dim(const egnn_layer_desc* d) { return d->out_dim ? d->out_dim : d->hidden; }

int check_desc(const egnn_layer_desc* d) {
  if (!d) return fail(EGNN_ERR_INVALID_ARG, "null layer descriptor");
  if (d->n_nodes < 0 || d->n_edges < 0 || d->n_nodes >= INT32_MAX || d->n_edges >= INT32_MAX)
    return fail(EGNN_ERR_INVALID_ARG, "N=%lld / E=%lld out of range", (long long)d->n_nodes,
                (long long)d->n_edges);
  if (!valid_hidden(d->hidden))
    return fail(EGNN_ERR_UNSUPPORTED, "hidden size %d not built (32, 64, 128, 256)", d->hidden);
  if (d->edge_attr_dim < 0 || d->edge_attr_dim > 16)
    return fail(EGNN_ERR_UNSUPPORTED, "edge_attr_dim %d not built (0..16)", d->edge_attr_dim);
  if (d->flags & ~31) return fail(EGNN_ERR_INVALID_ARG, "unknown flag bits 0x%x", d->flags);
  if (d->precision != EGNN_PREC_FP32 && d->precision != EGNN_PREC_BF16)
    return fail(EGNN_ERR_INVALID_ARG, "unknown precision %d", d->precision);
  if (d->in_dim < 0 || d->in_dim > 1024 || d->out_dim < 0 || d->out_dim > 1024)
    return fail(EGNN_ERR_UNSUPPORTED, "in_dim %d / out_dim %d not built (1..1024, 0 = hidden)", d->in_dim,
                d->out_dim);
  if ((d->flags & EGNN_FLAG_RESIDUAL) && in_dim(d) != out_dim(d))
    return fail(EGNN_ERR_INVALID_ARG, "the residual h + out needs in_dim == out_dim (%d, %d)", in_dim(d),
                out_dim(d));
  return EGNN_OK;
}

int resolve_sms(int num_sms) { return num_sms > 0 ? num_sms : num_sms_current(); }

// Upper bound on the edge-kernel CTA count (occupancy is at most 8 CTAs of
// 256 threads per SM).
int64_t max_ctas(int64_t E, int H, int num_sms) {
  const int T = edge_chunk(H);
  int64_t chunks = std::max<int64_t>(1, (E + T - 1) / T);
  return std::min<int64_t>(chunks, (int64_t)num_sms * 8);
}

// Prepared operands shared by the forward and the backward (I = input_nf,
// O = output_nf).
struct Prep {
  float4* xp; float* bias2; float* W2T; float* Wc1T; float* W2r; float* Wc1r; float* wr; float* We;
  float* WPQ;   // (2H, I): rows of edge_mlp.0 restricted to the h_i and h_j columns, contiguous
  // forward only: transposed weights (in x out), so that the forward node
  // GEMMs read their weight operand k-major like the backward ones
  float* Wn2T;  // (H, O):     node_mlp.2.weight^T
  float* Wn1T;  // (I + H, H): node_mlp.0.weight^T
  float* WPQT;  // (I, 2H):    WPQ^T
  // bf16 mode: the weight operands of the call's node GEMMs as split bf16
  // tile images (forward: WPQT, Wn1T, Wn2T; backward: node_mlp.2.weight,
  // node_mlp.0.weight, WPQ), built by prep_kernel
  BImage img[3];
};

enum { IMG_WPQT = 0, IMG_WN1T = 1, IMG_WN2T = 2, IMG_NW2 = 3, IMG_NW1 = 4, IMG_WPQ = 5 };

// Element (k, n) of the B operand an image holds (see Prep::img).
__device__ __forceinline__ float image_src(int kind, int64_t k, int64_t n, const egnn_layer_params& p, int H, int I,
                                           int64_t ld1) {
  switch (kind) {
    case IMG_WPQT: return n < H ? p.edge_w1[n * ld1 + k] : p.edge_w1[(n - H) * ld1 + I + k];
    case IMG_WN1T: return p.node_w1[n * (I + H) + k];
    case IMG_WN2T: return p.node_w2[n * H + k];
    case IMG_NW2: return p.node_w2[k * H + n];
    case IMG_NW1: return p.node_w1[k * (I + H) + n];
    default: return k < H ? p.edge_w1[k * ld1 + n] : p.edge_w1[(k - H) * ld1 + I + n];
  }
}

// 16-byte chunks (8 consecutive n) of the three images, in image order.
__host__ __device__ inline int64_t image_chunks(const BImage& b) { return b.base ? b.nkc * 64 * b.nb * 8 : 0; }

// `tc`: the tensor-core edge kernels read W2 and W_c1 as given, so the SIMT
// kernels' transposed / rounded copies are not made.
Prep carve_prep(Carver& c, int64_t N, int H, int I, int O, int d, bool bwd, bool tc, bool bf) {
  Prep p{};
  p.xp = c.take<float4>(std::max<int64_t>(N, 1));
  p.bias2 = c.take<float>(2 * H);
  p.W2T = tc ? nullptr : c.take<float>((size_t)H * H);
  p.Wc1T = tc ? nullptr : c.take<float>((size_t)H * H);
  p.W2r = (bwd && !tc) ? c.take<float>((size_t)H * H) : nullptr;
  p.Wc1r = (bwd && !tc) ? c.take<float>((size_t)H * H) : nullptr;
  p.wr = c.take<float>(H);
  p.We = c.take<float>((size_t)H * std::max(d, 1));
  p.WPQ = c.take<float>((size_t)2 * H * I);
  p.Wn2T = bwd ? nullptr : c.take<float>((size_t)H * O);
  p.Wn1T = bwd ? nullptr : c.take<float>((size_t)(I + H) * H);
  p.WPQT = bwd ? nullptr : c.take<float>((size_t)2 * H * I);
  if (bf) {
    const int64_t KN[3][2] = {{bwd ? O : I, bwd ? H : 2 * H}, {bwd ? H : I + H, bwd ? I + H : H},
                              {bwd ? 2 * H : H, bwd ? I : O}};
    for (int i = 0; i < 3; ++i) {
      p.img[i] = bimage_shape(KN[i][0], KN[i][1]);
      p.img[i].base = c.take<char>((size_t)p.img[i].bytes());
    }
  }
  return p;
}

__host__ __device__ inline int64_t prep_transposes(const Prep& o, int H, int I, int O) {
  return o.Wn2T ? (int64_t)H * O + (int64_t)(I + H) * H + 2LL * H * I : 0;
}
// The H x H copies of W2 / W_c1 the layout asks for: W2T, Wc1T, W2r, Wc1r in
// this order, the absent ones left out; sel[] lists the present ones.
__host__ __device__ inline int prep_copies(const Prep& o, int* sel) {
  int n = 0;
  if (o.W2T) sel[n++] = 0;
  if (o.Wc1T) sel[n++] = 1;
  if (o.W2r) sel[n++] = 2;
  if (o.Wc1r) sel[n++] = 3;
  return n;
}
__host__ __device__ inline int64_t prep_total(int64_t N, int H, int I, int O, int d, const Prep& o) {
  int sel[4];
  const int64_t HH = (int64_t)H * H;
  return N + 2 * H + prep_copies(o, sel) * HH + H + (int64_t)H * d + 2LL * H * I + prep_transposes(o, H, I, O);
}

// edge_mlp.0.weight (H, ld1 = 2I + 1 + d) columns: [0, I) h_i, [I, 2I) h_j,
// 2I the radial term, then the edge attributes.
__global__ void prep_kernel(int64_t N, int H, int I, int O, int d, int64_t ld1, int bf, egnn_layer_params p,
                            const float* x, Prep o) {
  pdl_enter();
  // the split bf16 images of the node GEMMs' weight operands
  {
    const int kind0 = o.Wn2T ? IMG_WPQT : IMG_NW2;
    const int64_t c0 = image_chunks(o.img[0]), c1 = image_chunks(o.img[1]), c2 = image_chunks(o.img[2]);
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < c0 + c1 + c2;
         idx += (int64_t)gridDim.x * blockDim.x) {
      int which = 0;
      int64_t t = idx;
      if (t >= c0) { t -= c0; which = 1; if (t >= c1) { t -= c1; which = 2; } }
      const BImage& b = o.img[which];
      const int64_t k = t / (b.nb * 8), n0 = (t % (b.nb * 8)) * 8;
      const int64_t kc = k >> 6, kr = k & 63, nb = n0 >> 6, nc = n0 & 63;
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int64_t n = n0 + 2 * q + u;
          v[u] = (k < b.K && n < b.N) ? image_src(kind0 + which, k, n, p, H, I, ld1) : 0.f;
        }
        const __nv_bfloat162 hp = __floats2bfloat162_rn(v[0], v[1]);
        const float2 hf = __bfloat1622float2(hp);
        const __nv_bfloat162 lp = __floats2bfloat162_rn(v[0] - hf.x, v[1] - hf.y);
        hw[q] = *reinterpret_cast<const uint32_t*>(&hp);
        lw[q] = *reinterpret_cast<const uint32_t*>(&lp);
      }
      // 128-byte swizzle: 16-byte chunk (nc / 8) of row kr at (nc / 8) ^ (kr % 8)
      const int64_t off = (kc * b.nb + nb) * 8192 + kr * 128 + (((nc >> 3) ^ (kr & 7)) << 4);
      *reinterpret_cast<uint4*>(b.base + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(b.base + b.part_bytes() + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
  const int64_t HH = (int64_t)H * H, HI = (int64_t)H * I, HO = (int64_t)H * O, IHH = (int64_t)(I + H) * H;
  int sel[4];
  const int ncopy = prep_copies(o, sel);
  const int64_t total = prep_total(N, H, I, O, d, o);
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = idx;
    if (o.Wn2T) {
      if (t < HO) {   // Wn2T[k][n] = node_w2[n][k], node_w2 is (O, H)
        o.Wn2T[t] = p.node_w2[(t % O) * H + t / O];
        continue;
      }
      t -= HO;
      if (t < IHH) {   // Wn1T[k][n] = node_w1[n][k], node_w1 is (H, I + H)
        o.Wn1T[t] = p.node_w1[(t % H) * (I + H) + t / H];
        continue;
      }
      t -= IHH;
      if (t < 2 * HI) {   // WPQT[k][n] = WPQ[n][k], k < I, n < 2H
        const int64_t k = t / (2 * H), n = t % (2 * H);
        o.WPQT[t] = n < H ? p.edge_w1[n * ld1 + k] : p.edge_w1[(n - H) * ld1 + I + k];
        continue;
      }
      t -= 2 * HI;
    }
    if (t < 2 * HI) {
      const int64_t r = t / I, c = t % I;   // WPQ[r][c]: r < H -> Wa, else Wb
      o.WPQ[t] = r < H ? p.edge_w1[r * ld1 + c] : p.edge_w1[(r - H) * ld1 + I + c];
      continue;
    }
    t -= 2 * HI;
    if (t < N) { o.xp[t] = make_float4(x[t * 3], x[t * 3 + 1], x[t * 3 + 2], 0.f); continue; }
    t -= N;
    if (t < 2 * H) { o.bias2[t] = t < H ? p.edge_b1[t] : 0.f; continue; }
    t -= 2 * H;
    if (t < ncopy * HH) {
      const int which = sel[t / HH];
      const int64_t r = t % HH, k = r / H, n = r % H;   // (k, n) of a [k][n] matrix
      float v;
      switch (which) {
        case 0: v = p.edge_w2[n * H + k]; o.W2T[r] = bf ? bf16_split(v) : v; break;
        case 1: v = p.coord_w1[n * H + k]; o.Wc1T[r] = bf ? bf16r(v) : v; break;
        case 2: v = p.edge_w2[r]; o.W2r[r] = bf ? bf16_split(v) : v; break;
        default: v = p.coord_w1[r]; o.Wc1r[r] = bf ? bf16r(v) : v; break;
      }
      continue;
    }
    t -= ncopy * HH;
    if (t < H) { o.wr[t] = p.edge_w1[t * ld1 + 2 * I]; continue; }
    t -= H;
    { const int64_t f = t / d, a = t % d; o.We[f * d + a] = p.edge_w1[f * ld1 + 2 * I + 1 + a]; }
  }
}

int launch_prep(int64_t N, int H, int I, int O, int d, int64_t ld1, bool bf, const egnn_layer_params* p,
                const float* x, const Prep& o, cudaStream_t s) {
  const int64_t total = std::max(prep_total(N, H, I, O, d, o),
                                 image_chunks(o.img[0]) + image_chunks(o.img[1]) + image_chunks(o.img[2]));
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 4096));
  TimerScope ts("prep", s);
  EGNN_CHECK_CUDA(launch_pdl(prep_kernel, dim3(blocks), dim3(256), 0, s, N, H, I, O, d, ld1, bf ? 1 : 0, *p, x,
                             o));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

// Node GEMMs: fp32 FFMA in fp32 mode, split-bf16 tensor cores in bf16 mode.
int node_gemm(const GemmArgs& g, bool bf, cudaStream_t s) {
  return (bf && gemm_tc_ok(g)) ? gemm_tc(g, s) : gemm(g, s);
}
int node_wgrad(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw, float* db, bool bf,
               float* part, cudaStream_t s) {
  return bf ? wgrad_tc(R, M, N, G, X, dW, lddw, db, part, s) : wgrad(R, M, N, G, X, dW, lddw, db, 0, part, s);
}

int gemm_pq(int64_t N, int H, int I, const float* h, const float* WPQT, const float* bias2, float* PQ, bool bf,
            const BImage& img, cudaStream_t s) {
  GemmArgs g;
  gemm_use_image(g, img);
  g.M = N; g.N = 2 * H; g.K = I;
  g.A = mat(h, I);
  g.B = mat(WPQT, 2 * H); g.b_t = 0;
  g.bias = bias2;
  g.C = PQ; g.ldc = 2 * H;
  g.round_bf16 = 0;
  return node_gemm(g, bf, s);
}

// Per-layer state the forward keeps for the backward (all per node):
// agg (N,H) | PQ (N,2H) | n1pre (N,H) | n1 (N,H).
struct Saved {
  float* agg; float* PQ; float* n1pre; float* n1;
};

Saved carve_saved(Carver& c, int64_t N, int H) {
  Saved v;
  const size_t n = (size_t)std::max<int64_t>(N, 1);
  v.agg = c.take<float>(n * H);
  v.PQ = c.take<float>(n * 2 * H);
  v.n1pre = c.take<float>(n * H);
  v.n1 = c.take<float>(n * H);
  return v;
}

struct FwdWs {
  Prep prep; float* carry; int32_t* carry_row; char* saved_tmp;
  RowsBufs rows;   // edge-row GEMM path only
};

FwdWs carve_fwd(Carver& c, const egnn_layer_desc* d, int num_sms) {
  const int64_t N = d->n_nodes, E = d->n_edges;
  const int H = d->hidden;
  FwdWs w;
  const bool rows = edge_rows_supported(H, d->edge_attr_dim, d->flags, d->precision);
  w.prep = carve_prep(c, N, H, in_dim(d), out_dim(d), d->edge_attr_dim, false,
                      rows || edge_tc_fwd_supported(H, d->edge_attr_dim, d->flags, d->precision),
                      d->precision == EGNN_PREC_BF16);
  const int64_t G = max_ctas(E, H, num_sms);
  w.carry = c.take<float>((size_t)G * 2 * (H + 4));
  w.carry_row = c.take<int32_t>((size_t)G * 2);
  Carver probe(nullptr);
  carve_saved(probe, N, H);
  w.saved_tmp = c.take<char>(probe.size());   // used when the caller keeps no state
  if (rows) w.rows = carve_rows(c, E, H, false, num_sms);
  return w;
}

// dL/dh from the node MLP and dL/dagg: one (N, I + H) product into ghg when
// I % 4 == 0; otherwise dL/dh (N, I) in ghg and dL/dagg (N, H) in gagg, so
// that the dL/dagg rows the edge kernels read 16 bytes at a time stay
// 16-byte aligned.
bool ghg_joint(int I) { return I % 4 == 0; }

struct BwdWs {
  Prep prep; float* g_n1pre; float* ghg; float* gagg;
  float* S_dst; float* S_src; float* gxd; float* gstore; float4* gdstore; float* carry;
  int32_t* carry_row; float* part; float* wpart;
  float* wpart_aux;   // split-K scratch of the weight gradients run on the side stream
  float* att_scr;     // attention only: per-CTA scratch of the SIMT edge backward
  RowsBufs rows;      // edge-row GEMM path only
};

// Split-K scratch of the layer's weight gradients: dW_n1 (H x (I + H)),
// dW_n2 (O x H), dW_a and dW_b (H x I).
int64_t wpart_floats(int64_t N, int H, int I, int O) {
  // slices of the FFMA split (wgrad) or of the tensor-core split (wgrad_tc)
  auto need = [&](int64_t M, int64_t K) {
    return std::max(wgrad_splits(N, M, K), wgrad_tc_splits(N, M, K)) * (M * K + M);
  };
  const int64_t c = colsum_splits(N) * (int64_t)std::max(I + H, O);
  return std::max<int64_t>({need(H, I + H), need(O, H), need(H, I), c, 1});
}

BwdWs carve_bwd(Carver& c, const egnn_layer_desc* d, int num_sms) {
  const int64_t N = std::max<int64_t>(d->n_nodes, 1), E = d->n_edges;
  const int H = d->hidden;
  BwdWs w;
  const int I = in_dim(d), O = out_dim(d);
  const bool rows = edge_rows_supported(H, d->edge_attr_dim, d->flags, d->precision);
  w.prep = carve_prep(c, N, H, I, O, d->edge_attr_dim, true,
                      rows || edge_tc_supported(H, d->edge_attr_dim, d->flags, d->precision),
                      d->precision == EGNN_PREC_BF16);
  w.g_n1pre = c.take<float>((size_t)N * H);
  w.ghg = c.take<float>((size_t)N * (ghg_joint(I) ? I + H : I));
  w.gagg = ghg_joint(I) ? w.ghg + I : c.take<float>((size_t)N * H);
  w.S_dst = c.take<float>((size_t)N * H);
  w.S_src = c.take<float>((size_t)N * H);
  w.gxd = c.take<float>((size_t)N * 3);
  w.gstore = c.take<float>((size_t)std::max<int64_t>(E, 1) * H);
  w.gdstore = c.take<float4>((size_t)std::max<int64_t>(E, 1));
  const int64_t G = max_ctas(E, H, num_sms);
  w.carry = c.take<float>((size_t)G * 2 * (H + 4));
  w.carry_row = c.take<int32_t>((size_t)G * 2);
  // the edge-row path keeps its per-CTA partials in w.rows.part
  w.part = rows ? nullptr : c.take<float>((size_t)G * edge_part_floats(H, d->edge_attr_dim));
  w.wpart = c.take<float>((size_t)wpart_floats(N, H, I, O));
  w.wpart_aux = c.take<float>((size_t)wpart_floats(N, H, I, O));
  w.att_scr = (d->flags & EGNN_FLAG_ATTENTION) ? c.take<float>((size_t)(G * edge_att_scratch_floats(H))) : nullptr;
  if (rows) w.rows = carve_rows(c, E, H, true, num_sms);
  return w;
}

// ---- side streams -----------------------------------------------------------------
// The backward forks work that no later kernel of the layer needs (the
// parameter gradients: node MLP, edge partial reduction, W1) onto two side
// streams, so that it fills SMs the edge kernels leave free and stays off the
// main chain.  Fork and join are event waits, which stream capture records as
// graph edges.
//
// Each caller stream gets its own pair of side streams and its own events
// (keyed by device and stream handle, and by thread for the per-thread
// default stream, whose handle every thread shares).  Calls on different
// streams therefore never record or wait on each other's events, and two host
// threads may run backwards concurrently on distinct streams.  Calls on the
// same stream are ordered by that stream; their host-side event records can
// only make one call wait for more of the other's work, never for less.  The
// streams and events of a new caller stream are created on its first call,
// with the thread switched to relaxed capture mode so that a first call made
// while that stream is being captured may create them.
struct SideStream {
  cudaStream_t stream = nullptr;    // node-MLP weight gradients, edge partials, dW_a
  cudaStream_t stream2 = nullptr;   // dW_b
  cudaEvent_t ev[8] = {};
};

struct SideKey {
  int dev;
  uintptr_t stream;
  std::thread::id thread;   // only for the per-thread default stream
  bool operator<(const SideKey& o) const {
    if (dev != o.dev) return dev < o.dev;
    if (stream != o.stream) return stream < o.stream;
    return thread < o.thread;
  }
};

int create_side(SideStream& ss) {
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  EGNN_CHECK_CUDA(cudaThreadExchangeStreamCaptureMode(&mode));
  cudaError_t e = cudaStreamCreateWithFlags(&ss.stream2, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking);
  for (auto& ev : ss.ev)
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaThreadExchangeStreamCaptureMode(&mode);
  EGNN_CHECK_CUDA(e);
  return EGNN_OK;
}

int side_stream(cudaStream_t caller, SideStream** out) {
  static std::mutex mu;
  static std::map<SideKey, SideStream*> sides;   // one entry per (device, caller stream); kept until exit
  int dev = 0;
  EGNN_CHECK_CUDA(cudaGetDevice(&dev));
  const uintptr_t h = reinterpret_cast<uintptr_t>(caller);
  const SideKey key{dev, h, h == reinterpret_cast<uintptr_t>(cudaStreamPerThread) ? std::this_thread::get_id()
                                                                                   : std::thread::id()};
  std::lock_guard<std::mutex> lk(mu);
  auto it = sides.find(key);
  if (it == sides.end()) {
    SideStream* ss = new SideStream();
    if (create_side(*ss) != EGNN_OK) {
      delete ss;
      return EGNN_ERR_CUDA;
    }
    it = sides.emplace(key, ss).first;
  }
  *out = it->second;
  return EGNN_OK;
}

// `to` waits for everything issued on `from` so far.
int stream_fork(cudaStream_t from, cudaStream_t to, cudaEvent_t ev) {
  EGNN_CHECK_CUDA(cudaEventRecord(ev, from));
  EGNN_CHECK_CUDA(cudaStreamWaitEvent(to, ev, 0));
  return EGNN_OK;
}

// Joins the side streams back into the main one when it goes out of scope
// (also on an early error return, so no capture is left forked).
struct SideJoin {
  cudaStream_t main_s;
  SideStream* side;
  ~SideJoin() {
    if (cudaEventRecord(side->ev[6], side->stream) == cudaSuccess) cudaStreamWaitEvent(main_s, side->ev[6], 0);
    if (cudaEventRecord(side->ev[7], side->stream2) == cudaSuccess) cudaStreamWaitEvent(main_s, side->ev[7], 0);
  }
};

bool missing_params(const egnn_layer_params* p, int flags) {
  return !p || !p->edge_w1 || !p->edge_b1 || !p->edge_w2 || !p->edge_b2 || !p->node_w1 ||
         !p->node_b1 || !p->node_w2 || !p->node_b2 || !p->coord_w1 || !p->coord_b1 || !p->coord_w2 ||
         ((flags & EGNN_FLAG_ATTENTION) && (!p->att_w || !p->att_b));
}

bool missing_graph(const egnn_graph* g, bool bwd, bool attr, int64_t E) {
  if (!g || !g->row_ptr) return true;
  if (bwd && !g->src_ptr) return true;
  if (E == 0) return false;   // per-edge arrays may be empty
  if (!g->col_idx || !g->row_idx) return true;
  if (attr && !g->edge_id) return true;
  if (bwd && !g->src_edge) return true;
  return false;
}

void fill_common(EdgeCommon& a, const egnn_layer_desc* d, const egnn_graph* g, const Prep& pr,
                 const float* PQ, const float* edge_attr, const egnn_layer_params* p, const EdgeGrid& eg) {
  a.N = d->n_nodes; a.E = d->n_edges;
  a.row_ptr = g->row_ptr; a.col_idx = g->col_idx; a.row_idx = g->row_idx; a.edge_id = g->edge_id;
  a.xp = pr.xp; a.PQ = PQ; a.wr = pr.wr; a.We = pr.We; a.attr = edge_attr; a.d = d->edge_attr_dim;
  a.W2T = pr.W2T; a.b2 = p->edge_b2; a.Wc1T = pr.Wc1T; a.bc1 = p->coord_b1; a.wc2 = p->coord_w2;
  a.W2_src = p->edge_w2; a.Wc1_src = p->coord_w1;
  a.wa = p->att_w; a.ba = p->att_b;
  a.flags = d->flags; a.epc = eg.epc;
}

}  // namespace
}  // namespace egnn

using namespace egnn;

extern "C" size_t egnn_saved_size(const egnn_layer_desc* d) {
  if (!d) return 0;
  Carver c(nullptr);
  carve_saved(c, d->n_nodes, d->hidden);
  return c.size();
}

extern "C" size_t egnn_workspace_size(const egnn_layer_desc* d, int which, int num_sms) {
  if (!d || check_desc(d) != EGNN_OK) return 0;
  const int sms = resolve_sms(num_sms);
  Carver c(nullptr);
  if (which == EGNN_WS_FWD) carve_fwd(c, d, sms); else carve_bwd(c, d, sms);
  return c.size();
}

extern "C" int egnn_layer_fwd(const egnn_layer_desc* d, const egnn_graph* g, const egnn_layer_params* p,
                              const float* h, const float* x, const float* edge_attr, float* h_out,
                              float* x_out, void* saved, void* ws, size_t ws_bytes, void* stream) {
  EGNN_TRY(check_desc(d));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t N = d->n_nodes, E = d->n_edges;
  const int H = d->hidden, dd = d->edge_attr_dim, I = in_dim(d), O = out_dim(d);
  const bool bf = d->precision == EGNN_PREC_BF16;
  if (N == 0) return EGNN_OK;
  if (missing_params(p, d->flags) || missing_graph(g, false, dd > 0, E) || !h || !x || !h_out || !x_out ||
      (dd > 0 && E > 0 && !edge_attr))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_layer_fwd: null pointer argument");
  const int sms = num_sms_current();
  Carver probe(nullptr);
  carve_fwd(probe, d, sms);
  if (!ws || ws_bytes < probe.size())
    return fail(EGNN_ERR_WORKSPACE, "egnn_layer_fwd: workspace %zu < %zu bytes", ws_bytes, probe.size());
  Carver c(ws);
  FwdWs w = carve_fwd(c, d, sms);
  const int64_t ld1 = 2 * I + 1 + dd;
  Carver sc(saved ? saved : static_cast<void*>(w.saved_tmp));
  const Saved sv = carve_saved(sc, N, H);
  float* agg = sv.agg;

  EGNN_TRY(launch_prep(N, H, I, O, dd, ld1, bf, p, x, w.prep, s));
  EGNN_TRY(gemm_pq(N, H, I, h, w.prep.WPQT, w.prep.bias2, sv.PQ, bf, w.prep.img[0], s));

  const bool rows = edge_rows_supported(H, dd, d->flags, d->precision);
  const bool tc = edge_tc_fwd_supported(H, dd, d->flags, d->precision);
  EdgeGrid eg{1, 0};
  if (tc) eg = edge_tc_grid(E, sms);
  else if (!rows) EGNN_TRY(edge_grid(H, false, bf, E, sms, &eg));
  EdgeFwdArgs a;
  fill_common(a, d, g, w.prep, sv.PQ, edge_attr, p, eg);
  a.carry = w.carry; a.carry_row = w.carry_row;
  a.x = x; a.agg = agg; a.x_out = x_out;
  if (rows) EGNN_TRY(edge_fwd_rows(a, w.rows, s));
  else if (tc) EGNN_TRY(edge_fwd_tc(H, a, eg, s));
  else EGNN_TRY(edge_fwd(H, bf, a, eg, s));

  GemmArgs n1;
  n1.M = N; n1.N = H; n1.K = I + H;
  n1.A = mat_cols(h, I, I, agg, H);
  n1.B = mat(w.prep.Wn1T, H); n1.b_t = 0;
  n1.bias = p->node_b1; n1.act = ACT_SILU;
  n1.pre = sv.n1pre; n1.ldp = H;
  n1.C = sv.n1; n1.ldc = H;
  gemm_use_image(n1, w.prep.img[1]);
  EGNN_TRY(node_gemm(n1, bf, s));

  GemmArgs n2;
  n2.M = N; n2.N = O; n2.K = H;
  n2.A = mat(sv.n1, H);
  n2.B = mat(w.prep.Wn2T, O); n2.b_t = 0;
  n2.bias = p->node_b2;
  if (d->flags & EGNN_FLAG_RESIDUAL) { n2.resid = h; n2.ldr = I; }   // I == O
  n2.C = h_out; n2.ldc = O;
  gemm_use_image(n2, w.prep.img[2]);
  EGNN_TRY(node_gemm(n2, bf, s));
  return EGNN_OK;
}

extern "C" int egnn_layer_bwd(const egnn_layer_desc* d, const egnn_graph* g, const egnn_layer_params* p,
                              const float* h, const float* x, const float* edge_attr, const void* saved,
                              const float* gh_out, const float* gx_out, float* grad_h, float* grad_x,
                              const egnn_layer_grads* gp, void* ws, size_t ws_bytes, void* stream) {
  EGNN_TRY(check_desc(d));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t N = d->n_nodes, E = d->n_edges;
  const int H = d->hidden, dd = d->edge_attr_dim, I = in_dim(d), O = out_dim(d);
  const bool bf = d->precision == EGNN_PREC_BF16;
  const bool residual = d->flags & EGNN_FLAG_RESIDUAL;
  if (missing_params(p, d->flags) || missing_graph(g, true, dd > 0, E) || !h || !x || !saved || !gh_out ||
      !gx_out || !grad_h || !grad_x || !gp || (dd > 0 && E > 0 && !edge_attr))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_layer_bwd: null pointer argument");
  if (!gp->edge_w1 || !gp->edge_b1 || !gp->edge_w2 || !gp->edge_b2 || !gp->node_w1 || !gp->node_b1 ||
      !gp->node_w2 || !gp->node_b2 || !gp->coord_w1 || !gp->coord_b1 || !gp->coord_w2 ||
      ((d->flags & EGNN_FLAG_ATTENTION) && (!gp->att_w || !gp->att_b)))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_layer_bwd: null gradient output");
  const int sms = num_sms_current();
  Carver probe(nullptr);
  carve_bwd(probe, d, sms);
  if (!ws || ws_bytes < probe.size())
    return fail(EGNN_ERR_WORKSPACE, "egnn_layer_bwd: workspace %zu < %zu bytes", ws_bytes, probe.size());
  Carver c(ws);
  BwdWs w = carve_bwd(c, d, sms);
  const int64_t ld1 = 2 * I + 1 + dd;
  Carver sc(const_cast<void*>(saved));
  const Saved sv = carve_saved(sc, N, H);
  const float* agg = sv.agg;
  if (N == 0) return EGNN_OK;

  EGNN_TRY(launch_prep(N, H, I, O, dd, ld1, bf, p, x, w.prep, s));
  SideStream* side = nullptr;
  EGNN_TRY(side_stream(s, &side));
  const cudaStream_t s2 = side->stream;
  SideJoin join{s, side};

  // ---- node MLP backward: h' = [h +] Wn2 silu(Wn1 [h, agg] + bn1) + bn2
  // dW_n2, db_n2 on the side stream (inputs ready at entry)
  EGNN_TRY(stream_fork(s, s2, side->ev[0]));
  EGNN_TRY(node_wgrad(N, O, H, mat(gh_out, O), mat(sv.n1, H), gp->node_w2, H, gp->node_b2, bf, w.wpart_aux, s2));
  {
    GemmArgs gn;
    gn.M = N; gn.N = H; gn.K = O;
    gn.A = mat(gh_out, O);
    gn.B = mat(p->node_w2, H); gn.b_t = 0;
    gn.act = ACT_DSILU; gn.aux = sv.n1pre; gn.ldaux = H;
    gn.C = w.g_n1pre; gn.ldc = H;
    gemm_use_image(gn, w.prep.img[0]);
    EGNN_TRY(node_gemm(gn, bf, s));
  }
  // dW_n1, db_n1 on the side stream once g_n1pre exists
  EGNN_TRY(stream_fork(s, s2, side->ev[1]));
  EGNN_TRY(node_wgrad(N, H, I + H, mat(w.g_n1pre, H), mat_cols(h, I, I, agg, H), gp->node_w1, I + H,
                      gp->node_b1, bf, w.wpart_aux, s2));
  const bool joint = ghg_joint(I);
  const int64_t ld_ghg = joint ? I + H : I;
  {
    // [dL/dh (MLP path) + residual | dL/dagg] = g_n1pre Wn1: one N x (I + H)
    // product, or its dL/dh columns here and the dL/dagg columns below
    GemmArgs gh;
    gh.M = N; gh.N = joint ? I + H : I; gh.K = H;
    gh.A = mat(w.g_n1pre, H);
    gh.B = mat(p->node_w1, I + H); gh.b_t = 0;
    if (residual) { gh.resid = gh_out; gh.ldr = O; gh.resid_cols = I; }   // I == O
    gh.C = w.ghg; gh.ldc = ld_ghg;
    gemm_use_image(gh, w.prep.img[1]);   // its columns start at the image's first block
    EGNN_TRY(node_gemm(gh, bf, s));
  }
  if (!joint) {
    GemmArgs ga;
    ga.M = N; ga.N = H; ga.K = H;
    ga.A = mat(w.g_n1pre, H);
    ga.B = mat(p->node_w1 + I, I + H); ga.b_t = 0;
    ga.C = w.gagg; ga.ldc = H;
    EGNN_TRY(node_gemm(ga, bf, s));
  }

  // ---- edge backward: dst pass, fix-up, partial reduction, src pass
  const bool rows = edge_rows_supported(H, dd, d->flags, d->precision);
  const bool tc = edge_tc_supported(H, dd, d->flags, d->precision);
  EdgeGrid eg{1, 0};
  if (tc) eg = edge_tc_grid(E, sms);
  else if (!rows) EGNN_TRY(edge_grid(H, true, bf, E, sms, &eg));
  EdgeBwdArgs a;
  fill_common(a, d, g, w.prep, sv.PQ, edge_attr, p, eg);
  a.carry = w.carry; a.carry_row = w.carry_row;
  a.W2 = bf ? w.prep.W2r : p->edge_w2;
  a.Wc1 = bf ? w.prep.Wc1r : p->coord_w1;
  a.gx_out = gx_out; a.g_agg = w.gagg; a.ld_gagg = joint ? I + H : H;
  a.S_dst = w.S_dst; a.gxd = w.gxd; a.gstore = w.gstore; a.gdstore = w.gdstore; a.part = w.part;
  a.att_scr = w.att_scr;
  if (rows) {
    EGNN_TRY(edge_bwd_rows(a, w.rows, s));
    // dW_c1, dW_2 and the partial reduction on the side stream
    EGNN_TRY(stream_fork(s, s2, side->ev[2]));
    EGNN_TRY(edge_wgrad_rows(E, w.rows, s2));
    EGNN_TRY(edge_part_reduce(H, dd, false, w.rows.G, w.rows.part, gp, ld1, 2 * I, s2));
  } else {
    if (tc) EGNN_TRY(edge_bwd_tc(H, a, eg, s));
    else EGNN_TRY(edge_bwd(H, bf, a, eg, s));
    // per-CTA weight-gradient partials -> parameter gradients, on the side stream
    EGNN_TRY(stream_fork(s, s2, side->ev[2]));
    EGNN_TRY(edge_part_reduce(H, dd, (d->flags & EGNN_FLAG_ATTENTION) != 0, eg.G, w.part, gp, ld1, 2 * I, s2));
  }
  if (tc || rows)
    EGNN_TRY(edge_node_pass_tc(H, N, g->row_ptr, g->src_ptr, g->src_edge, w.gstore, w.gdstore, gx_out, w.S_dst,
                               w.S_src, grad_x, s));
  else
    EGNN_TRY(edge_src_pass(H, N, g->src_ptr, g->src_edge, w.gstore, false, w.gdstore, gx_out, w.gxd, w.S_src,
                           grad_x, s));

  // ---- dL/dh = gh_acc + S_dst Wa + S_src Wb here; dWa, db1 and dWb on the two side streams
  EGNN_TRY(stream_fork(s, s2, side->ev[3]));
  EGNN_TRY(stream_fork(s, side->stream2, side->ev[4]));
  EGNN_TRY(node_wgrad(N, H, I, mat(w.S_src, H), mat(h, I), gp->edge_w1 + I, ld1, nullptr, bf, w.wpart,
                      side->stream2));
  EGNN_TRY(node_wgrad(N, H, I, mat(w.S_dst, H), mat(h, I), gp->edge_w1, ld1, gp->edge_b1, bf, w.wpart_aux, s2));
  {
    GemmArgs gh;
    gh.M = N; gh.N = I; gh.K = 2 * H;
    gh.A = mat_cols(w.S_dst, H, H, w.S_src, H);
    gh.B = mat(w.prep.WPQ, I); gh.b_t = 0;
    gh.resid = w.ghg; gh.ldr = ld_ghg;
    gh.C = grad_h; gh.ldc = I;
    gemm_use_image(gh, w.prep.img[2]);
    EGNN_TRY(node_gemm(gh, bf, s));
  }
  return EGNN_OK;
}

extern "C" int egnn_linear_fwd(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                               const float* b, float* y, void* stream) {
  if (m < 0 || k <= 0 || o <= 0) return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_fwd: bad shape");
  if (m == 0) return EGNN_OK;
  if (!x || !w || !y) return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_fwd: null pointer");
  if (linear_small_ok(o, k)) return linear_small(m, o, k, x, k, w, 1, b, y, o, (cudaStream_t)stream);
  GemmArgs g;
  g.M = m; g.N = o; g.K = k;
  g.A = mat(x, k);
  g.B = mat(w, k); g.b_t = 1;
  g.bias = b;
  g.C = y; g.ldc = o;
  return gemm(g, (cudaStream_t)stream);
}

extern "C" size_t egnn_linear_workspace_size(int64_t m, int32_t k, int32_t o) {
  Carver c(nullptr);
  c.take<float>((size_t)std::max<int64_t>(
      {wgrad_splits(m, o, k) * ((int64_t)o * k + o), colsum_splits(m) * (int64_t)o, 1}));
  return c.size();
}

extern "C" int egnn_linear_bwd(int64_t m, int32_t k, int32_t o, const float* x, const float* w,
                               const float* dy, float* dx, float* dw, float* db, void* ws,
                               size_t ws_bytes, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (m < 0 || k <= 0 || o <= 0) return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_bwd: bad shape");
  if (!x || !w || !dy || !dw) return fail(EGNN_ERR_INVALID_ARG, "egnn_linear_bwd: null pointer");
  if (!ws || ws_bytes < egnn_linear_workspace_size(m, k, o))
    return fail(EGNN_ERR_WORKSPACE, "egnn_linear_bwd: workspace too small");
  float* part = static_cast<float*>(ws);
  if (dx && m > 0) {
    if (linear_small_ok(k, o)) {
      EGNN_TRY(linear_small(m, k, o, dy, o, w, 0, nullptr, dx, k, s));
    } else {
      GemmArgs g;
      g.M = m; g.N = k; g.K = o;
      g.A = mat(dy, o);
      g.B = mat(w, k); g.b_t = 0;
      g.C = dx; g.ldc = k;
      EGNN_TRY(gemm(g, s));
    }
  }
  return wgrad(m, o, k, mat(dy, o), mat(x, k), dw, k, db, 0, part, s);
}
