// EGNN edge MLPs of a bf16-GEMM layer with H = 256 as edge-row GEMMs on the
// 5th-generation tensor cores.
//
// At H = 256 the two bf16 weight tiles of the fused edge kernels (W2 and
// W_c1, 128 KB each) do not fit one CTA's shared memory together, so each
// per-edge product runs as its own persistent GEMM over 128-edge tiles with
// ONE weight matrix resident in shared memory (128 KB) and a fused epilogue:
//
//   forward   u1 = silu(P_i + Q_j + w_r r)                gather kernel -> U
//             a2 = U W2^T;  m = silu(a2 + b2)             GEMM -> Mb (bf16) and fp32 m
//                                                         (backward: fp16 silu'(a2 + b2))
//             c1 = Mb Wc1^T; phi = wc2 . silu(c1 + bc1)   GEMM -> phi
//             agg_i = sum m, x'_i = x_i + s_i sum d phi   row kernel
//   backward  (recompute U, a2, m, c1 as above)
//             g_c1 = gphi wc2 silu'(c1)                   GEMM epilogue -> Gc1 (bf16)
//             g_a2 = (Gc1 Wc1 + g_agg[i]) silu'(a2)       GEMM -> Ga2 (bf16)
//             g_a1 = (Ga2 W2) silu'(a1)                   GEMM -> bf16 rows, g_d
//                    (silu'(a1) stored in fp16 by the backward's gather)
//             dWc1 = Gc1^T Mb, dW2 = Ga2^T U              split-K GEMMs over the edges
//
// The rounding points are those of the fused kernels (bf16 GEMM operands u1,
// m, g_c1, g_a2 and weights; fp32 accumulation; fp32 m in the row sums; bf16
// dL/da1 rows for the node pass; silu'(a2) kept in fp16 between kernels, as
// the fused kernels stage it), so the same rounding-exact model covers both
// paths.
//
// Operands move as "tiles": the bf16 (E, 256) matrices are stored tile-major,
// 64 KB per 128 edges, as four 16 KB column blocks of 128 rows x 64 features
// in the 128-byte swizzle (16-byte chunk c of row r at position c ^ (r % 8)),
// exactly the shared-memory image the MMA reads.  One cp.async.bulk copy
// (no tensor map, no multicast) moves a block; an mbarrier counts its bytes.
//
// GEMM kernel (one CTA per SM, 576 threads): warp 0 streams the A blocks of
// the CTA's tiles through a 3-stage ring, warp 1 issues tcgen05.mma (M = 128
// edges, N = 256, K = 16 per instruction) into one of two TMEM accumulators
// (2 x 256 columns), warps 2..17 run the epilogue of tile j while the MMAs of
// tile j + 1 run.  The three products with W2 (a2 in the forward and in the
// backward's recompute, g_u = G_a2 W2) multiply by W2 as a pair of bf16
// matrices, hi = bf16(W2) and lo = bf16(W2 - hi): a single bf16 W2 is one
// rounding shared by every edge, a systematic error that the coordinate-MLP
// weight gradients amplify far past the bf16 tolerance.  Both halves (256 KB)
// do not fit beside the ring, so these variants keep no weight resident: each
// ring stage carries an A block and the matching 64-deep K slice of W2 hi and
// lo (80 KB, two stages), copied from a bf16 image of W2 in global memory
// that stays in L2 (written per layer call by rows_wimg_kernel).  An epilogue thread owns one edge row and 64 features, so its
// row-major global traffic would touch 32 rows per warp instruction: stores and
// the fp16 side-row loads go through a 2 KB per-warp shared staging instead, so
// that each instruction moves whole 64- or 128-byte row pieces.  Every wait is
// bounded (2 s of global time); a thread that
// gives up raises a CTA abort flag that every other wait honours, the count
// is reported by egnn_device_status, and the CTA frees its TMEM and exits.
// Column sums (bias and w_c2 / w_r gradients) are per-warp transposing
// reductions kept per thread across tiles, then added per CTA in fixed order:
// results are bit-deterministic for a given GPU.
#include <algorithm>

#include "edge_rows.cuh"
#include "tc.cuh"

namespace egnn {

__device__ int g_rows_timeouts = 0;

namespace {

using namespace tc;

constexpr int kH = 256;
constexpr int kTile = 128 * kH * 2;   // bytes per 128-edge tile
constexpr int kBlk = 128 * 128;       // bytes per 64-feature column block of a tile
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`: false once 2 s have passed (the CTA's
// abort flag is raised and the event counted) or, when `abort_flag` is
// given, once another thread has raised it.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* raise_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (global_ns() - t0 > kWaitNs) {
      *reinterpret_cast<volatile int*>(raise_flag) = 1;
      atomicAdd(&g_rows_timeouts, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bulk copy global -> shared (16-byte aligned, size a multiple of 16), the
// bytes counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Named barriers of the 16 epilogue warps (512 threads).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }
__device__ __forceinline__ bool epi_any(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q, o;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred o, 2, 512, q;\n\t"
      "selp.u32 %0, 1, 0, o;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Warp-collective store of one 64-byte piece per row through the warp's 2 KB
// staging buffer: lane l owns row l's 16 words w[]; `dst` is that row's
// 64-byte destination (nullptr: not stored) and its logical 16-byte chunk c
// goes to position c ^ perm there.  Rows are written to the staging in an
// XOR-swizzled slot order (no bank conflicts) and read back four lanes per
// row, so every global store instruction covers eight whole 64-byte pieces
// (whole 32-byte sectors) instead of 16 bytes of 32 different rows.
__device__ __forceinline__ void store_rows64(char* stg, const uint32_t (&w)[16], char* dst, int perm) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  __syncwarp();
  const unsigned long long dv = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int hr = 8 * k + (lane >> 2), cc = lane & 3;
    const uint4 val = *reinterpret_cast<const uint4*>(stg + hr * 64 + ((cc ^ ((hr >> 1) & 3)) << 4));
    const unsigned long long d = __shfl_sync(0xffffffffu, dv, hr);
    const int pm = __shfl_sync(0xffffffffu, perm, hr);
    if (d) *reinterpret_cast<uint4*>(reinterpret_cast<char*>(d) + ((cc ^ pm) << 4)) = val;
  }
  __syncwarp();
}

// Warp-collective load of the 128-byte slices (fp16 features 64 cs .. + 63) of
// rows row0 .. row0 + 31 of a row-major (E, 256) fp16 matrix: lane l receives
// row row0 + l in side[].  Eight lanes read each slice (four whole 128-byte
// lines per load instruction), in two rounds of 16 rows through the warp's
// 2 KB staging (XOR-swizzled slots); rows >= E read row 0 (the caller masks them).
__device__ __forceinline__ void load_rows128(char* stg, const __half* base, int64_t row0, int64_t E, int cs,
                                             uint4 (&side)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int rr = 4 * k + (lane >> 3), c = lane & 7;
      const int64_t row = row0 + 16 * h + rr;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (row < E ? row : 0) * kH + cs * 64) + c);
      *reinterpret_cast<uint4*>(stg + rr * 128 + ((c ^ (rr & 7)) << 4)) = v;
    }
    __syncwarp();
    if ((lane >> 4) == h) {
      const int rr = lane & 15;
#pragma unroll
      for (int c = 0; c < 8; ++c) side[c] = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((c ^ (rr & 7)) << 4));
    }
    __syncwarp();
  }
}

// 32 values = features 64 cs + 32 p .. + 31 of row `el` of the tile at `tb`
// (in the 128-byte swizzle the piece is one aligned 64-byte half row whose
// chunks are permuted by el % 4).
__device__ __forceinline__ void st_tile_piece(char* stg, char* tb, int el, int cs, int p, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  store_rows64(stg, w, tb + cs * kBlk + el * 128 + ((((p << 2) ^ (el & 4))) << 4), el & 3);
}

// 32 values of a row-major row at `dst` (nullptr: row not stored).
__device__ __forceinline__ void st_f32_piece(char* stg, float* dst, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[16 * h + i]);
    store_rows64(stg, w, dst ? reinterpret_cast<char*>(dst + 16 * h) : nullptr, 0);
  }
}
__device__ __forceinline__ void st_f16_piece(char* stg, __half* dst, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  store_rows64(stg, w, reinterpret_cast<char*>(dst), 0);
}
__device__ __forceinline__ void st_bf16_piece(char* stg, __nv_bfloat16* dst, const float (&v)[32]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  store_rows64(stg, w, reinterpret_cast<char*>(dst), 0);
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Sum over the warp's 32 lanes of x[c]; lane l returns the sum for c = l.
__device__ __forceinline__ float colsum32(float (&x)[32]) {
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

// (256 x 256) fp32 W -> two bf16 tile images in global memory, the exact
// shared-memory image load_w256 writes: img = bf16(W), img + 128 KB =
// bf16(W - bf16(W)).
__global__ void __launch_bounds__(256) rows_wimg_kernel(const float* __restrict__ W, char* __restrict__ img) {
  pdl_enter();
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < kH * kH / 8; idx += gridDim.x * blockDim.x) {
    const int o = idx / (kH / 8), c8 = (idx % (kH / 8)) * 8;
    const float4 a = __ldg(reinterpret_cast<const float4*>(W + o * kH + c8));
    const float4 b = __ldg(reinterpret_cast<const float4*>(W + o * kH + c8 + 4));
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st_row8_bf16(img, kH, o, c8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] -= bf16r(v[k]);
    st_row8_bf16(img + kH * kH * 2, kH, o, c8, v);
  }
}

// (256 x 256) fp32 nn.Linear weight -> bf16 tile with rows = out, columns = in
// (K-major operand of x W^T, MN-major operand of g W).
__device__ void load_w256(char* tile, const float* __restrict__ W) {
  for (int idx = threadIdx.x; idx < kH * kH / 8; idx += blockDim.x) {
    const int o = idx / (kH / 8), c8 = (idx % (kH / 8)) * 8;
    const float4 a = __ldg(reinterpret_cast<const float4*>(W + o * kH + c8));
    const float4 b = __ldg(reinterpret_cast<const float4*>(W + o * kH + c8 + 4));
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st_row8_bf16(tile, kH, o, c8, v);
  }
}

// ---- gather: geometry and u1 = bf16(silu(P_i + Q_j + w_r r)) -------------------------
// A warp takes groups of EPW consecutive edges of the padded tile range, their
// coordinate and P / Q row loads all in flight together; lane owns features
// 8 lane .. + 7 (16 bytes of each tile row).  Padding rows (e >= E) are zero.
// With S1 (backward) the warp also stores silu'(a1) as fp16 rows (E, 256).
constexpr int EPW = 4;
template <bool WITH_S1>
__global__ void __launch_bounds__(256) rows_u_kernel(int64_t E, int64_t Epad, const int32_t* __restrict__ row_idx,
                                                     const int32_t* __restrict__ col_idx,
                                                     const float4* __restrict__ xp, const float* __restrict__ PQ,
                                                     const float* __restrict__ wr, char* __restrict__ U,
                                                     float4* __restrict__ geo, __half* __restrict__ S1,
                                                     const int32_t* __restrict__ row_ptr,
                                                     const float* __restrict__ gx_out, int flags,
                                                     float4* __restrict__ gtr) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t ngroups = Epad / EPW, gstride = (int64_t)gridDim.x * 8;
  int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (g >= ngroups) return;
  const float4 w0 = ldg4(wr + 8 * lane), w1 = ldg4(wr + 8 * lane + 4);
  const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  // grid-stride over groups of EPW edges; each iteration requests the next
  // group's indices while this group's rows are in flight
  int iv[EPW], jv[EPW];
#pragma unroll
  for (int k = 0; k < EPW; ++k) {
    const int64_t e = g * EPW + k;
    iv[k] = e < E ? row_idx[e] : 0;
    jv[k] = e < E ? col_idx[e] : 0;
  }
#pragma unroll 1
  for (; g < ngroups; g += gstride) {
    const int64_t e0 = g * EPW;
    // backward: lane k < EPW also forms edge e0 + k's coordinate-gradient
    // factors (its loads issued here, beside the row loads below)
    const bool gl = WITH_S1 && lane < EPW && e0 + lane < E;
    int mi = 0, mj = 0, rp0 = 0, rp1 = 0;
    float gxv[3] = {0.f, 0.f, 0.f}, myr = 0.f;
#pragma unroll
    for (int k = 0; k < EPW; ++k)
      if (lane == k) { mi = iv[k]; mj = jv[k]; }
    if (gl) {
      rp0 = row_ptr[mi];
      rp1 = row_ptr[mi + 1];
#pragma unroll
      for (int c = 0; c < 3; ++c) gxv[c] = gx_out[(int64_t)mi * 3 + c];
    }
    float4 xi[EPW], xj[EPW], pv[EPW][2], qv[EPW][2];
#pragma unroll
    for (int k = 0; k < EPW; ++k) {
      xi[k] = xp[iv[k]];
      xj[k] = xp[jv[k]];
      const float* P = PQ + (int64_t)iv[k] * 2 * kH + 8 * lane;
      const float* Q = PQ + (int64_t)jv[k] * 2 * kH + kH + 8 * lane;
      pv[k][0] = ldg4(P);
      pv[k][1] = ldg4(P + 4);
      qv[k][0] = ldg4(Q);
      qv[k][1] = ldg4(Q + 4);
    }
    const int64_t gn = g + gstride;
#pragma unroll
    for (int k = 0; k < EPW; ++k) {
      const int64_t e = gn * EPW + k;
      iv[k] = (gn < ngroups && e < E) ? row_idx[e] : 0;
      jv[k] = (gn < ngroups && e < E) ? col_idx[e] : 0;
    }
#pragma unroll
    for (int k = 0; k < EPW; ++k) {
      const int64_t e = e0 + k;
      const bool ok = e < E;
      const float dx = xi[k].x - xj[k].x, dy = xi[k].y - xj[k].y, dz = xi[k].z - xj[k].z;
      const float r = dx * dx + dy * dy + dz * dz;
      if (ok && lane == 0) geo[e] = make_float4(dx, dy, dz, r);
      if (lane == k) myr = r;
      const float pp[8] = {pv[k][0].x, pv[k][0].y, pv[k][0].z, pv[k][0].w,
                           pv[k][1].x, pv[k][1].y, pv[k][1].z, pv[k][1].w};
      const float qq[8] = {qv[k][0].x, qv[k][0].y, qv[k][0].z, qv[k][0].w,
                           qv[k][1].x, qv[k][1].y, qv[k][1].z, qv[k][1].w};
      float u[8], d[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float a1 = fmaf(w[c], r, pp[c] + qq[c]);
        if constexpr (WITH_S1) silu_grad_edge(a1, u[c], d[c]);
        else u[c] = silu_edge(a1);
        if (!ok) u[c] = 0.f;
      }
      const int64_t t = e >> 7;
      const int rl = (int)(e & 127), blk = lane >> 3, ch = lane & 7;
      const uint4 pk = make_uint4(pack_bf16x2(u[0], u[1]), pack_bf16x2(u[2], u[3]), pack_bf16x2(u[4], u[5]),
                                  pack_bf16x2(u[6], u[7]));
      *reinterpret_cast<uint4*>(U + t * kTile + blk * kBlk + rl * 128 + ((ch ^ (rl & 7)) << 4)) = pk;
      if (WITH_S1 && ok) {
        uint32_t hw[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const __half2 h2 = __floats2half2_rn(d[2 * c], d[2 * c + 1]);
          hw[c] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(S1 + e * kH + 8 * lane) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      }
    }
    if (gl) {   // (g_t s_i, 1 / (|d| + eps)) with the second term 0 on self-loops
      const float sc = (flags & EGNN_FLAG_COORDS_SUM) ? 1.f : 1.f / (float)max(rp1 - rp0, 1);
      const float inv = (flags & EGNN_FLAG_NORMALIZE) ? 1.f / (sqrtf(myr) + 1e-8f) : 1.f;
      gtr[e0 + lane] = make_float4(gxv[0] * sc, gxv[1] * sc, gxv[2] * sc, mi == mj ? 0.f : inv);
    }
  }
}

// ---- forward row sums: agg_i = sum m_e, x'_i = x_i + s_i sum d_e inv_e phi_e -----------
// Two warps per node, each owning 128 features (lane: 4 consecutive ones), its
// CSR row in order with four rows in flight; the first warp also sums the
// coordinate terms.
__global__ void __launch_bounds__(256) rows_agg_kernel(int64_t N, const int32_t* __restrict__ row_ptr,
                                                       const float* __restrict__ M32, const float* __restrict__ phi,
                                                       const float4* __restrict__ geo, const float* __restrict__ x,
                                                       int flags, float* __restrict__ agg,
                                                       float* __restrict__ x_out) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t v = gw >> 1;
  const int part = (int)(gw & 1);
  if (v >= N) return;
  const bool normalize = flags & EGNN_FLAG_NORMALIZE;
  const bool xl = part == 0 && lane < 3;   // lanes that sum a coordinate component
  const int k0 = row_ptr[v], k1 = row_ptr[v + 1];
  const int f0 = part * (kH / 2) + 4 * lane;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  float xs = 0.f;
  auto xterm = [&](int64_t k) {
    const float4 g = __ldg(geo + k);
    const float inv = normalize ? 1.f / (sqrtf(g.w) + 1e-8f) : 1.f;
    const float d = lane == 0 ? g.x : (lane == 1 ? g.y : g.z);
    return (d * inv) * __ldg(phi + k);
  };
  int k = k0;
  for (; k + 4 <= k1; k += 4) {
    float4 a[4];
    float xt[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      a[u] = ldg4(M32 + (int64_t)(k + u) * kH + f0);
      xt[u] = xl ? xterm(k + u) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[0] += a[u].x; s[1] += a[u].y; s[2] += a[u].z; s[3] += a[u].w;
      xs += xt[u];
    }
  }
  for (; k < k1; ++k) {
    const float4 a0 = ldg4(M32 + (int64_t)k * kH + f0);
    s[0] += a0.x; s[1] += a0.y; s[2] += a0.z; s[3] += a0.w;
    if (xl) xs += xterm(k);
  }
  *reinterpret_cast<float4*>(agg + v * kH + f0) = make_float4(s[0], s[1], s[2], s[3]);
  if (xl) {
    const float sc = (flags & EGNN_FLAG_COORDS_SUM) ? 1.f : 1.f / (float)max(k1 - k0, 1);
    x_out[v * 3 + lane] = x[v * 3 + lane] + xs * sc;
  }
}

// ---- persistent edge-row GEMM with fused epilogues ------------------------------------
enum { EPI_M_FWD = 0, EPI_M_BWD, EPI_PHI, EPI_GC1, EPI_GA2, EPI_GA1 };

struct RowsGemmArgs {
  const char* A = nullptr;        // tiles of the A operand (K-major, K = 256)
  const float* W = nullptr;       // (256, 256) fp32 weight [out][in]
  const char* Wimg = nullptr;     // W2 products: bf16 hi | lo images of W (rows_wimg_kernel)
  int64_t E = 0, ntiles = 0;
  const float* bias = nullptr;    // b2 (EPI_M_*) or bc1 (EPI_PHI, EPI_GC1)
  const float* wc2 = nullptr;
  const float* wr = nullptr;
  char* outb = nullptr;           // tiles written by the epilogue
  float* outf = nullptr;          // (E, 256) fp32 m (EPI_M_FWD)
  __half* outh = nullptr;         // (E, 256) fp16 silu'(a2 + b2) (EPI_M_BWD)
  __nv_bfloat16* gstore = nullptr;
  float* phi = nullptr;
  const float4* geo = nullptr;
  float4* gdstore = nullptr;
  const __half* aux = nullptr;    // (E, 256) fp16 silu'(a2 + b2) (EPI_GA2)
  const __half* s1 = nullptr;     // (E, 256) fp16 silu'(a1) (EPI_GA1)
  const float4* gtr = nullptr;    // (E) dL/dx'_i s_i, 1 / (|d| + eps) or 0 (EPI_GC1, EPI_GA1)
  const float* g_agg = nullptr;
  int64_t ld_gagg = 0;
  const int32_t* row_idx = nullptr;
  float* part = nullptr;
  int64_t PF = 0;
  int flags = 0;
};

constexpr int GM_NTH = 576;   // warp 0: loads; warp 1: MMA + TMEM; warps 2..17: epilogue
constexpr int kWBlk = kH * 128;   // 32 KB: one 64-deep K slice of a 256 x 256 bf16 weight
constexpr bool split_w(int epi) { return epi == EPI_M_FWD || epi == EPI_M_BWD || epi == EPI_GA1; }
// Resident weight: W (128 KB) | ring of 3 A blocks.  Split W2 products: no
// resident weight, a ring of 2 stages of [A block | W hi slice | W lo slice].
template <bool SPLIT>
struct GmLayout {
  static constexpr int S = SPLIT ? 2 : 3;                          // ring stages
  static constexpr int STAGE = SPLIT ? kBlk + 2 * kWBlk : kBlk;    // bytes per stage
  static constexpr int W = 0;
  static constexpr int A = SPLIT ? 0 : kH * kH * 2;
  static constexpr int BAR = A + S * STAGE;             // 180224 / 163840
  static constexpr int RED = BAR + 256;                 // float[2][4][128]
  static constexpr int VEC = RED + 2 * 4 * 128 * 4;     // float[3][256]: bias, w_c2, w_r
  static constexpr int STG = VEC + 3 * kH * 4;          // 16 epilogue warps x 2 KB store staging
  static constexpr size_t BYTES = STG + 16 * 2048 + 1024;
};

template <int EPI>
__global__ void __launch_bounds__(GM_NTH, 1) rows_gemm_kernel(RowsGemmArgs a) {
  constexpr bool BK = EPI <= EPI_GC1;   // B = W as [n][k] (x W^T), else W as [k][n] (g W)
  constexpr bool SPLIT = split_w(EPI);
  using L = GmLayout<SPLIT>;
  constexpr int GM_S = L::S;
  constexpr uint32_t IDESC = make_idesc_bf16(128, kH, 0, BK ? 0 : 1);
  constexpr int NV = EPI == EPI_GC1 ? 2 : (EPI == EPI_GA2 || EPI == EPI_GA1) ? 1 : 0;
  extern __shared__ __align__(1024) char rg_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(rg_raw) + 1023) & ~uintptr_t(1023));
  char* Wt = sm + L::W;
  char* Ast = sm + L::A;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* empty = full + GM_S;
  uint64_t* accf = empty + GM_S;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  uint32_t* tmem_s = reinterpret_cast<uint32_t*>(fin + 1);
  int* abort_s = reinterpret_cast<int*>(tmem_s + 1);
  float* red = reinterpret_cast<float*>(sm + L::RED);
  float* vbias = reinterpret_cast<float*>(sm + L::VEC);
  float* vwc2 = vbias + kH;
  float* vwr = vwc2 + kH;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t G = gridDim.x;
  const int64_t ntl = (int64_t)blockIdx.x < a.ntiles ? (a.ntiles - 1 - blockIdx.x) / G + 1 : 0;

  // prologue (parameters only, before the wait on the previous kernel)
  if constexpr (!SPLIT) load_w256(Wt, a.W);
  if (warp == 1) tmem_alloc(tmem_s, 512);
  if (tid == 0) {
    for (int s = 0; s < GM_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accf[0], 1);
    mbar_init(&accf[1], 1);
    mbar_init(&acce[0], 16);
    mbar_init(&acce[1], 16);
    mbar_init(fin, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_s;
  volatile int* abort_f = abort_s;
  pdl_enter();

  float acc0[2] = {0.f, 0.f}, acc1[2] = {0.f, 0.f};   // column sums (epilogue threads)
  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: A blocks of the CTA's tiles through the ring
      uint32_t it = 0;
      bool ok = true;
      for (int64_t j = 0; j < ntl && ok; ++j) {
        const char* src = a.A + (size_t)(blockIdx.x + j * G) * kTile;
        for (int b = 0; b < 4; ++b, ++it) {
          const int s = it % GM_S;
          if (it >= GM_S && !(ok = wait_bar(&empty[s], ((it / GM_S) - 1) & 1, abort_f, abort_s))) break;
          char* st = Ast + s * L::STAGE;
          mbar_expect_tx(&full[s], L::STAGE);
          bulk_g2s(st, src + b * kBlk, kBlk, &full[s]);
          if constexpr (SPLIT) {
            // K slice b of W hi and lo: rows 64 b .. + 63 of the [k][n] image
            // (4 column blocks of 8 KB) for g W, column block b of the [n][k]
            // image (32 KB) for x W^T
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const char* wsrc = a.Wimg + h * kH * kH * 2;
              char* wdst = st + kBlk + h * kWBlk;
              if constexpr (BK) {
                bulk_g2s(wdst, wsrc + b * kWBlk, kWBlk, &full[s]);
              } else {
#pragma unroll
                for (int cb = 0; cb < 4; ++cb)
                  bulk_g2s(wdst + cb * (kWBlk / 4), wsrc + cb * kWBlk + b * (kWBlk / 4), kWBlk / 4, &full[s]);
              }
            }
          }
        }
      }
      if (!ok)   // copies still in flight land before the CTA exits
        for (uint32_t k = it > GM_S ? it - GM_S : 0; k < it; ++k)
          wait_bar(&full[k % GM_S], (k / GM_S) & 1, nullptr, abort_s);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      const uint32_t wb = smem_u32(Wt), ab = smem_u32(Ast);
      uint32_t it = 0;
      bool ok = true;
      for (int64_t j = 0; j < ntl && ok; ++j) {
        const int buf = (int)(j & 1);
        if (j >= 2 && !(ok = wait_bar(&acce[buf], ((j >> 1) - 1) & 1, abort_f, abort_s))) break;
        fence_after_sync();
        const uint32_t d = tmem + buf * kH;
        for (int b = 0; b < 4; ++b, ++it) {
          const int s = it % GM_S;
          if (!(ok = wait_bar(&full[s], (it / GM_S) & 1, abort_f, abort_s))) break;
          fence_after_sync();
          const uint32_t sa = ab + s * L::STAGE;
          if constexpr (SPLIT) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t sw = sa + kBlk + h * kWBlk;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = make_desc(sa + kk * 32, 16, 1024);
                const uint64_t bd = BK ? make_desc(sw + kk * 32, 16, 1024)
                                       : make_desc(sw + kk * 2048, kWBlk / 4, 1024);
                mma_bf16(d, ad, bd, IDESC, (h | b | kk) ? 1u : 0u);
              }
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = make_desc(sa + kk * 32, 16, 1024);
              const uint64_t bd = BK ? make_desc(wb + b * (kH * 128) + kk * 32, 16, 1024)
                                     : make_desc(wb + (4 * b + kk) * 2048, kH * 128, 1024);
              mma_bf16(d, ad, bd, IDESC, (b | kk) ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&accf[buf]);
      }
      mma_commit(fin);   // every MMA of this thread has completed once fin flips
      wait_bar(fin, 0, nullptr, abort_s);
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread = (edge row el, 64-feature slice cs)
    const int q = warp & 3, cs = (warp - 2) >> 2, el = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    char* stg = sm + L::STG + (warp - 2) * 2048;
    const bool tanh_on = a.flags & EGNN_FLAG_TANH;
    // per-feature vectors (w_r comes from the prep kernel: read after the wait)
    for (int n = tid - 64; n < kH; n += 512) {
      vbias[n] = a.bias ? a.bias[n] : 0.f;
      vwc2[n] = a.wc2 ? a.wc2[n] : 0.f;
      vwr[n] = a.wr ? a.wr[n] : 0.f;
    }
    epi_sync();
    // variants with a named barrier inside the tile decide a timeout together;
    // the others per warp
    constexpr bool kJoint = EPI == EPI_PHI || EPI == EPI_GC1 || EPI == EPI_GA1;
    for (int64_t j = 0; j < ntl; ++j) {
      const int buf = (int)(j & 1);
      // g_a2 / g_a1: this thread's fp16 side row (silu'(a2) / silu'(a1), features
      // 64 cs .. + 63) is requested before the wait for the accumulator
      uint4 side[8];
      // g_c1 / g_a1: the edge's geometry and coordinate-gradient factors (and
      // phi for g_a1), likewise requested before the wait
      float4 pg = make_float4(0.f, 0.f, 0.f, 0.f), pt = pg;
      float pphi = 0.f;
      int prow = 0;   // g_a2: the edge's destination row of dL/dagg
      if constexpr (EPI == EPI_GA2) {
        const int64_t ep = (blockIdx.x + j * G) * 128 + el;
        if (ep < a.E) prow = a.row_idx[ep];
      }
      if constexpr (EPI == EPI_GC1 || EPI == EPI_GA1) {
        const int64_t ep = (blockIdx.x + j * G) * 128 + el;
        if (ep < a.E) {
          pg = a.geo[ep];
          pt = a.gtr[ep];
          if (EPI == EPI_GA1) pphi = a.phi[ep];
        }
      }
      if constexpr (EPI == EPI_GA2 || EPI == EPI_GA1)
        load_rows128(stg, EPI == EPI_GA2 ? a.aux : a.s1, (blockIdx.x + j * G) * 128 + q * 32, a.E, cs, side);
      const bool ok = wait_bar(&accf[buf], (j >> 1) & 1, abort_f, abort_s);
      if (kJoint ? epi_any(!ok) : !__all_sync(0xffffffffu, ok)) break;
      fence_after_sync();
      const int64_t t = blockIdx.x + j * G;
      const int64_t e = t * 128 + el;
      const bool valid = e < a.E;
      const uint32_t tacc = tmem + lane_base + buf * kH + cs * 64;
      char* tb = a.outb ? a.outb + t * kTile : nullptr;
      float* rbuf = red + (j & 1) * 512;
      auto release = [&]() {
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive1(&acce[buf]);
      };

      if constexpr (EPI == EPI_M_FWD || EPI == EPI_M_BWD) {
#pragma unroll 1
        for (int p = 0; p < 2; ++p) {
          float v[32];
          tmem_ld32(tacc + 32 * p, v);
          if (p == 1) release();
          const int n0 = cs * 64 + 32 * p;
#pragma unroll
          for (int t4 = 0; t4 < 32; t4 += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(vbias + n0 + t4);
            v[t4] += b4.x; v[t4 + 1] += b4.y; v[t4 + 2] += b4.z; v[t4 + 3] += b4.w;
          }
          if constexpr (EPI == EPI_M_BWD) {
            float d2[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              float yy, dy;
              silu_grad_edge(v[k], yy, dy);
              v[k] = valid ? yy : 0.f;
              d2[k] = dy;
            }
            st_f16_piece(stg, valid ? a.outh + e * kH + n0 : nullptr, d2);
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = valid ? silu_edge(v[k]) : 0.f;
            st_f32_piece(stg, valid ? a.outf + e * kH + n0 : nullptr, v);
          }
          st_tile_piece(stg, tb, el, cs, p, v);
        }
      } else if constexpr (EPI == EPI_PHI) {
        float part = 0.f;
#pragma unroll 1
        for (int p = 0; p < 2; ++p) {
          float v[32];
          tmem_ld32(tacc + 32 * p, v);
          if (p == 1) release();
          const int n0 = cs * 64 + 32 * p;
#pragma unroll
          for (int t4 = 0; t4 < 32; t4 += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(vbias + n0 + t4),
                         w4 = *reinterpret_cast<const float4*>(vwc2 + n0 + t4);
            part += w4.x * silu_edge(v[t4] + b4.x);
            part += w4.y * silu_edge(v[t4 + 1] + b4.y);
            part += w4.z * silu_edge(v[t4 + 2] + b4.z);
            part += w4.w * silu_edge(v[t4 + 3] + b4.w);
          }
        }
        rbuf[cs * 128 + el] = part;
        epi_sync();
        if (cs == 0 && valid) {
          float f = rbuf[el] + rbuf[128 + el] + rbuf[256 + el] + rbuf[384 + el];
          if (tanh_on) f = tanhf(f);
          a.phi[e] = f;
        }
      } else if constexpr (EPI == EPI_GC1) {
        // gphi_e = (g_t . d) inv, times (1 - phi^2) with tanh: only then does
        // it wait for phi (the row sum over the four slices)
        const float gbase = valid ? (pt.x * pg.x + pt.y * pg.y + pt.z * pg.z) * pt.w : 0.f;
        // g_c1 = gphi wc2 silu'(c1) -> Gc1; column sums of g_c1 and gphi silu(c1)
        auto grad_pass = [&](float gphi, float& part) {
#pragma unroll 1
          for (int p = 0; p < 2; ++p) {
            float v[32], y[32];
            tmem_ld32(tacc + 32 * p, v);
            if (p == 1) release();
            const int n0 = cs * 64 + 32 * p;
#pragma unroll
            for (int t4 = 0; t4 < 32; t4 += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(vbias + n0 + t4),
                           w4 = *reinterpret_cast<const float4*>(vwc2 + n0 + t4);
              const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                float yy, dy;
                silu_grad_edge(v[t4 + u] + bb[u], yy, dy);
                part += ww[u] * yy;
                v[t4 + u] = gphi * ww[u] * dy;
                y[t4 + u] = gphi * yy;
              }
            }
            st_tile_piece(stg, tb, el, cs, p, v);
            acc0[p] += colsum32(v);
            acc1[p] += colsum32(y);
          }
        };
        float part = 0.f;
        if (!tanh_on) {
          grad_pass(gbase, part);   // one pass: phi's partial sum rides along
          rbuf[cs * 128 + el] = part;
          epi_sync();
          if (cs == 0 && valid) a.phi[e] = rbuf[el] + rbuf[128 + el] + rbuf[256 + el] + rbuf[384 + el];
        } else {
#pragma unroll 1
          for (int p = 0; p < 2; ++p) {
            float v[32];
            tmem_ld32(tacc + 32 * p, v);
            const int n0 = cs * 64 + 32 * p;
#pragma unroll
            for (int t4 = 0; t4 < 32; t4 += 4) {
              const float4 b4 = *reinterpret_cast<const float4*>(vbias + n0 + t4),
                           w4 = *reinterpret_cast<const float4*>(vwc2 + n0 + t4);
              part += w4.x * silu_edge(v[t4] + b4.x);
              part += w4.y * silu_edge(v[t4 + 1] + b4.y);
              part += w4.z * silu_edge(v[t4 + 2] + b4.z);
              part += w4.w * silu_edge(v[t4 + 3] + b4.w);
            }
          }
          rbuf[cs * 128 + el] = part;
          epi_sync();
          const float f = tanhf(rbuf[el] + rbuf[128 + el] + rbuf[256 + el] + rbuf[384 + el]);
          if (cs == 0 && valid) a.phi[e] = f;
          float unused = 0.f;
          grad_pass(gbase * (1.f - f * f), unused);
        }
      } else if constexpr (EPI == EPI_GA2) {
        const int i = prow;
#pragma unroll 1
        for (int p = 0; p < 2; ++p) {
          float v[32];
          tmem_ld32(tacc + 32 * p, v);
          if (p == 1) release();
          const int n0 = cs * 64 + 32 * p;
          const float* ga = a.g_agg + (int64_t)i * a.ld_gagg + n0;
#pragma unroll
          for (int t8 = 0; t8 < 32; t8 += 8) {
            const float4 g0 = ldg4(ga + t8), g1 = ldg4(ga + t8 + 4);
            const uint4 hz = p ? side[4 + t8 / 8] : side[t8 / 8];
            const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const uint32_t hw[4] = {hz.x, hz.y, hz.z, hz.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hw[u]));
              v[t8 + 2 * u] = valid ? (v[t8 + 2 * u] + gg[2 * u]) * dd.x : 0.f;
              v[t8 + 2 * u + 1] = valid ? (v[t8 + 2 * u + 1] + gg[2 * u + 1]) * dd.y : 0.f;
            }
          }
          st_tile_piece(stg, tb, el, cs, p, v);
          acc0[p] += colsum32(v);
        }
      } else {   // EPI_GA1
        const float4 gq = pg;
        float grp = 0.f;
#pragma unroll 1
        for (int p = 0; p < 2; ++p) {
          float v[32], rr[32];
          tmem_ld32(tacc + 32 * p, v);
          if (p == 1) release();
          const int n0 = cs * 64 + 32 * p;
#pragma unroll
          for (int t8 = 0; t8 < 32; t8 += 8) {
            const uint4 hz = p ? side[4 + t8 / 8] : side[t8 / 8];
            const uint32_t hw[4] = {hz.x, hz.y, hz.z, hz.w};
            const float4 wa = *reinterpret_cast<const float4*>(vwr + n0 + t8),
                         wb = *reinterpret_cast<const float4*>(vwr + n0 + t8 + 4);
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hw[u]));
              const float g0 = valid ? v[t8 + 2 * u] * dd.x : 0.f;
              const float g1 = valid ? v[t8 + 2 * u + 1] * dd.y : 0.f;
              v[t8 + 2 * u] = g0;
              v[t8 + 2 * u + 1] = g1;
              grp += g0 * wv[2 * u] + g1 * wv[2 * u + 1];
              rr[t8 + 2 * u] = g0 * gq.w;
              rr[t8 + 2 * u + 1] = g1 * gq.w;
            }
          }
          st_bf16_piece(stg, valid ? a.gstore + e * kH + n0 : nullptr, v);
          acc0[p] += colsum32(rr);
        }
        rbuf[cs * 128 + el] = grp;
        epi_sync();
        if (cs == 0 && valid) {
          const float gr = rbuf[el] + rbuf[128 + el] + rbuf[256 + el] + rbuf[384 + el];
          const float coef = pphi * pt.w;   // pt.w is 0 on a self-loop: no coordinate gradient
          a.gdstore[e] = make_float4(pt.x * coef + 2.f * gr * gq.x, pt.y * coef + 2.f * gr * gq.y,
                                     pt.z * coef + 2.f * gr * gq.z, 0.f);
        }
      }
    }
  }
  __syncthreads();

  // ---- per-CTA column sums -> partial slots (the A ring is idle now)
  if constexpr (NV > 0) {
    float* cs_s = reinterpret_cast<float*>(Ast);   // [4 q][NV][256]
    if (warp >= 2) {
      const int q = warp & 3, cs = (warp - 2) >> 2;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int n = cs * 64 + 32 * p + lane;
        cs_s[(q * NV + 0) * kH + n] = acc0[p];
        if (NV == 2) cs_s[(q * NV + 1) * kH + n] = acc1[p];
      }
    }
    __syncthreads();
    const int64_t HH = (int64_t)kH * kH;
    for (int idx = tid; idx < NV * kH; idx += GM_NTH) {
      const int vv = idx / kH, n = idx % kH;
      const float s = cs_s[(0 * NV + vv) * kH + n] + cs_s[(1 * NV + vv) * kH + n] + cs_s[(2 * NV + vv) * kH + n] +
                      cs_s[(3 * NV + vv) * kH + n];
      int64_t slot;
      if (EPI == EPI_GC1) slot = vv == 0 ? 2 * HH : 2 * HH + 2 * kH;   // gbc1, gwc2
      else if (EPI == EPI_GA2) slot = 2 * HH + kH;                     // gb2
      else slot = 2 * HH + 3 * kH;                                      // gwr
      a.part[(int64_t)blockIdx.x * a.PF + slot + n] = s;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---- weight gradients: D = G^T X over the edges (split-K, one slice per CTA) ----------
// Each CTA takes a contiguous range of tiles in 32-edge slabs (a quarter
// tile: the 4 KB row range of each of the four column blocks of both
// operands, 32 KB per stage); one thread streams them through a 6-stage ring
// with five slabs in flight ahead of the MMAs, and issues the MMAs (A = G^T
// and B = X both MN-major, two M = 128 halves of the 256 output rows in
// 2 x 256 TMEM columns).
constexpr int WG_NTH = 256, WG_S = 6, WG_STAGE = 32768, WG_SLAB = 32 * 128;
constexpr size_t WG_BYTES = WG_S * WG_STAGE + 256 + 1024;

__global__ void __launch_bounds__(WG_NTH, 1) rows_wgrad_kernel(const char* __restrict__ Gt, const char* __restrict__ Xt,
                                                               int64_t ntiles, float* __restrict__ part, int64_t PF,
                                                               int64_t off) {
  constexpr uint32_t IDESC = make_idesc_bf16(128, kH, 1, 1);
  extern __shared__ __align__(1024) char wg_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(wg_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + WG_S * WG_STAGE);
  uint64_t* empty = full + WG_S;
  uint64_t* done = empty + WG_S;
  uint32_t* tmem_s = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_s = reinterpret_cast<int*>(tmem_s + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tpc = (ntiles + gridDim.x - 1) / gridDim.x;
  const int64_t t0 = std::min<int64_t>(ntiles, (int64_t)blockIdx.x * tpc);
  const int64_t t1 = std::min<int64_t>(ntiles, t0 + tpc);
  const int nslab = (int)(4 * (t1 - t0));

  if (warp == 0) tmem_alloc(tmem_s, 512);
  if (tid == 0) {
    for (int s = 0; s < WG_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_s;
  volatile int* abort_f = abort_s;
  pdl_enter();

  if (warp == 0) {
    if (lane == 0) {
      int filled = 0, used = 0;
      bool ok = true;
      for (int it = 0; it < nslab + WG_S - 1 && ok; ++it) {
        if (it < nslab) {
          const int s = it % WG_S;
          if (it >= WG_S && !(ok = wait_bar(&empty[s], ((it / WG_S) - 1) & 1, abort_f, abort_s))) break;
          char* st = sm + s * WG_STAGE;
          mbar_expect_tx(&full[s], WG_STAGE);
          const size_t src = (size_t)(t0 + (it >> 2)) * kTile + (size_t)(it & 3) * WG_SLAB;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            bulk_g2s(st + b * WG_SLAB, Gt + src + b * kBlk, WG_SLAB, &full[s]);
            bulk_g2s(st + WG_STAGE / 2 + b * WG_SLAB, Xt + src + b * kBlk, WG_SLAB, &full[s]);
          }
          filled = it + 1;
        }
        const int k = it - (WG_S - 1);
        if (k >= 0) {
          const int s = k % WG_S;
          if (!(ok = wait_bar(&full[s], (k / WG_S) & 1, abort_f, abort_s))) break;
          used = k + 1;
          fence_after_sync();
          const uint32_t gb = smem_u32(sm + s * WG_STAGE), xb = gb + WG_STAGE / 2;
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
#pragma unroll
            for (int mh = 0; mh < 2; ++mh)
              mma_bf16(tmem + mh * kH, make_desc(gb + mh * 2 * WG_SLAB + kk * 2048, WG_SLAB, 1024),
                       make_desc(xb + kk * 2048, WG_SLAB, 1024), IDESC, (k | kk) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
      }
      if (!ok)
        for (int k = used; k < filled; ++k) wait_bar(&full[k % WG_S], (k / WG_S) & 1, nullptr, abort_s);
      mma_commit(done);
    }
    __syncwarp();
  }
  wait_bar(done, 0, nullptr, abort_s);
  fence_after_sync();
  {
    const int q = warp & 3, mh = warp >> 2;
    const int m = mh * 128 + q * 32 + lane;
    float* dst = part + (int64_t)blockIdx.x * PF + off + (int64_t)m * kH;
    char* stg = sm + warp * 2048;   // the operand ring is idle once `done` has flipped
#pragma unroll 1
    for (int c = 0; c < kH / 32; ++c) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + mh * kH + 32 * c, v);
      if (nslab == 0) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = 0.f;
      }
      st_f32_piece(stg, dst + 32 * c, v);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int EPI>
int launch_gemm(const RowsGemmArgs& a, int G, cudaStream_t s, const char* name) {
  constexpr size_t bytes = GmLayout<split_w(EPI)>::BYTES;
  if (split_w(EPI) && !a.Wimg) return fail(EGNN_ERR_INVALID_ARG, "edge-row W2 product without its weight image");
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(
        cudaFuncSetAttribute(rows_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    attr_set |= bit;
  }
  {
    TimerScope ts(name, s);
    EGNN_CHECK_CUDA(launch_pdl(rows_gemm_kernel<EPI>, dim3(G), dim3(GM_NTH), bytes, s, a));
  }
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

// gx_out: the backward's dL/dx' (the gather then also writes S1 and gtr).
int launch_u(const EdgeCommon& a, const RowsBufs& b, const float* gx_out, cudaStream_t s) {
  const int64_t Epad = rows_tiles(a.E) * 128;
  if (Epad == 0) return EGNN_OK;
  TimerScope ts("edge_rows_u", s);
  // grid-stride: the 256-thread blocks that fit an SM by registers (about 60 per
  // thread in the forward variant, 128 in the backward one)
  const int64_t blocks = std::min<int64_t>(Epad / (8 * EPW), (gx_out ? 2 : 4) * (int64_t)num_sms_current());
  EGNN_CHECK_CUDA(launch_pdl(gx_out ? rows_u_kernel<true> : rows_u_kernel<false>, dim3((unsigned)blocks),
                             dim3(256), 0, s, a.E, Epad, a.row_idx, a.col_idx, a.xp, a.PQ, a.wr, b.U, b.geo, b.S1,
                             a.row_ptr, gx_out, a.flags, b.gtr));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

RowsGemmArgs gemm_common(const EdgeCommon& a, const RowsBufs& b) {
  RowsGemmArgs g;
  g.E = a.E;
  g.ntiles = rows_tiles(a.E);
  g.wc2 = a.wc2;
  g.wr = a.wr;
  g.geo = b.geo;
  g.gtr = b.gtr;
  g.phi = b.phi;
  g.row_idx = a.row_idx;
  g.part = b.part;
  g.PF = edge_part_floats(kH, 0);
  g.flags = a.flags;
  return g;
}

}  // namespace

bool edge_rows_supported(int H, int d, int flags, int precision) {
  return precision == EGNN_PREC_BF16 && H == kH && d == 0 && !(flags & EGNN_FLAG_ATTENTION);
}

int64_t rows_tiles(int64_t E) { return (E + 127) / 128; }

int rows_grid(int64_t E, int num_sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(num_sms, rows_tiles(E)));
}

RowsBufs carve_rows(Carver& c, int64_t E, int H, bool bwd, int num_sms) {
  RowsBufs b;
  b.W2img = c.take<char>((size_t)2 * kH * kH * 2);
  const size_t tiles = (size_t)std::max<int64_t>(rows_tiles(E), 1) * kTile;
  const size_t En = (size_t)std::max<int64_t>(E, 1);
  b.U = c.take<char>(tiles);
  b.Mb = c.take<char>(tiles);
  if (bwd) {
    b.Gc1 = c.take<char>(tiles);
    b.Ga2 = c.take<char>(tiles);
    b.D2 = c.take<__half>(En * H);
    b.S1 = c.take<__half>(En * H);
    b.gtr = c.take<float4>(En);
  } else {
    b.M32 = c.take<float>(En * H);
  }
  b.phi = c.take<float>(En);
  b.geo = c.take<float4>(En);
  b.G = rows_grid(E, num_sms);
  if (bwd) b.part = c.take<float>((size_t)b.G * edge_part_floats(H, 0));
  return b;
}

// bf16 hi / lo images of W2 for the split products.
int launch_wimg(const float* W2, char* img, cudaStream_t s) {
  TimerScope ts("edge_rows_wimg", s);
  EGNN_CHECK_CUDA(launch_pdl(rows_wimg_kernel, dim3(32), dim3(256), 0, s, W2, img));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

int edge_fwd_rows(const EdgeFwdArgs& a, const RowsBufs& b, cudaStream_t s) {
  if (a.E > 0) {
    EGNN_TRY(launch_wimg(a.W2_src, b.W2img, s));
    EGNN_TRY(launch_u(a, b, nullptr, s));
    RowsGemmArgs g = gemm_common(a, b);
    g.A = b.U;
    g.W = a.W2_src;
    g.Wimg = b.W2img;
    g.bias = a.b2;
    g.outb = b.Mb;
    g.outf = b.M32;
    EGNN_TRY(launch_gemm<EPI_M_FWD>(g, b.G, s, "edge_rows_gemm"));
    g.A = b.Mb;
    g.W = a.Wc1_src;
    g.bias = a.bc1;
    g.outb = nullptr;
    g.outf = nullptr;
    EGNN_TRY(launch_gemm<EPI_PHI>(g, b.G, s, "edge_rows_gemm"));
  }
  if (a.N > 0) {
    TimerScope ts("edge_rows_agg", s);
    EGNN_CHECK_CUDA(launch_pdl(rows_agg_kernel, dim3((unsigned)((2 * a.N + 7) / 8)), dim3(256), 0, s, a.N, a.row_ptr,
                               b.M32, b.phi, b.geo, a.x, a.flags, a.agg, a.x_out));
    EGNN_CHECK_LAUNCH();
  }
  return EGNN_OK;
}

int edge_bwd_rows(const EdgeBwdArgs& a, const RowsBufs& b, cudaStream_t s) {
  RowsGemmArgs g = gemm_common(a, b);
  g.Wimg = b.W2img;
  EGNN_TRY(launch_wimg(a.W2_src, b.W2img, s));
  if (a.E > 0) {
    EGNN_TRY(launch_u(a, b, a.gx_out, s));
    g.A = b.U;
    g.W = a.W2_src;
    g.bias = a.b2;
    g.outb = b.Mb;
    g.outh = b.D2;
    EGNN_TRY(launch_gemm<EPI_M_BWD>(g, b.G, s, "edge_rows_gemm"));
  }
  // the three gradient GEMMs also run without edges: they write the zero
  // column-sum slots of the partials
  g.A = b.Mb;
  g.W = a.Wc1_src;
  g.bias = a.bc1;
  g.outb = b.Gc1;
  g.outf = nullptr;
  EGNN_TRY(launch_gemm<EPI_GC1>(g, b.G, s, "edge_rows_gemm"));
  g.A = b.Gc1;
  g.bias = nullptr;
  g.outb = b.Ga2;
  g.aux = b.D2;
  g.g_agg = a.g_agg;
  g.ld_gagg = a.ld_gagg ? a.ld_gagg : kH;
  EGNN_TRY(launch_gemm<EPI_GA2>(g, b.G, s, "edge_rows_gemm"));
  g.A = b.Ga2;
  g.W = a.W2_src;
  g.outb = nullptr;
  g.s1 = b.S1;
  g.gstore = reinterpret_cast<__nv_bfloat16*>(a.gstore);
  g.gdstore = a.gdstore;
  EGNN_TRY(launch_gemm<EPI_GA1>(g, b.G, s, "edge_rows_gemm"));
  return EGNN_OK;
}

int edge_wgrad_rows(int64_t E, const RowsBufs& b, cudaStream_t s) {
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(
        cudaFuncSetAttribute(rows_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WG_BYTES));
    attr_set |= bit;
  }
  const int64_t T = rows_tiles(E), PF = edge_part_floats(kH, 0), HH = (int64_t)kH * kH;
  TimerScope ts("edge_rows_wgrad", s);
  EGNN_CHECK_CUDA(launch_pdl(rows_wgrad_kernel, dim3(b.G), dim3(WG_NTH), WG_BYTES, s, (const char*)b.Gc1,
                             (const char*)b.Mb, T, b.part, PF, (int64_t)0));
  EGNN_CHECK_LAUNCH();
  EGNN_CHECK_CUDA(launch_pdl(rows_wgrad_kernel, dim3(b.G), dim3(WG_NTH), WG_BYTES, s, (const char*)b.Ga2,
                             (const char*)b.U, T, b.part, PF, HH));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

int rows_take_timeouts() {
  int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_rows_timeouts, sizeof(int)) != cudaSuccess) return 0;
  if (n) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_rows_timeouts, &zero, sizeof(int));
  }
  return n;
}

}  // namespace egnn
