// Fused EGNN edge kernels (SIMT FFMA path): argument blocks and launchers.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace egnn {

// A warp reads / writes one H-float row with lane owning the H / 32
// consecutive features lane * (H / 32) .. (rows are H-float aligned).
template <int H>
__device__ __forceinline__ void load_row_slice(const float* row, int lane, float (&v)[H / 32]) {
  constexpr int VW = H / 32;
  const float* p = row + lane * VW;
  if constexpr (VW % 4 == 0) {
#pragma unroll
    for (int w = 0; w < VW; w += 4) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p + w));
      v[w] = a.x; v[w + 1] = a.y; v[w + 2] = a.z; v[w + 3] = a.w;
    }
  } else if constexpr (VW == 2) {
    const float2 a = __ldg(reinterpret_cast<const float2*>(p));
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = __ldg(p);
  }
}
// The same slice of a bf16 row (the tensor-core backward stores dL/da1 in bf16).
template <int H>
__device__ __forceinline__ void load_row_slice(const __nv_bfloat16* row, int lane, float (&v)[H / 32]) {
  constexpr int VW = H / 32;
  const __nv_bfloat16* p = row + lane * VW;
  if constexpr (VW % 8 == 0) {
#pragma unroll
    for (int w = 0; w < VW; w += 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p + w));
      const uint32_t x[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x[t]));
        v[w + 2 * t] = f.x; v[w + 2 * t + 1] = f.y;
      }
    }
  } else if constexpr (VW == 4) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  } else if constexpr (VW == 2) {
    const unsigned int u = __ldg(reinterpret_cast<const unsigned int*>(p));
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
    v[0] = f.x; v[1] = f.y;
  } else {
    v[0] = __bfloat162float(p[0]);
  }
}

template <int H>
__device__ __forceinline__ void store_row_slice(float* row, int lane, const float (&v)[H / 32]) {
  constexpr int VW = H / 32;
  float* p = row + lane * VW;
  if constexpr (VW % 4 == 0) {
#pragma unroll
    for (int w = 0; w < VW; w += 4) *reinterpret_cast<float4*>(p + w) = make_float4(v[w], v[w + 1], v[w + 2], v[w + 3]);
  } else if constexpr (VW == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
    p[0] = v[0];
  }
}

// Fields shared by the forward and backward edge kernels.
struct EdgeCommon {
  int64_t N = 0, E = 0;
  const int32_t* row_ptr = nullptr;
  const int32_t* col_idx = nullptr;
  const int32_t* row_idx = nullptr;
  const int32_t* edge_id = nullptr;
  const float4* xp = nullptr;    // (N) coordinates padded to 16 bytes
  const float* PQ = nullptr;     // (N, 2H): P = h Wa^T + b1 | Q = h Wb^T
  const float* wr = nullptr;     // (H) radial column of edge_mlp.0
  const float* We = nullptr;     // (H, d) edge_attr columns of edge_mlp.0
  const float* attr = nullptr;   // (E, d) edge attributes by original edge id
  int d = 0;
  const float* W2T = nullptr;    // (H,H) [k][o] = edge_mlp.2.weight[o][k]
  const float* b2 = nullptr;
  const float* Wc1T = nullptr;   // (H,H) [k][o] = coord_mlp.0.weight[o][k]
  const float* bc1 = nullptr;
  const float* wc2 = nullptr;    // (H) coord_mlp.2.weight
  const float* W2_src = nullptr; // (H,H) edge_mlp.2.weight as given (fp32, [out][in])
  const float* Wc1_src = nullptr;// (H,H) coord_mlp.0.weight as given
  const float* wa = nullptr;     // (H) att_mlp.0.weight (attention only)
  const float* ba = nullptr;     // (1) att_mlp.0.bias (attention only)
  int flags = 0;
  int64_t epc = 0;               // edges per CTA (multiple of the chunk size)
  float* carry = nullptr;        // (G, 2, H+4) partial rows at CTA range edges
  int32_t* carry_row = nullptr;  // (G, 2)
  // Tensor-core kernels: poll limit of the MMA-completion waits (-1: the
  // built-in limit).  Only a debugging aid sets it (EGNN_DEBUG_WAIT_POLLS),
  // to make the give-up path run; the drain wait that precedes freeing the
  // tensor memory always keeps the built-in limit.
  int wait_polls = -1;
  // Tensor-core kernels: 1-D tensor maps of row_idx and col_idx (int32, box of
  // 128), for the TMA loads of each chunk's index tiles; use_tma = 0 when the
  // arrays are not 16-byte aligned (the kernels then load them per thread).
  CUtensorMap tm_row;
  CUtensorMap tm_col;
  int use_tma = 0;
};

struct EdgeFwdArgs : EdgeCommon {
  const float* x = nullptr;      // (N,3)
  float* agg = nullptr;          // (N,H) out: sum of messages per row
  float* x_out = nullptr;        // (N,3) out
};

struct EdgeBwdArgs : EdgeCommon {
  const float* W2 = nullptr;     // (H,H) edge_mlp.2.weight (bf16-rounded in bf16 mode)
  const float* Wc1 = nullptr;    // (H,H) coord_mlp.0.weight (idem)
  const float* gx_out = nullptr; // (N,3) dL/dx'
  const float* g_agg = nullptr;  // (N, ld_gagg) dL/dagg from the node MLP backward
  int64_t ld_gagg = 0;           // row stride of g_agg (H when 0)
  float* S_dst = nullptr;        // (N,H) out: sum over each row of dL/da1
  float* gxd = nullptr;          // (N,3) out: sum over each row of dL/d(x_i - x_j)
  float* gstore = nullptr;       // (E,H) out: dL/da1 per CSR edge (bf16 rows on the tensor-core path)
  float4* gdstore = nullptr;     // (E) out: dL/d(x_i - x_j) per CSR edge
  float* part = nullptr;         // (G, part_floats(H,d)) per-CTA weight-gradient partials
  float* att_scr = nullptr;      // (G, edge_att_scratch_floats(H)) attention only: each CTA's
                                 // ungated messages of the current chunk and its gate-gradient sums
};

// Per-CTA partial layout (floats): gWc1 (H*H) | gW2 (H*H) | gbc1 | gb2 | gwc2 | gwr (H each)
// | gWe (H*d) | gwa (H) | gba (1); the last two only carry values with attention.
__host__ __device__ inline int64_t edge_part_att(int H, int d) { return 2LL * H * H + 4LL * H + (int64_t)H * d; }
__host__ __device__ inline int64_t edge_part_floats(int H, int d) {
  int64_t n = edge_part_att(H, d) + H + 1;
  return (n + 63) / 64 * 64;
}

// Per-CTA attention scratch of the SIMT backward (floats): the chunk's
// ungated messages (T x H) | gwa partial sums (TY x H) | gba partial sums (TY).
int64_t edge_att_scratch_floats(int H);

// Launch geometry for a given E: CTA count and edges per CTA.
struct EdgeGrid { int G; int64_t epc; };
int edge_grid(int H, bool bwd, bool bf16, int64_t E, int num_sms, EdgeGrid* out);
int edge_chunk(int H);

int edge_fwd(int H, bool bf16, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s);

// Boundary fix-up of the forward: rows cut by a CTA range boundary.
int edge_fixup_fwd(int H, const EdgeFwdArgs& a, const EdgeGrid& g, cudaStream_t s);
int edge_bwd(int H, bool bf16, const EdgeBwdArgs& a, const EdgeGrid& g, cudaStream_t s);

// Source-side pass of the backward: S_src[j] = sum of gstore over the
// out-edges of j (transpose CSR order), gx[j] = gx_out[j] + gxd[j] - sum gd.
// gstore holds fp32 rows, or bf16 rows when `bf16_rows` (tensor-core path).
int edge_src_pass(int H, int64_t N, const int32_t* src_ptr, const int32_t* src_edge,
                  const void* gstore, bool bf16_rows, const float4* gdstore, const float* gx_out,
                  const float* gxd, float* S_src, float* gx, cudaStream_t s);

// Reduce the G per-CTA partials in CTA order and scatter them into the
// parameter-gradient outputs.  edge_mlp.0.weight has row stride ld_w1; its
// radial column is c_r (= 2 input_nf), the edge-attribute columns follow.
int edge_part_reduce(int H, int d, bool att, int G, const float* part, const egnn_layer_grads* gp,
                     int64_t ld_w1, int64_t c_r, cudaStream_t s);

}  // namespace egnn
