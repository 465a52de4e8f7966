// Device graph builders: the step before the layer.
//
//  * egnn_fc_graph: fully connected intra-graph edges of a batch, in the order
//    of the reference's get_edges / get_edges_batch (egnn_clean.py:167-191),
//    written straight into a destination-sorted CSR (no sort needed).
//  * egnn_spatial_count / egnn_spatial_fill: radius graphs (optionally capped
//    at the nearest max_nbrs) and k-nearest-neighbour graphs over points,
//    split into graphs by graph_ptr, on a hashed uniform grid.
//  * egnn_morton_order: Morton codes and the stable order they induce.
//
// Exactness: distances are d2 = (dx*dx + dy*dy) + dz*dz in fp32 with every
// operation rounded (no contraction into FMA), ties broken by the smaller
// index, so the result is a pure function of the fp32 coordinates and a CPU
// restatement reproduces it bit for bit.  The k-nearest search grows its cube
// of cells until the k-th distance is provably inside it, and falls back to a
// scan of the whole graph.
//
// Work split: one warp per destination node.  A warp lists the candidate
// points of its cube of cells (lanes take one cell each, a warp prefix sum
// lays their bucket ranges end to end, lanes then stride over the candidates)
// and keeps the smallest keys in a shared-memory buffer that it sorts with a
// bitonic network when it fills up.
#include <algorithm>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace egnn {
namespace {

constexpr int kWarps = 8;           // warps per block of the query kernels
constexpr int kCap = 512;           // keys a warp buffers in shared memory
constexpr int kKeep = kCap / 2;     // keys a warp emits per pass
constexpr int kMaxK = kKeep;        // largest k of the nearest-neighbour mode

unsigned grid_for(int64_t n, int threads = 256) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 65535));
}

int pow2_at_least(int64_t v) {
  int b = 0;
  while ((1LL << b) < v) ++b;
  return b;
}

// Grid geometry shared by the count and fill phases (kept in the workspace).
struct GridParams {
  float s;            // cell edge
  float c2;           // cutoff^2 (fp32), radius modes
  uint32_t mask;      // bucket count - 1
  int pad;
};

struct SpatialArgs {
  int64_t N, G;
  const float* x;
  const int64_t* gp;  // (G+1) or null (one graph)
  int mode, k;        // k: max_nbrs (0 = uncapped radius) or the neighbour count
  const GridParams* prm;
  const int32_t* bstart;   // (mask+2) bucket ranges over the sorted points
  const float4* pts;       // sorted points: x, y, z, index bits
  const int4* cells;       // sorted points' cells: cx, cy, cz, graph
  int* err;
};

__device__ __forceinline__ float sqdist(float4 a, float4 b) {
  const float dx = __fsub_rn(a.x, b.x), dy = __fsub_rn(a.y, b.y), dz = __fsub_rn(a.z, b.z);
  return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

__device__ __forceinline__ int cell_of(float v, float s) {
  float q = floorf(__fdiv_rn(v, s));
  q = fminf(fmaxf(q, -1073741824.f), 1073741823.f);   // NaN -> lower clamp
  return (int)q;
}

__device__ __forceinline__ uint32_t cell_hash(int g, int cx, int cy, int cz, uint32_t mask) {
  uint32_t h = ((uint32_t)cx * 73856093u) ^ ((uint32_t)cy * 19349663u) ^ ((uint32_t)cz * 83492791u) ^
               ((uint32_t)g * 2654435761u);
  h ^= h >> 16;
  h *= 0x7feb352du;
  h ^= h >> 15;
  return h & mask;
}

// Graph of node i: the g with gp[g] <= i < gp[g+1] (0 without graph_ptr).
__device__ __forceinline__ int graph_of(const int64_t* gp, int64_t G, int64_t i) {
  if (!gp) return 0;
  int64_t lo = 0, hi = G - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (gp[mid] <= i) lo = mid; else hi = mid - 1;
  }
  return (int)lo;
}

__global__ void check_graph_ptr_kernel(int64_t N, int64_t G, const int64_t* gp, int* err) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g <= G; g += (int64_t)gridDim.x * blockDim.x) {
    if (g == 0 && gp[0] != 0) atomicOr(err, 1);
    if (g == G && gp[G] != N) atomicOr(err, 1);
    if (g < G && gp[g + 1] < gp[g]) atomicOr(err, 1);
  }
}

// ---- fully connected batches ----------------------------------------------------
__global__ void fc_counts_kernel(int64_t G, const int64_t* gp, int64_t* cnt) {
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g <= G; g += (int64_t)gridDim.x * blockDim.x) {
    if (g == G) { cnt[g] = 0; continue; }
    const int64_t n = gp[g + 1] - gp[g];
    cnt[g] = n > 1 ? n * (n - 1) : 0;
  }
}

// One warp per row i of graph g = [a, b): columns a..b-1 without i.
__global__ void fc_fill_kernel(int64_t N, int64_t G, const int64_t* gp, const int64_t* off, int64_t E,
                               int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; i < N; i += warps) {
    const int g = graph_of(gp, G, i);
    const int64_t a = gp[g], b = gp[g + 1];
    const int64_t deg = (b - a > 1) ? b - a - 1 : 0;
    const int64_t start = off[g] + (i - a) * deg;
    if (lane == 0) {
      row_ptr[i] = (int32_t)start;
      if (i == N - 1) {
        row_ptr[N] = (int32_t)off[G];
        if (off[G] != E) atomicOr(err, 2);
      }
    }
    for (int64_t t = lane; t < deg; t += 32) {
      const int64_t pos = start + t;
      if (pos >= E) { atomicOr(err, 2); break; }
      const int64_t j = a + t + (t >= i - a ? 1 : 0);
      col_idx[pos] = (int32_t)j;
      row_idx[pos] = (int32_t)i;
    }
  }
}

// ---- grid construction --------------------------------------------------------------
// Order-preserving uint encoding of floats for atomic min / max.
__device__ __forceinline__ uint32_t ord_enc(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_dec(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__global__ void bbox_kernel(int64_t N, const float* x, uint32_t* box) {
  float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x)
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const float v = x[i * 3 + a];
      if (v == v) { lo[a] = fminf(lo[a], v); hi[a] = fmaxf(hi[a], v); }
    }
#pragma unroll
  for (int a = 0; a < 3; ++a) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
      hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
    }
    if ((threadIdx.x & 31) == 0) {
      atomicMin(box + a, ord_enc(lo[a]));
      atomicMax(box + 3 + a, ord_enc(hi[a]));
    }
  }
}

// Cell edge: the cutoff (slightly enlarged) for radius graphs; for the
// nearest-neighbour mode the caller's hint, or an edge whose ball holds
// about 2 (k + 1) points of an average graph in the bounding box.
__global__ void params_kernel(int64_t N, int64_t G, int mode, int k, float cutoff, uint32_t mask,
                              const uint32_t* box, GridParams* p) {
  GridParams q;
  q.mask = mask;
  q.pad = 0;
  q.c2 = __fmul_rn(cutoff, cutoff);
  if (mode == EGNN_GRAPH_RADIUS) {
    q.s = cutoff * (1.f + 1.f / 4096.f);
  } else if (cutoff > 0.f) {
    q.s = cutoff;
  } else {
    double vol = 1.0;
    for (int a = 0; a < 3; ++a) {
      const double ext = (double)ord_dec(box[3 + a]) - (double)ord_dec(box[a]);
      vol *= (ext > 1e-6 && ext == ext) ? ext : 1e-6;
    }
    const double per_graph = (double)N / (double)(G > 0 ? G : 1);
    const double density = per_graph / vol;
    double s = cbrt(2.0 * (k + 1) / (4.18879 * (density > 0 ? density : 1.0)));
    if (!(s > 1e-6)) s = 1e-6;
    if (s > 1e30) s = 1e30;
    q.s = (float)s;
  }
  *p = q;
}

__global__ void point_key_kernel(const SpatialArgs a, uint32_t* keys, int32_t* vals) {
  const GridParams p = *a.prm;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.N; i += (int64_t)gridDim.x * blockDim.x) {
    const int g = graph_of(a.gp, a.G, i);
    keys[i] = cell_hash(g, cell_of(a.x[i * 3], p.s), cell_of(a.x[i * 3 + 1], p.s), cell_of(a.x[i * 3 + 2], p.s),
                        p.mask);
    vals[i] = (int32_t)i;
  }
}

// bstart[b] = first sorted position with key >= b, for b in [0, mask + 1].
__global__ void bucket_start_kernel(int64_t N, const uint32_t* sorted_keys, const GridParams* prm,
                                    int32_t* bstart) {
  const int64_t T = (int64_t)prm->mask + 1;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= T; b += (int64_t)gridDim.x * blockDim.x) {
    int64_t lo = 0, hi = N;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if ((int64_t)sorted_keys[mid] < b) lo = mid + 1; else hi = mid;
    }
    bstart[b] = (int32_t)lo;
  }
}

__global__ void gather_points_kernel(const SpatialArgs a, const int32_t* sorted_vals, float4* pts, int4* cells) {
  const float s = a.prm->s;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < a.N; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = sorted_vals[p];
    const float x = a.x[j * 3], y = a.x[j * 3 + 1], z = a.x[j * 3 + 2];
    pts[p] = make_float4(x, y, z, __int_as_float((int)j));
    cells[p] = make_int4(cell_of(x, s), cell_of(y, s), cell_of(z, s), graph_of(a.gp, a.G, j));
  }
}

// ---- per-warp candidate enumeration ------------------------------------------------
struct Query {
  float4 xi;
  int cx, cy, cz, g, i;
};

struct WarpScratch {
  int st[32];
  int ex[32];
  int4 cell[32];
  unsigned long long buf[kCap];
};

__device__ __forceinline__ Query make_query(const SpatialArgs& a, float s, int64_t i) {
  Query q;
  q.xi = make_float4(a.x[i * 3], a.x[i * 3 + 1], a.x[i * 3 + 2], 0.f);
  q.cx = cell_of(q.xi.x, s);
  q.cy = cell_of(q.xi.y, s);
  q.cz = cell_of(q.xi.z, s);
  q.g = graph_of(a.gp, a.G, i);
  q.i = (int)i;
  return q;
}

// Calls f(ok, j, d2) warp-collectively for every candidate j != i of the
// query's graph whose cell lies in the cube of half-width R around the
// query's cell (ok = false on lanes without a candidate).
template <class F>
__device__ __forceinline__ void for_cube(const SpatialArgs& a, const GridParams& p, const Query& q, int R,
                                         WarpScratch& ws, F&& f) {
  const int lane = threadIdx.x & 31;
  const int side = 2 * R + 1, ncell = side * side * side;
  for (int base = 0; base < ncell; base += 32) {
    const int c = base + lane;
    int st = 0, len = 0;
    int4 cc = make_int4(0, 0, 0, -1);
    if (c < ncell) {
      cc = make_int4(q.cx + c % side - R, q.cy + (c / side) % side - R, q.cz + c / (side * side) - R, q.g);
      const uint32_t b = cell_hash(cc.w, cc.x, cc.y, cc.z, p.mask);
      st = a.bstart[b];
      len = a.bstart[b + 1] - st;
    }
    int incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    ws.st[lane] = st;
    ws.ex[lane] = incl - len;
    ws.cell[lane] = cc;
    __syncwarp();
    for (int t0 = 0; t0 < total; t0 += 32) {
      const int t = t0 + lane;
      bool ok = false;
      int j = 0;
      float d2 = 0.f;
      if (t < total) {
        int lo = 0, hi = 31;   // largest owner with ex <= t
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (ws.ex[mid] <= t) lo = mid; else hi = mid - 1;
        }
        const int pidx = ws.st[lo] + (t - ws.ex[lo]);
        const int4 pc = a.cells[pidx];
        const int4 want = ws.cell[lo];
        if (pc.x == want.x && pc.y == want.y && pc.z == want.z && pc.w == want.w) {
          const float4 xp = a.pts[pidx];
          j = __float_as_int(xp.w);
          if (j != q.i) {
            ok = true;
            d2 = sqdist(q.xi, xp);
          }
        }
      }
      f(ok, j, d2);
    }
    __syncwarp();
  }
}

// Calls f(ok, j, d2) for every j != i in the node range [lo, hi).
template <class F>
__device__ __forceinline__ void for_range(const SpatialArgs& a, const Query& q, int64_t lo, int64_t hi, F&& f) {
  const int lane = threadIdx.x & 31;
  for (int64_t t0 = lo; t0 < hi; t0 += 32) {
    const int64_t j = t0 + lane;
    bool ok = false;
    float d2 = 0.f;
    if (j < hi && j != q.i) {
      ok = true;
      d2 = sqdist(q.xi, make_float4(a.x[j * 3], a.x[j * 3 + 1], a.x[j * 3 + 2], 0.f));
    }
    f(ok, (int)j, d2);
  }
}

// ---- per-warp selection of the smallest keys -----------------------------------------
__device__ void warp_sort(unsigned long long* buf, int n) {
  const int lane = threadIdx.x & 31;
  int P = 32;
  while (P < n) P <<= 1;
  for (int t = n + lane; t < P; t += 32) buf[t] = ~0ull;
  __syncwarp();
  for (int k = 2; k <= P; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int idx = lane; idx < P; idx += 32) {
        const int ixj = idx ^ j;
        if (ixj > idx) {
          const unsigned long long u = buf[idx], v = buf[ixj];
          const bool up = (idx & k) == 0;
          if ((u > v) == up) { buf[idx] = v; buf[ixj] = u; }
        }
      }
      __syncwarp();
    }
}

// Keeps (at least) the `keep` smallest keys above `floor_key` offered to it.
struct Select {
  unsigned long long* buf;
  int n, keep;
  unsigned long long bound, floor_key;
  bool has_floor;

  __device__ void offer(bool ok, unsigned long long key) {
    ok = ok && key < bound && (!has_floor || key > floor_key);
    unsigned m = __ballot_sync(0xffffffffu, ok);
    if (!m) return;
    if (n + __popc(m) > kCap) {            // full: sort, keep the smallest, tighten the bound
      warp_sort(buf, n);
      n = keep;
      bound = buf[keep - 1];
      ok = ok && key < bound;
      m = __ballot_sync(0xffffffffu, ok);
    }
    const int lane = threadIdx.x & 31;
    if (ok) buf[n + __popc(m & ((1u << lane) - 1u))] = key;
    n += __popc(m);
    __syncwarp();
  }
  // Sorts what is held and returns how many of the smallest are wanted and present.
  __device__ int finish(int want) {
    warp_sort(buf, n);
    return n < want ? n : want;
  }
};

__device__ __forceinline__ unsigned long long dist_key(float d2, int j) {
  return ((unsigned long long)__float_as_uint(d2) << 32) | (unsigned)j;
}

// Rows of the radius modes: number of j with d2 < cutoff^2 (capped).
__device__ __forceinline__ int radius_cube(const GridParams& p, const Query& q) {
  const float m = fmaxf(fabsf(q.xi.x), fmaxf(fabsf(q.xi.y), fabsf(q.xi.z)));
  return (m < 1024.f * p.s) ? 1 : 2;   // far from the origin the cell rounding can shift by one more
}

// Total of the row lengths in 64 bits; flags totals that do not fit int32.
__global__ void row_total_kernel(int64_t N, const int32_t* rowlen, unsigned long long* total, int* err) {
  unsigned long long t = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x)
    t += (unsigned)rowlen[i];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if ((threadIdx.x & 31) == 0 && t) {
    const unsigned long long prev = atomicAdd(total, t);
    if (prev + t >= (unsigned long long)INT32_MAX) atomicOr(err, 8);
  }
}

__global__ void __launch_bounds__(kWarps * 32) spatial_count_kernel(const SpatialArgs a, int32_t* rowlen) {
  __shared__ WarpScratch scratch[kWarps];
  WarpScratch& ws = scratch[threadIdx.x / 32];
  const GridParams p = *a.prm;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kWarps;
  for (int64_t i = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32; i < a.N; i += warps) {
    const Query q = make_query(a, p.s, i);
    int L;
    if (a.mode == EGNN_GRAPH_KNN) {
      const int64_t n_g = a.gp ? a.gp[q.g + 1] - a.gp[q.g] : a.N;
      L = (int)std::min<int64_t>(a.k, n_g - 1 > 0 ? n_g - 1 : 0);
    } else {
      int cnt = 0;
      for_cube(a, p, q, radius_cube(p, q), ws, [&](bool ok, int, float d2) {
        cnt += __popc(__ballot_sync(0xffffffffu, ok && d2 < p.c2));
      });
      L = (a.k > 0 && cnt > a.k) ? a.k : cnt;
    }
    if (lane == 0) rowlen[i] = L;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) rowlen[a.N] = 0;
}

// Squared radius of the ball around the query that the cube of half-width R
// is guaranteed to contain (less a margin for the rounding of the cells).
__device__ __forceinline__ double covered2(const Query& q, float s, int R) {
  const double S = s;
  const double xs[3] = {q.xi.x, q.xi.y, q.xi.z};
  const int cs[3] = {q.cx, q.cy, q.cz};
  double cov = 1e300;
  for (int a = 0; a < 3; ++a) {
    const double lo = (double)(cs[a] - R) * S, hi = (double)(cs[a] + R + 1) * S;
    const double margin = 1e-5 * (fabs(xs[a]) + (R + 1) * S);
    cov = fmin(cov, fmin(xs[a] - lo, hi - xs[a]) - margin);
  }
  return cov > 0 ? cov * cov * (1.0 - 1e-5) : 0.0;
}

__global__ void __launch_bounds__(kWarps * 32) spatial_fill_kernel(const SpatialArgs a, const int32_t* row_ptr,
                                                                   int32_t* col_idx, int32_t* row_idx) {
  __shared__ WarpScratch scratch[kWarps];
  WarpScratch& ws = scratch[threadIdx.x / 32];
  const GridParams p = *a.prm;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * kWarps;
  for (int64_t i = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32; i < a.N; i += warps) {
    const Query q = make_query(a, p.s, i);
    const int64_t start = row_ptr[i];
    const int L = row_ptr[i + 1] - row_ptr[i];
    if (L <= 0) continue;
    auto emit = [&](int from, int cnt) {
      for (int t = lane; t < cnt; t += 32) {
        col_idx[start + from + t] = (int32_t)(ws.buf[t] & 0xffffffffu);
        row_idx[start + from + t] = (int32_t)i;
      }
      __syncwarp();
    };
    if (a.mode == EGNN_GRAPH_KNN) {
      bool done = false;
      for (int R = 1; R <= 4 && !done; R <<= 1) {
        Select sel{ws.buf, 0, L, ~0ull, 0ull, false};
        for_cube(a, p, q, R, ws, [&](bool ok, int j, float d2) { sel.offer(ok, dist_key(d2, j)); });
        const int got = sel.finish(L);
        if (got == L && (double)__uint_as_float((unsigned)(ws.buf[L - 1] >> 32)) < covered2(q, p.s, R)) {
          emit(0, L);
          done = true;
        }
        __syncwarp();
      }
      if (!done) {   // exact fallback: the whole graph
        const int64_t lo = a.gp ? a.gp[q.g] : 0, hi = a.gp ? a.gp[q.g + 1] : a.N;
        Select sel{ws.buf, 0, L, ~0ull, 0ull, false};
        for_range(a, q, lo, hi, [&](bool ok, int j, float d2) { sel.offer(ok, dist_key(d2, j)); });
        const int got = sel.finish(L);
        emit(0, got);
        if (got != L && lane == 0) atomicOr(a.err, 4);
      }
    } else {
      // radius: keys j (increasing index) or (d2, j) when capped; rows longer
      // than one buffer go out in passes above the previous pass's last key
      const bool capped = a.k > 0;
      const int R = radius_cube(p, q);
      int emitted = 0;
      unsigned long long floor_key = 0;
      bool has_floor = false;
      while (emitted < L) {
        const int want = (L - emitted < kKeep) ? L - emitted : kKeep;
        Select sel{ws.buf, 0, want, ~0ull, floor_key, has_floor};
        for_cube(a, p, q, R, ws, [&](bool ok, int j, float d2) {
          const bool hit = ok && d2 < p.c2;
          sel.offer(hit, capped ? dist_key(d2, j) : (unsigned long long)(unsigned)j);
        });
        const int got = sel.finish(want);
        emit(emitted, got);
        if (got < want) {
          if (lane == 0) atomicOr(a.err, 4);
          break;
        }
        floor_key = ws.buf[got - 1];
        has_floor = true;
        emitted += got;
        __syncwarp();
      }
    }
  }
}

// ---- Morton order ----------------------------------------------------------------------
__global__ void morton_kernel(int64_t N, const float* x, double lo0, double lo1, double lo2, double hi0,
                              double hi1, double hi2, int bits, unsigned long long* code, int32_t* vals) {
  const double lo[3] = {lo0, lo1, lo2}, hi[3] = {hi0, hi1, hi2};
  const double scale = (double)(1ull << bits);
  const unsigned long long qmax = (1ull << bits) - 1ull;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    unsigned long long q[3];
    for (int a = 0; a < 3; ++a) {
      const double v = floor(__dmul_rn(__ddiv_rn(__dsub_rn((double)x[i * 3 + a], lo[a]), __dsub_rn(hi[a], lo[a])), scale));
      q[a] = !(v > 0.0) ? 0ull : (v >= (double)qmax ? qmax : (unsigned long long)v);
    }
    unsigned long long c = 0;
    for (int b = 0; b < bits; ++b)
      for (int a = 0; a < 3; ++a) c |= ((q[a] >> b) & 1ull) << (3 * b + a);
    code[i] = c;
    vals[i] = (int32_t)i;
  }
}

// ---- workspace layout ----------------------------------------------------------------------
struct SpatialWs {
  GridParams* prm; uint32_t* box; unsigned long long* total; int* err;
  uint32_t* kin; uint32_t* kout; int32_t* vin; int32_t* vout;
  int32_t* bstart; float4* pts; int4* cells; int32_t* rowlen;
  void* cub; size_t cub_bytes;
  int tbits;
};

size_t spatial_cub_bytes(int64_t N, int tbits) {
  size_t a = 0, b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, a, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)std::max<int64_t>(N, 1), 0,
                                  std::max(tbits, 1));
  cub::DeviceScan::ExclusiveSum(nullptr, b, (const int32_t*)nullptr, (int32_t*)nullptr,
                                (int)std::max<int64_t>(N + 1, 1));
  return std::max(a, b);
}

SpatialWs carve_spatial(Carver& c, int64_t N) {
  SpatialWs w;
  w.tbits = std::max(6, pow2_at_least(2 * std::max<int64_t>(N, 1)));
  const int64_t T = 1LL << w.tbits;
  const int64_t n = std::max<int64_t>(N, 1);
  w.prm = c.take<GridParams>(1);
  w.box = c.take<uint32_t>(8);
  w.total = c.take<unsigned long long>(1);
  w.err = c.take<int>(4);
  w.kin = c.take<uint32_t>(n);
  w.kout = c.take<uint32_t>(n);
  w.vin = c.take<int32_t>(n);
  w.vout = c.take<int32_t>(n);
  w.bstart = c.take<int32_t>(T + 1);
  w.pts = c.take<float4>(n);
  w.cells = c.take<int4>(n);
  w.rowlen = c.take<int32_t>(n + 1);
  w.cub_bytes = spatial_cub_bytes(N, w.tbits);
  w.cub = c.take<char>(w.cub_bytes);
  return w;
}

int check_spatial(const egnn_spatial_desc* d, const char* who) {
  if (!d) return fail(EGNN_ERR_INVALID_ARG, "%s: null descriptor", who);
  if (d->n_nodes < 0 || d->n_nodes > (1LL << 30))
    return fail(EGNN_ERR_INVALID_ARG, "%s: n_nodes %lld out of range", who, (long long)d->n_nodes);
  if (d->graph_ptr && d->n_graphs < 1)
    return fail(EGNN_ERR_INVALID_ARG, "%s: graph_ptr given with n_graphs < 1", who);
  if (d->n_nodes > 0 && !d->x) return fail(EGNN_ERR_INVALID_ARG, "%s: null coordinates", who);
  if (d->mode == EGNN_GRAPH_RADIUS) {
    if (!(d->cutoff > 0.f) || !(d->cutoff < 3.0e38f))
      return fail(EGNN_ERR_INVALID_ARG, "%s: radius mode needs a finite cutoff > 0", who);
    if (d->max_nbrs < 0) return fail(EGNN_ERR_INVALID_ARG, "%s: max_nbrs < 0", who);
  } else if (d->mode == EGNN_GRAPH_KNN) {
    if (d->max_nbrs < 0 || d->max_nbrs > kMaxK)
      return fail(EGNN_ERR_UNSUPPORTED, "%s: k = %d not built (0..%d)", who, d->max_nbrs, kMaxK);
    if (!(d->cutoff >= 0.f) || !(d->cutoff < 3.0e38f))
      return fail(EGNN_ERR_INVALID_ARG, "%s: cell size hint must be finite and >= 0", who);
  } else {
    return fail(EGNN_ERR_INVALID_ARG, "%s: unknown mode %d", who, d->mode);
  }
  return EGNN_OK;
}

SpatialArgs spatial_args(const egnn_spatial_desc* d, const SpatialWs& w) {
  SpatialArgs a;
  a.N = d->n_nodes;
  a.G = d->graph_ptr ? d->n_graphs : 1;
  a.x = d->x;
  a.gp = d->graph_ptr;
  a.mode = d->mode;
  a.k = d->max_nbrs;
  a.prm = w.prm;
  a.bstart = w.bstart;
  a.pts = w.pts;
  a.cells = w.cells;
  a.err = w.err;
  return a;
}

int read_err(const int* err, cudaStream_t s, int* out) {
  EGNN_CHECK_CUDA(cudaMemcpyAsync(out, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  EGNN_CHECK_CUDA(cudaStreamSynchronize(s));
  return EGNN_OK;
}

unsigned query_blocks(int64_t N) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((N + kWarps - 1) / kWarps, 148LL * 16));
}

}  // namespace
}  // namespace egnn

using namespace egnn;

extern "C" size_t egnn_fc_graph_workspace_size(int64_t n_graphs) {
  Carver c(nullptr);
  c.take<int>(4);
  c.take<int64_t>(std::max<int64_t>(n_graphs, 0) + 1);   // counts
  c.take<int64_t>(std::max<int64_t>(n_graphs, 0) + 1);   // offsets
  size_t b = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, b, (const int64_t*)nullptr, (int64_t*)nullptr,
                                (int)std::max<int64_t>(n_graphs + 1, 1));
  c.take<char>(b);
  return c.size();
}

extern "C" int egnn_fc_graph(int64_t n_nodes, int64_t n_graphs, const int64_t* graph_ptr, int64_t n_edges,
                             int32_t* row_ptr, int32_t* col_idx, int32_t* row_idx, void* ws, size_t ws_bytes,
                             void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n_nodes < 0 || n_edges < 0 || n_nodes >= INT32_MAX || n_edges >= INT32_MAX || n_graphs < 1 ||
      n_graphs >= INT32_MAX)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_fc_graph: sizes out of range");
  if (!graph_ptr || !row_ptr || (n_edges > 0 && (!col_idx || !row_idx)))
    return fail(EGNN_ERR_INVALID_ARG, "egnn_fc_graph: null pointer");
  if (!ws || ws_bytes < egnn_fc_graph_workspace_size(n_graphs))
    return fail(EGNN_ERR_WORKSPACE, "egnn_fc_graph: workspace too small");
  Carver c(ws);
  int* err = c.take<int>(4);
  int64_t* cnt = c.take<int64_t>(n_graphs + 1);
  int64_t* off = c.take<int64_t>(n_graphs + 1);
  size_t cb = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, cb, (const int64_t*)nullptr, (int64_t*)nullptr, (int)(n_graphs + 1));
  void* ctmp = c.take<char>(cb);
  EGNN_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  check_graph_ptr_kernel<<<grid_for(n_graphs + 1), 256, 0, s>>>(n_nodes, n_graphs, graph_ptr, err);
  EGNN_CHECK_LAUNCH();
  int herr = 0;
  EGNN_TRY(read_err(err, s, &herr));
  if (herr) return fail(EGNN_ERR_INDEX, "egnn_fc_graph: graph_ptr must rise from 0 to n_nodes");
  fc_counts_kernel<<<grid_for(n_graphs + 1), 256, 0, s>>>(n_graphs, graph_ptr, cnt);
  EGNN_CHECK_LAUNCH();
  EGNN_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(ctmp, cb, cnt, off, (int)(n_graphs + 1), s));
  count_launch();
  if (n_nodes == 0) {
    EGNN_CHECK_CUDA(cudaMemsetAsync(row_ptr, 0, sizeof(int32_t), s));
    return n_edges == 0 ? EGNN_OK : fail(EGNN_ERR_INVALID_ARG, "egnn_fc_graph: n_edges must be 0");
  }
  fc_fill_kernel<<<grid_for(n_nodes * 32), 256, 0, s>>>(n_nodes, n_graphs, graph_ptr, off, n_edges, row_ptr,
                                                        col_idx, row_idx, err);
  EGNN_CHECK_LAUNCH();
  EGNN_TRY(read_err(err, s, &herr));
  if (herr) return fail(EGNN_ERR_INVALID_ARG, "egnn_fc_graph: n_edges differs from sum n_g (n_g - 1)");
  return EGNN_OK;
}

extern "C" size_t egnn_spatial_workspace_size(int64_t n_nodes) {
  Carver c(nullptr);
  carve_spatial(c, std::max<int64_t>(n_nodes, 0));
  return c.size();
}

extern "C" int egnn_spatial_count(const egnn_spatial_desc* d, int32_t* row_ptr, void* ws, size_t ws_bytes,
                                  void* stream) {
  EGNN_TRY(check_spatial(d, "egnn_spatial_count"));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t N = d->n_nodes;
  if (!row_ptr) return fail(EGNN_ERR_INVALID_ARG, "egnn_spatial_count: null row_ptr");
  if (!ws || ws_bytes < egnn_spatial_workspace_size(N))
    return fail(EGNN_ERR_WORKSPACE, "egnn_spatial_count: workspace too small");
  Carver c(ws);
  SpatialWs w = carve_spatial(c, N);
  const SpatialArgs a = spatial_args(d, w);
  EGNN_CHECK_CUDA(cudaMemsetAsync(w.err, 0, sizeof(int), s));
  if (d->graph_ptr) {
    check_graph_ptr_kernel<<<grid_for(a.G + 1), 256, 0, s>>>(N, a.G, d->graph_ptr, w.err);
    EGNN_CHECK_LAUNCH();
    int herr = 0;
    EGNN_TRY(read_err(w.err, s, &herr));
    if (herr) return fail(EGNN_ERR_INDEX, "egnn_spatial_count: graph_ptr must rise from 0 to n_nodes");
  }
  if (N == 0) {
    EGNN_CHECK_CUDA(cudaMemsetAsync(row_ptr, 0, sizeof(int32_t), s));
    return EGNN_OK;
  }
  // bounding box (all ones / zeros encode +inf / -inf starts for min / max)
  EGNN_CHECK_CUDA(cudaMemsetAsync(w.box, 0xff, 3 * sizeof(uint32_t), s));
  EGNN_CHECK_CUDA(cudaMemsetAsync(w.box + 3, 0, 3 * sizeof(uint32_t), s));
  bbox_kernel<<<grid_for(N), 256, 0, s>>>(N, d->x, w.box);
  EGNN_CHECK_LAUNCH();
  params_kernel<<<1, 1, 0, s>>>(N, a.G, d->mode, d->max_nbrs, d->cutoff, (uint32_t)((1LL << w.tbits) - 1), w.box,
                                w.prm);
  EGNN_CHECK_LAUNCH();
  point_key_kernel<<<grid_for(N), 256, 0, s>>>(a, w.kin, w.vin);
  EGNN_CHECK_LAUNCH();
  size_t cb = w.cub_bytes;
  EGNN_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(w.cub, cb, w.kin, w.kout, w.vin, w.vout, (int)N, 0, w.tbits, s));
  count_launch();
  bucket_start_kernel<<<grid_for((1LL << w.tbits) + 1), 256, 0, s>>>(N, w.kout, w.prm, w.bstart);
  EGNN_CHECK_LAUNCH();
  gather_points_kernel<<<grid_for(N), 256, 0, s>>>(a, w.vout, w.pts, w.cells);
  EGNN_CHECK_LAUNCH();
  spatial_count_kernel<<<query_blocks(N), kWarps * 32, 0, s>>>(a, w.rowlen);
  EGNN_CHECK_LAUNCH();
  EGNN_CHECK_CUDA(cudaMemsetAsync(w.total, 0, sizeof(unsigned long long), s));
  row_total_kernel<<<grid_for(N), 256, 0, s>>>(N, w.rowlen, w.total, w.err);
  EGNN_CHECK_LAUNCH();
  int herr = 0;
  EGNN_TRY(read_err(w.err, s, &herr));
  if (herr) return fail(EGNN_ERR_UNSUPPORTED, "egnn_spatial_count: the graph has 2^31 edges or more");
  cb = w.cub_bytes;
  EGNN_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(w.cub, cb, w.rowlen, row_ptr, (int)(N + 1), s));
  count_launch();
  return EGNN_OK;
}

extern "C" int egnn_spatial_fill(const egnn_spatial_desc* d, const int32_t* row_ptr, int32_t* col_idx,
                                 int32_t* row_idx, void* ws, size_t ws_bytes, void* stream) {
  EGNN_TRY(check_spatial(d, "egnn_spatial_fill"));
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t N = d->n_nodes;
  if (!row_ptr) return fail(EGNN_ERR_INVALID_ARG, "egnn_spatial_fill: null row_ptr");
  if (!ws || ws_bytes < egnn_spatial_workspace_size(N))
    return fail(EGNN_ERR_WORKSPACE, "egnn_spatial_fill: workspace too small");
  if (N == 0) return EGNN_OK;
  Carver c(ws);
  SpatialWs w = carve_spatial(c, N);
  const SpatialArgs a = spatial_args(d, w);
  spatial_fill_kernel<<<query_blocks(N), kWarps * 32, 0, s>>>(a, row_ptr, col_idx, row_idx);
  EGNN_CHECK_LAUNCH();
  int herr = 0;
  EGNN_TRY(read_err(w.err, s, &herr));
  if (herr)
    return fail(EGNN_ERR_INVALID_ARG,
                "egnn_spatial_fill: rows differ from egnn_spatial_count (inputs or workspace changed in between)");
  return EGNN_OK;
}

extern "C" size_t egnn_morton_workspace_size(int64_t n_nodes) {
  const int64_t n = std::max<int64_t>(n_nodes, 1);
  Carver c(nullptr);
  c.take<unsigned long long>(n);   // sorted codes
  c.take<int32_t>(n);              // iota
  size_t b = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, b, (const unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 63);
  c.take<char>(b);
  return c.size();
}

extern "C" int egnn_morton_order(int64_t n_nodes, const float* x, const double* lo, const double* hi, int bits,
                                 uint64_t* codes, int32_t* perm, void* ws, size_t ws_bytes, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (n_nodes < 0 || n_nodes >= INT32_MAX || bits < 1 || bits > 21 || !lo || !hi)
    return fail(EGNN_ERR_INVALID_ARG, "egnn_morton_order: bad arguments");
  for (int a = 0; a < 3; ++a)
    if (!(hi[a] > lo[a])) return fail(EGNN_ERR_INVALID_ARG, "egnn_morton_order: hi must exceed lo on every axis");
  if (n_nodes == 0) return EGNN_OK;
  if (!x || !codes || !perm) return fail(EGNN_ERR_INVALID_ARG, "egnn_morton_order: null pointer");
  if (!ws || ws_bytes < egnn_morton_workspace_size(n_nodes))
    return fail(EGNN_ERR_WORKSPACE, "egnn_morton_order: workspace too small");
  Carver c(ws);
  unsigned long long* ksorted = c.take<unsigned long long>(n_nodes);
  int32_t* vin = c.take<int32_t>(n_nodes);
  size_t cb = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, cb, (const unsigned long long*)nullptr, (unsigned long long*)nullptr,
                                  (const int32_t*)nullptr, (int32_t*)nullptr, (int)n_nodes, 0, 63);
  void* ctmp = c.take<char>(cb);
  unsigned long long* kc = reinterpret_cast<unsigned long long*>(codes);
  morton_kernel<<<grid_for(n_nodes), 256, 0, s>>>(n_nodes, x, lo[0], lo[1], lo[2], hi[0], hi[1], hi[2], bits, kc, vin);
  EGNN_CHECK_LAUNCH();
  EGNN_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(ctmp, cb, kc, ksorted, vin, perm, (int)n_nodes, 0, 3 * bits, s));
  count_launch();
  return EGNN_OK;
}
