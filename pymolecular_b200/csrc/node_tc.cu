// Node-side GEMMs for bf16 mode on the 5th-generation tensor cores.
//
// Every fp32 operand is split into hi = bf16(x) and lo = bf16(x - hi) and the
// product is taken as hi*hi + hi*lo + lo*hi with fp32 accumulation in TMEM
// (about 16 bits of operand precision, ~1e-5 relative per output).
//
// Two persistent, warp-specialised kernels, one CTA per SM (288 threads):
//   warps 0-3  producers: load fp32 operand rows with coalesced 16-byte
//              loads, split them in registers and write the hi / lo SW128
//              tiles of a stage of the shared-memory ring;
//   warps 4-7  epilogue: drain the TMEM accumulator 32 columns at a time
//              through a shared staging tile and write whole row pieces;
//   warp 8     one thread issues the tcgen05.mma (3 per K-step) and commits.
// Stages are handed over with mbarriers (full: 128 producer arrivals; empty
// and accumulator-full: tcgen05.commit; accumulator-empty: 4 epilogue warps).
//
// Data GEMMs  C (M x N) = A (M x K) B (K x N) + epilogue, B = a weight held
//   row-major [k][n]: each CTA keeps one N-chunk of B (hi and lo, MN-major,
//   at most 128 KB) resident, splits it once, and walks row tiles of 128
//   with a double-buffered TMEM accumulator, so the epilogue of tile j
//   overlaps the loads and MMAs of tile j + 1.  CTAs that share a row tile
//   (one per N-chunk) run it at about the same time, so A is read from HBM
//   once.
// Weight gradients  dW (M x N) = sum_r G[r][m] X[r][n] over the node rows:
//   one output tile (128 x BN) per CTA and a contiguous slice of the rows
//   (split-K); both operands stream through the ring as MN-major tiles; the
//   slices are added in slice order by gemm_reduce, and db (the column sums
//   of G) is summed by the producers in a fixed order.
// Every wait is bounded (2 s of global time); a thread that gives up raises
// the CTA's abort flag, which every other wait honours; the event is counted
// (egnn_device_status) and the CTA drains its MMAs, frees its TMEM and exits.
#include <algorithm>

#include "node_tc.cuh"
#include "tc.cuh"

namespace egnn {

__device__ int g_node_tc_timeouts = 0;

namespace {

using namespace tc;

constexpr int kBM = 128;                  // rows of an output tile (MMA M)
constexpr int kBK = 64;                   // K per ring stage
constexpr int kNT = 288;                  // 4 producer + 4 epilogue warps + MMA warp
constexpr int kWMax = 128 * 1024;         // resident weight bytes (hi + lo)
constexpr int kStgLd = 33;                // staging row stride (floats)
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`; false once 2 s have passed (the abort
// flag is raised and the event counted) or once another thread raised it.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_f) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_f && *abort_f) return false;
    if (global_ns() - t0 > kWaitNs) {
      if (abort_f) *abort_f = 1;
      atomicAdd(&g_node_tc_timeouts, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier of the 4 epilogue warps.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Split 4 floats into hi / lo bf16 and store them (8 bytes each) at byte
// offset `off` of the hi and lo tiles.
__device__ __forceinline__ void st4_split(char* hi, char* lo, uint32_t off, float4 x) {
  const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
  const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
  const __nv_bfloat162 l01 = __floats2bfloat162_rn(x.x - f01.x, x.y - f01.y);
  const __nv_bfloat162 l23 = __floats2bfloat162_rn(x.z - f23.x, x.w - f23.y);
  uint2 uh, ul;
  uh.x = *reinterpret_cast<const uint32_t*>(&h01);
  uh.y = *reinterpret_cast<const uint32_t*>(&h23);
  ul.x = *reinterpret_cast<const uint32_t*>(&l01);
  ul.y = *reinterpret_cast<const uint32_t*>(&l23);
  *reinterpret_cast<uint2*>(hi + off) = uh;
  *reinterpret_cast<uint2*>(lo + off) = ul;
}

// Four consecutive elements X(r, c .. c + 3) of a row-major (possibly
// column-split) matrix; zero outside [0, rows) x [0, cols).  Callers keep
// c % 4 == 0 and the split on a multiple of 4, so the word lies in one part.
__device__ __forceinline__ float4 ld4(const Mat& X, int64_t r, int64_t c, int64_t rows, int64_t cols) {
  if (r >= rows || c >= cols) return make_float4(0.f, 0.f, 0.f, 0.f);
  const float* p = c < X.split ? X.p0 + r * X.ld0 + c : X.p1 + r * X.ld1 + (c - X.split);
  if (c + 4 <= cols) return __ldg(reinterpret_cast<const float4*>(p));
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < 4 && c + t < cols; ++t) v[t] = __ldg(p + t);
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Shared-memory layout of one kernel instance.
//   data: W hi | W lo (resident, kWMax bytes reserved) | ring of 2 stages of
//         the A chunk (128 m x 64 k, hi + lo) | staging | barriers
//   WG:   ring of 4 stages of [A^T chunk (32 k x 128 m, hi + lo) | X chunk
//         (32 k x BN, hi + lo)] | staging | db partials | barriers
constexpr int kBKW = 32;                  // node rows per weight-gradient stage
template <int BN, bool WG>
struct NL {
  static constexpr int KS = WG ? kBKW : kBK;                        // K per stage
  static constexpr int A_PART = kBM * KS * 2;                       // 16 / 8 KB
  static constexpr int B_PART = KS * BN * 2;                        // WG only
  static constexpr int STAGE = WG ? 2 * A_PART + 2 * B_PART : 2 * A_PART;
  static constexpr int S = WG ? 4 : 2;
  static constexpr int RING = WG ? 0 : kWMax;
  static constexpr int STG = RING + S * STAGE;                       // float[128][33]
  static constexpr int RED = STG + kBM * kStgLd * 4;                 // WG: db partials float[4][128]
  static constexpr int BAR = RED + 4 * kBM * 4;
  static constexpr size_t BYTES = BAR + 160 + 1024;
};

struct Bars {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* accf;
  uint64_t* acce;
  uint64_t* fin;
  uint32_t* tmem_s;
  int* abort_s;
  __device__ Bars(char* p) {
    full = reinterpret_cast<uint64_t*>(p);
    empty = full + 4;
    accf = empty + 4;
    acce = accf + 2;
    fin = acce + 2;
    tmem_s = reinterpret_cast<uint32_t*>(fin + 1);
    abort_s = reinterpret_cast<int*>(tmem_s + 1);
  }
};

__device__ __forceinline__ void init_bars(const Bars& b, int stages) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&b.full[s], 128);
    mbar_init(&b.empty[s], 1);
  }
  for (int s = 0; s < 2; ++s) {
    mbar_init(&b.accf[s], 1);
    mbar_init(&b.acce[s], 4);
  }
  mbar_init(b.fin, 1);
  *b.abort_s = 0;
  fence_mbar_init();
}

// Epilogue of one 128 x 32 slab: the thread's TMEM row (v[], row 32 q + lane)
// goes through the staging tile, then every thread moves 8 four-column words
// (consecutive threads on consecutive words: whole 128-byte row pieces per
// quarter warp).  `fetch(row, word, i)` issues the global loads word i needs
// (all 8 words' loads are in flight before the first result is formed) and
// `emit(row, word, i, float4)` applies the epilogue and stores.
template <class Fetch, class Emit>
__device__ __forceinline__ void slab_out(float* stg, int q, int lane, int etid, const float (&v)[32], Fetch fetch,
                                         Emit emit) {
  float* row = stg + (q * 32 + lane) * kStgLd;
#pragma unroll
  for (int i = 0; i < 8; ++i) fetch(i * 16 + (etid >> 3), etid & 7, i);
#pragma unroll
  for (int c = 0; c < 32; ++c) row[c] = v[c];
  epi_sync();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 16 + (etid >> 3), w = etid & 7;
    const float* src = stg + r * kStgLd + 4 * w;
    emit(r, w, i, make_float4(src[0], src[1], src[2], src[3]));
  }
  epi_sync();
}

// Per-word operands of the fused epilogue, loaded ahead of the math.
struct Side {
  float4 bias, aux, resid;
};

struct Epilogue {
  const float* bias;
  float* pre; int64_t ldp;
  int act;
  const float* aux; int64_t ldaux;
  const float* resid; int64_t ldr; int64_t resid_cols;
  float* C; int64_t ldc;
  int64_t M, N;
  int vec;
  __device__ __forceinline__ float one(int64_t m, int64_t n, float y) const {
    if (bias) y += bias[n];
    if (pre) pre[m * ldp + n] = y;
    if (act == ACT_SILU) {
      y = silu_fast(y);
    } else if (act == ACT_DSILU) {
      float yy, d;
      silu_grad_fast(aux[m * ldaux + n], yy, d);
      y *= d;
    }
    if (resid && n < resid_cols) y += resid[m * ldr + n];
    return y;
  }
  // vector path: the word's bias, SiLU' operand and residual
  __device__ __forceinline__ void fetch(int64_t m, int64_t n, Side& sd) const {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    sd.bias = sd.aux = sd.resid = z;
    if (!vec || m >= M || n >= N) return;
    if (bias) sd.bias = __ldg(reinterpret_cast<const float4*>(bias + n));
    if (act == ACT_DSILU) sd.aux = *reinterpret_cast<const float4*>(aux + m * ldaux + n);
    if (resid && n < resid_cols) sd.resid = *reinterpret_cast<const float4*>(resid + m * ldr + n);
  }
  __device__ __forceinline__ void apply4(int64_t m, int64_t n, float4 acc, const Side& sd) const {
    if (m >= M || n >= N) return;
    if (vec) {
      float y[4] = {acc.x + sd.bias.x, acc.y + sd.bias.y, acc.z + sd.bias.z, acc.w + sd.bias.w};
      if (pre) *reinterpret_cast<float4*>(pre + m * ldp + n) = make_float4(y[0], y[1], y[2], y[3]);
      if (act == ACT_SILU) {
#pragma unroll
        for (int t = 0; t < 4; ++t) y[t] = silu_fast(y[t]);
      } else if (act == ACT_DSILU) {
        const float zz[4] = {sd.aux.x, sd.aux.y, sd.aux.z, sd.aux.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float yy, d;
          silu_grad_fast(zz[t], yy, d);
          y[t] *= d;
        }
      }
      y[0] += sd.resid.x; y[1] += sd.resid.y; y[2] += sd.resid.z; y[3] += sd.resid.w;
      *reinterpret_cast<float4*>(C + m * ldc + n) = make_float4(y[0], y[1], y[2], y[3]);
    } else {
      const float a[4] = {acc.x, acc.y, acc.z, acc.w};
      for (int t = 0; t < 4; ++t)
        if (n + t < N) C[m * ldc + n + t] = one(m, n + t, a[t]);
    }
  }
};

// ---- data GEMM ------------------------------------------------------------------
struct DataArgs {
  Mat A, B;
  int64_t M, N, K, Kpad;
  int n_chunks;
  Epilogue epi;
};

template <int BN>
__global__ void __launch_bounds__(kNT, 1) nmm_data_kernel(DataArgs a) {
  using L = NL<BN, false>;
  constexpr uint32_t IDESC = make_idesc_bf16(kBM, BN, 0, 1);   // A K-major, B MN-major
  extern __shared__ __align__(1024) char nm_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(nm_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Bars bars(sm + L::BAR);
  const int Kp = (int)a.Kpad;
  char* w_hi = sm;   // resident weight: W hi | W lo, then the ring
  char* w_lo = w_hi + Kp * BN * 2;
  float* stg = reinterpret_cast<float*>(sm + L::STG);
  pdl_enter();   // the weight and the A rows may be the predecessor's output

  // CTA -> (N-chunk, first row tile, row-tile stride)
  const int nc = blockIdx.x % a.n_chunks;
  const int64_t stride = gridDim.x / a.n_chunks;
  const int64_t rt0 = blockIdx.x / a.n_chunks;
  const int64_t row_tiles = (a.M + kBM - 1) / kBM;
  const int64_t ntl = rt0 < row_tiles ? (row_tiles - 1 - rt0) / stride + 1 : 0;
  const int64_t n0 = (int64_t)nc * BN;
  const int nkc = Kp / kBK;

  // resident weight chunk B[0:Kpad][n0:n0+BN] -> hi / lo MN-major tiles,
  // eight 16-byte loads of every thread in flight per round
  for (int base = 0; base < Kp * BN / 4; base += 8 * kNT) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * kNT + tid, k = idx / (BN / 4), c = (idx % (BN / 4)) * 4;
      v[u] = idx < Kp * BN / 4 ? ld4(a.B, k, n0 + c, a.K, a.N) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * kNT + tid, k = idx / (BN / 4), c = (idx % (BN / 4)) * 4;
      if (idx < Kp * BN / 4) st4_split(w_hi, w_lo, sw128_offset(k, c, Kp), v[u]);
    }
  }
  if (warp == 8) tmem_alloc(bars.tmem_s, 2 * BN);
  if (tid == 0) init_bars(bars, L::S);
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *bars.tmem_s;
  volatile int* abort_f = bars.abort_s;

  if (warp < 4) {
    // ---- producers: A rows of each tile, 64 columns per stage.  Stage
    // it + 1 is loaded into the second register buffer before stage it waits
    // for its ring slot and is split, so 32-64 KB stay in flight per SM.
    const int ptid = tid;
    const int64_t total = ntl * nkc;
    auto load = [&](float4 (&v)[16], int64_t it) {
      const int64_t m0 = (rt0 + (it / nkc) * stride) * kBM;
      const int64_t k0 = (it % nkc) * kBK;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int idx = i * 128 + ptid, r = idx >> 4, c = (idx & 15) * 4;
        v[i] = ld4(a.A, m0 + r, k0 + c, a.M, a.K);
      }
    };
    auto put = [&](const float4 (&v)[16], int64_t it) -> bool {
      const int s = (int)(it & 1);
      if (it >= 2 && !wait_bar(&bars.empty[s], (uint32_t)((it >> 1) - 1) & 1, abort_f)) return false;
      char* st = sm + L::RING + s * L::STAGE;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int idx = i * 128 + ptid, r = idx >> 4, c = (idx & 15) * 4;
        st4_split(st, st + L::A_PART, sw128_offset(r, c, kBM), v[i]);
      }
      fence_proxy_async();
      mbar_arrive1(&bars.full[s]);
      return true;
    };
    float4 va[16], vb[16];
    if (total > 0) load(va, 0);
    for (int64_t it = 0; it < total; it += 2) {
      if (it + 1 < total) load(vb, it + 1);
      if (!put(va, it)) break;
      if (it + 1 >= total) break;
      if (it + 2 < total) load(va, it + 2);
      if (!put(vb, it + 1)) break;
    }
  } else if (warp < 8) {
    // ---- epilogue: thread = TMEM lane (row 32 q + lane) for the loads
    const int q = warp & 3, etid = tid - 128;
    for (int64_t j = 0; j < ntl; ++j) {
      const int buf = (int)(j & 1);
      const bool ok = wait_bar(&bars.accf[buf], (uint32_t)(j >> 1) & 1, abort_f);
      if (!__all_sync(0xffffffffu, ok)) break;
      fence_after_sync();
      const int64_t m0 = (rt0 + j * stride) * kBM;
#pragma unroll 1
      for (int cs = 0; cs < BN / 32; ++cs) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * BN + cs * 32, v);
        if (cs == BN / 32 - 1) {
          fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive1(&bars.acce[buf]);
        }
        Side sd[8];
        slab_out(
            stg, q, lane, etid, v,
            [&](int r, int w, int i) { a.epi.fetch(m0 + r, n0 + cs * 32 + 4 * w, sd[i]); },
            [&](int r, int w, int i, float4 val) { a.epi.apply4(m0 + r, n0 + cs * 32 + 4 * w, val, sd[i]); });
      }
    }
  } else if (lane == 0) {
    // ---- MMA issuer
    const uint32_t whi = smem_u32(w_hi), wlo = smem_u32(w_lo), ring = smem_u32(sm + L::RING);
    uint32_t it = 0;
    bool ok = true;
    for (int64_t j = 0; j < ntl && ok; ++j) {
      const int buf = (int)(j & 1);
      if (j >= 2 && !(ok = wait_bar(&bars.acce[buf], (uint32_t)((j >> 1) - 1) & 1, abort_f))) break;
      fence_after_sync();
      const uint32_t d = tmem + buf * BN;
      for (int kc = 0; kc < nkc; ++kc, ++it) {
        const int s = it & 1;
        if (!(ok = wait_bar(&bars.full[s], (it >> 1) & 1, abort_f))) break;
        fence_after_sync();
        const uint32_t ah = ring + s * L::STAGE, al = ah + L::A_PART;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t dah = make_desc(ah + kk * 32, 16, 1024), dal = make_desc(al + kk * 32, 16, 1024);
          const uint32_t boff = (kc * (kBK / 16) + kk) * 2048;
          const uint64_t dbh = make_desc(whi + boff, Kp * 128, 1024), dbl = make_desc(wlo + boff, Kp * 128, 1024);
          mma_bf16(d, dah, dbh, IDESC, (kc | kk) ? 1u : 0u);
          mma_bf16(d, dah, dbl, IDESC, 1u);
          mma_bf16(d, dal, dbh, IDESC, 1u);
        }
        mma_commit(&bars.empty[s]);
      }
      if (ok) mma_commit(&bars.accf[buf]);
    }
    mma_commit(bars.fin);   // every MMA of this thread has completed once fin flips
    wait_bar(bars.fin, 0, nullptr);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 8) tmem_dealloc(tmem, 2 * BN);
}

// ---- weight gradient --------------------------------------------------------------
struct WgArgs {
  Mat G, X;                 // G[r][m] (M columns), X[r][n] (N columns), r < R
  int64_t M, N, R;
  int ksplit;
  int64_t rows_per;         // node rows per split (a multiple of 32)
  float* C; int64_t ldc;    // ksplit == 1
  float* part;              // ksplit > 1: [ksplit][M][N]
  float* db;                // column sums of G (ksplit == 1)
  float* db_part;           // ksplit > 1: [ksplit][M]
};

template <int BN>
__global__ void __launch_bounds__(kNT, 1) nmm_wgrad_kernel(WgArgs a) {
  using L = NL<BN, true>;
  constexpr uint32_t IDESC = make_idesc_bf16(kBM, BN, 1, 1);   // both MN-major
  extern __shared__ __align__(1024) char nm_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(nm_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Bars bars(sm + L::BAR);
  float* stg = reinterpret_cast<float*>(sm + L::STG);
  float* red = reinterpret_cast<float*>(sm + L::RED);
  pdl_enter();

  const int64_t mb = blockIdx.x, nb = blockIdx.y, z = blockIdx.z;
  const int64_t m0 = mb * kBM, n0 = nb * BN;
  const int64_t r0 = std::min<int64_t>(a.R, z * a.rows_per), r1 = std::min<int64_t>(a.R, r0 + a.rows_per);
  const int nkc = (int)((r1 - r0 + kBKW - 1) / kBKW);
  const bool do_db = a.db != nullptr && nb == 0;

  if (warp == 8) tmem_alloc(bars.tmem_s, BN);
  if (tid == 0) init_bars(bars, L::S);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *bars.tmem_s;
  volatile int* abort_f = bars.abort_s;

  if (warp < 4) {
    // ---- producers: 32 node rows per stage of G (128 m columns) and X (BN n
    // columns), 8 + BN / 16 words per thread; the next stage is loaded into
    // the second register buffer before this one waits for its ring slot
    const int ptid = tid;
    constexpr int BW = BN / 4;                      // float4 words per X row
    constexpr int XW = kBKW * BW / 128;             // X words per thread: 4 or 8
    constexpr int NW = 8 + XW;
    float4 dbs = make_float4(0.f, 0.f, 0.f, 0.f);   // sums of columns m0 + 4 (ptid & 31) .. + 3
    auto load = [&](float4 (&v)[16], int kc) {
      const int64_t rb = r0 + (int64_t)kc * kBKW;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i * 128 + ptid, k = idx >> 5, c = (idx & 31) * 4;
        v[i] = ld4(a.G, rb + k, m0 + c, r1, a.M);
      }
#pragma unroll
      for (int i = 0; i < XW; ++i) {
        const int idx = i * 128 + ptid, k = idx / BW, c = (idx % BW) * 4;
        v[8 + i] = ld4(a.X, rb + k, n0 + c, r1, a.N);
      }
    };
    auto put = [&](const float4 (&v)[16], int kc) -> bool {
      const int s = kc & (L::S - 1);
      if (kc >= L::S && !wait_bar(&bars.empty[s], (uint32_t)((kc / L::S) - 1) & 1, abort_f)) return false;
      char* st = sm + s * L::STAGE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i * 128 + ptid, k = idx >> 5, c = (idx & 31) * 4;
        st4_split(st, st + L::A_PART, sw128_offset(k, c, kBKW), v[i]);
        dbs.x += v[i].x; dbs.y += v[i].y; dbs.z += v[i].z; dbs.w += v[i].w;
      }
      char* bst = st + 2 * L::A_PART;
#pragma unroll
      for (int i = 0; i < XW; ++i) {
        const int idx = i * 128 + ptid, k = idx / BW, c = (idx % BW) * 4;
        st4_split(bst, bst + L::B_PART, sw128_offset(k, c, kBKW), v[8 + i]);
      }
      fence_proxy_async();
      mbar_arrive1(&bars.full[s]);
      return true;
    };
    static_assert(NW <= 16, "one register buffer per stage");
    float4 va[16], vb[16];
    bool ok = true;
    if (nkc > 0) load(va, 0);
    for (int kc = 0; kc < nkc; kc += 2) {
      if (kc + 1 < nkc) load(vb, kc + 1);
      if (!(ok = put(va, kc))) break;
      if (kc + 1 >= nkc) break;
      if (kc + 2 < nkc) load(va, kc + 2);
      if (!(ok = put(vb, kc + 1))) break;
    }
    if (do_db && ok) {
      // the four threads of a column word (row classes ptid >> 5), combined in fixed order below
      reinterpret_cast<float4*>(red)[(ptid >> 5) * 32 + (ptid & 31)] = dbs;
    }
  } else if (warp == 8) {
    if (lane == 0) {
      const uint32_t ring = smem_u32(sm);
      bool ok = true;
      for (int kc = 0; kc < nkc; ++kc) {
        const int s = kc & (L::S - 1);
        if (!(ok = wait_bar(&bars.full[s], (uint32_t)(kc / L::S) & 1, abort_f))) break;
        fence_after_sync();
        const uint32_t ah = ring + s * L::STAGE, al = ah + L::A_PART, bh = ah + 2 * L::A_PART, bl = bh + L::B_PART;
#pragma unroll
        for (int kk = 0; kk < kBKW / 16; ++kk) {
          const uint32_t off = kk * 2048;
          const uint64_t dah = make_desc(ah + off, kBKW * 128, 1024), dal = make_desc(al + off, kBKW * 128, 1024);
          const uint64_t dbh = make_desc(bh + off, kBKW * 128, 1024), dbl = make_desc(bl + off, kBKW * 128, 1024);
          mma_bf16(tmem, dah, dbh, IDESC, (kc | kk) ? 1u : 0u);
          mma_bf16(tmem, dah, dbl, IDESC, 1u);
          mma_bf16(tmem, dal, dbh, IDESC, 1u);
        }
        mma_commit(&bars.empty[s]);
      }
      if (ok && nkc > 0) mma_commit(&bars.accf[0]);
      mma_commit(bars.fin);
      wait_bar(bars.fin, 0, nullptr);
    }
    __syncwarp();
  }
  __syncthreads();   // producers' db partials visible; the MMA thread has drained

  const bool aborted = *abort_f != 0;
  if (warp >= 4 && warp < 8 && !aborted) {
    const int q = warp & 3, etid = tid - 128;
    bool ok = true;
    if (nkc > 0) {
      ok = wait_bar(&bars.accf[0], 0, abort_f);
      fence_after_sync();
    }
    if (__all_sync(0xffffffffu, ok)) {
      float* out = a.ksplit > 1 ? a.part + z * a.M * a.N : a.C;
      const int64_t ld = a.ksplit > 1 ? a.N : a.ldc;
#pragma unroll 1
      for (int cs = 0; cs < BN / 32; ++cs) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + cs * 32, v);
        if (nkc == 0) {
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = 0.f;
        }
        slab_out(stg, q, lane, etid, v, [](int, int, int) {}, [&](int r, int w, int, float4 val) {
          const int64_t m = m0 + r, n = n0 + cs * 32 + 4 * w;
          if (m >= a.M || n >= a.N) return;
          float* dst = out + m * ld + n;
          if (n + 4 <= a.N && (ld & 3) == 0) {
            *reinterpret_cast<float4*>(dst) = val;
          } else {
            const float vv[4] = {val.x, val.y, val.z, val.w};
            for (int t = 0; t < 4 && n + t < a.N; ++t) dst[t] = vv[t];
          }
        });
      }
      if (do_db) {
        // column m0 + etid: word etid / 4, lane etid % 4 of it, row classes in order
        const float* f = red + (etid >> 2) * 4 + (etid & 3);
        const float sdb = ((f[0] + f[128]) + f[256]) + f[384];
        const int64_t m = m0 + etid;
        if (m < a.M) {
          if (a.ksplit > 1) a.db_part[z * a.M + m] = sdb;
          else a.db[m] = sdb;
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 8) tmem_dealloc(tmem, BN);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 16-byte words along the contiguous dimension: aligned bases, row strides and
// a column split that are multiples of 4 floats.
bool words_ok(const Mat& X) {
  if (X.split_rows || !aligned16(X.p0) || X.ld0 % 4) return false;
  if (X.p1 && (!aligned16(X.p1) || X.ld1 % 4 || X.split % 4)) return false;
  return true;
}

template <class K>
int set_smem(K kernel, size_t bytes) {
  EGNN_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return EGNN_OK;
}

// Resident weight chunk width: of 256 / 128 / 64 columns whose hi + lo tiles
// for all of K fit the 128 KB budget (K padded to 64), the widest that still
// gives at least one tile per SM (narrower chunks give small-M GEMMs more
// CTAs and less weight to load each; A is then re-read from L2).
int data_bn(int64_t M, int64_t N, int64_t Kpad, int sms) {
  const int64_t npad = (N + 63) / 64 * 64, row_tiles = (M + kBM - 1) / kBM;
  int best = 64;
  for (int bn : {64, 128, 256}) {
    if (bn > npad || Kpad * bn * 4 > kWMax) break;
    if (bn == 64 || row_tiles * ((N + bn - 1) / bn) >= sms) best = bn;
  }
  return best;
}

template <int BN>
int launch_data(const DataArgs& d, cudaStream_t s) {
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  constexpr size_t bytes = NL<BN, false>::BYTES;
  if (!(attr_set & bit)) {
    EGNN_TRY(set_smem(nmm_data_kernel<BN>, bytes));
    attr_set |= bit;
  }
  const int64_t row_tiles = (d.M + kBM - 1) / kBM;
  const int sms = num_sms_current();
  const int64_t per = std::max<int64_t>(1, std::min<int64_t>(sms / d.n_chunks, row_tiles));
  const unsigned grid = (unsigned)(per * d.n_chunks);
  TimerScope ts("node_gemm", s);
  EGNN_CHECK_CUDA(launch_pdl(nmm_data_kernel<BN>, dim3(grid), dim3(kNT), bytes, s, d));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

template <int BN>
int launch_wgrad(const WgArgs& w, cudaStream_t s) {
  static uint64_t attr_set = 0;
  const uint64_t bit = device_bit();
  constexpr size_t bytes = NL<BN, true>::BYTES;
  if (!(attr_set & bit)) {
    EGNN_TRY(set_smem(nmm_wgrad_kernel<BN>, bytes));
    attr_set |= bit;
  }
  const dim3 grid((unsigned)((w.M + kBM - 1) / kBM), (unsigned)((w.N + BN - 1) / BN), (unsigned)w.ksplit);
  TimerScope ts("node_gemm", s);
  EGNN_CHECK_CUDA(launch_pdl(nmm_wgrad_kernel<BN>, grid, dim3(kNT), bytes, s, w));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

int wgrad_bn(int64_t N) { return N > 64 ? 128 : 64; }

}  // namespace

bool gemm_tc_ok(const GemmArgs& a) {
  if (a.round_bf16 || a.K <= 0 || a.ksplit > 1) return false;
  // data GEMMs: A row-major [m][k], B a row-major [k][n] weight
  if (a.a_t != 0 || a.b_t != 0 || a.B.p1) return false;
  if (!words_ok(a.A) || !words_ok(a.B)) return false;
  const int64_t Kpad = (a.K + kBK - 1) / kBK * kBK;
  return Kpad * 64 * 4 <= kWMax;
}

int gemm_tc(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return EGNN_OK;
  if (!gemm_tc_ok(a)) return fail(EGNN_ERR_UNSUPPORTED, "gemm_tc: operand layout not supported");
  DataArgs d;
  d.A = a.A;
  d.B = a.B;
  d.M = a.M; d.N = a.N; d.K = a.K;
  d.Kpad = (a.K + kBK - 1) / kBK * kBK;
  const int bn = data_bn(a.M, a.N, d.Kpad, num_sms_current());
  d.n_chunks = (int)((a.N + bn - 1) / bn);
  Epilogue& e = d.epi;
  e.bias = a.bias;
  e.pre = a.pre; e.ldp = a.ldp;
  e.act = a.act;
  e.aux = a.aux; e.ldaux = a.ldaux;
  e.resid = a.resid; e.ldr = a.ldr; e.resid_cols = a.resid_cols;
  e.C = a.C; e.ldc = a.ldc;
  e.M = a.M; e.N = a.N;
  e.vec = (a.N % 4 == 0 && a.ldc % 4 == 0 && aligned16(a.C) && (!a.bias || aligned16(a.bias)) &&
           (!a.pre || (a.ldp % 4 == 0 && aligned16(a.pre))) &&
           (a.act != ACT_DSILU || (a.ldaux % 4 == 0 && aligned16(a.aux))) &&
           (!a.resid || (a.ldr % 4 == 0 && aligned16(a.resid) &&
                         (a.resid_cols == INT64_MAX || a.resid_cols % 4 == 0)))) ? 1 : 0;
  if (bn == 256) return launch_data<256>(d, s);
  if (bn == 128) return launch_data<128>(d, s);
  return launch_data<64>(d, s);
}

int64_t wgrad_tc_splits(int64_t R, int64_t M, int64_t N) {
  const int64_t tiles = std::max<int64_t>(1, ((M + 127) / 128) * ((N + wgrad_bn(N) - 1) / wgrad_bn(N)));
  const int64_t chunks = (R + 63) / 64;
  return std::max<int64_t>(1, std::min<int64_t>({148 / tiles, chunks / 2, 64}));
}

int wgrad_tc(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw, float* db, float* part,
             cudaStream_t s) {
  if (M <= 0 || N <= 0) return EGNN_OK;
  if (!words_ok(G) || !words_ok(X) || lddw < N) return wgrad(R, M, N, G, X, dW, lddw, db, 0, part, s);
  WgArgs w;
  w.G = G; w.X = X;
  w.M = M; w.N = N; w.R = R;
  // about one wave of output tiles x slices, at least 2 chunks of 64 rows per
  // slice, and no empty slices
  const int64_t chunks = (R + 63) / 64;
  const int64_t cap = wgrad_tc_splits(R, M, N);
  const int64_t per = std::max<int64_t>(1, (chunks + cap - 1) / cap);
  w.ksplit = (int)std::max<int64_t>(1, (chunks + per - 1) / per);
  w.rows_per = per * 64;
  w.C = dW; w.ldc = lddw;
  w.part = w.ksplit > 1 ? part : nullptr;
  w.db = db;
  w.db_part = (db && w.ksplit > 1) ? part + (int64_t)w.ksplit * M * N : nullptr;
  const int bn = wgrad_bn(N);
  if (bn == 128) EGNN_TRY(launch_wgrad<128>(w, s));
  else EGNN_TRY(launch_wgrad<64>(w, s));
  if (w.ksplit > 1) {
    GemmArgs r;
    r.M = M; r.N = N; r.K = R;
    r.C = dW; r.ldc = lddw;
    r.ksplit = w.ksplit;
    r.part = part;
    r.db = db;
    r.db_part = w.db_part;
    EGNN_TRY(gemm_reduce(r, s));
  }
  return EGNN_OK;
}

int node_tc_take_timeouts() {
  int n = 0;
  if (cudaMemcpyFromSymbol(&n, g_node_tc_timeouts, sizeof(int)) != cudaSuccess) return 0;
  if (n) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_node_tc_timeouts, &zero, sizeof(int));
  }
  return n;
}

}  // namespace egnn
