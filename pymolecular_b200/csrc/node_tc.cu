// Node-side GEMMs for bf16 mode on the 5th-generation tensor cores.
//
// C (M x N) = op(A) op(B) + epilogue, in 128 x BN output tiles (MMA M = 128,
// N = BN = 128, or 64 when 128-column tiles leave SMs idle; fp32 accumulator
// in BN TMEM columns), K in chunks of 64.
//
// Per CTA, three stages overlap:
//   1. cp.async copies raw fp32 chunks of A and B into a ring of NRAW shared
//      buffers, NRAW - 1 chunks ahead of the one being used;
//   2. all 256 threads split the current raw chunk into hi = bf16(x) and
//      lo = bf16(x - hi) SW128 tiles (shared to shared);
//   3. one thread issues hi*hi + hi*lo + lo*hi for the chunk's four K-steps
//      and commits to an mbarrier, waited for before the tiles are rewritten.
// Operand layouts map onto the two descriptor kinds without any transpose:
//   A row-major [m][k]                  -> K-major A tile (rows m, columns k)
//   A^T of a weight gradient, G[k][m]   -> MN-major A tile (rows k, columns m)
//   B = W[n][k]  (x W^T)                -> K-major B tile (rows n, columns k)
//   B = X[k][n]  (x W, G^T X)           -> MN-major B tile (rows k, columns n)
// Every mbarrier wait is bounded; a CTA that gives up counts it, waits once
// more for its MMAs, frees its TMEM and returns.
#include <algorithm>

#include "node_tc.cuh"
#include "tc.cuh"

namespace egnn {

__device__ int g_node_tc_timeouts = 0;

namespace {

using namespace tc;

constexpr int BMT = 128, BKT = 64, NTH = 512, NDB = NTH / 16;

// IMG: B arrives as bf16 hi / lo tiles from a prepared image (BImage) by
// bulk copies into two tile buffers; the raw ring then holds A alone and
// runs deeper (the data GEMMs, B = a weight; no db).
template <int BN, bool IMG = false>
struct TcShape {
  static constexpr int NRAW = IMG ? (BN == 64 ? 5 : (BN == 128 ? 4 : 2)) : (BN == 64 ? 3 : (BN == 128 ? 2 : 1));
  static constexpr int RAW_A = BMT * BKT * 4;          // 32 KB
  static constexpr int RAW_B = IMG ? 0 : BN * BKT * 4;
  static constexpr int RAW_STAGE = RAW_A + RAW_B;
  static constexpr int T_A = BMT * BKT * 2;            // one bf16 part of the A chunk: 16 KB
  static constexpr int T_B = BN * BKT * 2;
  static constexpr int TILES = 2 * T_A + (IMG ? 4 : 2) * T_B;   // A hi, A lo, B hi, B lo (two B buffers with IMG)
  static constexpr int OFF_RAW = TILES;
  static constexpr int OFF_BAR = OFF_RAW + NRAW * RAW_STAGE;
  static constexpr int OFF_DB = OFF_BAR + 64;          // float[NDB][128] (weight gradients only)
  static constexpr size_t SMEM_BYTES = OFF_DB + (IMG ? 0 : NDB * BMT * 4) + 1024;
};

__device__ __forceinline__ const float* mat_at(const Mat& X, int64_t r, int64_t c) {
  if (X.split_rows) return r < X.split ? X.p0 + r * X.ld0 + c : X.p1 + (r - X.split) * X.ld1 + c;
  return c < X.split ? X.p0 + r * X.ld0 + c : X.p1 + r * X.ld1 + (c - X.split);
}

__device__ __forceinline__ void cp_async16(void* dst, const float* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Raw chunk of one operand: ROWS (M or N index) x 64 (k) fp32, stored
// linearly as [tile row][tile column] with the tile's own orientation:
//   KMAJ: [r][k] (64 columns), element (r, k) at mat_at(X, r, k);
//   MN-major: [k][r] (ROWS columns), element (r, k) at mat_at(X, k, r).
// A thread's 16-byte words keep their tile position from chunk to chunk, so
// their source addresses are set up once and advance by k0 per chunk.
// Out-of-range words are zero-filled (whole words are in or out).
template <int ROWS, bool KMAJ>
struct RawCopier {
  static constexpr int COLS = KMAJ ? BKT : ROWS, WPR = COLS / 4;   // 16-byte words per raw row
  static constexpr int Q = ROWS * BKT / 4 / NTH;
  const float* src0[Q];   // KMAJ: row base in p0 (k < split); MN: &X[tr][r] in its buffer
  const float* src1[Q];   // KMAJ: row base in p1, minus split (k >= split)
  int64_t ldk[Q];         // MN: elements per k row of that buffer
  int64_t split;
  bool rok[Q];
  int tr_[Q];
  __device__ __forceinline__ RawCopier(const Mat& X, int64_t r0, int64_t rows) {
    split = X.split;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int w = threadIdx.x + NTH * q;
      const int tr = w / WPR, tc = (w % WPR) * 4;
      tr_[q] = tr;
      if (KMAJ) {
        const int64_t r = r0 + tr;
        rok[q] = r < rows;
        const int64_t rr = rok[q] ? r : 0;
        src0[q] = X.p0 + rr * X.ld0 + tc;
        src1[q] = X.p1 ? X.p1 + rr * X.ld1 + tc - X.split : src0[q];
      } else {
        const int64_t r = r0 + tc;
        rok[q] = r < rows;
        const int64_t rr = rok[q] ? r : 0;
        const bool hi = X.p1 && rr >= X.split;
        src0[q] = hi ? X.p1 + (int64_t)tr * X.ld1 + (rr - X.split) : X.p0 + (int64_t)tr * X.ld0 + rr;
        src1[q] = nullptr;
        ldk[q] = hi ? X.ld1 : X.ld0;
      }
    }
  }
  __device__ __forceinline__ void copy(float* raw, const Mat& X, int64_t k0, int64_t kend) const {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int w = threadIdx.x + NTH * q;
      const int tc = (w % WPR) * 4;
      if (KMAJ) {
        const int64_t k = k0 + tc;
        const bool ok = rok[q] && k < kend;
        const float* p = (k < split ? src0[q] : src1[q]) + k0;
        cp_async16(raw + tr_[q] * COLS + tc, ok ? p : X.p0, ok);
      } else {
        const int64_t k = k0 + tr_[q];
        const bool ok = rok[q] && k < kend;
        const float* p = src0[q] + k0 * ldk[q];
        cp_async16(raw + tr_[q] * COLS + tc, ok ? p : X.p0, ok);
      }
    }
  }
};

// Split a raw chunk into the hi / lo SW128 tiles; for MN-major chunks the
// thread may add each value to its per-column sums (a thread always sees
// the same 8 columns).
template <int ROWS, bool KMAJ>
__device__ __forceinline__ void split_raw(const float* raw, char* thi, char* tlo, float* colsum) {
  constexpr int COLS = KMAJ ? BKT : ROWS, RPR = COLS / 8;   // 8-element runs per raw row
  constexpr int RUNS = ROWS * BKT / 8;
#pragma unroll
  for (int q = 0; q < RUNS / NTH; ++q) {
    const int c = threadIdx.x + NTH * q;
    const int tr = c / RPR, tc8 = (c % RPR) * 8;
    const float4 x0 = *reinterpret_cast<const float4*>(raw + tr * COLS + tc8);
    const float4 x1 = *reinterpret_cast<const float4*>(raw + tr * COLS + tc8 + 4);
    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    uint32_t h[4], l[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const __nv_bfloat162 hp = __floats2bfloat162_rn(x[2 * t], x[2 * t + 1]);
      const float2 hf = __bfloat1622float2(hp);
      const __nv_bfloat162 lp = __floats2bfloat162_rn(x[2 * t] - hf.x, x[2 * t + 1] - hf.y);
      h[t] = *reinterpret_cast<const uint32_t*>(&hp);
      l[t] = *reinterpret_cast<const uint32_t*>(&lp);
    }
    const uint32_t off = sw128_offset(tr, tc8, KMAJ ? ROWS : BKT);
    *reinterpret_cast<uint4*>(thi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(tlo + off) = make_uint4(l[0], l[1], l[2], l[3]);
    if (!KMAJ && colsum) {
#pragma unroll
      for (int t = 0; t < 8; ++t) colsum[t] += x[t];
    }
  }
}

__device__ __forceinline__ uint64_t tdesc(const char* tile, bool kmaj, int kk) {
  return kmaj ? make_desc(smem_u32(tile) + kk * 32, 16, 1024)               // K-major, one 64-col block
              : make_desc(smem_u32(tile) + kk * 2048, BKT * 128, 1024);     // MN-major, 64 k-rows
}

// All-thread bounded wait for `bar` at parity `ph`.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t ph) {
  const bool ok = mbar_wait(bar, ph);
  return !__syncthreads_or(!ok);
}

template <int A_T, int B_T, int BNT, bool IMG = false>
__global__ void __launch_bounds__(NTH, 1) gemm_tc_kernel(GemmArgs a) {
  pdl_enter();
  using S = TcShape<BNT, IMG>;
  static_assert(!IMG || (A_T == 0 && B_T == 0), "image path: data GEMMs, MN-major B");
  extern __shared__ __align__(1024) char tsm_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~uintptr_t(1023));
  char* a_hi = sm;
  char* a_lo = sm + S::T_A;
  char* b_hi = sm + 2 * S::T_A;
  char* b_lo = sm + 2 * S::T_A + S::T_B;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + S::OFF_BAR);
  uint32_t* tmem_s = reinterpret_cast<uint32_t*>(sm + S::OFF_BAR + 16);
  uint64_t* bbar = reinterpret_cast<uint64_t*>(sm + S::OFF_BAR + 24);   // [2]: B tile buffers (IMG)
  int* babort = reinterpret_cast<int*>(sm + S::OFF_BAR + 40);          // a B wait gave up (IMG)
  auto b_buf = [&](int buf) { return sm + 2 * S::T_A + buf * 2 * S::T_B; };   // hi, then lo
  float* dbred = reinterpret_cast<float*>(sm + S::OFF_DB);      // [NDB][128]
  constexpr bool AK = A_T == 0, BK = B_T == 1;   // K-major operand tiles
  constexpr uint32_t IDESC = make_idesc_bf16(BMT, BNT, AK ? 0 : 1, BK ? 0 : 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.y * BMT, n0 = (int64_t)blockIdx.x * BNT;
  int64_t kbeg = 0, kend = a.K;
  if (a.ksplit > 1) {
    int64_t kc = (a.K + a.ksplit - 1) / a.ksplit;
    kc = (kc + BKT - 1) / BKT * BKT;
    kbeg = std::min<int64_t>(a.K, (int64_t)blockIdx.z * kc);
    kend = std::min<int64_t>(a.K, kbeg + kc);
  }
  const int nkc = (int)((kend - kbeg + BKT - 1) / BKT);
  auto raw_a = [&](int kc) { return reinterpret_cast<float*>(sm + S::OFF_RAW + (kc % S::NRAW) * S::RAW_STAGE); };
  auto raw_b = [&](int kc) { return raw_a(kc) + S::RAW_A / 4; };
  const RawCopier<BMT, AK> cpa(a.A, m0, a.M);
  const RawCopier<BNT, BK> cpb(a.B, n0, a.N);
  auto issue = [&](int kc) {
    if (kc < nkc) {
      const int64_t k0 = kbeg + (int64_t)kc * BKT;
      cpa.copy(raw_a(kc), a.A, k0, kend);
      if constexpr (!IMG) cpb.copy(raw_b(kc), a.B, k0, kend);
    }
    cp_async_commit();   // empty groups keep the group count uniform
  };
  // IMG, thread 0: the hi and lo tiles of chunk kc (its 64-column blocks are
  // contiguous in the image) into buffer kc & 1
  const int64_t nb0 = (int64_t)blockIdx.x * (BNT / 64);
  bool b_pend[2] = {false, false};   // thread 0: a copy into the buffer not yet waited for
  int b_last[2] = {0, 0};            // thread 0: the chunk last copied into the buffer
  auto issue_b = [&](int kc) {
    const int buf = kc & 1;
    const char* src = a.b_img + ((int64_t)kc * a.b_img_nb + nb0) * 8192;
    mbar_expect_tx_bytes(&bbar[buf], 2 * S::T_B);
    bulk_copy_g2s(b_buf(buf), src, S::T_B, &bbar[buf]);
    bulk_copy_g2s(b_buf(buf) + S::T_B, src + a.b_img_part, S::T_B, &bbar[buf]);
    b_pend[buf] = true;
    b_last[buf] = kc;
  };

  // raw chunks in flight while the TMEM and barrier set-up runs
#pragma unroll
  for (int p = 0; p < S::NRAW - 1; ++p) issue(p);
  if (warp == 0) tmem_alloc(tmem_s, BNT);
  if (tid == 0) {
    mbar_init(bar, 1);
    if constexpr (IMG) {
      mbar_init(&bbar[0], 1);
      mbar_init(&bbar[1], 1);
      *babort = 0;
    }
    fence_mbar_init();
    if constexpr (IMG) {
      if (nkc > 0) issue_b(0);
      if (nkc > 1) issue_b(1);
    }
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_s;
  // db of a weight gradient: A^T chunks are MN-major, each thread keeps the
  // sums of its 8 columns (first column tile only)
  const bool do_db = A_T == 1 && a.db != nullptr && blockIdx.x == 0;
  float colsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};

  uint32_t ph = 0;
  bool pending = false;   // a commit on bar not yet waited for
  bool ok = true;
#pragma unroll 1
  for (int kc = 0; kc < nkc; ++kc) {
    issue(kc + S::NRAW - 1);
    cp_async_wait<S::NRAW - 1>();   // this thread's copies of chunk kc have landed
    if (pending) {                  // the previous chunk's MMAs have released the tiles
      if (!(ok = wait_all(bar, ph))) break;
      ph ^= 1u;
      pending = false;
      fence_after_sync();
      if constexpr (IMG) {
        if (*babort) {              // set before the commit waited for above: the same in every thread
          ok = false;
          break;
        }
        if (tid == 0 && kc + 1 < nkc) issue_b(kc + 1);   // its buffer's last reader has completed
      }
    } else {
      __syncthreads();
    }
    split_raw<BMT, AK>(raw_a(kc), a_hi, a_lo, do_db ? colsum : nullptr);
    if constexpr (!IMG) split_raw<BNT, BK>(raw_b(kc), b_hi, b_lo, nullptr);
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();   // tiles complete; raw chunk kc free for chunk kc + NRAW
    fence_after_sync();
    if (tid == 0) {
      bool go = true;
      const char* bh = b_hi;
      const char* bl = b_lo;
      if constexpr (IMG) {
        const int buf = kc & 1;
        go = mbar_wait(&bbar[buf], (uint32_t)((kc >> 1) & 1));
        if (go) b_pend[buf] = false; else *babort = 1;
        bh = b_buf(buf);
        bl = bh + S::T_B;
      }
      if (go) {
#pragma unroll
        for (int kk = 0; kk < BKT / 16; ++kk) {
          mma_bf16(tmem, tdesc(a_hi, AK, kk), tdesc(bh, BK, kk), IDESC, (kc > 0 || kk > 0) ? 1u : 0u);
          mma_bf16(tmem, tdesc(a_hi, AK, kk), tdesc(bl, BK, kk), IDESC, 1u);
          mma_bf16(tmem, tdesc(a_lo, AK, kk), tdesc(bh, BK, kk), IDESC, 1u);
        }
      }
      mma_commit(bar);
    }
    pending = true;
  }
  cp_async_wait<0>();
  if (ok && pending) {
    ok = wait_all(bar, ph);
    if (ok) pending = false;
  }
  if constexpr (IMG) {
    if (ok && *babort) ok = false;
  }
  if (!ok) {
    if (tid == 0) {
      atomicAdd(&g_node_tc_timeouts, 1);
      if (pending) mbar_wait(bar, ph);
      if constexpr (IMG) {   // no bulk copy may still be landing when the CTA leaves
#pragma unroll
        for (int b = 0; b < 2; ++b)
          if (b_pend[b]) mbar_wait(&bbar[b], (uint32_t)((b_last[b] >> 1) & 1));
      }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, BNT);
    return;
  }
  fence_after_sync();

  // ---- db partials: NDB threads per 8-column group, added in fixed order
  if (do_db) {
    const int cg = tid & 15, j = tid >> 4;
#pragma unroll
    for (int t = 0; t < 8; ++t) dbred[j * BMT + cg * 8 + t] = colsum[t];
  }
  __syncthreads();
  if (do_db && tid < BMT) {
    float sum = 0.f;
    for (int j = 0; j < NDB; ++j) sum += dbred[j * BMT + tid];
    const int64_t m = m0 + tid;
    if (m < a.M) {
      if (a.ksplit > 1) a.db_part[(int64_t)blockIdx.z * a.M + m] = sum;
      else a.db[m] = sum;
    }
  }

  // ---- epilogue.  1: warp w moves TMEM lanes 32 (w % 4) .. (rows), column
  // quarter w / 4, into an fp32 staging tile over the (idle) raw ring.
  constexpr int NCW = BNT / 4;       // 64, 32 or 16 columns per warp
  constexpr int LDO = BNT + 4;       // staging row stride: 65, 33 or 17 16-byte words (odd)
  // the staging tile (128 x LDO floats) lies over the idle raw ring, or for
  // 256-column tiles over the operand tiles and the raw ring together
  float* ostage = reinterpret_cast<float*>(sm + (BNT == 256 ? 0 : S::OFF_RAW));
  static_assert((BNT == 256 ? 0 : S::OFF_RAW) + BMT * LDO * 4 <= S::OFF_BAR, "staging fits");
  {
    const int q = warp & 3, h = warp >> 2;
#pragma unroll 1
    for (int part = 0; part < (NCW > 32 ? NCW / 32 : 1); ++part) {
      constexpr int W = NCW > 32 ? 32 : NCW;
      float v[W];
      if constexpr (W == 32) tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + h * NCW + part * 32, v);
      else tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + h * NCW, v);
      if (nkc == 0) {   // empty K slice of a split: the accumulator was never written
#pragma unroll
        for (int t = 0; t < W; ++t) v[t] = 0.f;
      }
      float* dst = ostage + (q * 32 + lane) * LDO + h * NCW + part * 32;
#pragma unroll
      for (int t = 0; t < W; t += 4) *reinterpret_cast<float4*>(dst + t) = make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, BNT);
  // 2: whole rows out.  Thread -> (row, 4-column word), consecutive threads on
  // consecutive words of a row, so every global access of a warp is one
  // contiguous run; UR rows per thread have their operand loads in flight together.
  constexpr int G4 = BNT / 4, RPP = NTH / G4, UR = 4;
  const int cw = tid % G4, rr = tid / G4;
  const int64_t n = n0 + 4 * cw;
  const bool nin = n < a.N, nvec = a.vec && n + 3 < a.N;
  float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
  if (a.ksplit <= 1 && a.bias && nvec) bb = *reinterpret_cast<const float4*>(a.bias + n);
#pragma unroll 1
  for (int rb = 0; rb < BMT; rb += RPP * UR) {
    float4 acc[UR], aux[UR], rs[UR];
    int64_t mr[UR];
#pragma unroll
    for (int u = 0; u < UR; ++u) {
      const int row = rb + u * RPP + rr;
      mr[u] = m0 + row;
      acc[u] = *reinterpret_cast<const float4*>(ostage + row * LDO + 4 * cw);
      const bool live = nvec && mr[u] < a.M && a.ksplit <= 1;
      if (live && a.act == ACT_DSILU) aux[u] = *reinterpret_cast<const float4*>(a.aux + mr[u] * a.ldaux + n);
      if (live && a.resid && n < a.resid_cols) rs[u] = *reinterpret_cast<const float4*>(a.resid + mr[u] * a.ldr + n);
    }
#pragma unroll
    for (int u = 0; u < UR; ++u) {
      const int64_t m = mr[u];
      if (m >= a.M || !nin) continue;
      if (a.ksplit > 1) {   // raw split-K slice (N % 4 == 0 on this path)
        *reinterpret_cast<float4*>(a.part + (int64_t)blockIdx.z * a.M * a.N + m * a.N + n) = acc[u];
        continue;
      }
      if (nvec) {
        float y[4] = {acc[u].x + bb.x, acc[u].y + bb.y, acc[u].z + bb.z, acc[u].w + bb.w};
        if (a.pre) *reinterpret_cast<float4*>(a.pre + m * a.ldp + n) = make_float4(y[0], y[1], y[2], y[3]);
        if (a.act == ACT_SILU) {
#pragma unroll
          for (int t = 0; t < 4; ++t) y[t] = silu_fast(y[t]);
        } else if (a.act == ACT_DSILU) {
          const float z[4] = {aux[u].x, aux[u].y, aux[u].z, aux[u].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float yy, d;
            silu_grad_fast(z[t], yy, d);
            y[t] *= d;
          }
        }
        if (a.resid && n < a.resid_cols) { y[0] += rs[u].x; y[1] += rs[u].y; y[2] += rs[u].z; y[3] += rs[u].w; }
        *reinterpret_cast<float4*>(a.C + m * a.ldc + n) = make_float4(y[0], y[1], y[2], y[3]);
      } else {
        const float yv[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int64_t nn = n + t;
          if (nn >= a.N) continue;
          float y = yv[t];
          if (a.bias) y += a.bias[nn];
          if (a.pre) a.pre[m * a.ldp + nn] = y;
          if (a.act == ACT_SILU) {
            y = silu_fast(y);
          } else if (a.act == ACT_DSILU) {
            float yy, d;
            silu_grad_fast(a.aux[m * a.ldaux + nn], yy, d);
            y *= d;
          }
          if (a.resid && nn < a.resid_cols) y += a.resid[m * a.ldr + nn];
          a.C[m * a.ldc + nn] = y;
        }
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Words of 4 consecutive elements along the contiguous dimension must be
// 16-byte aligned and never straddle a split; runs of 8 along the tile
// columns need that extent to be a multiple of 8.
bool words_ok(const Mat& X, int64_t contiguous_extent) {
  if (contiguous_extent % 8 || !aligned16(X.p0) || X.ld0 % 4) return false;
  if (X.p1 && (!aligned16(X.p1) || X.ld1 % 4 || (!X.split_rows && X.split % 4))) return false;
  return true;
}

template <int A_T, int B_T, int BNT, bool IMG = false>
int launch_t(const GemmArgs& a, cudaStream_t s) {
  static uint64_t attr_set = 0;
  constexpr size_t bytes = TcShape<BNT, IMG>::SMEM_BYTES;
  static_assert(bytes <= 232448, "shared memory per CTA");
  const uint64_t bit = device_bit();
  if (!(attr_set & bit)) {
    EGNN_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<A_T, B_T, BNT, IMG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    attr_set |= bit;
  }
  const unsigned z = (unsigned)(a.ksplit > 1 ? a.ksplit : 1);
  const dim3 grid((unsigned)((a.N + BNT - 1) / BNT), (unsigned)((a.M + BMT - 1) / BMT), z);
  TimerScope ts(A_T == 1 ? "node_wgrad" : "node_gemm", s);   // weight gradients: the side streams
  EGNN_CHECK_CUDA(launch_pdl(gemm_tc_kernel<A_T, B_T, BNT, IMG>, grid, dim3(NTH), bytes, s, a));
  EGNN_CHECK_LAUNCH();
  return EGNN_OK;
}

// One CTA per SM: 64-column tiles while twice the CTAs still fit in one wave;
// 256-column tiles when 128-column tiles would need a second wave and
// 256-column ones do not (data GEMMs only: their K is short, so the one-deep
// raw ring of that shape costs less than the second wave); else 128.
template <int A_T, int B_T>
int launch_ab(const GemmArgs& a, cudaStream_t s) {
  const int64_t z = a.ksplit > 1 ? a.ksplit : 1;
  const int64_t rows = (a.M + BMT - 1) / BMT;
  const int64_t tiles128 = (a.N + 127) / 128 * rows * z;
  const int64_t tiles256 = (a.N + 255) / 256 * rows * z;
  const int sms = num_sms_current();
  if (2 * tiles128 <= sms) return launch_t<A_T, B_T, 64>(a, s);
  if (A_T == 0 && z == 1 && a.N > 128 && tiles128 > sms && tiles256 <= sms) return launch_t<A_T, B_T, 256>(a, s);
  return launch_t<A_T, B_T, 128>(a, s);
}

}  // namespace

bool gemm_tc_ok(const GemmArgs& a) {
  if (a.round_bf16 || a.K <= 0) return false;
  // A: row-major needs K-words (K % 8), the transposed form needs M-words
  if (a.A.split_rows || !words_ok(a.A, a.a_t == 0 ? a.K : a.M)) return false;
  // B: W[n][k] needs K-words; X[k][n] needs N-words
  if (a.B.split_rows || !words_ok(a.B, a.b_t == 1 ? a.K : a.N)) return false;
  if (a.ksplit > 1 && a.N % 4) return false;
  return true;
}

int gemm_tc(const GemmArgs& a_in, cudaStream_t s) {
  if (a_in.M <= 0 || a_in.N <= 0) return EGNN_OK;
  if (!gemm_tc_ok(a_in)) return fail(EGNN_ERR_UNSUPPORTED, "gemm_tc: operand layout not supported");
  GemmArgs a = a_in;
  a.vec = (a.N % 4 == 0 && a.ldc % 4 == 0 && aligned16(a.C) && (!a.bias || aligned16(a.bias)) &&
           (!a.pre || (a.ldp % 4 == 0 && aligned16(a.pre))) &&
           (a.act != ACT_DSILU || (a.ldaux % 4 == 0 && aligned16(a.aux))) &&
           (!a.resid || (a.ldr % 4 == 0 && aligned16(a.resid) &&
                         (a.resid_cols == INT64_MAX || a.resid_cols % 4 == 0)))) ? 1 : 0;
  if (a.b_img && a.a_t == 0 && a.b_t == 0 && a.ksplit <= 1) {
    // B from its prepared image; tile width chosen as in launch_ab
    const int64_t rows = (a.M + BMT - 1) / BMT;
    const int64_t tiles128 = (a.N + 127) / 128 * rows, tiles256 = (a.N + 255) / 256 * rows;
    const int sms = num_sms_current();
    if (2 * tiles128 <= sms) EGNN_TRY((launch_t<0, 0, 64, true>(a, s)));
    else if (a.N > 128 && tiles128 > sms && tiles256 <= sms) EGNN_TRY((launch_t<0, 0, 256, true>(a, s)));
    else EGNN_TRY((launch_t<0, 0, 128, true>(a, s)));
    return EGNN_OK;
  }
  if (a.a_t == 0 && a.b_t == 0) EGNN_TRY((launch_ab<0, 0>(a, s)));
  else if (a.a_t == 0 && a.b_t == 1) EGNN_TRY((launch_ab<0, 1>(a, s)));
  else if (a.a_t == 1 && a.b_t == 0) EGNN_TRY((launch_ab<1, 0>(a, s)));
  else EGNN_TRY((launch_ab<1, 1>(a, s)));
  if (a.ksplit > 1) EGNN_TRY(gemm_reduce(a, s));
  return EGNN_OK;
}

int64_t wgrad_tc_splits(int64_t R, int64_t M, int64_t N) {
  const int64_t tiles = std::max<int64_t>(1, ((M + 127) / 128) * ((N + 127) / 128));
  const int64_t chunks = (R + 63) / 64;
  return std::max<int64_t>(1, std::min<int64_t>({148 / tiles, chunks / 2, 64}));
}

int wgrad_tc(int64_t R, int64_t M, int64_t N, Mat G, Mat X, float* dW, int64_t lddw, float* db, float* part,
             cudaStream_t s) {
  GemmArgs a;
  a.M = M; a.N = N; a.K = R;
  a.A = G; a.a_t = 1;
  a.B = X; a.b_t = 0;
  a.C = dW; a.ldc = lddw;
  // about one wave of 128 x 128 tiles, at least 2 chunks of 64 rows per
  // split, and no empty splits
  const int64_t chunks = (R + 63) / 64;
  const int64_t cap = wgrad_tc_splits(R, M, N);
  const int64_t per = (chunks + cap - 1) / cap;
  a.ksplit = (int)std::max<int64_t>(1, (chunks + per - 1) / per);
  a.part = a.ksplit > 1 ? part : nullptr;
  if (!gemm_tc_ok(a)) return wgrad(R, M, N, G, X, dW, lddw, db, 0, part, s);
  a.db = db;
  a.db_part = (db && a.ksplit > 1) ? part + (int64_t)a.ksplit * M * N : nullptr;
  return gemm_tc(a, s);
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
