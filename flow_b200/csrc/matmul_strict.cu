// matmul_strict.cu — the matmul tile site, bit-identical to the interpreter.
//
// Site: `ta -> map { t -> (0.0, k) -> fold { acc, k -> acc + a[i*K + k] * b[k*N + j] } }`
// (benches/matmul/matmul1024_cap_f32.mapal:7-11; TileSite rows=M, c=N, k=K,
// a{ci=K, ck=1}, b{ck=N, clane=1}, crates/mapal-ir/src/algo.rs:335-345). The
// interpreter folds each cell from +0.0 with one rounded multiply and one
// rounded add per k, k ascending (crates/mapal-interp/src/eval.rs:326-359).
// Reordering or fusing any of those breaks bit-equality, so this kernel keeps
// every cell's chain intact and gets its speed from reuse and issue density:
//
//  * a CTA computes a BM x BN block of C; A and B panels stream through a
//    multi-stage cp.async ring in shared memory, so each global value is read
//    once per CTA instead of once per cell (rung 0 reads 2K values per cell);
//  * each thread owns TM x TN cells in registers and walks k in steps of 4:
//    one 128-bit load brings 4 k-values of an A row, one brings 4 columns of
//    a B row;
//  * two neighbouring cells advance together: one packed FMA with a -0.0
//    addend passed in at run time forms both rounded products, one packed
//    add accumulates them (2 issue slots per 2 MACs; f32x2.cuh gives the
//    argument that this is bit-identical to a rounded multiply then a
//    rounded add), leaving issue slots for the loads so the FP32 pipe, not
//    issue, is the bound;
//  * no split-K: k is never partitioned, so no cell is reassociated;
//  * the launch plan covers the site with whole waves of 128 x 128 tiles and
//    a remainder of 64 x 64 tiles, or with 128 x 112 tiles where 148 = 4 x 37
//    SMs leave the 128-wide plan a part-filled wave (row blocks of 512 or
//    1024 rows and 4096 columns, as a row-sharded 4096^2 site gives each GPU).
//
// The roofline is the FP32 pipe at one operation per lane per clock
// (148 SMs x 128 lanes), i.e. half the FFMA-counted peak: a strict MAC is two
// operations where an FMA would be one.
#include "common.cuh"
#include "f32x2.cuh"

namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(pred ? 16 : 0));
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 4 : 0));
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Copy 4 consecutive floats src[0..3] (valid ones: src[0..nvalid)) to dst.
// Full, aligned groups go as one 16-byte copy; a ragged edge goes per float,
// zero-filling the rest (zero-filled values are never used by a cell).
template <bool kVec>
__device__ __forceinline__ void copy4(uint32_t dst, const float* src, int nvalid) {
  if (kVec && nvalid >= 4) {
    cp_async16(dst, src, true);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) cp_async4(dst + 4 * e, nvalid > e ? src + e : src, nvalid > e);
  }
}

template <int BM, int BN, int BK, int TM, int TN, int STAGES>
struct Cfg {
  static constexpr int kThreadsM = BM / TM, kThreadsN = BN / TN;
  static constexpr int kThreads = kThreadsM * kThreadsN;
  static constexpr int kApad = 4, kBpad = 4;
  static constexpr int kAStride = BK + kApad;  // floats per A row in smem
  static constexpr int kBStride = BN + kBpad;  // floats per B row in smem
  static constexpr int kAStage = BM * kAStride, kBStage = BK * kBStride;
  static constexpr size_t kSmem = sizeof(float) * (size_t)STAGES * (kAStage + kBStage);
  static_assert(TM == 8 && TN == 8, "thread tile is 8x8: two 4x4 quadrants");
  static_assert(BK % 4 == 0, "k advances in steps of 4");
};

// Work is laid out on a grid of parent tiles of 128 rows and BN*split
// columns (tiles_m x tiles_n0 of them), split = 128/BM. A CTA covers one
// split^2-th of a parent tile: CTA u takes sub-tile u % split^2 of parent
// tile tile_base + u / split^2. Parent tiles are numbered in groups of
// kGroupRows tile rows, column-major inside a group, so the CTAs of one wave
// share a few row panels of A and a band of B's columns (at N = 16384 a
// row-major wave would stream all of B through L2 once per wave).
// With acc_from_c the cells start from the values already in C (a partial
// fold carried over from an earlier k range, bit-exact because the carried
// accumulator is the same f32 value) instead of from the seed.
constexpr int kGroupRows = 8;

template <int BM, int BN, int BK, int TM, int TN, int STAGES, bool kVec>
__global__ void __launch_bounds__(Cfg<BM, BN, BK, TM, TN, STAGES>::kThreads, 1)
    mm_strict_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                     int M, int N, int K, long long lda, long long ldb, long long ldc, float seed,
                     int tile_base, int tiles_m, int tiles_n0, int acc_from_c, float neg_zero) {
  using G = Cfg<BM, BN, BK, TM, TN, STAGES>;
  const f2 z2 = f2_splat(neg_zero);  // -0.0, unknown to the compiler: see f2_mac_z
  extern __shared__ __align__(16) float smem[];
  float* As = smem;                              // [STAGES][BM][kAStride]
  float* Bs = smem + STAGES * G::kAStage;        // [STAGES][BK][kBStride]

  const int tid = threadIdx.x;
  const int tx = tid % G::kThreadsN, ty = tid / G::kThreadsN;
  constexpr int kSplit = 128 / BM;
  static_assert(128 % BM == 0, "CTA rows divide the 128-row parent tile");
  const int parent = tile_base + (int)blockIdx.x / (kSplit * kSplit);
  const int sub = (int)blockIdx.x % (kSplit * kSplit);
  const int per_group = kGroupRows * tiles_n0;
  const int grp = parent / per_group, in_grp = parent % per_group;
  const int grp_rows = tiles_m - grp * kGroupRows < kGroupRows ? tiles_m - grp * kGroupRows : kGroupRows;
  const int pm = grp * kGroupRows + in_grp % grp_rows, pn = in_grp / grp_rows;
  const int m0 = pm * (BM * kSplit) + (sub / kSplit) * BM;
  const int n0 = pn * (BN * kSplit) + (sub % kSplit) * BN;
  const int KT = (K + BK - 1) / BK;

  // Loader coordinates: A tile BM x BK in 16-byte groups, B tile BK x BN.
  constexpr int kAGroups = BM * BK / 4, kBGroups = BK * BN / 4;

  auto load_tile = [&](int kt, int stage) {
    const int k0 = kt * BK;
    float* as = As + stage * G::kAStage;
    float* bs = Bs + stage * G::kBStage;
#pragma unroll
    for (int g = tid; g < kAGroups; g += G::kThreads) {
      const int row = g / (BK / 4), kq = g % (BK / 4);
      const int m = m0 + row, k = k0 + kq * 4;
      const int nvalid = (m < M) ? min(4, K - k) : 0;
      copy4<kVec>(smem_u32(as + row * G::kAStride + kq * 4), A + (long long)(m < M ? m : 0) * lda + (nvalid > 0 ? k : 0), nvalid);
    }
#pragma unroll
    for (int g = tid; g < kBGroups; g += G::kThreads) {
      const int kr = g / (BN / 4), nq = g % (BN / 4);
      const int k = k0 + kr, n = n0 + nq * 4;
      const int nvalid = (k < K) ? min(4, N - n) : 0;
      copy4<kVec>(smem_u32(bs + kr * G::kBStride + nq * 4), B + (long long)(k < K ? k : 0) * ldb + (nvalid > 0 ? n : 0), nvalid);
    }
  };

  // acc[i][q]: cells (row_i, cols 2q, 2q+1 of this thread's 8 columns).
  f2 acc[TM][TN / 2];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int q = 0; q < TN / 2; ++q) acc[i][q] = s2;

  // Row i of the thread tile: quadrant rows ty*4 + i (i < 4) and BM/2 + ty*4 + i-4.
  auto a_row = [&](int i) { return (i < 4 ? 0 : BM / 2) + ty * 4 + (i & 3); };

  if (acc_from_c) {
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int m = m0 + a_row(i);
#pragma unroll
      for (int q = 0; q < TN / 2; ++q) {
        const int n = n0 + (q < 2 ? 0 : BN / 2) + tx * 4 + 2 * (q & 1);
        const float* cp = C + (long long)(m < M ? m : 0) * ldc;
        const float lo = (m < M && n < N) ? cp[n] : 0.0f;
        const float hi = (m < M && n + 1 < N) ? cp[n + 1] : 0.0f;
        acc[i][q] = f2_pack(lo, hi);
      }
    }
  }

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < KT) load_tile(s, s);
    cp_commit();
  }

  for (int kt = 0; kt < KT; ++kt) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    {
      const int nt = kt + STAGES - 1;
      if (nt < KT) load_tile(nt, nt % STAGES);
      cp_commit();
    }
    const float* as = As + (kt % STAGES) * G::kAStage;
    const float* bs = Bs + (kt % STAGES) * G::kBStage;
    const int kvalid = min(BK, K - kt * BK);
    if (kvalid == BK) {
#pragma unroll
      for (int kq = 0; kq < BK / 4; ++kq) {
        float4 a[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i)
          a[i] = *reinterpret_cast<const float4*>(as + a_row(i) * G::kAStride + kq * 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float* brow = bs + (kq * 4 + kk) * G::kBStride;
          const float4 b0 = *reinterpret_cast<const float4*>(brow + tx * 4);
          const float4 b1 = *reinterpret_cast<const float4*>(brow + BN / 2 + tx * 4);
          const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
          for (int i = 0; i < TM; ++i) {
            const float av = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][q] = f2_mac_z(acc[i][q], f2_splat(av), f2_pack(bv[2 * q], bv[2 * q + 1]), z2);
          }
        }
      }
    } else {
      // Ragged last k-tile: exactly kvalid steps, still in ascending k.
      for (int kk = 0; kk < kvalid; ++kk) {
        const float* brow = bs + kk * G::kBStride;
        const float4 b0 = *reinterpret_cast<const float4*>(brow + tx * 4);
        const float4 b1 = *reinterpret_cast<const float4*>(brow + BN / 2 + tx * 4);
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float av = as[a_row(i) * G::kAStride + kk];
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[i][q] = f2_mac_z(acc[i][q], f2_splat(av), f2_pack(bv[2 * q], bv[2 * q + 1]), z2);
        }
      }
    }
  }
  cp_wait<0>();

  // Epilogue: each row's 8 cells are two runs of 4 columns.
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + a_row(i);
    if (m >= M) continue;
    float* crow = C + (long long)m * ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + h * (BN / 2) + tx * 4;
      const float v[4] = {f2_lo(acc[i][2 * h]), f2_hi(acc[i][2 * h]), f2_lo(acc[i][2 * h + 1]),
                          f2_hi(acc[i][2 * h + 1])};
      if (kVec && n + 3 < N) {
        *reinterpret_cast<float4*>(crow + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n + e < N) crow[n + e] = v[e];
      }
    }
  }
}

// 128 x 112 tiles. 148 SMs = 4 x 37 and 37 x 112 = 4144, so a block of
// 128·r rows and up to 4144 columns is r/4 waves with no partly empty wave
// (512 x 4096 is exactly one), where 128 x 128 tiles leave 20 of 148 SMs idle
// or run a part-filled extra wave. The threads stay 256 (8 warps, two per
// scheduler, as in the 128 x 128 kernel: 224 threads leave one scheduler with
// a single warp and run no faster than 128 x 128), laid out 32 x 8, each
// owning 4 rows x 14 columns: rows ty + 32i and columns 4tx .. 4tx+3,
// 32 + 4tx .., 64 + 4tx .. and 96 + 2tx, 96 + 2tx+1 of the tile. So a warp's
// B reads are three 128-byte and one 64-byte run per k, its A reads four
// consecutive rows, and the 14 columns pair into 7 packed cells per row.
// Every cell keeps its own chain: seed (or C), then one rounded product and
// one rounded add per k, k ascending.
constexpr int kNBM = 128, kNBN = 112, kNBK = 64, kNStages = 2, kNThreads = 256;
constexpr int kNAStride = kNBK + 4, kNBStride = kNBN + 4;
constexpr int kNAStage = kNBM * kNAStride, kNBStage = kNBK * kNBStride;
constexpr size_t kNSmem = sizeof(float) * (size_t)kNStages * (kNAStage + kNBStage);
static_assert((kNBM * kNBK / 4) % kNThreads == 0 && (kNBK * kNBN / 4) % kNThreads == 0, "whole loader trips");

template <bool kVec>
__global__ void __launch_bounds__(kNThreads, 1)
    mm_strict_n112_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M,
                          int N, int K, long long lda, long long ldb, long long ldc, float seed, int tile_base,
                          int tiles_m, int tiles_n0, int acc_from_c, float neg_zero) {
  const f2 z2 = f2_splat(neg_zero);  // -0.0, unknown to the compiler: see f2_mac_z
  extern __shared__ __align__(16) float smem[];
  float* As = smem;                          // [kNStages][128][kNAStride]
  float* Bs = smem + kNStages * kNAStage;    // [kNStages][64][kNBStride]

  const int tid = threadIdx.x;
  const int tx = tid % 8, ty = tid / 8;
  const int parent = tile_base + (int)blockIdx.x;
  const int per_group = kGroupRows * tiles_n0;
  const int grp = parent / per_group, in_grp = parent % per_group;
  const int grp_rows = tiles_m - grp * kGroupRows < kGroupRows ? tiles_m - grp * kGroupRows : kGroupRows;
  const int pm = grp * kGroupRows + in_grp % grp_rows, pn = in_grp / grp_rows;
  const int m0 = pm * kNBM, n0 = pn * kNBN;
  const int KT = (K + kNBK - 1) / kNBK;

  auto load_tile = [&](int kt, int stage) {
    const int k0 = kt * kNBK;
    float* as = As + stage * kNAStage;
    float* bs = Bs + stage * kNBStage;
#pragma unroll
    for (int g = tid; g < kNBM * kNBK / 4; g += kNThreads) {
      const int row = g / (kNBK / 4), kq = g % (kNBK / 4);
      const int m = m0 + row, k = k0 + kq * 4;
      const int nvalid = (m < M) ? min(4, K - k) : 0;
      copy4<kVec>(smem_u32(as + row * kNAStride + kq * 4),
                  A + (long long)(m < M ? m : 0) * lda + (nvalid > 0 ? k : 0), nvalid);
    }
#pragma unroll
    for (int g = tid; g < kNBK * kNBN / 4; g += kNThreads) {
      const int kr = g / (kNBN / 4), nq = g % (kNBN / 4);
      const int k = k0 + kr, n = n0 + nq * 4;
      const int nvalid = (k < K) ? min(4, N - n) : 0;
      copy4<kVec>(smem_u32(bs + kr * kNBStride + nq * 4),
                  B + (long long)(k < K ? k : 0) * ldb + (nvalid > 0 ? n : 0), nvalid);
    }
  };

  // acc[i][q]: row ty + 32i; q = 0..5 the column pairs of the three 4-column
  // runs (4tx + 32·(q/2) + 2·(q%2)), q = 6 the pair at 96 + 2tx.
  f2 acc[4][7];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int q = 0; q < 7; ++q) acc[i][q] = s2;
  auto col = [&](int q) { return q < 6 ? 32 * (q >> 1) + 4 * tx + 2 * (q & 1) : 96 + 2 * tx; };

  if (acc_from_c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty + 32 * i;
      const float* cp = C + (long long)(m < M ? m : 0) * ldc;
#pragma unroll
      for (int q = 0; q < 7; ++q) {
        const int n = n0 + col(q);
        const float lo = (m < M && n < N) ? cp[n] : 0.0f;
        const float hi = (m < M && n + 1 < N) ? cp[n + 1] : 0.0f;
        acc[i][q] = f2_pack(lo, hi);
      }
    }
  }

#pragma unroll
  for (int s = 0; s < kNStages - 1; ++s) {
    if (s < KT) load_tile(s, s);
    cp_commit();
  }

  auto step = [&](const float (&av)[4], const float* brow) {
    const float4 b0 = *reinterpret_cast<const float4*>(brow + 4 * tx);
    const float4 b1 = *reinterpret_cast<const float4*>(brow + 32 + 4 * tx);
    const float4 b2 = *reinterpret_cast<const float4*>(brow + 64 + 4 * tx);
    const float2 b3 = *reinterpret_cast<const float2*>(brow + 96 + 2 * tx);
    const f2 bp[7] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y), f2_pack(b1.z, b1.w),
                      f2_pack(b2.x, b2.y), f2_pack(b2.z, b2.w), f2_pack(b3.x, b3.y)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const f2 a2 = f2_splat(av[i]);
#pragma unroll
      for (int q = 0; q < 7; ++q) acc[i][q] = f2_mac_z(acc[i][q], a2, bp[q], z2);
    }
  };

  for (int kt = 0; kt < KT; ++kt) {
    cp_wait<kNStages - 2>();
    __syncthreads();
    {
      const int nt = kt + kNStages - 1;
      if (nt < KT) load_tile(nt, nt % kNStages);
      cp_commit();
    }
    const float* as = As + (kt % kNStages) * kNAStage;
    const float* bs = Bs + (kt % kNStages) * kNBStage;
    const int kvalid = min(kNBK, K - kt * kNBK);
    if (kvalid == kNBK) {
#pragma unroll
      for (int kq = 0; kq < kNBK / 4; ++kq) {
        float4 a[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          a[i] = *reinterpret_cast<const float4*>(as + (ty + 32 * i) * kNAStride + kq * 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          float av[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) av[i] = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
          step(av, bs + (kq * 4 + kk) * kNBStride);
        }
      }
    } else {
      // Ragged last k-tile: exactly kvalid steps, still in ascending k.
      for (int kk = 0; kk < kvalid; ++kk) {
        float av[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = as[(ty + 32 * i) * kNAStride + kk];
        step(av, bs + kk * kNBStride);
      }
    }
  }
  cp_wait<0>();

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 32 * i;
    if (m >= M) continue;
    float* crow = C + (long long)m * ldc + n0;
    const int nl = N - n0;  // columns of this tile inside C
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int c = 32 * r + 4 * tx;
      const f2 p0 = acc[i][2 * r], p1 = acc[i][2 * r + 1];
      if (kVec && c + 3 < nl) {
        *reinterpret_cast<float4*>(crow + c) = make_float4(f2_lo(p0), f2_hi(p0), f2_lo(p1), f2_hi(p1));
      } else {
        const float v[4] = {f2_lo(p0), f2_hi(p0), f2_lo(p1), f2_hi(p1)};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (c + e < nl) crow[c + e] = v[e];
      }
    }
    const int c = 96 + 2 * tx;
    if (kVec && c + 1 < nl) {
      *reinterpret_cast<float2*>(crow + c) = make_float2(f2_lo(acc[i][6]), f2_hi(acc[i][6]));
    } else {
      if (c < nl) crow[c] = f2_lo(acc[i][6]);
      if (c + 1 < nl) crow[c + 1] = f2_hi(acc[i][6]);
    }
  }
}

// Launch `ntiles` parent tiles starting at tile_base, each as (128/BM)^2 CTAs.
template <int BM, int BN, int BK, int STAGES, bool kVec>
int launch_cfg(cudaStream_t s, const float* A, const float* B, float* C, uint64_t M, uint64_t N,
               uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed, int tile_base, int ntiles,
               int tiles_n0, int acc_from_c) {
  using G = Cfg<BM, BN, BK, 8, 8, STAGES>;
  auto kern = mm_strict_kernel<BM, BN, BK, 8, 8, STAGES, kVec>;
  static std::atomic<uint64_t> attr_set{0};  // per template instance, one bit per device
  int dev = 0;
  MAPAL_CUDA(cudaGetDevice(&dev));
  MAPAL_TRY(ensure_smem_attr(attr_set, (const void*)kern, dev, G::kSmem, "cudaFuncSetAttribute(mm_strict)"));
  constexpr int kSplit = 128 / BM;
  const unsigned grid = (unsigned)ntiles * kSplit * kSplit;
  if (grid == 0) return 0;
  kern<<<grid, G::kThreads, G::kSmem, s>>>(A, B, C, (int)M, (int)N, (int)K, (long long)lda, (long long)ldb,
                                           (long long)ldc, seed, tile_base, (int)((M + 127) / 128), tiles_n0,
                                           acc_from_c, -0.0f);
  count_launch();
  return 0;
}

template <bool kVec>
int launch_balanced(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M, uint64_t N,
                    uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed, int acc_from_c,
                    int beside_collective) {
  const int tiles_n0 = (int)((N + 127) / 128);
  const int tiles = (int)((M + 127) / 128) * tiles_n0;
  // Whole waves of 128 x 128 CTAs (one per SM). The leftover tiles would run
  // as a partly empty last wave; when they are few (at most two 64 x 64 CTAs
  // per SM after a four-way split) they go as 64 x 64 CTAs instead, which
  // finish in about 0.65 of a 128 x 128 wave. Measured on B200 at
  // N = K = 4096 for M = 256..4096: the split wins at M = 256 and 2048
  // (a remainder of 64 and 68 tiles) and loses at 512, 1024 and 4096
  // (128, 108 and 136 tiles), where three or four 64 x 64 CTAs per SM take
  // longer than the partial wave.
  const int waves = tiles / sms, rem = tiles - waves * sms;
  const bool split = rem > 0 && (4 * rem + sms - 1) / sms <= 2;
  const int full = split ? waves * sms : tiles;
  // The same site in 128 x 112 tiles costs ceil(tiles112 / sms) waves of
  // kN112Wave each: a 128 x 112 CTA does 7/8 of a 128 x 128 CTA's work and
  // was measured on B200 (N = K = 4096) at 0.905 of its time, 0.559 against
  // 0.615 ms for a 512-row block (one wave each) and 4.35 against 4.21 ms
  // for 4096 rows (8 waves against 7). It wins where the 128-wide plan ends
  // in a part-filled wave that the narrower tiles fill: 512, 1024 and 1536 x
  // 4096 blocks (0.91 / 1.82 / 2.73 against 1 / 2 / 3 waves; measured 9-10 %
  // faster); 2048 x 4096 is a tie (3.64 against 3.65) and 4096 x 4096 stays
  // on 128 x 128 tiles (7.28 against 7).
  // Beside an SM-based collective (an NCCL kernel launched on another stream
  // next to this multiply) the 128-wide plan stays when its part-filled wave
  // leaves the collective kCollectiveCtas SMs, its CTA cap: the narrower tiles
  // fill every SM in every wave, and the collective then waits for the
  // multiply's end. Measured with the row-sharded 4096^2 site's B broadcast
  // at 4 GPUs (1024-row blocks, 40 SMs free in the second wave): keeping the
  // 128-wide plan beside it took the step from 1.29 to 1.23 ms.
  const int free_sms = rem > 0 && !split ? sms - rem : 0;
  if (!(beside_collective && free_sms >= kCollectiveCtas)) {
    constexpr double kN112Wave = 0.91, kSplitWave = 0.65;
    const int tiles_n112 = (int)((N + kNBN - 1) / kNBN);
    const long long t112 = (long long)((M + 127) / 128) * tiles_n112;
    const double cost128 = waves + (rem == 0 ? 0.0 : split ? kSplitWave : 1.0);
    const double cost112 = (double)((t112 + sms - 1) / sms) * kN112Wave;
    if (cost112 < cost128 - 0.01 && t112 <= 0x7fffffffll) {
      auto kern = mm_strict_n112_kernel<kVec>;
      static std::atomic<uint64_t> attr_set{0};
      int dev = 0;
      MAPAL_CUDA(cudaGetDevice(&dev));
      MAPAL_TRY(ensure_smem_attr(attr_set, (const void*)kern, dev, kNSmem, "cudaFuncSetAttribute(mm_strict_n112)"));
      kern<<<(unsigned)t112, kNThreads, kNSmem, s>>>(A, B, C, (int)M, (int)N, (int)K, (long long)lda,
                                                     (long long)ldb, (long long)ldc, seed, 0,
                                                     (int)((M + 127) / 128), tiles_n112, acc_from_c, -0.0f);
      count_launch();
      return 0;
    }
  }
  MAPAL_TRY((launch_cfg<128, 128, 64, 2, kVec>(s, A, B, C, M, N, K, lda, ldb, ldc, seed, 0, full, tiles_n0,
                                                acc_from_c)));
  return launch_cfg<64, 64, 16, 4, kVec>(s, A, B, C, M, N, K, lda, ldb, ldc, seed, full, tiles - full,
                                         tiles_n0, acc_from_c);
}

}  // namespace

// The whole site in the plan launch_balanced picks. With acc_from_c, cells
// continue from the partial folds stored in C (used to split K into ranges
// that overlap a B transfer).
int launch_matmul_strict_ex(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                            uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed,
                            int acc_from_c, int beside_collective) {
  if (M > 0x7fffffffull || N > 0x7fffffffull || K > 0x7fffffffull) return MAPAL_ERR_UNSUPPORTED;
  if ((M + 127) / 128 * ((N + 127) / 128) > 0x7fffffffull / 4) return MAPAL_ERR_UNSUPPORTED;
  const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && lda % 4 == 0 && ldb % 4 == 0 &&
                   ldc % 4 == 0;
  return vec ? launch_balanced<true>(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, acc_from_c, beside_collective)
             : launch_balanced<false>(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, acc_from_c, beside_collective);
}

int launch_matmul_strict(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                         uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed) {
  return launch_matmul_strict_ex(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, 0, 0);
}
