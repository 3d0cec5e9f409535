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
//  * no split-K: k is never partitioned, so no cell is reassociated.
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

// Launch `ntiles` parent tiles starting at tile_base, each as (128/BM)^2 CTAs.
template <int BM, int BN, int BK, int STAGES, bool kVec>
int launch_cfg(cudaStream_t s, const float* A, const float* B, float* C, uint64_t M, uint64_t N,
               uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed, int tile_base, int ntiles,
               int tiles_n0, int acc_from_c) {
  using G = Cfg<BM, BN, BK, 8, 8, STAGES>;
  auto kern = mm_strict_kernel<BM, BN, BK, 8, 8, STAGES, kVec>;
  static uint64_t attr_set = 0;  // per template instance, one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::kSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(mm_strict)");
    attr_set |= 1ull << dev;
  }
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
                    uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed, int acc_from_c) {
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
  // (128 x 112 tiles, 37 per 4144 columns so that four row bands fill 148
  // SMs, were measured too: with this kernel a wave of them takes as long as
  // a wave of 128 x 128 tiles, so they never beat the plan above.)
  const int full = split ? waves * sms : tiles;
  MAPAL_TRY((launch_cfg<128, 128, 64, 2, kVec>(s, A, B, C, M, N, K, lda, ldb, ldc, seed, 0, full, tiles_n0,
                                                acc_from_c)));
  return launch_cfg<64, 64, 16, 4, kVec>(s, A, B, C, M, N, K, lda, ldb, ldc, seed, full, tiles - full,
                                         tiles_n0, acc_from_c);
}

}  // namespace

// The whole site as whole waves of 128 x 128 tiles plus a remainder in
// 64 x 64 tiles. With acc_from_c, cells continue from the partial folds
// stored in C (used to split K into ranges that overlap a B broadcast).
int launch_matmul_strict_ex(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                            uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed,
                            int acc_from_c) {
  if (M > 0x7fffffffull || N > 0x7fffffffull || K > 0x7fffffffull) return MAPAL_ERR_UNSUPPORTED;
  if ((M + 127) / 128 * ((N + 127) / 128) > 0x7fffffffull / 4) return MAPAL_ERR_UNSUPPORTED;
  const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && lda % 4 == 0 && ldb % 4 == 0 &&
                   ldc % 4 == 0;
  return vec ? launch_balanced<true>(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, acc_from_c)
             : launch_balanced<false>(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, acc_from_c);
}

int launch_matmul_strict(cudaStream_t s, int sms, const float* A, const float* B, float* C, uint64_t M,
                         uint64_t N, uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed) {
  return launch_matmul_strict_ex(s, sms, A, B, C, M, N, K, lda, ldb, ldc, seed, 0);
}
