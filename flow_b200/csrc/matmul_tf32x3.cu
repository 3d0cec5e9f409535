// matmul_tf32x3.cu — the opt-in tensor-core matmul: 3xTF32 on tcgen05.
//
// ADR-0032 (docs/decisions/ADR-0032-precision-contracts-vs-backend-config.md)
// puts a `tf32-class` precision contract beside `exact`: a matmul site may
// be evaluated on tensor cores when the program opts in, within a stated
// error. This is that path (MAPAL_MATMUL_TF32X3); the default strict path
// stays bit-exact.
//
// Each f32 operand is split into two TF32 values and C = A*B is accumulated
// in f32 as Ahi*Bhi + Ahi*Blo + Alo*Bhi (the dropped Alo*Blo is ~2^-20
// relative), into two TMEM accumulators that alternate by k-block.
//
//  * B -> BhiT, BloT (transposed to N x K, K-major; hi = rna(x),
//    lo = rna(x - hi)) by a split pass into the context arena;
//  * A, when TMA can read it in place and N <= 8192: raw tiles are the hi
//    operand (the tensor pipe truncates an f32 to TF32) and the GEMM writes
//    the lo tiles in shared memory (mm_tf32x3_fused_kernel); otherwise A is
//    split into the arena as well (mm_tf32x3_kernel);
//  * GEMM: one CTA per 128 x 256 tile of C, 192 threads in three roles:
//      warp 0  TMA producer: 2-D tiled loads per k-block (16 k, 64-byte
//              swizzle) into a 4-stage shared-memory ring, one mbarrier per
//              stage with the transaction byte count;
//      warp 1  allocates 512 TMEM columns (two 128 x 256 f32 accumulators;
//              even k-blocks go to the first, odd ones to the second) and
//              one lane issues tcgen05.mma kind::tf32 (M128 N256 K8): three
//              products per k-step, two k-steps per stage; tcgen05.commit
//              frees a stage when its MMAs have read it;
//      warps 2-5 (fused kernel: first convert each stage's A lo tile) then
//              the epilogue: wait for the final commit, tcgen05.ld both
//              accumulators (each warp its 32-lane quarter), add them and
//              the seed, store C.
//  * no cluster multicast anywhere: every CTA fetches its own tiles.
//
// Every wait is bounded: a wait that runs out sets the device flag to
// kDeviceTimeout (reported as MAPAL_ERR_TIMEOUT), all roles leave their
// loops, in-flight copies and MMAs are waited for (bounded again) and TMEM
// is freed before the CTA exits.
#include <cuda.h>

#include "common.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 16, STAGES = 4;
constexpr int kThreads = 192;
// Two 128 x 256 f32 accumulators: k-blocks alternate between them and the
// epilogue adds the pair once with a rounded f32 add. The tensor pipe's
// accumulation error grows with the number of additions into one
// accumulator, so two half-length chains roughly halve it.
constexpr uint32_t kAccCols = 256;
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr int kATile = BM * BK * 4;  // bytes of one A tile (hi or lo)
constexpr int kBTile = BN * BK * 4;  // bytes of one B tile (hi or lo)
constexpr int kStageBytes = 2 * kATile + 2 * kBTile;
constexpr uint32_t kDeviceTimeout = 0x100u;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a wait gives up after 2 s

struct Smem {
  // stage buffers first, each 1024-byte aligned (the swizzle pattern repeats
  // every 512 bytes for the 64-byte swizzle)
  uint8_t stage[STAGES][kStageBytes];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(sa(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on a phase: false when kWaitLimitNs ran out, or (abort given)
// when another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(b, parity)) return true;
    if ((i & 255) == 255) {
      if (abort && *abort) return false;
      if (now_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          sa(dst)),
      "l"(map), "r"(x), "r"(y), "r"(sa(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major, 64-byte swizzle: rows of 64 bytes
// (16 tf32), 8-row groups 512 bytes apart (SBO), LBO 16 bytes (unused for
// swizzled K-major), version 1 (sm_100), layout type 4 = SWIZZLE_64B.
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  uint64_t addr = sa(p);
  uint64_t d = 0;
  d |= (addr & 0x3FFFFull) >> 4;          // start address
  d |= (uint64_t)(16 >> 4) << 16;         // leading byte offset
  d |= (uint64_t)(512 >> 4) << 32;        // stride byte offset
  d |= 1ull << 46;                        // version
  d |= 4ull << 61;                        // SWIZZLE_64B
  return d;
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Tile numbering: groups of kGroupRows tile rows, column-major inside a group,
// so the CTAs of one wave share a few row panels of A and a band of B's
// columns instead of every column of B (fewer L2 misses at large N and K).
constexpr int kGroupRows = 8;
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = kGroupRows * tiles_n;
  const int g = tile / per_group, r = tile % per_group;
  const int rows = tiles_m - g * kGroupRows < kGroupRows ? tiles_m - g * kGroupRows : kGroupRows;
  tm = g * kGroupRows + r % rows;
  tn = r / rows;
}

__global__ void __launch_bounds__(kThreads, 1)
    mm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                     const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                     float* __restrict__ C, int M, int N, int K, long long ldc, float seed, unsigned* flag,
                     int tiles_m, int tiles_n, int tile_base, int nsplit, float* __restrict__ part_out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // CTA -> (tile, k part); tile -> (tile row, tile column) by tile_coords.
  const int tile = tile_base + (int)blockIdx.x / nsplit, part = (int)blockIdx.x % nsplit;
  int tm, tn;
  tile_coords(tile, tiles_m, tiles_n, tm, tn);
  const int m0 = tm * BM, n0 = tn * BN;
  const int KT = (K + BK - 1) / BK;
  const int kt_lo = (int)((long long)KT * part / nsplit), nkt = (int)((long long)KT * (part + 1) / nsplit) - kt_lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int issued = 0;
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES && !mbar_wait(&sm.empty[s], ((kt / STAGES) - 1) & 1, abort)) {
        *abort = 1;
        break;
      }
      uint8_t* st = sm.stage[s];
      mbar_expect_tx(&sm.full[s], kStageBytes);
      const int k0 = (kt_lo + kt) * BK;
      tma_load_2d(st, &map_ahi, k0, m0, &sm.full[s]);
      tma_load_2d(st + kATile, &map_alo, k0, m0, &sm.full[s]);
      tma_load_2d(st + 2 * kATile, &map_bhi, k0, n0, &sm.full[s]);
      tma_load_2d(st + 2 * kATile + kBTile, &map_blo, k0, n0, &sm.full[s]);
      ++issued;
    }
    if (*abort) {
      // Let the copies already issued land before the CTA can exit.
      for (int kt = (issued > STAGES ? issued - STAGES : 0); kt < issued; ++kt)
        mbar_wait(&sm.full[kt % STAGES], (kt / STAGES) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt % STAGES;
      if (!mbar_wait(&sm.full[s], (kt / STAGES) & 1, abort)) {
        *abort = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t* st = sm.stage[s];
      const uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
      const uint64_t bhi = smem_desc(st + 2 * kATile), blo = smem_desc(st + 2 * kATile + kBTile);
      const uint32_t acc = tmem + (uint32_t)(kt & 1) * kAccCols;  // this k-block's accumulator
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint64_t adv = (uint64_t)((kk * 8 * 4) >> 4);  // 32 bytes along K
        mma_tf32(acc, ahi + adv, bhi + adv, (kt > 1 || kk > 0) ? 1u : 0u);
        mma_tf32(acc, ahi + adv, blo + adv, 1u);
        mma_tf32(acc, alo + adv, bhi + adv, 1u);
      }
      mma_commit(&sm.empty[s]);
    }
    // Final commit: arrives once every MMA issued above has completed.
    mma_commit(&sm.acc_full);
  } else if (warp >= 2) {
    // ---- epilogue: TMEM -> registers -> global ----
    const int quarter = warp % 4;  // TMEM lanes 32*quarter .. +31 are this warp's
    bool ready = mbar_wait(&sm.acc_full, 0, abort);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ready) {
      *abort = 1;
    } else {
      const int row = m0 + quarter * 32 + lane;
      // A k part writes its raw partial tile (row-major BM x BN) for the
      // reduction kernel; a whole-K CTA writes C with the seed.
      float* prow = nsplit > 1 ? part_out + (long long)blockIdx.x * (BM * BN) + (quarter * 32 + lane) * BN : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
        tmem_ld32(lane_base, v);
        if (nkt > 1) {  // the second accumulator holds the odd k-blocks
          float w[32];
          tmem_ld32(lane_base + kAccCols, w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], w[j]);
        }
        if (prow) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(prow + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else if (row < M) {
          float* crow = C + (long long)row * ldc + n0 + c0;
          const int nvalid = N - (n0 + c0);
          if (nvalid >= 32 && ((ldc & 3) == 0) && (((uintptr_t)C & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(crow + j) =
                  make_float4(v[j] + seed, v[j + 1] + seed, v[j + 2] + seed, v[j + 3] + seed);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) crow[j] = v[j] + seed;
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(flag, kDeviceTimeout);
    // MMAs still in flight must finish before their TMEM is released.
    if (warp == 1 && lane == 0) mbar_wait(&sm.acc_full, 0, nullptr);
    __syncwarp();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// C tile (tile_base + r) = seed + sum over parts p (in order) of the partial
// tiles part[(r * nsplit + p)], for the k-split remainder tiles. Fixed order,
// so the result is the same on every run.
__global__ void reduce_parts_kernel(const float* __restrict__ part, float* __restrict__ C, int M, int N,
                                    long long ldc, float seed, int tiles_m, int tiles_n, int tile_base, int ntiles,
                                    int nsplit) {
  const long long total = (long long)ntiles * BM * BN;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / (BM * BN)), within = (int)(e % (BM * BN));
    const int row = within / BN, col = within % BN;
    int tm, tn;
    tile_coords(tile_base + r, tiles_m, tiles_n, tm, tn);
    const int m = tm * BM + row, n = tn * BN + col;
    if (m >= M || n >= N) continue;
    float acc = 0.0f;
    for (int p = 0; p < nsplit; ++p) acc += part[((long long)r * nsplit + p) * (BM * BN) + within];
    C[(long long)m * ldc + n] = acc + seed;
  }
}

// ---- fused split of A: raw A converted in shared memory ---------------------------------------
//
// The tensor pipe reads a kind::tf32 operand as its top 19 bits (the low 13
// mantissa bits are ignored, i.e. the value is truncated toward zero to
// TF32; measured on a B200). So a raw f32 tile is itself a "hi" operand,
// hi = trunc(x), and lo = rna(x - hi) (x - hi is exact in f32) completes the
// split. This kernel reads A where it lies: TMA brings raw A tiles (K-major,
// 64-byte swizzle), and warps 2-5 write each stage's A lo tile at the same
// offsets plus 8 KiB (the layouts are identical, so the conversion is
// elementwise) before releasing the stage to the MMA warp; the same warps run
// the epilogue. B still comes pre-split and transposed (BhiT, BloT), because
// B read in place would be an MN-major operand, and the tensor pipe runs
// kind::tf32 with an MN-major B about 9 % slower than K-major (measured with
// mapal_gpu_probe_mma_peak kinds 0 and 2), more than the B split pass costs.
// Against the pre-split kernel: no A split pass and 8 KiB less L2 traffic
// per stage.

struct SmemF {
  uint8_t stage[STAGES][kStageBytes];  // per stage: A raw | A lo | BhiT | BloT
  uint64_t full[STAGES];               // TMA landed the stage
  uint64_t conv[STAGES];               // the A lo tile is written (128 converter arrivals)
  uint64_t empty[STAGES];              // the MMAs have read the stage
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
};
constexpr int kConvThreads = 128;
static_assert(kATile / 16 % kConvThreads == 0, "the converter's float4 share must be whole");
constexpr uint32_t kLoadStageBytes = kATile + 2 * kBTile;  // TMA bytes per stage

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}

// lo part of x for the truncated hi: x - trunc(x) is exact in f32 and is
// rounded to TF32 (nearest, ties away) with integer operations. A NaN or
// infinite x gives a NaN lo, kept as NaN, so every product that reads x is
// NaN (a NaN whose payload is only in the low 13 bits, which the tensor pipe
// reads as infinity, still yields NaN).
__device__ __forceinline__ float lo_rna(float x) {
  const float lo = __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
  const float r = __uint_as_float((__float_as_uint(lo) + 0x1000u) & 0xFFFFE000u);
  return lo == lo ? r : lo;
}

__global__ void __launch_bounds__(kThreads, 1)
    mm_tf32x3_fused_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_bhi,
                           const __grid_constant__ CUtensorMap map_blo, float* __restrict__ C, int M, int N, int K,
                           long long ldc, float seed, unsigned* flag, int tiles_m, int tiles_n, int tile_base,
                           int nsplit, float* __restrict__ part_out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SmemF& sm = *reinterpret_cast<SmemF*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = tile_base + (int)blockIdx.x / nsplit, part = (int)blockIdx.x % nsplit;
  int tm, tn;
  tile_coords(tile, tiles_m, tiles_n, tm, tn);
  const int m0 = tm * BM, n0 = tn * BN;
  const int KT = (K + BK - 1) / BK;
  const int kt_lo = (int)((long long)KT * part / nsplit), nkt = (int)((long long)KT * (part + 1) / nsplit) - kt_lo;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.conv[s], kConvThreads);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: raw A, BhiT, BloT ----
    int issued = 0;
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES && !mbar_wait(&sm.empty[s], ((kt / STAGES) - 1) & 1, abort)) {
        *abort = 1;
        break;
      }
      uint8_t* st = sm.stage[s];
      mbar_expect_tx(&sm.full[s], kLoadStageBytes);
      const int k0 = (kt_lo + kt) * BK;
      tma_load_2d(st, &map_a, k0, m0, &sm.full[s]);
      tma_load_2d(st + 2 * kATile, &map_bhi, k0, n0, &sm.full[s]);
      tma_load_2d(st + 2 * kATile + kBTile, &map_blo, k0, n0, &sm.full[s]);
      ++issued;
    }
    if (*abort) {
      for (int kt = (issued > STAGES ? issued - STAGES : 0); kt < issued; ++kt)
        mbar_wait(&sm.full[kt % STAGES], (kt / STAGES) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt % STAGES;
      if (!mbar_wait(&sm.conv[s], (kt / STAGES) & 1, abort)) {
        *abort = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t* st = sm.stage[s];
      const uint64_t ahi = smem_desc(st), alo = smem_desc(st + kATile);
      const uint64_t bhi = smem_desc(st + 2 * kATile), blo = smem_desc(st + 2 * kATile + kBTile);
      const uint32_t acc = tmem + (uint32_t)(kt & 1) * kAccCols;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint64_t adv = (uint64_t)((kk * 8 * 4) >> 4);  // 32 bytes along K
        mma_tf32(acc, ahi + adv, bhi + adv, (kt > 1 || kk > 0) ? 1u : 0u);
        mma_tf32(acc, ahi + adv, blo + adv, 1u);
        mma_tf32(acc, alo + adv, bhi + adv, 1u);
      }
      mma_commit(&sm.empty[s]);
    }
    mma_commit(&sm.acc_full);
  } else if (warp >= 2) {
    // ---- converter: the A lo tile of every stage, then the epilogue ----
    const int ct = threadIdx.x - 64;
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt % STAGES;
      if (!mbar_wait(&sm.full[s], (kt / STAGES) & 1, abort)) {
        *abort = 1;
        break;
      }
      uint8_t* st = sm.stage[s];
      float4 v[kATile / 16 / kConvThreads];
#pragma unroll
      for (int i = 0; i < kATile / 16 / kConvThreads; ++i)
        v[i] = *reinterpret_cast<const float4*>(st + (ct + i * kConvThreads) * 16);
#pragma unroll
      for (int i = 0; i < kATile / 16 / kConvThreads; ++i)
        *reinterpret_cast<float4*>(st + kATile + (ct + i * kConvThreads) * 16) =
            make_float4(lo_rna(v[i].x), lo_rna(v[i].y), lo_rna(v[i].z), lo_rna(v[i].w));
      // generic-proxy writes, then visible to the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sm.conv[s]);
    }
    const int quarter = warp % 4;
    bool ready = mbar_wait(&sm.acc_full, 0, abort);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ready) {
      *abort = 1;
    } else {
      const int row = m0 + quarter * 32 + lane;
      float* prow = nsplit > 1 ? part_out + (long long)blockIdx.x * (BM * BN) + (quarter * 32 + lane) * BN : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
        tmem_ld32(lane_base, v);
        if (nkt > 1) {
          float w[32];
          tmem_ld32(lane_base + kAccCols, w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], w[j]);
        }
        if (prow) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(prow + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else if (row < M) {
          float* crow = C + (long long)row * ldc + n0 + c0;
          const int nvalid = N - (n0 + c0);
          if (nvalid >= 32 && ((ldc & 3) == 0) && (((uintptr_t)C & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(crow + j) =
                  make_float4(v[j] + seed, v[j + 1] + seed, v[j + 2] + seed, v[j + 3] + seed);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) crow[j] = v[j] + seed;
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(flag, kDeviceTimeout);
    if (warp == 1 && lane == 0) mbar_wait(&sm.acc_full, 0, nullptr);
    __syncwarp();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// MN-major B for the probe (kind 2): 32-column chunks 2048 bytes apart (LBO),
// groups of 4 k rows 512 bytes apart (SBO), 128-byte rows, layout type 1
// (128-byte swizzle with 32-byte atoms, the only MN-major layout UMMA takes
// for 32-bit operands).
__device__ __forceinline__ uint64_t smem_desc_mn(const void* p) {
  uint64_t addr = sa(p);
  uint64_t d = 0;
  d |= (addr & 0x3FFFFull) >> 4;
  d |= (uint64_t)(2048 >> 4) << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= 1ull << 46;
  d |= 1ull << 61;
  return d;
}

constexpr uint32_t kIdescMN = kIdesc | (1u << 16);  // B MN-major

__device__ __forceinline__ void mma_tf32_mn(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdescMN), "r"(accumulate));
}

// ---- tensor-pipe probe ---------------------------------------------------------------------
//
// The roofline of the 3xTF32 GEMM is the tensor pipe's TF32 rate, which no
// datasheet figure gives for this part at its operating clock: this kernel
// measures it. One CTA per SM issues the GEMM's own MMA (M128 N256, operands
// K-major with the 64-byte swizzle in shared memory, f32 accumulator in TMEM)
// back to back with no memory traffic at all: `iters` rounds of 6 MMAs (two
// 8-deep k-steps x three products, as one stage of the GEMM). kind 1 issues
// the bf16 form of the same instruction shape (kind::f16, K16: the same
// 32 bytes of each operand row per MMA), to check the method against the
// measured cuBLAS bf16 rate.
constexpr uint32_t kIdescBf16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)(BM >> 4) << 24);
constexpr int kProbeThreads = 128;

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdescBf16), "r"(accumulate));
}

__global__ void __launch_bounds__(kProbeThreads, 1) probe_mma_kernel(int iters, int kind, unsigned* flag, float* sink) {
  // kind 2: kind::tf32 with B MN-major (the fused kernel's B layout: 128-byte
  // swizzle with 32-byte atoms, 32-column chunks 2 KiB apart)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // two operand sets (hi, lo) as in one GEMM stage: A 2 x 8 KiB, B 2 x 16 KiB
  uint32_t* words = reinterpret_cast<uint32_t*>(base);
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  for (int i = threadIdx.x; i < kStageBytes / 4; i += blockDim.x) {
    // finite values of either type: a bounded hash in [-1, 1) as f32, whose
    // 16-bit halves are ordinary bf16 values too
    uint32_t h = (uint32_t)i * 2654435761u + 12345u;
    h ^= h >> 13;
    words[i] = __float_as_uint((float)(h & 0xFFFF) * (1.0f / 32768.0f) - 1.0f) & 0xFFFFE000u;
  }
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) {
    const uint64_t ahi = smem_desc(base), alo = smem_desc(base + kATile);
    const uint64_t bhi = smem_desc(base + 2 * kATile), blo = smem_desc(base + 2 * kATile + kBTile);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint64_t adv = (uint64_t)((kk * 32) >> 4);
        if (kind == 0) {
          mma_tf32(tmem, ahi + adv, bhi + adv, (it > 0 || kk > 0) ? 1u : 0u);
          mma_tf32(tmem, ahi + adv, blo + adv, 1u);
          mma_tf32(tmem, alo + adv, bhi + adv, 1u);
        } else if (kind == 2) {
          const uint64_t bm = smem_desc_mn(base + 2 * kATile) + (uint64_t)((kk * 1024) >> 4);
          const uint64_t bl = smem_desc_mn(base + 2 * kATile + kBTile) + (uint64_t)((kk * 1024) >> 4);
          mma_tf32_mn(tmem, ahi + adv, bm, (it > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_mn(tmem, ahi + adv, bl, 1u);
          mma_tf32_mn(tmem, alo + adv, bm, 1u);
        } else {
          mma_bf16(tmem, ahi + adv, bhi + adv, (it > 0 || kk > 0) ? 1u : 0u);
          mma_bf16(tmem, ahi + adv, blo + adv, 1u);
          mma_bf16(tmem, alo + adv, bhi + adv, 1u);
        }
      }
    }
    mma_commit(&done);
    // bounded: a wait that runs out flags the launch, then waits once more
    // (bounded again) so no MMA is in flight when the columns are freed
    if (!mbar_wait(&done, 0, nullptr)) {
      atomicOr(flag, kDeviceTimeout);
      mbar_wait(&done, 0, nullptr);
    }
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  // one accumulator row per thread of warp 0..3 (lanes 32*warp + lane), first
  // 32 columns, folded into one value so the work has an observable result
  float v[32];
  tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) s += v[j];
  if (s == 12345.678f) sink[blockIdx.x] = s;  // practically never true; keeps the read
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---- split pass --------------------------------------------------------------------------

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi = rna(x), lo = rna(x - hi); non-finite values (and a hi that rounded up
// past the f32 range) keep lo = 0 so they propagate as hi*B alone. A NaN
// becomes the canonical NaN: rounding its mantissa could otherwise leave the
// bits of an infinity (a payload only in the low 13 bits).
__device__ __forceinline__ void split1(float x, float& hi, float& lo) {
  if (isnan(x)) {
    hi = __uint_as_float(0x7FFFFFFFu);
    lo = 0.0f;
    return;
  }
  hi = tf32_rna(x);
  if (isinf(hi) && !isinf(x)) hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = isfinite(hi) ? tf32_rna(__fsub_rn(x, hi)) : 0.0f;
}

// A (M x K, row stride lda) -> hi, lo (M x K, row stride kp). Blocks walk
// rows; threads walk a row in 16-byte groups when rows are 16-byte aligned.
__global__ void split_rows_kernel(const float* __restrict__ A, long long lda, int M, int K, float* __restrict__ hi,
                                  float* __restrict__ lo, long long kp) {
  const bool vec = (K & 3) == 0 && (lda & 3) == 0 && ((uintptr_t)A & 15) == 0;
  for (int r = blockIdx.x; r < M; r += gridDim.x) {
    const float* a = A + (long long)r * lda;
    float* h = hi + (long long)r * kp;
    float* l = lo + (long long)r * kp;
    if (vec) {
      for (int c = threadIdx.x; c < K / 4; c += blockDim.x) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(a) + c);
        float4 vh, vl;
        split1(v.x, vh.x, vl.x);
        split1(v.y, vh.y, vl.y);
        split1(v.z, vh.z, vl.z);
        split1(v.w, vh.w, vl.w);
        reinterpret_cast<float4*>(h)[c] = vh;
        reinterpret_cast<float4*>(l)[c] = vl;
      }
    } else {
      for (int c = threadIdx.x; c < K; c += blockDim.x) split1(__ldg(a + c), h[c], l[c]);
    }
  }
}

// B (K x N, row stride ldb) -> hiT, loT (N x K, row stride kp): 64x64 tiles
// through shared memory so both sides stay coalesced; 256 threads, 16
// elements each, all 16 loads in flight before the first shared store.
constexpr int kTT = 64, kTRows = 4;
__global__ void __launch_bounds__(kTT* kTRows) split_transpose_kernel(const float* __restrict__ B, long long ldb,
                                                                     int K, int N, float* __restrict__ hiT,
                                                                     float* __restrict__ loT, long long kp) {
  __shared__ float th[kTT][kTT + 1], tl[kTT][kTT + 1];
  const int k0 = blockIdx.y * kTT, n0 = blockIdx.x * kTT;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 64 x 4
  float v[kTT / kTRows];
#pragma unroll
  for (int p = 0; p < kTT / kTRows; ++p) {
    const int k = k0 + ty + kTRows * p, n = n0 + tx;
    v[p] = (k < K && n < N) ? __ldg(B + (long long)k * ldb + n) : 0.0f;
  }
#pragma unroll
  for (int p = 0; p < kTT / kTRows; ++p) {
    float h, l;
    split1(v[p], h, l);
    th[ty + kTRows * p][tx] = h;
    tl[ty + kTRows * p][tx] = l;
  }
  __syncthreads();
#pragma unroll
  for (int p = 0; p < kTT / kTRows; ++p) {
    const int n = n0 + ty + kTRows * p, k = k0 + tx;
    if (n < N && k < K) {
      hiT[(long long)n * kp + k] = th[tx][ty + kTRows * p];
      loT[(long long)n * kp + k] = tl[tx][ty + kTRows * p];
    }
  }
}

// ---- host: tensor maps ----------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's cuTensorMapEncodeTiled, looked up once (a function-local
// static is initialised exactly once, also when threads race to it).
EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (EncodeTiledFn)p;
    return (EncodeTiledFn) nullptr;
  }();
  return fn;
}

// rows x K f32 matrix with row stride kp (elements), box = box_rows x BK.
int make_map(CUtensorMap* map, const float* base, uint64_t rows, uint64_t K, uint64_t kp, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(MAPAL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {kp * 4};
  cuuint32_t box[2] = {BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MAPAL_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return 0;
}

}  // namespace

int launch_matmul_tf32x3(DeviceSlot& d, const float* A, const float* B, float* C, uint64_t M, uint64_t N,
                         uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed) {
  if (M > 0x7fffffffull || N > 0x7fffffffull || K > 0x7fffffffull) return set_error(MAPAL_ERR_UNSUPPORTED, "too large");
  if ((N + BN - 1) / BN > 0x7fffffffull || (M + BM - 1) / BM > 65535)
    return set_error(MAPAL_ERR_UNSUPPORTED, "matmul grid too large");
  const uint64_t kp = (K + 3) & ~3ull;  // TMA row strides must be multiples of 16 bytes
  // Tile plan: whole waves of 128 x 256 tiles; a partial last wave of R tiles
  // is split along K into nsplit parts (R * nsplit <= SMs) whose partial
  // tiles a reduction kernel sums in a fixed order.
  const int sms = d.prof.sm_count;
  const int tiles_n = (int)((N + BN - 1) / BN);
  const int tiles_m = (int)((M + BM - 1) / BM);
  const int tiles = tiles_m * tiles_n;
  const int KT = (int)((K + BK - 1) / BK);
  const int full = (tiles / sms) * sms, rem = tiles - full;
  int nsplit = 1;
  if (rem > 0 && rem <= sms / 2) {
    nsplit = sms / rem;
    if (nsplit > 4) nsplit = 4;
    if (nsplit > KT) nsplit = KT;
  }
  const uint64_t part_elems = nsplit > 1 ? (uint64_t)rem * nsplit * BM * BN : 0;
  const int whole = nsplit > 1 ? full : tiles;  // tiles computed over all of K

  // B is split and transposed into BhiT, BloT (N x K, K-major) in the arena.
  // A is read in place when TMA can address its rows (16-byte aligned base and
  // row stride) and N <= 8192: the GEMM then splits A in shared memory, which
  // costs about 2.5 % of the GEMM, while the A split pass it replaces costs a
  // share that falls as 1/N (5 % of the site at N = 4096, 1 % at 16384;
  // B200-measured: 4096^3 0.595 -> 0.578 ms, 16384^3 36.8 -> 37.4 ms).
  // Otherwise A is split into Ahi, Alo in the arena as well.
  const bool a_in_place = aligned16(A) && (lda & 3) == 0 && N <= 8192;
  const uint64_t a_elems = a_in_place ? 0 : 2 * M * kp;
  MAPAL_TRY(arena_reserve(d, (a_elems + 2 * N * kp + part_elems) * sizeof(float) + 4096));
  float* bhi = (float*)d.arena;
  float* blo = bhi + N * kp;
  float* ahi = blo + N * kp;
  float* alo = ahi + M * kp;
  float* parts = ahi + a_elems;
  // every operand base stays 16-byte aligned (kp is a multiple of 4 floats)
  dim3 tg((unsigned)((N + kTT - 1) / kTT), (unsigned)((K + kTT - 1) / kTT));
  if (tg.y > 65535) return set_error(MAPAL_ERR_UNSUPPORTED, "K too large for the split pass");
  split_transpose_kernel<<<tg, dim3(kTT, kTRows), 0, d.stream>>>(B, (long long)ldb, (int)K, (int)N, bhi, blo,
                                                                (long long)kp);
  count_launch();

  if (a_in_place) {
    CUtensorMap m_a, m_bhi, m_blo;
    MAPAL_TRY(make_map(&m_a, A, M, K, lda, BM));
    MAPAL_TRY(make_map(&m_bhi, bhi, N, K, kp, BN));
    MAPAL_TRY(make_map(&m_blo, blo, N, K, kp, BN));
    const size_t smem = sizeof(SmemF) + 1024;
    static std::atomic<uint64_t> attr_fused{0};
    MAPAL_TRY(ensure_smem_attr(attr_fused, (const void*)mm_tf32x3_fused_kernel, d.device, smem,
                               "cudaFuncSetAttribute(mm_tf32x3_fused_kernel)"));
    if (whole > 0) {
      mm_tf32x3_fused_kernel<<<(unsigned)whole, kThreads, smem, d.stream>>>(
          m_a, m_bhi, m_blo, C, (int)M, (int)N, (int)K, (long long)ldc, seed, d.trap, tiles_m, tiles_n, 0, 1, nullptr);
      count_launch();
    }
    if (nsplit > 1) {
      mm_tf32x3_fused_kernel<<<(unsigned)(rem * nsplit), kThreads, smem, d.stream>>>(
          m_a, m_bhi, m_blo, C, (int)M, (int)N, (int)K, (long long)ldc, seed, d.trap, tiles_m, tiles_n, full, nsplit,
          parts);
      count_launch();
      const uint64_t n_red = (uint64_t)rem * BM * BN;
      reduce_parts_kernel<<<stream_grid(n_red, 256, sms, 8), 256, 0, d.stream>>>(parts, C, (int)M, (int)N,
                                                                                (long long)ldc, seed, tiles_m, tiles_n,
                                                                                full, rem, nsplit);
      count_launch();
    }
    return 0;
  }

  split_rows_kernel<<<(unsigned)(M < (uint64_t)sms * 8 ? M : (uint64_t)sms * 8), 256, 0, d.stream>>>(
      A, (long long)lda, (int)M, (int)K, ahi, alo, (long long)kp);
  count_launch();

  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  MAPAL_TRY(make_map(&m_ahi, ahi, M, K, kp, BM));
  MAPAL_TRY(make_map(&m_alo, alo, M, K, kp, BM));
  MAPAL_TRY(make_map(&m_bhi, bhi, N, K, kp, BN));
  MAPAL_TRY(make_map(&m_blo, blo, N, K, kp, BN));

  const size_t smem = sizeof(Smem) + 1024;
  static std::atomic<uint64_t> attr_set{0};
  MAPAL_TRY(ensure_smem_attr(attr_set, (const void*)mm_tf32x3_kernel, d.device, smem,
                             "cudaFuncSetAttribute(mm_tf32x3_kernel)"));
  if (whole > 0) {
    mm_tf32x3_kernel<<<(unsigned)whole, kThreads, smem, d.stream>>>(m_ahi, m_alo, m_bhi, m_blo, C, (int)M, (int)N,
                                                                    (int)K, (long long)ldc, seed, d.trap, tiles_m,
                                                                    tiles_n, 0, 1, nullptr);
    count_launch();
  }
  if (nsplit > 1) {
    mm_tf32x3_kernel<<<(unsigned)(rem * nsplit), kThreads, smem, d.stream>>>(
        m_ahi, m_alo, m_bhi, m_blo, C, (int)M, (int)N, (int)K, (long long)ldc, seed, d.trap, tiles_m, tiles_n, full,
        nsplit, parts);
    count_launch();
    const uint64_t n_red = (uint64_t)rem * BM * BN;
    reduce_parts_kernel<<<stream_grid(n_red, 256, sms, 8), 256, 0, d.stream>>>(parts, C, (int)M, (int)N,
                                                                              (long long)ldc, seed, tiles_m, tiles_n,
                                                                              full, rem, nsplit);
    count_launch();
  }
  return 0;
}

// Tensor-pipe probe (see probe_mma_kernel): one CTA per SM, a warm-up launch,
// then one timed launch between two events on the context's stream.
extern "C" int mapal_gpu_probe_mma_peak(MapalGpuCtx* ctx, int kind, uint32_t iters, double* tflops) {
  MAPAL_TRY(enter(ctx, 0));
  if (!tflops) return set_error(MAPAL_ERR_INVALID, "tflops is null");
  if (kind < 0 || kind > 2) return set_error(MAPAL_ERR_INVALID, "kind must be 0 (tf32), 1 (bf16) or 2 (tf32, B MN-major)");
  if (iters == 0 || iters > (1u << 24)) return set_error(MAPAL_ERR_INVALID, "iters must be in [1, 2^24]");
  DeviceSlot& d = ctx->dev[0];
  // 120 KiB of dynamic shared memory: only one probe CTA fits on an SM
  const size_t smem = 120 * 1024;
  static std::atomic<uint64_t> attr_set{0};
  MAPAL_TRY(ensure_smem_attr(attr_set, (const void*)probe_mma_kernel, d.device, smem,
                             "cudaFuncSetAttribute(probe_mma_kernel)"));
  MAPAL_TRY(arena_reserve(d, (size_t)d.prof.sm_count * sizeof(float)));
  float* sink = static_cast<float*>(d.arena);
  cudaEvent_t e0, e1;
  MAPAL_CUDA(cudaEventCreate(&e0));
  MAPAL_CUDA(cudaEventCreate(&e1));
  const unsigned grid = (unsigned)d.prof.sm_count;
  probe_mma_kernel<<<grid, kProbeThreads, smem, d.stream>>>((int)(iters < 64 ? iters : 64), kind, d.trap, sink);
  count_launch();
  cudaEventRecord(e0, d.stream);
  probe_mma_kernel<<<grid, kProbeThreads, smem, d.stream>>>((int)iters, kind, d.trap, sink);
  count_launch();
  cudaEventRecord(e1, d.stream);
  cudaError_t le = cudaGetLastError();
  cudaError_t se = cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaError_t te = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (le != cudaSuccess) return cuda_fail(le, "probe_mma_kernel launch");
  if (se != cudaSuccess) return cuda_fail(se, "probe_mma_kernel");
  if (te != cudaSuccess) return cuda_fail(te, "cudaEventElapsedTime");
  MAPAL_TRY(drain(d));
  const double k_per_mma = kind == 1 ? 16.0 : 8.0;
  const double flops = (double)grid * iters * 6.0 * 2.0 * BM * BN * k_per_mma;
  *tflops = flops / (ms * 1e-3) / 1e12;
  return 0;
}
