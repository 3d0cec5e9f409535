// reduce.cu — the sum fold `(seed, x) -> fold { acc, v -> acc + v }`
// (benches/shapes/reduce_1048576.mapal:10).
//
// The reference runs every top-level fold as one device thread
// (<<<1,1>>>, crates/backends/cuda/src/kernel.rs:1484-1642; BC4 of the
// reference's docs/components/backend-cuda/DESIGN.md),
// because an f32 left fold is only bit-exact in sequence (ADR-0028 keeps f32
// folds sequential-pinned). This site is the one place the library trades
// bit-exactness for parallelism, under a stated tolerance: one launch, every
// SM streaming 128-bit loads, each thread summing its elements in f64, a
// fixed warp-shuffle + block tree, and the last block to finish combining the
// per-block partials in a fixed order. The shape of the tree depends only on
// n and the SM count, so the result is the same on every run.
#include "common.cuh"
#include "cpasync.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ double block_sum(double v, double* smem) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // smem may still be read by a previous call
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += smem[w];
  return t;  // valid in thread 0
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Warp 0 of the last block: lane q stores this rank's partial into rank q's
// block and raises its flag there, then waits (bounded) for rank q's flag in
// this device's block. Lane 0 adds the partials in rank order, so every rank
// writes the same value.
__device__ void peer_combine(double mine, float seed, float* out, const PeerArgs& P) {
  const int q = threadIdx.x;
  const int par = (int)(P.epoch & 1);
  unsigned err = 0;
  double v = 0.0;
  if (q < P.nranks) {
    PeerBlock* dst = P.blk[q];
    volatile PeerSlot* slot = &dst->val[par][P.rank];
    slot->v = mine;
    slot->epoch = P.epoch;
    st_release_sys(&dst->flag[P.rank], P.epoch);
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(&P.own->flag[q]) < P.epoch) {
      if (global_ns() - t0 > P.wait_ns) {  // a rank that has not published is reported, not waited for
        err = kPeerTimeout;
        break;
      }
      __nanosleep(32);
    }
    if (!err) {
      volatile const PeerSlot* src = &P.own->val[par][q];
      if (src->epoch != P.epoch) err = kPeerOutOfStep;
      v = src->v;
    }
  }
  err = __reduce_or_sync(0xffffffffu, err);
  double total = 0.0;
  for (int r = 0; r < P.nranks; ++r) total += __shfl_sync(0xffffffffu, v, r);
  if (q == 0) {
    if (err)
      atomicOr(P.trap, err);
    else
      *out = (float)((double)seed + total);
  }
}

template <bool kVec, bool kPeer>
__global__ void __launch_bounds__(kThreads) fold_sum_kernel(const float* __restrict__ x, uint64_t n,
                                                            float seed, double* partials,
                                                            unsigned* counter, float* out_f32,
                                                            double* out_f64, const __grid_constant__ PeerArgs P) {
  __shared__ double smem[kWarps];
  __shared__ bool last;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t gid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  double acc = 0.0;
  uint64_t tail = 0;
  if (kVec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const uint64_t n4 = n / 4;
    // Four 16-byte loads per thread per trip, issued together; the last,
    // partial trip loads a clamped (valid) index and zeroes what lies past
    // the end with a select, so its loads are not behind branches either and
    // a small input costs one memory round trip.
    uint64_t i = gid;
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(x4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc += (double)v[u].x;
        acc += (double)v[u].y;
        acc += (double)v[u].z;
        acc += (double)v[u].w;
      }
    }
    if (i < n4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint64_t j = i + u * stride;
        v[u] = __ldcs(x4 + (j < n4 ? j : n4 - 1));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool in = i + u * stride < n4;
        acc += in ? (double)v[u].x : 0.0;
        acc += in ? (double)v[u].y : 0.0;
        acc += in ? (double)v[u].z : 0.0;
        acc += in ? (double)v[u].w : 0.0;
      }
    }
    tail = n4 * 4;
  }
  for (uint64_t i = tail + gid; i < n; i += stride) acc += (double)__ldcs(x + i);

  double bsum = block_sum(acc, smem);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = bsum;
    // One acquire-release atomic: release publishes this block's partial,
    // and for the block that arrives last, acquire makes every partial
    // visible (to its other threads through the barrier below).
    unsigned ticket;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(ticket) : "l"(counter) : "memory");
    last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  // Last block: combine the partials in block order (fixed).
  double t = 0.0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) t += __ldcg(partials + b);
  double total = block_sum(t, smem);
  if (kPeer) {
    __shared__ double rank_total;
    if (threadIdx.x == 0) {
      rank_total = total;
      *counter = 0u;
    }
    __syncthreads();
    if (threadIdx.x < 32) peer_combine(rank_total, seed, out_f32, P);
    return;
  }
  if (threadIdx.x == 0) {
    if (out_f64) *out_f64 = total;
    if (out_f32) *out_f32 = (float)((double)seed + total);
    *counter = 0u;  // ready for the next launch on this stream
  }
}

// Blocks of one fold launch: up to 16 elements per thread (one trip of four
// 16-byte loads), at most 4 blocks per SM; beyond one wave's worth of SMs the
// count is a whole multiple of the SM count, so every SM streams the same
// share. Depends only on n and the SM count, so the tree is fixed.
unsigned fold_grid(uint64_t n, int sms) {
  uint64_t want = (n + (uint64_t)kThreads * 16 - 1) / ((uint64_t)kThreads * 16);
  uint64_t cap = (uint64_t)sms * 4;
  if (cap > (uint64_t)kFoldMaxBlocks) cap = kFoldMaxBlocks;
  if (want > (uint64_t)sms) want = (want + sms - 1) / sms * sms;
  return (unsigned)(want < 1 ? 1 : (want > cap ? cap : want));
}

__global__ void finalize_sum_kernel(const double* total, float seed, float* out) {
  *out = (float)((double)seed + *total);
}

}  // namespace

int launch_fold_sum(cudaStream_t s, int sms, const float* x, uint64_t n, float seed, double* partials,
                    unsigned* counter, float* out_f32, double* out_f64) {
  const unsigned grid = fold_grid(n, sms);
  if (n >= 4 && aligned16(x))
    fold_sum_kernel<true, false><<<grid, kThreads, 0, s>>>(x, n, seed, partials, counter, out_f32, out_f64,
                                                           PeerArgs{});
  else
    fold_sum_kernel<false, false><<<grid, kThreads, 0, s>>>(x, n, seed, partials, counter, out_f32, out_f64,
                                                            PeerArgs{});
  count_launch();
  return 0;
}

int launch_fold_sum_peer(cudaStream_t s, int sms, const float* x, uint64_t n, float seed, double* partials,
                         unsigned* counter, float* out, const PeerArgs& P) {
  // the same grid rule as launch_fold_sum: the rank's partial is the same tree
  const unsigned grid = fold_grid(n, sms);
  if (n >= 4 && aligned16(x))
    fold_sum_kernel<true, true><<<grid, kThreads, 0, s>>>(x, n, seed, partials, counter, out, nullptr, P);
  else
    fold_sum_kernel<false, true><<<grid, kThreads, 0, s>>>(x, n, seed, partials, counter, out, nullptr, P);
  count_launch();
  return 0;
}

namespace {

// The strict left fold: the block's threads stage chunks of x into a shared
// ring with cp.async, thread 0 adds them in order. The ring hides the load
// latency, leaving the chain of dependent adds as the only cost.
constexpr int kStrictThreads = 256;
constexpr int kStrictChunk = 2048;  // floats per stage
constexpr int kStrictStages = 4;

template <bool kAligned>
__global__ void __launch_bounds__(kStrictThreads) fold_sum_strict_kernel(const float* __restrict__ x,
                                                                         uint64_t n, float seed,
                                                                         float* out) {
  __shared__ __align__(16) float ring[kStrictStages][kStrictChunk];
  const uint64_t chunks = (n + kStrictChunk - 1) / kStrictChunk;
  auto issue = [&](uint64_t c) {
    if (c < chunks) {
      const uint64_t base = c * kStrictChunk;
      float* buf = ring[c % kStrictStages];
      for (int g = threadIdx.x; g < kStrictChunk / 4; g += kStrictThreads) {
        const uint64_t e = base + 4 * (uint64_t)g;
        const int64_t left = (int64_t)n - (int64_t)e;
        const int nvalid = left >= 4 ? 4 : (left > 0 ? (int)left : 0);
        copy4(smem_u32(buf + 4 * g), x + (nvalid ? e : 0), nvalid, kAligned);
      }
    }
    cp_commit();  // an empty group keeps the wait count uniform
  };
#pragma unroll
  for (int s = 0; s < kStrictStages - 1; ++s) issue(s);
  float acc = seed;
  for (uint64_t c = 0; c < chunks; ++c) {
    cp_wait<kStrictStages - 2>();
    __syncthreads();  // chunk c landed for every thread; chunk c-1's buffer is free
    issue(c + kStrictStages - 1);
    if (threadIdx.x == 0) {
      const float4* v = reinterpret_cast<const float4*>(ring[c % kStrictStages]);
      const uint64_t left = n - c * kStrictChunk;
      const int cnt = left < (uint64_t)kStrictChunk ? (int)left : kStrictChunk;
      int i = 0;
#pragma unroll 8
      for (; i + 4 <= cnt; i += 4) {
        const float4 q = v[i / 4];
        acc = __fadd_rn(acc, q.x);
        acc = __fadd_rn(acc, q.y);
        acc = __fadd_rn(acc, q.z);
        acc = __fadd_rn(acc, q.w);
      }
      for (; i < cnt; ++i) acc = __fadd_rn(acc, ring[c % kStrictStages][i]);
    }
  }
  cp_wait<0>();
  if (threadIdx.x == 0) *out = acc;
}

}  // namespace

int launch_fold_sum_strict(cudaStream_t s, const float* x, uint64_t n, float seed, float* out) {
  if (aligned16(x))
    fold_sum_strict_kernel<true><<<1, kStrictThreads, 0, s>>>(x, n, seed, out);
  else
    fold_sum_strict_kernel<false><<<1, kStrictThreads, 0, s>>>(x, n, seed, out);
  count_launch();
  return 0;
}

namespace {

// out = seed, then every block adds its wrapping partial sum atomically.
__global__ void set_i32_kernel(int32_t* out, int32_t v) { *out = v; }

__global__ void __launch_bounds__(kThreads) fold_sum_i32_kernel(const int32_t* __restrict__ x, uint64_t n,
                                                                int32_t* out) {
  __shared__ uint32_t part[kWarps];
  uint32_t acc = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads)
    acc += (uint32_t)__ldcs(x + i);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += part[w];
    atomicAdd(reinterpret_cast<unsigned*>(out), t);
  }
}

}  // namespace

extern "C" int mapal_gpu_fold_sum_i32(MapalGpuCtx* ctx, int32_t seed, const int32_t* x, uint64_t n,
                                      int32_t* out) {
  MAPAL_TRY(enter(ctx));
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (n && !x) return set_error(MAPAL_ERR_INVALID, "x is null");
  DeviceSlot& d = ctx->dev[0];
  set_i32_kernel<<<1, 1, 0, d.stream>>>(out, seed);
  count_launch();
  if (n) {
    fold_sum_i32_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 4), kThreads, 0, d.stream>>>(x, n, out);
    count_launch();
  }
  return finish(ctx, 0, false);
}

int launch_finalize_sum(cudaStream_t s, const double* total, float seed, float* out) {
  finalize_sum_kernel<<<1, 1, 0, s>>>(total, seed, out); count_launch();
  return 0;
}

extern "C" int mapal_gpu_fold_sum_f32(MapalGpuCtx* ctx, float seed, const float* x, uint64_t n,
                                      float* out) {
  MAPAL_TRY(enter(ctx));
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (n && !x) return set_error(MAPAL_ERR_INVALID, "x is null");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_fold_sum(d.stream, d.prof.sm_count, x, n, seed, d.fold_partials, d.fold_counter,
                            out, nullptr));
  return finish(ctx, 0, false);
}

// ---- launch floors of the streaming class ----------------------------------------------------
// What a 2^20-element site cannot beat: an empty kernel (the launch itself),
// and the fold's own grid and loads with no cross-block combine (one read of
// x at the rate the fold's loads reach).
namespace {
__global__ void floor_empty_kernel() {}

__global__ void __launch_bounds__(kThreads) floor_read_kernel(const float4* __restrict__ x4, uint64_t n4,
                                                              float* sink) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t gid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  float acc = 0.0f;
  uint64_t i = gid;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcs(x4 + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) acc += v[u].x + v[u].y + v[u].z + v[u].w;
  }
  if (i < n4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint64_t j = i + u * stride;
      v[u] = __ldcs(x4 + (j < n4 ? j : n4 - 1));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * stride < n4) acc += v[u].x + v[u].y + v[u].z + v[u].w;
  }
  if (acc == 1.2345e-30f) *sink = acc;  // practically never: keeps the loads
}

// n reads of x at hashed positions in [0, n_x), four per thread per trip, no
// index array and no output: the rate at which the memory system serves
// independent random 4-byte reads.
__global__ void __launch_bounds__(kThreads) floor_random_kernel(const float* __restrict__ x, uint64_t n_x,
                                                                uint64_t n, float* sink) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  float acc = 0.0f;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += 4 * stride) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint64_t h = (i + u * stride) * 0x9E3779B97F4A7C15ull;
      h ^= h >> 29;
      h *= 0xBF58476D1CE4E5B9ull;
      h ^= h >> 32;
      v[u] = (i + u * stride) < n ? __ldcs(x + h % n_x) : 0.0f;
    }
    acc += v[0] + v[1] + v[2] + v[3];
  }
  if (acc == 1.2345e-30f) *sink = acc;
}
}  // namespace

extern "C" int mapal_gpu_probe_launch_floor(MapalGpuCtx* ctx, int kind, const float* x, uint64_t n, float* sink) {
  MAPAL_TRY(enter(ctx));
  DeviceSlot& d = ctx->dev[0];
  if (kind == 0) {
    floor_empty_kernel<<<1, 32, 0, d.stream>>>();
  } else if (kind == 1) {
    if (!x || !sink || !aligned16(x) || (n & 3) != 0 || n == 0)
      return set_error(MAPAL_ERR_INVALID, "the read floor needs a 16-byte aligned x of 4k > 0 floats and a sink");
    floor_read_kernel<<<fold_grid(n, d.prof.sm_count), kThreads, 0, d.stream>>>(
        reinterpret_cast<const float4*>(x), n / 4, sink);
  } else if (kind == 2) {
    if (!x || !sink || n == 0) return set_error(MAPAL_ERR_INVALID, "the random-read floor needs x (n floats) and a sink");
    floor_random_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(x, n, n, sink);
  } else {
    return set_error(MAPAL_ERR_INVALID, "kind must be 0 (empty kernel), 1 (read) or 2 (random reads)");
  }
  count_launch();
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_fold_sum_f32_strict(MapalGpuCtx* ctx, float seed, const float* x, uint64_t n,
                                             float* out) {
  MAPAL_TRY(enter(ctx));
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (n && !x) return set_error(MAPAL_ERR_INVALID, "x is null");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_fold_sum_strict(d.stream, x, n, seed, out));
  return finish(ctx, 0, false);
}
