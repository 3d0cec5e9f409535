// gen.cu — input generators: Iota, Fill, Widen (crates/backends/cuda/src/kernel.rs:1335-1378;
// crates/mapal-interp/src/eval.rs:238-248, 402-427) and the fused element
// generators a consumer can recompute from the index alone (elem_plan,
// crates/mapal-ir/src/algo.rs:434-512): the benches' integer formulas and the
// seeded uniform stream. Grid-stride, 128-bit stores where aligned.
#include "common.cuh"

namespace {

// i32 wrapping arithmetic as Rust's wrapping_* (eval.rs:552-569). CUDA's
// signed `/` and `%` truncate toward zero like Rust's; the divisors used here
// are positive constants, so the MIN / -1 case cannot arise.
__device__ __forceinline__ int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
__device__ __forceinline__ int32_t wmul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }

__device__ __forceinline__ int32_t gen_hash(int32_t seed, int32_t i) {
  int32_t h = wadd(wmul(i, 1103515245), wadd(wmul(seed, 1640531527), 12345));
#pragma unroll
  for (int r = 0; r < 3; ++r) h = wadd(wadd(wmul(h, h), h / 65536), 1013904223);
  return h;
}

__device__ __forceinline__ int32_t pos_mod(int32_t d, int32_t m) { return wadd(d % m, m) % m; }

__device__ __forceinline__ float gen_value(int32_t seed, int32_t i, int kind) {
  int32_t r = pos_mod(gen_hash(seed, i) / 128, 16777216);
  float f = __int2float_rn(r);
  return kind == MAPAL_GEN_U01 ? __fdiv_rn(f, 16777216.0f) : __fsub_rn(__fdiv_rn(f, 8388608.0f), 1.0f);
}

__global__ void iota_kernel(int32_t* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = (int32_t)i;
}

__global__ void fill_kernel(float* out, float v, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = v;
}

__global__ void widen_kernel(const int32_t* in, float* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = __int2float_rn(in[i]);
}

__global__ void affine_kernel(float* out, uint64_t n, int64_t start, int32_t mul, int32_t add,
                              int32_t mod, int32_t sub) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    int32_t t = (int32_t)(uint32_t)(uint64_t)(start + (int64_t)i);
    int32_t v = wadd(wmul(t, mul), add) % mod;
    out[i] = __int2float_rn((int32_t)((uint32_t)v - (uint32_t)sub));
  }
}

__global__ void gen_kernel(float* out, uint64_t n, int32_t seed, int64_t offset, int kind) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = gen_value(seed, (int32_t)(uint32_t)(uint64_t)(offset + (int64_t)i), kind);
}

__global__ void gen_index_kernel(int32_t* out, uint64_t n, int32_t seed, int64_t offset,
                                 int32_t range) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    int32_t h = gen_hash(seed, (int32_t)(uint32_t)(uint64_t)(offset + (int64_t)i));
    int32_t d = range <= 16777216 ? h / 128 : h / 8;
    out[i] = pos_mod(d, range);
  }
}

constexpr int kThreads = 256;

}  // namespace

int launch_fill(cudaStream_t s, int sms, float* out, float v, uint64_t n) {
  if (n == 0) return 0;
  fill_kernel<<<stream_grid(n, kThreads, sms, 8), kThreads, 0, s>>>(out, v, n); count_launch();
  return 0;
}

int launch_gen_affine(cudaStream_t s, int sms, float* out, uint64_t n, int64_t start, int32_t mul,
                      int32_t add, int32_t mod, int32_t sub) {
  if (n == 0) return 0;
  affine_kernel<<<stream_grid(n, kThreads, sms, 8), kThreads, 0, s>>>(out, n, start, mul, add, mod, sub); count_launch();
  return 0;
}

int launch_gen_f32(cudaStream_t s, int sms, float* out, uint64_t n, int32_t seed, int64_t offset,
                   int kind) {
  if (n == 0) return 0;
  gen_kernel<<<stream_grid(n, kThreads, sms, 8), kThreads, 0, s>>>(out, n, seed, offset, kind); count_launch();
  return 0;
}

extern "C" int mapal_gpu_iota_i32(MapalGpuCtx* ctx, int32_t* out, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (n > (1ull << 31)) return set_error(MAPAL_ERR_INVALID, "iota count exceeds i32 range");
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  DeviceSlot& d = ctx->dev[0];
  iota_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(out, n); count_launch();
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_fill_f32(MapalGpuCtx* ctx, float* out, float v, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  DeviceSlot& d = ctx->dev[0];
  fill_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(out, v, n); count_launch();
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_widen_i32_f32(MapalGpuCtx* ctx, const int32_t* in, float* out, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (n == 0) return 0;
  if (!in || !out) return set_error(MAPAL_ERR_INVALID, "null buffer");
  DeviceSlot& d = ctx->dev[0];
  widen_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(in, out, n); count_launch();
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_gen_affine_f32(MapalGpuCtx* ctx, float* out, uint64_t n, int64_t start,
                                        int32_t mul, int32_t add, int32_t mod, int32_t sub) {
  MAPAL_TRY(enter(ctx));
  if (mod == 0) return set_error(MAPAL_TRAP_DIV_ZERO, "mapal trap: div_zero");
  if (mod < 0) return set_error(MAPAL_ERR_UNSUPPORTED, "negative modulus");
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_gen_affine(d.stream, d.prof.sm_count, out, n, start, mul, add, mod, sub));
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_gen_f32(MapalGpuCtx* ctx, float* out, uint64_t n, int32_t seed,
                                 int64_t offset, int kind) {
  MAPAL_TRY(enter(ctx));
  if (kind != MAPAL_GEN_U11 && kind != MAPAL_GEN_U01) return set_error(MAPAL_ERR_INVALID, "bad kind");
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_gen_f32(d.stream, d.prof.sm_count, out, n, seed, offset, kind));
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_gen_index_i32(MapalGpuCtx* ctx, int32_t* out, uint64_t n, int32_t seed,
                                       int64_t offset, int32_t range) {
  MAPAL_TRY(enter(ctx));
  if (range <= 0) return set_error(MAPAL_ERR_INVALID, "range must be positive");
  if (n == 0) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  DeviceSlot& d = ctx->dev[0];
  gen_index_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(
      out, n, seed, offset, range); count_launch();
  return finish(ctx, 0, false);
}
