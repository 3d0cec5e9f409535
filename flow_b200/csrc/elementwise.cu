// elementwise.cu — streaming sites: saxpy / zip-map, gather, move sites.
//
// Rung 0 in the reference launches one thread per element with scalar 4-byte
// accesses (crates/backends/cuda/src/kernel.rs:1156-1333, grid_expr :913) and,
// for saxpy, two kernels with a materialised pair array in between (zip then
// map). Here each site is one kernel moving 128-bit vectors, sized to keep
// every SM's memory pipeline full, with streaming cache hints (the data is
// touched once). All f32 arithmetic is separately rounded (__fmul_rn /
// __fadd_rn never contract into an FMA), matching eval.rs:572-585.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ float saxpy1(float a, float x, float y) { return __fadd_rn(__fmul_rn(a, x), y); }

// Two float4 per thread per trip keeps 32 bytes of loads in flight per
// operand per thread; with 2048 threads per SM that covers HBM latency.
__global__ void __launch_bounds__(kThreads) saxpy_vec_kernel(float a, const float4* __restrict__ x,
                                                             const float4* __restrict__ y0,
                                                             float4* __restrict__ y, uint64_t n4) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    float4 xa = ld_stream(x + i), xb = ld_stream(x + i + stride);
    float4 ya = ld_stream(y0 + i), yb = ld_stream(y0 + i + stride);
    float4 ra, rb;
    ra.x = saxpy1(a, xa.x, ya.x); ra.y = saxpy1(a, xa.y, ya.y);
    ra.z = saxpy1(a, xa.z, ya.z); ra.w = saxpy1(a, xa.w, ya.w);
    rb.x = saxpy1(a, xb.x, yb.x); rb.y = saxpy1(a, xb.y, yb.y);
    rb.z = saxpy1(a, xb.z, yb.z); rb.w = saxpy1(a, xb.w, yb.w);
    st_stream(y + i, ra);
    st_stream(y + i + stride, rb);
  }
  if (i < n4) {
    float4 xa = ld_stream(x + i), ya = ld_stream(y0 + i), ra;
    ra.x = saxpy1(a, xa.x, ya.x); ra.y = saxpy1(a, xa.y, ya.y);
    ra.z = saxpy1(a, xa.z, ya.z); ra.w = saxpy1(a, xa.w, ya.w);
    st_stream(y + i, ra);
  }
}

__global__ void saxpy_scalar_kernel(float a, const float* __restrict__ x, const float* __restrict__ y0,
                                    float* __restrict__ y, uint64_t lo, uint64_t n) {
  for (uint64_t i = lo + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = saxpy1(a, x[i], y0[i]);
}

__device__ __forceinline__ float zop(int op, float x, float y) {
  switch (op) {
    case MAPAL_OP_ADD: return __fadd_rn(x, y);
    case MAPAL_OP_SUB: return __fsub_rn(x, y);
    case MAPAL_OP_MUL: return __fmul_rn(x, y);
    case MAPAL_OP_DIV: return __fdiv_rn(x, y);
    default: return fmodf(x, y);  // Rust's f32 `%` is C fmod (exact)
  }
}

template <int OP>
__global__ void __launch_bounds__(kThreads) zip_vec_kernel(const float4* __restrict__ x,
                                                           const float4* __restrict__ y,
                                                           float4* __restrict__ out, uint64_t n4) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float4 a = ld_stream(x + i), b = ld_stream(y + i), r;
    r.x = zop(OP, a.x, b.x); r.y = zop(OP, a.y, b.y); r.z = zop(OP, a.z, b.z); r.w = zop(OP, a.w, b.w);
    st_stream(out + i, r);
  }
}

__global__ void zip_scalar_kernel(int op, const float* __restrict__ x, const float* __restrict__ y,
                                  float* __restrict__ out, uint64_t lo, uint64_t n) {
  for (uint64_t i = lo + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = zop(op, x[i], y[i]);
}

// Gather with the Index guard (kernel.rs:2655-2663): the 32-bit index is
// widened with sign and compared two-sided; a miss stores kind+1 = 2 into
// the trap flag and skips the element. idx/out move as int4/float4; the x
// reads are data-dependent 4-byte loads through the read-only path.
__device__ __forceinline__ bool in_range(int4 j, int64_t n_x) {
  return (int64_t)j.x >= 0 && (int64_t)j.x < n_x && (int64_t)j.y >= 0 && (int64_t)j.y < n_x &&
         (int64_t)j.z >= 0 && (int64_t)j.z < n_x && (int64_t)j.w >= 0 && (int64_t)j.w < n_x;
}

// Random x reads: read-only path, no L1 allocation (a gathered line is
// rarely reused by the same SM).
__device__ __forceinline__ float ld_gather(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float4 gather4(const float* __restrict__ x, int4 j) {
  return make_float4(ld_gather(x + j.x), ld_gather(x + j.y), ld_gather(x + j.z), ld_gather(x + j.w));
}

// Two index groups per trip, so eight independent x reads are in flight per
// thread behind the two index loads.
__global__ void __launch_bounds__(kThreads) gather_vec_kernel(const float* __restrict__ x, int64_t n_x,
                                                              const int4* __restrict__ idx,
                                                              float4* __restrict__ out, uint64_t n4,
                                                              unsigned* trap) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    const int4 ja = __ldcs(idx + i), jb = __ldcs(idx + i + stride);
    const bool oka = in_range(ja, n_x), okb = in_range(jb, n_x);
    if (!oka || !okb) *trap = 2u;
    if (oka) st_stream(out + i, gather4(x, ja));
    if (okb) st_stream(out + i + stride, gather4(x, jb));
  }
  if (i < n4) {
    const int4 ja = __ldcs(idx + i);
    if (in_range(ja, n_x))
      st_stream(out + i, gather4(x, ja));
    else
      *trap = 2u;
  }
}

__global__ void gather_scalar_kernel(const float* __restrict__ x, int64_t n_x,
                                     const int32_t* __restrict__ idx, float* __restrict__ out,
                                     uint64_t lo, uint64_t n, unsigned* trap) {
  for (uint64_t i = lo + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    int64_t j = (int64_t)idx[i];
    if (j < 0 || j >= n_x) {
      *trap = 2u;
      continue;
    }
    out[i] = __ldg(x + j);
  }
}

// Transpose-shaped move site (cq == 1): out[r][w] = in[w*cr + r] for an
// output of `rows` x `width`. Square tiles through shared memory padded by
// one column, so both the read (along r) and the write (along w) coalesce;
// each thread issues all of its loads before its first shared store. Large
// sites use 64x64 tiles (64x4 threads; 0.81-0.82 of the copy rate at 4096^2
// and 8192^2 on B200 against 0.69-0.72 with 32x32), small ones 32x32 tiles
// (32x8 threads: at 1024^2 the 64x64 grid is too short to fill the SMs).
template <int kTile, int kRowsPerPass>
__global__ void __launch_bounds__(kTile* kRowsPerPass) transpose_kernel(const float* __restrict__ in,
                                                                        float* __restrict__ out,
                                                                        uint64_t rows, uint64_t width,
                                                                        uint64_t cr) {
  __shared__ float tile[kTile][kTile + 1];
  const uint64_t r0 = (uint64_t)blockIdx.x * kTile;  // output row block (input column block)
  const uint64_t w0 = (uint64_t)blockIdx.y * kTile;  // output column block (input row block)
  const int tx = threadIdx.x, ty = threadIdx.y;
  float v[kTile / kRowsPerPass];
#pragma unroll
  for (int p = 0; p < kTile / kRowsPerPass; ++p) {
    const uint64_t w = w0 + ty + kRowsPerPass * p, r = r0 + tx;
    v[p] = (w < width && r < rows) ? __ldcs(in + w * cr + r) : 0.0f;
  }
#pragma unroll
  for (int p = 0; p < kTile / kRowsPerPass; ++p) tile[ty + kRowsPerPass * p][tx] = v[p];
  __syncthreads();
#pragma unroll
  for (int p = 0; p < kTile / kRowsPerPass; ++p) {
    const uint64_t r = r0 + ty + kRowsPerPass * p, w = w0 + tx;
    if (r < rows && w < width) __stcs(out + r * width + w, tile[tx][ty + kRowsPerPass * p]);
  }
}

template <int kTile, int kRowsPerPass>
int launch_transpose(cudaStream_t s, const float* in, float* out, uint64_t rows, uint64_t width, uint64_t cr) {
  dim3 grid((unsigned)((rows + kTile - 1) / kTile), (unsigned)((width + kTile - 1) / kTile));
  if (grid.y > 65535 || (rows + kTile - 1) / kTile > 0x7fffffffull)
    return set_error(MAPAL_ERR_UNSUPPORTED, "transpose too large");
  transpose_kernel<kTile, kRowsPerPass><<<grid, dim3(kTile, kRowsPerPass), 0, s>>>(in, out, rows, width, cr);
  count_launch();
  return 0;
}

// Any other move site: one thread per output element (addresses validated
// on the host, so no guard is needed).
__global__ void move_generic_kernel(const float* __restrict__ in, float* __restrict__ out, uint64_t n,
                                    uint64_t width, uint64_t cq, uint64_t cr) {
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < n;
       t += (uint64_t)gridDim.x * blockDim.x)
    out[t] = in[cq * (t / width) + cr * (t % width)];
}

}  // namespace

int launch_saxpy(cudaStream_t s, int sms, float a, const float* x, const float* y0, float* y,
                 uint64_t n) {
  if (n == 0) return 0;
  uint64_t done = 0;
  if (aligned16(x) && aligned16(y0) && aligned16(y)) {
    uint64_t n4 = n / 4;
    if (n4) {
      saxpy_vec_kernel<<<stream_grid((n4 + 1) / 2, kThreads, sms, 8), kThreads, 0, s>>>(
          a, (const float4*)x, (const float4*)y0, (float4*)y, n4); count_launch();
      done = n4 * 4;
    }
  }
  if (done < n) {
    saxpy_scalar_kernel<<<stream_grid(n - done, kThreads, sms, 8), kThreads, 0, s>>>(a, x, y0, y, done, n);
    count_launch();
  }
  return 0;
}

int launch_gather(cudaStream_t s, int sms, const float* x, uint64_t n_x, const int32_t* idx,
                  float* out, uint64_t n, unsigned* trap) {
  if (n == 0) return 0;
  uint64_t done = 0;
  if (aligned16(idx) && aligned16(out)) {
    uint64_t n4 = n / 4;
    if (n4) {
      // one index vector per thread until the grid reaches its cap (8 blocks
      // per SM): at 2^20 the random reads of more threads overlap (B200:
      // 7.22 -> 6.58 us); larger n is capped either way
      gather_vec_kernel<<<stream_grid(n4, kThreads, sms, 8), kThreads, 0, s>>>(
          x, (int64_t)n_x, (const int4*)idx, (float4*)out, n4, trap); count_launch();
      done = n4 * 4;
    }
  }
  if (done < n) {
    gather_scalar_kernel<<<stream_grid(n - done, kThreads, sms, 8), kThreads, 0, s>>>(
        x, (int64_t)n_x, idx, out, done, n, trap);
    count_launch();
  }
  return 0;
}

extern "C" int mapal_gpu_map_saxpy(MapalGpuCtx* ctx, float a, const float* x, const float* y0,
                                   float* y, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (n == 0) return 0;
  if (!x || !y0 || !y) return set_error(MAPAL_ERR_INVALID, "null buffer");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_saxpy(d.stream, d.prof.sm_count, a, x, y0, y, n));
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_zip_map_f32(MapalGpuCtx* ctx, int op, const float* x, const float* y,
                                     float* out, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (op < MAPAL_OP_ADD || op > MAPAL_OP_MOD) return set_error(MAPAL_ERR_INVALID, "unknown op");
  if (n == 0) return 0;
  if (!x || !y || !out) return set_error(MAPAL_ERR_INVALID, "null buffer");
  DeviceSlot& d = ctx->dev[0];
  int sms = d.prof.sm_count;
  uint64_t done = 0;
  if (aligned16(x) && aligned16(y) && aligned16(out) && n >= 4) {
    uint64_t n4 = n / 4;
    unsigned g = stream_grid(n4, kThreads, sms, 8);
    const float4 *x4 = (const float4*)x, *y4 = (const float4*)y;
    float4* o4 = (float4*)out;
    switch (op) {
      case MAPAL_OP_ADD: zip_vec_kernel<MAPAL_OP_ADD><<<g, kThreads, 0, d.stream>>>(x4, y4, o4, n4); count_launch(); break;
      case MAPAL_OP_SUB: zip_vec_kernel<MAPAL_OP_SUB><<<g, kThreads, 0, d.stream>>>(x4, y4, o4, n4); count_launch(); break;
      case MAPAL_OP_MUL: zip_vec_kernel<MAPAL_OP_MUL><<<g, kThreads, 0, d.stream>>>(x4, y4, o4, n4); count_launch(); break;
      case MAPAL_OP_DIV: zip_vec_kernel<MAPAL_OP_DIV><<<g, kThreads, 0, d.stream>>>(x4, y4, o4, n4); count_launch(); break;
      default: zip_vec_kernel<MAPAL_OP_MOD><<<g, kThreads, 0, d.stream>>>(x4, y4, o4, n4); count_launch(); break;
    }
    done = n4 * 4;
  }
  if (done < n) {
    zip_scalar_kernel<<<stream_grid(n - done, kThreads, sms, 8), kThreads, 0, d.stream>>>(op, x, y, out,
                                                                                        done, n);
    count_launch();
  }
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_gather(MapalGpuCtx* ctx, const float* x, uint64_t n_x, const int32_t* idx,
                                float* out, uint64_t n) {
  MAPAL_TRY(enter(ctx));
  if (n == 0) return 0;
  if (!x && n_x) return set_error(MAPAL_ERR_INVALID, "x is null");
  if (!idx || !out) return set_error(MAPAL_ERR_INVALID, "null buffer");
  DeviceSlot& d = ctx->dev[0];
  MAPAL_TRY(launch_gather(d.stream, d.prof.sm_count, x, n_x, idx, out, n, d.trap));
  return finish(ctx, 0, true);
}

extern "C" int mapal_gpu_transpose(MapalGpuCtx* ctx, const MapalMoveSite* site, const float* in,
                                   float* out) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  const uint64_t rows = site->rows, width = site->width;
  if (rows == 0 || width == 0) return 0;
  if (!in || !out) return set_error(MAPAL_ERR_INVALID, "null buffer");
  // The read address is affine with non-negative coefficients, so its maximum
  // is at the last row and last column: when that is in range every read is,
  // else the cell holding it traps index_oob (eval.rs:655-669) and, as the
  // interpreter evaluates every cell, so does the program.
  unsigned __int128 max_addr =
      (unsigned __int128)site->cq * (rows - 1) + (unsigned __int128)site->cr * (width - 1);
  if (max_addr >= site->len) return set_error(MAPAL_TRAP_INDEX_OOB, "mapal trap: index_oob");
  DeviceSlot& d = ctx->dev[0];
  if (site->cq == 1) {
    if (rows * width >= (4ull << 20))
      MAPAL_TRY((launch_transpose<64, 4>(d.stream, in, out, rows, width, site->cr)));
    else
      MAPAL_TRY((launch_transpose<32, 8>(d.stream, in, out, rows, width, site->cr)));
  } else {
    uint64_t n = rows * width;
    move_generic_kernel<<<stream_grid(n, kThreads, d.prof.sm_count, 8), kThreads, 0, d.stream>>>(
        in, out, n, width, site->cq, site->cr); count_launch();
  }
  return finish(ctx, 0, false);
}
