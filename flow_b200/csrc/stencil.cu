// stencil.cu — the FIR window site and the 3x3 conv2d site, bit-exact.
//
// Both are TileSites whose fold is a short dot product per output
// (benches/shapes/fir_1048576.mapal:10-12, conv2d_1024.mapal:11-15; records in
// crates/backends/llvm/tests/snapshots/tile_sites_pin__tile_record_content.snap).
// The reference evaluates each output as a per-thread loop over global memory
// (crates/backends/cuda/src/kernel.rs:2773-2886). Here a block stages its
// input window once into shared memory with asynchronous copies (all of a
// block's loads in flight at once) and each thread keeps a sliding window of
// inputs in registers. Every output keeps its exact fold order (acc from the
// seed, then acc + w[k]*x[...] for k ascending, each op rounded), so the
// results are bit-identical to the interpreter's.
//
// Each thread computes two outputs half a tile apart as one packed pair: two
// scalar rounded products and one packed rounded add (f32x2.cuh).
#include "common.cuh"
#include "cpasync.cuh"
#include "f32x2.cuh"

namespace {

// ---- FIR ---------------------------------------------------------------------

constexpr int kFirThreads = 64;
constexpr int kFirR = 8;                       // outputs per thread per lane
constexpr int kFirHalf = kFirThreads * kFirR;  // outputs per lane per block
constexpr int kFirTile = 2 * kFirHalf;         // outputs per block

__host__ __device__ constexpr int fir_wpad(int taps) { return (taps + 7) & ~7; }

// y[t] = fold_k(acc + w[k] * x[t + k]) from seed, t in [0, n_out).
__global__ void __launch_bounds__(kFirThreads) fir_kernel(const float* __restrict__ w, int taps,
                                                          const float* __restrict__ x, uint64_t x_len,
                                                          float* __restrict__ y, uint64_t n_out,
                                                          float seed) {
  extern __shared__ __align__(16) float fir_smem[];
  float* ws = fir_smem;                    // taps, zero-padded to a multiple of 8
  float* xs = fir_smem + fir_wpad(taps);   // x[t0 .. t0 + tile + taps + 16)
  const int span = (kFirTile + taps + 16 + 3) & ~3;  // staged floats, whole 16-byte groups
  const uint64_t t0 = (uint64_t)blockIdx.x * kFirTile;
  const bool xal = ((uintptr_t)x & 15) == 0, wal = ((uintptr_t)w & 15) == 0;

  for (int c = threadIdx.x; c < fir_wpad(taps) / 4; c += kFirThreads) {
    const int k = 4 * c;
    copy4(smem_u32(ws + k), w + (k < taps ? k : 0), taps - k, wal);
  }
  for (int c = threadIdx.x; c < span / 4; c += kFirThreads) {
    const uint64_t g = t0 + 4 * (uint64_t)c;
    const int nvalid = g < x_len ? (int)(x_len - g < 4 ? x_len - g : 4) : 0;
    copy4(smem_u32(xs + 4 * c), x + (nvalid > 0 ? g : 0), nvalid, xal);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();

  const int ba = threadIdx.x * kFirR, bb = kFirHalf + threadIdx.x * kFirR;
  f2 acc[kFirR];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int r = 0; r < kFirR; ++r) acc[r] = s2;
  float ca[kFirR], cb[kFirR], na[kFirR], nb[kFirR];
#pragma unroll
  for (int r = 0; r < kFirR; r += 4) {
    *reinterpret_cast<float4*>(ca + r) = *reinterpret_cast<const float4*>(xs + ba + r);
    *reinterpret_cast<float4*>(cb + r) = *reinterpret_cast<const float4*>(xs + bb + r);
  }
  for (int kg = 0; kg < taps; kg += kFirR) {
    float w8[kFirR];
#pragma unroll
    for (int r = 0; r < kFirR; r += 4) {
      *reinterpret_cast<float4*>(na + r) = *reinterpret_cast<const float4*>(xs + ba + kg + kFirR + r);
      *reinterpret_cast<float4*>(nb + r) = *reinterpret_cast<const float4*>(xs + bb + kg + kFirR + r);
      *reinterpret_cast<float4*>(w8 + r) = *reinterpret_cast<const float4*>(ws + kg + r);
    }
#pragma unroll
    for (int kk = 0; kk < kFirR; ++kk) {
      if (kg + kk < taps) {
#pragma unroll
        for (int r = 0; r < kFirR; ++r) {
          const float xa = (r + kk < kFirR) ? ca[r + kk] : na[r + kk - kFirR];
          const float xb = (r + kk < kFirR) ? cb[r + kk] : nb[r + kk - kFirR];
          acc[r] = f2_mac(acc[r], w8[kk], xa, w8[kk], xb);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kFirR; ++r) {
      ca[r] = na[r];
      cb[r] = nb[r];
    }
  }
#pragma unroll
  for (int r = 0; r < kFirR; ++r) {
    const uint64_t ta = t0 + ba + r, tb = t0 + bb + r;
    if (ta < n_out) y[ta] = f2_lo(acc[r]);
    if (tb < n_out) y[tb] = f2_hi(acc[r]);
  }
}

// ---- conv2d 3x3 ---------------------------------------------------------------

constexpr int kConvThreads = 64;         // one thread per column pair
constexpr int kConvHalf = kConvThreads;  // column pairs per block -> 128 columns
constexpr int kConvP = 8;                // output rows per thread
constexpr int kConvCols = 2 * kConvHalf;
constexpr int kConvPitch = kConvCols + 4;  // 130 used, 16-byte rows

// out[i, j] = fold_k(acc + w[k] * img[(i + k/3)*stride + j + k%3]) from seed.
__global__ void __launch_bounds__(kConvThreads) conv3x3_kernel(const float* __restrict__ w,
                                                               const float* __restrict__ img,
                                                               uint64_t img_len, uint64_t stride,
                                                               float* __restrict__ out, uint64_t rows,
                                                               uint64_t cols, float seed) {
  __shared__ __align__(16) float tile[kConvP + 2][kConvPitch];
  const uint64_t i0 = (uint64_t)blockIdx.y * kConvP;
  const uint64_t j0 = (uint64_t)blockIdx.x * kConvCols;
  const bool al = ((uintptr_t)img & 15) == 0 && (stride & 3) == 0;
  constexpr int kChunks = kConvPitch / 4;
  for (int e = threadIdx.x; e < (kConvP + 2) * kChunks; e += kConvThreads) {
    const int r = e / kChunks, c = 4 * (e % kChunks);
    const uint64_t row = i0 + r, col = j0 + c;
    int nvalid = 0;
    uint64_t g = 0;
    if (row < rows + 2 && col < cols + 2) {
      g = row * stride + col;
      const uint64_t lim_row = cols + 2 - col, lim_len = g < img_len ? img_len - g : 0;
      const uint64_t lim = lim_row < lim_len ? lim_row : lim_len;
      nvalid = (int)(lim < 4 ? lim : 4);
    }
    copy4(smem_u32(&tile[r][c]), img + (nvalid > 0 ? g : 0), nvalid, al);
  }
  cp_commit();
  float w9[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w9[k] = __ldg(w + k);
  cp_wait<0>();
  __syncthreads();

  const int c = threadIdx.x;
  f2 acc[kConvP];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int p = 0; p < kConvP; ++p) acc[p] = s2;
  // Input row r feeds output rows r-2..r (tap rows 2..0); walking r upward
  // applies each output's taps in ascending k (k = 3*dr + dc, dr = r - p).
#pragma unroll
  for (int r = 0; r < kConvP + 2; ++r) {
    const float a0 = tile[r][c], a1 = tile[r][c + 1], a2 = tile[r][c + 2];
    const float b0 = tile[r][kConvHalf + c], b1 = tile[r][kConvHalf + c + 1], b2 = tile[r][kConvHalf + c + 2];
#pragma unroll
    for (int dr = 0; dr < 3; ++dr) {
      const int p = r - dr;
      if (p >= 0 && p < kConvP) {
        acc[p] = f2_mac(acc[p], w9[3 * dr + 0], a0, w9[3 * dr + 0], b0);
        acc[p] = f2_mac(acc[p], w9[3 * dr + 1], a1, w9[3 * dr + 1], b1);
        acc[p] = f2_mac(acc[p], w9[3 * dr + 2], a2, w9[3 * dr + 2], b2);
      }
    }
  }
#pragma unroll
  for (int p = 0; p < kConvP; ++p) {
    const uint64_t i = i0 + p, ja = j0 + c, jb = j0 + kConvHalf + c;
    if (i < rows) {
      if (ja < cols) out[i * cols + ja] = f2_lo(acc[p]);
      if (jb < cols) out[i * cols + jb] = f2_hi(acc[p]);
    }
  }
}

}  // namespace

// Shared-memory bytes of one FIR block, 0 if the taps do not fit.
static size_t fir_smem_bytes(uint64_t taps) {
  if (taps > 8192) return 0;
  return sizeof(float) * ((size_t)fir_wpad((int)taps) + (((size_t)kFirTile + (size_t)taps + 16 + 3) & ~(size_t)3));
}

int launch_fir(cudaStream_t s, const float* w, uint64_t taps, const float* x, uint64_t x_len, float* y,
               uint64_t n_out, float seed) {
  size_t smem = fir_smem_bytes(taps);
  if (smem == 0) return MAPAL_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fir_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fir)");
  }
  uint64_t blocks = (n_out + kFirTile - 1) / kFirTile;
  if (blocks > 0x7fffffffull) return MAPAL_ERR_UNSUPPORTED;
  fir_kernel<<<(unsigned)blocks, kFirThreads, smem, s>>>(w, (int)taps, x, x_len, y, n_out, seed); count_launch();
  return 0;
}

int launch_conv3x3(cudaStream_t s, const float* w, const float* img, uint64_t img_len, uint64_t stride,
                   float* out, uint64_t rows, uint64_t cols, float seed) {
  dim3 grid((unsigned)((cols + kConvCols - 1) / kConvCols), (unsigned)((rows + kConvP - 1) / kConvP));
  if ((cols + kConvCols - 1) / kConvCols > 0x7fffffffull || (rows + kConvP - 1) / kConvP > 65535)
    return MAPAL_ERR_UNSUPPORTED;
  conv3x3_kernel<<<grid, kConvThreads, 0, s>>>(w, img, img_len, stride, out, rows, cols, seed); count_launch();
  return 0;
}
