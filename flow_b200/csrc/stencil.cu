// stencil.cu — the FIR window site and the 3x3 conv2d site, bit-exact.
//
// Both are TileSites whose fold is a short dot product per output
// (benches/shapes/fir_1048576.mapal:10-12, conv2d_1024.mapal:11-15; records in
// crates/backends/llvm/tests/snapshots/tile_sites_pin__tile_record_content.snap).
// The reference evaluates each output as a per-thread loop over global memory
// (crates/backends/cuda/src/kernel.rs:2773-2886). Here a block stages its
// input window once in shared memory and each thread keeps a sliding window
// of inputs in registers. Every output keeps its exact fold order (acc from
// the seed, then acc + w[k]*x[...] for k ascending, each op rounded), so the
// results are bit-identical to the interpreter's.
//
// Two outputs that are half a tile apart are computed as one packed pair
// (f32x2): shared memory holds the input as pairs (x[j], x[j + half]), so
// one 64-bit load feeds both lanes; the two products are scalar rounded
// multiplies and one packed rounded add advances both accumulators.
#include "common.cuh"
#include "f32x2.cuh"

namespace {

// ---- FIR ---------------------------------------------------------------------

constexpr int kFirThreads = 64;
constexpr int kFirR = 8;                              // outputs per thread per lane
constexpr int kFirHalf = kFirThreads * kFirR;         // outputs per lane per block
constexpr int kFirTile = 2 * kFirHalf;                // outputs per block

// y[t] = fold_k(acc + w[k] * x[t + k]) from seed, t in [0, n_out).
__global__ void __launch_bounds__(kFirThreads) fir_kernel(const float* __restrict__ w, int taps,
                                                          const float* __restrict__ x, uint64_t x_len,
                                                          float* __restrict__ y, uint64_t n_out,
                                                          float seed) {
  extern __shared__ __align__(16) unsigned char fir_smem[];
  float* ws = reinterpret_cast<float*>(fir_smem);  // w[k]
  const int span = kFirHalf + taps + kFirR;        // window pairs staged (tail padded)
  f2* xs = reinterpret_cast<f2*>(ws + ((taps + 1) & ~1));  // (x[t0 + j], x[t0 + half + j])
  const uint64_t t0 = (uint64_t)blockIdx.x * kFirTile;

  for (int k = threadIdx.x; k < taps; k += kFirThreads) ws[k] = w[k];
  for (int j = threadIdx.x; j < span; j += kFirThreads) {
    uint64_t ia = t0 + j, ib = t0 + kFirHalf + j;
    float va = ia < x_len ? __ldg(x + ia) : 0.0f;
    float vb = ib < x_len ? __ldg(x + ib) : 0.0f;
    xs[j] = f2_pack(va, vb);
  }
  __syncthreads();

  const int base = threadIdx.x * kFirR;
  f2 acc[kFirR];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int r = 0; r < kFirR; ++r) acc[r] = s2;
  f2 cur[kFirR], nxt[kFirR];
#pragma unroll
  for (int r = 0; r < kFirR; ++r) cur[r] = xs[base + r];
  for (int kg = 0; kg < taps; kg += kFirR) {
#pragma unroll
    for (int r = 0; r < kFirR; ++r) nxt[r] = xs[base + kg + kFirR + r];
#pragma unroll
    for (int kk = 0; kk < kFirR; ++kk) {
      if (kg + kk < taps) {
        const float wk = ws[kg + kk];
#pragma unroll
        for (int r = 0; r < kFirR; ++r) {
          const f2 xv = (r + kk < kFirR) ? cur[r + kk] : nxt[r + kk - kFirR];
          acc[r] = f2_mac(acc[r], wk, f2_lo(xv), wk, f2_hi(xv));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kFirR; ++r) cur[r] = nxt[r];
  }
#pragma unroll
  for (int r = 0; r < kFirR; ++r) {
    uint64_t ta = t0 + base + r, tb = t0 + kFirHalf + base + r;
    if (ta < n_out) y[ta] = f2_lo(acc[r]);
    if (tb < n_out) y[tb] = f2_hi(acc[r]);
  }
}

// ---- conv2d 3x3 ---------------------------------------------------------------

constexpr int kConvThreads = 64;   // one thread per column pair
constexpr int kConvHalf = kConvThreads;  // column pairs per block -> 128 columns
constexpr int kConvP = 8;          // output rows per thread
constexpr int kConvCols = 2 * kConvHalf;

// out[i, j] = fold_k(acc + w[k] * img[(i + k/3)*stride + j + k%3]) from seed.
__global__ void __launch_bounds__(kConvThreads) conv3x3_kernel(const float* __restrict__ w,
                                                               const float* __restrict__ img,
                                                               uint64_t img_len, uint64_t stride,
                                                               float* __restrict__ out, uint64_t rows,
                                                               uint64_t cols, float seed) {
  __shared__ f2 tile[kConvP + 2][kConvHalf + 2];
  const uint64_t i0 = (uint64_t)blockIdx.y * kConvP;
  const uint64_t j0 = (uint64_t)blockIdx.x * kConvCols;
  for (int e = threadIdx.x; e < (kConvP + 2) * (kConvHalf + 2); e += kConvThreads) {
    int r = e / (kConvHalf + 2), c = e % (kConvHalf + 2);
    uint64_t row = i0 + r;
    uint64_t ca = j0 + c, cb = j0 + kConvHalf + c;
    uint64_t aa = row * stride + ca, ab = row * stride + cb;
    bool ra = row < rows + 2 && ca < cols + 2 && aa < img_len;
    bool rb = row < rows + 2 && cb < cols + 2 && ab < img_len;
    tile[r][c] = f2_pack(ra ? __ldg(img + aa) : 0.0f, rb ? __ldg(img + ab) : 0.0f);
  }
  float w9[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w9[k] = __ldg(w + k);
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
    const f2 v0 = tile[r][c], v1 = tile[r][c + 1], v2 = tile[r][c + 2];
#pragma unroll
    for (int dr = 0; dr < 3; ++dr) {
      const int p = r - dr;
      if (p >= 0 && p < kConvP) {
        acc[p] = f2_mac(acc[p], w9[3 * dr + 0], f2_lo(v0), w9[3 * dr + 0], f2_hi(v0));
        acc[p] = f2_mac(acc[p], w9[3 * dr + 1], f2_lo(v1), w9[3 * dr + 1], f2_hi(v1));
        acc[p] = f2_mac(acc[p], w9[3 * dr + 2], f2_lo(v2), w9[3 * dr + 2], f2_hi(v2));
      }
    }
  }
#pragma unroll
  for (int p = 0; p < kConvP; ++p) {
    uint64_t i = i0 + p, ja = j0 + c, jb = j0 + kConvHalf + c;
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
  return sizeof(float) * (size_t)((taps + 1) & ~1ull) + sizeof(f2) * (size_t)(kFirHalf + taps + kFirR);
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
  fir_kernel<<<(unsigned)blocks, kFirThreads, smem, s>>>(w, (int)taps, x, x_len, y, n_out, seed);
  return 0;
}

int launch_conv3x3(cudaStream_t s, const float* w, const float* img, uint64_t img_len, uint64_t stride,
                   float* out, uint64_t rows, uint64_t cols, float seed) {
  dim3 grid((unsigned)((cols + kConvCols - 1) / kConvCols), (unsigned)((rows + kConvP - 1) / kConvP));
  if ((cols + kConvCols - 1) / kConvCols > 0x7fffffffull || (rows + kConvP - 1) / kConvP > 65535)
    return MAPAL_ERR_UNSUPPORTED;
  conv3x3_kernel<<<grid, kConvThreads, 0, s>>>(w, img, img_len, stride, out, rows, cols, seed);
  return 0;
}
