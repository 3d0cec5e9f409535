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
// Each thread computes pairs of outputs half a tile apart as packed values
// (f32x2.cuh): FIR forms both rounded products with one packed FMA whose
// addend is a run-time -0.0; conv2d uses two scalar rounded products; both
// accumulate with one packed rounded add.
#include "common.cuh"
#include "cpasync.cuh"
#include "f32x2.cuh"

namespace {

// ---- FIR ---------------------------------------------------------------------
//
// A block computes kFirTile consecutive outputs as two lanes of kFirHalf: a
// thread owns outputs j..j+3 of lane a and the same offsets of lane b, and
// advances each (lane a, lane b) output pair as one packed value. The input
// window is staged in shared memory interleaved, pair p = (x[t0 + p],
// x[t0 + kFirHalf + p]), and every tap is staged as the splat pair (w, w), so
// a 16-byte shared load yields two ready operand pairs and a MAC pair is one
// packed FMA with a run-time -0.0 addend (the two rounded products) plus one
// packed add (f32x2.cuh, f2_mac_z). The loads of the next tap group are issued
// a group ahead, and the 16-byte units are split into even and odd arrays so
// the units a warp reads in one instruction are consecutive (no bank
// conflicts).

constexpr int kFirThreads = 128;
constexpr int kFirR = 4;                       // outputs per thread per lane
constexpr int kFirHalf = kFirThreads * kFirR;  // outputs per lane per block
constexpr int kFirTile = 2 * kFirHalf;         // outputs per block

__host__ __device__ constexpr int fir_wpad(int taps) { return (taps + 3) & ~3; }
// pairs staged per block (a multiple of 4): the last thread's prefetch reads up
// to pair 4*(kFirThreads-1) + wpad + 7
__host__ __device__ constexpr int fir_npairs(int taps) { return kFirHalf + fir_wpad(taps) + 8; }

// y[t] = fold_k(acc + w[k] * x[t + k]) from seed, t in [0, n_out).
__global__ void __launch_bounds__(kFirThreads) fir_kernel(const float* __restrict__ w, int taps,
                                                          const float* __restrict__ x, uint64_t x_len,
                                                          float* __restrict__ y, uint64_t n_out,
                                                          float seed, float neg_zero) {
  extern __shared__ __align__(16) float fir_smem[];
  const int wpad = fir_wpad(taps), npairs = fir_npairs(taps);
  float* wp = fir_smem;                   // [wpad + 4] splat pairs (w[k], w[k]), zero past the taps
  float* xe = fir_smem + 2 * (wpad + 4);  // even 16-byte units of the pair array
  float* xo = xe + npairs;                // odd units
  const uint64_t t0 = (uint64_t)blockIdx.x * kFirTile;

  for (int k = threadIdx.x; k < wpad + 4; k += kFirThreads) {
    const bool ok = k < taps;
    cp_async4(smem_u32(wp + 2 * k), w + (ok ? k : 0), ok);
    cp_async4(smem_u32(wp + 2 * k + 1), w + (ok ? k : 0), ok);
  }
  // pair p = (x[t0 + p], x[t0 + kFirHalf + p]) lives in unit u = p/2 (two
  // pairs per 16 bytes); even units go to xe, odd ones to xo, so the units a
  // warp reads in one instruction are consecutive.
  for (int p = threadIdx.x; p < npairs; p += kFirThreads) {
    const uint64_t ga = t0 + p, gb = t0 + kFirHalf + p;
    const int u = p >> 1;
    float* dst = ((u & 1) ? xo : xe) + 4 * (u >> 1) + 2 * (p & 1);
    cp_async4(smem_u32(dst), x + (ga < x_len ? ga : 0), ga < x_len);
    cp_async4(smem_u32(dst + 1), x + (gb < x_len ? gb : 0), gb < x_len);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();

  const f2 z2 = f2_splat(neg_zero);  // -0.0, unknown to the compiler: see f2_mac_z
  const ulonglong2* ev = reinterpret_cast<const ulonglong2*>(xe) + threadIdx.x;
  const ulonglong2* ov = reinterpret_cast<const ulonglong2*>(xo) + threadIdx.x;
  const ulonglong2* wv = reinterpret_cast<const ulonglong2*>(wp);
  f2 acc[kFirR];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int r = 0; r < kFirR; ++r) acc[r] = s2;
  f2 win[8];  // pairs 4*tid + kg .. 4*tid + kg + 7
  {
    const ulonglong2 c0 = ev[0], c1 = ov[0];
    win[0] = c0.x, win[1] = c0.y, win[2] = c1.x, win[3] = c1.y;
  }
  // loads for the next tap group are issued one group ahead
  ulonglong2 pe = ev[1], po = ov[1], pw0 = wv[0], pw1 = wv[1];
  for (int kg = 0; kg < taps; kg += 4) {
    win[4] = pe.x, win[5] = pe.y, win[6] = po.x, win[7] = po.y;
    const f2 wk[4] = {pw0.x, pw0.y, pw1.x, pw1.y};
    pe = ev[kg / 4 + 2], po = ov[kg / 4 + 2], pw0 = wv[kg / 2 + 2], pw1 = wv[kg / 2 + 3];
    if (kg + 4 <= taps) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int r = 0; r < kFirR; ++r) acc[r] = f2_mac_z(acc[r], wk[kk], win[r + kk], z2);
    } else {
      // the last, partial tap group: exactly the remaining taps, in order
#pragma unroll
      for (int kk = 0; kk < 3; ++kk)
        if (kk < taps - kg)
#pragma unroll
          for (int r = 0; r < kFirR; ++r) acc[r] = f2_mac_z(acc[r], wk[kk], win[r + kk], z2);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) win[r] = win[r + 4];
  }
  const uint64_t j = t0 + (uint64_t)kFirR * threadIdx.x;
#pragma unroll
  for (int r = 0; r < kFirR; ++r) {
    if (j + r < n_out) y[j + r] = f2_lo(acc[r]);
    if (j + kFirHalf + r < n_out) y[j + kFirHalf + r] = f2_hi(acc[r]);
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
  return sizeof(float) * 2 * ((size_t)fir_wpad((int)taps) + 4 + (size_t)fir_npairs((int)taps));
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
  fir_kernel<<<(unsigned)blocks, kFirThreads, smem, s>>>(w, (int)taps, x, x_len, y, n_out, seed, -0.0f);
  count_launch();
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
