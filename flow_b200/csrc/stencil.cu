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
// addend is a run-time -0.0 (so does conv2d); both accumulate with one packed
// rounded add.
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
// TAPS > 0: the tap count is a compile-time constant and the tap loop fully
// unrolls (no register moves to slide the window; 64 taps: +7-9 % on B200).
template <int TAPS>
__global__ void __launch_bounds__(kFirThreads) fir_kernel(const float* __restrict__ w, int taps_rt,
                                                          const float* __restrict__ x, uint64_t x_len,
                                                          float* __restrict__ y, uint64_t n_out,
                                                          float seed, float neg_zero) {
  const int taps = TAPS ? TAPS : taps_rt;
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
#pragma unroll
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

constexpr int kConvThreads = 128;             // one thread per column pair (c, c + 128)
constexpr int kConvHalf = kConvThreads;
constexpr int kConvCols = 2 * kConvHalf;           // output columns per block
constexpr int kConvPitch = kConvCols + 8;          // 258 used after an alignment shift of up to 3
constexpr int kConvChunks = (kConvCols + 2 + 3 + 3) / 4;  // 16-byte chunks that cover a staged row

// Shift (in floats) of a row's first needed element above the 16-byte
// boundary below it: the staged row starts at that boundary.
__device__ __forceinline__ int conv_shift(const float* p) { return (int)(((uintptr_t)p >> 2) & 3); }

// Wait for phase 0 of a shared mbarrier, giving up after 1 s.
__device__ __forceinline__ bool conv_bar_wait(uint64_t* bar) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar))
        : "memory");
    if (ok) return true;
    if ((i & 63) == 63) {
      uint64_t t;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
      if (t - t0 > 1000000000ull) return false;
    }
  }
}

// out[i, j] = fold_k(acc + w[k] * img[(i + k/3)*stride + j + k%3]) from seed,
// for a strip of P output rows x kConvCols columns. The P + 2 input rows are
// staged (a warp per row) by 16-byte cp.async whatever the stride (elements outside the needed
// span are zero-filled and never read); each thread then walks the rows once,
// keeping P packed accumulators for its two columns, and every MAC pair is one
// packed FMA with a run-time -0.0 addend plus one packed add (f32x2.cuh).
template <int P>
__global__ void __launch_bounds__(kConvThreads) conv3x3_kernel(const float* __restrict__ w,
                                                               const float* __restrict__ img,
                                                               uint64_t img_len, uint64_t stride,
                                                               float* __restrict__ out, uint64_t rows,
                                                               uint64_t cols, float seed, float neg_zero,
                                                               unsigned* flag) {
  __shared__ __align__(16) float tile[P + 2][kConvPitch];
  const uint64_t i0 = (uint64_t)blockIdx.y * P;
  const uint64_t j0 = (uint64_t)blockIdx.x * kConvCols;
  const uint64_t need = cols + 2 - j0 < (uint64_t)(kConvCols + 2) ? cols + 2 - j0 : (uint64_t)(kConvCols + 2);
  const float* const img_end = img + img_len;
  __shared__ int shs[P + 2];  // each staged row's alignment shift
  __shared__ __align__(8) uint64_t bar;
  // Staging. A row whose 16-byte aligned span [rowp - sh, ...) lies inside
  // the image goes as one bulk copy (cp.async.bulk, completing on `bar`),
  // issued by thread 0; the image stride need not be a multiple of 4 floats,
  // which a 2-D tensor map would require. A row at the image's edge (its
  // aligned span would leave the array) is staged by a warp with 16- or
  // 4-byte cp.async, zero-filling what lies outside (never read).
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    uint32_t total = 0;
    uint32_t span[P + 2];
#pragma unroll
    for (int r = 0; r < P + 2; ++r) {
      const float* rowp = img + (i0 + r) * stride + j0;
      const int sh = conv_shift(rowp);
      shs[r] = sh;
      const float* lo = rowp - sh;
      const uint32_t nf = ((uint32_t)(sh + need) + 3u) & ~3u;  // floats, a whole number of 16-byte units
      span[r] = (i0 + r < rows + 2 && lo >= img && lo + nf <= img_end) ? nf * 4u : 0u;
      total += span[r];
    }
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&bar)), "r"(total)
                 : "memory");
#pragma unroll
    for (int r = 0; r < P + 2; ++r) {
      if (span[r] == 0) continue;
      const float* lo = img + (i0 + r) * stride + j0 - shs[r];
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(&tile[r][0])),
          "l"(lo), "r"(span[r]), "r"(smem_u32(&bar))
          : "memory");
    }
  }
  __syncthreads();  // shs[] and the barrier are set
  for (int r = warp; r < P + 2; r += kConvThreads / 32) {
    if (i0 + r >= rows + 2) continue;  // feeds no stored output: left unstaged
    const float* rowp = img + (i0 + r) * stride + j0;  // first needed element of staged row r
    const int sh = shs[r];
    const float* lo = rowp - sh;
    const uint32_t nf = ((uint32_t)(sh + need) + 3u) & ~3u;
    if (lo >= img && lo + nf <= img_end) continue;  // a bulk-copied row
    const float* hi = rowp + need < img_end ? rowp + need : img_end;
    for (int ch = lane; ch < kConvChunks; ch += 32) {
      const float* e0 = lo + 4 * ch;
      const uint32_t dst = smem_u32(&tile[r][4 * ch]);
      if (e0 >= rowp && e0 + 4 <= hi) {
        cp_async16(dst, e0, true);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const bool ok = e0 + q >= rowp && e0 + q < hi;
          cp_async4(dst + 4 * q, ok ? e0 + q : img, ok);
        }
      }
    }
  }
  cp_commit();
  f2 w9[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w9[k] = f2_splat(__ldg(w + k));
  const f2 z2 = f2_splat(neg_zero);  // -0.0, unknown to the compiler: see f2_mac_z
  cp_wait<0>();
  // Bounded wait for the bulk copies: 1 s on %globaltimer, then the launch
  // flags a timeout and the block skips its outputs (after a second bounded
  // wait, so no copy is still writing this block's shared memory at exit).
  bool landed = conv_bar_wait(&bar);
  if (!landed) {
    if (threadIdx.x == 0) atomicOr(flag, 0x100u);
    conv_bar_wait(&bar);
  }
  __syncthreads();
  if (!landed) return;

  const int c = threadIdx.x;
  f2 acc[P];
  const f2 s2 = f2_splat(seed);
#pragma unroll
  for (int p = 0; p < P; ++p) acc[p] = s2;
  // Input row r feeds output rows r-2..r (tap rows 2..0); walking r upward
  // applies each output's taps in ascending k (k = 3*dr + dc, dr = r - p).
#pragma unroll
  for (int r = 0; r < P + 2; ++r) {
    const float* tr = &tile[r][shs[r] + c];
    const f2 x0 = f2_pack(tr[0], tr[kConvHalf]), x1 = f2_pack(tr[1], tr[kConvHalf + 1]),
             x2 = f2_pack(tr[2], tr[kConvHalf + 2]);
#pragma unroll
    for (int dr = 0; dr < 3; ++dr) {
      const int p = r - dr;
      if (p >= 0 && p < P) {
        acc[p] = f2_mac_z(acc[p], w9[3 * dr + 0], x0, z2);
        acc[p] = f2_mac_z(acc[p], w9[3 * dr + 1], x1, z2);
        acc[p] = f2_mac_z(acc[p], w9[3 * dr + 2], x2, z2);
      }
    }
  }
  const uint64_t ja = j0 + c, jb = j0 + kConvHalf + c;
  const bool oka = ja < cols, okb = jb < cols;
  float* orow = out + i0 * cols + ja;
#pragma unroll
  for (int p = 0; p < P; ++p, orow += cols) {
    if (i0 + p < rows) {
      if (oka) __stcs(orow, f2_lo(acc[p]));
      if (okb) __stcs(orow + kConvHalf, f2_hi(acc[p]));
    }
  }
}


}  // namespace

// Shared-memory bytes of one FIR block, 0 if the taps do not fit.
static size_t fir_smem_bytes(uint64_t taps) {
  if (taps > 8192) return 0;
  return sizeof(float) * 2 * ((size_t)fir_wpad((int)taps) + 4 + (size_t)fir_npairs((int)taps));
}

template <int TAPS>
int launch_fir_t(cudaStream_t s, size_t smem, const float* w, uint64_t taps, const float* x, uint64_t x_len,
                 float* y, uint64_t n_out, float seed) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fir_kernel<TAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fir)");
  }
  const uint64_t blocks = (n_out + kFirTile - 1) / kFirTile;
  if (blocks > 0x7fffffffull) return MAPAL_ERR_UNSUPPORTED;
  fir_kernel<TAPS><<<(unsigned)blocks, kFirThreads, smem, s>>>(w, (int)taps, x, x_len, y, n_out, seed, -0.0f);
  count_launch();
  return 0;
}

int launch_fir(cudaStream_t s, const float* w, uint64_t taps, const float* x, uint64_t x_len, float* y,
               uint64_t n_out, float seed) {
  size_t smem = fir_smem_bytes(taps);
  if (smem == 0) return MAPAL_ERR_UNSUPPORTED;
  switch (taps) {  // the benches' tap counts get an unrolled kernel
    case 16: return launch_fir_t<16>(s, smem, w, taps, x, x_len, y, n_out, seed);
    case 32: return launch_fir_t<32>(s, smem, w, taps, x, x_len, y, n_out, seed);
    case 64: return launch_fir_t<64>(s, smem, w, taps, x, x_len, y, n_out, seed);
    default: return launch_fir_t<0>(s, smem, w, taps, x, x_len, y, n_out, seed);
  }
}

int launch_conv3x3(cudaStream_t s, int sms, const float* w, const float* img, uint64_t img_len, uint64_t stride,
                   float* out, uint64_t rows, uint64_t cols, float seed, unsigned* flag) {
  const uint64_t bx = (cols + kConvCols - 1) / kConvCols;
  if (bx > 0x7fffffffull) return MAPAL_ERR_UNSUPPORTED;
  // 10-row strips when they give every SM a few blocks, 2-row strips
  // otherwise. B200, bulk-copy staging, 4098^2 / 8194^2 images: 8, 9, 10, 11,
  // 12, 14, 16, 24 and 32 rows measured 28.7, 25.9, 25.7, 26.0, 27.1, 29.2,
  // 30.4, 31.5 and 34.9 us / 95.4, 86.1, 85.9, 85.6, 88.9, 90.9, 95.5, 100.1
  // and 118.2 us (0.80 / 0.95 of the copy rate at 10 rows); at 1026^2 the grid
  // is the limit: 2, 3, 4, 6 and 8 rows took 3.86, 4.06, 4.2-4.4, 4.20 and
  // 4.46 us (more, shorter blocks in flight).
  const uint64_t by10 = (rows + 9) / 10, by2 = (rows + 1) / 2;
  if (bx * by10 >= 4ull * (uint64_t)sms && by10 <= 65535) {
    conv3x3_kernel<10><<<dim3((unsigned)bx, (unsigned)by10), kConvThreads, 0, s>>>(w, img, img_len, stride, out,
                                                                                   rows, cols, seed, -0.0f, flag);
  } else {
    if (by2 > 65535) return MAPAL_ERR_UNSUPPORTED;
    conv3x3_kernel<2><<<dim3((unsigned)bx, (unsigned)by2), kConvThreads, 0, s>>>(w, img, img_len, stride, out,
                                                                                 rows, cols, seed, -0.0f, flag);
  }
  count_launch();
  return 0;
}
