// hostpath.cu — the matmul site on host-resident arrays, transfers overlapped
// with the multiply.
//
// The reference's emitted program keeps arrays on the device and moves host
// data across with one blocking cudaMemcpy per array (crates/backends/cuda/
// src/func.rs, the H2D / D2H seams of DESIGN BC1). Here a caller holding A, B
// and C in host memory makes one call: B goes up first (every row of C needs
// all of it), then A streams up in row blocks on a copy stream while earlier
// blocks multiply on the context stream, and each finished block of C streams
// down on a second copy stream. In strict mode with K deep enough the upload
// is cut along K instead: phase c brings up B's rows and A's columns of
// k-range c while phase c-1 multiplies, and the last phase runs in row blocks
// so C goes home block by block. With pinned host memory the two PCIe
// directions and the SMs all run at once; the exposed cost is the first
// phase's upload and the last C block.
#include "common.cuh"

namespace {

constexpr uint64_t kBlockAlign = 128;  // rows: a whole number of strict-kernel tiles per block
constexpr uint64_t kMaxBlocks = 8;
constexpr uint64_t kPhases = 5;        // k-ranges of the strict pipeline (at most)
constexpr uint64_t kPhaseMinK = 128;   // shallower ranges are not worth a launch each

int host_streams(DeviceSlot& d, size_t nevents) {
  MAPAL_CUDA(cudaSetDevice(d.device));
  if (!d.h2d_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.h2d_stream, cudaStreamNonBlocking));
  if (!d.d2h_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.d2h_stream, cudaStreamNonBlocking));
  while (d.host_events.size() < nevents) {
    cudaEvent_t e;
    MAPAL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    d.host_events.push_back(e);
  }
  return 0;
}

// The staging buffer grows (never shrinks); growth waits for every stream that
// may still touch the old buffer.
int stage_reserve(DeviceSlot& d, size_t bytes) {
  if (bytes <= d.stage_bytes) return 0;
  if (d.stage) {
    MAPAL_CUDA(cudaStreamSynchronize(d.stream));
    MAPAL_CUDA(cudaStreamSynchronize(d.h2d_stream));
    MAPAL_CUDA(cudaStreamSynchronize(d.d2h_stream));
    MAPAL_CUDA(cudaFree(d.stage));
    d.stage = nullptr;
    d.stage_bytes = 0;
  }
  const size_t round = (bytes + (64u << 20) - 1) & ~((size_t)(64u << 20) - 1);
  MAPAL_CUDA(cudaMalloc(&d.stage, round));
  d.stage_bytes = round;
  return 0;
}

size_t up256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

extern "C" int mapal_gpu_matmul_f32_host(MapalGpuCtx* ctx, const MapalTileSite* site, const float* A,
                                         const float* B, float* C, int mode) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  bool empty = false, shaped = false;
  MAPAL_TRY(validate_tile_site(site, A, B, C, &empty, &shaped));
  if (empty) return 0;
  if (site->k > 0 && !shaped)
    return set_error(MAPAL_ERR_UNSUPPORTED, "record is not matmul-shaped (a{ci>=K, ck=1}, b{ck>=N, clane=1})");
  DeviceSlot& d = ctx->dev[0];
  const uint64_t M = site->rows, N = site->c, K = site->k;
  const uint64_t lda = site->a.ci, ldb = site->b.ck;
  // spans read on the host: A rows [0, M), B rows [0, K), each from its base
  const uint64_t a_elems = K ? (M - 1) * lda + K : 0;
  const uint64_t b_elems = K ? (K - 1) * ldb + N : 0;
  const uint64_t c_elems = M * N;
  uint64_t rows_per = M;
  if (mode == MAPAL_MATMUL_STRICT && K > 0 && M > 2 * kBlockAlign) {
    rows_per = (M + kMaxBlocks - 1) / kMaxBlocks;
    rows_per = (rows_per + kBlockAlign - 1) / kBlockAlign * kBlockAlign;
  }
  const uint64_t nblocks = (M + rows_per - 1) / rows_per;
  MAPAL_TRY(host_streams(d, 2 * nblocks + kPhases + 2));
  MAPAL_TRY(stage_reserve(d, up256(a_elems * 4) + up256(b_elems * 4) + up256(c_elems * 4)));
  float* dA = (float*)d.stage;
  float* dB = (float*)((char*)d.stage + up256(a_elems * 4));
  float* dC = (float*)((char*)d.stage + up256(a_elems * 4) + up256(b_elems * 4));
  cudaEvent_t* ev = d.host_events.data();

  // Everything earlier on the context stream (including the previous call's
  // last C block, which the context stream waited for) precedes these copies.
  MAPAL_CUDA(cudaEventRecord(ev[0], d.stream));
  MAPAL_CUDA(cudaStreamWaitEvent(d.h2d_stream, ev[0], 0));
  MAPAL_CUDA(cudaStreamWaitEvent(d.d2h_stream, ev[0], 0));
  if (K == 0) {
    // a fold over an empty range is its seed
    MAPAL_TRY(launch_fill(d.stream, d.prof.sm_count, dC, site->seed, c_elems));
    MAPAL_CUDA(cudaEventRecord(ev[1], d.stream));
    MAPAL_CUDA(cudaStreamWaitEvent(d.d2h_stream, ev[1], 0));
    MAPAL_CUDA(cudaMemcpyAsync(C, dC, c_elems * 4, cudaMemcpyDeviceToHost, d.d2h_stream));
  } else if (mode == MAPAL_MATMUL_STRICT && nblocks > 1 && K >= 4 * kPhaseMinK) {
    // K in phases: phase c brings up B's rows and A's columns of k-range c
    // and multiplies them into C (each cell continues from the partial fold
    // the previous phase left in C, the same f32 value, so the result is
    // bit-identical to one pass). Only the first phase's transfer is exposed;
    // the last phase runs in row blocks whose C blocks go home as they finish.
    // Cuts at 1/16, 3/16, 6/16 and 10/16 of K (whole 64-deep k-tiles): the
    // first upload is small, each later one arrives before the multiply
    // reaches it (a k-step uploads in ~0.6 us at 55 GB/s and multiplies in
    // ~1 us at N = 4096), and the last phase is long enough to hide the
    // download of C behind its row blocks.
    uint64_t cut[kPhases + 2];
    uint64_t nph = 0;
    cut[0] = 0;
    for (uint64_t sixteenths : {1, 3, 6, 10}) {
      const uint64_t c = (K * sixteenths / 16 + 63) / 64 * 64;
      if (c > cut[nph] && c < K) cut[++nph] = c;
    }
    cut[++nph] = K;
    for (uint64_t c = 0; c < nph; ++c) {
      const uint64_t k0 = cut[c], kc = cut[c + 1] - cut[c];
      const uint64_t b_lo = k0 * ldb, b_hi = (k0 + kc - 1) * ldb + N;
      MAPAL_CUDA(cudaMemcpyAsync(dB + b_lo, B + site->b.base + b_lo, (b_hi - b_lo) * 4, cudaMemcpyHostToDevice,
                                 d.h2d_stream));
      MAPAL_CUDA(cudaMemcpy2DAsync(dA + k0, lda * 4, A + site->a.base + k0, lda * 4, kc * 4, M,
                                   cudaMemcpyHostToDevice, d.h2d_stream));
      MAPAL_CUDA(cudaEventRecord(ev[2 + c], d.h2d_stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.stream, ev[2 + c], 0));
      if (c + 1 < nph) {
        MAPAL_TRY(launch_matmul_strict_ex(d.stream, d.prof.sm_count, dA + k0, dB + b_lo, dC, M, N, kc, lda, ldb, N,
                                          site->seed, c > 0));
        continue;
      }
      for (uint64_t blk = 0; blk < nblocks; ++blk) {
        const uint64_t r0 = blk * rows_per;
        const uint64_t r1 = r0 + rows_per < M ? r0 + rows_per : M;
        cudaEvent_t done = ev[2 + nph + blk];
        MAPAL_TRY(launch_matmul_strict_ex(d.stream, d.prof.sm_count, dA + r0 * lda + k0, dB + b_lo, dC + r0 * N,
                                          r1 - r0, N, kc, lda, ldb, N, site->seed, c > 0));
        MAPAL_CUDA(cudaEventRecord(done, d.stream));
        MAPAL_CUDA(cudaStreamWaitEvent(d.d2h_stream, done, 0));
        MAPAL_CUDA(cudaMemcpyAsync(C + r0 * N, dC + r0 * N, (r1 - r0) * N * 4, cudaMemcpyDeviceToHost,
                                   d.d2h_stream));
      }
    }
  } else {
    MAPAL_CUDA(cudaMemcpyAsync(dB, B + site->b.base, b_elems * 4, cudaMemcpyHostToDevice, d.h2d_stream));
    for (uint64_t blk = 0; blk < nblocks; ++blk) {
      const uint64_t r0 = blk * rows_per;
      const uint64_t r1 = r0 + rows_per < M ? r0 + rows_per : M;
      const uint64_t a_lo = r0 * lda, a_hi = (r1 - 1) * lda + K;  // this block's A span
      cudaEvent_t up = ev[2 + 2 * blk], done = ev[3 + 2 * blk];
      MAPAL_CUDA(cudaMemcpyAsync(dA + a_lo, A + site->a.base + a_lo, (a_hi - a_lo) * 4, cudaMemcpyHostToDevice,
                                 d.h2d_stream));
      MAPAL_CUDA(cudaEventRecord(up, d.h2d_stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.stream, up, 0));
      if (mode == MAPAL_MATMUL_TF32X3)
        MAPAL_TRY(launch_matmul_tf32x3(d, dA + a_lo, dB, dC + r0 * N, r1 - r0, N, K, lda, ldb, N, site->seed));
      else
        MAPAL_TRY(launch_matmul_strict(d.stream, d.prof.sm_count, dA + a_lo, dB, dC + r0 * N, r1 - r0, N, K,
                                       lda, ldb, N, site->seed));
      MAPAL_CUDA(cudaEventRecord(done, d.stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.d2h_stream, done, 0));
      MAPAL_CUDA(cudaMemcpyAsync(C + r0 * N, dC + r0 * N, (r1 - r0) * N * 4, cudaMemcpyDeviceToHost,
                                 d.d2h_stream));
    }
  }
  // The context stream completes only after the last C block is home, so
  // synchronising the context (or its stream) covers the whole call.
  MAPAL_CUDA(cudaEventRecord(ev[1], d.d2h_stream));
  MAPAL_CUDA(cudaStreamWaitEvent(d.stream, ev[1], 0));
  return finish(ctx, 0, mode == MAPAL_MATMUL_TF32X3);
}
