// hostpath.cu — the matmul site on host-resident arrays, transfers overlapped
// with the multiply.
//
// The reference's emitted program keeps arrays on the device and moves host
// data across with one blocking cudaMemcpy per array (crates/backends/cuda/
// src/func.rs, the H2D / D2H seams; BC1 of the reference's
// docs/components/backend-cuda/DESIGN.md). Here a caller holding A, B
// and C in host memory makes one call: B goes up first (every row of C needs
// all of it), then A streams up in row blocks on a copy stream while earlier
// blocks multiply on the context stream, and each finished block of C streams
// down on a second copy stream. In strict mode with K deep enough the upload
// is cut along K instead: phase c brings up B's rows and A's columns of
// k-range c while phase c-1 multiplies, and the last phase runs in row blocks
// so C goes home block by block. With pinned host memory the two PCIe
// directions and the SMs all run at once; the exposed cost is the first
// phase's upload and the last C block.
//
// Over several GPUs (mapal_gpu_matmul_f32_host_sharded) each rank owns a row
// block of A and C, and B is needed whole by every rank: instead of every rank
// pushing all of B across its own PCIe link, each rank uploads 1/R of every
// k-phase's B rows and the ranks broadcast their slices to one another over
// NVLink on a comm stream, between the upload and the multiply of that phase
// (one in-place ncclAllGather when the slices are equal whole rows of a dense
// B, else one ncclBroadcast per owner in one group).
#include "common.cuh"

int finish_all(MapalGpuCtx* ctx, bool trap_capable);

namespace {

constexpr uint64_t kBlockAlign = 128;  // rows: a whole number of strict-kernel tiles per block
constexpr uint64_t kMaxBlocks = 8;
constexpr uint64_t kPhases = 5;        // k-ranges of the strict pipeline (at most)
constexpr uint64_t kPhaseMinK = 128;   // shallower ranges are not worth a launch each

int host_streams(DeviceSlot& d, size_t nevents) {
  MAPAL_CUDA(cudaSetDevice(d.device));
  if (!d.h2d_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.h2d_stream, cudaStreamNonBlocking));
  if (!d.d2h_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.d2h_stream, cudaStreamNonBlocking));
  if (!d.aux_stream) MAPAL_CUDA(cudaStreamCreateWithFlags(&d.aux_stream, cudaStreamNonBlocking));
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
    MAPAL_CUDA(cudaStreamSynchronize(d.aux_stream));
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

// k-phase cuts of the strict pipeline: 0, then 1/16, 3/16, 6/16 and 10/16 of K
// rounded up to whole 64-deep k-tiles, then K. Returns the number of phases.
uint64_t phase_cuts(uint64_t K, uint64_t* cut) {
  uint64_t nph = 0;
  cut[0] = 0;
  for (uint64_t sixteenths : {1, 3, 6, 10}) {
    const uint64_t c = (K * sixteenths / 16 + 63) / 64 * 64;
    if (c > cut[nph] && c < K) cut[++nph] = c;
  }
  cut[++nph] = K;
  return nph;
}

// Row blocks of the last phase (strict) or of the whole call.
uint64_t rows_per_block(uint64_t M, int mode, uint64_t K) {
  uint64_t rows_per = M;
  if (mode == MAPAL_MATMUL_STRICT && K > 0 && M > 2 * kBlockAlign) {
    rows_per = (M + kMaxBlocks - 1) / kMaxBlocks;
    rows_per = (rows_per + kBlockAlign - 1) / kBlockAlign * kBlockAlign;
  }
  return rows_per;
}

int check_host_site(const MapalTileSite* site, const float* A, const float* B, float* C, bool* empty) {
  bool shaped = false;
  MAPAL_TRY(validate_tile_site(site, A, B, C, empty, &shaped));
  if (!*empty && site->k > 0 && !shaped)
    return set_error(MAPAL_ERR_UNSUPPORTED, "record is not matmul-shaped (a{ci>=K, ck=1}, b{ck>=N, clane=1})");
  return 0;
}

// The whole single-device pipeline on local device i, issued without waiting.
int host_one(MapalGpuCtx* ctx, int i, const MapalTileSite* site, const float* A, const float* B, float* C,
             int mode) {
  MAPAL_TRY(enter(ctx, i));
  DeviceSlot& d = ctx->dev[i];
  const uint64_t M = site->rows, N = site->c, K = site->k;
  const uint64_t lda = site->a.ci, ldb = site->b.ck;
  // spans read on the host: A rows [0, M), B rows [0, K), each from its base
  const uint64_t a_elems = K ? (M - 1) * lda + K : 0;
  const uint64_t b_elems = K ? (K - 1) * ldb + N : 0;
  const uint64_t c_elems = M * N;
  const uint64_t rows_per = rows_per_block(M, mode, K);
  const uint64_t nblocks = (M + rows_per - 1) / rows_per;
  MAPAL_TRY(host_streams(d, 2 * nblocks + kPhases + 3));
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
    const uint64_t nph = phase_cuts(K, cut);
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
                                          site->seed, c > 0, 0));
        continue;
      }
      // the row blocks alternate between two streams, so one block's last
      // partial wave shares the SMs with the next block's first
      MAPAL_CUDA(cudaEventRecord(ev[2 + nph + nblocks], d.stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.aux_stream, ev[2 + nph + nblocks], 0));
      for (uint64_t blk = 0; blk < nblocks; ++blk) {
        const uint64_t r0 = blk * rows_per;
        const uint64_t r1 = r0 + rows_per < M ? r0 + rows_per : M;
        cudaEvent_t done = ev[2 + nph + blk];
        cudaStream_t cs = blk % 2 ? d.aux_stream : d.stream;
        MAPAL_TRY(launch_matmul_strict_ex(cs, d.prof.sm_count, dA + r0 * lda + k0, dB + b_lo, dC + r0 * N,
                                          r1 - r0, N, kc, lda, ldb, N, site->seed, c > 0, 0));
        MAPAL_CUDA(cudaEventRecord(done, cs));
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
  return 0;
}

// Rows [lo, hi) of k-phase [k0, k0 + kc) whose B rows rank r uploads.
void b_slice(uint64_t k0, uint64_t kc, int r, int R, uint64_t* lo, uint64_t* hi) {
  *lo = k0 + kc * (uint64_t)r / (uint64_t)R;
  *hi = k0 + kc * (uint64_t)(r + 1) / (uint64_t)R;
}

}  // namespace

extern "C" int mapal_gpu_matmul_f32_host(MapalGpuCtx* ctx, const MapalTileSite* site, const float* A,
                                         const float* B, float* C, int mode) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  bool empty = false;
  MAPAL_TRY(check_host_site(site, A, B, C, &empty));
  if (empty) return 0;
  MAPAL_TRY(host_one(ctx, 0, site, A, B, C, mode));
  return finish(ctx, 0, mode == MAPAL_MATMUL_TF32X3);
}

extern "C" int mapal_gpu_matmul_f32_host_sharded(MapalGpuCtx* ctx, const MapalTileSite* site,
                                                 const float* const* A, const float* const* B, float* const* C,
                                                 const uint64_t* m, int mode) {
  if (!ctx || !site || !A || !B || !C || !m) return set_error(MAPAL_ERR_INVALID, "null argument");
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  const int L = (int)ctx->dev.size(), R = ctx->nranks;
  std::vector<MapalTileSite> local(L);
  std::vector<bool> empty(L);
  for (int i = 0; i < L; ++i) {
    // the device's site: its own row block (A[i] points at the block's first
    // row), the same columns, k order and B record
    local[i] = *site;
    local[i].rows = m[i];
    local[i].a.base = 0;
    local[i].a.len = m[i] ? (m[i] - 1) * site->a.ci + site->k : 0;
    bool e = false;
    MAPAL_TRY(check_host_site(&local[i], A[i], B[i], C[i], &e));
    empty[i] = e;
  }
  const uint64_t N = site->c, K = site->k, lda = site->a.ci, ldb = site->b.ck;
  // Every rank takes the same branch: the test reads only what all ranks share.
  const bool shared_b = R > 1 && mode == MAPAL_MATMUL_STRICT && K >= 4 * kPhaseMinK && N > 0;
  if (!shared_b) {
    for (int i = 0; i < L; ++i)
      if (!empty[i]) MAPAL_TRY(host_one(ctx, i, &local[i], A[i], B[i], C[i], mode));
    return finish_all(ctx, mode == MAPAL_MATMUL_TF32X3);
  }
  for (int i = 0; i < L; ++i)
    if (!B[i]) return set_error(MAPAL_ERR_INVALID, "every rank needs B's host copy");
  NcclApi* nc = nccl_api();
  if (!nc->loaded) return set_error(MAPAL_ERR_NCCL, nc->error);
  uint64_t cut[kPhases + 2];
  const uint64_t nph = phase_cuts(K, cut);
  const uint64_t b_elems = (K - 1) * ldb + N;
  std::vector<float*> dA(L), dB(L), dC(L);
  std::vector<uint64_t> rows_per(L), nblocks(L);
  // host_events: 0 start, 1 end, 2 + 2c B slice up, 3 + 2c A columns up, then
  // one per C block; d.events: one per phase, the slices gathered
  for (int i = 0; i < L; ++i) {
    DeviceSlot& d = ctx->dev[i];
    const uint64_t M = m[i];
    rows_per[i] = M ? rows_per_block(M, mode, K) : 1;
    nblocks[i] = M ? (M + rows_per[i] - 1) / rows_per[i] : 0;
    MAPAL_TRY(host_streams(d, 3 + 2 * nph + nblocks[i]));
    MAPAL_TRY(slot_events(d, nph));
    const uint64_t a_elems = M ? (M - 1) * lda + K : 0;
    MAPAL_TRY(stage_reserve(d, up256(a_elems * 4) + up256(b_elems * 4) + up256(M * N * 4)));
    dA[i] = (float*)d.stage;
    dB[i] = (float*)((char*)d.stage + up256(a_elems * 4));
    dC[i] = (float*)((char*)d.stage + up256(a_elems * 4) + up256(b_elems * 4));
    cudaEvent_t* ev = d.host_events.data();
    MAPAL_CUDA(cudaEventRecord(ev[0], d.stream));
    for (cudaStream_t st : {d.h2d_stream, d.d2h_stream, d.comm_stream}) MAPAL_CUDA(cudaStreamWaitEvent(st, ev[0], 0));
  }
  for (uint64_t c = 0; c < nph; ++c) {
    const uint64_t k0 = cut[c], kc = cut[c + 1] - cut[c];
    for (int i = 0; i < L; ++i) {
      DeviceSlot& d = ctx->dev[i];
      MAPAL_TRY(enter(ctx, i));
      cudaEvent_t* ev = d.host_events.data();
      uint64_t s0, s1;
      b_slice(k0, kc, ctx->rank0 + i, R, &s0, &s1);
      if (s1 > s0)
        MAPAL_CUDA(cudaMemcpyAsync(dB[i] + s0 * ldb, B[i] + site->b.base + s0 * ldb, ((s1 - s0 - 1) * ldb + N) * 4,
                                   cudaMemcpyHostToDevice, d.h2d_stream));
      MAPAL_CUDA(cudaEventRecord(ev[2 + 2 * c], d.h2d_stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.comm_stream, ev[2 + 2 * c], 0));
      if (m[i])
        MAPAL_CUDA(cudaMemcpy2DAsync(dA[i] + k0, lda * 4, A[i] + k0, lda * 4, kc * 4, m[i], cudaMemcpyHostToDevice,
                                     d.h2d_stream));
      MAPAL_CUDA(cudaEventRecord(ev[3 + 2 * c], d.h2d_stream));
    }
    // the phase's B rows, gathered: one in-place all-gather when every rank's
    // slice is the same whole number of dense rows, else every owner
    // broadcasts its slice
    const bool equal = ldb == N && kc % (uint64_t)R == 0;
    int rc = nc->GroupStart();
    if (rc) return set_error(MAPAL_ERR_NCCL, "ncclGroupStart failed");
    for (int i = 0; i < L && !rc; ++i) {
      DeviceSlot& d = ctx->dev[i];
      if (equal) {
        const uint64_t per = kc / (uint64_t)R * N;
        float* base = dB[i] + k0 * N;
        rc = nc->AllGather(base + per * (uint64_t)(ctx->rank0 + i), base, per, kNcclFloat32, d.comm, d.comm_stream);
        continue;
      }
      for (int r = 0; r < R && !rc; ++r) {
        uint64_t t0, t1;
        b_slice(k0, kc, r, R, &t0, &t1);
        if (t1 == t0) continue;
        float* p = dB[i] + t0 * ldb;
        rc = nc->Broadcast(p, p, (t1 - t0 - 1) * ldb + N, kNcclFloat32, r, d.comm, d.comm_stream);
      }
    }
    const int rc2 = nc->GroupEnd();
    if (rc || rc2) return set_error(MAPAL_ERR_NCCL, "gathering a phase's B slices failed");
    for (int i = 0; i < L; ++i) {
      DeviceSlot& d = ctx->dev[i];
      MAPAL_TRY(enter(ctx, i));
      cudaEvent_t* ev = d.host_events.data();
      MAPAL_CUDA(cudaEventRecord(d.events[c], d.comm_stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.stream, d.events[c], 0));
      MAPAL_CUDA(cudaStreamWaitEvent(d.stream, ev[3 + 2 * c], 0));
      const uint64_t M = m[i];
      if (!M) continue;
      const float* bk = dB[i] + k0 * ldb;
      if (c + 1 < nph) {
        // the next phase's B rows are gathered by NCCL beside this multiply
        MAPAL_TRY(launch_matmul_strict_ex(d.stream, d.prof.sm_count, dA[i] + k0, bk, dC[i], M, N, kc, lda, ldb, N,
                                          site->seed, c > 0, 1));
        continue;
      }
      MAPAL_CUDA(cudaEventRecord(ev[2 + 2 * nph + nblocks[i]], d.stream));
      MAPAL_CUDA(cudaStreamWaitEvent(d.aux_stream, ev[2 + 2 * nph + nblocks[i]], 0));
      for (uint64_t blk = 0; blk < nblocks[i]; ++blk) {
        const uint64_t r0 = blk * rows_per[i];
        const uint64_t r1 = r0 + rows_per[i] < M ? r0 + rows_per[i] : M;
        cudaEvent_t done = ev[2 + 2 * nph + blk];
        cudaStream_t cs = blk % 2 ? d.aux_stream : d.stream;
        MAPAL_TRY(launch_matmul_strict_ex(cs, d.prof.sm_count, dA[i] + r0 * lda + k0, bk, dC[i] + r0 * N,
                                          r1 - r0, N, kc, lda, ldb, N, site->seed, c > 0, 0));
        MAPAL_CUDA(cudaEventRecord(done, cs));
        MAPAL_CUDA(cudaStreamWaitEvent(d.d2h_stream, done, 0));
        MAPAL_CUDA(cudaMemcpyAsync(C[i] + r0 * N, dC[i] + r0 * N, (r1 - r0) * N * 4, cudaMemcpyDeviceToHost,
                                   d.d2h_stream));
      }
    }
  }
  for (int i = 0; i < L; ++i) {
    DeviceSlot& d = ctx->dev[i];
    MAPAL_TRY(enter(ctx, i));
    MAPAL_CUDA(cudaEventRecord(d.host_events[1], d.d2h_stream));
    MAPAL_CUDA(cudaStreamWaitEvent(d.stream, d.host_events[1], 0));
  }
  return finish_all(ctx, false);
}
