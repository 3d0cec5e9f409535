// sharded.cu — the auto-partitioner's multi-GPU sites.
//
// The reference is one process with no multi-GPU path. Its bulk sites split
// naturally, and only where they do does this library shard them:
//  * saxpy: contiguous equal shards, no exchange;
//  * sum:   contiguous shards, one f64 partial per rank, combined over peer
//           memory in the fold kernel (or one NCCL all-reduce);
//  * gather: idx sharded, x replicated (NCCL broadcast, done once by the caller);
//  * matmul: A row blocks, B replicated by NCCL broadcast, C row blocks stay put.
// A context spans either several devices of one process (arrays hold one
// pointer per local device) or one device of a multi-process job (arrays of
// length 1); the collectives run over the context's communicator either way.
#include "common.cuh"

int nccl_allreduce_f64(MapalGpuCtx* ctx, double* const* buf, size_t count);
int nccl_broadcast_f32(MapalGpuCtx* ctx, float* const* buf, size_t count, int root);
int tile_site_on(MapalGpuCtx* ctx, int local, const MapalTileSite* site, const float* a, const float* b,
                 float* out, int mode);

// Finish a multi-device call: launch errors, then (sync mode) every device's
// completion and trap flag. The first nonzero status wins.
int finish_all(MapalGpuCtx* ctx, bool trap_capable) {
  int first = 0;
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    int rc = enter(ctx, i);
    if (!rc) rc = finish(ctx, i, trap_capable);
    if (rc && !first) first = rc;
  }
  return first;
}

namespace {

int check_arrays(MapalGpuCtx* ctx, const void* a, const void* b, const void* c) {
  if (!ctx) return set_error(MAPAL_ERR_INVALID, "ctx is null");
  if (!a || !b || !c) return set_error(MAPAL_ERR_INVALID, "null pointer array");
  return 0;
}

// Strict row-block matmul with the B broadcast overlapped: K is cut into up
// to kChunks ranges, [0, K/8), [K/8, 3K/8), [3K/8, K) (cuts rounded up to
// whole 64-deep k-tiles); the broadcast of B's rows for range c runs on the
// comm stream while range c-1 is multiplied on the compute stream, so only
// the first eighth of B's transfer is exposed and each range's multiply is
// longer than the next range's transfer. Range c > 0 continues every cell
// from the partial fold range c-1 left in C, so each cell still folds
// k = 0..K-1 in order from the seed: bit-identical to one pass.
constexpr int kChunks = 3;

int matmul_sharded_overlapped(MapalGpuCtx* ctx, const MapalTileSite* site, const float* const* A,
                              float* const* B, float* const* C, const uint64_t* m, int root) {
  const uint64_t K = site->k, lda = site->a.ci, ldb = site->b.ck, N = site->c;
  const int nd = (int)ctx->dev.size();
  // Validate every device's record before anything is enqueued.
  for (int i = 0; i < nd; ++i) {
    MapalTileSite local = *site;
    local.rows = m[i];
    local.a.base = 0;
    local.a.len = m[i] ? (m[i] - 1) * lda + K : 0;
    bool empty = false, mm = false;
    MAPAL_TRY(validate_tile_site(&local, A[i], B[i], C[i], &empty, &mm));
    if (!empty && !mm) return set_error(MAPAL_ERR_UNSUPPORTED, "record is not matmul-shaped");
  }
  // The broadcast must not overwrite B while earlier work on the compute
  // stream may still read it.
  for (int i = 0; i < nd; ++i) {
    DeviceSlot& d = ctx->dev[i];
    MAPAL_TRY(enter(ctx, i));
    MAPAL_TRY(slot_events(d, kChunks + 1));
    MAPAL_CUDA(cudaEventRecord(d.events[kChunks], d.stream));
    MAPAL_CUDA(cudaStreamWaitEvent(d.comm_stream, d.events[kChunks], 0));
  }
  uint64_t k_lo[kChunks + 1];
  int nchunks = 0;
  {
    const uint64_t eighths[kChunks] = {0, 1, 3};
    k_lo[0] = 0;
    for (int c = 1; c < kChunks; ++c) {
      uint64_t cut = (K * eighths[c] / 8 + 63) / 64 * 64;
      if (cut > k_lo[nchunks] && cut < K) k_lo[++nchunks] = cut;
    }
    k_lo[++nchunks] = K;
  }
  for (int c = 0; c < nchunks; ++c) {
    // B rows [k_lo[c], k_lo[c+1]) within the B record's extent.
    const uint64_t lo = site->b.base + k_lo[c] * ldb;
    uint64_t hi = site->b.base + k_lo[c + 1] * ldb;
    if (c == nchunks - 1 || hi > site->b.len) hi = site->b.len;
    MAPAL_TRY(nccl_broadcast_f32_on(ctx, B, lo, hi - lo, root, true));
    for (int i = 0; i < nd; ++i) {
      MAPAL_TRY(enter(ctx, i));
      MAPAL_CUDA(cudaEventRecord(ctx->dev[i].events[c], ctx->dev[i].comm_stream));
    }
  }
  for (int c = 0; c < nchunks; ++c) {
    for (int i = 0; i < nd; ++i) {
      DeviceSlot& d = ctx->dev[i];
      MAPAL_TRY(enter(ctx, i));
      MAPAL_CUDA(cudaStreamWaitEvent(d.stream, d.events[c], 0));
      if (m[i] == 0) continue;
      const uint64_t k0 = k_lo[c], kc = k_lo[c + 1] - k_lo[c];
      MAPAL_TRY(launch_matmul_strict_ex(d.stream, d.prof.sm_count, A[i] + k0, B[i] + site->b.base + k0 * ldb,
                                        C[i], m[i], N, kc, lda, ldb, N, site->seed, c > 0 ? 1 : 0,
                                        c + 1 < nchunks ? 1 : 0));
    }
  }
  return finish_all(ctx, false);
}

}  // namespace

extern "C" int mapal_gpu_saxpy_sharded(MapalGpuCtx* ctx, float a, const float* const* x,
                                       const float* const* y0, float* const* y, const uint64_t* n) {
  MAPAL_TRY(check_arrays(ctx, x, y0, y));
  if (!n) return set_error(MAPAL_ERR_INVALID, "n is null");
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    MAPAL_TRY(enter(ctx, i));
    if (n[i] && (!x[i] || !y0[i] || !y[i])) return set_error(MAPAL_ERR_INVALID, "null shard");
    DeviceSlot& d = ctx->dev[i];
    MAPAL_TRY(launch_saxpy(d.stream, d.prof.sm_count, a, x[i], y0[i], y[i], n[i]));
  }
  return finish_all(ctx, false);
}

extern "C" int mapal_gpu_fold_sum_f32_sharded(MapalGpuCtx* ctx, float seed, const float* const* x,
                                              const uint64_t* n, float* const* out) {
  MAPAL_TRY(check_arrays(ctx, x, n, out));
  for (int i = 0; i < (int)ctx->dev.size(); ++i)
    if ((n[i] && !x[i]) || !out[i]) return set_error(MAPAL_ERR_INVALID, "null shard");
  MAPAL_TRY(peer_setup(ctx));
  if (ctx->peer_state == 1) {
    // one kernel per rank: the fold, then the partials exchanged over peer
    // memory and added in rank order by the fold's last block
    const unsigned long long epoch = ++ctx->xepoch;
    for (int i = 0; i < (int)ctx->dev.size(); ++i) {
      MAPAL_TRY(enter(ctx, i));
      DeviceSlot& d = ctx->dev[i];
      PeerArgs P{};
      for (int q = 0; q < ctx->nranks; ++q) P.blk[q] = d.peer_blk[q];
      P.own = d.xblk;
      P.nranks = ctx->nranks;
      P.rank = ctx->rank0 + i;
      P.epoch = epoch;
      P.wait_ns = ctx->peer_wait_ns;
      P.trap = d.trap;
      MAPAL_TRY(launch_fold_sum_peer(d.stream, d.prof.sm_count, x[i], n[i], seed, d.fold_partials,
                                     d.fold_counter, out[i], P));
    }
    return finish_all(ctx, true);
  }
  std::vector<double*> totals(ctx->dev.size());
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    MAPAL_TRY(enter(ctx, i));
    if ((n[i] && !x[i]) || !out[i]) return set_error(MAPAL_ERR_INVALID, "null shard");
    DeviceSlot& d = ctx->dev[i];
    totals[i] = d.fold_total;
    MAPAL_TRY(launch_fold_sum(d.stream, d.prof.sm_count, x[i], n[i], 0.0f, d.fold_partials,
                              d.fold_counter, nullptr, d.fold_total));
  }
  MAPAL_TRY(nccl_allreduce_f64(ctx, totals.data(), 1));
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    MAPAL_TRY(enter(ctx, i));
    MAPAL_TRY(launch_finalize_sum(ctx->dev[i].stream, ctx->dev[i].fold_total, seed, out[i]));
  }
  return finish_all(ctx, false);
}

extern "C" int mapal_gpu_broadcast_f32(MapalGpuCtx* ctx, float* const* buf, uint64_t n, int root) {
  if (!ctx || !buf) return set_error(MAPAL_ERR_INVALID, "null argument");
  if (root < 0 || root >= ctx->nranks) return set_error(MAPAL_ERR_INVALID, "root out of range");
  if (n == 0) return 0;
  for (int i = 0; i < (int)ctx->dev.size(); ++i)
    if (!buf[i]) return set_error(MAPAL_ERR_INVALID, "null buffer");
  MAPAL_TRY(nccl_broadcast_f32(ctx, buf, n, root));
  return finish_all(ctx, false);
}

extern "C" int mapal_gpu_gather_sharded(MapalGpuCtx* ctx, const float* const* x, uint64_t n_x,
                                        const int32_t* const* idx, float* const* out, const uint64_t* n) {
  MAPAL_TRY(check_arrays(ctx, x, idx, out));
  if (!n) return set_error(MAPAL_ERR_INVALID, "n is null");
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    MAPAL_TRY(enter(ctx, i));
    if (n[i] && (!idx[i] || !out[i] || (n_x && !x[i]))) return set_error(MAPAL_ERR_INVALID, "null shard");
    DeviceSlot& d = ctx->dev[i];
    MAPAL_TRY(launch_gather(d.stream, d.prof.sm_count, x[i], n_x, idx[i], out[i], n[i], d.trap));
  }
  return finish_all(ctx, true);
}

extern "C" int mapal_gpu_matmul_f32_sharded(MapalGpuCtx* ctx, const MapalTileSite* site,
                                            const float* const* A, float* const* B, float* const* C,
                                            const uint64_t* m, int root, int mode) {
  MAPAL_TRY(check_arrays(ctx, A, B, C));
  if (!site || !m) return set_error(MAPAL_ERR_INVALID, "null argument");
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  if (root < 0 || root >= ctx->nranks) return set_error(MAPAL_ERR_INVALID, "root out of range");
  const uint64_t b_elems = site->b.len;
  if (mode == MAPAL_MATMUL_STRICT && ctx->nranks > 1 && site->k >= 512)
    return matmul_sharded_overlapped(ctx, site, A, B, C, m, root);
  // B is replicated first: every rank's full B buffer receives root's.
  MAPAL_TRY(nccl_broadcast_f32(ctx, B, b_elems, root));
  for (int i = 0; i < (int)ctx->dev.size(); ++i) {
    MAPAL_TRY(enter(ctx, i));
    // The device's site: its own row block (A[i] points at the block's first
    // row), the same columns, k order and B record.
    MapalTileSite local = *site;
    local.rows = m[i];
    local.a.base = 0;
    local.a.len = m[i] ? (m[i] - 1) * site->a.ci + site->k : 0;
    MAPAL_TRY(tile_site_on(ctx, i, &local, A[i], B[i], C[i], mode));
  }
  return finish_all(ctx, mode == MAPAL_MATMUL_TF32X3);
}
