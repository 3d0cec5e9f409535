// tile.cu — TileSite entry points: record validation, shape recognition and
// dispatch, and the generic one-thread-per-cell site kernel.
//
// The reference recognizes three tile-site shapes from the record
// (crates/mapal-ir/src/algo.rs:949-1079, pinned by
// crates/backends/llvm/tests/snapshots/tile_sites_pin__tile_record_content.snap):
// matmul (a{ci, ck=1}, b{ck, clane=1}), the FIR window (rows=1, a{ck=1},
// b{ck=1, clane=1}) and the 3x3 conv (b with a k/3, k%3 split). Each gets a
// specialised kernel here; any other record runs the generic kernel, which
// is the reference's rung-0 shape (one thread per cell, kernel.rs:2773-2886)
// and equally bit-exact.
#include "common.cuh"

int launch_fir(cudaStream_t s, const float* w, uint64_t taps, const float* x, uint64_t x_len, float* y,
               uint64_t n_out, float seed);
int launch_conv3x3(cudaStream_t s, int sms, const float* w, const float* img, uint64_t img_len, uint64_t stride,
                   float* out, uint64_t rows, uint64_t cols, float seed, unsigned* flag);

namespace {

typedef unsigned __int128 u128;

// Largest address a read reaches over i < rows, lane < c, k < K. Every
// coefficient is non-negative, so i and lane peak at their last values; the
// k part ck*k + cq*(k/div) + cr*(k%div) peaks either at k = K-1 or at the
// last element of the last complete div-group.
u128 max_addr(const MapalTileRead& r, uint64_t rows, uint64_t c, uint64_t K) {
  auto kpart = [&](uint64_t k) -> u128 {
    u128 v = (u128)r.ck * k;
    if (r.ksplit.div) v += (u128)r.ksplit.cq * (k / r.ksplit.div) + (u128)r.ksplit.cr * (k % r.ksplit.div);
    return v;
  };
  u128 kmax = kpart(K - 1);
  if (r.ksplit.div && K >= r.ksplit.div) {
    uint64_t k2 = ((K - 1) / r.ksplit.div) * r.ksplit.div;  // first k of the last group
    if (k2 > 0) {
      u128 alt = kpart(k2 - 1);
      if (alt > kmax) kmax = alt;
    }
  }
  return (u128)r.base + (u128)r.ci * (rows - 1) + (u128)r.clane * (c - 1) + kmax;
}

struct GenericRead {
  uint64_t base, ci, ck, clane, div, cq, cr;
};

__device__ __forceinline__ uint64_t gaddr(const GenericRead& r, uint64_t i, uint64_t lane, uint64_t k) {
  uint64_t a = r.base + r.ci * i + r.clane * lane + r.ck * k;
  if (r.div) a += r.cq * (k / r.div) + r.cr * (k % r.div);
  return a;
}

__global__ void tile_generic_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                    float* __restrict__ out, uint64_t cells, uint64_t c, uint64_t K,
                                    GenericRead ra, GenericRead rb, float seed, int mul_a_first,
                                    int add_acc_first) {
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < cells;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / c, lane = t % c;
    float acc = seed;
    for (uint64_t k = 0; k < K; ++k) {
      const float x = __ldg(a + gaddr(ra, i, lane, k)), y = __ldg(b + gaddr(rb, i, lane, k));
      const float p = mul_a_first ? __fmul_rn(x, y) : __fmul_rn(y, x);
      acc = add_acc_first ? __fadd_rn(acc, p) : __fadd_rn(p, acc);
    }
    out[t] = acc;
  }
}

GenericRead to_generic(const MapalTileRead& r) {
  return {r.base, r.ci, r.ck, r.clane, r.ksplit.div, r.ksplit.cq, r.ksplit.cr};
}

bool plain(const MapalTileRead& r) { return r.ksplit.div == 0; }

bool is_matmul(const MapalTileSite& s) {
  return plain(s.a) && plain(s.b) && s.a.ck == 1 && s.a.clane == 0 && s.b.ci == 0 && s.b.clane == 1 &&
         s.a.ci >= s.k && s.b.ck >= s.c;
}

bool is_fir(const MapalTileSite& s) {
  return s.rows == 1 && plain(s.a) && plain(s.b) && s.a.ck == 1 && s.a.clane == 0 && s.b.ck == 1 &&
         s.b.clane == 1;
}

bool is_conv3x3(const MapalTileSite& s) {
  return s.k == 9 && plain(s.a) && s.a.ck == 1 && s.a.ci == 0 && s.a.clane == 0 && s.b.ck == 0 &&
         s.b.clane == 1 && s.b.ksplit.div == 3 && s.b.ksplit.cr == 1 && s.b.ksplit.cq == s.b.ci &&
         s.b.ci >= s.c + 2;
}

// Common checks: null record, empty site, bounds (a read outside its array
// is an index_oob trap for the whole program, as every cell is evaluated).
int check_site(const MapalTileSite* s, const void* a, const void* b, const void* out, bool* empty) {
  if (!s) return set_error(MAPAL_ERR_INVALID, "site is null");
  *empty = s->rows == 0 || s->c == 0;
  if (*empty) return 0;
  if (!out) return set_error(MAPAL_ERR_INVALID, "out is null");
  if (s->k == 0) return 0;
  if (!a || !b) return set_error(MAPAL_ERR_INVALID, "null operand");
  if (max_addr(s->a, s->rows, s->c, s->k) >= s->a.len || max_addr(s->b, s->rows, s->c, s->k) >= s->b.len)
    return set_error(MAPAL_TRAP_INDEX_OOB, "mapal trap: index_oob");
  return 0;
}

int launch_generic(DeviceSlot& d, const MapalTileSite& s, const float* a, const float* b, float* out) {
  const uint64_t cells = s.rows * s.c;
  tile_generic_kernel<<<stream_grid(cells, 256, d.prof.sm_count, 8), 256, 0, d.stream>>>(
      a, b, out, cells, s.c, s.k, to_generic(s.a), to_generic(s.b), s.seed, s.mul_a_first,
      s.add_acc_first); count_launch();
  return 0;
}

int run_site(MapalGpuCtx* ctx, int local, const MapalTileSite& s, const float* a, const float* b,
             float* out, int mode) {
  DeviceSlot& d = ctx->dev[local];
  if (s.k == 0) {
    // A fold over an empty range is its seed.
    return launch_fill(d.stream, d.prof.sm_count, out, s.seed, s.rows * s.c);
  }
  if (is_matmul(s)) {
    const float* A = a + s.a.base;
    const float* B = b + s.b.base;
    if (mode == MAPAL_MATMUL_TF32X3)
      return launch_matmul_tf32x3(d, A, B, out, s.rows, s.c, s.k, s.a.ci, s.b.ck, s.c, s.seed);
    return launch_matmul_strict(d.stream, d.prof.sm_count, A, B, out, s.rows, s.c, s.k, s.a.ci, s.b.ck,
                                s.c, s.seed);
  }
  if (is_fir(s)) {
    int rc = launch_fir(d.stream, a + s.a.base, s.k, b + s.b.base, s.b.len - s.b.base, out, s.c, s.seed);
    if (rc != MAPAL_ERR_UNSUPPORTED) return rc;
  }
  if (is_conv3x3(s)) {
    int rc = launch_conv3x3(d.stream, d.prof.sm_count, a + s.a.base, b + s.b.base, s.b.len - s.b.base, s.b.ci, out, s.rows,
                            s.c, s.seed, d.trap);
    if (rc != MAPAL_ERR_UNSUPPORTED) return rc;
  }
  return launch_generic(d, s, a, b, out);
}

}  // namespace

int validate_tile_site(const MapalTileSite* site, const void* a, const void* b, const void* out, bool* empty,
                       bool* matmul_shaped) {
  MAPAL_TRY(check_site(site, a, b, out, empty));
  *matmul_shaped = site->k > 0 && is_matmul(*site);
  return 0;
}

int tile_site_on(MapalGpuCtx* ctx, int local, const MapalTileSite* site, const float* a, const float* b,
                 float* out, int mode) {
  bool empty = false;
  MAPAL_TRY(check_site(site, a, b, out, &empty));
  if (empty) return 0;
  return run_site(ctx, local, *site, a, b, out, mode);
}

extern "C" int mapal_gpu_tile_site_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* a,
                                       const float* b, float* out, int mode) {
  MAPAL_TRY(enter(ctx));
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  MAPAL_TRY(tile_site_on(ctx, 0, site, a, b, out, mode));
  return finish(ctx, 0, mode == MAPAL_MATMUL_TF32X3);
}

extern "C" int mapal_gpu_matmul_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* A,
                                    const float* B, float* C, int mode) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  if (mode != MAPAL_MATMUL_STRICT && mode != MAPAL_MATMUL_TF32X3)
    return set_error(MAPAL_ERR_INVALID, "unknown matmul mode");
  if (site->k > 0 && !is_matmul(*site))
    return set_error(MAPAL_ERR_UNSUPPORTED, "record is not matmul-shaped (a{ci>=K, ck=1}, b{ck>=N, clane=1})");
  MAPAL_TRY(tile_site_on(ctx, 0, site, A, B, C, mode));
  return finish(ctx, 0, mode == MAPAL_MATMUL_TF32X3);
}

extern "C" int mapal_gpu_fir_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* w,
                                 const float* x, float* out) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  if (site->k > 0 && !is_fir(*site))
    return set_error(MAPAL_ERR_UNSUPPORTED, "record is not a FIR window (rows=1, a{ck=1}, b{ck=1, clane=1})");
  MAPAL_TRY(tile_site_on(ctx, 0, site, w, x, out, MAPAL_MATMUL_STRICT));
  return finish(ctx, 0, false);
}

extern "C" int mapal_gpu_conv2d_3x3_f32(MapalGpuCtx* ctx, const MapalTileSite* site, const float* w,
                                        const float* img, float* out) {
  MAPAL_TRY(enter(ctx));
  if (!site) return set_error(MAPAL_ERR_INVALID, "site is null");
  if (!is_conv3x3(*site))
    return set_error(MAPAL_ERR_UNSUPPORTED, "record is not a 3x3 conv (k=9, b{ci=S, clane=1, ksplit div3 cqS cr1})");
  MAPAL_TRY(tile_site_on(ctx, 0, site, w, img, out, MAPAL_MATMUL_STRICT));
  return finish(ctx, 0, false);
}
