/*
 * mapal_oracle.c — CPU restatement of the Mapal interpreter for the bulk-site
 * classes (TEST INFRASTRUCTURE ONLY: the oracle, never the product).
 *
 * Build flags matter: -ffp-contract=off -fno-fast-math, so every float `+`
 * and `*` below is one separately rounded IEEE binary32 operation, as Rust's
 * `x + y` / `x * y` on f32 are in crates/mapal-interp/src/eval.rs:572-585.
 * On x86-64 float arithmetic is SSE (no excess precision).
 */
#include "mapal_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- i32 wrapping arithmetic: eval.rs:552-569 -------------------------- */

int32_t or_i32_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
int32_t or_i32_sub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
int32_t or_i32_mul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }

/* wrapping_div: truncation toward zero; i32::MIN / -1 wraps to i32::MIN. */
int or_i32_div(int32_t a, int32_t b, int32_t* out) {
  if (b == 0) return MAPAL_TRAP_DIV_ZERO;
  if (a == INT32_MIN && b == -1) {
    *out = INT32_MIN;
    return 0;
  }
  *out = a / b;
  return 0;
}

/* wrapping_rem: sign of the dividend; i32::MIN % -1 == 0. */
int or_i32_rem(int32_t a, int32_t b, int32_t* out) {
  if (b == 0) return MAPAL_TRAP_DIV_ZERO;
  if (b == -1) {
    *out = 0;
    return 0;
  }
  *out = a % b;
  return 0;
}

/* ---- the seeded stream ---------------------------------------------------- */

int32_t or_gen_hash(int32_t seed, int32_t i) {
  int32_t h = or_i32_add(or_i32_mul(i, 1103515245),
                         or_i32_add(or_i32_mul(seed, 1640531527), 12345));
  for (int r = 0; r < 3; ++r) {
    int32_t sq = or_i32_mul(h, h);
    int32_t d;
    or_i32_div(h, 65536, &d);
    h = or_i32_add(or_i32_add(sq, d), 1013904223);
  }
  return h;
}

static int32_t pos_mod(int32_t d, int32_t m) {
  int32_t r;
  or_i32_rem(d, m, &r);
  r = or_i32_add(r, m);
  or_i32_rem(r, m, &r);
  return r;
}

static int32_t gen_r24(int32_t seed, int32_t i) {
  int32_t q;
  or_i32_div(or_gen_hash(seed, i), 128, &q);
  return pos_mod(q, 16777216);
}

float or_gen_u11(int32_t seed, int32_t i) {
  float r = (float)gen_r24(seed, i); /* Widen i32 -> f32, eval.rs:238-248 */
  float u = r / 8388608.0f;
  return u - 1.0f;
}

float or_gen_u01(int32_t seed, int32_t i) {
  float r = (float)gen_r24(seed, i);
  return r / 16777216.0f;
}

int32_t or_gen_index(int32_t seed, int32_t i, int32_t range) {
  int32_t h = or_gen_hash(seed, i);
  int32_t d;
  if (range <= 16777216)
    or_i32_div(h, 128, &d);
  else
    or_i32_div(h, 8, &d);
  return pos_mod(d, range);
}

void or_fill_gen(float* out, int64_t n, int32_t seed, int64_t offset, int kind) {
  for (int64_t i = 0; i < n; ++i) {
    int32_t pos = (int32_t)(uint32_t)(uint64_t)(offset + i);
    out[i] = kind == MAPAL_GEN_U01 ? or_gen_u01(seed, pos) : or_gen_u11(seed, pos);
  }
}

void or_fill_index(int32_t* out, int64_t n, int32_t seed, int64_t offset, int32_t range) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = or_gen_index(seed, (int32_t)(uint32_t)(uint64_t)(offset + i), range);
}

void or_fill_affine(float* out, int64_t n, int64_t start, int32_t mul, int32_t add, int32_t mod,
                    int32_t sub) {
  for (int64_t i = 0; i < n; ++i) {
    int32_t t = (int32_t)(uint32_t)(uint64_t)(start + i);
    int32_t v = or_i32_add(or_i32_mul(t, mul), add);
    or_i32_rem(v, mod, &v);
    out[i] = (float)or_i32_sub(v, sub);
  }
}

/* ---- elementwise ------------------------------------------------------------ */

void or_saxpy(float a, const float* x, const float* y0, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float p = a * x[i];
    y[i] = p + y0[i];
  }
}

int or_zip_map(int op, const float* x, const float* y, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    switch (op) {
      case MAPAL_OP_ADD: out[i] = x[i] + y[i]; break;
      case MAPAL_OP_SUB: out[i] = x[i] - y[i]; break;
      case MAPAL_OP_MUL: out[i] = x[i] * y[i]; break;
      case MAPAL_OP_DIV: out[i] = x[i] / y[i]; break;
      case MAPAL_OP_MOD: out[i] = fmodf(x[i], y[i]); break;
      default: return MAPAL_ERR_INVALID;
    }
  }
  return 0;
}

/* ---- move site and gather: Index eval.rs:655-669 ------------------------------ */

int or_move_site(const MapalMoveSite* s, const float* in, float* out) {
  uint64_t n = s->rows * s->width;
  for (uint64_t t = 0; t < n; ++t) {
    uint64_t addr = s->cq * (t / s->width) + s->cr * (t % s->width);
    if (addr >= s->len) return MAPAL_TRAP_INDEX_OOB;
    out[t] = in[addr];
  }
  return 0;
}

int or_gather(const float* x, int64_t n_x, const int32_t* idx, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    int64_t j = (int64_t)idx[i]; /* sign-extending widening, eval.rs:721-728 */
    if (j < 0 || j >= n_x) return MAPAL_TRAP_INDEX_OOB;
    out[i] = x[j];
  }
  return 0;
}

/* ---- fold: eval.rs:326-359 ------------------------------------------------------ */

float or_fold_sum(float seed, const float* x, int64_t n) {
  float acc = seed;
  for (int64_t i = 0; i < n; ++i) acc = acc + x[i];
  return acc;
}

double or_sum_f64(float seed, const float* x, int64_t n) {
  double acc = (double)seed;
  for (int64_t i = 0; i < n; ++i) acc += (double)x[i];
  return acc;
}

double or_sum_abs_f64(const float* x, int64_t n) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) acc += fabs((double)x[i]);
  return acc;
}

/* ---- tile sites: algo.rs:221-345, Map eval.rs:297-324, Fold eval.rs:326-359 ---- */

static uint64_t tile_addr(const MapalTileRead* r, uint64_t i, uint64_t lane, uint64_t k) {
  uint64_t addr = r->base + r->ci * i + r->clane * lane + r->ck * k;
  if (r->ksplit.div != 0) addr += r->ksplit.cq * (k / r->ksplit.div) + r->ksplit.cr * (k % r->ksplit.div);
  return addr;
}

int or_tile_site(const MapalTileSite* s, const float* a, const float* b, float* out) {
  uint64_t cells = s->rows * s->c;
  for (uint64_t t = 0; t < cells; ++t) {
    uint64_t i = t / s->c, lane = t % s->c;
    float acc = s->seed;
    for (uint64_t k = 0; k < s->k; ++k) {
      uint64_t ia = tile_addr(&s->a, i, lane, k);
      uint64_t ib = tile_addr(&s->b, i, lane, k);
      if (ia >= s->a.len || ib >= s->b.len) return MAPAL_TRAP_INDEX_OOB;
      float p = s->mul_a_first ? a[ia] * b[ib] : b[ib] * a[ia];
      acc = s->add_acc_first ? acc + p : p + acc;
    }
    out[t] = acc;
  }
  return 0;
}

/* ---- specialised sites (same per-cell order as or_tile_site) -------------------- */

float or_matmul_cell(const float* A, const float* B, int64_t N, int64_t K, int64_t i, int64_t j) {
  float acc = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    float p = A[i * K + k] * B[k * N + j];
    acc = acc + p;
  }
  return acc;
}

typedef struct {
  const float *A, *B;
  float* C;
  int64_t N, K, r0, r1;
} mm_job;

/* Rows are independent and each cell keeps its k order, so any row split is
 * bit-identical. The j loop is blocked so a panel of B rows stays cached; the
 * per-cell accumulation is still acc = acc + a*b over k ascending. */
static void* mm_worker(void* p) {
  mm_job* j = (mm_job*)p;
  enum { JB = 256 };
  float acc[JB];
  for (int64_t i = j->r0; i < j->r1; ++i) {
    const float* arow = j->A + i * j->K;
    for (int64_t j0 = 0; j0 < j->N; j0 += JB) {
      int64_t jn = j->N - j0 < JB ? j->N - j0 : JB;
      for (int64_t jj = 0; jj < jn; ++jj) acc[jj] = 0.0f;
      for (int64_t k = 0; k < j->K; ++k) {
        float av = arow[k];
        const float* brow = j->B + k * j->N + j0;
        for (int64_t jj = 0; jj < jn; ++jj) {
          float p = av * brow[jj];
          acc[jj] = acc[jj] + p;
        }
      }
      for (int64_t jj = 0; jj < jn; ++jj) j->C[i * j->N + j0 + jj] = acc[jj];
    }
  }
  return NULL;
}

void or_matmul_rows(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    int64_t row0, int64_t row1, int threads) {
  (void)M;
  if (threads < 1) threads = 1;
  int64_t rows = row1 - row0;
  if (rows <= 0) return;
  if (threads > rows) threads = (int)rows;
  pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  mm_job* jobs = (mm_job*)calloc((size_t)threads, sizeof(mm_job));
  for (int t = 0; t < threads; ++t) {
    jobs[t].A = A;
    jobs[t].B = B;
    jobs[t].C = C;
    jobs[t].N = N;
    jobs[t].K = K;
    jobs[t].r0 = row0 + rows * t / threads;
    jobs[t].r1 = row0 + rows * (t + 1) / threads;
    if (threads == 1)
      mm_worker(&jobs[t]);
    else
      pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
  }
  if (threads > 1)
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(tid);
  free(jobs);
}

void or_fir(const float* w, int64_t taps, const float* x, float* y, int64_t n_out) {
  for (int64_t t = 0; t < n_out; ++t) {
    float acc = 0.0f;
    for (int64_t k = 0; k < taps; ++k) {
      float p = w[k] * x[t + k];
      acc = acc + p;
    }
    y[t] = acc;
  }
}

void or_conv2d_3x3(const float* w, const float* img, int64_t stride, float* out,
                   int64_t out_rows, int64_t out_cols) {
  for (int64_t i = 0; i < out_rows; ++i)
    for (int64_t j = 0; j < out_cols; ++j) {
      float acc = 0.0f;
      for (int64_t k = 0; k < 9; ++k) {
        float p = w[k] * img[(i + k / 3) * stride + j + k % 3];
        acc = acc + p;
      }
      out[i * out_cols + j] = acc;
    }
}

/* ---- general map body: Map eval.rs:297-324, arith eval.rs:544-596 ---------------- */

static uint32_t fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static float bitsf(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int or_map_expr(const MapalExprOp* prog, uint32_t nops, const void* const* arrays, const uint64_t* lens,
                uint32_t narrays, void* out, uint64_t n) {
  (void)narrays;
  for (uint64_t t = 0; t < n; ++t) {
    uint32_t st[16];
    int sp = 0;
    for (uint32_t pc = 0; pc < nops; ++pc) {
      const MapalExprOp* op = &prog[pc];
      switch (op->code) {
        case MAPAL_X_T_I32: st[sp++] = (uint32_t)t; break;
        case MAPAL_X_CONST_I32: st[sp++] = (uint32_t)op->i; break;
        case MAPAL_X_CONST_F32: st[sp++] = fbits(op->f); break;
        case MAPAL_X_IN_I32:
        case MAPAL_X_IN_F32: st[sp++] = ((const uint32_t*)arrays[op->slot])[t]; break;
        case MAPAL_X_LOAD_I32:
        case MAPAL_X_LOAD_F32: {
          int64_t j = (int64_t)(int32_t)st[sp - 1];
          if (j < 0 || (uint64_t)j >= lens[op->slot]) return MAPAL_TRAP_INDEX_OOB;
          st[sp - 1] = ((const uint32_t*)arrays[op->slot])[j];
          break;
        }
        case MAPAL_X_NEG_I32: st[sp - 1] = (uint32_t)or_i32_sub(0, (int32_t)st[sp - 1]); break;
        case MAPAL_X_NEG_F32: st[sp - 1] = fbits(-bitsf(st[sp - 1])); break;
        case MAPAL_X_WIDEN_I32_F32: st[sp - 1] = fbits((float)(int32_t)st[sp - 1]); break;
        case MAPAL_X_STORE_I32:
        case MAPAL_X_STORE_F32: ((uint32_t*)out)[t] = st[--sp]; break;
        default: {
          uint32_t b = st[--sp], a = st[sp - 1];
          int32_t r32;
          switch (op->code) {
            case MAPAL_X_ADD_I32: st[sp - 1] = (uint32_t)or_i32_add((int32_t)a, (int32_t)b); break;
            case MAPAL_X_SUB_I32: st[sp - 1] = (uint32_t)or_i32_sub((int32_t)a, (int32_t)b); break;
            case MAPAL_X_MUL_I32: st[sp - 1] = (uint32_t)or_i32_mul((int32_t)a, (int32_t)b); break;
            case MAPAL_X_DIV_I32:
              if (or_i32_div((int32_t)a, (int32_t)b, &r32)) return MAPAL_TRAP_DIV_ZERO;
              st[sp - 1] = (uint32_t)r32;
              break;
            case MAPAL_X_REM_I32:
              if (or_i32_rem((int32_t)a, (int32_t)b, &r32)) return MAPAL_TRAP_DIV_ZERO;
              st[sp - 1] = (uint32_t)r32;
              break;
            case MAPAL_X_ADD_F32: st[sp - 1] = fbits(bitsf(a) + bitsf(b)); break;
            case MAPAL_X_SUB_F32: st[sp - 1] = fbits(bitsf(a) - bitsf(b)); break;
            case MAPAL_X_MUL_F32: st[sp - 1] = fbits(bitsf(a) * bitsf(b)); break;
            case MAPAL_X_DIV_F32: st[sp - 1] = fbits(bitsf(a) / bitsf(b)); break;
            case MAPAL_X_REM_F32: st[sp - 1] = fbits(fmodf(bitsf(a), bitsf(b))); break;
            default: return MAPAL_ERR_INVALID;
          }
        }
      }
    }
  }
  return 0;
}

/* ---- Rust Display of floats: value.rs:90-100 ------------------------------------ */

/* Shortest digit string d (p digits, decimal exponent e: value = d.ddd x 10^e)
 * that parses back to v; among candidates of that length the nearest one.
 * Found by trying lengths 1..maxp with the correctly rounded p-digit decimal
 * and its two neighbours. */
static int shortest_digits(double v, int is_f32, char* digits, int* exp10) {
  int maxp = is_f32 ? 9 : 17;
  char buf[64], cand[64];
  for (int p = 1; p <= maxp; ++p) {
    snprintf(buf, sizeof buf, "%.*e", p - 1, v);
    /* buf = d[.ddd]e[+-]xx */
    char mant[32];
    int m = 0;
    const char* s = buf;
    while (*s && *s != 'e') {
      if (*s != '.') mant[m++] = *s;
      ++s;
    }
    mant[m] = 0;
    int e = atoi(s + 1);
    long long D = atoll(mant);
    long long lo = 1, hi = 10;
    for (int q = 1; q < p; ++q) lo *= 10, hi *= 10;
    if (p == 1) lo = 1;
    long long tries[3] = {D, D - 1, D + 1};
    for (int c = 0; c < 3; ++c) {
      long long Dc = tries[c];
      int ec = e;
      if (Dc < lo) { /* 10..0 - 1 -> 9.99..9 one decade down */
        Dc = hi - 1;
        ec = e - 1;
      }
      if (Dc >= hi) { Dc = lo; ec = e + 1; }
      char ds[32];
      snprintf(ds, sizeof ds, "%lld", Dc);
      snprintf(cand, sizeof cand, "%c.%se%d", ds[0], ds + 1, ec);
      int ok = is_f32 ? (strtof(cand, NULL) == (float)v) : (strtod(cand, NULL) == v);
      if (ok) {
        strcpy(digits, ds);
        *exp10 = ec;
        return p;
      }
    }
  }
  return -1;
}

static int render(double v, int is_f32, char* buf, int cap) {
  char out[400];
  int n = 0;
  if (isnan(v)) {
    n = snprintf(out, sizeof out, "NaN");
  } else if (isinf(v)) {
    n = snprintf(out, sizeof out, v < 0 ? "-inf" : "inf");
  } else if (v == 0.0) {
    n = snprintf(out, sizeof out, signbit(v) ? "-0" : "0");
  } else {
    char digits[32];
    int e;
    double av = fabs(v);
    int p = shortest_digits(av, is_f32, digits, &e);
    if (p < 0) return -1;
    if (signbit(v)) out[n++] = '-';
    if (e >= p - 1) {
      memcpy(out + n, digits, (size_t)p);
      n += p;
      for (int z = 0; z < e - (p - 1); ++z) out[n++] = '0';
    } else if (e >= 0) {
      memcpy(out + n, digits, (size_t)(e + 1));
      n += e + 1;
      out[n++] = '.';
      memcpy(out + n, digits + e + 1, (size_t)(p - e - 1));
      n += p - e - 1;
    } else {
      out[n++] = '0';
      out[n++] = '.';
      for (int z = 0; z < -e - 1; ++z) out[n++] = '0';
      memcpy(out + n, digits, (size_t)p);
      n += p;
    }
    out[n] = 0;
  }
  if (n + 1 > cap) return -1;
  memcpy(buf, out, (size_t)n + 1);
  return n;
}

int or_render_f32(float v, char* buf, int cap) { return render((double)v, 1, buf, cap); }
int or_render_f64(double v, char* buf, int cap) { return render(v, 0, buf, cap); }
