/*
 * mapal_oracle.h — CPU restatement of the Mapal interpreter's semantics for
 * the bulk-site classes that libmapal_gpu accelerates.
 *
 * TEST INFRASTRUCTURE ONLY. This is the oracle: only tests/, the smoke
 * check and the bench's CPU-baseline leg load it. No product code path
 * calls it, and libmapal_gpu has no CPU fallback to it.
 *
 * Every function cites the reference file:line whose behaviour it restates
 * (paths relative to the reference project root). Parity of this oracle is
 * pinned against the reference's own known answers and its own C++ baseline
 * programs, compiled from the reference sources by oracle/Makefile; see
 * tests/test_oracle_golden.py.
 */
#ifndef MAPAL_ORACLE_H
#define MAPAL_ORACLE_H

#include <stdint.h>

#include "../include/mapal_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* i32 wrapping arithmetic (eval.rs:552-569: wrapping_add/sub/mul; div and rem
 * truncate toward zero, MIN / -1 wraps, a zero divisor traps div_zero).
 * or_i32_div / or_i32_rem return 0 or MAPAL_TRAP_DIV_ZERO. */
int32_t or_i32_add(int32_t a, int32_t b);
int32_t or_i32_sub(int32_t a, int32_t b);
int32_t or_i32_mul(int32_t a, int32_t b);
int or_i32_div(int32_t a, int32_t b, int32_t* out);
int or_i32_rem(int32_t a, int32_t b, int32_t* out);

/* The seeded stream, written only with Mapal's i32 wrapping `* + / %`:
 *   h = i*1103515245 + (seed*1640531527 + 12345)
 *   3 times: h = h*h + h/65536 + 1013904223
 *   q = h/128;  r = ((q % 2^24) + 2^24) % 2^24
 *   u11 = widen_f32(r)/8388608.0 - 1.0,  u01 = widen_f32(r)/16777216.0
 *   index in [0, range): ((d % range) + range) % range with d = q when
 *   range <= 2^24, else d = h/8. */
int32_t or_gen_hash(int32_t seed, int32_t i);
float or_gen_u11(int32_t seed, int32_t i);
float or_gen_u01(int32_t seed, int32_t i);
int32_t or_gen_index(int32_t seed, int32_t i, int32_t range);
void or_fill_gen(float* out, int64_t n, int32_t seed, int64_t offset, int kind);
void or_fill_index(int32_t* out, int64_t n, int32_t seed, int64_t offset, int32_t range);

/* The benches' integer generators: out[i] = widen_f32((t*mul + add) % mod - sub),
 * t = start + i, i32 wrapping (e.g. benches/shapes/saxpy_1048576.mapal:8-9). */
void or_fill_affine(float* out, int64_t n, int64_t start, int32_t mul, int32_t add, int32_t mod,
                    int32_t sub);

/* saxpy y[i] = a*x[i] + y0[i], each op rounded (saxpy_1048576.mapal:11;
 * Zip eval.rs:371-385 then Map eval.rs:297-324). */
void or_saxpy(float a, const float* x, const float* y0, float* y, int64_t n);

/* out[i] = x[i] OP y[i] (float arith, eval.rs:572-585; MOD is fmodf). */
int or_zip_map(int op, const float* x, const float* y, float* out, int64_t n);

/* Move site out[t] = in[cq*(t/width) + cr*(t%width)] (transpose_1024.mapal:11);
 * returns MAPAL_TRAP_INDEX_OOB at the first out-of-range address (eval.rs:655-669). */
int or_move_site(const MapalMoveSite* site, const float* in, float* out);

/* Gather out[i] = x[idx[i]]; index_oob at the first idx outside [0, n_x)
 * (gather_1048576.mapal:11; eval.rs:655-669). */
int or_gather(const float* x, int64_t n_x, const int32_t* idx, float* out, int64_t n);

/* Left fold acc = acc + x[i] from seed (eval.rs:326-359). */
float or_fold_sum(float seed, const float* x, int64_t n);
/* The same sum in f64 (an accuracy reference, not an interpreter op). */
double or_sum_f64(float seed, const float* x, int64_t n);
/* sum |x| in f64 */
double or_sum_abs_f64(const float* x, int64_t n);

/* Any TileSite, cell by cell in cell order, fold strictly left to right
 * (algo.rs:221-345 record semantics; Map eval.rs:297-324; Fold eval.rs:326-359).
 * a has site->a.len elements and b site->b.len. Returns 0 or
 * MAPAL_TRAP_INDEX_OOB (the first cell whose read is out of range, out is then
 * partially written). */
int or_tile_site(const MapalTileSite* site, const float* a, const float* b, float* out);

/* Row-major matmul rows [row0, row1) of C = A*B (A M x K, B K x N), each cell
 * acc = +0.0, then acc = acc + a*b for k ascending, every op rounded: the
 * matmul tile site (matmul1024_cap_f32.mapal:7-11). `threads` > 1 splits rows
 * over POSIX threads (a cell's k order never changes). */
void or_matmul_rows(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    int64_t row0, int64_t row1, int threads);
/* One cell of the same matmul. */
float or_matmul_cell(const float* A, const float* B, int64_t N, int64_t K, int64_t i, int64_t j);

/* FIR y[t] = fold_k(acc + w[k]*x[t+k]) from 0.0, t < n_out (fir_1048576.mapal:10-12). */
void or_fir(const float* w, int64_t taps, const float* x, float* y, int64_t n_out);

/* 3x3 conv2d out[i,j] = fold_k(acc + w[k]*img[(i+k/3)*stride + j + k%3]),
 * out is out_rows x out_cols (conv2d_1024.mapal:11-15). */
void or_conv2d_3x3(const float* w, const float* img, int64_t stride, float* out,
                   int64_t out_rows, int64_t out_cols);

/* A map body given as a MAPAL_X_* stack program (include/mapal_gpu.h),
 * evaluated element by element in order (Map eval.rs:297-324; arithmetic
 * eval.rs:544-596). out holds 32-bit values (i32 or f32 bits). Returns 0, or
 * the trap of the first element that traps (MAPAL_TRAP_DIV_ZERO /
 * MAPAL_TRAP_INDEX_OOB); elements before it are written. */
int or_map_expr(const MapalExprOp* prog, uint32_t nops, const void* const* arrays, const uint64_t* lens,
                uint32_t narrays, void* out, uint64_t n);

/* Rust `Display` of an f32 / f64 (value.rs:90-100): shortest round-trip
 * digits, positional notation, "NaN", "inf", "-inf", "-0". Returns length. */
int or_render_f32(float v, char* buf, int cap);
int or_render_f64(double v, char* buf, int cap);

#ifdef __cplusplus
}
#endif

#endif /* MAPAL_ORACLE_H */
