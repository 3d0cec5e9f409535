/*
 * mapal_rt.h — the runtime symbols every emitted Mapal program links,
 * re-exported by libmapal_gpu with the reference's semantics (the Rust
 * staticlib crates/mapal-rt cannot be built without a Rust toolchain).
 *
 * Declared by the emitted prelude at crates/backends/cuda/src/module.rs:47-59;
 * defined at crates/mapal-rt/src/lib.rs:27-81 (prints, trap) and :393 (time).
 */
#ifndef MAPAL_RT_H
#define MAPAL_RT_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every symbol declared here is exported even when the library is built with
 * hidden default visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Print `v` as Rust's Display does (mapal-rt/src/lib.rs:38-53): integers in
 * decimal, bool as true/false, floats as the shortest round-trip decimal in
 * positional notation ("4080", "5.375", "0.33333334", "NaN", "inf", "-0"),
 * then a newline if `newline`; stdout is flushed on every call. */
void mapal_print_i32(int32_t v, bool newline);
void mapal_print_i64(int64_t v, bool newline);
void mapal_print_u8(uint8_t v, bool newline);
void mapal_print_bool(bool v, bool newline);
void mapal_print_f32(float v, bool newline);
void mapal_print_f64(double v, bool newline);
/* Print exactly `len` bytes of UTF-8 at `ptr` (lib.rs:63). */
void mapal_print_str(const uint8_t* ptr, size_t len, bool newline);

/* A defined trap (lib.rs:71-81): flush stdout, write "mapal trap: div_zero"
 * (kind 0) / "mapal trap: index_oob" (kind 1) / "mapal trap: unknown" to
 * stderr, exit(101). */
#ifdef __cplusplus
[[noreturn]]
#endif
void mapal_trap(uint32_t kind);

/* Milliseconds on a monotonic clock since the first call in the process
 * (lib.rs:393; the `time` builtin's seam). */
double mapal_time_ms(void);

/* Render helpers (no I/O): write the Display text of `v` into buf (NUL
 * terminated, at most cap bytes); return its length, or -1 if cap is too
 * small. Float Display needs at most 48 bytes for f32 and 330 for f64. */
int mapal_render_f32(float v, char* buf, size_t cap);
int mapal_render_f64(double v, char* buf, size_t cap);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MAPAL_RT_H */
