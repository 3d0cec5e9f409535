// rt.cpp — the mapal-rt symbols an emitted Mapal program links
// (crates/mapal-rt/src/lib.rs:27-81 prints and trap, :393 time), re-exported
// with the same observable behaviour: stdout bytes, stderr message, exit code.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <charconv>
#include <chrono>
#include <cinttypes>
#include <mutex>

#include "../../include/mapal_rt.h"

namespace {

// Rust's `Display` for floats: the shortest digit string that round-trips,
// laid out positionally (never an exponent) with zeros filling the places
// past the last significant digit, no trailing ".0", and the spellings
// "NaN", "inf", "-inf", "-0" (crates/mapal-interp/src/value.rs:90-100 renders
// through the same formatter). So 623573888.0f32 prints "623573900" and
// f32::MAX "340282350000000000000000000000000000000". std::to_chars in
// scientific form supplies the shortest round-trip digits and the exponent;
// the positional layout is assembled here.
template <typename T>
int render(T v, char* buf, size_t cap) {
  char tmp[400];
  size_t n = 0;
  if (isnan(v)) {
    n = (size_t)snprintf(tmp, sizeof tmp, "NaN");
  } else if (isinf(v)) {
    n = (size_t)snprintf(tmp, sizeof tmp, "%s", v < 0 ? "-inf" : "inf");
  } else if (v == 0) {
    n = (size_t)snprintf(tmp, sizeof tmp, "%s", signbit(v) ? "-0" : "0");
  } else {
    char sci[64];
    auto r = std::to_chars(sci, sci + sizeof sci - 1, v < 0 ? -v : v, std::chars_format::scientific);
    if (r.ec != std::errc()) return -1;
    *r.ptr = 0;
    char digits[40];
    int p = 0;
    const char* s = sci;
    for (; *s && *s != 'e'; ++s)
      if (*s != '.') digits[p++] = *s;
    int e = atoi(s + 1);  // value = d.ddd x 10^e
    if (v < 0) tmp[n++] = '-';
    if (e >= p - 1) {  // integral: digits then zeros
      memcpy(tmp + n, digits, (size_t)p);
      n += (size_t)p;
      for (int z = 0; z < e - (p - 1); ++z) tmp[n++] = '0';
    } else if (e >= 0) {  // point inside the digits
      memcpy(tmp + n, digits, (size_t)e + 1);
      n += (size_t)e + 1;
      tmp[n++] = '.';
      memcpy(tmp + n, digits + e + 1, (size_t)(p - e - 1));
      n += (size_t)(p - e - 1);
    } else {  // 0.000ddd
      tmp[n++] = '0';
      tmp[n++] = '.';
      for (int z = 0; z < -e - 1; ++z) tmp[n++] = '0';
      memcpy(tmp + n, digits, (size_t)p);
      n += (size_t)p;
    }
  }
  tmp[n] = 0;
  if (n + 1 > cap) return -1;
  memcpy(buf, tmp, n + 1);
  return (int)n;
}

void emit(const char* s, size_t len, bool newline) {
  fwrite(s, 1, len, stdout);
  if (newline) fputc('\n', stdout);
  fflush(stdout);
}

}  // namespace

extern "C" {

int mapal_render_f32(float v, char* buf, size_t cap) { return render<float>(v, buf, cap); }
int mapal_render_f64(double v, char* buf, size_t cap) { return render<double>(v, buf, cap); }

void mapal_print_i32(int32_t v, bool newline) {
  char b[32];
  int n = snprintf(b, sizeof b, "%" PRId32, v);
  emit(b, (size_t)n, newline);
}

void mapal_print_i64(int64_t v, bool newline) {
  char b[32];
  int n = snprintf(b, sizeof b, "%" PRId64, v);
  emit(b, (size_t)n, newline);
}

void mapal_print_u8(uint8_t v, bool newline) {
  char b[8];
  int n = snprintf(b, sizeof b, "%u", (unsigned)v);
  emit(b, (size_t)n, newline);
}

void mapal_print_bool(bool v, bool newline) {
  if (v)
    emit("true", 4, newline);
  else
    emit("false", 5, newline);
}

void mapal_print_f32(float v, bool newline) {
  char b[64];
  int n = mapal_render_f32(v, b, sizeof b);
  emit(b, (size_t)(n < 0 ? 0 : n), newline);
}

void mapal_print_f64(double v, bool newline) {
  char b[400];
  int n = mapal_render_f64(v, b, sizeof b);
  emit(b, (size_t)(n < 0 ? 0 : n), newline);
}

void mapal_print_str(const uint8_t* ptr, size_t len, bool newline) {
  emit(reinterpret_cast<const char*>(ptr), len, newline);
}

[[noreturn]] void mapal_trap(uint32_t kind) {
  const char* msg = kind == 0 ? "div_zero" : kind == 1 ? "index_oob" : "unknown";
  fflush(stdout);
  fprintf(stderr, "mapal trap: %s\n", msg);
  fflush(stderr);
  exit(101);
}

double mapal_time_ms(void) {
  using clock = std::chrono::steady_clock;
  static std::once_flag once;
  static clock::time_point epoch;
  std::call_once(once, [] { epoch = clock::now(); });
  return std::chrono::duration<double, std::milli>(clock::now() - epoch).count();
}

}  // extern "C"
