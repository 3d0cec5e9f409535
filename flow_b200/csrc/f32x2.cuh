// f32x2.cuh — packed pairs of binary32 values for sm_100's two-lane FP32
// instructions (PTX mul.rn.f32x2 / add.rn.f32x2). Each lane is one IEEE
// round-to-nearest-even operation, exactly what __fmul_rn / __fadd_rn give
// one value at a time; the explicit .rn keeps the compiler from contracting
// a multiply and an add into an FMA. One instruction handles two lanes, so a
// strict multiply-then-add costs one issue slot per value pair instead of
// two per value, and leaves issue slots for the loads.
#pragma once

#include <stdint.h>

typedef uint64_t f2;  // lane 0 in the low 32 bits

__device__ __forceinline__ f2 f2_pack(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ f2 f2_splat(float v) { return f2_pack(v, v); }

__device__ __forceinline__ float f2_lo(f2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}

__device__ __forceinline__ float f2_hi(f2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}

__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// acc + (a * b), two separately rounded operations per lane.
__device__ __forceinline__ f2 f2_mac(f2 acc, f2 a, f2 b) { return f2_add(acc, f2_mul(a, b)); }
