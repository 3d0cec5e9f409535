// f32x2.cuh — packed pairs of binary32 values for sm_100's two-lane FP32 add
// (PTX add.rn.f32x2), used by the strict (bit-exact) kernels.
//
// A strict MAC is acc = acc + (a * b) with both operations rounded to
// nearest-even, never an FMA. On this toolchain the code generator fuses a
// packed multiply (mul.rn.f32x2, or even fma.rn.f32x2 with a -0 addend)
// followed by a packed add into a packed FMA, whatever -fmad says; a scalar
// __fmul_rn feeding a packed add.rn.f32x2 stays two roundings (measured on
// B200: bit-identical to the separately rounded CPU chain on 8192 random
// 64-step chains, and the packed-packed forms matched the FMA chain instead).
// So products are scalar __fmul_rn (documented never to merge into an FMA)
// and only the accumulation is packed: 3 issue slots per 2 MACs instead of 4.
//
// f2_mac_z goes one step further: the two products are one packed FMA whose
// addend is a -0.0 that the kernel receives as a parameter. a*b + (-0) is
// exact for every a*b (a zero product keeps its sign, infinities and NaNs
// pass through, subnormal products are formed exactly before the single
// rounding), so the FMA returns the rounded product; and since the compiler
// cannot know the addend, it cannot turn the FMA and the following add into
// one fused operation. 2 issue slots per 2 MACs, bit-identical to the scalar
// form (checked on B200 over every cell of a 4096^3 product and against a
// separately rounded CPU chain).
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
  (void)hi;
  return lo;
}

__device__ __forceinline__ float f2_hi(f2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  (void)lo;
  return hi;
}

__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// (acc.lo + a0*b0, acc.hi + a1*b1): two rounded scalar products, one packed
// rounded add.
__device__ __forceinline__ f2 f2_mac(f2 acc, float a0, float b0, float a1, float b1) {
  return f2_add(acc, f2_pack(__fmul_rn(a0, b0), __fmul_rn(a1, b1)));
}

// (acc.lo + a.lo*b.lo, acc.hi + a.hi*b.hi) with z = (-0.0, -0.0) held in a
// register whose value only the caller knows: one packed FMA forms the
// rounded products, one packed add accumulates them.
__device__ __forceinline__ f2 f2_mac_z(f2 acc, f2 a, f2 b, f2 z) {
  f2 p;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(a), "l"(b), "l"(z));
  return f2_add(acc, p);
}
