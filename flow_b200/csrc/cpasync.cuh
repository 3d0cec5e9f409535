// cpasync.cuh — asynchronous global-to-shared copies (cp.async, sm_80+ form,
// still the lightest way to stage small irregular tiles on sm_100).
#pragma once

#include <stdint.h>

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16 bytes, or zero-fill when !pred (src is then not read).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0));
}

// 4 bytes, or zero-fill when !pred.
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 4 : 0));
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Copy floats src[0..3] to dst where the first `nvalid` are readable
// (nvalid <= 0: all zero). A full group at a 16-byte aligned source goes as
// one 16-byte copy; otherwise one 4-byte copy per float, zero-filling the rest.
__device__ __forceinline__ void copy4(uint32_t dst, const float* src, int nvalid, bool aligned) {
  if (aligned && nvalid >= 4) {
    cp_async16(dst, src, true);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) cp_async4(dst + 4 * e, nvalid > e ? src + e : src, nvalid > e);
  }
}
