// matmul_tf32x3.cu — opt-in tensor-core matmul (3xTF32 on tcgen05); see below.
#include "common.cuh"

int launch_matmul_tf32x3(DeviceSlot& d, const float* A, const float* B, float* C, uint64_t M, uint64_t N,
                         uint64_t K, uint64_t lda, uint64_t ldb, uint64_t ldc, float seed) {
  (void)d; (void)A; (void)B; (void)C; (void)M; (void)N; (void)K; (void)lda; (void)ldb; (void)ldc;
  (void)seed;
  return set_error(MAPAL_ERR_UNSUPPORTED, "3xTF32 matmul not built yet");
}
