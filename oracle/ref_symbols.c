/* TEST INFRASTRUCTURE ONLY: the two scalar reference GEMMs the reference's own test programs
 * (tools/test_bf16.cpp, tools/test_int8_epi.cpp of hit-droid/Acfun) call as their correctness
 * baseline, provided by this repository's C oracle so those programs can be compiled
 * unmodified against libacfun_b200.so (oracle/Makefile `dropin`).
 *   acfun_gemm_ref           reference src/gemm_ref.cpp (plain triple loop, C = A * B)
 *   acfun_gemm_int8_epi_ref  reference src/gemm_int8.cpp scalar path ((float)acc*alpha + beta)
 * Never linked into the product library. */
#include <stddef.h>
#include <stdint.h>

#include "acfun_oracle.h"

void acfun_gemm_ref(int M, int N, int K, const float* A, const float* B, float* C) {
  orc_gemm_f32(M, N, K, A, B, C, NULL, 0);
}

void acfun_gemm_int8_epi_ref(int M, int N, int K, const uint8_t* A, const int8_t* B, float* C,
                             const float* alpha, const float* beta, int act) {
  orc_gemm_int8_epi(M, N, K, A, B, C, alpha, beta, act);
}
