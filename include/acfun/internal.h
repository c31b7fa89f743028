/*
 * internal.h — the include name the reference's own test programs and tools use for its
 * non-installed symbols (reference src/internal.h).  A caller built against the reference
 * that writes `#include "internal.h"` compiles unchanged against this directory: the
 * symbols libacfun_b200.so exports are declared in acfun_internal.h.
 *
 * Two scalar reference GEMMs that the reference's tests use as their correctness baseline
 * are declared here too (internal.h:10-11 and :141-143 of the reference); they are NOT part
 * of libacfun_b200.so.  A test program that calls them links a CPU implementation of its own
 * choosing (this repository's test-only oracle provides one, oracle/Makefile `dropin`).
 */
#ifndef ACFUN_B200_INTERNAL_COMPAT_H
#define ACFUN_B200_INTERNAL_COMPAT_H

#include "acfun_internal.h"

#ifdef __cplusplus
extern "C" {
#endif

/* internal.h:10-11 — C = A * B, scalar (not in libacfun_b200.so) */
void acfun_gemm_ref(int M, int N, int K, const float* A, const float* B, float* C);
/* internal.h:141-143 — scalar int8 GEMM + dequant epilogue (not in libacfun_b200.so) */
void acfun_gemm_int8_epi_ref(int M, int N, int K, const uint8_t* A, const int8_t* B, float* C,
                             const float* alpha, const float* beta, int act);

#ifdef __cplusplus
}
#endif
#endif
