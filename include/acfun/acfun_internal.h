/*
 * acfun_internal.h — the reference's non-installed int8 / runtime symbols that its tests
 * and tools bind (reference src/internal.h), exported by libacfun_b200.so with
 * identical signatures.  Pointers may be host or device, as for acfun.h.
 */
#ifndef ACFUN_INTERNAL_H
#define ACFUN_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* internal.h:111-112 — kept for ABI; the CUDA backend ignores CPU thread counts */
void acfun_set_num_threads_runtime(int n);
int acfun_get_num_threads_runtime(void);
/* internal.h:115 */
int acfun_pick_threads(int M, int N, int K);
/* internal.h:225 */
int acfun_effective_cores(void);

/* internal.h:119 — u8 x s8 -> s32, exact */
void acfun_gemm_int8(int M, int N, int K, const uint8_t* A, const int8_t* B, int32_t* C);
/* internal.h:138 — C = (float)acc * alpha[j] + beta[j] (two roundings, no FMA), ReLU if act */
void acfun_gemm_int8_epi(int M, int N, int K, const uint8_t* A, const int8_t* B, float* C,
                         const float* alpha, const float* beta, int act);
/* internal.h:152 — out = clamp(rne(in*inv_s) + zp, 0, 255) (the AVX-512 path's rounding) */
void acfun_quantize_u8(const float* in, uint8_t* out, size_t n, float inv_s, int zp);
/* internal.h:164 — direct u8 conv (pad cells read zp = 128) + mul-then-add epilogue */
void acfun_conv2d_int8_direct(const uint8_t* inQ, int N, int H, int W, int Cin,
                              const int8_t* wq, const float* alpha, const float* beta,
                              int KH, int KW, int Cout, int stride, int pad,
                              int OH, int OW, float* output, int act);
/* internal.h:185 — 1x1 stride-1 u8 conv, A[M,K] zero-copy */
void acfun_conv1x1_int8(const uint8_t* inQ, int M, int K, int Cout, const int8_t* wq,
                        const float* alpha, const float* beta, float* output, int act);
/* internal.h:198 — int8 Winograd F(2,3) route (float input quantised inside) */
void acfun_winograd_conv3x3_int8(const float* input, int N, int H, int W, int Cin,
                                 const int8_t* wq, const float* wscale, const float* bias,
                                 int Cout, float s_in, float inv_s, float* output, int act);
/* internal.h:45-60 — fp32 3x3 s1 p1 Winograd routes */
void acfun_winograd_conv3x3(const float* input, int N, int H, int W, int Cin,
                            const float* weight, const float* bias, int Cout, float* output,
                            int act);
void acfun_winograd43_conv3x3(const float* input, int N, int H, int W, int Cin,
                              const float* weight, const float* bias, int Cout, float* output,
                              int act);
/* internal.h:90 — grouped direct conv, weight [g][KH*KW*Cin_per][Cout_per] */
void acfun_conv2d_grouped(const float* input, int N, int H, int W, int Cin,
                          const float* weight, const float* bias, int KH, int KW, int Cout,
                          int stride, int pad, int groups, float* output, int act);

#ifdef __cplusplus
}
#endif
#endif
