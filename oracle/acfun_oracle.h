/*
 * acfun_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded CPU restatement of the Acfun reference algorithms on the
 * conv/GEMM inference path.  It is the parity checker for the CUDA library
 * (libacfun_b200.so) and is never linked into, loaded by, or called from the product.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs may use it.
 *
 * Every function cites the reference file:line it restates (paths relative to the
 * hit-droid/Acfun source tree).  Rounding is reproduced exactly for the integer paths:
 *   - mul-then-add epilogues are compiled with -ffp-contract=off (reference TUs use the
 *     same flag, CMakeLists.txt:55,62,65);
 *   - the int8 Winograd dequant uses fmaf (winograd_int8.cpp:166).
 * The oracle is pinned against the reference library built from its own sources
 * (oracle/_ref) and against committed golden vectors (tests/golden).
 */
#ifndef ACFUN_ORACLE_H
#define ACFUN_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- GEMM family ---------------- */
void orc_gemm_f32(int M, int N, int K, const float* A, const float* B, float* C,
                  const float* bias, int act);
uint16_t orc_f32_to_bf16(float f);
void orc_gemm_bf16(int M, int N, int K, const float* A, const float* B, float* C);
void orc_gemm_int8(int M, int N, int K, const uint8_t* A, const int8_t* B, int32_t* C);
void orc_gemm_int8_epi(int M, int N, int K, const uint8_t* A, const int8_t* B, float* C,
                       const float* alpha, const float* beta, int act);
void orc_gemm_s8_requant(int M, int N, int K, const int8_t* A, const int8_t* B,
                         const int32_t* bias, const float* scale, int8_t* C, int act);
int8_t orc_requant_s8(int32_t acc, int32_t bias, float scale, int act);

/* ---------------- quantization ---------------- */
void orc_quantize_u8(const float* in, uint8_t* out, size_t n, float inv_s, int zp, int rne);
void orc_quantize_weights(const float* w, int K, int N, float* scales, int8_t* wq);

/* ---------------- int8 convolution (router + every route) ---------------- */
void orc_conv2d_int8(const float* input, int N, int H, int W, int Cin,
                     const int8_t* wq, const float* wscale, const float* bias,
                     int KH, int KW, int Cout, int stride, int pad,
                     float s_in, float* output, int act);
void orc_winograd_int8(const float* input, int N, int H, int W, int Cin,
                       const int8_t* wq, const float* wscale, const float* bias, int Cout,
                       float s_in, float inv_s, float* output, int act);
void orc_conv2d_int8_direct(const uint8_t* inQ, int N, int H, int W, int Cin,
                            const int8_t* wq, const float* alpha, const float* beta,
                            int KH, int KW, int Cout, int stride, int pad,
                            int OH, int OW, float* output, int act);
void orc_conv1x1_int8(const uint8_t* inQ, int M, int K, int Cout, const int8_t* wq,
                      const float* alpha, const float* beta, float* output, int act);
/* route id the reference's conv_int8.cpp:63-148 would take on an AVX-512F host:
 * 0 zero-output (max|x|<1e-12), 1 winograd-int8, 2 direct, 3 conv1x1, 4 im2col+GEMM-epi */
int  orc_conv2d_int8_route(const float* input, int N, int H, int W, int Cin,
                           int KH, int KW, int Cout, int stride, int pad);

/* ---------------- float convolution family ---------------- */
/* direct convolution, any groups; weight layouts exactly as the reference reads them */
void orc_conv2d(const float* input, int N, int H, int W, int Cin,
                const float* weight, const float* bias, int KH, int KW, int Cout,
                int stride, int pad, int groups, float* output, int act);
void orc_winograd23(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int Cout, float* output, int act);
void orc_winograd43(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int Cout, float* output, int act);
void orc_conv2d_dw(const float* input, int N, int H, int W, int C, const float* weight,
                   const float* bias, int KH, int KW, int stride, int pad, float* output, int act);
void orc_group_conv(const float* input, int N, int H, int W, int Cin, const float* weight,
                    const float* bias, int KH, int KW, int Cout, int stride, int pad,
                    int groups, float* output, int act);
/* route id of layers.cpp:106-195: 1 dw, 2 grouped-direct, 3 grouped-split, 4 conv1x1,
 * 5 winograd F(4,3), 6 winograd F(2,3), 7 im2col+GEMM, 0 empty output */
int  orc_conv2d_route(int N, int H, int W, int Cin, int KH, int KW, int Cout,
                      int stride, int pad, int groups);

/* ---------------- layers ---------------- */
void orc_fc(const float* input, int N, int Cin, const float* weight, const float* bias,
            int Cout, float* output, int act);
void orc_relu(float* d, size_t n);
void orc_relu6(float* d, size_t n);
void orc_maxpool(const float* in, int N, int H, int W, int C, int pool, int stride, int pad,
                 float* out, int post_relu);
void orc_softmax(const float* in, int rows, int cols, float* out);
void orc_batchnorm(float* d, int size, int channels, const float* mean, const float* var,
                   const float* gamma, const float* beta, float eps);
/* BN fold of model.cpp:69-95 applied to a Conv/FC/grouped weight block */
void orc_fold_bn(float* w, float* b, size_t wn, int Cout, int groups, const float* mean,
                 const float* var, const float* gamma, const float* beta);

#ifdef __cplusplus
}
#endif
#endif
