/*
 * acfun.h — public C API of the B200 (sm_100a) implementation of the Acfun inference path.
 *
 * Drop-in for the reference's include/acfun/acfun.h: every declaration below keeps the
 * reference signature, argument meaning, layouts and error behaviour (void functions
 * return silently on invalid shapes; acfun_model_load returns NULL on failure;
 * acfun_model_infer returns 0 for a NULL model).  The comment on each names the
 * reference declaration it replaces (path:line in the hit-droid/Acfun tree).
 *
 * Memory: every tensor argument may be a host pointer (pageable or pinned) or a CUDA
 * device pointer, detected per call.  Host-pointer calls are synchronous, like the
 * reference.  Calls whose tensors are all device-resident are stream-ordered on the
 * stream set with acfun_set_stream() (default: the legacy default stream) and return
 * without synchronising; call acfun_synchronize() before reading results on the host.
 *
 * Layouts (row-major, NHWC activations):
 *   GEMM         A[M,K], B[K,N], C[M,N]
 *   conv weight  [KH*KW*Cin, Cout]      index ((kh*KW+kw)*Cin+ic)*Cout+oc
 *   depthwise    [C, KH, KW]
 *   grouped      [groups][KH*KW*Cin_per][Cout_per]
 *   FC weight    [Cin, Cout]
 */
#ifndef ACFUN_ACFUN_H
#define ACFUN_ACFUN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime / dispatch (reference acfun.h:19-30) ---- */
void acfun_set_threads(int n);                 /* acfun.h:20 — kept for ABI; CPU thread count has no meaning here */
int acfun_backend(void);                       /* acfun.h:23 — returns 4 (ACFUN_BACKEND_CUDA_SM100A) */
const char* acfun_backend_name(void);          /* acfun.h:24 — "CUDA-sm100a" */
/* acfun.h:29 — measures, on the current GPU, the fastest tcgen05 tile variant of the plain
 * fp32 (3xBF16), bf16 and int8 GEMMs per shape class (M, N, K rounded up to powers of two) and
 * writes the table to $ACFUN_TUNE_CACHE or ~/.cache/acfun/tile_table_<gpu>.txt; later runs load
 * it on first use.  Without a table the built-in size heuristics choose.  Results do not
 * depend on the table (it only picks among tested kernels). */
void acfun_autotune(void);
/* acfun.h:30 — "tuned: <n> shape classes ..." or "static heuristics: ..." */
const char* acfun_tune_status(void);

#define ACFUN_BACKEND_CUDA_SM100A 4

/* ---- GEMM (reference acfun.h:33-51) ---- */
/* acfun.h:33 — fp32 C = A*B; computed as 3xBF16 on tcgen05 tensor cores (3xTF32 with
 * acfun_set_fp32_math(1)), fp32-class error */
void acfun_gemm(int M, int N, int K, const float* A, const float* B, float* C);
/* acfun.h:43 — C = A*B + bias[j] (bias may be NULL), then ReLU if act==1 */
void acfun_gemm_epi(int M, int N, int K, const float* A, const float* B, float* C,
                    const float* bias, int act);
/* acfun.h:51 — fp32 in/out, operands rounded to bf16 (RNE), fp32 accumulation */
void acfun_gemm_bf16(int M, int N, int K, const float* A, const float* B, float* C);

/* ---- convolution (reference acfun.h:61-97) ---- */
/* acfun.h:61 */
void acfun_conv2d(const float* input, int N, int H, int W, int Cin,
                  const float* weight, const float* bias,
                  int KH, int KW, int Cout, int stride, int pad, float* output);
/* acfun.h:67 */
void acfun_conv2d_relu(const float* input, int N, int H, int W, int Cin,
                       const float* weight, const float* bias,
                       int KH, int KW, int Cout, int stride, int pad, float* output);
/* acfun.h:77 — depthwise, weight [C,KH,KW] */
void acfun_conv2d_dw(const float* input, int N, int H, int W, int C,
                     const float* weight, const float* bias,
                     int KH, int KW, int stride, int pad, float* output, int act);
/* acfun.h:86 — grouped; groups==Cin==Cout routes to depthwise */
void acfun_conv2d_g(const float* input, int N, int H, int W, int Cin,
                    const float* weight, const float* bias,
                    int KH, int KW, int Cout, int stride, int pad, int groups,
                    float* output, int act);
/* acfun.h:92 — out[N,Cout] = in[N,Cin] * W[Cin,Cout] + bias */
void acfun_fc(const float* input, int N, int Cin, const float* weight, const float* bias,
              int Cout, float* output);
/* acfun.h:97 — FC + bias + ReLU */
void acfun_fc_relu(const float* input, int N, int Cin, const float* weight, const float* bias,
                   int Cout, float* output);

/* ---- elementwise / pooling / normalisation (reference acfun.h:101-117) ---- */
void acfun_relu(float* data, size_t len);      /* acfun.h:101 */
void acfun_relu6(float* data, size_t len);     /* acfun.h:102 */
/* acfun.h:105 — NHWC max pool, square window */
void acfun_maxpool(const float* input, int N, int H, int W, int C,
                   int pool, int stride, int pad, float* output);
/* acfun.h:111 — max pool with ReLU applied to the pooled value */
void acfun_maxpool_relu(const float* input, int N, int H, int W, int C,
                        int pool, int stride, int pad, float* output);
/* acfun.h:114 — row softmax over the last dimension */
void acfun_softmax(const float* input, int rows, int cols, float* output);
/* acfun.h:117 — in place y = (x-mean)/sqrt(var+eps)*gamma + beta over NHWC channels */
void acfun_batchnorm(float* data, int size, int channels, const float* mean, const float* var,
                     const float* gamma, const float* beta, float eps);

/* ---- int8 (reference acfun.h:126-131) ---- */
/* acfun.h:126 — per-column symmetric weight quantisation (host-side, exact lroundf) */
void acfun_quantize_weights(const float* w, int K, int N, float* scales, int8_t* wq);
/* acfun.h:128 — int8 conv with per-tensor dynamic activation scale (s_in is ignored,
 * as in the reference), per-channel weight scales, fp32 output */
void acfun_conv2d_int8(const float* input, int N, int H, int W, int Cin,
                       const int8_t* wq, const float* wscale, const float* bias,
                       int KH, int KW, int Cout, int stride, int pad,
                       float s_in, float* output, int act);

/* ---- model (reference acfun.h:136-144) ---- */
typedef struct AcfunModel AcfunModel;
AcfunModel* acfun_model_load(const char* path);                          /* acfun.h:138 */
void acfun_model_destroy(AcfunModel* m);                                 /* acfun.h:139 */
int acfun_model_infer(AcfunModel* m, const float* input, float* output); /* acfun.h:141 */
int acfun_model_output_size(AcfunModel* m);                              /* acfun.h:142 */
void acfun_model_input_dims(AcfunModel* m, int* Cin, int* Hin, int* Win); /* acfun.h:144 */

/* ======================= extensions (no reference counterpart) ======================= */

/* Batched inference: n images of [Hin,Win,Cin] -> n * output_size floats.  Each image is
 * processed with batch-1 semantics (Softmax per image).  Returns the per-image output
 * element count, 0 on error. */
int acfun_model_infer_batch(AcfunModel* m, int n, const float* input, float* output);

/* int8 mode for a loaded model (no counterpart in the reference, whose int8 path has no
 * model format): enable != 0 runs every dense convolution through the int8 router
 * (acfun_quantize_weights of the folded weights + acfun_conv2d_int8) with one activation
 * scale per image -- the result of the reference harness that calls acfun_conv2d_int8 per
 * image -- while FC, pooling, BN and softmax stay fp32; 0 switches back to fp32.  Returns
 * 0 or an error code. */
int acfun_model_set_int8(AcfunModel* m, int enable);

/* s8 x s8 GEMM with int32 accumulation and a fused requantising epilogue:
 *   C[i,j] = sat_s8(rne(relu?((float)(acc[i,j] + bias[j]) * scale[j])))
 * bias may be NULL.  This is the int8 GEMM the BASELINE int8 config names; the reference
 * expresses it as acfun_gemm_int8 on A+128 followed by a -128*colsum(B) correction. */
void acfun_gemm_s8_requant(int M, int N, int K, const int8_t* A, const int8_t* B,
                           const int32_t* bias, const float* scale, int8_t* C, int act);

/* acfun_gemm_epi for callers that cannot allocate device memory (no counterpart in the
 * reference).  Such callers exist: processes that reserve all device memory up front in
 * their own pool, code running in an out-of-memory handler or allocator callback, and
 * latency-critical loops where cudaMalloc/cudaFree would synchronise the device.  Same
 * result as acfun_gemm_epi in 3xTF32 mode (acfun_set_fp32_math(1)), but nothing is
 * allocated: the 3xTF32 operand copies live in one
 * fixed 16 MiB device array compiled into the library (held by every GPU that loads it),
 * so 2*(M*K + K*N) must stay <= 4 Mi floats (K, N rounded up to 4).  All tensors must be
 * device pointers on the acfun device.  The first call on a device resolves the array's
 * address.  Calls share the array: calls that overlap on the GPU race.  Runs on the acfun
 * stream and synchronises with it before returning (so it cannot be called while that
 * stream is being captured): returns 0, or an error code. */
int acfun_gemm_epi_noalloc(int M, int N, int K, const float* A, const float* B, float* C,
                           const float* bias, int act);

/* fp32 math on tensor cores.  Every fp32 product is split into hi + lo parts and three
 * tensor-core products are accumulated in fp32 (the dropped lo*lo term and the split residuals
 * bound the error):
 *   1  3xTF32 everywhere   (tf32 parts, ~2^-21 relative per product)
 *   2  3xBF16 everywhere   (bf16 parts, ~2^-17 per product; twice the tensor rate and half the
 *                           operand bytes of 3xTF32)
 *   0  default: 3xBF16 everywhere (measured max-rel vs float64 on the parity shapes is at
 *      or below 3xTF32's there: the fp32 accumulation dominates both).
 * The initial mode comes from $ACFUN_FP32_MATH ("tf32x3" / "bf16x3").  Returns 0 or 1 (bad
 * mode).  Process-wide. */
int acfun_set_fp32_math(int mode);

/* Stream for device-pointer calls (a cudaStream_t passed as void*; NULL = legacy default). */
void acfun_set_stream(void* stream);
void* acfun_get_stream(void);
/* Select the CUDA device used by subsequent calls of this thread (default: device 0 or
 * $ACFUN_DEVICE). */
int acfun_set_device(int device);
/* Wait for all work issued on the current stream; returns 0 on success, else the error
 * code also reported by acfun_last_error(). */
int acfun_synchronize(void);
/* Last error of this thread (0 / "" when none); acfun_clear_error() resets it.
 * Codes: 1 invalid argument, 2 CUDA runtime error, 3 device-side wait timeout,
 *        4 out of memory, 5 model format error. */
int acfun_last_error_code(void);
const char* acfun_last_error(void);
void acfun_clear_error(void);

#ifdef __cplusplus
}
#endif

#endif /* ACFUN_ACFUN_H */
