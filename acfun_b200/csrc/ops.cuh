// ops.cuh — device-pointer entry points of the bandwidth kernels (ops.cu), shared by the
// public API wrappers, the convolution router and the model executor.
#pragma once
#include "runtime.cuh"

namespace acf {
bool relu_dev(Call& c, float* d, long long n, int six);
struct SplitAct;
// os != NULL: write the result as the next convolution's split input (C % 16 == 0)
bool maxpool_dev(Call& c, const float* in, int N, int H, int W, int C, int pool, int stride,
                 int pad, float* out, int post_relu, const SplitAct* os = nullptr);
bool softmax_dev(Call& c, const float* in, int rows, int cols, float* out);
bool batchnorm_dev(Call& c, float* d, int size, int channels, const float* mean,
                   const float* var, const float* gamma, const float* beta, float eps);
bool quantize_u8_dev(Call& c, const float* in, uint8_t* out, long long n, float inv_s, int zp);
// d[0..n) = v
bool fill_u32_dev(Call& c, unsigned* d, unsigned v, long long n);
bool dw_dev(Call& c, const float* in, int N, int H, int W, int C, const float* w,
            const float* bias, int KH, int KW, int stride, int pad, float* out, int act);
// depthwise 3x3 / stride 1 / pad 1 fed by TMA halo boxes (dw_tma.cu); dw3_tma_ok says whether
// the shape and pointers take it
bool dw3_tma_ok(const float* in, const float* out, const float* bias, int N, int H, int W, int C,
                int KH, int KW, int stride, int pad, int sm_count);
bool dw3_tma_dev(Call& c, const float* in, int N, int H, int W, int C, const float* w, const float* bias,
                 float* out, int act);
bool group_dev(Call& c, const float* in, int N, int H, int W, int Cin, const float* w,
               const float* bias, int KH, int KW, int Cout, int stride, int pad, int groups,
               float* out, int act);
// fp32 GEMM on device operands on tensor cores (3xTF32 or 3xBF16 per fp32_math, gemm.cu)
// b_split: B already split for 3xBF16 (to_bf16x2), used when that mode is active.
enum class Fp32Use;
struct Operand;
bool gemm_f32(Call& c, const float* dA, long long lda, const float* dB, long long ldb, int M,
              int N, int K, float* dC, long long ldc, const float* dbias, int act, Fp32Use use,
              const Operand* b_split = nullptr);
}  // namespace acf
