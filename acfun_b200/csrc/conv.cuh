// conv.cuh — convolution entry points on device pointers (conv.cu, conv_int8.cu), shared
// by the public API and the model executor.
#pragma once
#include "runtime.cuh"

namespace acf {

enum ConvRoute {
  kRouteDepthwise = 1,
  kRouteGroupedDirect = 2,
  kRouteGroupedSplit = 3,
  kRoute1x1 = 4,
  kRouteWino43 = 5,
  kRouteWino23 = 6,
  kRouteIm2col = 7,
};

// routing of conv2d_impl (layers.cpp:106-195)
int conv_route(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad, int groups);
size_t conv_weight_elems(int Cin, int KH, int KW, int Cout, int groups);

// fp32 conv (any groups, reference weight layouts), fused bias / ReLU.
bool conv2d_dev(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                const float* bias, int KH, int KW, int Cout, int stride, int pad, int groups,
                float* out, int act);
// one dense conv over channels [coff, coff+Cg) of an NHWC tensor with Cs channels; output
// rows have stride ldc.  Weights [KH*KW*Cg][Cout_g] with row stride ldw.
bool conv_f32_dev(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cg,
                  const float* w, long long ldw, const float* bias, int KH, int KW, int Cout_g,
                  int stride, int pad, float* out, long long ldc, int act);

// Dense conv (groups 1) immediately followed by max-pool(pool, pst, ppd, post_relu), fused when
// the conv takes the CUDA-core small-K route and the pool is 2x2 / stride 2 / pad 0 (sets
// *handled; otherwise nothing is launched).  Same result as the two layers run in turn.
bool conv_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                   const float* bias, int KH, int KW, int Cout, int stride, int pad, int act,
                   int pool, int pst, int ppd, int post_relu, float* out, bool* handled);

// The same router over a batch with one activation scale per image, i.e. N separate
// calls of acfun_conv2d_int8 (the reference's per-image model harness) in one pass.
bool conv2d_int8_batch_dev(Call& c, const float* x, int N, int H, int W, int Cin,
                           const int8_t* wq, const float* wscale, const float* bias, int KH,
                           int KW, int Cout, int stride, int pad, float* out, int act);

// conv2d_int8_batch_dev immediately followed by max-pool(2, 2, 0, post_relu), fused for small-K
// non-Winograd routes (sets *handled; otherwise nothing is launched).  Bit-identical to the two
// layers run in turn.
bool conv_int8_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                        const float* wscale, const float* bias, int KH, int KW, int Cout,
                        int stride, int pad, int act, int pool, int pst, int ppd, int post_relu,
                        float* out, bool* handled);

// int8 conv router (conv_int8.cpp:63-148) on device pointers.
bool conv2d_int8_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                     const float* wscale, const float* bias, int KH, int KW, int Cout, int stride,
                     int pad, float* out, int act);

}  // namespace acf
