// conv.cuh — convolution entry points on device pointers (conv.cu, conv_int8.cu), shared
// by the public API and the model executor.
#pragma once
#include "runtime.cuh"

namespace acf {

struct ConvGeom;

enum ConvRoute {
  kRouteDepthwise = 1,
  kRouteGroupedDirect = 2,
  kRouteGroupedSplit = 3,
  kRoute1x1 = 4,
  kRouteWino43 = 5,
  kRouteWino23 = 6,
  kRouteIm2col = 7,
};

// Narrow stride-1 fp32 convolution (Cin, Cout <= 64, KH*KW <= 9) as one 3xBF16 tcgen05 kernel
// with resident weights and in-kernel operand conversion (conv_halo.cu).
bool conv_halo_ok(int Cin, int KH, int KW, int Cout, int stride);
// 1x1 stride-1 fp32 convolution (Cin <= 192, a multiple of 4; Cout <= 64) on tensor cores in
// 3xBF16 (conv_pw_tc.cu); x is [M][Cin] contiguous.
bool conv_pw_tc_ok(const float* x, int Cs, int coff, int Cin, int Cout, long long M);
bool conv_pw_tc_dev(Call& c, const float* x, long long M, int Cin, const float* w, long long ldw,
                    const float* bias, int Cout, float* out, long long ldc, int act);
// Small-K int8 convolution + 2x2/2 max-pool on tensor cores (conv_i8_pool_tc.cu): per-image
// scales (ab = [N][2][Cout] alpha / beta, img_inv, img_zero from k_absmax_img).
bool conv_i8_pool_tc_ok(const float* x, int W, int Cin, int KH, int KW, int Cout, int stride, int PW);
bool conv_i8_pool_tc_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                         int KH, int KW, int Cout, int pad, int PH, int PW, const float* ab,
                         const float* img_inv, const int* img_zero, float* out, int act,
                         int post_relu, unsigned* out_max);
bool conv_halo_f32_dev(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cin,
                       const float* w, long long ldw, const float* bias, int KH, int KW, int Cout,
                       int pad, float* out, long long ldc, int act);

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

// An activation held as the zero-padded bf16 hi / lo planes a 3xBF16 implicit convolution
// reads: [2][N][H + 2*pad][W + 2*pad][C] (C a multiple of 64), the lo plane `plane` elements
// after the hi plane.  Borders are zero.
struct SplitAct {
  void* base = nullptr;
  long long plane = 0;
  int N = 0, H = 0, W = 0, C = 0, pad = 0;
};
// Bytes such an activation takes.
inline long long split_act_bytes(int N, int H, int W, int C, int pad) {
  return 2LL * 2 * N * (H + 2LL * pad) * (W + 2LL * pad) * C;
}
// Whether a dense convolution runs as the 3xBF16 implicit GEMM that split activations feed:
// the model executor then keeps its input (and, when the next layer is one too, its output)
// in split form.
bool conv_split_ok(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad);
// Zero the padding border of `a` (both planes).
bool split_border_dev(Call& c, const SplitAct& a);
// fp32 weights [taps*Cin][Cout] -> the [2][taps*Cin][Np] bf16 split the implicit GEMM takes
// (Np = Cout rounded up to 8).  `dst` holds split_weight_bytes.
long long split_weight_bytes(int taps, int Cin, int Cout);

// Row-pair tiling of a stride-1 implicit convolution over N images of padded height Hp whose
// OH x OW output is max-pooled 2x2 / stride 2 (ConvGeom::pair): fills cg's pair fields and
// returns the GEMM's virtual row count (256 per tile), or 0 when the shape does not qualify
// (odd Hp, output narrower than 2).
long long pair_geometry(ConvGeom& cg, int N, int Hp, int OH, int OW);
bool split_weights_dev(Call& c, const float* w, int taps, int Cin, int Cout, void* dst);
// conv_split_ok convolution from fp32 x (padded + split here) or the split activation xs
// (xs->pad == pad), with pre-split weights ws (or NULL: split here), into fp32 out or, when
// os is given, the next convolution's split input.  pool: the 2x2 / stride-2 / pad-0 max-pool
// that follows runs in the epilogue (output (OH/2) x (OW/2); needs H + 2*pad even), its
// post-ReLU folded into act.
bool conv_tc_split_dev(Call& c, const float* x, const SplitAct* xs, int N, int H, int W,
                       int Cin, const float* w, const void* ws, const float* bias, int KH,
                       int KW, int Cout, int pad, float* out, const SplitAct* os, int act,
                       bool pool = false);

// Dense conv (groups 1) immediately followed by max-pool(pool, pst, ppd, post_relu), fused when
// the conv takes the CUDA-core small-K route and the pool is 2x2 / stride 2 / pad 0 (sets
// *handled; otherwise nothing is launched).  Same result as the two layers run in turn.
// os != NULL: write the pooled result as the next convolution's split input (3x3 / Cin 3 /
// stride 1 / pad 1 kernel only; otherwise nothing is launched).
bool conv_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                   const float* bias, int KH, int KW, int Cout, int stride, int pad, int act,
                   int pool, int pst, int ppd, int post_relu, float* out, bool* handled,
                   const SplitAct* os = nullptr);

// The same router over a batch with one activation scale per image, i.e. N separate
// calls of acfun_conv2d_int8 (the reference's per-image model harness) in one pass.
// in_max: the input's per-image max |x| already accumulated by its producer (skips the absmax
// pass); out_max: accumulate the output's per-image max |y| (zeroed by the caller) for the next
// int8 layer.
// pool: the 2x2 / stride-2 / pad-0 max-pool that follows runs in the GEMM epilogue (output
// (OH/2) x (OW/2)) when int8_pool_ok holds for the shape; its post-ReLU folded into act.
bool conv2d_int8_batch_dev(Call& c, const float* x, int N, int H, int W, int Cin,
                           const int8_t* wq, const float* wscale, const float* bias, int KH,
                           int KW, int Cout, int stride, int pad, float* out, int act,
                           const unsigned* in_max = nullptr, unsigned* out_max = nullptr,
                           bool pool = false);
bool int8_pool_ok(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad);

// conv2d_int8_batch_dev immediately followed by max-pool(2, 2, 0, post_relu), fused for small-K
// non-Winograd routes (sets *handled; otherwise nothing is launched).  Bit-identical to the two
// layers run in turn.  in_max: the per-image input maximum, given instead of measured.
bool conv_int8_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                        const float* wscale, const float* bias, int KH, int KW, int Cout,
                        int stride, int pad, int act, int pool, int pst, int ppd, int post_relu,
                        float* out, bool* handled, unsigned* out_max = nullptr,
                        const unsigned* in_max = nullptr);

// int8 conv router (conv_int8.cpp:63-148) on device pointers.
bool conv2d_int8_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                     const float* wscale, const float* bias, int KH, int KW, int Cout, int stride,
                     int pad, float* out, int act);

}  // namespace acf
