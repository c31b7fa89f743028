// conv_int8.cu — int8 convolution: router, quantisation kernels and the exact integer
// convolution on tcgen05 kind::i8 tensor cores.
//
// Reference (hit-droid/Acfun): conv_int8.cpp:63-148 (router), winograd_int8.cpp:245-350,
// conv_int8_direct.cpp:20-59, conv1x1_int8.cpp:21-36, int8_quantize_avx512.cpp:8-35.
//
// Every route of the reference computes an exact integer correlation of the u8 activations
// (zero point 128, out-of-image taps read 128) with the s8 weights, then dequantises:
//   direct / 1x1 / im2col routes: out = (float)acc * alpha[j] + beta[j]       (mul, then add)
//   Winograd F(2,3) route:        out = fmaf(4*(float)(acc - 128*Sw[j]), wso[j], bias[j])
// The Winograd route's transforms are exact in integers (G~ = 2G is integral, so the
// output transform yields exactly 4x the centred correlation), which is why one integer
// implicit GEMM serves every route bit-exactly; the routes differ only in the activation
// rounding (round-half-even vs the Winograd path's half-away) and in the dequant formula.
// Per-call scalars (max|x|, inv_s = 127/max, s_a = max/127) and per-channel factors are
// derived on the device so a call never synchronises with the host mid-way.
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "api_export.cuh"
#include "conv.cuh"
#include "gemm.cuh"
#include "ops.cuh"

namespace acf {

struct Int8Scalars {
  float inv_s;         // 127 / maxa
  float sa;            // maxa / 127
  int zero;            // maxa < 1e-12: the reference writes an all-zero output
};

// Per-output-channel dequantisation factors, derived on the device once sa is known (same
// expressions as k_int8_colparams).
struct Int8ColArgs {
  const float* wscale;
  const float* bias;
  const int* Sw;
  int Cout;
  int wino;  // 1: f0 = wso; 0: f0 = alpha, f1 = beta
  float* f0;
  float* f1;
};

static int grid_n(Call& c, long long work) {
  long long b = (work + 255) / 256, cap = (long long)c.sm_count() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// conv_int8.cpp:75-77: maxa = max(maxa, |x|) (std::max keeps maxa when |x| is NaN).
// One block's share of max|x| over x[0, n): grid-stride over float4 with four loads in flight
// per thread; returns the block maximum (valid in every thread).
__device__ float block_absmax(const float* __restrict__ x, long long n, int b, int nb) {
  __shared__ float sh[33];
  float m = 0.0f;
  const long long step = (long long)nb * blockDim.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const long long n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    long long i = b * (long long)blockDim.x + threadIdx.x;
    for (; i + 3 * step < n4; i += 4 * step) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldg(x4 + i + u * step);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float a = fabsf(q[u].x), bb = fabsf(q[u].y), cc = fabsf(q[u].z), d = fabsf(q[u].w);
        m = (m < a) ? a : m;
        m = (m < bb) ? bb : m;
        m = (m < cc) ? cc : m;
        m = (m < d) ? d : m;
      }
    }
    for (; i < n4; i += step) {
      const float4 q = __ldg(x4 + i);
      const float a = fabsf(q.x), bb = fabsf(q.y), cc = fabsf(q.z), d = fabsf(q.w);
      m = (m < a) ? a : m;
      m = (m < bb) ? bb : m;
      m = (m < cc) ? cc : m;
      m = (m < d) ? d : m;
    }
    for (long long k = (n4 << 2) + b * (long long)blockDim.x + threadIdx.x; k < n; k += step) {
      const float v = fabsf(x[k]);
      m = (m < v) ? v : m;
    }
  } else {
    for (long long k = b * (long long)blockDim.x + threadIdx.x; k < n; k += step) {
      const float v = fabsf(x[k]);
      m = (m < v) ? v : m;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, m, o);
    m = (m < u) ? u : m;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, m, o);
      m = (m < u) ? u : m;
    }
    if (threadIdx.x == 0) sh[32] = m;
  }
  __syncthreads();
  return sh[32];
}

// Weight preparation for one output channel (a block): s8 [taps*Cin][Cout] -> K-major row n of
// [Cout][taps*Cpad] (each tap's Cin weights, then zeros up to Cpad) and its column sum Sw[n].
__device__ void wprep_channel(const int8_t* __restrict__ w, int taps, int Cin, int Cout, int Cpad,
                              int n, int8_t* __restrict__ dst, int* __restrict__ Sw) {
  __shared__ int red[32];
  const int K4 = taps * Cpad / 4;
  uint32_t* row = reinterpret_cast<uint32_t*>(dst + (size_t)n * taps * Cpad);
  int sum = 0;
  for (int i = threadIdx.x; i < K4; i += blockDim.x) {
    const int k = i * 4, tap = k / Cpad, c0 = k - tap * Cpad;
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + e;
      const int8_t v = c < Cin ? w[((long long)tap * Cin + c) * Cout + n] : (int8_t)0;
      sum += v;
      packed |= (uint32_t)(uint8_t)v << (8 * e);
    }
    row[i] = packed;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    Sw[n] = t;
  }
}

// First launch of a per-call int8 convolution: blocks [0, Cout) prepare the weights (one
// output channel each), blocks [Cout, Cout + nparts) write part[b - Cout] = the maximum of
// |x| over their share.  The partial maxima need no clearing and no counter; the quantiser
// that runs next reduces them (Int8Derive).
__global__ void k_int8_prep_absmax(const int8_t* __restrict__ w, int taps, int Cin, int Cout,
                                   int Cpad, int8_t* __restrict__ wk, int* __restrict__ Sw,
                                   const float* __restrict__ x, long long n, float* __restrict__ part,
                                   int nparts) {
  dev::grid_dep_launch();  // the quantiser may start its prologue now
  if ((int)blockIdx.x < Cout) {
    wprep_channel(w, taps, Cin, Cout, Cpad, blockIdx.x, wk, Sw);
    return;
  }
  const int b = (int)blockIdx.x - Cout;
  const float m = block_absmax(x, n, b, nparts);
  if (threadIdx.x == 0) part[b] = m;
}

// Per-call activation scalars from k_int8_prep_absmax's partial maxima, derived by every block
// of the kernel that quantises the activation (so no launch waits on a single block):
// maxa = max(part[]), inv_s = 127/maxa; block 0 also stores inv_s, sa = maxa/127 and the
// all-zero flag in *s and the per-channel dequantisation factors of ca.
struct Int8Derive {
  const float* part = nullptr;
  int nparts = 0;
  Int8Scalars* s = nullptr;
  Int8ColArgs ca{};
};

__device__ float derive_inv_s(const Int8Derive& d) {
  __shared__ float sh[33];
  float m = 0.0f;
  for (int i = threadIdx.x; i < d.nparts; i += blockDim.x) {
    const float v = d.part[i];
    m = (m < v) ? v : m;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, m, o);
    m = (m < u) ? u : m;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, m, o);
      m = (m < u) ? u : m;
    }
    if (threadIdx.x == 0) sh[32] = m;
  }
  __syncthreads();
  const float maxa = sh[32];
  if (blockIdx.x == 0) {
    const float sa = __fdiv_rn(maxa, 127.0f);
    if (threadIdx.x == 0) {
      d.s->zero = maxa < 1e-12f ? 1 : 0;
      d.s->inv_s = __fdiv_rn(127.0f, maxa);
      d.s->sa = sa;
    }
    const Int8ColArgs& ca = d.ca;
    for (int j = threadIdx.x; j < ca.Cout; j += blockDim.x) {
      if (ca.wino) {
        ca.f0[j] = __fmul_rn(__fmul_rn(sa, 0.25f), ca.wscale[j]);
      } else {
        const float a = __fmul_rn(sa, ca.wscale[j]);
        const float corr = __fmul_rn(__fmul_rn(a, 128.0f), (float)ca.Sw[j]);
        ca.f0[j] = a;
        ca.f1[j] = __fsub_rn(ca.bias ? ca.bias[j] : 0.0f, corr);
      }
    }
  }
  return __fdiv_rn(127.0f, maxa);
}

// The activation scale a quantiser uses: derived from partial maxima, else inv_host.
__device__ __forceinline__ float quant_inv_all(const Int8Derive& d, float inv_host) {
  return d.part ? derive_inv_s(d) : inv_host;
}

// Per output channel j (one warp each): Sw = sum_k wq[k][j]; alpha = sa*ws; beta =
// bias - (alpha*128)*Sw (conv_int8.cpp:100-107, no contraction); wso = (sa*0.25)*ws
// (winograd_int8.cpp:155), for a caller-supplied sa.
__global__ void k_int8_colparams(const int8_t* __restrict__ wq, int K, int Cout,
                                 const float* __restrict__ wscale, const float* __restrict__ bias,
                                 float sa, float* alpha, float* beta, float* wso, int* Sw) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= Cout) return;
  const int j = warp;
  int sum = 0;
  for (int k = lane; k < K; k += 32) sum += wq[(long long)k * Cout + j];
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) {
    const float a = __fmul_rn(sa, wscale[j]);
    const float corr = __fmul_rn(__fmul_rn(a, 128.0f), (float)sum);
    if (alpha) alpha[j] = a;
    if (beta) beta[j] = __fsub_rn(bias ? bias[j] : 0.0f, corr);
    if (wso) wso[j] = __fmul_rn(__fmul_rn(sa, 0.25f), wscale[j]);
    if (Sw) Sw[j] = sum;
  }
}

// lroundf semantics (ties away from zero), exact for |t| < 2^31
__device__ __forceinline__ int round_half_away(float t) {
  const float a = fabsf(t);
  const float f = floorf(a);
  const float r = (a - f >= 0.5f) ? f + 1.0f : f;
  return (int)copysignf(r, t);
}

__device__ __forceinline__ uint8_t clamp_u8(int v) {
  return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
}

// Activation quantisation (zp = 128) into a spatially padded NHWC buffer [N*Hp*Wp][Cpad];
// border cells and padding channels hold the zero point.
//   mode 0: cvt_rne(x*inv_s) + 128            (int8_quantize_avx512.cpp:16)
//   mode 1: channels < Cin&~15: trunc(t + copysign(0.5, t)); tail channels: lroundf(t)
//           (winograd_int8.cpp:306-325)
__global__ void k_quant_pad_u8(const float* __restrict__ x, int N, int H, int W, int Cin, int pad,
                               int Hp, int Wp, int Cpad, Int8Derive dv, float inv_host,
                               const float* __restrict__ img_inv, int mode,
                               uint8_t* __restrict__ dst) {
  const float inv_all = quant_inv_all(dv, inv_host);
  const int cvec = Cin & ~15;
  const long long total = (long long)N * Hp * Wp * Cpad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % Cpad);
    long long p = i / Cpad;
    const int wp = (int)(p % Wp);
    p /= Wp;
    const int hp = (int)(p % Hp);
    const int n = (int)(p / Hp);
    const int ih = hp - pad, iw = wp - pad;
    uint8_t q = 128;
    if (c < Cin && ih >= 0 && ih < H && iw >= 0 && iw < W) {
      const float inv_s = img_inv ? img_inv[n] : inv_all;
      const float t = __fmul_rn(x[(((long long)n * H + ih) * W + iw) * Cin + c], inv_s);
      int v;
      if (mode == 0) {
        v = (fabsf(t) < 2147483648.0f) ? __float2int_rn(t) : (int)0x80000000;
      } else if (c < cvec) {
        const float r = __fadd_rn(t, copysignf(0.5f, t));
        v = (fabsf(r) < 2147483648.0f) ? (int)truncf(r) : (int)0x80000000;
      } else {
        v = round_half_away(t);
      }
      q = clamp_u8((int)((unsigned)v + 128u));
    }
    dst[i] = q;
  }
}

__device__ __forceinline__ uint8_t quant_one(float xv, float inv_s, int mode, bool vec_lane) {
  const float t = __fmul_rn(xv, inv_s);
  int v;
  if (mode == 0) {
    v = (fabsf(t) < 2147483648.0f) ? __float2int_rn(t) : (int)0x80000000;
  } else if (vec_lane) {
    const float r = __fadd_rn(t, copysignf(0.5f, t));
    v = (fabsf(r) < 2147483648.0f) ? (int)truncf(r) : (int)0x80000000;
  } else {
    v = round_half_away(t);
  }
  return clamp_u8((int)((unsigned)v + 128u));
}

// Integer rounding on the FMA pipe (no conversion-unit instruction): adding 1.5 * 2^23
// (resp. 2^23 with round-toward-zero) leaves the rounded value in the low mantissa bits.
// rne_small: round-half-even of t, |t| <= 2^22.  floor_small: floor of a in [0, 2^23).
__device__ __forceinline__ int rne_small(float t) {
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}
__device__ __forceinline__ int floor_small(float a) {
  return __float_as_int(__fadd_rz(a, 8388608.0f)) - 0x4B000000;
}

// Same result as quant_one for a vector lane (mode 0: cvt_rne; mode 1: trunc(t + copysign(.5,
// t))), |t| >= 2^31 and NaN giving the x86 "integer indefinite" INT_MIN, i.e. byte 0.
template <int MODE>
__device__ __forceinline__ uint32_t quant_fast(float xv, float inv_s) {
  const float t = __fmul_rn(xv, inv_s);
  int v;
  if constexpr (MODE == 0) {
    if (!(fabsf(t) < 2147483648.0f)) return 0u;
    v = rne_small(fminf(fmaxf(t, -256.0f), 256.0f));
  } else {
    const float r = __fadd_rn(t, copysignf(0.5f, t));
    if (!(fabsf(r) < 2147483648.0f)) return 0u;
    const int f = floor_small(fminf(fabsf(r), 256.0f));
    v = r < 0.0f ? -f : f;
  }
  v += 128;
  return (uint32_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
}

// k_quant_pad_u8 with one thread per (padded pixel, 16 channels), 32-bit index math and one
// 16-byte store (Cpad is a multiple of 16); used when the tensor has < 2^31 such groups.
template <int MODE>
__global__ void k_quant_pad_u8_16(const float* __restrict__ x, int H, int W, int Cin, int pad,
                                  int Hp, int Wp, int C16, unsigned total, int vec_in,
                                  Int8Derive dv, float inv_host,
                                  const float* __restrict__ img_inv, uint4* __restrict__ dst) {
  dev::grid_dep_wait();    // launched as the dependent of the kernel producing x / the scalars
  dev::grid_dep_launch();  // and the conv after it may start its prologue
  const float inv_all = quant_inv_all(dv, inv_host);
  const int cvec = Cin & ~15;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const unsigned cg = i % C16, p = i / C16;
    const unsigned wp = p % Wp, t = p / Wp;
    const unsigned hp = t % Hp, n = t / Hp;
    const int ih = (int)hp - pad, iw = (int)wp - pad, c0 = (int)cg * 16;
    uint32_t w[4] = {0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u};
    if (c0 < Cin && ih >= 0 && ih < H && iw >= 0 && iw < W) {
      const float* src = x + (((size_t)n * H + ih) * W + iw) * Cin + c0;
      const float inv_s = img_inv ? img_inv[n] : inv_all;
      if (vec_in && c0 + 16 <= Cin) {
        // whole group of vector lanes: no per-lane checks
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(src + 4 * k));
          w[k] = quant_fast<MODE>(q.x, inv_s) | (quant_fast<MODE>(q.y, inv_s) << 8) |
                 (quant_fast<MODE>(q.z, inv_s) << 16) | (quant_fast<MODE>(q.w, inv_s) << 24);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint8_t q =
              (c0 + k < Cin) ? quant_one(src[k], inv_s, MODE, c0 + k < cvec) : (uint8_t)128;
          w[k >> 2] = (w[k >> 2] & ~(0xFFu << (8 * (k & 3)))) | ((uint32_t)q << (8 * (k & 3)));
        }
      }
    }
    dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// k_quant_pad_u8_16 for 64-channel rows (Cin == Cpad == 64, 16-byte aligned input): a block walks
// whole padded grid rows (n, hp), so the image / row arithmetic is done once per row and a thread
// takes (pixel, 16-channel group) = (item >> 2, item & 3) of the row -- no per-item division.
template <int MODE>
__global__ void k_quant_pad_rows64(const float* __restrict__ x, int H, int W, int pad, int Hp, int Wp,
                                   int nrows, Int8Derive dv, float inv_host,
                                   const float* __restrict__ img_inv, uint4* __restrict__ dst) {
  dev::grid_dep_wait();    // launched as the dependent of the kernel producing x / the scalars
  dev::grid_dep_launch();  // and the conv after it may start its prologue
  const float inv_all = quant_inv_all(dv, inv_host);
  const int items = Wp * 4;
  for (int row = blockIdx.x; row < nrows; row += gridDim.x) {
    const int n = row / Hp, ih = row - n * Hp - pad;
    const bool row_in = ih >= 0 && ih < H;
    const float inv_s = img_inv ? img_inv[n] : inv_all;
    const float* src_row = x + ((size_t)n * H + (row_in ? ih : 0)) * W * 64;
    uint4* dst_row = dst + (size_t)row * items;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
      const int iw = (it >> 2) - pad, cg = it & 3;
      uint32_t w[4] = {0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u};
      if (row_in && iw >= 0 && iw < W) {
        const float4* src = reinterpret_cast<const float4*>(src_row + (size_t)iw * 64 + cg * 16);
        float4 q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = __ldg(src + k);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          w[k] = quant_fast<MODE>(q[k].x, inv_s) | (quant_fast<MODE>(q[k].y, inv_s) << 8) |
                 (quant_fast<MODE>(q[k].z, inv_s) << 16) | (quant_fast<MODE>(q[k].w, inv_s) << 24);
      }
      dst_row[it] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// pre-quantised u8 NHWC -> padded [N*Hp*Wp][Cpad] (border = zero point)
__global__ void k_pad_u8(const uint8_t* __restrict__ xq, int N, int H, int W, int Cin, int pad,
                         int Hp, int Wp, int Cpad, uint8_t* __restrict__ dst) {
  const long long total = (long long)N * Hp * Wp * Cpad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % Cpad);
    long long p = i / Cpad;
    const int wp = (int)(p % Wp);
    p /= Wp;
    const int hp = (int)(p % Hp);
    const int n = (int)(p / Hp);
    const int ih = hp - pad, iw = wp - pad;
    uint8_t q = 128;
    if (c < Cin && ih >= 0 && ih < H && iw >= 0 && iw < W)
      q = xq[(((long long)n * H + ih) * W + iw) * Cin + c];
    dst[i] = q;
  }
}

// u8 im2col (im2col_u8, conv_int8.cpp:42-61): out-of-image taps hold the zero point
__global__ void k_im2col_u8(const uint8_t* __restrict__ xq, int N, int H, int W, int Cin, int KH,
                            int KW, int stride, int pad, int OH, int OW, int Kpad,
                            uint8_t* __restrict__ dst) {
  const long long total = (long long)N * OH * OW * Kpad;
  const int K = KH * KW * Cin;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % Kpad);
    long long m = i / Kpad;
    const int ow = (int)(m % OW);
    m /= OW;
    const int oh = (int)(m % OH);
    const int n = (int)(m / OH);
    uint8_t q = 128;
    if (k < K) {
      const int tap = k / Cin, c = k - tap * Cin;
      const int ih = oh * stride - pad + tap / KW, iw = ow * stride - pad + tap % KW;
      if (ih >= 0 && ih < H && iw >= 0 && iw < W) q = xq[(((long long)n * H + ih) * W + iw) * Cin + c];
    }
    dst[i] = q;
  }
}

// k_im2col_u8 with one thread per (output pixel, 16 K bytes): 32-bit index math, the tap /
// channel position advanced incrementally, one 16-byte store (Kpad is a multiple of 16).
__global__ void k_im2col_u8_16(const uint8_t* __restrict__ xq, int H, int W, int Cin, int KH,
                               int KW, int stride, int pad, int OH, int OW, int K16,
                               unsigned total, uint4* __restrict__ dst) {
  const int K = KH * KW * Cin;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const unsigned g = i % K16, m = i / K16;
    const unsigned ow = m % OW, r = m / OW, oh = r % OH, n = r / OH;
    int k = (int)g * 16;
    int tap = k / Cin, c = k - tap * Cin;
    int kh = tap / KW, kw = tap - kh * KW;
    const uint8_t* img = xq + (size_t)n * H * W * Cin;
    uint32_t wv[4] = {0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u};
#pragma unroll
    for (int e = 0; e < 16; ++e, ++k) {
      if (k < K) {
        const int ih = (int)oh * stride - pad + kh, iw = (int)ow * stride - pad + kw;
        if (ih >= 0 && ih < H && iw >= 0 && iw < W) {
          const uint32_t q = img[((size_t)ih * W + iw) * Cin + c];
          wv[e >> 2] = (wv[e >> 2] & ~(0xFFu << (8 * (e & 3)))) | (q << (8 * (e & 3)));
        }
        if (++c == Cin) {
          c = 0;
          if (++kw == KW) {
            kw = 0;
            ++kh;
          }
        }
      }
    }
    dst[i] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// Dense (unpadded) u8 quantisation of a whole NHWC tensor, 4 elements per thread (float4 in,
// one 32-bit store): the same rounding as k_quant_pad_u8 (vector lanes = channels below
// Cin & ~15 in mode 1), one scale per image when img_inv is given.
template <int MODE>
__global__ void k_quant_u8_flat4(const float4* __restrict__ x, unsigned n4, int Cin,
                                 unsigned per_img, Int8Derive dv, float inv_host,
                                 const float* __restrict__ img_inv, uint32_t* __restrict__ dst) {
  const float inv_all = quant_inv_all(dv, inv_host);
  const int cvec = Cin & ~15;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    const float4 v = __ldg(x + i);
    const float xv[4] = {v.x, v.y, v.z, v.w};
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const unsigned idx = i * 4 + e;
      const float inv_s = img_inv ? img_inv[idx / per_img] : inv_all;
      const int c = (int)(idx % (unsigned)Cin);
      w |= (uint32_t)quant_one(xv[e], inv_s, MODE, c < cvec) << (8 * e);
    }
    dst[i] = w;
  }
}

// s8 weights [taps*Cin][Cout] -> K-major [Cout][taps*Cpad] (row n holds output channel n's
// taps, each tap's Cin weights followed by zeros up to Cpad).  One thread per 4 K bytes.
__global__ void k_weights_s8k(const int8_t* __restrict__ w, int taps, int Cin, int Cout, int Cpad,
                              int8_t* __restrict__ dst) {
  const int K4 = taps * Cpad / 4;
  const long long total = (long long)Cout * K4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K4), k = (int)(i - (long long)n * K4) * 4;
    const int tap = k / Cpad, c0 = k - tap * Cpad;
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + e;
      const int8_t v = c < Cin ? w[((long long)tap * Cin + c) * Cout + n] : (int8_t)0;
      packed |= (uint32_t)(uint8_t)v << (8 * e);
    }
    reinterpret_cast<uint32_t*>(dst)[i] = packed;
  }
}

// wprep_channel for every output channel (one block each); block 0 also clears the nclear
// words that k_absmax_img accumulates into.
__global__ void k_int8_wprep(const int8_t* __restrict__ w, int taps, int Cin, int Cout, int Cpad,
                             int8_t* __restrict__ dst, int* __restrict__ Sw,
                             unsigned* __restrict__ clear, int nclear) {
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nclear; i += blockDim.x) clear[i] = 0u;
  wprep_channel(w, taps, Cin, Cout, Cpad, blockIdx.x, dst, Sw);
}

// 64-byte K blocks when they cut the channel padding (Cin mod 128 in 1..64), else 128
static int int8_kblock(int k) { return (k % 128 != 0 && k % 128 <= 64) ? 64 : 128; }

// Quantised input + exact integer conv + dequant epilogue.
//   xf / xq: float input (quantised here with `qmode`, scalars from `s` or inv_host) or
//            pre-quantised u8 input.
struct Int8ConvArgs {
  const float* xf = nullptr;
  const uint8_t* xq = nullptr;
  int qmode = 0;
  Int8Derive dv;       // per-call scalars derived in the quantiser (else inv_host)
  float inv_host = 0.0f;
  Epi epi = Epi::F32_AB;
  const float* f0 = nullptr;  // alpha | wso
  const float* f1 = nullptr;  // beta | bias
  const int* i0 = nullptr;    // Sw (Winograd epilogue)
  const int* zero_flag = nullptr;
  // one activation scale per image (batch-1 semantics): 127/max and max/127 of image n,
  // its all-zero flag; f0 / f1 / i0 are then weight scale / bias / Sw
  const float* img_inv = nullptr;
  const float* img_sa = nullptr;
  const int* img_zero = nullptr;
  // per-image max |output| accumulator for the next int8 layer (EpiParams::img_absmax)
  unsigned* out_max = nullptr;
};

// K-major weight layout a convolution's GEMM uses: implicit route (stride 1, Cin >= 32):
// `taps` taps of Cpad channels; im2col route: one "tap" of Cpad = align(KH*KW*Cin, 16).
struct Int8BLayout {
  bool implicit;
  int taps, cin, cpad, bkb;
};
static Int8BLayout int8_b_layout(int Cin, int KH, int KW, int stride) {
  Int8BLayout L;
  L.implicit = stride == 1 && Cin >= 32;
  if (L.implicit) {
    L.taps = KH * KW;
    L.cin = Cin;
    L.bkb = int8_kblock(Cin);
    L.cpad = (int)align_up((size_t)Cin, L.bkb);
  } else {
    L.taps = 1;
    L.cin = KH * KW * Cin;
    L.cpad = (int)align_up((size_t)L.cin, 16);
    L.bkb = int8_kblock(L.cpad);
  }
  return L;
}

// wk: weights already in int8_b_layout's K-major form (else prepared here from wq)
static bool int8_conv_gemm(Call& c, const Int8ConvArgs& a, int N, int H, int W, int Cin,
                           const int8_t* wq, int KH, int KW, int Cout, int stride, int pad,
                           float* out, int act, const int8_t* wk = nullptr, bool pool = false) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return true;
  const int taps = KH * KW;
  EpiParams ep{};
  ep.C = out;
  ep.ldc = Cout;
  ep.f0 = a.f0;
  ep.f1 = a.f1;
  ep.i0 = a.i0;
  ep.act = act;
  ep.zero_flag = a.zero_flag;
  ep.img_sa = a.img_sa;
  ep.img_zero = a.img_zero;
  ep.img_absmax = a.out_max;
  uint8_t* xq_dense = nullptr;  // unpadded u8 input for the gather path
  const Int8BLayout lay = int8_b_layout(Cin, KH, KW, stride);
  if (lay.implicit) {
    // implicit GEMM over the zero-point-padded tensor
    const int bkb = lay.bkb, Cpad = lay.cpad;
    const int Hp = H + 2 * pad, Wp = W + 2 * pad;
    const long long rows = (long long)N * Hp * Wp;
    uint8_t* A = (uint8_t*)c.scratch((size_t)rows * Cpad);
    int8_t* B = wk ? const_cast<int8_t*>(wk) : (int8_t*)c.scratch((size_t)Cout * taps * Cpad);
    if (!A || !B) return false;
    if (a.xf && rows * (Cpad / 16) < (1LL << 31)) {
      const long long g16 = rows * (Cpad / 16);
      // one resident wave when every block first derives the scalars from partial maxima
      int gq = grid_n(c, g16);
      if (a.dv.part && gq > 8 * c.sm_count()) gq = 8 * c.sm_count();
      const int vec_in = (Cin % 4 == 0) && aligned16(a.xf);
      const long long nrows = (long long)N * Hp;
      const bool rows64 = Cin == 64 && Cpad == 64 && vec_in && a.dv.part && nrows < (1LL << 31);
      const int gr = (int)std::min<long long>(nrows, 8LL * c.sm_count());
      const cudaError_t e =
          rows64 ? (a.qmode == 0 ? launch_pdl(k_quant_pad_rows64<0>, dim3(gr), dim3(256), 0, c.stream(), a.xf, H, W,
                                              pad, Hp, Wp, (int)nrows, a.dv, a.inv_host, a.img_inv, (uint4*)A)
                                 : launch_pdl(k_quant_pad_rows64<1>, dim3(gr), dim3(256), 0, c.stream(), a.xf, H, W,
                                              pad, Hp, Wp, (int)nrows, a.dv, a.inv_host, a.img_inv, (uint4*)A))
          : a.qmode == 0
              ? launch_pdl(k_quant_pad_u8_16<0>, dim3(gq), dim3(256), 0, c.stream(), a.xf, H, W, Cin, pad,
                           Hp, Wp, Cpad / 16, (unsigned)g16, vec_in, a.dv, a.inv_host, a.img_inv, (uint4*)A)
              : launch_pdl(k_quant_pad_u8_16<1>, dim3(gq), dim3(256), 0, c.stream(), a.xf, H, W, Cin, pad,
                           Hp, Wp, Cpad / 16, (unsigned)g16, vec_in, a.dv, a.inv_host, a.img_inv, (uint4*)A);
      if (!ACF_CUDA_OK(e)) {
        c.fail();
        return false;
      }
    } else if (a.xf)
      k_quant_pad_u8<<<grid_n(c, rows * Cpad), 256, 0, c.stream()>>>(
          a.xf, N, H, W, Cin, pad, Hp, Wp, Cpad, a.dv, a.inv_host, a.img_inv, a.qmode, A);
    else
      k_pad_u8<<<grid_n(c, rows * Cpad), 256, 0, c.stream()>>>(a.xq, N, H, W, Cin, pad, Hp, Wp,
                                                               Cpad, A);
    if (!wk)
      k_weights_s8k<<<grid_n(c, (long long)Cout * taps * Cpad / 4), 256, 0, c.stream()>>>(
          wq, taps, Cin, Cout, Cpad, B);
    if (!c.launched("int8 implicit prep")) return false;
    // narrow convolutions: resident weights, one staged slab of input rows per tile
    static const bool halo_on = [] {
      const char* e = getenv("ACFUN_CONV_HALO");
      return !(e && !strcmp(e, "0"));
    }();
    if (halo_on && !pool && rows < (1LL << 31) - 4096 &&
        conv_halo_i8_ok(Cpad, KH, KW, Cout, stride, Wp))
      return conv_halo_i8_dev(c, a.epi, A, B, N, Hp, Wp, KH, KW, OH, OW, Cout, ep);
    Operand Ao, Bo;
    Ao.p = A;
    Ao.ld = Cpad;
    Bo.p = B;
    Bo.ld = (long long)taps * Cpad;
    ep.remap = 1;
    ep.img_rows = Hp * Wp;
    ep.Wp = Wp;
    ep.OH = OH;
    ep.OW = OW;
    ConvGeom cg{1, Cpad / bkb, KW, Wp, Cpad, taps};
    long long M = rows;
    if (pool) {  // 2x2 / stride-2 max-pool in the epilogue (int8_pool_ok)
      M = pair_geometry(cg, N, Hp, OH, OW);
      if (M <= 0 || M >= (1LL << 31)) {
        set_error(kInvalid, "%s: pooled int8 conv geometry", c.name());
        c.fail();
        return false;
      }
      ep.remap = 0;
      ep.ph = OH / 2;
      ep.pw = OW / 2;
    }
    return gemm_launch_i8k(c, a.epi, Ao, Bo, (int)M, Cout, taps * Cpad, ep, cg, bkb);
  }
  if (pool) {
    set_error(kInvalid, "%s: pooled int8 conv needs the implicit route", c.name());
    c.fail();
    return false;
  }
  // explicit im2col over the quantised input
  const uint8_t* src = a.xq;
  if (a.xf) {
    const long long nel = (long long)N * H * W * Cin;
    xq_dense = (uint8_t*)c.scratch((size_t)nel);
    if (!xq_dense) return false;
    if (nel % 4 == 0 && nel < (1LL << 32) && aligned16(a.xf)) {
      const unsigned n4 = (unsigned)(nel / 4), per = (unsigned)((long long)H * W * Cin);
      if (a.qmode == 0)
        k_quant_u8_flat4<0><<<grid_n(c, n4), 256, 0, c.stream()>>>(
            (const float4*)a.xf, n4, Cin, per, a.dv, a.inv_host, a.img_inv, (uint32_t*)xq_dense);
      else
        k_quant_u8_flat4<1><<<grid_n(c, n4), 256, 0, c.stream()>>>(
            (const float4*)a.xf, n4, Cin, per, a.dv, a.inv_host, a.img_inv, (uint32_t*)xq_dense);
    } else {
      k_quant_pad_u8<<<grid_n(c, nel), 256, 0, c.stream()>>>(
          a.xf, N, H, W, Cin, 0, H, W, Cin, a.dv, a.inv_host, a.img_inv, a.qmode, xq_dense);
    }
    src = xq_dense;
  }
  const long long M = (long long)N * OH * OW;
  const int K = lay.cin, Kpad = lay.cpad;
  uint8_t* A = (uint8_t*)c.scratch((size_t)M * Kpad);
  int8_t* B = wk ? const_cast<int8_t*>(wk) : (int8_t*)c.scratch((size_t)Cout * Kpad);
  if (!A || !B) return false;
  if (M * (Kpad / 16) < (1LL << 31) && (long long)H * W * Cin < (1LL << 31)) {
    const unsigned tot16 = (unsigned)(M * (Kpad / 16));
    k_im2col_u8_16<<<grid_n(c, tot16), 256, 0, c.stream()>>>(src, H, W, Cin, KH, KW, stride, pad,
                                                              OH, OW, Kpad / 16, tot16, (uint4*)A);
  } else {
    k_im2col_u8<<<grid_n(c, M * Kpad), 256, 0, c.stream()>>>(src, N, H, W, Cin, KH, KW, stride,
                                                             pad, OH, OW, Kpad, A);
  }
  if (!wk)
    k_weights_s8k<<<grid_n(c, (long long)Cout * Kpad / 4), 256, 0, c.stream()>>>(wq, 1, K, Cout,
                                                                                Kpad, B);
  if (!c.launched("int8 im2col prep")) return false;
  ep.img_rows = OH * OW;  // GEMM rows per image (per-image scales; no remap on this route)
  Operand Ao, Bo;
  Ao.p = A;
  Ao.ld = Kpad;
  Bo.p = B;
  Bo.ld = Kpad;
  return gemm_launch_i8k(c, a.epi, Ao, Bo, (int)M, Cout, Kpad, ep, ConvGeom{}, lay.bkb);
}

static bool is_wino_route(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad) {
  return KH == 3 && KW == 3 && stride == 1 && pad == 1 && H >= 3 && W >= 3 && Cin >= 4 && Cout >= 4;
}

bool conv2d_int8_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                     const float* wscale, const float* bias, int KH, int KW, int Cout, int stride,
                     int pad, float* out, int act) {
  // 3 launches: weights -> K-major + Sw next to the partial maxima of |x|; quantise + pad
  // (every block derives inv_s from the partials, block 0 also sa and the per-channel
  // factors); the integer GEMM with its epilogue.
  const Int8BLayout lay = int8_b_layout(Cin, KH, KW, stride);
  const long long n = (long long)N * H * W * Cin;
  long long np = (n / 4 + 511) / 512;
  const long long np_cap = 2LL * c.sm_count();
  np = np < 1 ? 1 : (np > np_cap ? np_cap : np);
  Int8Scalars* s = (Int8Scalars*)c.scratch(sizeof(Int8Scalars));
  float* part = (float*)c.scratch((size_t)np * 4);
  float* f0 = (float*)c.scratch((size_t)Cout * 4);
  float* f1 = (float*)c.scratch((size_t)Cout * 4);
  int* Sw = (int*)c.scratch((size_t)Cout * 4);
  int8_t* wk = (int8_t*)c.scratch((size_t)Cout * lay.taps * lay.cpad);
  if (!s || !part || !f0 || !f1 || !Sw || !wk) return false;
  k_int8_prep_absmax<<<(unsigned)(Cout + np), 512, 0, c.stream()>>>(
      wq, lay.taps, lay.cin, Cout, lay.cpad, wk, Sw, x, n, part, (int)np);
  if (!c.launched("int8 params")) return false;
  const bool wino = is_wino_route(H, W, Cin, KH, KW, Cout, stride, pad);
  Int8ConvArgs a;
  a.xf = x;
  // Winograd: f0 = wso, f1 = bias (or NULL); others: f0 = alpha, f1 = beta
  a.dv.part = part;
  a.dv.nparts = (int)np;
  a.dv.s = s;
  a.dv.ca = Int8ColArgs{wscale, bias, Sw, Cout, wino ? 1 : 0, f0, f1};
  a.zero_flag = &s->zero;
  if (wino) {
    a.qmode = 1;
    a.epi = Epi::I8_WINO;
    a.f0 = f0;
    a.f1 = bias;
    a.i0 = Sw;
  } else {
    a.qmode = 0;
    a.epi = Epi::F32_AB;
    a.f0 = f0;
    a.f1 = f1;
  }
  return int8_conv_gemm(c, a, N, H, W, Cin, wq, KH, KW, Cout, stride, pad, out, act, wk);
}

// Per-image max|x| for an int8 convolution over a batch with batch-1 semantics (the reference
// quantises per call, conv_int8.cpp:75-81, and its model harness calls per image): grid
// (blocks, images); the last block of image n derives inv[n] = 127/max, sa[n] = max/127 and
// zero[n].  maxa[] and done[] are cleared by k_int8_wprep.
// preset (optional): a given per-image maximum (the bits of a non-negative float) used instead of
// reading x -- a model's stored static activation range; launch with per_img = 0 then.
__global__ void k_absmax_img(const float* __restrict__ x, long long per_img, unsigned* maxa,
                             unsigned* done, float* inv, float* sa, int* zero,
                             const float* __restrict__ wscale, const float* __restrict__ bias,
                             const int* __restrict__ Sw, int Cout, float* __restrict__ ab,
                             const unsigned* __restrict__ preset) {
  dev::grid_dep_launch();  // a programmatic dependent may start its prologue now
  __shared__ float sh[32];
  __shared__ int last;
  const int n = blockIdx.y;
  const float* xi = x + (size_t)n * per_img;
  float m = 0.0f;
  long long i0 = 0;
  if ((reinterpret_cast<uintptr_t>(xi) & 15) == 0) {
    const long long n4 = per_img >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(xi);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
      const float4 q = __ldg(x4 + i);
      const float a = fabsf(q.x), b = fabsf(q.y), cc = fabsf(q.z), d = fabsf(q.w);
      m = (m < a) ? a : m;
      m = (m < b) ? b : m;
      m = (m < cc) ? cc : m;
      m = (m < d) ? d : m;
    }
    i0 = n4 << 2;
  }
  for (long long i = i0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < per_img;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = fabsf(xi[i]);
    m = (m < v) ? v : m;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, m, o);
    m = (m < u) ? u : m;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, m, o);
      m = (m < u) ? u : m;
    }
    if (threadIdx.x == 0) {
      unsigned mv = __float_as_uint(m);
      if (preset) mv = mv < preset[n] ? preset[n] : mv;
      atomicMax(&maxa[n], mv);
      __threadfence();
      last = (atomicAdd(&done[n], 1u) == gridDim.x - 1) ? 1 : 0;
    }
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float mx = __uint_as_float(atomicOr(&maxa[n], 0u));
  const float s_a = __fdiv_rn(mx, 127.0f);
  if (threadIdx.x == 0) {
    zero[n] = mx < 1e-12f ? 1 : 0;
    inv[n] = __fdiv_rn(127.0f, mx);
    sa[n] = s_a;
  }
  // optional per-image alpha / beta table ab[n][0..Cout) / [Cout..2Cout): the expressions of
  // k_int8_colparams (alpha = sa*ws, beta = bias - (alpha*128)*Sw)
  if (ab)
    for (int j = threadIdx.x; j < Cout; j += blockDim.x) {
      const float a = __fmul_rn(s_a, wscale[j]);
      ab[(size_t)n * 2 * Cout + j] = a;
      ab[(size_t)n * 2 * Cout + Cout + j] =
          __fsub_rn(bias ? bias[j] : 0.0f, __fmul_rn(__fmul_rn(a, 128.0f), (float)Sw[j]));
    }
}

// k_absmax_img's per-image derivation from a maximum its producer already accumulated
// (EpiParams::img_absmax, k_maxpool4, k_conv_int8_pool): the same expressions.
__global__ void k_int8_img_scalars(const unsigned* __restrict__ maxa, int N, float* inv, float* sa,
                                   int* zero) {
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    const float mx = __uint_as_float(maxa[n]);
    zero[n] = mx < 1e-12f ? 1 : 0;
    inv[n] = __fdiv_rn(127.0f, mx);
    sa[n] = __fdiv_rn(mx, 127.0f);
  }
}

bool int8_pool_ok(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  return int8_b_layout(Cin, KH, KW, stride).implicit && Cout > 64 && (H + 2 * pad) % 2 == 0 &&
         OH >= 2 && OW >= 2;
}

bool conv2d_int8_batch_dev(Call& c, const float* x, int N, int H, int W, int Cin,
                           const int8_t* wq, const float* wscale, const float* bias, int KH,
                           int KW, int Cout, int stride, int pad, float* out, int act,
                           const unsigned* in_max, unsigned* out_max, bool pool) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0 || N <= 0) return true;
  if (N > 65535) {
    set_error(kInvalid, "%s: at most 65535 images per int8 batch call", c.name());
    c.fail();
    return false;
  }
  const Int8BLayout lay = int8_b_layout(Cin, KH, KW, stride);
  unsigned* words = (unsigned*)c.scratch((size_t)N * 2 * 4);  // maxa[N], done[N]
  float* inv = (float*)c.scratch((size_t)N * 4);
  float* sa = (float*)c.scratch((size_t)N * 4);
  int* zero = (int*)c.scratch((size_t)N * 4);
  int* Sw = (int*)c.scratch((size_t)Cout * 4);
  int8_t* wk = (int8_t*)c.scratch((size_t)Cout * lay.taps * lay.cpad);
  if (!words || !inv || !sa || !zero || !Sw || !wk) return false;
  k_int8_wprep<<<Cout, 128, 0, c.stream()>>>(wq, lay.taps, lay.cin, Cout, lay.cpad, wk, Sw, words,
                                              2 * N);
  if (in_max) {
    k_int8_img_scalars<<<(N + 127) / 128, 128, 0, c.stream()>>>(in_max, N, inv, sa, zero);
  } else {
    const long long per = (long long)H * W * Cin;
    long long bx = per / (4 * 256 * 4);
    bx = bx < 1 ? 1 : (bx > 64 ? 64 : bx);
    k_absmax_img<<<dim3((unsigned)bx, (unsigned)N), 256, 0, c.stream()>>>(
        x, per, words, words + N, inv, sa, zero, nullptr, nullptr, nullptr, 0, nullptr, nullptr);
  }
  if (!c.launched("int8 per-image params")) return false;
  const bool wino = is_wino_route(H, W, Cin, KH, KW, Cout, stride, pad);
  Int8ConvArgs a;
  a.xf = x;
  a.img_inv = inv;
  a.img_sa = sa;
  a.img_zero = zero;
  a.qmode = wino ? 1 : 0;
  a.epi = wino ? Epi::I8_WINO : Epi::F32_AB;
  a.f0 = wscale;
  a.f1 = bias;
  a.i0 = Sw;
  a.out_max = out_max;
  return int8_conv_gemm(c, a, N, H, W, Cin, wq, KH, KW, Cout, stride, pad, out, act, wk, pool);
}

// s8 weights [taps*Cin][Cout] -> 4-byte words wpk[tap][cw][Cout] (channels 4cw..4cw+3 of a
// tap, zero past Cin) for k_conv_int8_pool, and the column sums Sw (one block per output
// channel); block 0 also clears the nclear words k_absmax_img accumulates into.
__global__ void k_int8_pool_wpack(const int8_t* __restrict__ wq, int taps, int Cin, int CW,
                                  int Cout, uint32_t* __restrict__ wpk, int* __restrict__ Sw,
                                  unsigned* __restrict__ clear, int nclear) {
  __shared__ int red[32];
  const int j = blockIdx.x;
  if (j == 0)
    for (int i = threadIdx.x; i < nclear; i += blockDim.x) clear[i] = 0u;
  int sum = 0;
  for (int r = threadIdx.x; r < taps * CW; r += blockDim.x) {
    const int tap = r / CW, cw = r - tap * CW;
    uint32_t wv = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = cw * 4 + e;
      if (c < Cin) {
        const int8_t v = wq[(size_t)(tap * Cin + c) * Cout + j];
        sum += v;
        wv |= (uint32_t)(uint8_t)v << (8 * e);
      }
    }
    wpk[(size_t)r * Cout + j] = wv;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    Sw[j] = t;
  }
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Small-K int8 convolution (non-Winograd route) fused with the 2x2 / stride-2 / pad-0 max-pool
// that follows it, for the per-image int8 model path.  A block owns one pooled row of one image:
// it quantises the input rows that row needs straight from fp32 (RNE, the image's inv_s, zero
// point 128 -- also outside the image, as the reference's u8 im2col pads) into a padded tile of
// 4-byte pixel words (channels c..c+3 of a pixel, CW words per pixel) and stages the s8 weights
// packed in matching words [tap][cw][Cout] (k_int8_pool_wpack) and this image's alpha / beta
// (k_absmax_img).  One thread per
// (16-channel block, pooled pixel) then accumulates the exact integer correlation of its four
// conv pixels with dp4a, dequantises as the F32_AB epilogue does ((float)acc*alpha then +
// beta), applies act and the pool (start -1e30, window
// order (0,0) (0,1) (1,0) (1,1)), then the pool's post-ReLU.  Integer sums do not depend on the
// order, so the output equals the unfused im2col GEMM + max-pool bit for bit.
template <int CW>
__global__ void __launch_bounds__(128) k_conv_int8_pool(
    const float* __restrict__ x, int H, int W, int Cin, const uint32_t* __restrict__ wpk,
    const float* __restrict__ ab, int Cout, int KH, int KW, int stride, int pad, int PH, int PW,
    const float* __restrict__ img_inv, const int* __restrict__ img_zero, float* __restrict__ out,
    int act, int post_relu, unsigned* __restrict__ out_max) {
  extern __shared__ uint4 ip_sm4[];
  __shared__ float am_red[4];
  float am = 0.0f;  // max |stored value| of this block (one image): out_max
  const int taps = KH * KW;
  const int Wp = W + 2 * pad, ROWS = stride + KH;
  uint32_t* wsm = reinterpret_cast<uint32_t*>(ip_sm4);  // [taps][CW][Cout]
  float* alpha = reinterpret_cast<float*>(wsm + taps * CW * Cout);
  float* beta = alpha + Cout;
  uint32_t* tile = reinterpret_cast<uint32_t*>(beta + Cout);  // [ROWS][Wp][CW]
  const int n = blockIdx.x / PH, ph = blockIdx.x - n * PH;
  const float inv_s = img_inv[n];
  const bool zero = img_zero[n] != 0;
  // packed weights and this image's alpha / beta: all of a thread's loads before its stores
  {
    constexpr int U = 8;
    const int nw = taps * CW * Cout, na = 2 * Cout;
    const float* abn = ab + (size_t)n * 2 * Cout;
    for (int b0 = threadIdx.x; b0 < nw + na; b0 += U * blockDim.x) {
      uint32_t v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        v[u] = 0u;
        if (i < nw) v[u] = __ldg(wpk + i);
        else if (i < nw + na) v[u] = __float_as_uint(__ldg(abn + (i - nw)));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        if (i < nw + na) wsm[i] = v[u];  // alpha / beta follow the weights in smem
      }
    }
  }
  const int r0 = 2 * ph * stride - pad;  // input row of tile row 0
  const float* img = x + (size_t)n * H * W * Cin;
  {
    constexpr int U = 4;
    const int nt = ROWS * Wp * CW;
    for (int b0 = threadIdx.x; b0 < nt; b0 += U * blockDim.x) {
      float v[U][4];
      bool in[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        const int cw = i % CW, rc = i / CW, pc = rc % Wp, tr = rc / Wp;
        const int ih = r0 + tr, iw = pc - pad;
        in[u] = i < nt && ih >= 0 && ih < H && iw >= 0 && iw < W;
        const float* src = in[u] ? img + ((size_t)ih * W + iw) * Cin : img;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = cw * 4 + e;
          v[u][e] = (in[u] && c < Cin) ? __ldg(src + c) : 0.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        if (i >= nt) continue;
        const int cw = i % CW;
        uint32_t wv = 0x80808080u;
        if (in[u]) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t q = (cw * 4 + e < Cin) ? quant_fast<0>(v[u][e], inv_s) : 128u;
            wv = (wv & ~(0xFFu << (8 * e))) | (q << (8 * e));
          }
        }
        tile[i] = wv;
      }
    }
  }
  __syncthreads();
  const int nb = Cout / 16, items = PW * nb;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int cb = it / PW, pw = it - cb * PW;
    int acc[4][16];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[p][j] = 0;
    for (int kh = 0; kh < KH; ++kh)
      for (int kw = 0; kw < KW; ++kw)
#pragma unroll
        for (int cw = 0; cw < CW; ++cw) {
          const uint4* wr = reinterpret_cast<const uint4*>(wsm + ((kh * KW + kw) * CW + cw) * Cout + cb * 16);
          uint32_t wv[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 t = wr[q];
            wv[4 * q] = t.x; wv[4 * q + 1] = t.y; wv[4 * q + 2] = t.z; wv[4 * q + 3] = t.w;
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int tr = (p >> 1) * stride + kh;              // conv row 2ph + dy
            const int pc = (2 * pw + (p & 1)) * stride + kw;    // padded column
            const uint32_t xv = tile[(tr * Wp + pc) * CW + cw];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[p][j] = dp4a_us(xv, wv[j], acc[p][j]);
          }
        }
    float m[16];
    // The window maximum of the int32 sums, then one dequantisation: (float)acc*alpha + beta
    // is non-decreasing in acc (alpha = sa*ws >= 0) and so is ReLU, so this is the maximum of
    // the four dequantised values bit for bit -- except that with alpha == 0 and beta == +-0
    // the four values are zeros whose signs follow the sums' signs; such a channel (only
    // without ReLU, which maps both zeros to +0) takes the per-pixel maximum.
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float al = alpha[cb * 16 + j], be = beta[cb * 16 + j];
      float v;
      if (act || al > 0.0f || be != 0.0f) {
        const int a = max(max(acc[0][j], acc[1][j]), max(acc[2][j], acc[3][j]));
        v = __fadd_rn(__fmul_rn(__int2float_rn(a), al), be);
        if (act) v = v > 0.0f ? v : 0.0f;
      } else {
        v = -1e30f;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float u = __fadd_rn(__fmul_rn(__int2float_rn(acc[p][j]), al), be);
          v = v > u ? v : u;
        }
      }
      m[j] = zero ? 0.0f : v;
    }
    float* dst = out + (((size_t)n * PH + ph) * PW + pw) * Cout + cb * 16;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 r = make_float4(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3]);
      if (post_relu) {
        r.x = r.x > 0.f ? r.x : 0.f; r.y = r.y > 0.f ? r.y : 0.f;
        r.z = r.z > 0.f ? r.z : 0.f; r.w = r.w > 0.f ? r.w : 0.f;
      }
      reinterpret_cast<float4*>(dst)[q] = r;
      amax_acc(am, r.x);
      amax_acc(am, r.y);
      amax_acc(am, r.z);
      amax_acc(am, r.w);
    }
  }
  if (out_max) {  // block-uniform
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, am, o);
      am = (am < u) ? u : am;
    }
    if ((threadIdx.x & 31) == 0) am_red[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) am = (am < am_red[w]) ? am_red[w] : am;
      if (am > 0.0f) atomicMax(&out_max[n], __float_as_uint(am));
    }
  }
}


bool conv_int8_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                        const float* wscale, const float* bias, int KH, int KW, int Cout,
                        int stride, int pad, int act, int pool, int pst, int ppd, int post_relu,
                        float* out, bool* handled, unsigned* out_max, const unsigned* in_max) {
  *handled = false;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (pool != 2 || pst != 2 || ppd != 0 || OH < 2 || OW < 2 || N <= 0 || N > 65535) return true;
  // the Winograd route quantises half-away and dequantises differently: not fused here
  if (is_wino_route(H, W, Cin, KH, KW, Cout, stride, pad)) return true;
  const int taps = KH * KW, K = taps * Cin, CW = (Cin + 3) / 4;
  if (K > 64 || Cin > 16 || Cout % 16 != 0 || Cout > 64 || !aligned16(out)) return true;
  const int PH = (OH - 2) / 2 + 1, PW = (OW - 2) / 2 + 1;
  const long long Wp = (long long)W + 2 * pad, ROWS = stride + KH;
  const long long smem = ((long long)taps * CW * Cout + 2LL * Cout + ROWS * Wp * CW) * 4;
  if (smem > 48 * 1024 || (long long)N * PH >= (1LL << 31)) return true;
  unsigned* words = (unsigned*)c.scratch((size_t)N * 2 * 4);  // maxa[N], done[N]
  float* inv = (float*)c.scratch((size_t)N * 4);
  float* sa = (float*)c.scratch((size_t)N * 4);
  int* zero = (int*)c.scratch((size_t)N * 4);
  int* Sw = (int*)c.scratch((size_t)Cout * 4);
  uint32_t* wpk = (uint32_t*)c.scratch((size_t)taps * CW * Cout * 4);
  float* ab = (float*)c.scratch((size_t)N * 2 * Cout * 4);
  if (!words || !inv || !sa || !zero || !Sw || !wpk || !ab) return false;
  k_int8_pool_wpack<<<Cout, 64, 0, c.stream()>>>(wq, taps, Cin, CW, Cout, wpk, Sw, words, 2 * N);
  // the per-image maximum: measured from x, or given (in_max) without reading x
  const long long per = in_max ? 0 : (long long)H * W * Cin;
  long long bx = per / (4 * 256 * 4);
  bx = bx < 1 ? 1 : (bx > 64 ? 64 : bx);
  k_absmax_img<<<dim3((unsigned)bx, (unsigned)N), 256, 0, c.stream()>>>(
      x, per, words, words + N, inv, sa, zero, wscale, bias, Sw, Cout, ab, in_max);
  if (conv_i8_pool_tc_ok(x, W, Cin, KH, KW, Cout, stride, PW)) {
    *handled = true;
    if (!c.launched("int8 pool params")) return false;
    return conv_i8_pool_tc_dev(c, x, N, H, W, Cin, wq, KH, KW, Cout, pad, PH, PW, ab, inv, zero, out,
                               act, post_relu, out_max);
  }
#define ACF_I8POOL(CWV)                                                                        \
  k_conv_int8_pool<CWV><<<N * PH, 128, (size_t)smem, c.stream()>>>(                            \
      x, H, W, Cin, wpk, ab, Cout, KH, KW, stride, pad, PH, PW, inv, zero, out, act, post_relu,  \
      out_max)
  if (CW == 1)
    ACF_I8POOL(1);
  else if (CW == 2)
    ACF_I8POOL(2);
  else if (CW == 3)
    ACF_I8POOL(3);
  else
    ACF_I8POOL(4);
#undef ACF_I8POOL
  *handled = true;
  return c.launched("k_conv_int8_pool");
}

}  // namespace acf

using namespace acf;

// conv_int8.cpp:24-37 — host-side: exact IEEE division + lroundf, like the reference.
extern "C" void acfun_quantize_weights(const float* w, int K, int N, float* scales, int8_t* wq) {
  if (!w || !scales || !wq || K <= 0 || N <= 0) return;
  // device pointers are accepted too: stage through host memory
  const bool dev_in = ptr_kind(w) == PtrKind::Device;
  const bool dev_s = ptr_kind(scales) == PtrKind::Device;
  const bool dev_q = ptr_kind(wq) == PtrKind::Device;
  std::vector<float> hw, hs;
  std::vector<int8_t> hq;
  const float* W = w;
  float* S = scales;
  int8_t* Q = wq;
  if (dev_in) {
    hw.resize((size_t)K * N);
    if (!ACF_CUDA_OK(cudaMemcpy(hw.data(), w, hw.size() * 4, cudaMemcpyDeviceToHost))) return;
    W = hw.data();
  }
  if (dev_s) {
    hs.resize(N);
    S = hs.data();
  }
  if (dev_q) {
    hq.resize((size_t)K * N);
    Q = hq.data();
  }
  for (int j = 0; j < N; ++j) {
    float maxa = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float v = fabsf(W[(size_t)k * N + j]);
      maxa = (maxa < v) ? v : maxa;
    }
    float s = maxa / 127.0f;
    if (s <= 0.0f) s = 1.0f;
    S[j] = s;
    for (int k = 0; k < K; ++k) {
      int v = (int)lroundf(W[(size_t)k * N + j] / s);
      if (v > 127) v = 127;
      else if (v < -128) v = -128;
      Q[(size_t)k * N + j] = (int8_t)v;
    }
  }
  if (dev_s) ACF_CUDA_OK(cudaMemcpy(scales, hs.data(), (size_t)N * 4, cudaMemcpyHostToDevice));
  if (dev_q) ACF_CUDA_OK(cudaMemcpy(wq, hq.data(), (size_t)K * N, cudaMemcpyHostToDevice));
}

extern "C" void acfun_conv2d_int8(const float* input, int N, int H, int W, int Cin,
                                  const int8_t* wq, const float* wscale, const float* bias, int KH,
                                  int KW, int Cout, int stride, int pad, float s_in, float* output,
                                  int act) {
  (void)s_in;  // ignored, as in the reference (conv_int8.cpp:63-81)
  if (!input || !wq || !wscale || !output || N <= 0 || Cin <= 0 || Cout <= 0 || KH <= 0 ||
      KW <= 0 || stride <= 0)
    return;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return;
  Call c("acfun_conv2d_int8");
  if (!c.ok()) return;
  const float* dx = (const float*)c.in(input, (size_t)N * H * W * Cin * 4);
  const int8_t* dw = (const int8_t*)c.in(wq, (size_t)KH * KW * Cin * Cout);
  const float* ds = (const float*)c.in(wscale, (size_t)Cout * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * OH * OW * Cout * 4);
  if (!c.ok()) return;
  conv2d_int8_dev(c, dx, N, H, W, Cin, dw, ds, db, KH, KW, Cout, stride, pad, dout, act);
  c.finish();
}

// internal.h:164 — pre-quantised u8 input, caller-supplied alpha / beta
extern "C" void acfun_conv2d_int8_direct(const uint8_t* inQ, int N, int H, int W, int Cin,
                                         const int8_t* wq, const float* alpha, const float* beta,
                                         int KH, int KW, int Cout, int stride, int pad, int OH,
                                         int OW, float* output, int act) {
  if (!inQ || !wq || !alpha || !beta || !output || N <= 0 || Cin <= 0 || Cout <= 0 || KH <= 0 ||
      KW <= 0 || stride <= 0 || OH <= 0 || OW <= 0)
    return;
  if (OH != (H + 2 * pad - KH) / stride + 1 || OW != (W + 2 * pad - KW) / stride + 1) {
    set_error(kInvalid, "acfun_conv2d_int8_direct: OH/OW do not match the geometry");
    return;
  }
  Call c("acfun_conv2d_int8_direct");
  if (!c.ok()) return;
  const uint8_t* dx = (const uint8_t*)c.in(inQ, (size_t)N * H * W * Cin);
  const int8_t* dw = (const int8_t*)c.in(wq, (size_t)KH * KW * Cin * Cout);
  const float* da = (const float*)c.in(alpha, (size_t)Cout * 4);
  const float* db = (const float*)c.in(beta, (size_t)Cout * 4);
  float* dout = (float*)c.out(output, (size_t)N * OH * OW * Cout * 4);
  if (!c.ok()) return;
  Int8ConvArgs a;
  a.xq = dx;
  a.epi = Epi::F32_AB;
  a.f0 = da;
  a.f1 = db;
  int8_conv_gemm(c, a, N, H, W, Cin, dw, KH, KW, Cout, stride, pad, dout, act);
  c.finish();
}

// internal.h:185 — 1x1 s1 p0 over A[M][K] = the fused int8 GEMM epilogue
extern "C" void acfun_conv1x1_int8(const uint8_t* inQ, int M, int K, int Cout, const int8_t* wq,
                                   const float* alpha, const float* beta, float* output, int act) {
  acfun_gemm_int8_epi(M, Cout, K, inQ, wq, output, alpha, beta, act);
}

// internal.h:198 — Winograd F(2,3) int8 route with caller-supplied s_in / inv_s
extern "C" void acfun_winograd_conv3x3_int8(const float* input, int N, int H, int W, int Cin,
                                            const int8_t* wq, const float* wscale,
                                            const float* bias, int Cout, float s_in, float inv_s,
                                            float* output, int act) {
  if (!input || !wq || !wscale || !output || N <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0)
    return;
  Call c("acfun_winograd_conv3x3_int8");
  if (!c.ok()) return;
  const float* dx = (const float*)c.in(input, (size_t)N * H * W * Cin * 4);
  const int8_t* dw = (const int8_t*)c.in(wq, (size_t)9 * Cin * Cout);
  const float* ds = (const float*)c.in(wscale, (size_t)Cout * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * H * W * Cout * 4);
  float* wso = (float*)c.scratch((size_t)Cout * 4);
  int* Sw = (int*)c.scratch((size_t)Cout * 4);
  if (!c.ok()) return;
  k_int8_colparams<<<(Cout * 32 + 255) / 256, 256, 0, c.stream()>>>(
      dw, 9 * Cin, Cout, ds, db, s_in, nullptr, nullptr, wso, Sw);
  if (!c.launched("int8 params")) return;
  Int8ConvArgs a;
  a.xf = dx;
  a.qmode = 1;
  a.inv_host = inv_s;
  a.epi = Epi::I8_WINO;
  a.f0 = wso;
  a.f1 = db;
  a.i0 = Sw;
  int8_conv_gemm(c, a, N, H, W, Cin, dw, 3, 3, Cout, 1, 1, dout, act);
  c.finish();
}
