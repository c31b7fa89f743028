// ops.cu — bandwidth-bound NHWC kernels: ReLU / ReLU6, max-pool (+ReLU), softmax,
// batch-norm, u8 activation quantisation, depthwise and grouped direct convolution.
//
// Each kernel reproduces the rounding sequence of the reference's routed AVX path so that
// results are bit-identical where the reference is deterministic:
//   depthwise   acc = bias; acc = fma(x_or_0, w, acc) over kh, kw   (dw_avx512.cpp:99-124)
//   grouped     acc = bias; acc = fma(x, w, acc) over kh, kw, ic    (group_conv_avx2.cpp:241-258)
//               (mul-then-add when Cout_per < 8: the scalar kernel, group_conv.cpp:16-55)
//   batch-norm  (x - mean) * (gamma / sqrtf(var + eps)) + beta      (layers.cpp:285-296)
//   quantize    clamp(cvt_rne(x * inv_s) + zp, 0, 255)               (int8_quantize_avx512.cpp:8-35)
//   max-pool    vector lanes: acc = acc > v ? acc : v (vmaxps);       (maxpool_avx512.cpp:15-66)
//               scalar tail lanes: if (v > mx) mx = v
#include <algorithm>
#include <float.h>

#include "api_export.cuh"
#include "conv.cuh"
#include "numerics.cuh"
#include "ops.cuh"
#include "runtime.cuh"

namespace acf {

static inline int grid_for(Call& c, long long work, int block = 256) {
  long long b = (work + block - 1) / block;
  long long cap = (long long)c.sm_count() * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

#define GRID_STRIDE(i, n)                                                               \
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (n); \
       i += (long long)gridDim.x * blockDim.x)

// ------------------------------------------------------------------ relu / relu6
__global__ void k_relu(float* d, long long n, int six) {
  GRID_STRIDE(i, n) {
    float v = d[i];
    if (v < 0.0f) v = 0.0f;
    else if (six && v > 6.0f) v = 6.0f;
    d[i] = v;
  }
}

bool relu_dev(Call& c, float* d, long long n, int six) {
  if (n <= 0) return true;
  k_relu<<<grid_for(c, n), 256, 0, c.stream()>>>(d, n, six);
  return c.launched("k_relu");
}

// ------------------------------------------------------------------ max pool
__global__ void k_maxpool(const float* __restrict__ in, int N, int H, int W, int C, int pool,
                          int stride, int pad, int OH, int OW, int cfull, float* __restrict__ out,
                          int post_relu) {
  const long long total = (long long)N * OH * OW * C;
  GRID_STRIDE(idx, total) {
    const int c = (int)(idx % C);
    long long p = idx / C;
    const int ow = (int)(p % OW);
    p /= OW;
    const int oh = (int)(p % OH);
    const int n = (int)(p / OH);
    const bool vec = c < cfull;
    float mx = -1e30f;
    for (int ph = 0; ph < pool; ++ph) {
      const int ih = oh * stride - pad + ph;
      if (ih < 0 || ih >= H) continue;
      for (int pw = 0; pw < pool; ++pw) {
        const int iw = ow * stride - pad + pw;
        if (iw < 0 || iw >= W) continue;
        const float v = in[(((long long)n * H + ih) * W + iw) * C + c];
        if (vec) mx = (mx > v) ? mx : v;
        else if (v > mx) mx = v;
      }
    }
    if (post_relu) {
      if (vec) mx = (mx > 0.0f) ? mx : 0.0f;
      else if (mx < 0.0f) mx = 0.0f;
    }
    out[idx] = mx;
  }
}

// float4 variant for whole vector-lane channel groups (C % 4 == 0, all lanes vectorised).
// out_split != NULL: the result goes, split into bf16 hi / lo, into the next convolution's
// zero-padded input planes (pixel (n, oh, ow) at ((n*sHp + oh + spad)*sWp + ow + spad)) instead
// of `out`; nx_store_split4 is the split k_pad_split4 makes, so the next layer reads the same.
__global__ void k_maxpool4(const float4* __restrict__ in, int N, int H, int W, int C4, int pool,
                           int stride, int pad, int OH, int OW, float4* __restrict__ out,
                           int post_relu, void* out_split, long long split_plane, int sHp,
                           int sWp, int spad) {
  const long long total = (long long)N * OH * OW * C4;
  GRID_STRIDE(idx, total) {
    const int c = (int)(idx % C4);
    long long p = idx / C4;
    const int ow = (int)(p % OW);
    p /= OW;
    const int oh = (int)(p % OH);
    const int n = (int)(p / OH);
    float4 m = make_float4(-1e30f, -1e30f, -1e30f, -1e30f);
    for (int ph = 0; ph < pool; ++ph) {
      const int ih = oh * stride - pad + ph;
      if (ih < 0 || ih >= H) continue;
      for (int pw = 0; pw < pool; ++pw) {
        const int iw = ow * stride - pad + pw;
        if (iw < 0 || iw >= W) continue;
        const float4 v = in[(((long long)n * H + ih) * W + iw) * C4 + c];
        m.x = m.x > v.x ? m.x : v.x;
        m.y = m.y > v.y ? m.y : v.y;
        m.z = m.z > v.z ? m.z : v.z;
        m.w = m.w > v.w ? m.w : v.w;
      }
    }
    if (post_relu) {
      m.x = m.x > 0.f ? m.x : 0.f;
      m.y = m.y > 0.f ? m.y : 0.f;
      m.z = m.z > 0.f ? m.z : 0.f;
      m.w = m.w > 0.f ? m.w : 0.f;
    }
    if (out_split) {
      const float v[4] = {m.x, m.y, m.z, m.w};
      const size_t i4 = (((size_t)n * sHp + oh + spad) * sWp + ow + spad) * C4 + c;
      nx_store_split4<true>(out_split, i4, (size_t)split_plane, v);
    } else {
      out[idx] = m;
    }
  }
}

bool maxpool_dev(Call& c, const float* in, int N, int H, int W, int C, int pool, int stride,
                 int pad, float* out, int post_relu, const SplitAct* os) {
  const int OH = (H + 2 * pad - pool) / stride + 1, OW = (W + 2 * pad - pool) / stride + 1;
  if (OH <= 0 || OW <= 0 || N <= 0 || C <= 0) return true;
  // lanes handled by the reference's vector kernels (maxpool_impl, layers.cpp:250-258)
  const int cfull = C >= 16 ? (C & ~15) : (C >= 8 ? (C & ~7) : 0);
  if (cfull == C && C % 4 == 0 && aligned16(in) && aligned16(out)) {
    const long long total = (long long)N * OH * OW * (C / 4);
    k_maxpool4<<<grid_for(c, total), 256, 0, c.stream()>>>(
        (const float4*)in, N, H, W, C / 4, pool, stride, pad, OH, OW, (float4*)out, post_relu,
        os ? os->base : nullptr, os ? os->plane : 0, os ? os->H + 2 * os->pad : 0,
        os ? os->W + 2 * os->pad : 0, os ? os->pad : 0);
    return c.launched("k_maxpool4");
  }
  if (os) {
    set_error(kInvalid, "%s: split max-pool output needs whole 16-channel groups", c.name());
    c.fail();
    return false;
  }
  const long long total = (long long)N * OH * OW * C;
  k_maxpool<<<grid_for(c, total), 256, 0, c.stream()>>>(in, N, H, W, C, pool, stride, pad, OH,
                                                        OW, cfull, out, post_relu);
  return c.launched("k_maxpool");
}

// ------------------------------------------------------------------ softmax
__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = (threadIdx.x < nw) ? sh[threadIdx.x] : (is_max ? -FLT_MAX : 0.0f);
  if (w == 0) {
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, u) : v + u;
    }
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

// layers.cpp:272-283: one block per row; max, e = expf(x - max), sum, out = e * (1/sum).
__global__ void k_softmax(const float* __restrict__ in, int cols, float* __restrict__ out) {
  __shared__ float sh[32];
  const float* ri = in + (long long)blockIdx.x * cols;
  float* ro = out + (long long)blockIdx.x * cols;
  float m = -FLT_MAX;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) m = fmaxf(m, ri[j]);
  m = block_reduce(m, true, sh);
  float s = 0.0f;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) {
    const float e = expf(ri[j] - m);
    ro[j] = e;
    s += e;
  }
  s = block_reduce(s, false, sh);
  const float inv = 1.0f / s;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) ro[j] = ro[j] * inv;
}

bool softmax_dev(Call& c, const float* in, int rows, int cols, float* out) {
  if (rows <= 0 || cols <= 0) return true;
  k_softmax<<<rows, 256, 0, c.stream()>>>(in, cols, out);
  return c.launched("k_softmax");
}

// ------------------------------------------------------------------ batch norm
__global__ void k_batchnorm(float* d, long long n, int channels, const float* mean,
                            const float* var, const float* gamma, const float* beta, float eps) {
  GRID_STRIDE(i, n) {
    const int c = (int)(i % channels);
    const float scale = gamma ? gamma[c] : 1.0f;
    const float shift = beta ? beta[c] : 0.0f;
    const float inv = __fdiv_rn(scale, __fsqrt_rn(__fadd_rn(var[c], eps)));
    d[i] = __fadd_rn(__fmul_rn(__fsub_rn(d[i], mean[c]), inv), shift);
  }
}

bool batchnorm_dev(Call& c, float* d, int size, int channels, const float* mean,
                   const float* var, const float* gamma, const float* beta, float eps) {
  if (channels <= 0 || size <= 0) return true;
  const long long n = (long long)(size / channels) * channels;  // the reference's `spatial` floor
  if (n <= 0) return true;
  k_batchnorm<<<grid_for(c, n), 256, 0, c.stream()>>>(d, n, channels, mean, var, gamma, beta, eps);
  return c.launched("k_batchnorm");
}

// ------------------------------------------------------------------ u8 quantisation
__device__ __forceinline__ uint8_t quant_rne(float x, float inv_s, int zp) {
  const float t = __fmul_rn(x, inv_s);
  // cvtps2dq: |t| >= 2^31 or NaN gives the integer indefinite 0x80000000
  const int q = (fabsf(t) < 2147483648.0f) ? __float2int_rn(t) : (int)0x80000000;
  const int v = (int)((unsigned)q + (unsigned)zp);
  return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
}

__global__ void k_quantize_u8(const float* __restrict__ in, uint8_t* __restrict__ out, long long n,
                              float inv_s, int zp) {
  const long long n4 = n / 4;
  GRID_STRIDE(i, n4) {
    const float4 v = reinterpret_cast<const float4*>(in)[i];
    uchar4 q;
    q.x = quant_rne(v.x, inv_s, zp);
    q.y = quant_rne(v.y, inv_s, zp);
    q.z = quant_rne(v.z, inv_s, zp);
    q.w = quant_rne(v.w, inv_s, zp);
    reinterpret_cast<uchar4*>(out)[i] = q;
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const long long i = n4 * 4 + threadIdx.x;
    out[i] = quant_rne(in[i], inv_s, zp);
  }
}

__global__ void k_quantize_u8_scalar(const float* __restrict__ in, uint8_t* __restrict__ out,
                                     long long n, float inv_s, int zp) {
  GRID_STRIDE(i, n) out[i] = quant_rne(in[i], inv_s, zp);
}

bool quantize_u8_dev(Call& c, const float* in, uint8_t* out, long long n, float inv_s, int zp) {
  if (n <= 0) return true;
  if (aligned16(in) && (reinterpret_cast<uintptr_t>(out) & 3) == 0) {
    k_quantize_u8<<<grid_for(c, n / 4 + 1), 256, 0, c.stream()>>>(in, out, n, inv_s, zp);
  } else {
    k_quantize_u8_scalar<<<grid_for(c, n), 256, 0, c.stream()>>>(in, out, n, inv_s, zp);
  }
  return c.launched("k_quantize_u8");
}

__global__ void k_fill_u32(unsigned* __restrict__ d, unsigned v, long long n) {
  GRID_STRIDE(i, n) d[i] = v;
}

bool fill_u32_dev(Call& c, unsigned* d, unsigned v, long long n) {
  if (n <= 0) return true;
  k_fill_u32<<<grid_for(c, n), 256, 0, c.stream()>>>(d, v, n);
  return c.launched("k_fill_u32");
}

// ------------------------------------------------------------------ depthwise conv
// One thread per (output pixel, 4 channels): coalesced NHWC float4 reads / writes.
__global__ void k_dw4(const float* __restrict__ in, int N, int H, int W, int C,
                      const float* __restrict__ w, const float* __restrict__ bias, int KH, int KW,
                      int stride, int pad, int OH, int OW, float* __restrict__ out, int act) {
  const int C4 = C / 4;
  const long long total = (long long)N * OH * OW * C4;
  const int K = KH * KW;
  GRID_STRIDE(idx, total) {
    const int c4 = (int)(idx % C4);
    long long p = idx / C4;
    const int ow = (int)(p % OW);
    p /= OW;
    const int oh = (int)(p % OH);
    const int n = (int)(p / OH);
    const int c = c4 * 4;
    float4 acc = bias ? *reinterpret_cast<const float4*>(bias + c) : make_float4(0, 0, 0, 0);
    const float* w0 = w + (long long)c * K;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        const int k = kh * KW + kw;
        float4 x = make_float4(0, 0, 0, 0);
        if (ih >= 0 && ih < H && iw >= 0 && iw < W)
          x = *reinterpret_cast<const float4*>(in + (((long long)n * H + ih) * W + iw) * C + c);
        acc.x = __fmaf_rn(x.x, __ldg(w0 + k), acc.x);
        acc.y = __fmaf_rn(x.y, __ldg(w0 + K + k), acc.y);
        acc.z = __fmaf_rn(x.z, __ldg(w0 + 2 * K + k), acc.z);
        acc.w = __fmaf_rn(x.w, __ldg(w0 + 3 * K + k), acc.w);
      }
    }
    if (act == 1) {
      acc.x = acc.x > 0.f ? acc.x : 0.f;
      acc.y = acc.y > 0.f ? acc.y : 0.f;
      acc.z = acc.z > 0.f ? acc.z : 0.f;
      acc.w = acc.w > 0.f ? acc.w : 0.f;
    }
    *reinterpret_cast<float4*>(out + (((long long)n * OH + oh) * OW + ow) * C + c) = acc;
  }
}

// One block per output row (n, oh): the block transposes the weights to wT[k][C] in shared
// memory once, then threads walk (ow, 4-channel group) items of the row with float4 loads.
// Same per-lane FMA chain as k_dw4 (bias, then taps in kh, kw order, zeros outside).
__global__ void k_dw_row(const float* __restrict__ in, int H, int W, int C,
                         const float* __restrict__ w, const float* __restrict__ bias, int KH,
                         int KW, int stride, int pad, int OH, int OW, float* __restrict__ out,
                         int act) {
  extern __shared__ float4 dsm4[];
  float* wT = reinterpret_cast<float*>(dsm4);
  const int K = KH * KW;
  float* bs = wT + K * C;
  for (int i = threadIdx.x; i < K * C; i += blockDim.x) {
    const int k = i / C, c = i - k * C;
    wT[i] = w[c * K + k];
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) bs[i] = bias ? bias[i] : 0.0f;
  __syncthreads();
  const int n = blockIdx.x / OH, oh = blockIdx.x - n * OH;
  const int C4 = C >> 2, items = OW * C4;
  const float* img = in + (size_t)n * H * W * C;
  float* orow = out + ((size_t)n * OH + oh) * OW * C;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int ow = it / C4, c = (it - ow * C4) * 4;
    float4 acc = *reinterpret_cast<const float4*>(bs + c);
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      const bool rok = ih >= 0 && ih < H;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rok && iw >= 0 && iw < W)
          x = __ldg(reinterpret_cast<const float4*>(img + ((size_t)ih * W + iw) * C + c));
        const float4 wv = *reinterpret_cast<const float4*>(wT + (kh * KW + kw) * C + c);
        acc.x = __fmaf_rn(x.x, wv.x, acc.x);
        acc.y = __fmaf_rn(x.y, wv.y, acc.y);
        acc.z = __fmaf_rn(x.z, wv.z, acc.z);
        acc.w = __fmaf_rn(x.w, wv.w, acc.w);
      }
    }
    if (act == 1) {
      acc.x = acc.x > 0.f ? acc.x : 0.f;
      acc.y = acc.y > 0.f ? acc.y : 0.f;
      acc.z = acc.z > 0.f ? acc.z : 0.f;
      acc.w = acc.w > 0.f ? acc.w : 0.f;
    }
    *reinterpret_cast<float4*>(orow + (size_t)ow * C + c) = acc;
  }
}

// Register-tiled depthwise: one block per output row, one thread per (strip of TW outputs
// along W, 4 channels).  For each kernel row the thread loads the (TW-1)*stride+KW input
// columns of its strip once and reuses them across the window; per output the FMA order is
// the reference's (bias, then kh outer, kw inner, zeros for taps outside the image), so the
// result is bit-identical to k_dw_row.  KW and the stride are template parameters so the
// column window stays in registers.
template <int TW, int KW, int STRIDE>
__global__ void k_dw_strip(const float* __restrict__ in, int H, int W, int C,
                           const float* __restrict__ w, const float* __restrict__ bias, int KH,
                           int pad, int OH, int OW, float* __restrict__ out, int act) {
  constexpr int NCOL = (TW - 1) * STRIDE + KW;
  constexpr int stride = STRIDE;
  extern __shared__ float4 dss4[];
  float* wT = reinterpret_cast<float*>(dss4);
  const int K = KH * KW;
  float* bs = wT + K * C;
  {
    // every thread issues its U loads before its stores: one memory round trip per U
    // elements instead of one per element
    constexpr int U = 8;
    const int tot = K * C + C;
    for (int b0 = threadIdx.x; b0 < tot; b0 += U * blockDim.x) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        v[u] = 0.0f;
        if (i < K * C) {
          const int k = i / C, c = i - k * C;
          v[u] = __ldg(w + c * K + k);
        } else if (i < tot && bias) {
          v[u] = __ldg(bias + (i - K * C));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        if (i < tot) wT[i] = v[u];  // bs follows wT
      }
    }
  }
  __syncthreads();
  const int n = blockIdx.x / OH, oh = blockIdx.x - n * OH;
  const int C4 = C >> 2, strips = (OW + TW - 1) / TW, items = strips * C4;
  const float* img = in + (size_t)n * H * W * C;
  float* orow = out + ((size_t)n * OH + oh) * OW * C;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int s = it / C4, c = (it - s * C4) * 4;
    const int ow0 = s * TW, iw0 = ow0 * stride - pad;
    float4 acc[TW];
    const float4 b4 = *reinterpret_cast<const float4*>(bs + c);
#pragma unroll
    for (int t = 0; t < TW; ++t) acc[t] = b4;
    // strips whose input columns all lie inside the image take a branch-free body
    const bool inner = iw0 >= 0 && iw0 + NCOL <= W;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      if (ih < 0 || ih >= H) continue;  // out-of-image taps are skipped, not multiplied by 0
      float4 xc[NCOL];
      unsigned ok = (1u << NCOL) - 1u;
      if (inner) {
        const float* rowp = img + ((size_t)ih * W + iw0) * C + c;
#pragma unroll
        for (int j = 0; j < NCOL; ++j)
          xc[j] = __ldg(reinterpret_cast<const float4*>(rowp + (size_t)j * C));
      } else {
        ok = 0;
#pragma unroll
        for (int j = 0; j < NCOL; ++j) {
          const int iw = iw0 + j;
          xc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (iw >= 0 && iw < W) {
            xc[j] = __ldg(reinterpret_cast<const float4*>(img + ((size_t)ih * W + iw) * C + c));
            ok |= 1u << j;
          }
        }
      }
#pragma unroll
      for (int kw = 0; kw < KW; ++kw) {
        const float4 wv = *reinterpret_cast<const float4*>(wT + (kh * KW + kw) * C + c);
#pragma unroll
        for (int t = 0; t < TW; ++t) {
          if (!inner && !((ok >> (t * STRIDE + kw)) & 1u)) continue;
          const float4 x = xc[t * STRIDE + kw];
          // two packed fmas (lanes x,y and z,w): bit-identical to four __fmaf_rn
          const float2 lo = nx_ffma2(make_float2(x.x, x.y), make_float2(wv.x, wv.y),
                                     make_float2(acc[t].x, acc[t].y));
          const float2 hi = nx_ffma2(make_float2(x.z, x.w), make_float2(wv.z, wv.w),
                                     make_float2(acc[t].z, acc[t].w));
          acc[t] = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TW; ++t) {
      if (ow0 + t >= OW) break;
      float4 a = acc[t];
      if (act == 1) {
        a.x = a.x > 0.f ? a.x : 0.f;
        a.y = a.y > 0.f ? a.y : 0.f;
        a.z = a.z > 0.f ? a.z : 0.f;
        a.w = a.w > 0.f ? a.w : 0.f;
      }
      *reinterpret_cast<float4*>(orow + (size_t)(ow0 + t) * C + c) = a;
    }
  }
}

// 3x3 stride-1 depthwise, rolling window: a thread owns 4 channels of a strip of 4 output
// columns over TH consecutive output rows and reads each input row of that range once (6 float4
// columns), folding it into the three output rows it feeds -- kh = 0 of the newest row, 1 of the
// previous, 2 of the oldest, which is then complete and stored.  Rows are visited in order, so
// every output still gets bias, then kh = 0, 1, 2 (kw = 0, 1, 2 within each), one fma per
// in-image tap: k_dw_strip's arithmetic.  The 9 weights and the bias of the 4 channels stay in
// registers; the next input row is loaded while the current one is folded in.
template <int TH>
__global__ void __launch_bounds__(384, 1) k_dw3_roll(const float* __restrict__ in, int N, int H,
                                                     int W, int C, const float* __restrict__ w,
                                                     const float* __restrict__ bias, int pad, int OH,
                                                     int OW, float* __restrict__ out, int act) {
  const int C4 = C >> 2, strips = (OW + 3) >> 2, segs = (OH + TH - 1) / TH;
  const long long items = (long long)N * segs * strips * C4;
  for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < items;
       it += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(it % C4) * 4;
    long long r = it / C4;
    const int st = (int)(r % strips);
    r /= strips;
    const int sg = (int)(r % segs), n = (int)(r / segs);
    const int oh0 = sg * TH, oh1 = min(oh0 + TH, OH);
    const int ow0 = st * 4, iw0 = ow0 - pad;
    unsigned cok = 0;
#pragma unroll
    for (int j = 0; j < 6; ++j)
      if (iw0 + j >= 0 && iw0 + j < W) cok |= 1u << j;
    float4 wv[9];
#pragma unroll
    for (int k = 0; k < 9; ++k)
      wv[k] = make_float4(__ldg(w + (c + 0) * 9 + k), __ldg(w + (c + 1) * 9 + k),
                          __ldg(w + (c + 2) * 9 + k), __ldg(w + (c + 3) * 9 + k));
    const float4 b4 = bias ? __ldg(reinterpret_cast<const float4*>(bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float* img = in + (size_t)n * H * W * C + c;
    float* obase = out + (size_t)n * OH * OW * C + c;
    auto load_row = [&](int ih, float4 (&xr)[6]) {
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        xr[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ih >= 0 && ih < H && ((cok >> j) & 1u))
          xr[j] = __ldg(reinterpret_cast<const float4*>(img + ((size_t)ih * W + iw0 + j) * C));
      }
    };
    // a0: output row ih + pad - 2 (gets kh = 2, then complete), a1: ih + pad - 1 (kh = 1),
    // a2: ih + pad (kh = 0, starts from the bias)
    float4 a0[4], a1[4], a2[4];
    const int ih_first = oh0 - pad, ih_last = oh1 - 1 - pad + 2;
    float4 xn[6];
    load_row(ih_first, xn);
    for (int ih = ih_first; ih <= ih_last; ++ih) {
      float4 xr[6];
#pragma unroll
      for (int j = 0; j < 6; ++j) xr[j] = xn[j];
      if (ih < ih_last) load_row(ih + 1, xn);  // in flight while this row is folded in
      const bool row_in = ih >= 0 && ih < H;
#pragma unroll
      for (int t = 0; t < 4; ++t) a2[t] = b4;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        float4* acc = kh == 0 ? a2 : (kh == 1 ? a1 : a0);
        if (!row_in) break;  // out-of-image rows contribute nothing
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          const float4 wk = wv[kh * 3 + kw];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (!((cok >> (t + kw)) & 1u)) continue;
            const float4 x = xr[t + kw];
            const float2 lo = nx_ffma2(make_float2(x.x, x.y), make_float2(wk.x, wk.y),
                                       make_float2(acc[t].x, acc[t].y));
            const float2 hi = nx_ffma2(make_float2(x.z, x.w), make_float2(wk.z, wk.w),
                                       make_float2(acc[t].z, acc[t].w));
            acc[t] = make_float4(lo.x, lo.y, hi.x, hi.y);
          }
        }
      }
      const int od = ih + pad - 2;  // complete output row
      if (od >= oh0 && od < oh1) {
        float* orow = obase + (size_t)od * OW * C;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (ow0 + t >= OW) break;
          float4 v = a0[t];
          if (act == 1) {
            v.x = v.x > 0.f ? v.x : 0.f;
            v.y = v.y > 0.f ? v.y : 0.f;
            v.z = v.z > 0.f ? v.z : 0.f;
            v.w = v.w > 0.f ? v.w : 0.f;
          }
          *reinterpret_cast<float4*>(orow + (size_t)(ow0 + t) * C) = v;
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        a0[t] = a1[t];
        a1[t] = a2[t];
      }
    }
  }
}

__global__ void k_dw1(const float* __restrict__ in, int N, int H, int W, int C,
                      const float* __restrict__ w, const float* __restrict__ bias, int KH, int KW,
                      int stride, int pad, int OH, int OW, float* __restrict__ out, int act) {
  const long long total = (long long)N * OH * OW * C;
  const int K = KH * KW;
  GRID_STRIDE(idx, total) {
    const int c = (int)(idx % C);
    long long p = idx / C;
    const int ow = (int)(p % OW);
    p /= OW;
    const int oh = (int)(p % OH);
    const int n = (int)(p / OH);
    float acc = bias ? bias[c] : 0.0f;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        float x = 0.0f;
        if (ih >= 0 && ih < H && iw >= 0 && iw < W) x = in[(((long long)n * H + ih) * W + iw) * C + c];
        acc = __fmaf_rn(x, w[(long long)c * K + kh * KW + kw], acc);
      }
    }
    if (act == 1) acc = acc > 0.f ? acc : 0.f;
    out[idx] = acc;
  }
}

bool dw_dev(Call& c, const float* in, int N, int H, int W, int C, const float* w,
            const float* bias, int KH, int KW, int stride, int pad, float* out, int act) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0 || N <= 0 || C <= 0) return true;
  const size_t smem = ((size_t)KH * KW * C + C) * 4;
  const bool rowk = C % 4 == 0 && aligned16(in) && aligned16(out) && smem <= 48 * 1024 &&
                    (long long)N * OH < (1LL << 31) && (long long)H * W * C < (1LL << 31);
  static const bool dw_tma_on = [] {
    const char* e = getenv("ACFUN_DW_TMA");
    return !(e && !strcmp(e, "0"));
  }();
  if (dw_tma_on && dw3_tma_ok(in, out, bias, N, H, W, C, KH, KW, stride, pad, c.sm_count()))
    return dw3_tma_dev(c, in, N, H, W, C, w, bias, out, act);
  if (rowk && KH == 3 && KW == 3 && stride == 1 && (!bias || aligned16(bias))) {
    // rows per item: 8 for tall maps (1.25 row reads per output row), fewer for short ones
    const long long per8 = (long long)N * ((OH + 7) / 8) * ((OW + 3) / 4) * (C / 4);
    const long long cap = 384LL * c.sm_count();
    const int grid = (int)std::min<long long>((per8 + 383) / 384, (long long)c.sm_count());
    if (OH >= 16) {
      k_dw3_roll<8><<<grid, 384, 0, c.stream()>>>(in, N, H, W, C, w, bias, pad, OH, OW, out, act);
    } else {
      const long long per4 = (long long)N * ((OH + 3) / 4) * ((OW + 3) / 4) * (C / 4);
      k_dw3_roll<4><<<(int)std::min<long long>((per4 + 383) / 384, cap / 384), 384, 0, c.stream()>>>(
          in, N, H, W, C, w, bias, pad, OH, OW, out, act);
    }
    return c.launched("k_dw3_roll");
  }
  if (rowk && KW == 3 && (stride == 1 || stride == 2)) {
    if (stride == 1)
      k_dw_strip<4, 3, 1><<<N * OH, 256, smem, c.stream()>>>(in, H, W, C, w, bias, KH, pad, OH, OW,
                                                             out, act);
    else
      k_dw_strip<4, 3, 2><<<N * OH, 256, smem, c.stream()>>>(in, H, W, C, w, bias, KH, pad, OH, OW,
                                                             out, act);
    return c.launched("k_dw_strip");
  }
  if (rowk) {
    k_dw_row<<<N * OH, 256, smem, c.stream()>>>(in, H, W, C, w, bias, KH, KW, stride, pad, OH, OW,
                                                out, act);
    return c.launched("k_dw_row");
  }
  if (C % 4 == 0 && aligned16(in) && aligned16(out) && (!bias || aligned16(bias))) {
    const long long total = (long long)N * OH * OW * (C / 4);
    k_dw4<<<grid_for(c, total), 256, 0, c.stream()>>>(in, N, H, W, C, w, bias, KH, KW, stride, pad,
                                                      OH, OW, out, act);
    return c.launched("k_dw4");
  }
  const long long total = (long long)N * OH * OW * C;
  k_dw1<<<grid_for(c, total), 256, 0, c.stream()>>>(in, N, H, W, C, w, bias, KH, KW, stride, pad,
                                                    OH, OW, out, act);
  return c.launched("k_dw1");
}

// ------------------------------------------------------------------ grouped conv
__global__ void k_group(const float* __restrict__ in, int N, int H, int W, int Cin,
                        const float* __restrict__ w, const float* __restrict__ bias, int KH,
                        int KW, int Cout, int stride, int pad, int groups, int OH, int OW,
                        float* __restrict__ out, int act, int fma_chain) {
  const int Cin_p = Cin / groups, Cout_p = Cout / groups;
  const long long total = (long long)N * OH * OW * Cout;
  const long long wg_stride = (long long)Cout_p * KH * KW * Cin_p;
  GRID_STRIDE(idx, total) {
    const int oc_g = (int)(idx % Cout);
    long long p = idx / Cout;
    const int ow = (int)(p % OW);
    p /= OW;
    const int oh = (int)(p % OH);
    const int n = (int)(p / OH);
    const int g = oc_g / Cout_p, oc = oc_g - g * Cout_p;
    const float* wg = w + g * wg_stride + oc;
    float s = bias ? bias[oc_g] : 0.0f;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      if (ih < 0 || ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        if (iw < 0 || iw >= W) continue;
        const float* ip = in + (((long long)n * H + ih) * W + iw) * Cin + (long long)g * Cin_p;
        const float* wp = wg + (long long)((kh * KW + kw) * Cin_p) * Cout_p;
        for (int ic = 0; ic < Cin_p; ++ic) {
          const float x = ip[ic], wv = __ldg(wp + (long long)ic * Cout_p);
          s = fma_chain ? __fmaf_rn(x, wv, s) : __fadd_rn(s, __fmul_rn(x, wv));
        }
      }
    }
    if (act == 1) s = fma_chain ? (s > 0.f ? s : 0.f) : (s < 0.f ? 0.f : s);
    out[idx] = s;
  }
}

// Grouped conv, one block per output row (n, oh): all groups' weights (+ bias) staged in shared
// memory with the per-group stride padded so that the groups one warp touches fall in
// different banks; thread item = (ow, output channel), consecutive threads write consecutive
// channels.  Same accumulation as k_group (bias, then kh -> kw -> ic).
__global__ void k_group_row(const float* __restrict__ in, int H, int W, int Cin,
                            const float* __restrict__ w, const float* __restrict__ bias, int KH,
                            int KW, int Cout, int stride, int pad, int groups, int OH, int OW,
                            int sstride, float* __restrict__ out, int act, int fma_chain) {
  extern __shared__ float gs[];
  const int Cin_p = Cin / groups, Cout_p = Cout / groups;
  const int wg = Cout_p * KH * KW * Cin_p;
  float* bs = gs + groups * sstride;
  for (int i = threadIdx.x; i < groups * wg; i += blockDim.x) {
    const int g = i / wg, r = i - g * wg;
    gs[g * sstride + r] = w[i];
  }
  for (int i = threadIdx.x; i < Cout; i += blockDim.x) bs[i] = bias ? bias[i] : 0.0f;
  __syncthreads();
  const int n = blockIdx.x / OH, oh = blockIdx.x - n * OH;
  const float* img = in + (size_t)n * H * W * Cin;
  float* orow = out + ((size_t)n * OH + oh) * OW * Cout;
  const int items = OW * Cout;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int ow = it / Cout, oc_g = it - ow * Cout;
    const int g = oc_g / Cout_p, oc = oc_g - g * Cout_p;
    const float* wgp = gs + g * sstride + oc;
    float s = bs[oc_g];
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      if (ih < 0 || ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        if (iw < 0 || iw >= W) continue;
        const float* ip = img + ((size_t)ih * W + iw) * Cin + g * Cin_p;
        const float* wp = wgp + (kh * KW + kw) * Cin_p * Cout_p;
        for (int ic = 0; ic < Cin_p; ++ic) {
          const float x = __ldg(ip + ic), wv = wp[ic * Cout_p];
          s = fma_chain ? __fmaf_rn(x, wv, s) : __fadd_rn(s, __fmul_rn(x, wv));
        }
      }
    }
    if (act == 1) s = fma_chain ? (s > 0.f ? s : 0.f) : (s < 0.f ? 0.f : s);
    orow[it] = s;
  }
}

// Grouped conv, one thread per (output pixel, group) computing all COUT_P channels of the group.
// A block owns R consecutive output rows of one image: it first stages, with one cooperative
// load, the group weights ([tap][ic][COUT_P] per group, per-group stride = 4 (mod 32) floats so
// a warp's groups read float4s from distinct banks) and the input rows those outputs touch;
// the accumulation then reads shared memory only.  Per-output arithmetic as k_group: bias, then
// kh -> kw -> ic over in-image taps, fma chain for COUT_P >= 8, mul+add below.
template <int COUT_P, int CIN_P>  // CIN_P = Cin/groups when known at compile time, else 0
__global__ void __launch_bounds__(256) k_group_tile(const float* __restrict__ in, int H, int W,
                                                    int Cin, const float* __restrict__ w,
                                                    const float* __restrict__ bias, int KH, int KW,
                                                    int stride, int pad, int groups, int OH, int OW,
                                                    int R, int sstride, float* __restrict__ out,
                                                    int act) {
  static_assert(COUT_P % 4 == 0, "float4 weight rows");
  extern __shared__ float4 gs4[];
  float* gs = reinterpret_cast<float*>(gs4);
  const int Cin_p = CIN_P > 0 ? CIN_P : Cin / groups, Cout = groups * COUT_P;
  const int wg = COUT_P * KH * KW * Cin_p;
  float* bs = gs + groups * sstride;
  float* tile = bs + ((Cout + 3) & ~3);
  const int blocks_per_img = (OH + R - 1) / R;
  const int n = blockIdx.x / blocks_per_img, oh0 = (blockIdx.x - n * blocks_per_img) * R;
  const int oh1 = min(OH, oh0 + R);
  const int ih0 = max(0, oh0 * stride - pad), ih1 = min(H, (oh1 - 1) * stride - pad + KH);
  // staging: every thread issues all of its 16-byte loads before its first shared store, so
  // the block waits for one memory round trip instead of one per loop iteration
  constexpr int U = 4;
  const int wg4 = wg / 4, w_tot4 = groups * wg4;  // wg and sstride are multiples of 4
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int base = threadIdx.x; base < w_tot4; base += U * blockDim.x) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < w_tot4) v[u] = __ldg(w4 + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < w_tot4) {
        const int g = i / wg4;
        gs4[g * (sstride / 4) + (i - g * wg4)] = v[u];
      }
    }
  }
  for (int i = threadIdx.x; i < Cout; i += blockDim.x) bs[i] = bias ? bias[i] : 0.0f;
  const int tile_4 = (ih1 - ih0) * W * Cin / 4;  // W * Cin is a multiple of 4
  const float4* src4 = reinterpret_cast<const float4*>(in + ((size_t)n * H + ih0) * W * Cin);
  float4* tile4 = reinterpret_cast<float4*>(tile);
  for (int base = threadIdx.x; base < tile_4; base += U * blockDim.x) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < tile_4) v[u] = __ldg(src4 + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < tile_4) tile4[i] = v[u];
    }
  }
  __syncthreads();
  const int items = (oh1 - oh0) * OW * groups;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int g = it % groups;
    const int p = it / groups;
    const int oh = oh0 + p / OW, ow = p % OW;
    float acc[COUT_P];
#pragma unroll
    for (int oc = 0; oc < COUT_P; ++oc) acc[oc] = bs[g * COUT_P + oc];
    const float* wgp = gs + g * sstride;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * stride - pad + kh;
      if (ih < 0 || ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * stride - pad + kw;
        if (iw < 0 || iw >= W) continue;
        const float* ip = tile + ((ih - ih0) * W + iw) * Cin + g * Cin_p;
        const float4* wp = reinterpret_cast<const float4*>(wgp + (kh * KW + kw) * Cin_p * COUT_P);
        float xs[CIN_P > 0 ? CIN_P : 1];
        if constexpr (CIN_P % 4 == 0 && CIN_P > 0) {
#pragma unroll
          for (int i = 0; i < CIN_P; i += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(ip + i);
            xs[i] = q4.x; xs[i + 1] = q4.y; xs[i + 2] = q4.z; xs[i + 3] = q4.w;
          }
        }
#pragma unroll
        for (int ic = 0; ic < (CIN_P > 0 ? CIN_P : Cin_p); ++ic) {
          float x;
          if constexpr (CIN_P % 4 == 0 && CIN_P > 0)
            x = xs[ic];
          else
            x = ip[ic];
#pragma unroll
          for (int q = 0; q < COUT_P / 4; ++q) {
            const float4 wv = wp[ic * (COUT_P / 4) + q];
            if constexpr (COUT_P >= 8) {
              acc[4 * q] = __fmaf_rn(x, wv.x, acc[4 * q]);
              acc[4 * q + 1] = __fmaf_rn(x, wv.y, acc[4 * q + 1]);
              acc[4 * q + 2] = __fmaf_rn(x, wv.z, acc[4 * q + 2]);
              acc[4 * q + 3] = __fmaf_rn(x, wv.w, acc[4 * q + 3]);
            } else {
              acc[4 * q] = __fadd_rn(acc[4 * q], __fmul_rn(x, wv.x));
              acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __fmul_rn(x, wv.y));
              acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __fmul_rn(x, wv.z));
              acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __fmul_rn(x, wv.w));
            }
          }
        }
      }
    }
    float* op = out + (((size_t)n * OH + oh) * OW + ow) * Cout + g * COUT_P;
#pragma unroll
    for (int q = 0; q < COUT_P / 4; ++q) {
      float4 v = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      if (act == 1) {
        if constexpr (COUT_P >= 8) {
          v.x = v.x > 0.f ? v.x : 0.f; v.y = v.y > 0.f ? v.y : 0.f;
          v.z = v.z > 0.f ? v.z : 0.f; v.w = v.w > 0.f ? v.w : 0.f;
        } else {
          v.x = v.x < 0.f ? 0.f : v.x; v.y = v.y < 0.f ? 0.f : v.y;
          v.z = v.z < 0.f ? 0.f : v.z; v.w = v.w < 0.f ? 0.f : v.w;
        }
      }
      reinterpret_cast<float4*>(op)[q] = v;
    }
  }
}

bool group_dev(Call& c, const float* in, int N, int H, int W, int Cin, const float* w,
               const float* bias, int KH, int KW, int Cout, int stride, int pad, int groups,
               float* out, int act) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0 || N <= 0) return true;
  const int Cout_p = Cout / groups;
  const long long total = (long long)N * OH * OW * Cout;
  const long long wg = (long long)Cout_p * KH * KW * (Cin / groups);
  // pad the per-group stride to Cout_p (mod 32) so a warp's groups hit different banks
  const long long sstride = Cout_p < 32 ? wg + (((Cout_p - wg % 32) % 32) + 32) % 32 : wg;
  const long long smem = (groups * sstride + Cout) * 4;
  // k_group_tile: R output rows per block (about 256 items), weights + input rows in smem
  const long long sstride4 = wg + (((4 - wg % 32) % 32) + 32) % 32;  // = 4 (mod 32)
  const long long per_row = (long long)OW * groups;
  const int R = (int)(per_row >= 256 ? 1 : (256 / per_row < OH ? 256 / per_row : OH));
  const long long rows_in = std::min<long long>(H, (long long)(R - 1) * stride + KH);
  const long long smem_t = (groups * sstride4 + ((Cout + 3) & ~3) + rows_in * W * Cin) * 4;
  if ((Cout_p == 4 || Cout_p == 8 || Cout_p == 16) && smem_t <= 48 * 1024 && aligned16(in) &&
      aligned16(w) && (W * Cin) % 4 == 0 &&
      (long long)N * ((OH + R - 1) / R) < (1LL << 31) && (long long)N * H * W * Cin < (1LL << 31) &&
      aligned16(out)) {
    const int grid = N * ((OH + R - 1) / R);
#define ACF_GROUP_TILE(CP, CI)                                                               \
  k_group_tile<CP, CI><<<grid, 256, (size_t)smem_t, c.stream()>>>(                           \
      in, H, W, Cin, w, bias, KH, KW, stride, pad, groups, OH, OW, R, (int)sstride4, out, act)
    // Cin/groups = 4 (with 16-byte aligned group slices) gets a compile-time channel loop
    const bool ci4 = Cin / groups == 4;
    if (Cout_p == 4) {
      if (ci4) ACF_GROUP_TILE(4, 4); else ACF_GROUP_TILE(4, 0);
    } else if (Cout_p == 8) {
      if (ci4) ACF_GROUP_TILE(8, 4); else ACF_GROUP_TILE(8, 0);
    } else {
      if (ci4) ACF_GROUP_TILE(16, 4); else ACF_GROUP_TILE(16, 0);
    }
#undef ACF_GROUP_TILE
    return c.launched("k_group_tile");
  }
  if (smem <= 48 * 1024 && (long long)H * W * Cin < (1LL << 31) && (long long)N * OH < (1LL << 31) &&
      (long long)OW * Cout < (1LL << 31)) {
    k_group_row<<<N * OH, 256, (size_t)smem, c.stream()>>>(
        in, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, groups, OH, OW, (int)sstride, out, act,
        Cout_p >= 8 ? 1 : 0);
    return c.launched("k_group_row");
  }
  k_group<<<grid_for(c, total), 256, 0, c.stream()>>>(in, N, H, W, Cin, w, bias, KH, KW, Cout,
                                                      stride, pad, groups, OH, OW, out, act,
                                                      Cout_p >= 8 ? 1 : 0);
  return c.launched("k_group");
}

}  // namespace acf

using namespace acf;

// ============================================================== C API wrappers
static void relu_api(const char* name, float* d, size_t len, int six) {
  if (!d || len == 0) return;
  Call c(name);
  if (!c.ok()) return;
  float* dd = (float*)c.inout(d, len * 4);
  if (!c.ok()) return;
  relu_dev(c, dd, (long long)len, six);
  c.finish();
}
extern "C" void acfun_relu(float* data, size_t len) { relu_api("acfun_relu", data, len, 0); }
extern "C" void acfun_relu6(float* data, size_t len) { relu_api("acfun_relu6", data, len, 1); }

static void maxpool_api(const char* name, const float* in, int N, int H, int W, int C, int pool,
                        int stride, int pad, float* out, int post) {
  if (N <= 0 || C <= 0 || pool <= 0 || stride <= 0 || !in || !out) return;
  const int OH = (H + 2 * pad - pool) / stride + 1, OW = (W + 2 * pad - pool) / stride + 1;
  if (OH <= 0 || OW <= 0) return;
  Call c(name);
  if (!c.ok()) return;
  const float* di = (const float*)c.in(in, (size_t)N * H * W * C * 4);
  float* dout = (float*)c.out(out, (size_t)N * OH * OW * C * 4);
  if (!c.ok()) return;
  maxpool_dev(c, di, N, H, W, C, pool, stride, pad, dout, post);
  c.finish();
}
extern "C" void acfun_maxpool(const float* in, int N, int H, int W, int C, int pool, int stride,
                              int pad, float* out) {
  maxpool_api("acfun_maxpool", in, N, H, W, C, pool, stride, pad, out, 0);
}
extern "C" void acfun_maxpool_relu(const float* in, int N, int H, int W, int C, int pool,
                                   int stride, int pad, float* out) {
  maxpool_api("acfun_maxpool_relu", in, N, H, W, C, pool, stride, pad, out, 1);
}

extern "C" void acfun_softmax(const float* in, int rows, int cols, float* out) {
  if (rows <= 0 || cols <= 0 || !in || !out) return;
  Call c("acfun_softmax");
  if (!c.ok()) return;
  const size_t bytes = (size_t)rows * cols * 4;
  const float* di;
  float* dout;
  if (in == out) {  // in-place use (model.cpp:335)
    dout = (float*)c.inout(out, bytes);
    di = dout;
  } else {
    di = (const float*)c.in(in, bytes);
    dout = (float*)c.out(out, bytes);
  }
  if (!c.ok()) return;
  softmax_dev(c, di, rows, cols, dout);
  c.finish();
}

extern "C" void acfun_batchnorm(float* d, int size, int channels, const float* mean,
                                const float* var, const float* gamma, const float* beta,
                                float eps) {
  if (!d || size <= 0 || channels <= 0 || !mean || !var) return;
  Call c("acfun_batchnorm");
  if (!c.ok()) return;
  float* dd = (float*)c.inout(d, (size_t)size * 4);
  const float* dm = (const float*)c.in(mean, (size_t)channels * 4);
  const float* dv = (const float*)c.in(var, (size_t)channels * 4);
  const float* dg = gamma ? (const float*)c.in(gamma, (size_t)channels * 4) : nullptr;
  const float* db = beta ? (const float*)c.in(beta, (size_t)channels * 4) : nullptr;
  if (!c.ok()) return;
  batchnorm_dev(c, dd, size, channels, dm, dv, dg, db, eps);
  c.finish();
}

extern "C" void acfun_quantize_u8(const float* in, uint8_t* out, size_t n, float inv_s, int zp) {
  if (!in || !out || n == 0) return;
  Call c("acfun_quantize_u8");
  if (!c.ok()) return;
  const float* di = (const float*)c.in(in, n * 4);
  uint8_t* dout = (uint8_t*)c.out(out, n);
  if (!c.ok()) return;
  quantize_u8_dev(c, di, dout, (long long)n, inv_s, zp);
  c.finish();
}

extern "C" void acfun_conv2d_dw(const float* input, int N, int H, int W, int C,
                                const float* weight, const float* bias, int KH, int KW, int stride,
                                int pad, float* output, int act) {
  if (KH <= 0 || KW <= 0 || N <= 0 || C <= 0 || stride <= 0 || !input || !weight || !output)
    return;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return;
  Call c("acfun_conv2d_dw");
  if (!c.ok()) return;
  const float* di = (const float*)c.in(input, (size_t)N * H * W * C * 4);
  const float* dw = (const float*)c.in(weight, (size_t)C * KH * KW * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)C * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * OH * OW * C * 4);
  if (!c.ok()) return;
  dw_dev(c, di, N, H, W, C, dw, db, KH, KW, stride, pad, dout, act);
  c.finish();
}

extern "C" void acfun_conv2d_grouped(const float* input, int N, int H, int W, int Cin,
                                     const float* weight, const float* bias, int KH, int KW,
                                     int Cout, int stride, int pad, int groups, float* output,
                                     int act) {
  if (groups <= 1 || KH <= 0 || KW <= 0 || N <= 0 || stride <= 0 || !input || !weight || !output)
    return;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return;
  Call c("acfun_conv2d_grouped");
  if (!c.ok()) return;
  const int Cin_p = Cin / groups, Cout_p = Cout / groups;
  const float* di = (const float*)c.in(input, (size_t)N * H * W * Cin * 4);
  const float* dw =
      (const float*)c.in(weight, (size_t)groups * Cout_p * KH * KW * Cin_p * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * OH * OW * Cout * 4);
  if (!c.ok()) return;
  group_dev(c, di, N, H, W, Cin, dw, db, KH, KW, Cout, stride, pad, groups, dout, act);
  c.finish();
}
