// conv.cu — fp32 convolution router and FC.
//
// Routing mirrors conv2d_impl (hit-droid/Acfun src/layers.cpp:106-195):
//   groups == Cin == Cout                   -> depthwise kernel           (layers.cpp:112-116)
//   groups > 1, Cin/g <= 64, Cout/g <= 128  -> grouped direct kernel      (:126-130)
//   groups > 1 otherwise                    -> per-group GEMM conv        (:134-153)
//   1x1                                     -> GEMM, zero-copy when s1 p0 (:157-160, :66-101)
//   3x3 s1 p1, H,W >= 3, Cin,Cout >= 4      -> the reference's Winograd F(4,3)/F(2,3) routes
//   otherwise                               -> im2col + GEMM               (:178-194)
// On B200 every GEMM-shaped route runs on tcgen05 tensor cores in 3xTF32 (fp32-class
// error).  Stride-1 convolutions (the Winograd routes, 1x1, any KxK) are implicit GEMMs
// over a zero-padded copy of the input: each K block is one (tap, 32-channel block), the
// TMA producer shifts the A rows by kh*Wp + kw, and the epilogue keeps only the GEMM rows
// that land on real output pixels.  Strided convolutions gather an explicit im2col matrix.
// Bias and ReLU are fused into the TMEM drain.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include "api_export.cuh"
#include "conv.cuh"
#include "gemm.cuh"
#include "numerics.cuh"
#include "ops.cuh"

namespace {
// im2col bytes per chunk of images on the tensor-core conv + pool route (kept in L2)
constexpr long long kPoolIm2colChunkBytes = 96LL << 20;
}  // namespace

namespace acf {

static int grid_ew(Call& c, long long work) {
  long long b = (work + 255) / 256, cap = (long long)c.sm_count() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// x: NHWC with channel stride Cs and channel offset coff (Cg channels used) ->
// [2][N*Hp*Wp][Cpad] split planes (hi, lo), zero in the spatial border and in channels >= Cg.
// One thread per (padded pixel, 4 channels); 32-bit index math (callers check the size).
template <bool BF>
__global__ void k_pad_split4(const float* __restrict__ x, int H, int W, int Cs, int coff, int Cg,
                             int pad, int Hp, int Wp, int C4, unsigned total, int vec_in,
                             void* __restrict__ dst, size_t op_stride) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const unsigned c4 = i % C4, p = i / C4;
    const unsigned wp = p % Wp, t = p / Wp;
    const unsigned hp = t % Hp, n = t / Hp;
    const int ih = (int)hp - pad, iw = (int)wp - pad, c = (int)c4 * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < Cg && ih >= 0 && ih < H && iw >= 0 && iw < W) {
      const float* src = x + (((size_t)n * H + ih) * W + iw) * Cs + coff + c;
      if (vec_in && c + 4 <= Cg) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(src));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = (c + k < Cg) ? src[k] : 0.f;
      }
    }
    nx_store_split4<BF>(dst, i, op_stride, v);
  }
}

// im2col for strided convs: row m = (n, oh, ow), column k = (kh*KW + kw)*Cg + c -> [2][M][Kpad]
template <bool BF>
__global__ void k_im2col_split(const float* __restrict__ x, int N, int H, int W, int Cs, int coff,
                               int Cg, int KH, int KW, int stride, int pad, int OH, int OW,
                               int Kpad, void* __restrict__ dst, long long op_stride) {
  const long long total = (long long)N * OH * OW * Kpad;
  const int K = KH * KW * Cg;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % Kpad);
    long long m = i / Kpad;
    const int ow = (int)(m % OW);
    m /= OW;
    const int oh = (int)(m % OH);
    const int n = (int)(m / OH);
    float v = 0.0f;
    if (k < K) {
      const int tap = k / Cg, c = k - tap * Cg;
      const int ih = oh * stride - pad + tap / KW, iw = ow * stride - pad + tap % KW;
      if (ih >= 0 && ih < H && iw >= 0 && iw < W)
        v = x[(((long long)n * H + ih) * W + iw) * Cs + coff + c];
    }
    nx_store_split1<BF>(dst, (size_t)i, (size_t)op_stride, v);
  }
}

// weights [taps*Cg][Cout_g] (row stride ldw) -> [2][taps*Cpad][Np], zero rows for c >= Cg
template <bool BF>
__global__ void k_weights_split(const float* __restrict__ w, int taps, int Cg, int Cout_g,
                                long long ldw, int Cpad, int Np, void* __restrict__ dst,
                                long long op_stride) {
  const long long total = (long long)taps * Cpad * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % Np);
    const long long r = i / Np;
    const int tap = (int)(r / Cpad), c = (int)(r % Cpad);
    float v = 0.0f;
    if (c < Cg && j < Cout_g) v = w[((long long)tap * Cg + c) * ldw + j];
    nx_store_split1<BF>(dst, (size_t)i, (size_t)op_stride, v);
  }
}

// Narrow convolutions on CUDA cores: Cout <= NB (64) and either a 1x1 pad-0 conv (any
// stride) or a small reduction (KH*KW*Cin <= 64, e.g. the 3-channel first layer of VGG).
// These are HBM-bound, so the activations are read once with no padded or split copy; one
// thread per output pixel keeps NB fp32 accumulators and the weights [taps*Cin][Cout] sit in
// shared memory as warp-wide broadcasts.  out = relu?(sum_taps,k x*w + bias[j]) with an fp32
// FMA chain (taps outside the image are skipped).
// S threads share a pixel, each owning NB/S of its output channels (more warps in flight for
// layers with few pixels per SM).
template <int NB, int S>
__global__ void __launch_bounds__(128) k_conv_simt(const float* __restrict__ x, int H, int W,
                                                   int Cs, int coff, int Cin,
                                                   const float* __restrict__ w, long long ldw,
                                                   const float* __restrict__ bias, int Cout, int KH,
                                                   int KW, int stride, int pad, int OH, int OW,
                                                   unsigned M, float* __restrict__ out,
                                                   long long ldc, int act, int vec_in, int vec_out) {
  extern __shared__ float4 cs_sm4[];
  float* ws = reinterpret_cast<float*>(cs_sm4);  // [taps*Cin][NB]
  const int K = KH * KW * Cin;
  float* bs = ws + K * NB;
  stage_block<16>(ws, K * NB, [&](int i) {
    const int k = i / NB, j = i - k * NB;
    return (j < Cout) ? __ldg(w + (long long)k * ldw + j) : 0.0f;
  });
  for (int j = threadIdx.x; j < NB; j += blockDim.x) bs[j] = (bias && j < Cout) ? bias[j] : 0.0f;
  __syncthreads();
  constexpr int NBT = NB / S;  // accumulators per thread
  static_assert(NBT % 4 == 0, "16-byte weight broadcasts");
  for (unsigned q = blockIdx.x * blockDim.x + threadIdx.x; q < M * S; q += gridDim.x * blockDim.x) {
    const unsigned m = q / S, g0 = (q % S) * NBT;
    const unsigned ow = m % OW, t = m / OW, oh = t % OH, n = t / OH;
    float acc[NBT];
#pragma unroll
    for (int j = 0; j < NBT; ++j) acc[j] = 0.0f;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = (int)oh * stride - pad + kh;
      if (ih < 0 || ih >= H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = (int)ow * stride - pad + kw;
        if (iw < 0 || iw >= W) continue;
        const float* src = x + (((size_t)n * H + ih) * W + iw) * Cs + coff;
        const float* wt = ws + (kh * KW + kw) * Cin * NB + g0;
        int k = 0;
        if (vec_in) {
          for (; k + 4 <= Cin; k += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + k));
            const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              // weight rows are NB (a multiple of 4) floats: 16-byte broadcasts feed two FMA2s
              const float4* wr4 = reinterpret_cast<const float4*>(wt + (k + u) * NB);
              const float2 x2 = make_float2(xv[u], xv[u]);
#pragma unroll
              for (int j = 0; j < NBT; j += 4) {
                const float4 w4 = wr4[j / 4];
                const float2 r0 = nx_ffma2(x2, make_float2(w4.x, w4.y), make_float2(acc[j], acc[j + 1]));
                const float2 r1 = nx_ffma2(x2, make_float2(w4.z, w4.w), make_float2(acc[j + 2], acc[j + 3]));
                acc[j] = r0.x;
                acc[j + 1] = r0.y;
                acc[j + 2] = r1.x;
                acc[j + 3] = r1.y;
              }
            }
          }
        }
        for (; k < Cin; ++k) {
          const float xv = src[k];
          const float* wr = wt + k * NB;
          const float2 x2 = make_float2(xv, xv);
#pragma unroll
          for (int j = 0; j < NBT; j += 2) {
            const float2 r2 = nx_ffma2(x2, make_float2(wr[j], wr[j + 1]), make_float2(acc[j], acc[j + 1]));
            acc[j] = r2.x;
            acc[j + 1] = r2.y;
          }
        }
      }
    }
    float* dst = out + (size_t)m * ldc + g0;
#pragma unroll
    for (int j = 0; j < NBT; ++j) {
      const float v = __fadd_rn(acc[j], bs[g0 + j]);
      acc[j] = act ? (v > 0.0f ? v : 0.0f) : v;
    }
    if (vec_out) {
#pragma unroll
      for (int j = 0; j < NBT; j += 4)
        if ((int)g0 + j < Cout)
          *reinterpret_cast<float4*>(dst + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < NBT; ++j)
        if ((int)g0 + j < Cout) dst[j] = acc[j];
    }
  }
}

static __device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(sdst)),
               "l"(gsrc)
               : "memory");
}

// 1x1 pad-0 convolution (any stride) with few output channels on CUDA cores, through shared
// memory.  A block of NW warps (4 in the dispatch: 6 and 8 measured slower) owns a run of
// TP = 32*PX*(NW/S) output pixels per tile: its input
// rows (Cin floats each) are copied into shared memory once with coalesced 16-byte cp.async
// (rows padded to an odd number of 16-byte chunks, so lane-per-pixel reads are conflict-free),
// each warp then computes NBT = NB/S output channels of 32*PX of those pixels (pixel p*32+lane
// of its set) with every weight load a warp-uniform broadcast, and the finished tile goes out
// through a padded shared-memory tile as coalesced 16-byte stores.  The next tile's input
// copy overlaps this tile's epilogue.  Per output the arithmetic is k_conv_simt's: an fp32 fma
// chain from 0 over the input channels, then + bias, then ReLU.
template <int NB, int S, int PX, int NW>
__global__ void __launch_bounds__(32 * NW, 16 / NW) k_pw_tile(const float* __restrict__ x, int H, int W, int Cs,
                                                 int coff, int Cin, const float* __restrict__ w,
                                                 long long ldw, const float* __restrict__ bias,
                                                 int Cout, int stride, int OH, int OW, unsigned M,
                                                 float* __restrict__ out, long long ldc, int act) {
  constexpr int NBT = NB / S, SETS = NW / S, TP = 32 * PX * SETS, NB4 = NB / 4, RO = NB4 | 1;
  static_assert(NBT * S == NB && NBT % 4 == 0 && SETS * S == NW, "16-byte weight broadcasts, S divides the warps");
  extern __shared__ float4 pt_sm4[];
  const int C4 = Cin >> 2, RS = C4 | 1, CO4 = Cout >> 2;
  float4* ws4 = pt_sm4;                     // [Cin][NB4] weights
  float4* bs4 = ws4 + Cin * NB4;            // [NB4] bias
  float4* xs = bs4 + NB4;                   // [TP][RS] input rows
  float4* os = xs + TP * RS;                // [TP][RO] output rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g0 = (warp % S) * NBT, row0 = (warp / S) * 32 * PX + lane;
  const unsigned tiles = (M + TP - 1) / TP;
  // row copies: with at most 32 chunks a row, one warp pass moves 32 / chunks rows (lane ->
  // row offset, chunk); wider rows are walked 32 chunks at a time
  const int rpi = C4 <= 32 ? 32 / C4 : 1, isub = C4 <= 32 ? lane / C4 : 0;
  const int ic = C4 <= 32 ? lane - isub * C4 : lane;
  const int rpo = 32 / CO4, osub = lane / CO4, oc = lane - osub * CO4;
  auto fill = [&](unsigned t) {
    if (isub >= rpi) return;
    for (int r = warp * rpi + isub; r < TP; r += NW * rpi) {
      const unsigned m = t * TP + r;
      if (m >= M) break;
      const unsigned ow = m % OW, tt = m / OW, oh = tt % OH, n = tt / OH;
      const float* src = x + (((size_t)n * H + oh * stride) * W + ow * stride) * Cs + coff;
      for (int c = ic; c < C4; c += 32) cp_async16(xs + r * RS + c, src + 4 * c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (blockIdx.x < tiles) fill(blockIdx.x);
  stage_block<16>(reinterpret_cast<float*>(ws4), Cin * NB, [&](int i) {
    const int k = i / NB, j = i - k * NB;
    return (j < Cout) ? __ldg(w + (long long)k * ldw + j) : 0.0f;
  });
  for (int j = threadIdx.x; j < NB; j += blockDim.x)
    reinterpret_cast<float*>(bs4)[j] = (bias && j < Cout) ? bias[j] : 0.0f;
  for (unsigned t = blockIdx.x; t < tiles; t += gridDim.x) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    float acc[PX][NBT];
#pragma unroll
    for (int p = 0; p < PX; ++p)
#pragma unroll
      for (int j = 0; j < NBT; ++j) acc[p][j] = 0.0f;
#pragma unroll 2
    for (int k4 = 0; k4 < C4; ++k4) {
      float4 xc[PX];
#pragma unroll
      for (int p = 0; p < PX; ++p) xc[p] = xs[(row0 + 32 * p) * RS + k4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4* wr4 = ws4 + (4 * k4 + u) * NB4 + g0 / 4;
#pragma unroll
        for (int j = 0; j < NBT; j += 4) {
          const float4 w4 = wr4[j / 4];
#pragma unroll
          for (int p = 0; p < PX; ++p) {
            const float xv = u == 0 ? xc[p].x : (u == 1 ? xc[p].y : (u == 2 ? xc[p].z : xc[p].w));
            const float2 x2 = make_float2(xv, xv);
            const float2 r0 = nx_ffma2(x2, make_float2(w4.x, w4.y), make_float2(acc[p][j], acc[p][j + 1]));
            const float2 r1 = nx_ffma2(x2, make_float2(w4.z, w4.w), make_float2(acc[p][j + 2], acc[p][j + 3]));
            acc[p][j] = r0.x;
            acc[p][j + 1] = r0.y;
            acc[p][j + 2] = r1.x;
            acc[p][j + 3] = r1.y;
          }
        }
      }
    }
    __syncthreads();  // every warp is done with xs
    if (t + gridDim.x < tiles) fill(t + gridDim.x);
#pragma unroll
    for (int p = 0; p < PX; ++p) {
#pragma unroll
      for (int j = 0; j < NBT; j += 4) {
        const float4 b4 = bs4[(g0 + j) / 4];
        float4 v;
        v.x = __fadd_rn(acc[p][j], b4.x);
        v.y = __fadd_rn(acc[p][j + 1], b4.y);
        v.z = __fadd_rn(acc[p][j + 2], b4.z);
        v.w = __fadd_rn(acc[p][j + 3], b4.w);
        if (act) {
          v.x = v.x > 0.0f ? v.x : 0.0f;
          v.y = v.y > 0.0f ? v.y : 0.0f;
          v.z = v.z > 0.0f ? v.z : 0.0f;
          v.w = v.w > 0.0f ? v.w : 0.0f;
        }
        os[(row0 + 32 * p) * RO + (g0 + j) / 4] = v;
      }
    }
    __syncthreads();  // the tile's outputs are in os
    if (osub < rpo) {
      for (int r = warp * rpo + osub; r < TP; r += NW * rpo) {
        const unsigned m = t * TP + r;
        if (m >= M) break;
        *reinterpret_cast<float4*>(out + (size_t)m * ldc + 4 * oc) = os[r * RO + oc];
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Small-K convolution fused with the 2x2 / stride-2 / pad-0 max-pool that follows it (an ACFUN0
// Conv -> MaxPool pair): a block owns one pooled output row; it stages the conv weights
// [K][Cout], the bias and the input rows that row needs in shared memory, then one thread per
// (pooled pixel, 16-channel block) computes the four conv outputs of its pool window (weights
// loaded once per k and reused by the four) and writes only their maximum.  Per conv output
// the arithmetic is k_conv_simt's: fma chain from 0 over k = (kh, kw, ic) of the in-image
// taps, + bias, then act; the pool is k_maxpool4's: start -1e30, window order (0,0) (0,1)
// (1,0) (1,1), then the pool's post-ReLU.
template <int CB>
__global__ void __launch_bounds__(128) k_conv_pool_simt(
    const float* __restrict__ x, int H, int W, int Cin, const float* __restrict__ w,
    const float* __restrict__ bias, int Cout, int KH, int KW, int stride, int pad, int PH, int PW,
    int rows_in, float* __restrict__ out, int act, int post_relu) {
  extern __shared__ float4 cp_sm4[];
  float* ws = reinterpret_cast<float*>(cp_sm4);  // [K][Cout]
  const int K = KH * KW * Cin;
  float* bs = ws + K * Cout;
  float* tile = bs + ((Cout + 3) & ~3);
  const int n = blockIdx.x / PH, ph = blockIdx.x - n * PH;
  const int ih0 = max(0, 2 * ph * stride - pad);
  const int ih1 = min(H, (2 * ph + 1) * stride - pad + KH);
  for (int i = threadIdx.x; i < K * Cout; i += blockDim.x) ws[i] = w[i];
  for (int i = threadIdx.x; i < Cout; i += blockDim.x) bs[i] = bias ? bias[i] : 0.0f;
  {
    const int tn = (ih1 - ih0) * W * Cin;
    const float* src = x + ((size_t)n * H + ih0) * W * Cin;
    constexpr int U = 8;
    for (int base = threadIdx.x; base < tn; base += U * blockDim.x) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < tn) v[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < tn) tile[i] = v[u];
      }
    }
  }
  (void)rows_in;
  __syncthreads();
  const int nb = Cout / CB, items = PW * nb;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int pw = it / nb, cb = it - pw * nb;
    float acc[4][CB];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int j = 0; j < CB; ++j) acc[p][j] = 0.0f;
    for (int kh = 0; kh < KH; ++kh) {
      for (int kw = 0; kw < KW; ++kw) {
        // the pool window's four conv pixels: (2ph + dy, 2pw + dx)
        int xoff[4];
        bool ok[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int ih = (2 * ph + (p >> 1)) * stride - pad + kh;
          const int iw = (2 * pw + (p & 1)) * stride - pad + kw;
          ok[p] = ih >= 0 && ih < H && iw >= 0 && iw < W;
          xoff[p] = ((ih - ih0) * W + iw) * Cin;
        }
        for (int ic = 0; ic < Cin; ++ic) {
          const float4* wr = reinterpret_cast<const float4*>(ws + ((kh * KW + kw) * Cin + ic) * Cout + cb * CB);
          float wv[CB];
#pragma unroll
          for (int q = 0; q < CB / 4; ++q) {
            const float4 t = wr[q];
            wv[4 * q] = t.x; wv[4 * q + 1] = t.y; wv[4 * q + 2] = t.z; wv[4 * q + 3] = t.w;
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            if (!ok[p]) continue;
            const float xv = tile[xoff[p] + ic];
#pragma unroll
            for (int j = 0; j < CB; ++j) acc[p][j] = __fmaf_rn(xv, wv[j], acc[p][j]);
          }
        }
      }
    }
    float m[CB];
#pragma unroll
    for (int j = 0; j < CB; ++j) m[j] = -1e30f;
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        float v = __fadd_rn(acc[p][j], bs[cb * CB + j]);
        v = act ? (v > 0.0f ? v : 0.0f) : v;
        m[j] = m[j] > v ? m[j] : v;
      }
    float* dst = out + (((size_t)n * PH + ph) * PW + pw) * Cout + cb * CB;
#pragma unroll
    for (int q = 0; q < CB / 4; ++q) {
      float4 r = make_float4(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3]);
      if (post_relu) {
        r.x = r.x > 0.f ? r.x : 0.f; r.y = r.y > 0.f ? r.y : 0.f;
        r.z = r.z > 0.f ? r.z : 0.f; r.w = r.w > 0.f ? r.w : 0.f;
      }
      reinterpret_cast<float4*>(dst)[q] = r;
    }
  }
}

// k_conv_pool_simt specialised at compile time for the first layer of an image network
// (3x3, stride 1, pad 1, Cin = 3): the input tile is split by column parity and keeps the
// channels of a pixel together ([row][iw & 1][iw >> 1][CIN]), so for every tap the four
// pixels of a pool window read fixed offsets from one per-thread base and a warp's reads
// are CIN words apart (conflict-free for odd CIN); all 27 taps unroll.  Border items take
// the bounds-checked loop.  Arithmetic identical to k_conv_pool_simt.
template <int CIN, int CB>
__global__ void __launch_bounds__(128) k_conv_pool_3x3s1(
    const float* __restrict__ x, int H, int W, const float* __restrict__ w,
    const float* __restrict__ bias, int Cout, int PH, int PW, float* __restrict__ out, int act,
    int post_relu, void* out_split, long long split_plane, int sHp, int sWp, int spad) {
  constexpr int KH = 3, KW = 3, K = KH * KW * CIN, ROWS = 1 + KH;  // stride 1, pad 1
  extern __shared__ float4 cf_sm4[];
  float* ws = reinterpret_cast<float*>(cf_sm4);  // [K][Cout]
  float* bs = ws + K * Cout;
  float* tile = bs + ((Cout + 3) & ~3);  // [ROWS][2][hw][CIN]
  const int hw = (W + 1) >> 1, plane = hw * CIN;
  const int n = blockIdx.x / PH, ph = blockIdx.x - n * PH;
  const int r0 = 2 * ph - 1;  // input row of tile row 0
  const int ih0 = max(0, r0), ih1 = min(H, r0 + ROWS);
  for (int i = threadIdx.x; i < K * Cout; i += blockDim.x) ws[i] = w[i];
  for (int i = threadIdx.x; i < Cout; i += blockDim.x) bs[i] = bias ? bias[i] : 0.0f;
  {
    const int tn = (ih1 - ih0) * W * CIN;
    const float* src = x + ((size_t)n * H + ih0) * W * CIN;
    const int base_r = ih0 - r0;
    constexpr int U = 8;
    for (int b0 = threadIdx.x; b0 < tn; b0 += U * blockDim.x) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        if (i < tn) v[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = b0 + u * blockDim.x;
        if (i < tn) {
          const int pix = i / CIN, ic = i - pix * CIN;
          const int r = pix / W, iw = pix - r * W;
          tile[((base_r + r) * 2 + (iw & 1)) * plane + (iw >> 1) * CIN + ic] = v[u];
        }
      }
    }
  }
  __syncthreads();
  const int nb = Cout / CB, items = PW * nb;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int cb = it / PW, pw = it - cb * PW;
    float2 acc[4][CB / 2];  // channel pairs (2j, 2j+1), one packed fma per pair
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int j = 0; j < CB / 2; ++j) acc[p][j] = make_float2(0.0f, 0.0f);
    const bool interior = r0 >= 0 && r0 + ROWS <= H && pw >= 1 && 2 * pw + 2 < W;
    if (interior) {
      // pixel (dy, dx), tap (kh, kw): tile row dy + kh, column 2pw + dx - 1 + kw
      const float* tb = tile + (pw - 1) * CIN;
#pragma unroll
      for (int kh = 0; kh < KH; ++kh)
#pragma unroll
        for (int kw = 0; kw < KW; ++kw)
#pragma unroll
          for (int ic = 0; ic < CIN; ++ic) {
            const int k = (kh * KW + kw) * CIN + ic;
            const float4* wr = reinterpret_cast<const float4*>(ws + k * Cout + cb * CB);
            float2 wv[CB / 2];
#pragma unroll
            for (int q = 0; q < CB / 4; ++q) {
              const float4 t = wr[q];
              wv[2 * q] = make_float2(t.x, t.y);
              wv[2 * q + 1] = make_float2(t.z, t.w);
            }
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const int dy = p >> 1, dx = p & 1;
              const int col = 2 + dx - 1 + kw;  // column relative to 2*(pw-1)
              const float xv = tb[((dy + kh) * 2 + (col & 1)) * plane + (col >> 1) * CIN + ic];
              const float2 x2 = make_float2(xv, xv);
#pragma unroll
              for (int j = 0; j < CB / 2; ++j) acc[p][j] = nx_ffma2(x2, wv[j], acc[p][j]);
            }
          }
    } else {
      for (int kh = 0; kh < KH; ++kh)
        for (int kw = 0; kw < KW; ++kw)
#pragma unroll
          for (int ic = 0; ic < CIN; ++ic) {
            const int k = (kh * KW + kw) * CIN + ic;
            const float4* wr = reinterpret_cast<const float4*>(ws + k * Cout + cb * CB);
            float2 wv[CB / 2];
#pragma unroll
            for (int q = 0; q < CB / 4; ++q) {
              const float4 t = wr[q];
              wv[2 * q] = make_float2(t.x, t.y);
              wv[2 * q + 1] = make_float2(t.z, t.w);
            }
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const int dy = p >> 1, dx = p & 1;
              const int ih = 2 * ph + dy - 1 + kh, iw = 2 * pw + dx - 1 + kw;
              if (ih < 0 || ih >= H || iw < 0 || iw >= W) continue;
              const float xv = tile[((ih - r0) * 2 + (iw & 1)) * plane + (iw >> 1) * CIN + ic];
              const float2 x2 = make_float2(xv, xv);
#pragma unroll
              for (int j = 0; j < CB / 2; ++j) acc[p][j] = nx_ffma2(x2, wv[j], acc[p][j]);
            }
          }
    }
    float m[CB];
#pragma unroll
    for (int j = 0; j < CB; ++j) m[j] = -1e30f;
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        float v = __fadd_rn((j & 1) ? acc[p][j / 2].y : acc[p][j / 2].x, bs[cb * CB + j]);
        v = act ? (v > 0.0f ? v : 0.0f) : v;
        m[j] = m[j] > v ? m[j] : v;
      }
    if (post_relu) {
#pragma unroll
      for (int j = 0; j < CB; ++j) m[j] = m[j] > 0.f ? m[j] : 0.f;
    }
    if (out_split) {
      // the next convolution's split input (hi = bf16(v), lo = bf16(v - hi): k_pad_split4's
      // split), CB channels per plane in 16-byte stores
      uint32_t ph2[CB / 2], pl2[CB / 2];
#pragma unroll
      for (int j = 0; j < CB; j += 2) nx_split_bf16x2(m[j], m[j + 1], ph2[j / 2], pl2[j / 2]);
      uint16_t* hi = reinterpret_cast<uint16_t*>(out_split) +
                     (((size_t)n * sHp + ph + spad) * sWp + pw + spad) * Cout + cb * CB;
      uint16_t* lo = hi + split_plane;
#pragma unroll
      for (int q = 0; q < CB / 8; ++q) {
        reinterpret_cast<uint4*>(hi)[q] = make_uint4(ph2[4 * q], ph2[4 * q + 1], ph2[4 * q + 2], ph2[4 * q + 3]);
        reinterpret_cast<uint4*>(lo)[q] = make_uint4(pl2[4 * q], pl2[4 * q + 1], pl2[4 * q + 2], pl2[4 * q + 3]);
      }
    } else {
      float* dst = out + (((size_t)n * PH + ph) * PW + pw) * Cout + cb * CB;
#pragma unroll
      for (int q = 0; q < CB / 4; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3]);
    }
  }
}

// im2col of a small-K convolution in pooled-window order, as the 3xBF16 split: row
// ((n*PH + py)*PW + px)*4 + d holds the patch of output pixel (2py + d/2, 2px + d%2), K in
// (kh, kw, ci) order zero-padded to KP, bf16 hi = bf16(v) and lo = bf16(v - hi) planes
// (k_pad_split4's split).  The pooling GEMM epilogue then reduces each group of four rows.
template <int KP>
__global__ void k_im2col_pool_split(const float* __restrict__ x, int H, int W, int Cin, int KH,
                                    int KW, int stride, int pad, int PH, int PW, long long rows,
                                    uint16_t* __restrict__ hi, long long plane) {
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < rows;
       r += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(r & 3);
    long long P = r >> 2;
    const int px = (int)(P % PW);
    P /= PW;
    const int py = (int)(P % PH);
    const long long n = P / PH;
    const int iy0 = (2 * py + (d >> 1)) * stride - pad, ix0 = (2 * px + (d & 1)) * stride - pad;
    const float* xn = x + n * H * W * Cin;
    float v[KP];
    int kh = 0, kw = 0, ci = 0;
#pragma unroll
    for (int k = 0; k < KP; ++k) {
      float t = 0.0f;
      if (kh < KH) {
        const int iy = iy0 + kh, ix = ix0 + kw;
        if (iy >= 0 && iy < H && ix >= 0 && ix < W) t = xn[((long long)iy * W + ix) * Cin + ci];
        if (++ci == Cin) {
          ci = 0;
          if (++kw == KW) {
            kw = 0;
            ++kh;
          }
        }
      }
      v[k] = t;
    }
    uint32_t ph[KP / 2], pl[KP / 2];
#pragma unroll
    for (int k = 0; k < KP; k += 2) nx_split_bf16x2(v[k], v[k + 1], ph[k / 2], pl[k / 2]);
    uint4* dh = reinterpret_cast<uint4*>(hi + r * KP);
    uint4* dl = reinterpret_cast<uint4*>(hi + plane + r * KP);
#pragma unroll
    for (int q = 0; q < KP / 8; ++q) {
      dh[q] = make_uint4(ph[4 * q], ph[4 * q + 1], ph[4 * q + 2], ph[4 * q + 3]);
      dl[q] = make_uint4(pl[4 * q], pl[4 * q + 1], pl[4 * q + 2], pl[4 * q + 3]);
    }
  }
}

// k_im2col_pool_split<32> for the 3x3 / stride 1 / pad 1 / 3-channel case.  A block of 64
// threads takes 64 consecutive pooled pixels, one each: the pixel's 4x4x3 input patch is read
// once and its window's four rows (256 bytes per plane) go to shared memory; the block's rows
// are contiguous in both planes, so they leave in coalesced 16-byte stores.
constexpr int kIm2colPix = 64;
constexpr int kIm2colRowB = 272;  // 256 bytes per pixel + 16: conflict-free 16-byte writes
__global__ void __launch_bounds__(kIm2colPix) k_im2col_pool_3x3c3(
    const float* __restrict__ x, int H, int W, int PH, int PW, long long pooled,
    uint16_t* __restrict__ hi, long long plane) {
  __shared__ __align__(16) uint8_t st[2][kIm2colPix * kIm2colRowB];
  const int t = threadIdx.x;
  for (long long base = (long long)blockIdx.x * kIm2colPix; base < pooled;
       base += (long long)gridDim.x * kIm2colPix) {
    const long long P = base + t;
    if (P < pooled) {
      const int px = (int)(P % PW);
      const long long q = P / PW;
      const int py = (int)(q % PH);
      const long long n = q / PH;
      const int y0 = 2 * py - 1, x0 = 2 * px - 1;
      const float* xn = x + n * H * W * 3;
      const bool inside = y0 >= 0 && y0 + 4 <= H && x0 >= 0 && x0 + 4 <= W;
      float p[4][12];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 12; ++c) {
          const int iy = y0 + r, ix = x0 + c / 3;
          p[r][c] = (inside || (iy >= 0 && iy < H && ix >= 0 && ix < W))
                        ? xn[((long long)iy * W + x0) * 3 + c]
                        : 0.0f;
        }
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        const int dy = d >> 1, dx = d & 1;
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; ++k)
          v[k] = k < 27 ? p[dy + k / 9][(dx + (k / 3) % 3) * 3 + k % 3] : 0.0f;
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) nx_split_bf16x2(v[k], v[k + 1], ph[k / 2], pl[k / 2]);
        uint4* sh = reinterpret_cast<uint4*>(st[0] + t * kIm2colRowB + d * 64);
        uint4* sl = reinterpret_cast<uint4*>(st[1] + t * kIm2colRowB + d * 64);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sh[u] = make_uint4(ph[4 * u], ph[4 * u + 1], ph[4 * u + 2], ph[4 * u + 3]);
          sl[u] = make_uint4(pl[4 * u], pl[4 * u + 1], pl[4 * u + 2], pl[4 * u + 3]);
        }
      }
    }
    __syncthreads();
    const int npix = (int)(pooled - base < kIm2colPix ? pooled - base : kIm2colPix);
    uint4* gh = reinterpret_cast<uint4*>(hi + base * 4 * 32);
    uint4* gl = reinterpret_cast<uint4*>(hi + plane + base * 4 * 32);
    for (int u = t; u < npix * 16; u += kIm2colPix) {
      const int off = (u >> 4) * kIm2colRowB + (u & 15) * 16;
      gh[u] = *reinterpret_cast<const uint4*>(st[0] + off);
      gl[u] = *reinterpret_cast<const uint4*>(st[1] + off);
    }
    __syncthreads();
  }
}

// Conv (K <= 64) + 2x2/2 max-pool on the tensor cores: pooled-order im2col, then a 3xBF16
// GEMM whose epilogue takes each window's maximum before bias and activation (max commutes
// with the per-channel bias add and ReLU, both monotone).  Images go in chunks whose im2col
// stays in L2 between its producer and the GEMM.
static bool conv_pool_tc(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                         const float* bias, int KH, int KW, int Cout, int stride, int pad, int act,
                         int PH, int PW, float* out, const SplitAct* os) {
  const int K = KH * KW * Cin, KP = K <= 32 ? 32 : 64;
  const int Np = (int)align_up((size_t)Cout, 8);
  const long long img_rows = 4LL * PH * PW;
  const long long img_bytes = img_rows * KP * 2 * 2;
  const int chunk = (int)std::max<long long>(1, std::min<long long>(N, kPoolIm2colChunkBytes / img_bytes));
  const long long plane = (long long)chunk * img_rows * KP;
  uint16_t* a = static_cast<uint16_t*>(c.scratch((size_t)(2 * plane * 2 + split_weight_bytes(1, KP, Cout))));
  if (!a) return false;
  void* b = a + 2 * plane;
  k_weights_split<true><<<grid_ew(c, (long long)KP * Np), 256, 0, c.stream()>>>(
      w, 1, K, Cout, Cout, KP, Np, b, (long long)KP * Np);
  if (!c.launched("k_weights_split")) return false;
  EpiParams ep{};
  ep.f0 = bias;
  ep.act = act;
  ep.pool4 = 1;
  ep.ph = PH;
  ep.pw = PW;
  ep.ldc = Cout;
  if (os) {
    ep.split_plane = os->plane;
    ep.sHp = os->H + 2 * os->pad;
    ep.sWp = os->W + 2 * os->pad;
    ep.spad = os->pad;
    ep.sC = os->C;
    ep.ldc = os->C;
  }
  Operand A, B;
  A.p = a;
  A.ld = KP;
  A.op_stride = plane;
  B.p = b;
  B.ld = Np;
  B.op_stride = (long long)KP * Np;
  for (int n0 = 0; n0 < N; n0 += chunk) {
    const int nc = std::min(chunk, N - n0);
    const long long rows = nc * img_rows;
    if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && Cin == 3)
      k_im2col_pool_3x3c3<<<(unsigned)std::min<long long>((rows / 4 + kIm2colPix - 1) / kIm2colPix,
                                                          64LL * c.sm_count()),
                            kIm2colPix, 0, c.stream()>>>(
          x + (long long)n0 * H * W * Cin, H, W, PH, PW, rows / 4, a, plane);
    else if (KP == 32)
      k_im2col_pool_split<32><<<grid_ew(c, rows), 256, 0, c.stream()>>>(
          x + (long long)n0 * H * W * Cin, H, W, Cin, KH, KW, stride, pad, PH, PW, rows, a, plane);
    else
      k_im2col_pool_split<64><<<grid_ew(c, rows), 256, 0, c.stream()>>>(
          x + (long long)n0 * H * W * Cin, H, W, Cin, KH, KW, stride, pad, PH, PW, rows, a, plane);
    if (!c.launched("k_im2col_pool_split")) return false;
    if (os)
      ep.split_out = static_cast<uint16_t*>(os->base) + (long long)n0 * ep.sHp * ep.sWp * ep.sC;
    else
      ep.C = out + (long long)n0 * PH * PW * Cout;
    if (!gemm_launch(c, GemmKind::BF16X3, Epi::F32_BIAS, A, B, (int)rows, Cout, KP, ep))
      return false;
  }
  return true;
}

bool conv_pool_dev(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                   const float* bias, int KH, int KW, int Cout, int stride, int pad, int act,
                   int pool, int pst, int ppd, int post_relu, float* out, bool* handled,
                   const SplitAct* os) {
  *handled = false;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (pool != 2 || pst != 2 || ppd != 0 || OH < 2 || OW < 2 || Cout % 16 != 0) return true;
  const int K = KH * KW * Cin;
  const int PH = (OH - 2) / 2 + 1, PW = (OW - 2) / 2 + 1;
  // tensor-core route once the GEMM fills the GPU (two 128-row sub-tiles per CTA)
  if (K <= 64 && fp32_math(Fp32Use::Conv) == Fp32Math::BF16X3 &&
      4LL * N * PH * PW >= 256LL * c.sm_count() && 4LL * PH * PW * 64 * 4 <= kPoolIm2colChunkBytes) {
    *handled = true;
    return conv_pool_tc(c, x, N, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, act | post_relu, PH,
                        PW, out, os);
  }
  if (K > 64 || Cout > 64 || !aligned16(w) || !aligned16(out) || (long long)N * PH >= (1LL << 31))
    return true;
  if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && Cin == 3) {
    const long long smem3 = ((long long)K * Cout + ((Cout + 3) & ~3) + 4LL * 2 * ((W + 1) / 2) * 3) * 4;
    if (smem3 <= 48 * 1024 && (long long)4 * W * 3 < (1LL << 31)) {
      k_conv_pool_3x3s1<3, 16><<<N * PH, 128, (size_t)smem3, c.stream()>>>(
          x, H, W, w, bias, Cout, PH, PW, out, act, post_relu, os ? os->base : nullptr,
          os ? os->plane : 0, os ? os->H + 2 * os->pad : 0, os ? os->W + 2 * os->pad : 0,
          os ? os->pad : 0);
      *handled = true;
      return c.launched("k_conv_pool_3x3s1");
    }
  }
  if (os) return true;  // split output only from the 3x3 / Cin 3 kernel
  const long long rows_in = std::min<long long>(H, (long long)stride + KH);
  const long long smem = ((long long)K * Cout + ((Cout + 3) & ~3) + rows_in * W * Cin) * 4;
  // same cases as conv_simt (K <= 64, Cout <= 64), so the fused result equals conv + pool
  if (smem > 48 * 1024 || (long long)rows_in * W * Cin >= (1LL << 31)) return true;
  k_conv_pool_simt<16><<<N * PH, 128, (size_t)smem, c.stream()>>>(
      x, H, W, Cin, w, bias, Cout, KH, KW, stride, pad, PH, PW, (int)rows_in, out, act, post_relu);
  *handled = true;
  return c.launched("k_conv_pool_simt");
}

// Returns true when the CUDA-core path applies (and has been launched).
static bool conv_simt(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cg,
                      const float* w, long long ldw, const float* bias, int KH, int KW, int Cout,
                      int stride, int pad, float* out, long long ldc, int act, bool* handled) {
  *handled = false;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  const long long M = (long long)N * OH * OW;
  const int K = KH * KW * Cg;
  const bool narrow = (KH == 1 && KW == 1 && pad == 0) || K <= 64;
  const int NB = Cout <= 16 ? 16 : Cout <= 24 ? 24 : Cout <= 32 ? 32 : Cout <= 48 ? 48 : 64;
  const size_t smem = ((size_t)K * NB + NB) * 4;
  if (!narrow || Cout > 64 || smem > 48 * 1024 || M >= (1LL << 30)) return true;
  *handled = true;
  const int vec_in = (Cs % 4 == 0) && (coff % 4 == 0) && aligned16(x);
  const int vec_out = (Cout % 4 == 0) && (ldc % 4 == 0) && aligned16(out);
  // 1x1 stride 1 over enough pixels to fill the GPU: tensor cores (3xBF16), one read of x
  if (KH == 1 && KW == 1 && pad == 0 && stride == 1 && fp32_math(Fp32Use::Conv) == Fp32Math::BF16X3 &&
      conv_pw_tc_ok(x, Cs, coff, Cg, Cout, M))
    return conv_pw_tc_dev(c, x, M, Cg, w, ldw, bias, Cout, out, ldc, act);
  if (KH == 1 && KW == 1 && pad == 0 && vec_in && vec_out && Cg % 4 == 0 && Cout % 4 == 0 &&
      (NB == 24 || NB == 64)) {
    // 1x1: blocks of NW warps over shared-memory tiles of 32*PX*(NW/S) output pixels
    constexpr int S64 = 4, PX64 = 2, NW64 = 4, S24 = 2, PX24 = 1, NW24 = 4;
    const int TP = NB == 24 ? 32 * PX24 * (NW24 / S24) : 32 * PX64 * (NW64 / S64);
    const int NWv = NB == 24 ? NW24 : NW64;
    const size_t tsmem = smem + (size_t)TP * ((Cg / 4) | 1) * 16 + (size_t)TP * ((NB / 4) | 1) * 16;
    auto kern = NB == 24 ? k_pw_tile<24, S24, PX24, NW24> : k_pw_tile<64, S64, PX64, NW64>;
    static bool attr_done[64][2] = {};
    const int dv = current_device(), ki = NB == 24;
    if (tsmem > 48 * 1024 && dv >= 0 && dv < 64 && !attr_done[dv][ki]) {
      if (!ACF_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024))) {
        c.fail();
        return false;
      }
      attr_done[dv][ki] = true;
    }
    const long long per_sm =
        std::max<long long>(1, std::min<long long>(16 / NWv, (227 * 1024) / (long long)(tsmem + 1024)));
    const int grid = (int)std::min<long long>((M + TP - 1) / TP, per_sm * c.sm_count());
    kern<<<grid, 32 * NWv, tsmem, c.stream()>>>(x, H, W, Cs, coff, Cg, w, ldw, bias, Cout, stride, OH, OW,
                                               (unsigned)M, out, ldc, act);
    return c.launched("k_pw_tile");
  }
  // a few resident blocks per SM, each walking many pixels: the weight staging is paid once
  // per block
  const int grid = (int)std::min<long long>((2 * M + 127) / 128, 8LL * c.sm_count());
#define ACF_CONV_SIMT(NBV)                                                                      \
  k_conv_simt<NBV, 2><<<grid, 128, smem, c.stream()>>>(x, H, W, Cs, coff, Cg, w, ldw, bias, Cout,  \
                                                       KH, KW, stride, pad, OH, OW, (unsigned)M, \
                                                       out, ldc, act, vec_in, vec_out)
  if (NB == 16)
    ACF_CONV_SIMT(16);
  else if (NB == 24)
    ACF_CONV_SIMT(24);
  else if (NB == 32)
    ACF_CONV_SIMT(32);
  else if (NB == 48)
    ACF_CONV_SIMT(48);
  else
    ACF_CONV_SIMT(64);
#undef ACF_CONV_SIMT
  return c.launched("k_conv_simt");
}

template <bool BF>
static bool conv_tc(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cg,
                    const float* w, long long ldw, const float* bias, int KH, int KW, int Cout_g,
                    int stride, int pad, float* out, long long ldc, int act) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  const int taps = KH * KW;
  const int E = BF ? 2 : 4;             // bytes per split element
  const int BKE = BF ? 64 : 32;         // channels per 128-byte K block
  const int Np = (int)align_up((size_t)Cout_g, BF ? 8 : 4);
  const GemmKind kind = BF ? GemmKind::BF16X3 : GemmKind::TF32X3;
  EpiParams ep{};
  ep.C = out;
  ep.ldc = ldc;
  ep.f0 = bias;
  ep.act = act;
  Operand A, B;
  if constexpr (BF) {
    // narrow convolutions: resident weights, the activation converted inside the kernel
    static const bool halo_on = [] {
      const char* e = getenv("ACFUN_CONV_HALO");
      return !(e && !strcmp(e, "0"));
    }();
    if (halo_on && conv_halo_ok(Cg, KH, KW, Cout_g, stride))
      return conv_halo_f32_dev(c, x, N, H, W, Cs, coff, Cg, w, ldw, bias, KH, KW, Cout_g, pad, out,
                               ldc, act);
  }
  if (stride == 1) {
    const int Hp = H + 2 * pad, Wp = W + 2 * pad;
    const int Cpad = (int)align_up((size_t)Cg, BKE);
    const long long rows = (long long)N * Hp * Wp;
    const long long groups4 = rows * (Cpad / 4);
    if (rows >= (1LL << 31) || groups4 >= (1LL << 32)) {
      set_error(kInvalid, "%s: tensor too large", c.name());
      c.fail();
      return false;
    }
    void* a = c.scratch((size_t)2 * rows * Cpad * E);
    void* b = c.scratch((size_t)2 * taps * Cpad * Np * E);
    if (!a || !b) return false;
    const int vec_in = (Cs % 4 == 0) && (coff % 4 == 0) && aligned16(x);
    k_pad_split4<BF><<<grid_ew(c, groups4), 256, 0, c.stream()>>>(
        x, H, W, Cs, coff, Cg, pad, Hp, Wp, Cpad / 4, (unsigned)groups4, vec_in, a, (size_t)(rows * Cpad));
    k_weights_split<BF><<<grid_ew(c, (long long)taps * Cpad * Np), 256, 0, c.stream()>>>(
        w, taps, Cg, Cout_g, ldw, Cpad, Np, b, (long long)taps * Cpad * Np);
    if (!c.launched("conv prep")) return false;
    A.p = a;
    A.ld = Cpad;
    A.op_stride = rows * Cpad;
    B.p = b;
    B.ld = Np;
    B.op_stride = (long long)taps * Cpad * Np;
    ep.remap = 1;
    ep.img_rows = Hp * Wp;
    ep.Wp = Wp;
    ep.OH = OH;
    ep.OW = OW;
    ConvGeom cg{1, Cpad / BKE, KW, Wp, Cpad, taps};
    return gemm_launch(c, kind, Epi::F32_BIAS, A, B, (int)rows, Cout_g, taps * Cpad, ep, cg);
  }
  const long long M = (long long)N * OH * OW;
  const int K = taps * Cg, Kpad = (int)align_up((size_t)K, BF ? 8 : 4);
  void* a = c.scratch((size_t)2 * M * Kpad * E);
  void* b = c.scratch((size_t)2 * K * Np * E);
  if (!a || !b) return false;
  k_im2col_split<BF><<<grid_ew(c, M * Kpad), 256, 0, c.stream()>>>(x, N, H, W, Cs, coff, Cg, KH, KW,
                                                                   stride, pad, OH, OW, Kpad, a, M * Kpad);
  k_weights_split<BF><<<grid_ew(c, (long long)K * Np), 256, 0, c.stream()>>>(w, 1, K, Cout_g, ldw, K,
                                                                            Np, b, (long long)K * Np);
  if (!c.launched("im2col prep")) return false;
  A.p = a;
  A.ld = Kpad;
  A.op_stride = M * Kpad;
  B.p = b;
  B.ld = Np;
  B.op_stride = (long long)K * Np;
  return gemm_launch(c, kind, Epi::F32_BIAS, A, B, (int)M, Cout_g, K, ep);
}

// ------------------------------------------------------------------ split activations
bool conv_split_ok(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad) {
  if (fp32_math(Fp32Use::Conv) != Fp32Math::BF16X3) return false;
  if (stride != 1 || Cin % 64 != 0 || Cout % 64 != 0 || KH <= 0 || KW <= 0 || pad < 0) return false;
  const int OH = H + 2 * pad - KH + 1, OW = W + 2 * pad - KW + 1;
  if (OH <= 0 || OW <= 0) return false;
  // the CUDA-core route takes narrow layers (conv_simt's condition)
  const int K = KH * KW * Cin;
  const bool narrow = (KH == 1 && KW == 1 && pad == 0) || K <= 64;
  if (narrow && Cout <= 64) return false;
  return true;
}

// one thread per (border pixel, 8 channels) of each plane
__global__ void k_split_border(uint4* __restrict__ base, long long plane8, int N, int Hp, int Wp,
                               int C8, int pad, long long total) {
  const int bw = 2 * pad * Wp + 2 * pad * (Hp - 2 * pad);  // border pixels per image
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % C8);
    long long r = i / C8;
    const int b = (int)(r % bw);
    r /= bw;
    const int n = (int)(r % N), p = (int)(r / N);
    int hp, wp;
    if (b < pad * Wp) {
      hp = b / Wp;
      wp = b % Wp;
    } else if (b < 2 * pad * Wp) {
      hp = Hp - pad + (b - pad * Wp) / Wp;
      wp = (b - pad * Wp) % Wp;
    } else {
      const int q = b - 2 * pad * Wp, side = q % (2 * pad);
      hp = pad + q / (2 * pad);
      wp = side < pad ? side : Wp - 2 * pad + side;
    }
    base[p * plane8 + (((long long)n * Hp + hp) * Wp + wp) * C8 + c8] = make_uint4(0, 0, 0, 0);
  }
}

bool split_border_dev(Call& c, const SplitAct& a) {
  if (a.pad == 0) return true;
  const int Hp = a.H + 2 * a.pad, Wp = a.W + 2 * a.pad, C8 = a.C / 8;
  const long long bw = 2LL * a.pad * Wp + 2LL * a.pad * (Hp - 2 * a.pad);
  const long long total = 2 * (long long)a.N * bw * C8;
  k_split_border<<<grid_ew(c, total), 256, 0, c.stream()>>>((uint4*)a.base, a.plane / 8, a.N, Hp, Wp,
                                                             C8, a.pad, total);
  return c.launched("k_split_border");
}

long long split_weight_bytes(int taps, int Cin, int Cout) {
  return 2LL * 2 * taps * Cin * (long long)align_up((size_t)Cout, 8);
}

bool split_weights_dev(Call& c, const float* w, int taps, int Cin, int Cout, void* dst) {
  const int Np = (int)align_up((size_t)Cout, 8);
  k_weights_split<true><<<grid_ew(c, (long long)taps * Cin * Np), 256, 0, c.stream()>>>(
      w, taps, Cin, Cout, Cout, Cin, Np, dst, (long long)taps * Cin * Np);
  return c.launched("k_weights_split");
}

long long pair_geometry(ConvGeom& cg, int N, int Hp, int OH, int OW) {
  if (Hp % 2 != 0 || OH < 2 || OW < 2) return 0;
  // Tile width 2^bxl: the widest whose column blocks cover the 2*(OW/2) pooled columns with
  // at most 3 % padding (every padding column is MMA work for a discarded lane), else the
  // least padded; e.g. OW 112 -> 16 (7 blocks), 56 -> 8, 28 -> 4, 14 -> 2.
  const int used = 2 * (OW / 2);
  int bxl = 0;
  double best = -1.0;
  for (int l = 7; l >= 1; --l) {
    const int bx = 1 << l, blocks = (used + bx - 1) / bx;
    const double util = (double)used / ((double)blocks * bx);
    if (util >= 0.97) {
      bxl = l;
      break;
    }
    if (util > best) {
      best = util;
      bxl = l;
    }
  }
  cg.pair = 1;
  cg.bxl = bxl;
  cg.by = 128 >> bxl;
  cg.xb = (used + (1 << bxl) - 1) >> bxl;
  cg.hp2 = Hp / 2;
  cg.npr = N * (Hp / 2);
  const long long pb = (cg.npr + cg.by - 1) / cg.by;
  return pb * cg.xb * 256;
}

bool conv_tc_split_dev(Call& c, const float* x, const SplitAct* xs, int N, int H, int W,
                       int Cin, const float* w, const void* ws, const float* bias, int KH,
                       int KW, int Cout, int pad, float* out, const SplitAct* os, int act,
                       bool pool) {
  const int OH = H + 2 * pad - KH + 1, OW = W + 2 * pad - KW + 1;
  const int taps = KH * KW, Hp = H + 2 * pad, Wp = W + 2 * pad, Cpad = Cin;
  const int Np = (int)align_up((size_t)Cout, 8);
  const long long rows = (long long)N * Hp * Wp;
  if (rows >= (1LL << 31) || rows * (Cpad / 4) >= (1LL << 32) || (xs && xs->pad != pad)) {
    set_error(kInvalid, "%s: split conv geometry", c.name());
    c.fail();
    return false;
  }
  const void* a = xs ? xs->base : nullptr;
  long long plane = xs ? xs->plane : rows * Cpad;
  if (!a) {
    void* s = c.scratch((size_t)2 * rows * Cpad * 2);
    if (!s) return false;
    const long long groups4 = rows * (Cpad / 4);
    const int vec_in = aligned16(x);
    k_pad_split4<true><<<grid_ew(c, groups4), 256, 0, c.stream()>>>(
        x, H, W, Cin, 0, Cin, pad, Hp, Wp, Cpad / 4, (unsigned)groups4, vec_in, s, (size_t)plane);
    a = s;
  }
  if (!ws) {
    void* s = c.scratch((size_t)split_weight_bytes(taps, Cin, Cout));
    if (!s || !split_weights_dev(c, w, taps, Cin, Cout, s)) return false;
    ws = s;
  }
  if (!c.launched("split conv prep")) return false;
  EpiParams ep{};
  ep.C = out;
  ep.ldc = Cout;
  ep.f0 = bias;
  ep.act = act;
  ep.remap = 1;
  ep.img_rows = Hp * Wp;
  ep.Wp = Wp;
  ep.OH = OH;
  ep.OW = OW;
  if (os) {
    ep.split_out = os->base;
    ep.split_plane = os->plane;
    ep.sHp = os->H + 2 * os->pad;
    ep.sWp = os->W + 2 * os->pad;
    ep.spad = os->pad;
    ep.sC = os->C;
    ep.ldc = os->C;
  }
  Operand A, B;
  A.p = a;
  A.ld = Cpad;
  A.op_stride = plane;
  B.p = ws;
  B.ld = Np;
  B.op_stride = (long long)taps * Cpad * Np;
  ConvGeom cg{1, Cpad / 64, KW, Wp, Cpad, taps};
  long long M = rows;
  if (pool) {
    // the 2x2 / stride-2 max-pool in the epilogue: output (N, OH/2, OW/2, Cout), fp32 `out`
    // or the split planes `os` of that size
    M = pair_geometry(cg, N, Hp, OH, OW);
    if (M <= 0 || M >= (1LL << 31)) {
      set_error(kInvalid, "%s: pooled split conv geometry", c.name());
      c.fail();
      return false;
    }
    ep.remap = 0;
    ep.ph = OH / 2;
    ep.pw = OW / 2;
  }
  return gemm_launch(c, GemmKind::BF16X3, Epi::F32_BIAS, A, B, (int)M, Cout, taps * Cpad, ep, cg);
}

bool conv_f32_dev(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cg,
                  const float* w, long long ldw, const float* bias, int KH, int KW, int Cout_g,
                  int stride, int pad, float* out, long long ldc, int act) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0 || N <= 0 || Cout_g <= 0) return true;
  bool handled = false;
  if (!conv_simt(c, x, N, H, W, Cs, coff, Cg, w, ldw, bias, KH, KW, Cout_g, stride, pad, out, ldc,
                 act, &handled))
    return false;
  if (handled) return true;
  if (fp32_math(Fp32Use::Conv) == Fp32Math::BF16X3)
    return conv_tc<true>(c, x, N, H, W, Cs, coff, Cg, w, ldw, bias, KH, KW, Cout_g, stride, pad, out,
                         ldc, act);
  return conv_tc<false>(c, x, N, H, W, Cs, coff, Cg, w, ldw, bias, KH, KW, Cout_g, stride, pad, out,
                        ldc, act);
}

int conv_route(int H, int W, int Cin, int KH, int KW, int Cout, int stride, int pad, int groups) {
  if (groups > 1) {
    if (groups == Cin && groups == Cout) return kRouteDepthwise;
    if (Cin / groups <= 64 && Cout / groups <= 128) return kRouteGroupedDirect;
    return kRouteGroupedSplit;
  }
  if (KH == 1 && KW == 1) return kRoute1x1;
  if (KH == 3 && KW == 3 && stride == 1 && pad == 1 && H >= 3 && W >= 3 && Cin >= 4 && Cout >= 4)
    return (H >= 112 && W >= 112 && Cin >= 64 && Cout >= 64) ? kRouteWino43 : kRouteWino23;
  return kRouteIm2col;
}

// conv2d_impl on device pointers; weights in the reference layouts.
bool conv2d_dev(Call& c, const float* x, int N, int H, int W, int Cin, const float* w,
                const float* bias, int KH, int KW, int Cout, int stride, int pad, int groups,
                float* out, int act) {
  const int route = conv_route(H, W, Cin, KH, KW, Cout, stride, pad, groups);
  switch (route) {
    case kRouteDepthwise:
      return dw_dev(c, x, N, H, W, Cin, w, bias, KH, KW, stride, pad, out, act);
    case kRouteGroupedDirect:
      return group_dev(c, x, N, H, W, Cin, w, bias, KH, KW, Cout, stride, pad, groups, out, act);
    case kRouteGroupedSplit: {
      const int Cin_p = Cin / groups, Cout_p = Cout / groups;
      for (int g = 0; g < groups; ++g) {
        const float* wg = w + (size_t)g * Cout_p * KH * KW * Cin_p;
        if (!conv_f32_dev(c, x, N, H, W, Cin, g * Cin_p, Cin_p, wg, Cout_p,
                          bias ? bias + (size_t)g * Cout_p : nullptr, KH, KW, Cout_p, stride, pad,
                          out + (size_t)g * Cout_p, Cout, act))
          return false;
      }
      return true;
    }
    default:
      return conv_f32_dev(c, x, N, H, W, Cin, 0, Cin, w, Cout, bias, KH, KW, Cout, stride, pad, out,
                          Cout, act);
  }
}

size_t conv_weight_elems(int Cin, int KH, int KW, int Cout, int groups) {
  if (groups > 1 && groups == Cin && groups == Cout) return (size_t)Cin * KH * KW;
  if (groups < 1) groups = 1;
  return (size_t)KH * KW * (Cin / groups) * Cout;
}

}  // namespace acf

using namespace acf;

static void conv_api(const char* name, const float* input, int N, int H, int W, int Cin,
                     const float* weight, const float* bias, int KH, int KW, int Cout, int stride,
                     int pad, int groups, float* output, int act) {
  if (!input || !weight || !output || N <= 0 || KH <= 0 || KW <= 0 || stride <= 0 || Cin <= 0 ||
      Cout <= 0)
    return;
  if (groups < 1) groups = 1;
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return;
  Call c(name);
  if (!c.ok()) return;
  const float* dx = (const float*)c.in(input, (size_t)N * H * W * Cin * 4);
  const float* dw =
      (const float*)c.in(weight, conv_weight_elems(Cin, KH, KW, Cout, groups) * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * OH * OW * Cout * 4);
  if (!c.ok()) return;
  conv2d_dev(c, dx, N, H, W, Cin, dw, db, KH, KW, Cout, stride, pad, groups, dout, act);
  c.finish();
}

extern "C" void acfun_conv2d(const float* input, int N, int H, int W, int Cin, const float* weight,
                             const float* bias, int KH, int KW, int Cout, int stride, int pad,
                             float* output) {
  conv_api("acfun_conv2d", input, N, H, W, Cin, weight, bias, KH, KW, Cout, stride, pad, 1, output,
           0);
}

extern "C" void acfun_conv2d_relu(const float* input, int N, int H, int W, int Cin,
                                  const float* weight, const float* bias, int KH, int KW, int Cout,
                                  int stride, int pad, float* output) {
  conv_api("acfun_conv2d_relu", input, N, H, W, Cin, weight, bias, KH, KW, Cout, stride, pad, 1,
           output, 1);
}

extern "C" void acfun_conv2d_g(const float* input, int N, int H, int W, int Cin,
                               const float* weight, const float* bias, int KH, int KW, int Cout,
                               int stride, int pad, int groups, float* output, int act) {
  conv_api("acfun_conv2d_g", input, N, H, W, Cin, weight, bias, KH, KW, Cout, stride, pad,
           groups > 1 ? groups : 1, output, act);
}

// internal.h:45-60 — the reference's Winograd entry points (3x3, s1, p1); here the same
// implicit-GEMM convolution.
static void wino_api(const char* name, const float* input, int N, int H, int W, int Cin,
                     const float* weight, const float* bias, int Cout, float* output, int act) {
  if (!input || !weight || !output || N <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0) return;
  Call c(name);
  if (!c.ok()) return;
  const float* dx = (const float*)c.in(input, (size_t)N * H * W * Cin * 4);
  const float* dw = (const float*)c.in(weight, (size_t)9 * Cin * Cout * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * H * W * Cout * 4);
  if (!c.ok()) return;
  conv_f32_dev(c, dx, N, H, W, Cin, 0, Cin, dw, Cout, db, 3, 3, Cout, 1, 1, dout, Cout, act);
  c.finish();
}

extern "C" void acfun_winograd_conv3x3(const float* input, int N, int H, int W, int Cin,
                                       const float* weight, const float* bias, int Cout,
                                       float* output, int act) {
  wino_api("acfun_winograd_conv3x3", input, N, H, W, Cin, weight, bias, Cout, output, act);
}

extern "C" void acfun_winograd43_conv3x3(const float* input, int N, int H, int W, int Cin,
                                         const float* weight, const float* bias, int Cout,
                                         float* output, int act) {
  wino_api("acfun_winograd43_conv3x3", input, N, H, W, Cin, weight, bias, Cout, output, act);
}

// acfun.h:92-97 (layers.cpp:19-36): FC = GEMM + bias (+ ReLU), fused into the drain.
static void fc_api(const char* name, const float* input, int N, int Cin, const float* weight,
                   const float* bias, int Cout, float* output, int act) {
  if (!input || !weight || !output || N <= 0 || Cin <= 0 || Cout <= 0) return;
  Call c(name);
  if (!c.ok()) return;
  const float* dx = (const float*)c.in(input, (size_t)N * Cin * 4);
  const float* dw = (const float*)c.in(weight, (size_t)Cin * Cout * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)Cout * 4) : nullptr;
  float* dout = (float*)c.out(output, (size_t)N * Cout * 4);
  if (!c.ok()) return;
  gemm_f32(c, dx, Cin, dw, Cout, N, Cout, Cin, dout, Cout, db, act, Fp32Use::Conv);
  c.finish();
}

extern "C" void acfun_fc(const float* input, int N, int Cin, const float* weight,
                         const float* bias, int Cout, float* output) {
  fc_api("acfun_fc", input, N, Cin, weight, bias, Cout, output, 0);
}

extern "C" void acfun_fc_relu(const float* input, int N, int Cin, const float* weight,
                              const float* bias, int Cout, float* output) {
  fc_api("acfun_fc_relu", input, N, Cin, weight, bias, Cout, output, 1);
}
