// dw_tma.cu — depthwise 3x3, stride 1, pad 1 convolution (the reference's dw_conv3x3 route,
// dw_avx512.cpp:20-74) fed by TMA, for NHWC maps whose tiles fit one wave of CTAs.
//
// A tile is (image n, strip of R output rows, strip of WT output columns, group of CG channels:
// all of them when C <= 256, so each box row is one contiguous run of pixels).  One 4-D TMA box
// brings its whole input halo -- R + 2 rows x (WT + 2) columns x CG channels, zero-filled past
// the image border -- into shared memory (two buffers: a CTA with more than one tile has the next
// box in flight while it computes), with no register spent on the copy.  A CTA walks a
// contiguous range of tiles.  Compute thread = 4 channels x QW output columns, walking the R + 2
// input rows with three rolling accumulator rows; per output the arithmetic is k_dw3_roll's (the
// bias, then the in-image taps in (kh, kw) order as fp32 fma, then ReLU), so the two kernels give
// the same bits.  Measured (same-process A/B against k_dw3_roll, bit-identical): 1.6-2x faster
// when the tiles fit one wave (9-10 us against 14-18 us per call at 4x112x112x32, 2x17x13x12,
// 1x30x33x40, 3x16x250x8); slower once each CTA walks several tiles (cfg4, 1024 tiles: 34.9
// against 30.7 us), where a CTA's compute warps are too few to hide their own latency -- so the
// dispatch takes this kernel only for single-wave grids.  Every wait is bounded (ptx.cuh); on
// expiry the error word is flagged and the CTA drains its copies and leaves.
#include <algorithm>

#include "gemm.cuh"
#include "numerics.cuh"
#include "ops.cuh"

namespace acf {
namespace dwt {
constexpr int R = 7;         // output rows per tile
constexpr int MAX_SMEM = 227 * 1024;
constexpr int MAX_THREADS = 384;  // producer warp + compute warps
constexpr int QW = 2;             // output columns per compute thread (4 measured slower)
}  // namespace dwt

struct DwtArgs {
  int N, H, W, C, CG, WT, act;
  int ngrp, nstrip, ncs, tiles;  // C / CG, ceil(H / R), ceil(W / WT), N * nstrip * ncs * ngrp
  int ncomp;                     // compute threads: (CG / 4) * (WT / QW)
  uint32_t box_bytes;
  const float* w;                // [C][9]
  const float* bias;             // [C] or null
  float* out;                    // NHWC, H x W
};

// One input row of the rolling window: loads the thread's QW + 2 columns (only in-image ones, so
// every read stays inside the box row), starts a2 from the bias and folds the row into a2 / a1 /
// a0 as taps kh = 0 / 1 / 2 in kw order, skipping out-of-image taps (k_dw3_roll's order).
template <int QW>
__device__ __forceinline__ void dwt_row(const float* boxrow, int CG, unsigned cok, bool row_in,
                                        const float4 (&wv)[9], float4 b4, float4 (&a0)[QW],
                                        float4 (&a1)[QW], float4 (&a2)[QW]) {
  float4 xr[QW + 2];
#pragma unroll
  for (int j = 0; j < QW + 2; ++j)
    xr[j] = ((cok >> j) & 1u) ? *reinterpret_cast<const float4*>(boxrow + j * CG) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < QW; ++q) a2[q] = b4;
  if (!row_in) return;  // out-of-image rows contribute nothing
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    float4* acc = kh == 0 ? a2 : (kh == 1 ? a1 : a0);
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const float4 wk = wv[kh * 3 + kw];
#pragma unroll
      for (int q = 0; q < QW; ++q) {
        if (!((cok >> (q + kw)) & 1u)) continue;
        const float4 x = xr[q + kw];
        const float2 lo = nx_ffma2(make_float2(x.x, x.y), make_float2(wk.x, wk.y), make_float2(acc[q].x, acc[q].y));
        const float2 hi = nx_ffma2(make_float2(x.z, x.w), make_float2(wk.z, wk.w), make_float2(acc[q].z, acc[q].w));
        acc[q] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
    }
  }
}

__global__ void __launch_bounds__(dwt::MAX_THREADS, 1)
    k_dw3_tma(const __grid_constant__ CUtensorMap tm, DwtArgs a, unsigned* err) {
  using namespace dwt;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t buf_bytes = (a.box_bytes + 1023u) & ~1023u;
  float* bufs[2] = {reinterpret_cast<float*>(smem), reinterpret_cast<float*>(smem + buf_bytes)};
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * buf_bytes);
  uint64_t* empty = full + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int comp_warps = (a.ncomp + 31) >> 5;
  // this CTA's contiguous tile range
  const int t0 = (int)((long long)a.tiles * blockIdx.x / gridDim.x);
  const int t1 = (int)((long long)a.tiles * (blockIdx.x + 1) / gridDim.x);

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      dev::mbar_init(&full[b], 1);
      dev::mbar_init(&empty[b], comp_warps);
    }
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tm);
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int t = t0; t < t1; ++t, ++issued) {
        const int b = issued & 1;
        const uint32_t ph = (uint32_t)(issued >> 1) & 1u;
        if (*abort_flag || !dev::mbar_wait(&empty[b], ph ^ 1u, err)) {
          *abort_flag = 1;
          break;
        }
        const int g = t % a.ngrp, cs = (t / a.ngrp) % a.ncs, s = (t / (a.ngrp * a.ncs)) % a.nstrip,
                  n = t / (a.ngrp * a.ncs * a.nstrip);
        dev::mbar_arrive_expect_tx(&full[b], a.box_bytes);
        dev::tma_load_4d(bufs[b], &tm, &full[b], g * a.CG, cs * a.WT - 1, s * R - 1, n);
      }
      // every copy must land before the CTA can release its shared memory
      for (int k = issued > 2 ? issued - 2 : 0; k < issued; ++k)
        dev::mbar_wait(&full[k & 1], (uint32_t)(k >> 1) & 1u, nullptr, 200000000ull);
    }
    return;
  }

  // ---------------- compute: thread = 4 channels x QW output columns of the tile
  const int ct = threadIdx.x - 32;
  const int cq4 = a.CG >> 2;
  const bool active = ct < a.ncomp;
  const int cl = active ? (ct % cq4) * 4 : 0;   // channel within the group
  const int oc0 = active ? (ct / cq4) * QW : 0;  // first output column within the tile
  const int rowf = (a.WT + 2) * a.CG;             // floats per box row
  int done = 0;
  for (int t = t0; t < t1; ++t, ++done) {
    const int b = done & 1;
    const uint32_t ph = (uint32_t)(done >> 1) & 1u;
    if (*abort_flag || !dev::mbar_wait(&full[b], ph, err)) {
      *abort_flag = 1;
      break;
    }
    const int g = t % a.ngrp, cs = (t / a.ngrp) % a.ncs, s = (t / (a.ngrp * a.ncs)) % a.nstrip,
              n = t / (a.ngrp * a.ncs * a.nstrip);
    const int oh0 = s * R, oh1 = min(oh0 + R, a.H);
    const int ow0 = cs * a.WT + oc0;  // first output column of this thread
    unsigned cok = 0;                 // input columns ow0 - 1 + j inside the image
#pragma unroll
    for (int j = 0; j < QW + 2; ++j)
      if (ow0 - 1 + j >= 0 && ow0 - 1 + j < a.W) cok |= 1u << j;
    if (active) {
      const int c = g * a.CG + cl;
      float4 wv[9];
#pragma unroll
      for (int k = 0; k < 9; ++k)
        wv[k] = make_float4(__ldg(a.w + (c + 0) * 9 + k), __ldg(a.w + (c + 1) * 9 + k),
                            __ldg(a.w + (c + 2) * 9 + k), __ldg(a.w + (c + 3) * 9 + k));
      const float4 b4 = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float* box = bufs[b] + oc0 * a.CG + cl;  // box column oc0 = input column ow0 - 1
      float* obase = a.out + (size_t)n * a.H * a.W * a.C + c;
      // a0: output row ih - 1 (gets kh = 2, then complete), a1: ih (kh = 1), a2: ih + 1 (kh = 0,
      // starts from the bias) -- k_dw3_roll's rolling window with pad 1
      float4 a0[QW], a1[QW], a2[QW];
      const int nrows = oh1 - oh0 + 2;
#pragma unroll
      for (int rr = 0; rr < R + 2; ++rr) {
        if (rr >= nrows) break;
        const int ih = oh0 - 1 + rr;
        const bool row_in = ih >= 0 && ih < a.H;
        dwt_row<QW>(box + (size_t)rr * rowf, a.CG, cok, row_in, wv, b4, a0, a1, a2);
        const int od = ih - 1;  // complete output row
        if (od >= oh0 && od < oh1) {
          float* orow = obase + (size_t)od * a.W * a.C;
#pragma unroll
          for (int q = 0; q < QW; ++q) {
            if (ow0 + q >= a.W) break;
            float4 v = a0[q];
            if (a.act == 1) {
              v.x = v.x > 0.f ? v.x : 0.f;
              v.y = v.y > 0.f ? v.y : 0.f;
              v.z = v.z > 0.f ? v.z : 0.f;
              v.w = v.w > 0.f ? v.w : 0.f;
            }
            *reinterpret_cast<float4*>(orow + (size_t)(ow0 + q) * a.C) = v;
          }
        }
#pragma unroll
        for (int q = 0; q < QW; ++q) {
          a0[q] = a1[q];
          a1[q] = a2[q];
        }
      }
    }
    __syncwarp();
    if (lane == 0) dev::mbar_arrive(&empty[b]);
  }
}

// Tile shape for a C-channel map of width W: all C channels (the box rows are then whole runs of
// pixels, contiguous in memory) when C <= 256, else the largest channel divisor that fits; the
// column strip WT the widest that keeps two boxes in shared memory and the compute threads in
// one block, preferring a divisor of W.  Returns false if nothing fits.
static bool dwt_shape(int C, int W, int* cg_out, int* wt_out) {
  for (int cg = std::min(C, 256); cg >= 4; cg -= 4) {
    if (C % cg) continue;
    int best = 0;
    for (int wt = dwt::QW; wt <= W + dwt::QW - 1; wt += dwt::QW) {
      const long long box = (long long)(dwt::R + 2) * (wt + 2) * cg * 4;
      const long long smem = 1024 + 2 * ((box + 1023) / 1024 * 1024) + 64;
      const int ncomp = (cg / 4) * (wt / dwt::QW);
      if (smem > dwt::MAX_SMEM || 32 + ((ncomp + 31) / 32) * 32 > dwt::MAX_THREADS || wt > 254) break;
      if (W % wt == 0 || wt >= W) best = wt;  // whole strips
      else if (best == 0 || W % best != 0) best = wt;
    }
    if (best > 0) {
      *cg_out = cg;
      *wt_out = std::min(best, (W + dwt::QW - 1) / dwt::QW * dwt::QW);
      return true;
    }
  }
  return false;
}

bool dw3_tma_ok(const float* in, const float* out, const float* bias, int N, int H, int W, int C,
                int KH, int KW, int stride, int pad, int sm_count) {
  int cg = 0, wt = 0;
  if (!(KH == 3 && KW == 3 && stride == 1 && pad == 1 && C % 4 == 0 && N >= 1 && H >= 1 && W >= 1 &&
        aligned16(in) && aligned16(out) && (!bias || aligned16(bias)) && dwt_shape(C, W, &cg, &wt) &&
        (long long)H * W * C < (1LL << 31)))
    return false;
  const long long tiles = (long long)N * (C / cg) * ((H + dwt::R - 1) / dwt::R) * ((W + wt - 1) / wt);
  return tiles <= sm_count;  // one wave: where it beats k_dw3_roll
}

bool dw3_tma_dev(Call& c, const float* in, int N, int H, int W, int C, const float* w, const float* bias,
                 float* out, int act) {
  DwtArgs a{};
  a.N = N;
  a.H = H;
  a.W = W;
  a.C = C;
  if (!dwt_shape(C, W, &a.CG, &a.WT)) {
    c.fail();
    return false;
  }
  a.act = act;
  a.ngrp = C / a.CG;
  a.nstrip = (H + dwt::R - 1) / dwt::R;
  a.ncs = (W + a.WT - 1) / a.WT;
  const long long tiles = (long long)N * a.ngrp * a.nstrip * a.ncs;
  if (tiles >= (1LL << 31)) {
    set_error(kInvalid, "%s: tensor too large", c.name());
    c.fail();
    return false;
  }
  a.tiles = (int)tiles;
  a.ncomp = (a.CG / 4) * (a.WT / dwt::QW);
  a.box_bytes = (uint32_t)((dwt::R + 2) * (a.WT + 2) * a.CG * 4);
  a.w = w;
  a.bias = bias;
  a.out = out;
  CUtensorMap tm;
  const uint64_t d[4] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)N};
  const uint64_t st[3] = {(uint64_t)C * 4, (uint64_t)W * C * 4, (uint64_t)H * W * C * 4};
  const uint32_t bx[4] = {(uint32_t)a.CG, (uint32_t)(a.WT + 2), (uint32_t)(dwt::R + 2), 1u};
  if (!encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, in, d, st, bx, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    c.fail();
    return false;
  }
  const uint32_t buf_bytes = (a.box_bytes + 1023u) & ~1023u;
  const size_t smem = 1024 + 2 * (size_t)buf_bytes + 64;
  static bool attr_done[64] = {};
  const int dv = current_device();
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(k_dw3_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, dwt::MAX_SMEM))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  const int threads = 32 + ((a.ncomp + 31) / 32) * 32;
  const int grid = std::min(a.tiles, c.sm_count());
  k_dw3_tma<<<grid, threads, smem, c.stream()>>>(tm, a, c.err());
  return c.launched("k_dw3_tma");
}

}  // namespace acf
