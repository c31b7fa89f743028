// conv_i8_pool_tc.cu — small-K int8 convolution fused with the 2x2 / stride-2 max-pool after
// it (the per-image int8 model path's first layer, e.g. VGG conv1: 3x3x3 -> 64 at 224x224), on
// tcgen05 kind::i8 tensor cores.  Same results as k_conv_int8_pool (conv_int8.cu), bit for bit:
// the exact integer correlation of the u8 activations (RNE quantisation with the image's
// inv_s, zero point 128 -- also outside the image, as the reference's u8 im2col pads) with
// the s8 weights, the 2x2 window maximum taken on the int32 sums, then one dequantisation
// ((float)acc*alpha + beta), act, the pool's post-ReLU (conv_int8.cpp:63-148 followed by
// pooling.cpp's max-pool).
//
// A tile is 8 pooled rows x 16 pooled columns of one image: 128 GEMM rows, one per pooled
// pixel, whose 128-byte A row holds the four im2col patches of the pixel's 2x2 window (32 bytes
// each, K = KH*KW*Cin <= 32, zeros past K).  Four MMAs per tile (M=128, N=Cout, K=32) multiply
// patch p by the weights into TMEM columns 64p.., so every window's four sums sit in one TMEM
// lane: the pool is a per-thread maximum, with no exchange between lanes.
//   * A TMA warp brings each tile's fp32 input window (18 x 34 pixels for a 3x3 kernel, rows of
//     the [N][H][W*Cin] view from a 16-byte-aligned start; zero fill outside the image, which
//     quantises to the zero point) into a ring of stages.
//   * Two groups of four converter warps take alternate tiles: a group quantises a window into
//     u8 bytes in shared memory, then each thread builds the A row of one pooled pixel in the
//     no-swizzle K-major core-matrix layout.
//   * One thread issues the four MMAs per tile into one of two 256-column TMEM accumulators;
//     the s8 weights ([Cout][32], same layout) stay resident.
//   * Eight epilogue warps (a TMEM lane quadrant and half of the channels each) take the
//     window maximum per channel, dequantise, and store; they also fold each image's
//     max |stored value| into out_max for the next int8 layer (a running maximum per warp, one
//     atomic when the image changes: a CTA takes a contiguous range of tiles).
// Every wait is bounded (ptx.cuh); on expiry the kernel flags the error word and drains.
#include <algorithm>

#include "conv.cuh"
#include "gemm.cuh"

namespace acf {
namespace i8p {
constexpr int TPR = 8, TPC = 16;             // pooled rows / columns of a tile (128 pixels)
constexpr int CR = 2 * TPR, CC = 2 * TPC;    // conv rows / columns of a tile
constexpr int MAXK = 32;                     // bytes of one patch
constexpr int MAXKS = 3;                     // kernel extent (KH, KW <= 3)
constexpr int IR = CR + MAXKS - 1, IC = CC + MAXKS - 1;  // input window (stride 1)
constexpr int MAXCIN = 4;
constexpr int STAGE_IN = IR * IC * MAXCIN + 16;  // the quantised window (rows padded to 4 bytes)
constexpr int MAXBXW = 144;                  // floats of one TMA window row (>= IC*Cin + 3)
constexpr int RAW_BYTES = 10368;             // >= IR * MAXBXW * 4, a multiple of 128
constexpr int NIN = 6;                       // input-window stages
constexpr int NA = 3;                        // A stages
constexpr int NBUF = 2;                      // TMEM accumulators (4 x 64 columns each)
constexpr int A_BYTES = 128 * 4 * MAXK;      // 16 KB: 128 rows x 4 patches
constexpr int CONV_GROUPS = 2;               // converter groups of 4 warps, alternate tiles
constexpr int CONV_WARPS = 4 * CONV_GROUPS, EPI_WARPS = 8;
constexpr int TMA_WARP = 1 + CONV_WARPS + EPI_WARPS;
constexpr int THREADS = 32 * (TMA_WARP + 1);
// barriers: b_ready, a_full[NA], a_empty[NA], t_full[NBUF], t_empty[NBUF], in_full[NIN],
// in_empty[NIN], drain
constexpr int BAR_BYTES = (1 + 2 * NA + 2 * NBUF + 2 * NIN + 1) * 8;
constexpr int SMEM = 1024 + NA * A_BYTES + NIN * RAW_BYTES + 64 * MAXK +
                     2 * CONV_GROUPS * STAGE_IN + BAR_BYTES + 16;
static_assert(IR * MAXBXW * 4 <= RAW_BYTES && RAW_BYTES % 128 == 0, "window stage");
static_assert(A_BYTES % 1024 == 0 && STAGE_IN % 16 == 0, "alignment");
}  // namespace i8p

struct I8PoolArgs {
  int H, W, Cin, KH, KW, pad, K;
  const int8_t* wq;        // [K][Cout] s8
  int Cout;
  const float* ab;         // [N][2][Cout]: alpha, beta of image n
  const float* img_inv;    // [N] 127 / max|x|
  const int* img_zero;     // [N]
  float* out;              // [N][PH][PW][Cout]
  int PH, PW;
  int act, post_relu;
  unsigned* out_max;       // [N] or null
  int segs, prb;           // tiles per pooled-row block, pooled-row blocks per image
  int num_tiles;
  int bxw;                 // floats of a TMA window row
};

// Core-matrix (no swizzle) K-major offset of 16-byte chunk k16 (0..7) of row m: 8-row groups
// 1024 bytes apart, chunks of a group 128 bytes apart.
__device__ __forceinline__ int i8p_off(int m, int k16) { return (m >> 3) * 1024 + k16 * 128 + (m & 7) * 16; }

__device__ __forceinline__ uint8_t i8p_quant(float xv, float inv_s) {
  // RNE of x*inv_s + 128, clamped (quant_fast<0>'s rounding, conv_int8.cu)
  const float t = __fmul_rn(xv, inv_s);
  if (!(fabsf(t) < 2147483648.0f)) return 0u;
  int v = __float_as_int(__fadd_rn(fminf(fmaxf(t, -256.0f), 256.0f), 12582912.0f)) - 0x4B400000;
  v += 128;
  return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
}

template <bool ACT, bool POST>
__global__ void __launch_bounds__(i8p::THREADS, 1)
    k_conv_i8_pool_tc(const __grid_constant__ CUtensorMap tmX, I8PoolArgs a, unsigned* err) {
  using namespace i8p;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sRaw = sA + NA * A_BYTES;
  uint8_t* sB = sRaw + NIN * RAW_BYTES;
  uint8_t* sIn = sB + 64 * MAXK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sIn + 2 * CONV_GROUPS * STAGE_IN);
  uint64_t* b_ready = bars;
  uint64_t* a_full = bars + 1;
  uint64_t* a_empty = a_full + NA;
  uint64_t* t_full = a_empty + NA;
  uint64_t* t_empty = t_full + NBUF;
  uint64_t* in_full = t_empty + NBUF;
  uint64_t* in_empty = in_full + NIN;
  uint64_t* drain = in_empty + NIN;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    dev::mbar_init(b_ready, CONV_WARPS);
    for (int s = 0; s < NA; ++s) {
      dev::mbar_init(&a_full[s], 4);  // the four warps of the group that built the stage
      dev::mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&t_full[b], 1);
      dev::mbar_init(&t_empty[b], EPI_WARPS);
    }
    for (int s = 0; s < NIN; ++s) {
      dev::mbar_init(&in_full[s], 1);
      dev::mbar_init(&in_empty[s], 1);
    }
    dev::mbar_init(drain, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmX);
  }
  if (warp == 0) {
    dev::tmem_alloc(tmem_slot, NBUF * 256);
    dev::tmem_relinquish();
  }
  // the prologue above may overlap the per-image scalar kernel; nothing it produced is read before this
  dev::grid_dep_wait();
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tiles_img = a.prb * a.segs;
  // a contiguous range of tiles per CTA (few image changes, neighbouring windows in L2)
  const int t_begin = (int)((long long)a.num_tiles * blockIdx.x / gridDim.x);
  const int t_end = (int)((long long)a.num_tiles * (blockIdx.x + 1) / gridDim.x);

  if (warp == 0) {
    // ---------------- MMA issuer: four M=128, N=Cout, K=32 MMAs per tile (one per patch)
    if (lane == 0) {
      const uint32_t idesc = dev::umma_idesc(2u, 0u, 1u, 0u, 0u, 128u, (uint32_t)a.Cout);
      const uint64_t ad0 = dev::umma_sdesc(dev::smem_u32(sA), 128, 1024, 0u);
      const uint64_t bd = dev::umma_sdesc(dev::smem_u32(sB), 128, 256, 0u);
      bool ok = dev::mbar_wait(b_ready, 0, err);
      dev::tc_fence_after();
      uint32_t local = 0;
      for (int t = t_begin; t < t_end && ok; ++t, ++local) {
        const uint32_t s = local % NA, sph = (local / NA) & 1;
        const uint32_t buf = local % NBUF, use = local / NBUF;
        if (*abort_flag || !dev::mbar_wait(&t_empty[buf], (use & 1) ^ 1, err) ||
            !dev::mbar_wait(&a_full[s], sph, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint64_t as = ad0 + (uint64_t)((s * A_BYTES) >> 4);
#pragma unroll
        for (int p = 0; p < 4; ++p)  // patch p: 16-byte chunks 2p, 2p+1
          dev::umma<dev::MmaKind::I8>(tmem + buf * 256 + 64 * p, as + (uint64_t)((2 * p * 128) >> 4), bd,
                                      idesc, 0u);
        dev::umma_commit(&a_empty[s]);
        dev::umma_commit(&t_full[buf]);
      }
      if (!ok) {
        *abort_flag = 1;
        dev::umma_commit(drain);
        dev::mbar_wait(drain, 0, nullptr, 200000000ull);
        for (int b = 0; b < NBUF; ++b) dev::mbar_arrive(&t_full[b]);
      }
    }
  } else if (warp <= CONV_WARPS) {
    // ---------------- converters: group g (4 warps) takes the range's tiles g, g+2, ...
    const int cw = warp - 1, g = cw >> 2, ct = threadIdx.x - 32 - 128 * g;  // ct: A row (pooled pixel)
    // resident weights: B[j][k] = wq[k][j] (zero for k >= K and j >= Cout); [64][32] core matrices
    {
      // all of a thread's weight loads in flight at once (one load latency, not eight)
      constexpr int WU = 64 * MAXK / (32 * CONV_WARPS);
      int8_t v[WU];
#pragma unroll
      for (int u = 0; u < WU; ++u) {
        const int e = threadIdx.x - 32 + u * 32 * CONV_WARPS, j = e / MAXK, k = e % MAXK;
        v[u] = (k < a.K && j < a.Cout) ? a.wq[k * a.Cout + j] : (int8_t)0;
      }
#pragma unroll
      for (int u = 0; u < WU; ++u) {
        const int e = threadIdx.x - 32 + u * 32 * CONV_WARPS, j = e / MAXK, k = e % MAXK;
        sB[(j >> 3) * 256 + (k >> 4) * 128 + (j & 7) * 16 + (k & 15)] = (uint8_t)v[u];
      }
    }
    dev::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) dev::mbar_arrive(b_ready);
    const int ir = CR + a.KH - 1, ic = CC + a.KW - 1, rowb = ic * a.Cin;
    const int rp = (rowb + 3) & ~3, wpr = rp >> 2, nw = ir * wpr;  // byte-window row pitch, words
    // this thread's pooled pixel (pi, pj) of the tile; byte k = (kh*KW + kw)*Cin + ci of patch
    // p = 2*dy + dx is window byte base + pofs[p] + kh*rp + kw*Cin + ci
    const int pi = ct / TPC, pj = ct % TPC;
    const bool k333 = a.KH == 3 && a.KW == 3 && a.Cin == 3;  // 9-byte kernel rows: word gathers
    const int base = 2 * pi * rp + 2 * pj * a.Cin;
    const int pofs[4] = {0, a.Cin, rp, rp + a.Cin};
    // the window words this thread quantises: e = ct + 128*j -> row e / wpr, word e % wpr
    const int q_r0 = ct / wpr, q_c0 = ct - (ct / wpr) * wpr, q_sr = 128 / wpr, q_sc = 128 % wpr;
    uint32_t local = g, lt = 0;
    for (int t = t_begin + g; t < t_end; t += CONV_GROUPS, local += CONV_GROUPS, ++lt) {
      const int n = t / tiles_img, rem = t - n * tiles_img;
      const int sg = rem - (rem / a.segs) * a.segs;
      const int x0 = (2 * TPC * sg - a.pad) * a.Cin;   // window column 0, in floats
      const int off = x0 - (x0 & ~3);                 // the TMA box starts at x0 & ~3
      const uint32_t si = local % NIN, iph = (local / NIN) & 1;
      const uint32_t s = local % NA, sph = (local / NA) & 1;
      // the window and a free A stage; every thread of the group agrees before going on (one
      // that gave up must not leave the others waiting at the group's named barrier)
      const uint32_t mine = (!*abort_flag && dev::mbar_wait(&in_full[si], iph, err) &&
                             dev::mbar_wait(&a_empty[s], sph ^ 1, err)) ? 1u : 0u;
      uint8_t* st = sIn + (2 * g + (lt & 1)) * STAGE_IN;
      if (mine) {
        const float inv_s = a.img_inv[n];
        const float* raw = reinterpret_cast<const float*>(sRaw + si * RAW_BYTES) + off;
        // quantised window [ir][rp], four values per word; zero fill outside the image
        // quantises to 128 (bytes past rowb in a row are never used)
        int rr = q_r0, cc = q_c0;
        for (int e = ct; e < nw; e += 128) {
          const float* src = raw + rr * a.bxw + 4 * cc;
          const uint32_t wv = (uint32_t)i8p_quant(src[0], inv_s) | ((uint32_t)i8p_quant(src[1], inv_s) << 8) |
                              ((uint32_t)i8p_quant(src[2], inv_s) << 16) |
                              ((uint32_t)i8p_quant(src[3], inv_s) << 24);
          reinterpret_cast<uint32_t*>(st)[e] = wv;
          rr += q_sr;
          cc += q_sc;
          if (cc >= wpr) {
            cc -= wpr;
            ++rr;
          }
        }
      }
      uint32_t all;
      asm volatile(
          "{\n\t.reg .pred q, r;\n\tsetp.ne.u32 q, %1, 0;\n\t"
          "barrier.cta.red.and.pred r, %2, 128, q;\n\tselp.u32 %0, 1, 0, r;\n\t}"
          : "=r"(all)
          : "r"(mine), "r"(1 + g)
          : "memory");
      if (!all) {
        *abort_flag = 1;
        break;
      }
      if (ct == 0) dev::mbar_arrive(&in_empty[si]);  // the fp32 window has been read
      uint8_t* dstA = sA + s * A_BYTES;
      if (k333) {
        // 3x3x3: each kernel row's 9 bytes come from three aligned words and two funnel shifts
        const uint32_t* stw = reinterpret_cast<const uint32_t*>(st);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint32_t r[3][3];
#pragma unroll
          for (int kh = 0; kh < 3; ++kh) {
            const int o = base + pofs[p] + kh * rp;
            const int wi = o >> 2;
            const uint32_t sh = (uint32_t)(o & 3) * 8u;
            const uint32_t w0 = stw[wi], w1 = stw[wi + 1], w2 = stw[wi + 2];
            r[kh][0] = __funnelshift_r(w0, w1, sh);
            r[kh][1] = __funnelshift_r(w1, w2, sh);
            r[kh][2] = (w2 >> sh) & 0xFFu;
          }
          // bytes 0-8 | 9-17 | 18-26 of the patch, zeros after
          const uint32_t W0 = r[0][0], W1 = r[0][1];
          const uint32_t W2 = r[0][2] | (r[1][0] << 8);
          const uint32_t W3 = (r[1][0] >> 24) | (r[1][1] << 8);
          const uint32_t W4 = (r[1][1] >> 24) | (r[1][2] << 8) | (r[2][0] << 16);
          const uint32_t W5 = (r[2][0] >> 16) | (r[2][1] << 16);
          const uint32_t W6 = (r[2][1] >> 16) | (r[2][2] << 16);
          *reinterpret_cast<uint4*>(dstA + i8p_off(ct, 2 * p)) = make_uint4(W0, W1, W2, W3);
          *reinterpret_cast<uint4*>(dstA + i8p_off(ct, 2 * p + 1)) = make_uint4(W4, W5, W6, 0u);
        }
      } else {
        int offs[MAXK];
#pragma unroll
        for (int k = 0; k < MAXK; ++k) {
          const int kk = k < a.K ? k : 0;
          const int kh = kk / (a.KW * a.Cin), r2 = kk - kh * a.KW * a.Cin;
          offs[k] = base + kh * rp + r2;
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint8_t* src = st + pofs[p];
          uint32_t w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
          for (int k = 0; k < MAXK; ++k)
            if (k < a.K) w[k >> 2] |= (uint32_t)src[offs[k]] << (8 * (k & 3));
          *reinterpret_cast<uint4*>(dstA + i8p_off(ct, 2 * p)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(dstA + i8p_off(ct, 2 * p + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      dev::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&a_full[s]);
    }
  } else if (warp == TMA_WARP) {
    // ---------------- TMA producer: one fp32 input window per tile
    if (lane == 0) {
      const uint32_t wbytes = (uint32_t)((CR + a.KH - 1) * a.bxw * 4);
      uint32_t local = 0;
      for (int t = t_begin; t < t_end; ++t, ++local) {
        const int n = t / tiles_img, rem = t - n * tiles_img;
        const int pr = rem / a.segs, sg = rem - pr * a.segs;
        const int r0 = 2 * TPR * pr - a.pad, xs = ((2 * TPC * sg - a.pad) * a.Cin) & ~3;
        const uint32_t si = local % NIN, iph = (local / NIN) & 1;
        if (*abort_flag || !dev::mbar_wait(&in_empty[si], iph ^ 1, err)) {
          *abort_flag = 1;
          break;
        }
        dev::mbar_arrive_expect_tx(&in_full[si], wbytes);
        dev::tma_load_3d(sRaw + si * RAW_BYTES, &tmX, &in_full[si], xs, r0, n);
      }
      // the copies in flight must land before the CTA releases its shared memory
      for (uint32_t k = local > (uint32_t)NIN ? local - NIN : 0; k < local; ++k)
        dev::mbar_wait(&in_full[k % NIN], (k / NIN) & 1, nullptr, 200000000ull);
    }
  } else {
    // ---------------- epilogue: window maximum, dequantisation, pooled stores
    // warp (q, h): TMEM lane quadrant q (pooled pixels 32q..32q+31), channels 32h..32h+31
    const int ew = warp - 1 - CONV_WARPS;  // 0..7
    const int q = warp & 3, h = ew >> 2;
    // out_max: a running maximum per lane while the tiles stay in one image, then one atomic
    // per warp
    float am = 0.0f;
    int n_run = -1;
    auto flush = [&]() {
      if (!a.out_max || n_run < 0) return;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, am, o);
        am = (am < u) ? u : am;
      }
      if (lane == 0 && am > 0.0f) atomicMax(&a.out_max[n_run], __float_as_uint(am));
      am = 0.0f;
    };
    const int m = q * 32 + lane;
    const int pi = m / TPC, pj = m % TPC;
    // per image: the all-zero flag and whether any of this warp's channels has a dequantisation
    // that is not increasing (alpha <= 0 with beta == +-0 and no ReLU: the zeros' signs follow
    // the sums', so such a channel pools its four dequantised values one by one)
    bool zero = false, slow_any = false;
    uint32_t local = 0;
    for (int t = t_begin; t < t_end; ++t, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      const bool ok = dev::mbar_wait(&t_full[buf], use & 1, err);
      dev::tc_fence_after();
      if (!ok || *abort_flag) break;
      const int n = t / tiles_img, rem = t - n * tiles_img;
      const float* abn = a.ab + (size_t)n * 2 * a.Cout;
      if (n != n_run) {  // warp-uniform
        flush();
        n_run = n;
        zero = a.img_zero[n] != 0;
        bool sl = false;
        if (!ACT && 32 * h + lane < a.Cout)
          sl = !(abn[32 * h + lane] > 0.0f) && abn[a.Cout + 32 * h + lane] == 0.0f;
        slow_any = __any_sync(0xffffffffu, sl);
      }
      const int pr = rem / a.segs, sg = rem - pr * a.segs;
      const int ph = TPR * pr + pi, pw = TPC * sg + pj;
      const bool store = ph < a.PH && pw < a.PW;
      float* dst = a.out + (((size_t)n * a.PH + ph) * a.PW + pw) * a.Cout;
      const uint32_t tl = tmem + buf * 256 + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c0 = 32 * h; c0 < 32 * h + 32; c0 += 8) {
        if (c0 >= a.Cout) break;  // warp-uniform
        uint32_t v0[8], v1[8], v2[8], v3[8];
        dev::tmem_ld8(tl + c0, v0);
        dev::tmem_ld8(tl + 64 + c0, v1);
        dev::tmem_ld8(tl + 128 + c0, v2);
        dev::tmem_ld8(tl + 192 + c0, v3);
        dev::tmem_ld_wait();
        float y[8];
        if (zero) {
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = 0.0f;
        } else {
          float al[8], be[8];
          {
            const float4 a0 = __ldg(reinterpret_cast<const float4*>(abn + c0));
            const float4 a1 = __ldg(reinterpret_cast<const float4*>(abn + c0 + 4));
            const float4 b0 = __ldg(reinterpret_cast<const float4*>(abn + a.Cout + c0));
            const float4 b1 = __ldg(reinterpret_cast<const float4*>(abn + a.Cout + c0 + 4));
            al[0] = a0.x; al[1] = a0.y; al[2] = a0.z; al[3] = a0.w;
            al[4] = a1.x; al[5] = a1.y; al[6] = a1.z; al[7] = a1.w;
            be[0] = b0.x; be[1] = b0.y; be[2] = b0.z; be[3] = b0.w;
            be[4] = b1.x; be[5] = b1.y; be[6] = b1.z; be[7] = b1.w;
          }
          if (!slow_any) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int mx = max(max((int)v0[j], (int)v1[j]), max((int)v2[j], (int)v3[j]));
              float r = __fadd_rn(__fmul_rn(__int2float_rn(mx), al[j]), be[j]);
              if (ACT) r = r > 0.0f ? r : 0.0f;
              y[j] = r;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float r;
              if (ACT || al[j] > 0.0f || be[j] != 0.0f) {
                const int mx = max(max((int)v0[j], (int)v1[j]), max((int)v2[j], (int)v3[j]));
                r = __fadd_rn(__fmul_rn(__int2float_rn(mx), al[j]), be[j]);
                if (ACT) r = r > 0.0f ? r : 0.0f;
              } else {
                const int vv[4] = {(int)v0[j], (int)v1[j], (int)v2[j], (int)v3[j]};
                r = -1e30f;
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                  const float uu = __fadd_rn(__fmul_rn(__int2float_rn(vv[pp]), al[j]), be[j]);
                  r = r > uu ? r : uu;
                }
              }
              y[j] = r;
            }
          }
        }
        if (POST) {
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = y[j] > 0.0f ? y[j] : 0.0f;
        }
        if (store) {
#pragma unroll
          for (int j = 0; j < 8; ++j) amax_acc(am, y[j]);
          if ((reinterpret_cast<uintptr_t>(dst + c0) & 31) == 0) {
            dev::st_global_v8(dst + c0, reinterpret_cast<const uint32_t*>(y));  // a whole sector
          } else {
            *reinterpret_cast<float4*>(dst + c0) = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4*>(dst + c0 + 4) = make_float4(y[4], y[5], y[6], y[7]);
          }
        }
      }
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&t_empty[buf]);
    }
    flush();
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, NBUF * 256);
  }
}

static int i8p_bxw(int Cin, int KW) { return ((i8p::CC + KW - 1) * Cin + 3 + 3) & ~3; }

bool conv_i8_pool_tc_ok(const float* x, int W, int Cin, int KH, int KW, int Cout, int stride, int PW) {
  return stride == 1 && Cin >= 1 && Cin <= i8p::MAXCIN && KH >= 1 && KW >= 1 && KH <= i8p::MAXKS &&
         KW <= i8p::MAXKS && KH * KW * Cin <= i8p::MAXK && Cout >= 16 && Cout <= 64 && Cout % 16 == 0 &&
         PW >= 1 && (long long)W * Cin % 4 == 0 && aligned16(x) && i8p_bxw(Cin, KW) <= i8p::MAXBXW;
}

bool conv_i8_pool_tc_dev(Call& c, const float* x, int N, int H, int W, int Cin, const int8_t* wq,
                         int KH, int KW, int Cout, int pad, int PH, int PW, const float* ab,
                         const float* img_inv, const int* img_zero, float* out, int act,
                         int post_relu, unsigned* out_max) {
  I8PoolArgs a;
  a.H = H;
  a.W = W;
  a.Cin = Cin;
  a.KH = KH;
  a.KW = KW;
  a.pad = pad;
  a.K = KH * KW * Cin;
  a.wq = wq;
  a.Cout = Cout;
  a.ab = ab;
  a.img_inv = img_inv;
  a.img_zero = img_zero;
  a.out = out;
  a.PH = PH;
  a.PW = PW;
  a.act = act;
  a.post_relu = post_relu;
  a.out_max = out_max;
  a.segs = (PW + i8p::TPC - 1) / i8p::TPC;
  a.prb = (PH + i8p::TPR - 1) / i8p::TPR;
  const long long tiles = (long long)N * a.prb * a.segs;
  if (tiles >= (1LL << 31)) {
    set_error(kInvalid, "%s: too many tiles", c.name());
    c.fail();
    return false;
  }
  a.num_tiles = (int)tiles;
  a.bxw = i8p_bxw(Cin, KW);
  CUtensorMap tx;
  {
    // [N][H][W*Cin] fp32 view; a box is bxw floats x (CR + KH - 1) rows of one image
    const uint64_t d[3] = {(uint64_t)W * Cin, (uint64_t)H, (uint64_t)N};
    const uint64_t st[2] = {(uint64_t)W * Cin * 4, (uint64_t)H * W * Cin * 4};
    const uint32_t bx[3] = {(uint32_t)a.bxw, (uint32_t)(i8p::CR + KH - 1), 1u};
    if (!encode_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, x, d, st, bx, CU_TENSOR_MAP_SWIZZLE_NONE)) {
      c.fail();
      return false;
    }
  }
  auto kern = act ? (post_relu ? k_conv_i8_pool_tc<true, true> : k_conv_i8_pool_tc<true, false>)
                 : (post_relu ? k_conv_i8_pool_tc<false, true> : k_conv_i8_pool_tc<false, false>);
  static bool attr_done[4][64] = {};
  const int dv = current_device(), kv = (act ? 2 : 0) + (post_relu ? 1 : 0);
  if (dv >= 0 && dv < 64 && !attr_done[kv][dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, i8p::SMEM))) {
      c.fail();
      return false;
    }
    attr_done[kv][dv] = true;
  }
  const int grid = (int)std::min<long long>(tiles, c.sm_count());
  if (!ACF_CUDA_OK(launch_pdl(kern, dim3(grid), dim3(i8p::THREADS), (size_t)i8p::SMEM, c.stream(), tx, a,
                              c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("k_conv_i8_pool_tc");
}

}  // namespace acf
