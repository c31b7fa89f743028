// conv_halo.cu — narrow stride-1 fp32 convolutions (at most 64 input and 64 output channels,
// KH*KW <= 9: the reference's Winograd F(2,3) / F(4,3) routes at the cfg3 shapes,
// winograd_avx512.cpp:186-250 and winograd43_avx512.cpp:218-280) as one persistent tcgen05
// kernel in 3xBF16, with no preparation pass over the activation.
//
// GEMM view: row r = a pixel of the zero-padded input grid (N x Hp x Wp, NHWC), 64 channels
// per row; output pixel (oh, ow) of image n is row r = (n*Hp + oh)*Wp + ow, and tap (kh, kw)
// reads row r + kh*Wp + kw.  A tile is 128 consecutive rows x 64 output channels.
//   * The split weights of every tap ([2][taps][64 channels][64 columns] bf16 hi / lo, 16 KB a
//     tap) are loaded by TMA once per CTA and stay resident in shared memory.
//   * For each kernel row kh, converter warps read the tile's 128 + KW - 1 input rows
//     (a "slab") straight from the fp32 NHWC tensor -- zero outside the image and past the
//     channels -- split them into bf16 hi / lo and store them in the 128-byte-swizzled
//     K-major layout the tensor core reads; two slab buffers let the next slab be converted
//     while the MMAs consume the current one.
//   * One thread issues, per slab, the MMAs of its KW taps: the A operand of tap kw is the
//     slab's rows kw .. kw + 127, a descriptor whose start is shifted by kw rows, so each
//     input row is converted and staged once per kernel row instead of once per tap.  3xBF16
//     in two MMAs per K-step: hi * [hi | lo] as one 128-column operand (the two weight copies
//     are the two 64-column chunks of an MN-major B whose chunk stride is one copy) and
//     lo * hi, into three fp32 partial accumulators in TMEM (two buffers of 256 columns).
//   * Epilogue warps drain TMEM, sum the partials ((lo*hi + hi*lo) + hi*hi), add the bias,
//     apply ReLU and store the rows that land on output pixels.
// Every wait is bounded (ptx.cuh); on expiry the kernel flags the error word and drains.
#include "conv.cuh"
#include "gemm.cuh"

namespace acf {
namespace halo {
constexpr int BN = 64;                          // output channels of a tile
constexpr int CP = 64;                          // input channels of a row (zero-padded)
constexpr int MAXTAPS = 9;
constexpr int SLAB_ROWS = 136;                  // >= 128 + KW - 1, a multiple of 8
constexpr int ROWB = 128;                       // bytes of one bf16 row
constexpr int TAPB = CP * ROWB;                 // 8 KB: one tap of one weight copy
constexpr int B_COPY = MAXTAPS * TAPB;
constexpr int B_BYTES = 2 * B_COPY;             // hi + lo weights, resident
constexpr int SLAB_COPY = SLAB_ROWS * ROWB;
constexpr int SLAB = 2 * SLAB_COPY;             // hi + lo
constexpr int NSLAB = 2;
constexpr int NBUF = 2;                         // TMEM buffers of 3 partials (256 columns)
constexpr int CONV_WARPS = 10, EPI_WARPS = 4;
constexpr int CONV_THREADS = 32 * CONV_WARPS;
constexpr int THREADS = 64 + 32 * (CONV_WARPS + EPI_WARPS);
constexpr int UNITS = (SLAB_ROWS * 4 + CONV_THREADS - 1) / CONV_THREADS;  // 16-channel units
// barriers: b_full, slab_full[2], slab_empty[2], t_full[4], t_empty[4], drain
constexpr int BAR_BYTES = 16 * 8;
constexpr int SMEM = 1024 + B_BYTES + NSLAB * SLAB + BAR_BYTES + 16 + BN * 4;
static_assert(SMEM <= 232448, "shared memory");
static_assert(B_COPY % 1024 == 0 && SLAB_COPY % 1024 == 0, "swizzle-atom alignment");
}  // namespace halo

struct HaloArgs {
  const float* x;        // NHWC input, channels [coff, coff + Cin) of Cs
  int H, W, Cs, coff, Cin;
  int pad, Wp, KH, KW;
  unsigned img_rows;     // Hp * Wp
  unsigned rows;         // N * Hp * Wp (< 2^31)
  float* out;
  long long ldc;
  int act, OH, OW, Cout;
};

// split weights: w [taps*Cin][Cout] (row stride ldw) -> [2][taps*64][64] bf16 hi / lo, zero for
// channels >= Cin and columns >= Cout
__global__ void k_halo_wsplit(const float* __restrict__ w, int taps, int Cin, int Cout, long long ldw,
                              uint16_t* __restrict__ dst) {
  const int total = taps * halo::CP * halo::BN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int j = i % halo::BN, r = i / halo::BN, tap = r / halo::CP, ch = r % halo::CP;
    const float v = (ch < Cin && j < Cout) ? w[((long long)tap * Cin + ch) * ldw + j] : 0.0f;
    nx_store_split1<true>(dst, (size_t)i, (size_t)total, v);
  }
}

// 128-byte-swizzle descriptor of a matrix starting at `addr`.  The start may lie on any 128-byte
// row: the tensor core takes the swizzle phase of each row from the absolute shared-memory address
// bits, as TMA and the converters wrote it, so the descriptor's base-offset field stays 0 (setting
// it to the start's phase, (addr >> 7) & 7, measurably reads the wrong rows).
__device__ __forceinline__ uint64_t halo_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return dev::umma_sdesc(addr, lbo, sbo, dev::UMMA_SW128);
}

template <bool VEC>
__global__ void __launch_bounds__(halo::THREADS, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tmB, HaloArgs a, const float* __restrict__ bias,
                     int num_tiles, unsigned* err) {
  using namespace halo;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sA = smem + B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + NSLAB * SLAB);
  uint64_t* b_full = bars;
  uint64_t* slab_full = bars + 1;
  uint64_t* slab_empty = bars + 3;
  uint64_t* t_full = bars + 5;
  uint64_t* t_empty = bars + 9;
  uint64_t* drain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + B_BYTES + NSLAB * SLAB + BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbias = reinterpret_cast<float*>(smem + B_BYTES + NSLAB * SLAB + BAR_BYTES + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int taps = a.KH * a.KW;
  if (threadIdx.x == 0) {
    dev::mbar_init(b_full, 1);
    for (int s = 0; s < NSLAB; ++s) {
      dev::mbar_init(&slab_full[s], CONV_WARPS);
      dev::mbar_init(&slab_empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&t_full[b], 1);
      dev::mbar_init(&t_empty[b], EPI_WARPS);
    }
    dev::mbar_init(drain, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmB);
  }
  if (threadIdx.x < BN) sbias[threadIdx.x] = (bias && (int)threadIdx.x < a.Cout) ? bias[threadIdx.x] : 0.0f;
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, 512);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- resident weights: one TMA box per (copy, tap)
    if (lane == 0) {
      dev::mbar_arrive_expect_tx(b_full, (uint32_t)(2 * taps * TAPB));
      for (int op = 0; op < 2; ++op)
        for (int t = 0; t < taps; ++t)
          dev::tma_load_3d(sB + op * B_COPY + t * TAPB, &tmB, b_full, 0, t * CP, op);
      // the copies must land before the CTA can exit
      dev::mbar_wait(b_full, 0, err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    // One thread's serial instruction stream: descriptors are built once and advanced by
    // adding to their 14-bit start-address field (addresses stay below 256 KB, no carry).
    if (lane == 0) {
      constexpr uint32_t idesc = dev::umma_idesc(1u, 1u, 1u, 0u, 1u, 128u, (uint32_t)BN);
      constexpr uint32_t idesc2 = dev::umma_idesc(1u, 1u, 1u, 0u, 1u, 128u, 128u);
      const uint64_t ad0 = halo_desc(dev::smem_u32(sA), 16, 1024);
      // [B_hi | B_lo] as one 128-column MN-major operand: chunk 1 (columns 64..127) sits one
      // weight copy after chunk 0
      const uint64_t bd0 = halo_desc(dev::smem_u32(sB), B_COPY, 1024);
      bool ok = dev::mbar_wait(b_full, 0, err);
      dev::tc_fence_after();
      uint32_t sl = 0, local = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local % NBUF, use = local / NBUF;
        if (*abort_flag || !dev::mbar_wait(&t_empty[buf], (use & 1) ^ 1, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t d_tmem = tmem + buf * 256, d2 = d_tmem + 128;
        uint64_t bd = bd0;  // tap (kh, kw) of the hi copy
        for (int kh = 0; kh < a.KH; ++kh, ++sl) {
          const uint32_t s = sl & 1, ph = (sl >> 1) & 1;
          if (!dev::mbar_wait(&slab_full[s], ph, err)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          uint64_t ad = ad0 + (uint64_t)((s * SLAB) >> 4);  // slab s, hi copy, row 0
          for (int kw = 0; kw < a.KW; ++kw, ad += ROWB >> 4, bd += TAPB >> 4) {
            const uint32_t first = (kh | kw) == 0;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              // hi * [hi | lo] (128 columns), lo * hi (64 columns)
              dev::umma<dev::MmaKind::F16>(d_tmem, ad + ((ks * 32) >> 4),
                                           bd + ((ks * 16 * ROWB) >> 4), idesc2, (ks != 0) || !first);
              dev::umma<dev::MmaKind::F16>(d2, ad + ((SLAB_COPY + ks * 32) >> 4),
                                           bd + ((ks * 16 * ROWB) >> 4), idesc, (ks != 0) || !first);
            }
          }
          dev::umma_commit(&slab_empty[s]);
        }
        if (ok) dev::umma_commit(&t_full[buf]);
      }
      if (!ok) {
        *abort_flag = 1;
        dev::umma_commit(drain);
        dev::mbar_wait(drain, 0, nullptr, 200000000ull);
        for (int b = 0; b < NBUF; ++b) dev::mbar_arrive(&t_full[b]);
      }
    }
  } else if (warp < 2 + CONV_WARPS) {
    // ---------------- converters: fp32 NHWC -> swizzled bf16 hi / lo slab rows
    // unit = (slab row, 16 channels): 64 contiguous input bytes, two 16-byte chunks per copy.
    // Slab k of this CTA is (tile blockIdx.x + (k / KH) * gridDim.x, kernel row k % KH); the
    // loads of slab k + 1 are issued before slab k is stored, so two slabs of loads overlap.
    const int ct = threadIdx.x - 64;
    const int R = 128 + a.KW - 1, NU = 4 * R;
    const int my_tiles = num_tiles > (int)blockIdx.x
                             ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nslabs = my_tiles * a.KH;
    auto load_slab = [&](int k, float4 (&v)[UNITS][4]) {
      const int t = (int)blockIdx.x + (k / a.KH) * (int)gridDim.x, kh = k - (k / a.KH) * a.KH;
      const unsigned r0 = (unsigned)t * 128u + (unsigned)(kh * a.Wp);
#pragma unroll
      for (int u = 0; u < UNITS; ++u) {
        const int idx = ct + u * CONV_THREADS, row = idx >> 2, ch = (idx & 3) * 16;
#pragma unroll
        for (int e = 0; e < 4; ++e) v[u][e] = make_float4(0.f, 0.f, 0.f, 0.f);
        const unsigned g = r0 + (unsigned)row;
        if (idx < NU && g < a.rows && ch < a.Cin) {
          const unsigned n = g / a.img_rows, q = g - n * a.img_rows;
          const unsigned hp = q / a.Wp;
          const int ih = (int)hp - a.pad, iw = (int)(q - hp * a.Wp) - a.pad;
          if (ih >= 0 && ih < a.H && iw >= 0 && iw < a.W) {
            const float* src = a.x + (((size_t)n * a.H + ih) * a.W + iw) * a.Cs + a.coff + ch;
            if constexpr (VEC) {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (ch + 4 * e < a.Cin) v[u][e] = __ldg(reinterpret_cast<const float4*>(src) + e);
            } else {
              float* f = reinterpret_cast<float*>(v[u]);
#pragma unroll
              for (int e = 0; e < 16; ++e) f[e] = (ch + e < a.Cin) ? __ldg(src + e) : 0.0f;
            }
          }
        }
      }
    };
    auto store_slab = [&](int k, const float4 (&v)[UNITS][4]) -> bool {
      const uint32_t s = (uint32_t)k & 1, ph = ((uint32_t)k >> 1) & 1;
      if (*abort_flag || !dev::mbar_wait(&slab_empty[s], ph ^ 1, err)) {
        *abort_flag = 1;
        return false;
      }
      uint8_t* hi = sA + s * SLAB;
#pragma unroll
      for (int u = 0; u < UNITS; ++u) {
        const int idx = ct + u * CONV_THREADS, row = idx >> 2, c16 = (idx & 3) * 2;
        if (idx < NU) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float4 p0 = v[u][2 * hh], p1 = v[u][2 * hh + 1];
            uint32_t h[4], l[4];
            nx_split_bf16x2(p0.x, p0.y, h[0], l[0]);
            nx_split_bf16x2(p0.z, p0.w, h[1], l[1]);
            nx_split_bf16x2(p1.x, p1.y, h[2], l[2]);
            nx_split_bf16x2(p1.z, p1.w, h[3], l[3]);
            const int off = row * ROWB + (((c16 + hh) ^ (row & 7)) << 4);
            *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(hi + SLAB_COPY + off) = make_uint4(l[0], l[1], l[2], l[3]);
          }
        }
      }
      dev::fence_proxy_async_smem();  // generic-proxy stores -> the tensor core's reads
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&slab_full[s]);
      return true;
    };
    float4 va[UNITS][4], vb[UNITS][4];
    if (nslabs > 0) load_slab(0, va);
    for (int k = 0; k < nslabs; k += 2) {
      if (k + 1 < nslabs) load_slab(k + 1, vb);
      if (!store_slab(k, va)) break;
      if (k + 1 >= nslabs) break;
      if (k + 2 < nslabs) load_slab(k + 2, va);
      if (!store_slab(k + 1, vb)) break;
    }
  } else {
    // ---------------- epilogue: TMEM -> +bias, ReLU -> output pixels
    const int q = warp & 3;
    uint32_t local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      const bool ok = dev::mbar_wait(&t_full[buf], use & 1, err);
      dev::tc_fence_after();
      if (!ok || *abort_flag) break;
      const unsigned r = (unsigned)t * 128u + (unsigned)(q * 32 + lane);
      const unsigned n = r / a.img_rows, qq = r - n * a.img_rows;
      const int oh = (int)(qq / (unsigned)a.Wp), ow = (int)qq - oh * a.Wp;
      const bool store = r < a.rows && oh < a.OH && ow < a.OW;
      float* dst = a.out + (((long long)n * a.OH + oh) * a.OW + ow) * a.ldc;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32) {
        if (c0 >= a.Cout) break;  // warp-uniform
        uint32_t v[32], v1[32], v2[32];
        const uint32_t tb = tmem + buf * 256 + (uint32_t)c0 + ((uint32_t)(q * 32) << 16);
        dev::tmem_ld32(tb, v);          // hi*hi
        dev::tmem_ld32(tb + 64, v1);    // hi*lo
        dev::tmem_ld32(tb + 128, v2);   // lo*hi
        dev::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          v[i] = __float_as_uint(__fadd_rn(__fadd_rn(__uint_as_float(v2[i]), __uint_as_float(v1[i])),
                                           __uint_as_float(v[i])));
        if (!store) continue;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float y = __fadd_rn(__uint_as_float(v[i]), sbias[c0 + i]);
          if (a.act) y = relu_max(y);
          o[i] = y;
        }
        if (c0 + 32 <= a.Cout && (reinterpret_cast<uintptr_t>(dst + c0) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + c0 + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
        } else {
          for (int i = 0; i < 32; ++i)
            if (c0 + i < a.Cout) dst[c0 + i] = o[i];
        }
      }
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&t_empty[buf]);
    }
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, 512);
  }
}

bool conv_halo_ok(int Cin, int KH, int KW, int Cout, int stride) {
  return stride == 1 && Cin >= 1 && Cin <= halo::CP && Cout >= 1 && Cout <= halo::BN && KH >= 1 &&
         KW >= 1 && KH * KW <= halo::MAXTAPS && 128 + KW - 1 <= halo::SLAB_ROWS;
}

bool conv_halo_f32_dev(Call& c, const float* x, int N, int H, int W, int Cs, int coff, int Cin,
                       const float* w, long long ldw, const float* bias, int KH, int KW, int Cout,
                       int pad, float* out, long long ldc, int act) {
  const int Hp = H + 2 * pad, Wp = W + 2 * pad, OH = Hp - KH + 1, OW = Wp - KW + 1;
  if (OH <= 0 || OW <= 0 || N <= 0) return true;
  const long long rows = (long long)N * Hp * Wp;
  if (rows >= (1LL << 31) - 1024 || (long long)Hp * Wp >= (1LL << 31)) {
    set_error(kInvalid, "%s: tensor too large", c.name());
    c.fail();
    return false;
  }
  const int taps = KH * KW;
  uint16_t* ws = static_cast<uint16_t*>(c.scratch((size_t)2 * taps * halo::CP * halo::BN * 2));
  if (!ws) return false;
  k_halo_wsplit<<<(taps * halo::CP * halo::BN + 255) / 256, 256, 0, c.stream()>>>(w, taps, Cin, Cout,
                                                                                  ldw, ws);
  if (!c.launched("k_halo_wsplit")) return false;
  CUtensorMap tb;
  const uint64_t dB[3] = {(uint64_t)halo::BN, (uint64_t)taps * halo::CP, 2};
  const uint64_t sB[2] = {(uint64_t)halo::BN * 2, (uint64_t)taps * halo::CP * halo::BN * 2};
  const uint32_t bB[3] = {(uint32_t)halo::BN, (uint32_t)halo::CP, 1u};
  if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ws, dB, sB, bB,
                   CU_TENSOR_MAP_SWIZZLE_128B)) {
    c.fail();
    return false;
  }
  HaloArgs a;
  a.x = x;
  a.H = H;
  a.W = W;
  a.Cs = Cs;
  a.coff = coff;
  a.Cin = Cin;
  a.pad = pad;
  a.Wp = Wp;
  a.KH = KH;
  a.KW = KW;
  a.img_rows = (unsigned)(Hp * Wp);
  a.rows = (unsigned)rows;
  a.out = out;
  a.ldc = ldc;
  a.act = act;
  a.OH = OH;
  a.OW = OW;
  a.Cout = Cout;
  const bool vec = Cin % 4 == 0 && Cs % 4 == 0 && coff % 4 == 0 && aligned16(x);
  const int tiles = (int)((rows + 127) / 128);
  const int grid = tiles < c.sm_count() ? tiles : c.sm_count();
  static bool attr_done[2][64] = {};
  const int dv = current_device();
  auto kern = vec ? conv_halo_kernel<true> : conv_halo_kernel<false>;
  if (dv >= 0 && dv < 64 && !attr_done[vec][dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, halo::SMEM))) {
      c.fail();
      return false;
    }
    attr_done[vec][dv] = true;
  }
  kern<<<grid, halo::THREADS, halo::SMEM, c.stream()>>>(tb, a, bias, tiles, c.err());
  return c.launched("conv_halo_kernel");
}

}  // namespace acf

