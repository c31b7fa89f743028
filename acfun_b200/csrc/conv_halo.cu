// conv_halo.cu — narrow stride-1 fp32 convolutions (at most 64 input and 64 output channels,
// KH*KW <= 9: the reference's Winograd F(2,3) / F(4,3) routes at the cfg3 shapes,
// winograd_avx512.cpp:186-250 and winograd43_avx512.cpp:218-280) as a split pass plus one
// persistent tcgen05 kernel in 3xBF16.
//
// GEMM view: row r = a pixel of the zero-padded input grid (N x Hp x Wp, NHWC), 64 channels
// per row; output pixel (oh, ow) of image n is row r = (n*Hp + oh)*Wp + ow, and tap (kh, kw)
// reads row r + kh*Wp + kw.  A tile is 128 consecutive rows x 64 output channels.
//   * k_halo_split writes the padded grid once as bf16 hi / lo planes ([2][rows][64], zero in
//     the border and past the channels), a bandwidth pass whose output stays in L2, and the
//     split weights; the conv kernel is launched as its programmatic dependent, so its prologue
//     (barriers, tensor memory) overlaps the pass.
//   * The split weights of every tap ([2][taps][64 channels][64 columns] bf16 hi / lo, 16 KB a
//     tap) are loaded by TMA once per CTA and stay resident in shared memory.
//   * For each kernel row kh one TMA box brings the tile's 128 + KW - 1 rows of both planes
//     (a "slab", 128-byte swizzled K-major); the A operand of tap kw is the slab from row kw
//     on, a descriptor whose start is shifted by kw rows, so a row is staged once per kernel
//     row instead of once per tap.  3xBF16 in two MMAs per K-step: hi * [hi | lo] as one
//     128-column operand (the two weight copies are the two 64-column chunks of an MN-major B
//     whose chunk stride is one copy) and lo * hi, into three fp32 partial accumulators in
//     TMEM (two buffers of 256 columns).
//   * Eight epilogue warps (two per TMEM lane quadrant, one 32-column chunk each) sum the
//     partials ((lo*hi + hi*lo) + hi*hi), add the bias, apply ReLU and store the rows that
//     land on output pixels.
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
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
// barriers: b_full, slab_full[2], slab_empty[2], t_full[2], t_empty[2], drain
constexpr int BAR_BYTES = 16 * 8;
constexpr int SMEM = 1024 + B_BYTES + NSLAB * SLAB + BAR_BYTES + 16 + BN * 4;
static_assert(SMEM <= 232448, "shared memory");
static_assert(B_COPY % 1024 == 0 && SLAB_COPY % 1024 == 0, "swizzle-atom alignment");
}  // namespace halo

struct HaloArgs {
  int KH, KW, Wp;
  unsigned img_rows;     // Hp * Wp
  unsigned rows;         // N * Hp * Wp (< 2^31)
  float* out;
  long long ldc;
  int act, OH, OW, Cout;
};

// x: NHWC (channel stride Cs, channels [coff, coff + Cin)) -> [2][rows][64] bf16 hi / lo planes of
// the zero-padded grid; one thread per (grid row, 8 channels): two 16-byte loads, one 16-byte
// store per plane.
// The same launch splits the weights: w [taps*Cin][Cout] (row stride ldw) -> [2][taps*64][64] bf16
// hi / lo, zero for channels >= Cin and columns >= Cout.
template <bool VEC>
__global__ void k_halo_split(const float* __restrict__ x, int H, int W, int Cs, int coff, int Cin,
                             int pad, int Wp, unsigned img_rows, unsigned total,
                             uint4* __restrict__ dst, unsigned plane16,
                             const float* __restrict__ w, int taps, int Cout, long long ldw,
                             uint16_t* __restrict__ wdst) {
  dev::grid_dep_launch();  // the conv kernel may start its prologue now
  const int wtotal = taps * halo::CP * halo::BN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < wtotal; i += gridDim.x * blockDim.x) {
    const int j = i % halo::BN, r = i / halo::BN, tap = r / halo::CP, ch = r % halo::CP;
    const float v = (ch < Cin && j < Cout) ? w[((long long)tap * Cin + ch) * ldw + j] : 0.0f;
    nx_store_split1<true>(wdst, (size_t)i, (size_t)wtotal, v);
  }
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const unsigned g = i >> 3, c8 = (i & 7) * 8;
    const unsigned n = g / img_rows, q = g - n * img_rows;
    const unsigned hp = q / (unsigned)Wp;
    const int ih = (int)hp - pad, iw = (int)(q - hp * (unsigned)Wp) - pad;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if ((int)c8 < Cin && ih >= 0 && ih < H && iw >= 0 && iw < W) {
      const float* src = x + (((size_t)n * H + ih) * W + iw) * Cs + coff + c8;
      if (VEC && (int)c8 + 8 <= Cin) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = ((int)c8 + e < Cin) ? __ldg(src + e) : 0.0f;
      }
    }
    uint32_t h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) nx_split_bf16x2(v[2 * k], v[2 * k + 1], h[k], l[k]);
    dst[i] = make_uint4(h[0], h[1], h[2], h[3]);
    dst[i + plane16] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// 128-byte-swizzle descriptor of a matrix starting at `addr`.  The start may lie on any 128-byte
// row: the tensor core takes the swizzle phase of each row from the absolute shared-memory address
// bits, as TMA wrote it, so the descriptor's base-offset field stays 0 (setting it to the start's
// phase, (addr >> 7) & 7, measurably reads the wrong rows).
__device__ __forceinline__ uint64_t halo_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return dev::umma_sdesc(addr, lbo, sbo, dev::UMMA_SW128);
}

__global__ void __launch_bounds__(halo::THREADS, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     HaloArgs a, const float* __restrict__ bias, int num_tiles, unsigned* err) {
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
  uint64_t* t_empty = bars + 7;
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + B_BYTES + NSLAB * SLAB + BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbias = reinterpret_cast<float*>(smem + B_BYTES + NSLAB * SLAB + BAR_BYTES + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int taps = a.KH * a.KW;
  if (threadIdx.x == 0) {
    dev::mbar_init(b_full, 1);
    for (int s = 0; s < NSLAB; ++s) {
      dev::mbar_init(&slab_full[s], 1);
      dev::mbar_init(&slab_empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&t_full[b], 1);
      dev::mbar_init(&t_empty[b], EPI_WARPS);
    }
    dev::mbar_init(drain, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmA);
    dev::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, 512);
    dev::tmem_relinquish();
  }
  // the prologue above may overlap the split pass; nothing it produced is read before this
  dev::grid_dep_wait();
  if (threadIdx.x < BN) sbias[threadIdx.x] = (bias && (int)threadIdx.x < a.Cout) ? bias[threadIdx.x] : 0.0f;
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: resident weights, then one slab per (tile, kernel row)
    if (lane == 0) {
      dev::mbar_arrive_expect_tx(b_full, (uint32_t)(2 * taps * TAPB));
      for (int op = 0; op < 2; ++op)
        for (int t = 0; t < taps; ++t)
          dev::tma_load_3d(sB + op * B_COPY + t * TAPB, &tmB, b_full, 0, t * CP, op);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        for (int kh = 0; kh < a.KH; ++kh, ++it) {
          const uint32_t s = it & 1, ph = (it >> 1) & 1;
          if (*abort_flag || !dev::mbar_wait(&slab_empty[s], ph ^ 1, err)) {
            *abort_flag = 1;
            break;
          }
          dev::mbar_arrive_expect_tx(&slab_full[s], (uint32_t)SLAB);
          dev::tma_load_3d(sA + s * SLAB, &tmA, &slab_full[s], 0, t * 128 + kh * a.Wp, 0);
        }
        if (*abort_flag) break;
      }
      // every copy must land before the CTA can release its shared memory
      dev::mbar_wait(b_full, 0, nullptr, 200000000ull);
      if (*abort_flag)
        for (uint32_t k = it > (uint32_t)NSLAB ? it - NSLAB : 0; k < it; ++k)
          dev::mbar_wait(&slab_full[k & 1], (k >> 1) & 1, nullptr, 200000000ull);
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
  } else {
    // ---------------- epilogue: TMEM -> +bias, ReLU -> output pixels
    const int q = warp & 3;                // TMEM lane quadrant this warp may access
    const int c0 = ((warp - 2) >> 2) * 32;  // this warp's 32 output columns
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
      if (c0 < a.Cout) {  // warp-uniform
        uint32_t v[32], v1[32], v2[32];
        const uint32_t tb = tmem + buf * 256 + (uint32_t)c0 + ((uint32_t)(q * 32) << 16);
        dev::tmem_ld32(tb, v);          // hi*hi
        dev::tmem_ld32(tb + 64, v1);    // hi*lo
        dev::tmem_ld32(tb + 128, v2);   // lo*hi
        dev::tmem_ld_wait();
        if (store) {
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float y = __fadd_rn(__fadd_rn(__uint_as_float(v2[i]), __uint_as_float(v1[i])),
                                __uint_as_float(v[i]));
            y = __fadd_rn(y, sbias[c0 + i]);
            if (a.act) y = relu_max(y);
            o[i] = y;
          }
          if (c0 + 32 <= a.Cout && (reinterpret_cast<uintptr_t>(dst + c0) & 31) == 0) {
            // 32-byte stores: a whole sector per lane
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              dev::st_global_v8(dst + c0 + i, reinterpret_cast<const uint32_t*>(o + i));
          } else if (c0 + 32 <= a.Cout && (reinterpret_cast<uintptr_t>(dst + c0) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + c0 + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          } else {
            for (int i = 0; i < 32; ++i)
              if (c0 + i < a.Cout) dst[c0 + i] = o[i];
          }
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
  if (rows >= (1LL << 29) || (long long)Hp * Wp >= (1LL << 31)) {
    set_error(kInvalid, "%s: tensor too large", c.name());
    c.fail();
    return false;
  }
  const int taps = KH * KW;
  uint16_t* ws = static_cast<uint16_t*>(c.scratch((size_t)2 * taps * halo::CP * halo::BN * 2));
  uint4* xs = static_cast<uint4*>(c.scratch((size_t)2 * rows * halo::CP * 2));
  if (!ws || !xs) return false;
  const unsigned total = (unsigned)(rows * 8);
  const bool vec = Cin % 4 == 0 && Cs % 4 == 0 && coff % 4 == 0 && aligned16(x);
  long long gb = (total + 255) / 256, cap = (long long)c.sm_count() * 8;
  const int grid_s = (int)(gb < cap ? gb : cap);
  if (vec)
    k_halo_split<true><<<grid_s, 256, 0, c.stream()>>>(x, H, W, Cs, coff, Cin, pad, Wp,
                                                       (unsigned)(Hp * Wp), total, xs, total, w, taps,
                                                       Cout, ldw, ws);
  else
    k_halo_split<false><<<grid_s, 256, 0, c.stream()>>>(x, H, W, Cs, coff, Cin, pad, Wp,
                                                        (unsigned)(Hp * Wp), total, xs, total, w, taps,
                                                        Cout, ldw, ws);
  if (!c.launched("conv halo prep")) return false;
  CUtensorMap ta, tb;
  {
    const uint64_t d[3] = {(uint64_t)halo::CP, (uint64_t)rows, 2};
    const uint64_t st[2] = {(uint64_t)halo::CP * 2, (uint64_t)rows * halo::CP * 2};
    const uint32_t bx[3] = {(uint32_t)halo::CP, (uint32_t)halo::SLAB_ROWS, 2u};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, xs, d, st, bx,
                     CU_TENSOR_MAP_SWIZZLE_128B)) {
      c.fail();
      return false;
    }
  }
  {
    const uint64_t d[3] = {(uint64_t)halo::BN, (uint64_t)taps * halo::CP, 2};
    const uint64_t st[2] = {(uint64_t)halo::BN * 2, (uint64_t)taps * halo::CP * halo::BN * 2};
    const uint32_t bx[3] = {(uint32_t)halo::BN, (uint32_t)halo::CP, 1u};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ws, d, st, bx,
                     CU_TENSOR_MAP_SWIZZLE_128B)) {
      c.fail();
      return false;
    }
  }
  HaloArgs a;
  a.KH = KH;
  a.KW = KW;
  a.Wp = Wp;
  a.img_rows = (unsigned)(Hp * Wp);
  a.rows = (unsigned)rows;
  a.out = out;
  a.ldc = ldc;
  a.act = act;
  a.OH = OH;
  a.OW = OW;
  a.Cout = Cout;
  const int tiles = (int)((rows + 127) / 128);
  const int grid = tiles < c.sm_count() ? tiles : c.sm_count();
  static bool attr_done[64] = {};
  const int dv = current_device();
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(conv_halo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          halo::SMEM))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  if (!ACF_CUDA_OK(launch_pdl(conv_halo_kernel, dim3(grid), dim3(halo::THREADS), halo::SMEM, c.stream(), ta,
                              tb, a, bias, tiles, c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("conv_halo_kernel");
}

}  // namespace acf
