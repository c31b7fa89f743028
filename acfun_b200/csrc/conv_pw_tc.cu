// conv_pw_tc.cu — 1x1 stride-1 fp32 convolutions with few output channels (the reference's
// zero-copy GEMM route, conv1x1_impl, layers.cpp:66-101: out[p][j] = sum_c x[p][c] * w[c][j]
// + b[j], then act) as one persistent tcgen05 kernel in 3xBF16, reading the fp32 activation
// once.  The cfg4 pointwise layer (144 -> 24 at 56x56, 32 images) is HBM-bound: 57.8 MB in,
// 9.6 MB out, 0.69 GFLOP.
//
// GEMM view: row = pixel (M = N*H*W), K = input channels in 64-channel blocks (zero past Cin),
// N = output channels padded to Np (a multiple of 16, <= 64).  A tile is 128 pixels.
//   * A TMA warp brings each (tile, K block) as a [128 pixels][64 channels] fp32 box (zero fill
//     past Cin and past the last pixel) into a ring of fp32 stages, as many as shared memory
//     holds (4 at the cfg4 shape): the HBM latency is covered only by the bytes in flight.
//   * Eight converter warps split each box into bf16 hi / lo tiles in the 128-byte-swizzled
//     K-major layout (one 16-byte chunk of 8 channels per unit, 8 threads per pixel row), into
//     a second ring; the split weights of every K block ([2*Np][64] K-major: the hi rows, then
//     the lo rows), prepared once per call by k_pw_wsplit in their shared-memory image, arrive
//     by one bulk copy and stay resident (built inside each CTA they cost ~25 us of ALU work).
//   * One thread issues per K-step two MMAs: hi x [B_hi ; B_lo] (N = 2*Np: the hi*hi and hi*lo
//     partials in adjacent column blocks) and lo x B_hi (N = Np), into one of two TMEM buffers.
//   * Four epilogue warps sum the partials ((lo*hi + hi*lo) + hi*hi), add the bias, apply act
//     and store the pixel's Cout outputs.
// Every wait is bounded (ptx.cuh); on expiry the kernel flags the error word and drains.
#include <algorithm>

#include "conv.cuh"
#include "gemm.cuh"

namespace acf {
namespace pw {
constexpr int BKC = 64;                        // channels of a K block
constexpr int MAXKB = 3;                       // K blocks (Cin <= 192)
constexpr int MAXNP = 64;                      // padded output channels
constexpr int F_BYTES = 128 * BKC * 4;         // 32 KB fp32 box
constexpr int H_BYTES = 128 * BKC * 2;         // 16 KB: one bf16 copy of a K block
constexpr int S_BYTES = 2 * H_BYTES;           // hi + lo
constexpr int MAXNF = 6, NS = 2, NBUF = 2;    // fp32 stages: as many as fit (>= 2)
constexpr int B_BLOCK_MAX = 2 * MAXNP * 128;   // [2*Np rows][128 bytes] per K block
constexpr int CONV_WARPS = 8, EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * (CONV_WARPS + EPI_WARPS);
// barriers: f_full[MAXNF], f_empty[MAXNF], s_full[NS], s_empty[NS], t_full[NBUF], t_empty[NBUF],
// b_ready, drain
constexpr int BAR_BYTES = (2 * MAXNF + 2 * NS + 2 * NBUF + 2) * 8;
constexpr int SMEM_MAX = 232448;
constexpr int FIXED = 1024 + NS * S_BYTES + BAR_BYTES + 16 + MAXNP * 4;
static_assert(FIXED + MAXKB * B_BLOCK_MAX + 2 * F_BYTES <= SMEM_MAX, "shared memory");
}  // namespace pw

struct PwArgs {
  const uint8_t* wimg;     // split weights in their shared-memory image (k_pw_wsplit)
  const float* bias;
  int Cin, Cout, Np, kb;   // kb: K blocks
  int nf;                  // fp32 stages
  unsigned M;              // pixels
  float* out;
  long long ldc;
  int act;
  int num_tiles;
};

__global__ void __launch_bounds__(pw::THREADS, 1)
    conv_pw_tc_kernel(const __grid_constant__ CUtensorMap tmX, PwArgs a, unsigned* err) {
  using namespace pw;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int NF = a.nf, B_BLOCK = 2 * a.Np * 128;
  uint8_t* sS = smem;
  uint8_t* sB = sS + NS * S_BYTES;
  uint8_t* sF = sB + a.kb * B_BLOCK;  // 1024-aligned: B_BLOCK is a multiple of 4 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sF + NF * F_BYTES);
  uint64_t* f_full = bars;
  uint64_t* f_empty = f_full + MAXNF;
  uint64_t* s_full = f_empty + MAXNF;
  uint64_t* s_empty = s_full + NS;
  uint64_t* t_full = s_empty + NS;
  uint64_t* t_empty = t_full + NBUF;
  uint64_t* b_ready = t_empty + NBUF;
  uint64_t* drain = b_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + BAR_BYTES + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Np = a.Np, B_ROWS = 2 * Np;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NF; ++s) {
      dev::mbar_init(&f_full[s], 1);
      dev::mbar_init(&f_empty[s], CONV_WARPS);
    }
    for (int s = 0; s < NS; ++s) {
      dev::mbar_init(&s_full[s], CONV_WARPS);
      dev::mbar_init(&s_empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&t_full[b], 1);
      dev::mbar_init(&t_empty[b], EPI_WARPS);
    }
    dev::mbar_init(b_ready, 1);
    dev::mbar_init(drain, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, 512);
    dev::tmem_relinquish();
  }
  // the prologue above may overlap the weight preparation; nothing it produced is read before this
  dev::grid_dep_wait();
  if (threadIdx.x < MAXNP) sbias[threadIdx.x] = (a.bias && (int)threadIdx.x < a.Cout) ? a.bias[threadIdx.x] : 0.0f;
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: one fp32 box per (tile, K block)
    if (lane == 0) {
      // the split weights: one bulk copy of the image k_pw_wsplit prepared
      const uint32_t bbytes = (uint32_t)(a.kb * B_BLOCK);
      dev::mbar_arrive_expect_tx(b_ready, bbytes);
      dev::bulk_load(sB, a.wimg, bbytes, b_ready);
      uint32_t it = 0;
      for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x) {
        for (int kb = 0; kb < a.kb; ++kb, ++it) {
          const uint32_t s = it % NF, ph = (it / NF) & 1;
          if (*abort_flag || !dev::mbar_wait(&f_empty[s], ph ^ 1, err)) {
            *abort_flag = 1;
            break;
          }
          dev::mbar_arrive_expect_tx(&f_full[s], (uint32_t)F_BYTES);
          dev::tma_load_2d(sF + s * F_BYTES, &tmX, &f_full[s], kb * BKC, t * 128);
        }
        if (*abort_flag) break;
      }
      dev::mbar_wait(b_ready, 0, nullptr, 200000000ull);
      for (uint32_t k = it > (uint32_t)NF ? it - NF : 0; k < it; ++k)
        dev::mbar_wait(&f_full[k % NF], (k / NF) & 1, nullptr, 200000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_a = dev::umma_idesc(1u, 1u, 1u, 0u, 0u, 128u, (uint32_t)B_ROWS);
      const uint32_t idesc_b = dev::umma_idesc(1u, 1u, 1u, 0u, 0u, 128u, (uint32_t)Np);
      const uint64_t ad0 = dev::umma_sdesc(dev::smem_u32(sS), 16, 1024, dev::UMMA_SW128);
      const uint64_t bd0 = dev::umma_sdesc(dev::smem_u32(sB), 16, 1024, dev::UMMA_SW128);
      bool ok = dev::mbar_wait(b_ready, 0, err);
      dev::tc_fence_after();
      uint32_t it = 0, local = 0;
      for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local % NBUF, use = local / NBUF;
        if (*abort_flag || !dev::mbar_wait(&t_empty[buf], (use & 1) ^ 1, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t d0 = tmem + buf * 256, d1 = d0 + (uint32_t)B_ROWS;
        for (int kb = 0; kb < a.kb; ++kb, ++it) {
          const uint32_t s = it % NS, ph = (it / NS) & 1;
          if (!dev::mbar_wait(&s_full[s], ph, err)) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
          const uint64_t ah = ad0 + (uint64_t)((s * S_BYTES) >> 4), al = ah + (uint64_t)(H_BYTES >> 4);
          const uint64_t bb = bd0 + (uint64_t)((kb * B_BLOCK) >> 4);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {  // 16 channels (32 bytes) per MMA
            const uint32_t acc = (kb | ks) != 0;
            dev::umma<dev::MmaKind::F16>(d0, ah + (uint64_t)ks * 2, bb + (uint64_t)ks * 2, idesc_a, acc);
            dev::umma<dev::MmaKind::F16>(d1, al + (uint64_t)ks * 2, bb + (uint64_t)ks * 2, idesc_b, acc);
          }
          dev::umma_commit(&s_empty[s]);
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
    // ---------------- converters: fp32 box -> swizzled bf16 hi / lo
    const int ct = threadIdx.x - 64;  // 0..255
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.num_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < a.kb; ++kb, ++it) {
        const uint32_t f = it % NF, fph = (it / NF) & 1;
        const uint32_t s = it % NS, sph = (it / NS) & 1;
        if (*abort_flag || !dev::mbar_wait(&f_full[f], fph, err) ||
            !dev::mbar_wait(&s_empty[s], sph ^ 1, err)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        const float* src = reinterpret_cast<const float*>(sF + f * F_BYTES);
        uint8_t* hi = sS + s * S_BYTES;
        uint8_t* lo = hi + H_BYTES;
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // 1024 (row, 8-channel chunk) units per box
          const int unit = ct + 256 * u, r = unit >> 3, chunk = unit & 7;
          const float4 p0 = *reinterpret_cast<const float4*>(src + r * BKC + chunk * 8);
          const float4 p1 = *reinterpret_cast<const float4*>(src + r * BKC + chunk * 8 + 4);
          uint32_t h[4], l[4];
          nx_split_bf16x2(p0.x, p0.y, h[0], l[0]);
          nx_split_bf16x2(p0.z, p0.w, h[1], l[1]);
          nx_split_bf16x2(p1.x, p1.y, h[2], l[2]);
          nx_split_bf16x2(p1.z, p1.w, h[3], l[3]);
          const int o = r * 128 + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(hi + o) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(lo + o) = make_uint4(l[0], l[1], l[2], l[3]);
        }
        dev::fence_proxy_async_smem();  // generic-proxy stores -> the tensor core's reads
        __syncwarp();
        if (lane == 0) {
          dev::mbar_arrive(&f_empty[f]);
          dev::mbar_arrive(&s_full[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> +bias, act -> output pixels
    const int q = warp & 3;
    uint32_t local = 0;
    for (int t = blockIdx.x; t < a.num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      const bool ok = dev::mbar_wait(&t_full[buf], use & 1, err);
      dev::tc_fence_after();
      if (!ok || *abort_flag) break;
      const unsigned r = (unsigned)t * 128u + (unsigned)(q * 32 + lane);
      const bool store = r < a.M;
      float* dst = a.out + (long long)r * a.ldc;
      const uint32_t tb = tmem + buf * 256 + ((uint32_t)(q * 32) << 16);
      for (int c0 = 0; c0 < Np; c0 += 16) {
        uint32_t v[16], v1[16], v2[16];
        dev::tmem_ld16(tb + c0, v);                        // hi*hi
        dev::tmem_ld16(tb + (uint32_t)Np + c0, v1);        // hi*lo
        dev::tmem_ld16(tb + (uint32_t)B_ROWS + c0, v2);    // lo*hi
        dev::tmem_ld_wait();
        if (!store) continue;
        float o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float y = __fadd_rn(__fadd_rn(__uint_as_float(v2[i]), __uint_as_float(v1[i])),
                              __uint_as_float(v[i]));
          y = __fadd_rn(y, sbias[c0 + i]);
          if (a.act) y = relu_max(y);
          o[i] = y;
        }
#pragma unroll
        for (int i = 0; i < 16; i += 8) {  // 8 columns at a time: one 32-byte store when whole
          float* d = dst + c0 + i;
          if (c0 + i + 8 <= a.Cout && (reinterpret_cast<uintptr_t>(d) & 31) == 0) {
            dev::st_global_v8(d, reinterpret_cast<const uint32_t*>(o + i));
          } else if (c0 + i + 8 <= a.Cout && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
            *reinterpret_cast<float4*>(d) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
            *reinterpret_cast<float4*>(d + 4) = make_float4(o[i + 4], o[i + 5], o[i + 6], o[i + 7]);
          } else {
            for (int e = 0; e < 8; ++e)
              if (c0 + i + e < a.Cout) d[e] = o[i + e];
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

// Split weights in the kernel's shared-memory image: K block kb, row r < Np holds the bf16 hi
// of output column r, row Np + r its lo; 128-byte rows of 64 channels, 16-byte chunks
// XOR-swizzled by (row & 7) as the tensor core's 128-byte K-major layout expects.
__global__ void k_pw_wsplit(const float* __restrict__ w, long long ldw, int Cin, int Cout, int Np, int kb,
                            uint8_t* __restrict__ img) {
  dev::grid_dep_launch();  // the conv kernel may start its prologue now
  const int rows = 2 * Np, total = kb * rows * pw::BKC;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int b = e / (rows * pw::BKC), rem = e - b * rows * pw::BKC;
    const int r = rem / pw::BKC, k = rem - r * pw::BKC;
    const int j = r < Np ? r : r - Np, c = b * pw::BKC + k;
    const float v = (j < Cout && c < Cin) ? w[(long long)c * ldw + j] : 0.0f;
    const uint16_t hb = nx_bf16_rne(v);
    const uint16_t bits = r < Np ? hb : nx_bf16_rne(v - nx_bf16_val(hb));
    uint8_t* row = img + (size_t)b * rows * 128 + (size_t)r * 128;
    *reinterpret_cast<uint16_t*>(row + ((((k >> 3) ^ (r & 7)) << 4) | ((k & 7) << 1))) = bits;
  }
}

bool conv_pw_tc_ok(const float* x, int Cs, int coff, int Cin, int Cout, long long M) {
  return coff == 0 && Cs == Cin && Cin % 4 == 0 && Cin >= 4 && Cin <= pw::MAXKB * pw::BKC &&
         Cout >= 1 && Cout <= pw::MAXNP && aligned16(x) && M >= 128LL * 148 && M < (1LL << 31) - 256;
}

bool conv_pw_tc_dev(Call& c, const float* x, long long M, int Cin, const float* w, long long ldw,
                    const float* bias, int Cout, float* out, long long ldc, int act) {
  PwArgs a;
  a.bias = bias;
  a.Cin = Cin;
  a.Cout = Cout;
  a.Np = (Cout + 15) & ~15;
  a.kb = (Cin + pw::BKC - 1) / pw::BKC;
  a.M = (unsigned)M;
  a.out = out;
  a.ldc = ldc;
  a.act = act;
  a.num_tiles = (int)((M + 127) / 128);
  const int bbytes = a.kb * 2 * a.Np * 128;
  uint8_t* img = static_cast<uint8_t*>(c.scratch((size_t)bbytes));
  if (!img) return false;
  k_pw_wsplit<<<(bbytes / 2 + 255) / 256, 256, 0, c.stream()>>>(w, ldw, Cin, Cout, a.Np, a.kb, img);
  if (!c.launched("k_pw_wsplit")) return false;
  a.wimg = img;
  a.nf = std::min(pw::MAXNF, (pw::SMEM_MAX - pw::FIXED - bbytes) / pw::F_BYTES);
  const int smem = pw::FIXED + bbytes + a.nf * pw::F_BYTES;
  CUtensorMap tx;
  const uint64_t d[2] = {(uint64_t)Cin, (uint64_t)M};
  const uint64_t st[1] = {(uint64_t)Cin * 4};
  const uint32_t bx[2] = {(uint32_t)pw::BKC, 128u};
  if (!encode_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, x, d, st, bx, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    c.fail();
    return false;
  }
  static bool attr_done[64] = {};
  const int dv = current_device();
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(conv_pw_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          pw::SMEM_MAX))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  const int grid = std::min(a.num_tiles, c.sm_count());
  if (!ACF_CUDA_OK(launch_pdl(conv_pw_tc_kernel, dim3(grid), dim3(pw::THREADS), (size_t)smem, c.stream(), tx, a,
                              c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("conv_pw_tc_kernel");
}

}  // namespace acf
