// conv_halo_i8.cu — narrow stride-1 int8 convolutions (at most 64 input and 128 output
// channels): the exact integer correlation of the reference's int8 routes (Winograd F(2,3),
// winograd_int8.cpp:245-350; direct, conv_int8_direct.cpp:20-59; 1x1, conv1x1_int8.cpp:21-36)
// as one persistent tcgen05 kind::i8 kernel that stages every input row once per tile.
//
// GEMM view (the same as the implicit route of conv_int8.cu): row r = a pixel of the
// zero-point-padded u8 grid (N x Hp x Wp, 64 bytes a row); output pixel (oh, ow) of image n is
// row r = (n*Hp + oh)*Wp + ow and tap (kh, kw) reads row r + kh*Wp + kw.  A tile is 128
// consecutive rows x BN output channels.
//   * The K-major s8 weights of every tap ([taps][BN rows][64 bytes], 64-byte swizzle) are
//     loaded by TMA once per CTA and stay resident in shared memory.
//   * Per tile, TMA brings one slab: the tile's 128 rows plus the (KH-1)*Wp + KW-1 rows its
//     taps reach past them, in 128-row boxes.  The A operand of tap (kh, kw) is the slab from
//     row kh*Wp + kw on: a descriptor whose start is shifted by that many 64-byte rows (the
//     tensor core takes each row's swizzle phase from the absolute address bits, as TMA wrote
//     it), so the nine taps read one staged copy instead of nine.
//   * Two MMAs (K = 32 bytes each) per tap accumulate u8 x s8 into int32 TMEM columns; four
//     accumulator buffers let the MMAs run up to four tiles ahead of the epilogue.
//   * Eight epilogue warps (two per TMEM lane quadrant, splitting the 32-column chunks) apply
//     the dequantisation of conv_int8.cu (F32_AB or I8_WINO, per-call or per-image scales,
//     ReLU, optional per-image max |out|) and store the rows that land on output pixels.
// Every wait is bounded (ptx.cuh); on expiry the kernel flags the error word and drains.
#include "conv.cuh"
#include "gemm.cuh"

namespace acf {
namespace h8 {
constexpr int CP = 64;                 // bytes (u8 channels) of one grid row
constexpr int BOX = 128;               // rows of one TMA box
constexpr int BOXB = BOX * CP;         // 8 KB
constexpr int MAXBOX = 4;              // slab of at most 512 rows
constexpr int MAXST = 8;               // slab stages
constexpr int NBUF = 4;                // TMEM accumulator buffers
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int SMEM_MAX = 232448;
// b_full, full[MAXST], empty[MAXST], tfull[NBUF], tempty[NBUF], drain
constexpr int BAR_BYTES = (1 + 2 * MAXST + 2 * NBUF + 1) * 8;
constexpr int MISC = 16;               // TMEM slot, abort flag
template <int BN>
struct Cfg {
  static constexpr int TAPB = BN * CP;                    // one tap of resident weights
  static constexpr int CHUNKS_PER_WARP = (BN / 32 + 1) / 2;
  static constexpr int PARAM_BYTES = EPI_WARPS * CHUNKS_PER_WARP * (int)sizeof(ColSlice);
  static constexpr int TMEM_COLS = NBUF * BN;
  static_assert(BN == 64 || BN == 128, "tile width");
  static_assert(TMEM_COLS <= 512, "TMEM capacity");
};
}  // namespace h8

struct H8Geom {
  int KH, KW, taps;
  int Wp;
  unsigned img_rows;   // Hp * Wp
  unsigned rows;       // N * Hp * Wp (< 2^31)
  int OH, OW, Cout;
  int nbox, nst;       // boxes per slab, slab stages
};

template <int BN, Epi EPI>
__global__ void __launch_bounds__(h8::THREADS, 1)
    conv_halo_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        EpiParams ep, H8Geom g, int num_tiles, unsigned* err) {
  using namespace h8;
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int slab_bytes = g.nbox * BOXB;
  uint8_t* sB = smem;
  uint8_t* sA = smem + g.taps * C::TAPB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + g.nst * slab_bytes);
  uint64_t* b_full = bars;
  uint64_t* full = bars + 1;
  uint64_t* empty = full + MAXST;
  uint64_t* tfull = empty + MAXST;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  ColSlice* col_slices = reinterpret_cast<ColSlice*>(reinterpret_cast<uint8_t*>(bars) + BAR_BYTES + MISC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    dev::mbar_init(b_full, 1);
    for (int s = 0; s < g.nst; ++s) {
      dev::mbar_init(&full[s], 1);
      dev::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&tfull[b], 1);
      dev::mbar_init(&tempty[b], EPI_WARPS);
    }
    dev::mbar_init(drain, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmA);
    dev::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, C::TMEM_COLS);
    dev::tmem_relinquish();
  }
  // the prologue above may overlap the quantiser; nothing it produced is read before this
  dev::grid_dep_wait();
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: resident weights, then one slab per tile
    if (lane == 0) {
      dev::mbar_arrive_expect_tx(b_full, (uint32_t)(g.taps * C::TAPB));
      for (int t = 0; t < g.taps; ++t)
        dev::tma_load_2d(sB + t * C::TAPB, &tmB, b_full, t * CP, 0);
      uint32_t it = 0, s = 0, ph = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
        if (*abort_flag || !dev::mbar_wait(&empty[s], ph ^ 1, err)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* dst = sA + s * slab_bytes;
        dev::mbar_arrive_expect_tx(&full[s], (uint32_t)slab_bytes);
        for (int b = 0; b < g.nbox; ++b)
          dev::tma_load_2d(dst + b * BOXB, &tmA, &full[s], 0, t * BOX + b * BOX);
        if (++s == (uint32_t)g.nst) {
          s = 0;
          ph ^= 1;
        }
      }
      // every copy must land before the CTA can release its shared memory
      dev::mbar_wait(b_full, 0, nullptr, 200000000ull);
      const uint32_t first = it > (uint32_t)g.nst ? it - g.nst : 0;
      if (*abort_flag)
        for (uint32_t k = first; k < it; ++k)
          dev::mbar_wait(&full[k % g.nst], (k / g.nst) & 1, nullptr, 200000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      // s32 accumulator, u8 A (zero point 128), s8 B, both K-major
      constexpr uint32_t idesc = dev::umma_idesc(2u, 0u, 1u, 0u, 0u, 128u, (uint32_t)BN);
      const uint64_t ad0 = dev::umma_sdesc(dev::smem_u32(sA), 16, 8 * CP, dev::UMMA_SW64);
      const uint64_t bd0 = dev::umma_sdesc(dev::smem_u32(sB), 16, 8 * CP, dev::UMMA_SW64);
      bool ok = dev::mbar_wait(b_full, 0, err);
      dev::tc_fence_after();
      uint32_t s = 0, ph = 0, local = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local % NBUF, use = local / NBUF;
        if (*abort_flag || !dev::mbar_wait(&tempty[buf], (use & 1) ^ 1, err) ||
            !dev::mbar_wait(&full[s], ph, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        const uint64_t as = ad0 + (uint64_t)((s * (uint32_t)slab_bytes) >> 4);
        int tap = 0;
        for (int kh = 0; kh < g.KH; ++kh) {
          for (int kw = 0; kw < g.KW; ++kw, ++tap) {
            const uint64_t ad = as + (uint64_t)(((kh * g.Wp + kw) * CP) >> 4);
            const uint64_t bd = bd0 + (uint64_t)((tap * C::TAPB) >> 4);
            dev::umma<dev::MmaKind::I8>(d, ad, bd, idesc, tap != 0);
            dev::umma<dev::MmaKind::I8>(d, ad + 2, bd + 2, idesc, 1u);  // bytes 32..63 of the row
          }
        }
        dev::umma_commit(&empty[s]);
        dev::umma_commit(&tfull[buf]);
        if (++s == (uint32_t)g.nst) {
          s = 0;
          ph ^= 1;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        dev::umma_commit(drain);
        dev::mbar_wait(drain, 0, nullptr, 200000000ull);
        for (int b = 0; b < NBUF; ++b) dev::mbar_arrive(&tfull[b]);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> dequantised fp32 output pixels
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int h = (warp - 2) >> 2;    // chunk parity: columns h*32 + 64*k
    ColSlice* my = col_slices + (warp - 2) * C::CHUNKS_PER_WARP;
#pragma unroll
    for (int k = 0; k < C::CHUNKS_PER_WARP; ++k)
      epi_stage_cols<EPI>(ep, h * 32 + 64 * k + lane, g.Cout, lane, my[k]);
    __syncwarp();
    uint32_t local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      const bool ok = dev::mbar_wait(&tfull[buf], use & 1, err);
      dev::tc_fence_after();
      if (!ok || *abort_flag) break;
      const unsigned r = (unsigned)t * BOX + (unsigned)(q * 32 + lane);
      const unsigned n = r / g.img_rows, qq = r - n * g.img_rows;
      const int oh = (int)(qq / (unsigned)g.Wp), ow = (int)qq - oh * g.Wp;
      const bool store = r < g.rows && oh < g.OH && ow < g.OW;
      const long long orow = ((long long)n * g.OH + oh) * g.OW + ow;
      bool zero_out = ep.zero_flag && *ep.zero_flag;
      float img_sa = 0.0f;
      if (ep.img_sa && store) {
        img_sa = ep.img_sa[n];
        zero_out = ep.img_zero[n] != 0;
      }
      float am = 0.0f;
#pragma unroll
      for (int k = 0; k < C::CHUNKS_PER_WARP; ++k) {
        const int c0 = h * 32 + 64 * k;
        if (c0 >= BN || c0 >= g.Cout) break;  // warp-uniform
        uint32_t v[32];
        dev::tmem_ld32(tmem + buf * BN + (uint32_t)c0 + ((uint32_t)(q * 32) << 16), v);
        dev::tmem_ld_wait();
        if (store) epi_store32<EPI>(ep, orow, c0, g.Cout, v, my[k], zero_out, img_sa, am);
      }
      if (ep.img_absmax) amax_flush(ep.img_absmax, store ? (int)n : -1, am);  // warp-uniform
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&tempty[buf]);
    }
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

static int h8_nbox(int KH, int KW, int Wp) {
  const long long span = 128LL + (long long)(KH - 1) * Wp + (KW - 1);
  return (int)((span + h8::BOX - 1) / h8::BOX);
}

static int h8_smem_fixed(int taps, int BN) {
  const int params = h8::EPI_WARPS * ((BN / 32 + 1) / 2) * (int)sizeof(ColSlice);
  return 1024 + taps * BN * h8::CP + h8::BAR_BYTES + h8::MISC + params;
}

bool conv_halo_i8_ok(int Cpad, int KH, int KW, int Cout, int stride, int Wp) {
  if (stride != 1 || Cpad != h8::CP || Cout < 1 || Cout > 128 || KH < 1 || KW < 1) return false;
  const int nbox = h8_nbox(KH, KW, Wp);
  if (nbox > h8::MAXBOX) return false;
  const int BN = Cout <= 64 ? 64 : 128;
  // at least two slab stages next to the resident weights
  return h8_smem_fixed(KH * KW, BN) + 2 * nbox * h8::BOXB <= h8::SMEM_MAX;
}

template <int BN, Epi EPI>
static bool launch_h8(Call& c, const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& ep,
                      H8Geom g, int tiles) {
  const int fixed = h8_smem_fixed(g.taps, BN);
  g.nst = (h8::SMEM_MAX - fixed) / (g.nbox * h8::BOXB);
  if (g.nst > h8::MAXST) g.nst = h8::MAXST;
  const int smem = fixed + g.nst * g.nbox * h8::BOXB;
  static bool attr_done[64] = {};
  const int dv = current_device();
  auto kern = conv_halo_i8_kernel<BN, EPI>;
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, h8::SMEM_MAX))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  const int grid = tiles < c.sm_count() ? tiles : c.sm_count();
  if (!ACF_CUDA_OK(launch_pdl(kern, dim3(grid), dim3(h8::THREADS), (size_t)smem, c.stream(), ta, tb, ep, g,
                              tiles, c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("conv_halo_i8_kernel");
}

bool conv_halo_i8_dev(Call& c, Epi epi, const uint8_t* A, const int8_t* wk, int N, int Hp, int Wp,
                      int KH, int KW, int OH, int OW, int Cout, const EpiParams& ep) {
  const long long rows = (long long)N * Hp * Wp;
  if (rows <= 0 || OH <= 0 || OW <= 0) return true;
  if (rows >= (1LL << 31) - 4096 || !conv_halo_i8_ok(h8::CP, KH, KW, Cout, 1, Wp) ||
      (epi != Epi::F32_AB && epi != Epi::I8_WINO)) {
    set_error(kInvalid, "%s: shape outside the narrow int8 kernel", c.name());
    c.fail();
    return false;
  }
  const int taps = KH * KW;
  const int BN = Cout <= 64 ? 64 : 128;
  CUtensorMap ta, tb;
  {
    const uint64_t d[2] = {(uint64_t)h8::CP, (uint64_t)rows};
    const uint64_t s[1] = {(uint64_t)h8::CP};
    const uint32_t b[2] = {(uint32_t)h8::CP, (uint32_t)h8::BOX};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, A, d, s, b, CU_TENSOR_MAP_SWIZZLE_64B)) {
      c.fail();
      return false;
    }
  }
  {
    // [Cout][taps*64] K-major; rows past Cout read as zero
    const uint64_t d[2] = {(uint64_t)taps * h8::CP, (uint64_t)Cout};
    const uint64_t s[1] = {(uint64_t)taps * h8::CP};
    const uint32_t b[2] = {(uint32_t)h8::CP, (uint32_t)BN};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, wk, d, s, b, CU_TENSOR_MAP_SWIZZLE_64B)) {
      c.fail();
      return false;
    }
  }
  H8Geom g;
  g.KH = KH;
  g.KW = KW;
  g.taps = taps;
  g.Wp = Wp;
  g.img_rows = (unsigned)(Hp * Wp);
  g.rows = (unsigned)rows;
  g.OH = OH;
  g.OW = OW;
  g.Cout = Cout;
  g.nbox = h8_nbox(KH, KW, Wp);
  g.nst = 0;
  const int tiles = (int)((rows + h8::BOX - 1) / h8::BOX);
  if (BN == 64)
    return epi == Epi::I8_WINO ? launch_h8<64, Epi::I8_WINO>(c, ta, tb, ep, g, tiles)
                               : launch_h8<64, Epi::F32_AB>(c, ta, tb, ep, g, tiles);
  return epi == Epi::I8_WINO ? launch_h8<128, Epi::I8_WINO>(c, ta, tb, ep, g, tiles)
                             : launch_h8<128, Epi::F32_AB>(c, ta, tb, ep, g, tiles);
}

}  // namespace acf
