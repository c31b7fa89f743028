// gemm_tc.cuh — tcgen05 (5th-gen tensor core) GEMM for sm_100a.
//
// One CTA computes a 128 x BN tile of C = A[M,K] * B[K,N]:
//   warp 0        TMA producer: per 128-byte (SW128) or 64-byte (SW64) K block, the A tile
//                 (128 rows, K-major) and the B tile (K rows x BN MN-major in 128-byte N
//                 chunks, or BN rows K-major like A) into a STAGES-deep shared-memory ring
//                 guarded by full/empty mbarriers;
//   warp 1        TMEM owner + single-thread UMMA issuer (cta_group::1, M=128, N=BN),
//                 one MMA per 32-byte K-step; tcgen05.commit frees a stage as soon
//                 as its MMAs retire and finally signals the epilogue;
//   warps 2..9    epilogue: tcgen05.ld 32 columns at a time from their TMEM lane quadrant
//                 (two warps per quadrant, even / odd 32-column chunks),
//                 fused epilogue (int32 store / dequant mul+add / requant to s8 / bias +
//                 ReLU / int8-Winograd dequant fma), vectorised global stores.
// 3xTF32 (NPASS = 3): A and B arrive as [2][rows][cols] (hi, lo) pairs; each K-step issues
// lo*hi + hi*lo + hi*hi into the same fp32 accumulator.
//
// Rows of C may be remapped (implicit convolution over a padded NHWC tensor): GEMM row r
// is output pixel r when remap is off; otherwise r indexes the padded grid and only rows
// that land on a real output pixel are stored.
#pragma once
#include "numerics.cuh"
#include "ptx.cuh"

namespace acf {

enum class Epi : int { S32 = 0, F32_AB = 1, S8_REQ = 2, F32_BIAS = 3, I8_WINO = 4 };

struct EpiParams {
  void* C;               // output base
  long long ldc;         // output row stride in elements
  const float* f0;       // F32_AB alpha | S8_REQ scale | I8_WINO wso | F32_BIAS bias
  const float* f1;       // F32_AB beta  | I8_WINO bias
  const int32_t* i0;     // S8_REQ int32 bias | I8_WINO column sums of the u8-zp weights
  int act;
  // implicit-convolution row remap (remap != 0): GEMM row r -> image n = r / img_rows,
  // q = r % img_rows, oh = q / Wp, ow = q % Wp; stored iff oh < OH && ow < OW at
  // output row (n*OH + oh)*OW + ow.
  int remap;
  int img_rows, Wp, OH, OW;
  // when non-NULL and *zero_flag != 0 every stored value is 0 (int8 router: max|x| < 1e-12)
  const int* zero_flag;
  // int8 convolution over a batch with one activation scale per image (batch-1 semantics):
  // image n = r / img_rows (remap or not); F32_AB and I8_WINO then take f0 = per-column
  // weight scale, f1 = bias (or NULL), i0 = column sums, and derive alpha / beta / wso from
  // img_sa[n] in the same expressions the single-call router precomputes; img_zero[n]
  // replaces zero_flag.
  const float* img_sa;
  const int* img_zero;
  // F32_BIAS with split_out (implicit convolution only): the result is written as its bf16
  // hi / lo split -- the 3xBF16 operand of the next convolution -- into that convolution's
  // zero-padded input planes instead of C: output pixel (n, oh, ow), channel j at element
  // ((n*sHp + oh + spad)*sWp + ow + spad)*sC + j of the hi plane; the lo plane follows
  // split_plane elements later.
  void* split_out;
  long long split_plane;
  int sHp, sWp, spad, sC;
  // F32_BIAS with pool4 (plain GEMM rows, no remap): rows come in groups of four, the 2x2
  // window of one pooled pixel; the group's maximum is biased / activated and stored as
  // pooled row r/4 -- of a ph x pw grid per image when it goes to split_out.
  int pool4;
  int ph, pw;
  // when non-NULL (float epilogues): img_absmax[n] = max(img_absmax[n], max |stored value| of
  // image n = r / img_rows), an atomicMax on the bits of a non-negative float -- the next int8
  // convolution's per-image activation maximum, folded into the producer.
  unsigned* img_absmax;
};

// Implicit convolution (stride 1) over a padded NHWC tensor viewed as A[rows][Cpad]:
// K block kb = (tap, channel block); the A rows are shifted by kh*Wp + kw and the B rows
// (weights [taps][Cpad][Cout]) start at tap*Cpad.
struct ConvGeom {
  int enabled;
  int cblocks;  // Cpad / BKE
  int KW;
  int Wp;
  int cpad;     // channels per tap in B
  int taps;
  // Row-pair tiling (MT = 2; a convolution followed by a 2x2 / stride-2 max-pool): A is viewed
  // as [pairs][2][Wp][cpad] (padded rows 2p, 2p+1; the hi / lo copy outermost for 3xBF16) and
  // a tile is `by` pairs x 2^bxl columns of output pixels, sub-tile i holding the rows of
  // parity i, so each 2x2 window sits in lanes (l, l^1) of the two sub-tiles.  xb = column
  // blocks per pair block, hp2 = pairs per image (Hp / 2), npr = pairs in the tensor.
  int pair, bxl, by, xb, hp2, npr;
  // Split-K (plain GEMMs only): tile t covers K blocks of split t / (tiles_m*tiles_n), whose
  // raw accumulator goes to rows ks*M + r of C (partials [ksplit][M][ldc], summed by the caller)
  int ksplit;
  // Column split of the last wave (plain GEMMs, MT = 1, MN-major B): tiles [0, tfull) run
  // whole; each remaining tile -- the last, partial wave of the persistent walk -- becomes
  // nsplit units of BN / nsplit columns (the same K loop and MMA per column, so the same
  // bits), which spreads that wave over up to nsplit times as many SMs.
  int nsplit, tfull;
};

// One unit of a CTA's persistent walk: a whole tile, one split-K slice of it, or column part
// `part` (>= 0) of a last-wave tile; K blocks [kb0, kb1).
struct TileUnit {
  int tt, ks, kb0, kb1, part;
};

__device__ __forceinline__ TileUnit tile_unit(int t, int tiles_mn, int nkb_all, int nkb_s,
                                              int nsplit, int tfull) {
  TileUnit u;
  if (nsplit > 1 && t >= tfull) {
    const int v = t - tfull;
    u.tt = tfull + v / nsplit;
    u.part = v - (u.tt - tfull) * nsplit;
    u.ks = 0;
    u.kb0 = 0;
    u.kb1 = nkb_all;
  } else {
    u.tt = t % tiles_mn;
    u.ks = t / tiles_mn;
    u.part = -1;
    u.kb0 = u.ks * nkb_s;
    u.kb1 = min(nkb_all, u.kb0 + nkb_s);
  }
  return u;
}

// Per-column epilogue parameters of one 32-column chunk, staged in the epilogue warp's own
// shared-memory slice: pa / pb (float) and pc (int32), 32 entries each, zero past column N.
//   S8_REQ: pa = scale, pc = int32 bias | F32_AB: pa = alpha, pb = beta | F32_BIAS: pa = bias
//   I8_WINO: pa = wso, pb = bias, pc = column sums of the weights
struct ColSlice {
  float a[32];
  float b[32];
  int32_t c[32];
};

template <dev::MmaKind KIND>
struct KindTraits;
template <>
struct KindTraits<dev::MmaKind::I8> {
  static constexpr int ELEM = 1;
};
template <>
struct KindTraits<dev::MmaKind::F16> {
  static constexpr int ELEM = 2;
};
template <>
struct KindTraits<dev::MmaKind::TF32> {
  static constexpr int ELEM = 4;
};

// BKB_ = K bytes per pipeline block (128: SW128 K-major rows; 64: SW64, for operands whose
// K run per tap is 64 bytes).  B_KMAJ: B is stored [N][K] (K contiguous) and loaded like A as
// one BN-row tile; otherwise B is [K][N] (MN-major) and loaded in 128-byte N chunks.
// MT: 128-row sub-tiles per CTA tile (BM = 128*MT); they share every B stage, each with its
// own TMEM accumulator (MT*BN columns), which divides the B bytes per MAC by MT.
template <dev::MmaKind KIND, int BN, int STAGES, int NPASS, int BKB_ = 128, bool B_KMAJ = false,
          int MT_ = 1>
struct GemmShape {
  static constexpr int ELEM = KindTraits<KIND>::ELEM;
  static constexpr int MT = MT_;
  static constexpr int BM = 128 * MT;
  static constexpr int BKB = BKB_;                     // K bytes per block
  static constexpr int BKE = BKB / ELEM;               // K elements per block
  static constexpr int KSTEPS = BKB / 32;              // 32-byte MMA K-steps per block
  static constexpr int NOPS = (NPASS == 3) ? 2 : 1;    // hi/lo operand copies
  static constexpr int A_TILE = 128 * BKB;             // one sub-tile
  static constexpr int A_OP = MT * A_TILE;               // all sub-tiles of one operand copy
  static constexpr uint32_t K_LAYOUT = (BKB == 128) ? dev::UMMA_SW128 : dev::UMMA_SW64;
  static constexpr int K_SBO = 8 * BKB;                // 8-row core-matrix group stride
  static constexpr int NCHUNK = B_KMAJ ? 1 : BN * ELEM / 128;  // TMA boxes per B tile
  static constexpr int CHUNK_B = B_KMAJ ? BN * BKB : BKE * 128;
  static constexpr int B_TILE = NCHUNK * CHUNK_B;
  static constexpr int STAGE = NOPS * (A_OP + B_TILE);
  // B descriptor advance per MMA K-step
  static constexpr int KSTEP_B = B_KMAJ ? 32 : (32 / ELEM) * 128;
  // MN-major 32-bit (tf32) operands only exist in the 128B swizzle with 32-byte atoms
  // (4-row / 512-byte pattern, TMA SWIZZLE_128B_ATOM_32B); 8/16-bit use the 128B swizzle
  // with 16-byte atoms (8-row / 1024-byte pattern).  K-major B uses A's layout.
  static constexpr uint32_t B_LAYOUT =
      B_KMAJ ? K_LAYOUT : (ELEM == 4) ? dev::UMMA_SW128_B32 : dev::UMMA_SW128;
  static constexpr int B_SBO = B_KMAJ ? K_SBO : (ELEM == 4) ? 512 : 1024;
  static constexpr int B_LBO = B_KMAJ ? 16 : CHUNK_B;
  static constexpr int ACC_COLS = MT * BN;   // one accumulator buffer
  // accumulator buffers in TMEM: 4 when they fit (short-K tiles then keep the MMA several
  // tiles ahead of the epilogue), else 2
  static constexpr int NBUF = ACC_COLS <= 128 ? 4 : 2;
  static constexpr int TMEM_COLS = NBUF * ACC_COLS;
  // warps 0 (TMA) and 1 (MMA / TMEM), then EPI_WARPS epilogue warps: two per TMEM lane
  // quadrant, splitting the tile's 32-column chunks between them (even / odd chunks)
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int CHUNKS_PER_WARP = (BN / 32 + 1) / 2;
  // full/empty per stage, tfull[2], tempty[2], drain; TMEM slot; abort flag
  static constexpr int BAR_BYTES = ((2 * STAGES + 2 * NBUF + 1) * 8 + 8 + 15) / 16 * 16;
  static constexpr int PARAM_BYTES = EPI_WARPS * CHUNKS_PER_WARP * (int)sizeof(ColSlice);
  static constexpr int SMEM = 1024 + STAGES * STAGE + BAR_BYTES + PARAM_BYTES;
  static_assert(BKB == 128 || (BKB == 64 && (B_KMAJ ? NPASS == 1 : ELEM == 2)),
                "64-byte K blocks: K-major int8 B or MN-major bf16 B");
  static_assert(B_KMAJ || BN * ELEM % 128 == 0, "B tile must be whole 128-byte chunks");
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "TMEM columns");
  static_assert((MT == 1 || MT == 2 || MT == 4) && TMEM_COLS <= 512, "TMEM capacity");
};

__device__ __forceinline__ float relu_max(float v) { return v > 0.0f ? v : 0.0f; }

template <Epi EPI>
__device__ __forceinline__ void epi_stage_cols(const EpiParams& ep, int col, int N, int lane,
                                               ColSlice& s) {
  const bool in = col < N;
  if constexpr (EPI == Epi::S8_REQ) {
    s.a[lane] = in ? ep.f0[col] : 0.0f;
    s.c[lane] = (in && ep.i0) ? ep.i0[col] : 0;
  } else if constexpr (EPI == Epi::F32_AB) {
    s.a[lane] = in ? ep.f0[col] : 0.0f;
    s.b[lane] = (in && ep.f1) ? ep.f1[col] : 0.0f;
    s.c[lane] = (in && ep.i0) ? ep.i0[col] : 0;
  } else if constexpr (EPI == Epi::F32_BIAS) {
    s.a[lane] = (in && ep.f0) ? ep.f0[col] : 0.0f;
  } else if constexpr (EPI == Epi::I8_WINO) {
    s.a[lane] = in ? ep.f0[col] : 0.0f;
    s.b[lane] = (in && ep.f1) ? ep.f1[col] : 0.0f;
    s.c[lane] = in ? ep.i0[col] : 0;
  }
}

template <typename T>
__device__ __forceinline__ void lds32(const T* p, T (&o)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint4 u = *reinterpret_cast<const uint4*>(p + i);  // warp-wide broadcast
    o[i] = __builtin_bit_cast(T, u.x);
    o[i + 1] = __builtin_bit_cast(T, u.y);
    o[i + 2] = __builtin_bit_cast(T, u.z);
    o[i + 3] = __builtin_bit_cast(T, u.w);
  }
}

// Fold one warp's row maxima (lane's image n, or -1 for a row it does not store) into
// img_absmax: one atomic per warp when the rows share an image.
__device__ __forceinline__ void amax_flush(unsigned* img_absmax, int n, float am) {
  const int n0 = __shfl_sync(0xffffffffu, n, 0);
  if (__all_sync(0xffffffffu, n == n0 || n < 0)) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(0xffffffffu, am, o);
      am = (am < u) ? u : am;
    }
    if ((threadIdx.x & 31) == 0 && n0 >= 0 && am > 0.0f) atomicMax(&img_absmax[n0], __float_as_uint(am));
  } else if (n >= 0 && am > 0.0f) {
    atomicMax(&img_absmax[n], __float_as_uint(am));
  }
}

// The float epilogues' values for 32 columns j0..j0+31 of one row (F32_AB, F32_BIAS, I8_WINO):
// dequantisation / bias, act, the all-zero override; folds max |value| into am when the
// per-image maximum is wanted.  epi_store32 stores them; kernels that stage rows in shared
// memory call it directly.
template <Epi EPI>
__device__ __forceinline__ void epi_values32(const EpiParams& ep, int j0, int N, const uint32_t (&r)[32],
                                             const ColSlice& P, bool zero, float img_sa, float& am,
                                             float (&v)[32]) {
  float p0[32], p1[32];
  int32_t pi[32];
  if constexpr (EPI == Epi::F32_AB) {
    lds32(P.a, p0);
    lds32(P.b, p1);
    if (ep.img_sa) {
      // alpha = sa*ws, beta = bias - (alpha*128)*Sw: k_int8_colparams's expressions
      lds32(P.c, pi);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = __fmul_rn(img_sa, p0[i]);
        p1[i] = __fsub_rn(p1[i], __fmul_rn(__fmul_rn(a, 128.0f), (float)pi[i]));
        p0[i] = a;
      }
    }
  } else if constexpr (EPI == Epi::F32_BIAS) {
    lds32(P.a, p0);
  } else {  // I8_WINO
    lds32(P.a, p0);
    lds32(P.b, p1);
    lds32(P.c, pi);
    if (ep.img_sa) {
      // wso = (sa*0.25)*ws (winograd_int8.cpp:155)
      const float q = __fmul_rn(img_sa, 0.25f);
#pragma unroll
      for (int i = 0; i < 32; ++i) p0[i] = __fmul_rn(q, p0[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float x;
    if constexpr (EPI == Epi::F32_AB) {
      x = __fadd_rn(__fmul_rn(__int2float_rn((int32_t)r[i]), p0[i]), p1[i]);
    } else if constexpr (EPI == Epi::F32_BIAS) {
      x = __fadd_rn(__uint_as_float(r[i]), p0[i]);
    } else {  // I8_WINO
      const int32_t c = (int32_t)r[i] - 128 * pi[i];
      x = __fmaf_rn(__fmul_rn(4.0f, __int2float_rn(c)), p0[i], p1[i]);
    }
    if (ep.act) x = relu_max(x);
    v[i] = zero ? 0.0f : x;
  }
  if (ep.img_absmax) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (j0 + i < N) amax_acc(am, v[i]);
  }
}

template <Epi EPI>
__device__ __forceinline__ void epi_store32(const EpiParams& ep, long long orow, int j0, int N,
                                            const uint32_t (&r)[32], const ColSlice& P,
                                            bool zero, float img_sa, float& am) {
  // 32 outputs for columns j0..j0+31 of output row `orow`
  const bool full = (j0 + 32 <= N);
  if constexpr (EPI == Epi::S32) {
    int32_t* dst = reinterpret_cast<int32_t*>(ep.C) + orow * ep.ldc + j0;
    if (full && ((reinterpret_cast<uintptr_t>(dst) & 31) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) dev::st_global_v8(dst + i, r + i);
    } else if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<uint4*>(dst + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (j0 + i < N) dst[i] = (int32_t)r[i];
    }
  } else if constexpr (EPI == Epi::S8_REQ) {
    float sc[32];
    int32_t bi[32];
    lds32(P.a, sc);
    lds32(P.c, bi);
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      uint32_t w = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int32_t s = (int32_t)((uint32_t)r[i + t] + (uint32_t)bi[i + t]);
        float v = __fmul_rn(__int2float_rn(s), sc[i + t]);
        if (ep.act) v = relu_max(v);
        int q = __float2int_rn(v);
        q = q > 127 ? 127 : (q < -128 ? -128 : q);
        w |= (uint32_t)(q & 0xFF) << (8 * t);
      }
      packed[i / 4] = w;
    }
    int8_t* dst = reinterpret_cast<int8_t*>(ep.C) + orow * ep.ldc + j0;
    if (full && ((reinterpret_cast<uintptr_t>(dst) & 31) == 0)) {
      dev::st_global_v8(dst, packed);  // one 32-byte store: a whole sector per lane
    } else if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      *reinterpret_cast<uint4*>(dst + 16) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (j0 + i < N) dst[i] = (int8_t)((packed[i / 4] >> (8 * (i % 4))) & 0xFF);
    }
  } else {
    float v[32];
    epi_values32<EPI>(ep, j0, N, r, P, zero, img_sa, am, v);
    if constexpr (EPI == Epi::F32_BIAS) {
      if (ep.split_out) {
        // hi = bf16(v), lo = bf16(v - hi): the split k_pad_split4 makes of an fp32 input
        uint16_t* hi = reinterpret_cast<uint16_t*>(ep.split_out) + orow * ep.ldc + j0;
        uint16_t* lo = hi + ep.split_plane;
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) nx_split_bf16x2(v[i], v[i + 1], ph[i / 2], pl[i / 2]);
        if (full && ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 31) == 0) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            dev::st_global_v8(hi + 16 * q, ph + 8 * q);
            dev::st_global_v8(lo + 16 * q, pl + 8 * q);
          }
        } else if (full) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            reinterpret_cast<uint4*>(hi)[q] = make_uint4(ph[4 * q], ph[4 * q + 1], ph[4 * q + 2], ph[4 * q + 3]);
            reinterpret_cast<uint4*>(lo)[q] = make_uint4(pl[4 * q], pl[4 * q + 1], pl[4 * q + 2], pl[4 * q + 3]);
          }
        } else {
          for (int i = 0; i < 32; ++i)
            if (j0 + i < N) {
              hi[i] = (uint16_t)(ph[i / 2] >> (16 * (i & 1)));
              lo[i] = (uint16_t)(pl[i / 2] >> (16 * (i & 1)));
            }
        }
        return;
      }
    }
    float* dst = reinterpret_cast<float*>(ep.C) + orow * ep.ldc + j0;
    if (full && ((reinterpret_cast<uintptr_t>(dst) & 31) == 0)) {
      // 32-byte stores: a whole sector per lane
#pragma unroll
      for (int i = 0; i < 32; i += 8) dev::st_global_v8(dst + i, reinterpret_cast<const uint32_t*>(v + i));
    } else if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (j0 + i < N) dst[i] = v[i];
    }
  }
}

// Window maximum of two accumulator words: fp32 (F32_BIAS) or int32 (F32_AB, I8_WINO, whose
// dequantisation is non-decreasing in the accumulator -- every scale is >= 0 -- so the maximum
// may be taken before it; bias and ReLU are monotone too).
template <Epi EPI>
__device__ __forceinline__ uint32_t acc_max(uint32_t a, uint32_t b) {
  if constexpr (EPI == Epi::F32_BIAS)
    return __float_as_uint(fmaxf(__uint_as_float(a), __uint_as_float(b)));
  else
    return (int32_t)a > (int32_t)b ? a : b;
}

// Pooled epilogue: NC columns j0..j0+NC-1 of pooled row `orow` from window maxima m (accumulator
// words), the columns' parameters at P.{a,b,c}[cs..cs+NC); epi_store32's arithmetic per EPI.
template <Epi EPI, int NC>
__device__ __forceinline__ void epi_store_pool(const EpiParams& ep, long long orow, int j0, int N,
                                               const uint32_t (&m)[NC], const ColSlice& P, int cs,
                                               bool zero, float img_sa, float& am) {
  static_assert(EPI == Epi::F32_BIAS || EPI == Epi::F32_AB || EPI == Epi::I8_WINO, "float out");
  float v[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    float x;
    if constexpr (EPI == Epi::F32_BIAS) {
      x = __fadd_rn(__uint_as_float(m[i]), P.a[cs + i]);
    } else if constexpr (EPI == Epi::F32_AB) {
      float a = P.a[cs + i], b = P.b[cs + i];
      if (ep.img_sa) {
        a = __fmul_rn(img_sa, a);
        b = __fsub_rn(b, __fmul_rn(__fmul_rn(a, 128.0f), (float)P.c[cs + i]));
      }
      x = __fadd_rn(__fmul_rn(__int2float_rn((int32_t)m[i]), a), b);
    } else {
      float w = P.a[cs + i];
      if (ep.img_sa) w = __fmul_rn(__fmul_rn(img_sa, 0.25f), w);
      const int32_t c = (int32_t)m[i] - 128 * P.c[cs + i];
      x = __fmaf_rn(__fmul_rn(4.0f, __int2float_rn(c)), w, P.b[cs + i]);
    }
    if (ep.act) x = relu_max(x);
    v[i] = zero ? 0.0f : x;
  }
  if (ep.img_absmax) {
#pragma unroll
    for (int i = 0; i < NC; ++i)
      if (j0 + i < N) amax_acc(am, v[i]);
  }
  const bool full = j0 + NC <= N;
  if constexpr (EPI == Epi::F32_BIAS) {
    if (ep.split_out) {
      uint16_t* hi = reinterpret_cast<uint16_t*>(ep.split_out) + orow * ep.ldc + j0;
      uint16_t* lo = hi + ep.split_plane;
      uint32_t ph[NC / 2], pl[NC / 2];
#pragma unroll
      for (int i = 0; i < NC; i += 2) nx_split_bf16x2(v[i], v[i + 1], ph[i / 2], pl[i / 2]);
      if (NC % 16 == 0 && full && ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 31) == 0) {
#pragma unroll
        for (int q = 0; q < NC / 16; ++q) {
          dev::st_global_v8(hi + 16 * q, ph + 8 * q);
          dev::st_global_v8(lo + 16 * q, pl + 8 * q);
        }
      } else if (full && ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) == 0) {
#pragma unroll
        for (int q = 0; q < NC / 8; ++q) {
          reinterpret_cast<uint4*>(hi)[q] = make_uint4(ph[4 * q], ph[4 * q + 1], ph[4 * q + 2], ph[4 * q + 3]);
          reinterpret_cast<uint4*>(lo)[q] = make_uint4(pl[4 * q], pl[4 * q + 1], pl[4 * q + 2], pl[4 * q + 3]);
        }
      } else {
        for (int i = 0; i < NC; ++i)
          if (j0 + i < N) {
            hi[i] = (uint16_t)(ph[i / 2] >> (16 * (i & 1)));
            lo[i] = (uint16_t)(pl[i / 2] >> (16 * (i & 1)));
          }
      }
      return;
    }
  }
  float* dst = reinterpret_cast<float*>(ep.C) + orow * ep.ldc + j0;
  if (NC % 8 == 0 && full && (reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
#pragma unroll
    for (int q = 0; q < NC / 8; ++q) dev::st_global_v8(dst + 8 * q, reinterpret_cast<const uint32_t*>(v + 8 * q));
  } else if (full && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < NC / 4; ++q)
      reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    for (int i = 0; i < NC; ++i)
      if (j0 + i < N) dst[i] = v[i];
  }
}

// Persistent kernel: grid = min(#tiles, #SMs); CTA b walks tiles b, b+grid, ...  The smem
// ring runs continuously across tiles, and the accumulator has NBUF buffers in TMEM
// (NBUF x MT*BN columns): the UMMA warp fills buffer i % NBUF while the epilogue warps drain
// the earlier ones, so a tile's epilogue overlaps the next tiles' MMAs.
template <dev::MmaKind KIND, int BN, int STAGES, int NPASS, Epi EPI, bool A_SIGNED, int BKB = 128,
          bool B_KMAJ = false, int MT = 1>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   EpiParams ep, ConvGeom cg, int M, int N, int K, unsigned* err) {
  using S = GemmShape<KIND, BN, STAGES, NPASS, BKB, B_KMAJ, MT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;     // [NBUF] accumulator ready for the epilogue
  uint64_t* tempty_bar = tfull_bar + S::NBUF;   // [NBUF] accumulator drained
  uint64_t* drain_bar = tempty_bar + S::NBUF;   // error-path MMA drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  ColSlice* col_slices = reinterpret_cast<ColSlice*>(smem + STAGES * S::STAGE + S::BAR_BYTES);
  static_assert(S::THREADS == 320, "launch bounds");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (M + S::BM - 1) / S::BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_mn = tiles_m * tiles_n;
  const int ksplit = (!cg.enabled && cg.ksplit > 1) ? cg.ksplit : 1;
  const int nsplit =
      (MT == 1 && !B_KMAJ && !cg.enabled && ksplit == 1 && cg.nsplit > 1) ? cg.nsplit : 0;
  const int num_tiles = nsplit ? cg.tfull + (tiles_mn - cg.tfull) * nsplit : tiles_mn * ksplit;
  const int nkb_all = cg.enabled ? cg.taps * cg.cblocks : (K + S::BKE - 1) / S::BKE;
  const int nkb_s = (nkb_all + ksplit - 1) / ksplit;  // K blocks per split

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(&full_bar[s], 1);
      dev::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < S::NBUF; ++b) {
      dev::mbar_init(&tfull_bar[b], 1);
      dev::mbar_init(&tempty_bar[b], S::EPI_WARPS);  // one arrive per epilogue warp
    }
    dev::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmA);
    dev::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    dev::tmem_alloc(tmem_slot, S::TMEM_COLS);
    dev::tmem_relinquish();
  }
  // launched as a programmatic dependent: the prologue above (barriers, tensor memory) may
  // overlap the previous kernel; nothing it produced is read, and nothing is written, before this
  dev::grid_dep_wait();
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    // The loop body is one thread's serial instruction stream, so it carries no divisions:
    // ring slot / phase and the convolution's (tap, channel block) advance incrementally.
    uint32_t it = 0;  // global K-block counter (ring position)
    uint32_t s = 0, ph = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < num_tiles && !stop; t += gridDim.x) {
      if (*abort_flag) break;
      const TileUnit u = tile_unit(t, tiles_mn, nkb_all, nkb_s, nsplit, cg.tfull);
      const int tt = u.tt;
      // a column part loads the first NCHUNK / nsplit B chunks of its own column range
      const int nch = u.part >= 0 ? S::NCHUNK / nsplit : S::NCHUNK;
      const uint32_t stage_bytes =
          u.part >= 0 ? (uint32_t)(S::NOPS * (S::A_OP + nch * S::CHUNK_B)) : (uint32_t)S::STAGE;
      const int m0 = (tt / tiles_n) * S::BM;
      const int n0 = (tt % tiles_n) * BN + (u.part > 0 ? u.part * (BN / nsplit) : 0);
      const int kb0 = u.kb0, nkb = u.kb1;
      // conv: channel block, kw, kh, A row shift, B k
      int cb = 0, kw = 0, kh = 0, row_off = 0, tap_k = 0;
      int pr0 = 0, px0 = 0;  // row-pair tiling: first pair and first column of the tile
      if (MT == 2 && cg.pair) {
        const int tm = tt / tiles_n, pb = tm / cg.xb;
        pr0 = pb * cg.by;
        px0 = (tm - pb * cg.xb) << cg.bxl;
      }
      for (int kb = kb0; kb < nkb; ++kb) {
        if (!dev::mbar_wait(&empty_bar[s], ph ^ 1, err)) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        uint8_t* st = smem + s * S::STAGE;
        dev::mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
        int kx, ay, by;
        const int akw = kw, akh = kh;  // this block's tap
        if (cg.enabled) {
          kx = cb * S::BKE;
          ay = m0 + row_off;
          by = tap_k + kx;
          if (++cb == cg.cblocks) {
            cb = 0;
            tap_k += cg.cpad;
            ++row_off;
            if (++kw == cg.KW) {
              kw = 0;
              ++kh;
              row_off += cg.Wp - cg.KW;
            }
          }
        } else {
          kx = kb * S::BKE;
          ay = m0;
          by = kx;
        }
#pragma unroll
        for (int op = 0; op < S::NOPS; ++op) {
          uint8_t* a_dst = st + op * S::A_OP;
          uint8_t* b_dst = st + S::NOPS * S::A_OP + op * S::B_TILE;
          bool a_done = false;
          if constexpr (MT == 2) {
            if (cg.pair) {
              // output rows 2p + i read padded rows 2p + i + kh: pair p + (i+kh)/2, parity (i+kh)&1
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int pi = i + akh;
                if constexpr (S::NOPS == 1)
                  dev::tma_load_4d(a_dst + i * S::A_TILE, &tmA, &full_bar[s], kx, px0 + akw,
                                   pi & 1, pr0 + (pi >> 1));
                else
                  dev::tma_load_5d(a_dst + i * S::A_TILE, &tmA, &full_bar[s], kx, px0 + akw,
                                   pi & 1, pr0 + (pi >> 1), op);
              }
              a_done = true;
            }
          }
          if constexpr (B_KMAJ) {
            if (!a_done) {
#pragma unroll
              for (int i = 0; i < MT; ++i)
                dev::tma_load_2d(a_dst + i * S::A_TILE, &tmA, &full_bar[s], kx, ay + 128 * i);
            }
            dev::tma_load_2d(b_dst, &tmB, &full_bar[s], by, n0);
          } else if constexpr (S::NOPS == 1) {
            if (!a_done) {
#pragma unroll
              for (int i = 0; i < MT; ++i)
                dev::tma_load_2d(a_dst + i * S::A_TILE, &tmA, &full_bar[s], kx, ay + 128 * i);
            }
#pragma unroll
            for (int c = 0; c < S::NCHUNK; ++c)
              if (c < nch)
                dev::tma_load_2d(b_dst + c * S::CHUNK_B, &tmB, &full_bar[s],
                                 n0 + c * (128 / S::ELEM), by);
          } else {
            if (!a_done) {
#pragma unroll
              for (int i = 0; i < MT; ++i)
                dev::tma_load_3d(a_dst + i * S::A_TILE, &tmA, &full_bar[s], kx, ay + 128 * i, op);
            }
#pragma unroll
            for (int c = 0; c < S::NCHUNK; ++c)
              if (c < nch)
                dev::tma_load_3d(b_dst + c * S::CHUNK_B, &tmB, &full_bar[s],
                                 n0 + c * (128 / S::ELEM), by, op);
          }
        }
        ++it;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    if (*abort_flag) {
      // drain copies that may still be in flight before the CTA releases its smem
      const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
      for (uint32_t k = first; k < it; ++k)
        dev::mbar_wait(&full_bar[k % STAGES], (k / STAGES) & 1, nullptr, 200000000ull);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer
    constexpr uint32_t c_fmt = (KIND == dev::MmaKind::I8) ? 2u : 1u;
    constexpr uint32_t a_fmt = (KIND == dev::MmaKind::I8) ? (A_SIGNED ? 1u : 0u)
                               : (KIND == dev::MmaKind::F16) ? 1u : 2u;
    constexpr uint32_t b_fmt = (KIND == dev::MmaKind::I8) ? 1u
                               : (KIND == dev::MmaKind::F16) ? 1u : 2u;
    constexpr uint32_t idesc_full =
        dev::umma_idesc(c_fmt, a_fmt, b_fmt, 0u, B_KMAJ ? 0u : 1u, 128u, (uint32_t)BN);
    const uint32_t idesc_part = nsplit ? dev::umma_idesc(c_fmt, a_fmt, b_fmt, 0u, B_KMAJ ? 0u : 1u,
                                                         128u, (uint32_t)(BN / nsplit))
                                       : idesc_full;
    // Shared-memory descriptors are built once; a stage / K-step / operand offset is an add
    // to the 14-bit start-address field (addresses are below 256 KB, so it never carries).
    const uint32_t smem_base = dev::smem_u32(smem);
    const uint64_t a_desc0 = dev::umma_sdesc(smem_base, 16, S::K_SBO, S::K_LAYOUT);
    const uint64_t b_desc0 = dev::umma_sdesc(smem_base + S::NOPS * S::A_OP, S::B_LBO, S::B_SBO,
                                             S::B_LAYOUT);
    bool ok = true;
    uint32_t it = 0, local = 0;
    uint32_t s = 0, ph = 0;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
      const uint32_t buf = local % S::NBUF, use = local / S::NBUF;
      if (*abort_flag || !dev::mbar_wait(&tempty_bar[buf], (use & 1) ^ 1, err)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      const uint32_t d_tmem = tmem + buf * S::ACC_COLS;
      const TileUnit u = tile_unit(t, tiles_mn, nkb_all, nkb_s, nsplit, cg.tfull);
      const int kb0 = u.kb0, nkb = u.kb1;
      const uint32_t idesc = u.part >= 0 ? idesc_part : idesc_full;  // N = this unit's columns
      for (int kb = kb0; kb < nkb; ++kb, ++it) {
        if (!dev::mbar_wait(&full_bar[s], ph, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint64_t soff = (uint64_t)((s * (uint32_t)S::STAGE) >> 4);
#pragma unroll
        for (int ks = 0; ks < S::KSTEPS; ++ks) {
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            if constexpr (NPASS == 1) {
              const uint64_t ad = a_desc0 + soff + (uint64_t)((i * S::A_TILE + ks * 32) / 16);
              const uint64_t bd = b_desc0 + soff + (uint64_t)(ks * S::KSTEP_B / 16);
              dev::umma<KIND>(d_tmem + i * BN, ad, bd, idesc, ((kb - kb0) | ks) != 0);
            } else {
              // (a_op, b_op): lo*hi, hi*lo, hi*hi
              const int aop[3] = {1, 0, 0}, bop[3] = {0, 1, 0};
#pragma unroll
              for (int p = 0; p < 3; ++p) {
                const uint64_t ad = a_desc0 + soff +
                                    (uint64_t)((aop[p] * S::A_OP + i * S::A_TILE + ks * 32) / 16);
                const uint64_t bd =
                    b_desc0 + soff + (uint64_t)((bop[p] * S::B_TILE + ks * S::KSTEP_B) / 16);
                dev::umma<KIND>(d_tmem + i * BN, ad, bd, idesc, ((kb - kb0) | ks | p) != 0);
              }
            }
          }
        }
        dev::umma_commit(&empty_bar[s]);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1;
        }
      }
      if (ok) dev::umma_commit(&tfull_bar[buf]);
    }
    if (!ok) {
      *abort_flag = 1;
      dev::umma_commit(drain_bar);
      dev::mbar_wait(drain_bar, 0, nullptr, 200000000ull);
      for (int b = 0; b < S::NBUF; ++b)
        dev::mbar_arrive(&tfull_bar[b]);  // release epilogue warps (they see abort_flag)
    }
  } else if (warp >= 2) {
    // ---------------- epilogue
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int h = (warp - 2) >> 2;    // chunk parity: columns h*32 + 64*k
    ColSlice* my = col_slices + (warp - 2) * S::CHUNKS_PER_WARP;
    uint32_t local = 0;
    int staged_n0 = -1;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local % S::NBUF, use = local / S::NBUF;
      const TileUnit u = tile_unit(t, tiles_mn, nkb_all, nkb_s, nsplit, cg.tfull);
      const int tt = u.tt, ksp = u.ks;
      const int nw = u.part >= 0 ? BN / nsplit : BN;  // this unit's columns
      const int m0 = (tt / tiles_n) * S::BM;
      const int n0 = (tt % tiles_n) * BN + (u.part > 0 ? u.part * nw : 0);
      if constexpr (EPI != Epi::S32) {
        // per-column parameters of this tile's chunks, loaded before the accumulator is
        // ready (and only when the column block changes)
        if (n0 != staged_n0) {
          __syncwarp();
#pragma unroll
          for (int k = 0; k < S::CHUNKS_PER_WARP; ++k)
            epi_stage_cols<EPI>(ep, n0 + h * 32 + 64 * k + lane, N, lane, my[k]);
          __syncwarp();
          staged_n0 = n0;
        }
      }
      const bool ok = dev::mbar_wait(&tfull_bar[buf], use & 1, err);
      dev::tc_fence_after();
      if (!ok || *abort_flag) break;
      if constexpr (MT == 2 && (EPI == Epi::F32_BIAS || EPI == Epi::F32_AB ||
                                EPI == Epi::I8_WINO)) {
        if (cg.pair) {
          // Row-pair tile: lane l of both sub-tiles is output pixel (2*pr + i, x) with pr =
          // pr0 + l / 2^bxl, x = x0 + l % 2^bxl; the 2x2 window of pooled pixel (pr, x/2) is
          // lanes (l, l^1) of the two sub-tiles.
          const int tm = tt / tiles_n, pb = tm / cg.xb;
          const int l = q * 32 + lane, lby = l >> cg.bxl;
          const int pr = pb * cg.by + lby;
          const int xx = ((tm - pb * cg.xb) << cg.bxl) + (l & ((1 << cg.bxl) - 1));
          const int n = pr / cg.hp2, py = pr - n * cg.hp2, px = xx >> 1;
          const bool store = lby < cg.by && pr < cg.npr && py < ep.ph && px < ep.pw;
          const long long orow = ep.split_out
                                     ? ((long long)n * ep.sHp + py + ep.spad) * ep.sWp + px + ep.spad
                                     : ((long long)n * ep.ph + py) * ep.pw + px;
          bool zero_out = ep.zero_flag && *ep.zero_flag;
          float img_sa = 0.0f;
          if (ep.img_sa && store) {
            img_sa = ep.img_sa[n];
            zero_out = ep.img_zero[n] != 0;
          }
          float am = 0.0f;
          const int hs = lane & 1;  // this lane keeps columns 16*hs..16*hs+15 of each chunk
#pragma unroll 1
          for (int k = 0; k < S::CHUNKS_PER_WARP; ++k) {
            const int c0 = h * 32 + 64 * k;
            if (c0 >= BN || n0 + c0 >= N) break;  // warp-uniform
            uint32_t v0[32], v1[32];
            const uint32_t ta = tmem + buf * S::ACC_COLS + (uint32_t)c0 + ((uint32_t)(q * 32) << 16);
            dev::tmem_ld32(ta, v0);
            dev::tmem_ld32(ta + BN, v1);
            dev::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) v0[j] = acc_max<EPI>(v0[j], v1[j]);
            uint32_t m16[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t send = hs ? v0[j] : v0[16 + j], keep = hs ? v0[16 + j] : v0[j];
              m16[j] = acc_max<EPI>(keep, __shfl_xor_sync(0xffffffffu, send, 1));
            }
            if (store)
              epi_store_pool<EPI, 16>(ep, orow, n0 + c0 + 16 * hs, N, m16, my[k], 16 * hs, zero_out,
                                      img_sa, am);
          }
          if (ep.img_absmax) amax_flush(ep.img_absmax, store ? n : -1, am);  // warp-uniform
          dev::tc_fence_before();
          __syncwarp();
          if (lane == 0) dev::mbar_arrive(&tempty_bar[buf]);
          continue;
        }
      }
#pragma unroll 1
      for (int i = 0; i < MT; ++i) {  // 128-row sub-tiles
        const int r = m0 + 128 * i + q * 32 + lane;
        bool zero_out = ep.zero_flag && *ep.zero_flag;
        float img_sa = 0.0f;
        long long orow = r + (long long)ksp * M;  // split-K partial rows
        bool store = r < M;
        if (ep.img_sa && store) {
          const int n = r / ep.img_rows;
          img_sa = ep.img_sa[n];
          zero_out = ep.img_zero[n] != 0;
        }
        if (ep.remap && store) {
          const int n = r / ep.img_rows, qq = r - n * ep.img_rows;
          const int oh = qq / ep.Wp, ow = qq - oh * ep.Wp;
          store = (oh < ep.OH) && (ow < ep.OW);
          orow = ep.split_out ? ((long long)n * ep.sHp + oh + ep.spad) * ep.sWp + ow + ep.spad
                              : ((long long)n * ep.OH + oh) * ep.OW + ow;
        }
        if (ep.pool4) {
          const int P = r >> 2;
          orow = P;
          if (ep.split_out) {
            const int per = ep.ph * ep.pw, n = P / per, rem = P - n * per, py = rem / ep.pw;
            orow = ((long long)n * ep.sHp + py + ep.spad) * ep.sWp + (rem - py * ep.pw) + ep.spad;
          }
        }
        float am = 0.0f;  // this row's max |stored value| (img_absmax)
        const int nimg = (ep.img_absmax && store) ? r / ep.img_rows : -1;
#pragma unroll 1
        for (int k = 0; k < S::CHUNKS_PER_WARP; ++k) {
          const int c0 = h * 32 + 64 * k;
          if (c0 >= nw || n0 + c0 >= N) break;  // warp-uniform
          uint32_t v[32];
          dev::tmem_ld32(
              tmem + buf * S::ACC_COLS + (uint32_t)(i * BN + c0) + ((uint32_t)(q * 32) << 16), v);
          dev::tmem_ld_wait();
          if constexpr (EPI == Epi::F32_BIAS) {
            if (ep.pool4) {
              // warp-uniform.  The window's four rows are lanes 4g..4g+3: a reduce-scatter
              // over them leaves lane 4g+s with the maxima of columns 8s..8s+7.
              const int s4 = lane & 3;
              const bool up = (s4 & 2) != 0, odd = (s4 & 1) != 0;
              uint32_t k16[16], m8[8];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t send = up ? v[j] : v[16 + j], keep = up ? v[16 + j] : v[j];
                k16[j] = acc_max<EPI>(keep, __shfl_xor_sync(0xffffffffu, send, 2));
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t send = odd ? k16[j] : k16[8 + j], keep = odd ? k16[8 + j] : k16[j];
                m8[j] = acc_max<EPI>(keep, __shfl_xor_sync(0xffffffffu, send, 1));
              }
              if (store)
                epi_store_pool<EPI, 8>(ep, orow, n0 + c0 + 8 * s4, N, m8, my[k], 8 * s4, zero_out,
                                       img_sa, am);
              continue;
            }
          }
          if (store) epi_store32<EPI>(ep, orow, n0 + c0, N, v, my[k], zero_out, img_sa, am);
        }
        if (ep.img_absmax) amax_flush(ep.img_absmax, nimg, am);  // warp-uniform
      }
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0) dev::mbar_arrive(&tempty_bar[buf]);
    }
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace acf
