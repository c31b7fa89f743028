// gemm.cu — GEMM-family entry points and the tcgen05 GEMM launcher.
//
// Entry points (reference behaviour in brackets, hit-droid/Acfun paths):
//   acfun_gemm / acfun_gemm_epi   fp32, 3xBF16 (or 3xTF32)     [gemm.cpp:90-99,138-148]
//   acfun_gemm_bf16               bf16 RNE operands, f32 acc   [gemm_bf16_avx512.cpp:171-232]
//   acfun_gemm_int8               u8 x s8 -> s32, exact        [gemm_int8.cpp:45-50]
//   acfun_gemm_int8_epi           + (float)acc*alpha + beta    [gemm_int8.cpp:69-75]
//   acfun_gemm_s8_requant         s8 x s8 -> requantised s8    [no counterpart]
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "api_export.cuh"
#include "gemm.cuh"

namespace acf {

// ------------------------------------------------------------------ operand preparation
Operand tma_operand(Call& c, const void* src, int rows, int cols, int elem) {
  Operand o;
  if (!c.ok()) return o;
  const size_t pitch = (size_t)cols * elem;
  const bool dev = ptr_kind(src) == PtrKind::Device;
  if (dev && aligned16(src) && pitch % 16 == 0) {
    o.p = src;
    o.ld = cols;
    return o;
  }
  const size_t ldp = align_up(pitch, 16);
  void* d = c.scratch((size_t)rows * ldp);
  if (!d) return o;
  if (!ACF_CUDA_OK(cudaMemcpy2DAsync(d, ldp, src, pitch, pitch, rows, cudaMemcpyDefault,
                                     c.stream()))) {
    c.fail();
    return o;
  }
  if (!dev) c.note_host();
  o.p = d;
  o.ld = (long long)(ldp / elem);
  return o;
}

__device__ __forceinline__ uint16_t bf16_bits_ref(float f) {
  // gemm_bf16_avx512.cpp:37-44: add 0x7fff + lsb(bit 16), keep the top half (wrapping)
  const uint32_t x = __float_as_uint(f);
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float tf32_rne(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  u += 0xfffu + ((u >> 13) & 1u);
  return __uint_as_float(u & 0xffffe000u);
}

__global__ void k_to_tf32x2(const float* __restrict__ src, long long lds, int rows, int cols,
                            float* __restrict__ dst, long long ldp, long long op_stride) {
  dev::grid_dep_launch();  // the GEMM after it may start its prologue
  const long long groups = ldp / 4;
  const long long total = (long long)rows * groups;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const long long r = g / groups;
    const int j = (int)(g - r * groups) * 4;
    const float* s = src + r * lds;
    float hi[4], lo[4];
    if (j + 4 <= cols && ((reinterpret_cast<uintptr_t>(s + j) & 15) == 0)) {
      const float4 v = *reinterpret_cast<const float4*>(s + j);
      const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        hi[t] = tf32_rne(x[t]);
        lo[t] = tf32_rne(x[t] - hi[t]);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float x = (j + t < cols) ? s[j + t] : 0.0f;
        hi[t] = tf32_rne(x);
        lo[t] = tf32_rne(x - hi[t]);
      }
    }
    float* d = dst + r * ldp + j;
    *reinterpret_cast<float4*>(d) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<float4*>(d + op_stride) = make_float4(lo[0], lo[1], lo[2], lo[3]);
  }
}

static int ew_grid(Call& c, long long work) {
  long long b = (work + 255) / 256;
  long long cap = (long long)c.sm_count() * 8;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

// One launch converts one or two fp32 matrices (job 1's 8-column groups follow job 0's).
struct Bf16Job {
  const float* src;
  long long lds;
  int rows, cols;
  uint16_t* dst;
  long long ldp;
};
__global__ void k_to_bf16(Bf16Job j0, Bf16Job j1, long long g0, long long gt) {
  dev::grid_dep_launch();  // the GEMM after it may start its prologue
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < gt;
       g += (long long)gridDim.x * blockDim.x) {
    const bool sec = g >= g0;
    const float* src = sec ? j1.src : j0.src;
    const long long lds = sec ? j1.lds : j0.lds, ldp = sec ? j1.ldp : j0.ldp;
    const int cols = sec ? j1.cols : j0.cols;
    uint16_t* dst = sec ? j1.dst : j0.dst;
    const long long gg = sec ? g - g0 : g, groups = ldp / 8;
    const long long r = gg / groups;
    const int j = (int)(gg - r * groups) * 8;
    const float* s = src + r * lds + j;
    float v[8];
    if (j + 8 <= cols && (reinterpret_cast<uintptr_t>(s) & 15) == 0) {
      const float4 p = __ldg(reinterpret_cast<const float4*>(s));
      const float4 q = __ldg(reinterpret_cast<const float4*>(s + 4));
      v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
      v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = j + u < cols ? s[u] : 0.0f;
    }
    uint32_t w[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint16_t lo = j + 2 * t < cols ? bf16_bits_ref(v[2 * t]) : 0;
      const uint16_t hi = j + 2 * t + 1 < cols ? bf16_bits_ref(v[2 * t + 1]) : 0;
      w[t] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(dst + r * ldp + j) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
static bool bf16_job(Call& c, const float* src, int rows, int cols, long long lds, Bf16Job& j,
                     Operand& o) {
  const long long ldp = (long long)align_up((size_t)cols, 8);
  uint16_t* d = (uint16_t*)c.scratch((size_t)rows * ldp * 2);
  if (!d) return false;
  j = Bf16Job{src, lds, rows, cols, d, ldp};
  o.p = d;
  o.ld = ldp;
  return true;
}
Operand to_bf16(Call& c, const float* src, int rows, int cols, long long lds) {
  Operand o;
  Bf16Job j{};
  if (!c.ok() || !bf16_job(c, src, rows, cols, lds, j, o)) return Operand{};
  const long long g = (long long)rows * (j.ldp / 8);
  k_to_bf16<<<ew_grid(c, g), 256, 0, c.stream()>>>(j, j, g, g);
  if (!c.launched("k_to_bf16")) return Operand{};
  return o;
}

Operand to_tf32x2(Call& c, const float* src, int rows, int cols, long long lds) {
  Operand o;
  if (!c.ok()) return o;
  const long long ldp = (long long)align_up((size_t)cols, 4);
  float* d = (float*)c.scratch((size_t)2 * rows * ldp * 4);
  if (!d) return o;
  k_to_tf32x2<<<ew_grid(c, rows * (ldp / 4)), 256, 0, c.stream()>>>(src, lds, rows, cols, d, ldp,
                                                                      (long long)rows * ldp);
  if (!c.launched("k_to_tf32x2")) return o;
  o.p = d;
  o.ld = ldp;
  o.op_stride = (long long)rows * ldp;
  return o;
}

// 3xBF16 split: x = hi + lo + r with hi = bf16(x), lo = bf16(x - hi), |r| <= 2^-18 |x|;
// fp32 [rows][cols] -> [2][rows][ldp] bf16, zero padding (ldp a multiple of 8).  One launch
// splits one or two matrices (job 1's 4-column groups follow job 0's).
struct Bf16x2Job {
  const float* src;
  long long lds;
  int rows, cols;
  uint16_t* dst;
  long long ldp, op_stride;
};
__global__ void k_to_bf16x2(Bf16x2Job j0, Bf16x2Job j1, long long g0, long long gt) {
  dev::grid_dep_launch();  // the GEMM after it may start its prologue
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < gt;
       g += (long long)gridDim.x * blockDim.x) {
    const bool sec = g >= g0;
    const float* src = sec ? j1.src : j0.src;
    const long long lds = sec ? j1.lds : j0.lds, ldp = sec ? j1.ldp : j0.ldp;
    const int cols = sec ? j1.cols : j0.cols;
    uint16_t* dst = sec ? j1.dst : j0.dst;
    const long long ops = sec ? j1.op_stride : j0.op_stride;
    const long long gg = sec ? g - g0 : g, groups = ldp / 4;
    const long long r = gg / groups;
    const int j = (int)(gg - r * groups) * 4;
    const float* s = src + r * lds + j;
    float v[4];
    if (j + 4 <= cols && (reinterpret_cast<uintptr_t>(s) & 15) == 0) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(s));
      v[0] = q.x;
      v[1] = q.y;
      v[2] = q.z;
      v[3] = q.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = j + u < cols ? s[u] : 0.0f;
    }
    uint32_t h0, l0, h1, l1;
    nx_split_bf16x2(v[0], v[1], h0, l0);
    nx_split_bf16x2(v[2], v[3], h1, l1);
    *reinterpret_cast<uint2*>(dst + r * ldp + j) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(dst + ops + r * ldp + j) = make_uint2(l0, l1);
  }
}

long long bf16x2_bytes(int rows, int cols) {
  return 2LL * rows * (long long)align_up((size_t)cols, 8) * 2;
}

static bool bf16x2_job(Call& c, const float* src, int rows, int cols, long long lds, void* into,
                       Bf16x2Job& j, Operand& o) {
  const long long ldp = (long long)align_up((size_t)cols, 8);
  uint16_t* d = into ? (uint16_t*)into : (uint16_t*)c.scratch((size_t)2 * rows * ldp * 2);
  if (!d) return false;
  j = Bf16x2Job{src, lds, rows, cols, d, ldp, (long long)rows * ldp};
  o.p = d;
  o.ld = ldp;
  o.op_stride = (long long)rows * ldp;
  return true;
}

Operand to_bf16x2(Call& c, const float* src, int rows, int cols, long long lds, void* into) {
  Operand o;
  Bf16x2Job j{};
  if (!c.ok() || !bf16x2_job(c, src, rows, cols, lds, into, j, o)) return Operand{};
  const long long g = (long long)rows * (j.ldp / 4);
  k_to_bf16x2<<<ew_grid(c, g), 256, 0, c.stream()>>>(j, j, g, g);
  if (!c.launched("k_to_bf16x2")) return Operand{};
  return o;
}

// Both operands of a 3xBF16 GEMM in one launch.
static bool to_bf16x2_pair(Call& c, const float* a, int ar, int ac, long long lda, const float* b,
                           int br, int bc, long long ldb, Operand& oa, Operand& ob) {
  Bf16x2Job ja{}, jb{};
  if (!c.ok() || !bf16x2_job(c, a, ar, ac, lda, nullptr, ja, oa) ||
      !bf16x2_job(c, b, br, bc, ldb, nullptr, jb, ob))
    return false;
  const long long g0 = (long long)ar * (ja.ldp / 4), gt = g0 + (long long)br * (jb.ldp / 4);
  k_to_bf16x2<<<ew_grid(c, gt), 256, 0, c.stream()>>>(ja, jb, g0, gt);
  return c.launched("k_to_bf16x2");
}

// 0 (default) and 2: 3xBF16 everywhere; 1: 3xTF32 everywhere.  Initialised from
// ACFUN_FP32_MATH, changed by acfun_set_fp32_math.
static std::atomic<int> g_fp32_mode{-1};

static int fp32_mode() {
  int m = g_fp32_mode.load();
  if (m < 0) {
    const char* e = getenv("ACFUN_FP32_MATH");
    m = !e ? 0 : (!strcmp(e, "tf32x3") ? 1 : (!strcmp(e, "bf16x3") ? 2 : 0));
    int expect = -1;
    g_fp32_mode.compare_exchange_strong(expect, m);
    m = g_fp32_mode.load();
  }
  return m;
}

Fp32Math fp32_math(Fp32Use use) {
  const int m = fp32_mode();
  if (m == 1) return Fp32Math::TF32X3;
  if (m == 2) return Fp32Math::BF16X3;
  (void)use;
  return Fp32Math::BF16X3;
}

// Column split of the persistent walk's last wave (ConvGeom::nsplit): on unless
// ACFUN_TAIL_SPLIT=0.
// ACFUN_GEMM_2SM=0: plain GEMMs stay on one SM per tile instead of the SM-pair kernel
static bool two_sm_on() {
  static const bool on = [] {
    const char* e = getenv("ACFUN_GEMM_2SM");
    return !(e && !strcmp(e, "0"));
  }();
  return on;
}

static bool tail_split_on() {
  static const bool on = [] {
    const char* e = getenv("ACFUN_TAIL_SPLIT");
    return !(e && !strcmp(e, "0"));
  }();
  return on;
}

// ------------------------------------------------------------------ launcher
template <dev::MmaKind KIND, int BN, int STAGES, int NPASS, Epi EPI, bool AS, int BKB = 128,
          bool BKM = false, int MT = 1>
static bool launch_one(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                       const EpiParams& ep, const ConvGeom& cg) {
  using S = GemmShape<KIND, BN, STAGES, NPASS, BKB, BKM, MT>;
  static_assert(S::SMEM <= 232448, "shared memory budget");
  const CUtensorMapDataType dt = (KIND == dev::MmaKind::I8) ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : (KIND == dev::MmaKind::F16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap ta, tb;
  const uint64_t E = S::ELEM;
  const CUtensorMapSwizzle kswz =
      (BKB == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapSwizzle bswz = BKM ? kswz
                                  : (S::ELEM == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                   : CU_TENSOR_MAP_SWIZZLE_128B;
  if (MT == 2 && cg.enabled && cg.pair) {
    // row-pair view of the padded activation [pairs][2][Wp][cpad] (+ the hi / lo copy):
    // box = 1 parity x `by` pairs x 2^bxl columns x BKE channels = 128 rows
    const uint64_t C = (uint64_t)A.ld, Wp = (uint64_t)cg.Wp;
    const uint64_t dA[5] = {C, Wp, 2, (uint64_t)cg.npr, 2};
    const uint64_t sA[4] = {C * E, Wp * C * E, 2 * Wp * C * E, (uint64_t)A.op_stride * E};
    const uint32_t bA[5] = {(uint32_t)S::BKE, 1u << cg.bxl, 1u, (uint32_t)cg.by, 1u};
    const int rank = NPASS == 1 ? 4 : 5;
    if ((1 << cg.bxl) * cg.by != 128 || !encode_tmap(&ta, dt, rank, A.p, dA, sA, bA, kswz)) {
      set_error(kInvalid, "%s: row-pair tensor map", c.name());
      c.fail();
      return false;
    }
    if (NPASS == 1) {
      const uint64_t dB[2] = {BKM ? (uint64_t)K : (uint64_t)N, BKM ? (uint64_t)N : (uint64_t)K};
      const uint64_t sB[1] = {(uint64_t)B.ld * E};
      const uint32_t bB[2] = {BKM ? (uint32_t)S::BKE : (uint32_t)(128 / S::ELEM),
                              BKM ? (uint32_t)BN : (uint32_t)S::BKE};
      if (!encode_tmap(&tb, dt, 2, B.p, dB, sB, bB, bswz)) {
        c.fail();
        return false;
      }
    } else {
      const uint64_t dB[3] = {(uint64_t)N, (uint64_t)K, 2};
      const uint64_t sB[2] = {(uint64_t)B.ld * E, (uint64_t)B.op_stride * E};
      const uint32_t bB[3] = {(uint32_t)(128 / S::ELEM), (uint32_t)S::BKE, 1u};
      if (!encode_tmap(&tb, dt, 3, B.p, dB, sB, bB, bswz)) {
        c.fail();
        return false;
      }
    }
  } else if (NPASS == 1) {
    const uint64_t dA[2] = {(uint64_t)K, (uint64_t)M}, sA[1] = {(uint64_t)A.ld * E};
    const uint32_t bA[2] = {(uint32_t)S::BKE, 128u};
    // K-major B: [N][K] rows, one BN-row box; MN-major B: [K][N], 128-byte N chunks
    const uint64_t dB[2] = {BKM ? (uint64_t)K : (uint64_t)N, BKM ? (uint64_t)N : (uint64_t)K};
    const uint64_t sB[1] = {(uint64_t)B.ld * E};
    const uint32_t bB[2] = {BKM ? (uint32_t)S::BKE : (uint32_t)(128 / S::ELEM),
                            BKM ? (uint32_t)BN : (uint32_t)S::BKE};
    if (!encode_tmap(&ta, dt, 2, A.p, dA, sA, bA, kswz) ||
        !encode_tmap(&tb, dt, 2, B.p, dB, sB, bB, bswz)) {
      c.fail();
      return false;
    }
  } else {
    const uint64_t dA[3] = {(uint64_t)K, (uint64_t)M, 2};
    const uint64_t sA[2] = {(uint64_t)A.ld * E, (uint64_t)A.op_stride * E};
    const uint32_t bA[3] = {(uint32_t)S::BKE, 128u, 1u};
    const uint64_t dB[3] = {(uint64_t)N, (uint64_t)K, 2};
    const uint64_t sB[2] = {(uint64_t)B.ld * E, (uint64_t)B.op_stride * E};
    const uint32_t bB[3] = {(uint32_t)(128 / S::ELEM), (uint32_t)S::BKE, 1u};
    if (!encode_tmap(&ta, dt, 3, A.p, dA, sA, bA, kswz) ||
        !encode_tmap(&tb, dt, 3, B.p, dB, sB, bB, bswz)) {
      c.fail();
      return false;
    }
  }
  auto kern = gemm_tc_kernel<KIND, BN, STAGES, NPASS, EPI, AS, BKB, BKM, MT>;
  static bool attr_done[64] = {false};
  const int dv = current_device();
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  const long long tiles_mn = (long long)((M + S::BM - 1) / S::BM) * ((N + BN - 1) / BN);
  long long tiles = tiles_mn * ((!cg.enabled && cg.ksplit > 1) ? cg.ksplit : 1);
  if (tiles >= (1LL << 31)) {
    set_error(kInvalid, "%s: problem too large", c.name());
    c.fail();
    return false;
  }
  // the implicit convolution walks cpad channels per tap in blocks of this variant's BKE
  ConvGeom g = cg;
  if (g.enabled) g.cblocks = g.cpad / S::BKE;
  const int sms = c.sm_count();
  g.nsplit = 0;
  g.tfull = 0;
  if (MT == 1 && !BKM && !g.enabled && g.ksplit <= 1 && tail_split_on()) {
    // the last wave holds rem < sms tiles: run them as rem * ns column parts (whole B
    // chunks, >= 64 columns each) when those still fit in one wave
    const long long rem = tiles_mn % sms;
    int ns = 1;
    while (ns < 4 && S::NCHUNK % (2 * ns) == 0 && BN / (2 * ns) >= 64 && rem * 2 * ns <= sms)
      ns *= 2;
    if (rem > 0 && ns > 1) {
      g.nsplit = ns;
      g.tfull = (int)(tiles_mn - rem);
      tiles = g.tfull + rem * ns;
    }
  }
  // persistent: one CTA per SM (1 CTA/SM by shared memory), tiles strided over the grid
  const dim3 grid((unsigned)(tiles < sms ? tiles : sms));
  if (!ACF_CUDA_OK(launch_pdl(kern, dim3(grid), dim3(S::THREADS), (size_t)S::SMEM, c.stream(), ta, tb, ep, g,
                              M, N, K, c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("gemm_tc_kernel");
}

static long long tiles(int M, int N, int bn, int bm = 128) {
  return (long long)((M + bm - 1) / bm) * ((N + bn - 1) / bn);
}

// Split-K partial sums [S][M][N] -> out = act(sum_s part[s] + bias), summed in split order;
// VEC: 4 consecutive columns per thread (N and ldc multiples of 4, 16-byte aligned buffers).
template <bool VEC>
__global__ void k_splitk_reduce(const float* __restrict__ part, int S, int M, int N,
                                const float* __restrict__ bias, int act, float* __restrict__ out,
                                long long ldc) {
  const long long mn = (long long)M * N;
  constexpr int V = VEC ? 4 : 1;
  for (long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * V; i < mn;
       i += (long long)gridDim.x * blockDim.x * V) {
    const int m = (int)(i / N), n = (int)(i - (long long)m * N);
    float v[V];
    if constexpr (VEC) {
      const float4 p = *reinterpret_cast<const float4*>(part + i);
      v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
      for (int s = 1; s < S; ++s) {
        const float4 q = *reinterpret_cast<const float4*>(part + s * mn + i);
        v[0] = __fadd_rn(v[0], q.x); v[1] = __fadd_rn(v[1], q.y);
        v[2] = __fadd_rn(v[2], q.z); v[3] = __fadd_rn(v[3], q.w);
      }
    } else {
      v[0] = part[i];
      for (int s = 1; s < S; ++s) v[0] = __fadd_rn(v[0], part[s * mn + i]);
    }
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const float x = __fadd_rn(v[u], bias ? bias[n + u] : 0.0f);
      v[u] = act ? (x > 0.0f ? x : 0.0f) : x;
    }
    float* o = out + (long long)m * ldc + n;
    if constexpr (VEC)
      *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
    else
      o[0] = v[0];
  }
}

// 3xBF16 GEMMs with few output tiles and a long K (FC layers at small batch): K is split over
// 256x128 tiles so every SM streams a K range; fp32 partials, then k_splitk_reduce.
static bool gemm_bf16x3_splitk(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                               const EpiParams& ep, int tiles_mn) {
  using MK = dev::MmaKind;
  const int nkb = (K + 31) / 32;  // 64-byte bf16 K blocks
  int S = std::max(2, std::min(std::min(c.sm_count() / std::max(1, tiles_mn), nkb / 8), 16));
  const int per = (nkb + S - 1) / S;
  S = (nkb + per - 1) / per;  // no empty split
  float* part = static_cast<float*>(c.scratch((size_t)S * M * N * 4));
  if (!part) return false;
  EpiParams pe{};
  pe.C = part;
  pe.ldc = N;
  ConvGeom g{};
  g.ksplit = S;
  if (!launch_one<MK::F16, 128, 4, 3, Epi::F32_BIAS, false, 64, false, 2>(c, A, B, M, N, K, pe, g))
    return false;
  const long long mn = (long long)M * N;
  const bool vec = N % 4 == 0 && ep.ldc % 4 == 0 && aligned16(ep.C);
  const unsigned grid =
      (unsigned)std::min<long long>((mn / (vec ? 4 : 1) + 255) / 256, 16LL * c.sm_count());
  if (vec)
    k_splitk_reduce<true><<<grid, 256, 0, c.stream()>>>(part, S, M, N, ep.f0, ep.act,
                                                        static_cast<float*>(ep.C), ep.ldc);
  else
    k_splitk_reduce<false><<<grid, 256, 0, c.stream()>>>(part, S, M, N, ep.f0, ep.act,
                                                         static_cast<float*>(ep.C), ep.ldc);
  return c.launched("k_splitk_reduce");
}

int gemm_bke(GemmKind kind) {
  return (kind == GemmKind::BF16 || kind == GemmKind::BF16X3) ? 64
         : kind == GemmKind::TF32X3 ? 32 : 128;
}

template <Epi EPI>
static bool launch_i8k(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                       const EpiParams& ep, const ConvGeom& cg, int bkb) {
  using MK = dev::MmaKind;
  const int sms = c.sm_count();
  const int bn = N <= 64 ? 64 : (N <= 128 ? (tiles(M, N, 128) >= sms ? 128 : 64)
                                          : (tiles(M, N, 256) >= sms ? 256 : 128));
  if (bkb == 64) {
    if (bn == 64) return launch_one<MK::I8, 64, 16, 1, EPI, false, 64, true>(c, A, B, M, N, K, ep, cg);
    return launch_one<MK::I8, 128, 12, 1, EPI, false, 64, true>(c, A, B, M, N, K, ep, cg);
  }
  if (bn == 64) return launch_one<MK::I8, 64, 8, 1, EPI, false, 128, true>(c, A, B, M, N, K, ep, cg);
  if (bn == 128) return launch_one<MK::I8, 128, 6, 1, EPI, false, 128, true>(c, A, B, M, N, K, ep, cg);
  return launch_one<MK::I8, 256, 4, 1, EPI, false, 128, true>(c, A, B, M, N, K, ep, cg);
}

// Row-pair (pooled) implicit convolutions: two 128-row sub-tiles of 128 columns per CTA.
template <Epi EPI>
static bool launch_i8k_pair(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                            const EpiParams& ep, const ConvGeom& cg, int bkb) {
  using MK = dev::MmaKind;
  if (bkb == 64)
    return launch_one<MK::I8, 128, 8, 1, EPI, false, 64, true, 2>(c, A, B, M, N, K, ep, cg);
  return launch_one<MK::I8, 128, 4, 1, EPI, false, 128, true, 2>(c, A, B, M, N, K, ep, cg);
}

bool gemm_launch_i8k(Call& c, Epi epi, const Operand& A, const Operand& B, int M, int N, int K,
                     const EpiParams& ep, const ConvGeom& cg, int bkb) {
  if (!c.ok() || !A.p || !B.p || (bkb != 64 && bkb != 128)) {
    c.fail();
    return false;
  }
  if (cg.enabled && cg.pair && N <= 64) {
    set_error(kInvalid, "%s: row-pair int8 convolution needs more than 64 output channels", c.name());
    c.fail();
    return false;
  }
  switch (epi) {
    case Epi::F32_AB:
      return cg.pair ? launch_i8k_pair<Epi::F32_AB>(c, A, B, M, N, K, ep, cg, bkb)
                     : launch_i8k<Epi::F32_AB>(c, A, B, M, N, K, ep, cg, bkb);
    case Epi::I8_WINO:
      return cg.pair ? launch_i8k_pair<Epi::I8_WINO>(c, A, B, M, N, K, ep, cg, bkb)
                     : launch_i8k<Epi::I8_WINO>(c, A, B, M, N, K, ep, cg, bkb);
    default:
      set_error(kInvalid, "%s: unsupported int8 epilogue", c.name());
      c.fail();
      return false;
  }
}

bool gemm_launch(Call& c, GemmKind kind, Epi epi, const Operand& A, const Operand& B, int M,
                 int N, int K, const EpiParams& ep, const ConvGeom& cg) {
  if (!c.ok() || !A.p || !B.p) {
    c.fail();
    return false;
  }
  const int sms = c.sm_count();
  using MK = dev::MmaKind;
  // plain GEMMs may take the tile variant of the measured tile table (gemm.cuh)
  const bool plain = !cg.enabled && !ep.remap && !ep.split_out && !ep.pool4 && !ep.img_absmax;
  auto pick = [&](TuneFamily f) {
    const int v = plain ? tune_variant(c, f, M, N, K) : -1;
    return (v >= 0 && tune_variant_valid(f, v, M, N, K)) ? v : -1;
  };
  switch (kind) {
    case GemmKind::I8U: {
      const int v = pick(TuneFamily::I8);
      const bool wide = v >= 0 ? v == 1 : (N > 128 && tiles(M, N, 256) >= sms);
      switch (epi) {
        case Epi::S32:
          return wide ? launch_one<MK::I8, 256, 4, 1, Epi::S32, false>(c, A, B, M, N, K, ep, cg)
                      : launch_one<MK::I8, 128, 6, 1, Epi::S32, false>(c, A, B, M, N, K, ep, cg);
        case Epi::F32_AB:
          return wide ? launch_one<MK::I8, 256, 4, 1, Epi::F32_AB, false>(c, A, B, M, N, K, ep, cg)
                      : launch_one<MK::I8, 128, 6, 1, Epi::F32_AB, false>(c, A, B, M, N, K, ep, cg);
        case Epi::I8_WINO:
          return wide ? launch_one<MK::I8, 256, 4, 1, Epi::I8_WINO, false>(c, A, B, M, N, K, ep, cg)
                      : launch_one<MK::I8, 128, 6, 1, Epi::I8_WINO, false>(c, A, B, M, N, K, ep, cg);
        default:
          break;
      }
      break;
    }
    case GemmKind::I8S: {
      const int v = pick(TuneFamily::I8);
      const bool wide = v >= 0 ? v == 1 : (N > 128 && tiles(M, N, 256) >= sms);
      // plain requantising GEMMs that fill the GPU with 256 x 256 tiles: the 2-SM MMA
      if (epi == Epi::S8_REQ && plain && two_sm_on() && v < 0 && M >= 256 && N >= 256 &&
          tiles(M, N, 256, 256) * 2 >= sms)
        return gemm_s8req_2sm(c, A, B, M, N, K, ep);
      if (epi == Epi::S8_REQ)
        return wide ? launch_one<MK::I8, 256, 4, 1, Epi::S8_REQ, true>(c, A, B, M, N, K, ep, cg)
                    : launch_one<MK::I8, 128, 6, 1, Epi::S8_REQ, true>(c, A, B, M, N, K, ep, cg);
      break;
    }
    case GemmKind::BF16: {
      if (epi != Epi::F32_BIAS) break;
      const int v = pick(TuneFamily::BF16);
      // plain GEMMs with two or more waves of 256 x 256 tiles and a long K: the 2-SM MMA
      // (4096^3: 136 against 147 us per call; at K = 333 and 1.2 waves the 1-SM kernel wins)
      if (plain && two_sm_on() && v < 0 && M >= 256 && N >= 256 && K >= 1024 && tiles(M, N, 256, 256) >= sms)
        return gemm_bf16_2sm(c, A, B, M, N, K, ep);
      if (v == 2 || (v < 0 && N > 128 && tiles(M, N, 256) >= sms))
        return launch_one<MK::F16, 256, 4, 1, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
      if (v == 1 || (v < 0 && N > 64 && tiles(M, N, 128) >= sms))
        return launch_one<MK::F16, 128, 6, 1, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
      return launch_one<MK::F16, 64, 8, 1, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
    }
    case GemmKind::BF16X3: {
      if (epi != Epi::F32_BIAS) break;
      switch (pick(TuneFamily::F32)) {
        case 0:
          return launch_one<MK::F16, 64, 4, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
        case 1:
          return launch_one<MK::F16, 64, 5, 3, Epi::F32_BIAS, false, 64, false, 2>(c, A, B, M, N,
                                                                                  K, ep, cg);
        case 2:
          return launch_one<MK::F16, 128, 3, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
        case 3:
          return launch_one<MK::F16, 128, 4, 3, Epi::F32_BIAS, false, 64, false, 2>(c, A, B, M, N,
                                                                                   K, ep, cg);
        case 4:
          return launch_one<MK::F16, 256, 4, 3, Epi::F32_BIAS, false, 64>(c, A, B, M, N, K, ep, cg);
        case 5:
          return gemm_bf16x3_splitk(c, A, B, M, N, K, ep, (int)tiles(M, N, 128, 256));
        default:
          break;
      }
      if (plain && K >= 2048 && 2 * tiles(M, N, 128, 256) <= sms && (long long)M * N < (1LL << 31))
        return gemm_bf16x3_splitk(c, A, B, M, N, K, ep, (int)tiles(M, N, 128, 256));
      if (cg.enabled && cg.pair)  // row-pair (pooled) convolution: two sub-tiles per CTA
        return N > 64 ? launch_one<MK::F16, 128, 4, 3, Epi::F32_BIAS, false, 64, false, 2>(
                            c, A, B, M, N, K, ep, cg)
                      : launch_one<MK::F16, 64, 5, 3, Epi::F32_BIAS, false, 64, false, 2>(
                            c, A, B, M, N, K, ep, cg);
      // 256-column tiles in 64-byte K blocks: a quarter fewer operand bytes per MAC than
      // 128-column tiles (the 3xBF16 main loop is bound by shared-memory fill from L2)
      if (N > 128 && tiles(M, N, 256) >= sms)
        return launch_one<MK::F16, 256, 4, 3, Epi::F32_BIAS, false, 64>(c, A, B, M, N, K, ep, cg);
      // narrower N: two 128-row sub-tiles per CTA share each B stage, for the same bytes
      // per MAC as the 256-column tile
      if (N > 64 && tiles(M, N, 128, 256) >= sms)
        return launch_one<MK::F16, 128, 4, 3, Epi::F32_BIAS, false, 64, false, 2>(c, A, B, M, N, K,
                                                                                 ep, cg);
      if (N > 64 && tiles(M, N, 128) >= sms)
        return launch_one<MK::F16, 128, 3, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
      if (N > 32 && tiles(M, N, 64, 256) >= sms)
        return launch_one<MK::F16, 64, 5, 3, Epi::F32_BIAS, false, 64, false, 2>(c, A, B, M, N, K,
                                                                                ep, cg);
      return launch_one<MK::F16, 64, 4, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
    }
    case GemmKind::TF32X3: {
      if (epi != Epi::F32_BIAS) break;
      if (N > 64 && tiles(M, N, 128) >= sms)
        return launch_one<MK::TF32, 128, 3, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
      if (N > 32)
        return launch_one<MK::TF32, 64, 4, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
      return launch_one<MK::TF32, 32, 5, 3, Epi::F32_BIAS, false>(c, A, B, M, N, K, ep, cg);
    }
  }
  set_error(kInvalid, "%s: unsupported GEMM kind/epilogue combination", c.name());
  c.fail();
  return false;
}

// fp32 GEMM (+bias, +ReLU) on device operands, used by GEMM, FC and conv routes.
bool gemm_f32(Call& c, const float* dA, long long lda, const float* dB, long long ldb, int M,
              int N, int K, float* dC, long long ldc, const float* dbias, int act, Fp32Use use,
              const Operand* b_split) {
  const bool bf = fp32_math(use) == Fp32Math::BF16X3;
  Operand a, b;
  if (bf && !b_split) {
    if (!to_bf16x2_pair(c, dA, M, K, lda, dB, K, N, ldb, a, b)) return false;
  } else {
    a = bf ? to_bf16x2(c, dA, M, K, lda) : to_tf32x2(c, dA, M, K, lda);
    b = (bf && b_split) ? *b_split
                        : bf ? to_bf16x2(c, dB, K, N, ldb) : to_tf32x2(c, dB, K, N, ldb);
  }
  EpiParams ep{};
  ep.C = dC;
  ep.ldc = ldc;
  ep.f0 = dbias;
  ep.act = act;
  return gemm_launch(c, bf ? GemmKind::BF16X3 : GemmKind::TF32X3, Epi::F32_BIAS, a, b, M, N, K, ep);
}

}  // namespace acf

using namespace acf;

static bool bad_ptrs(const char* fn, const void* a, const void* b, const void* c) {
  if (!a || !b || !c) {
    set_error(kInvalid, "%s: NULL tensor argument", fn);
    return true;
  }
  return false;
}

extern "C" void acfun_gemm_epi(int M, int N, int K, const float* A, const float* B, float* C,
                               const float* bias, int act) {
  if (M <= 0 || N <= 0 || K <= 0 || bad_ptrs("acfun_gemm_epi", A, B, C)) return;
  Call c("acfun_gemm_epi");
  if (!c.ok()) return;
  const float* dA = (const float*)c.in(A, (size_t)M * K * 4);
  const float* dB = (const float*)c.in(B, (size_t)K * N * 4);
  const float* db = bias ? (const float*)c.in(bias, (size_t)N * 4) : nullptr;
  float* dC = (float*)c.out(C, (size_t)M * N * 4);
  if (!c.ok()) return;
  gemm_f32(c, dA, K, dB, N, M, N, K, dC, N, db, act ? 1 : 0, Fp32Use::GemmApi, nullptr);
  c.finish();
}

extern "C" void acfun_gemm(int M, int N, int K, const float* A, const float* B, float* C) {
  acfun_gemm_epi(M, N, K, A, B, C, nullptr, 0);
}

extern "C" void acfun_gemm_bf16(int M, int N, int K, const float* A, const float* B, float* C) {
  if (M <= 0 || N <= 0 || K <= 0 || bad_ptrs("acfun_gemm_bf16", A, B, C)) return;
  Call c("acfun_gemm_bf16");
  if (!c.ok()) return;
  const float* dA = (const float*)c.in(A, (size_t)M * K * 4);
  const float* dB = (const float*)c.in(B, (size_t)K * N * 4);
  float* dC = (float*)c.out(C, (size_t)M * N * 4);
  if (!c.ok()) return;
  // both operands converted in one launch
  Operand a, b;
  Bf16Job ja{}, jb{};
  if (!bf16_job(c, dA, M, K, K, ja, a) || !bf16_job(c, dB, K, N, N, jb, b)) {
    c.finish();
    return;
  }
  const long long g0 = (long long)M * (ja.ldp / 8), gt = g0 + (long long)K * (jb.ldp / 8);
  k_to_bf16<<<ew_grid(c, gt), 256, 0, c.stream()>>>(ja, jb, g0, gt);
  if (!c.launched("k_to_bf16")) {
    c.finish();
    return;
  }
  EpiParams ep{};
  ep.C = dC;
  ep.ldc = N;
  gemm_launch(c, GemmKind::BF16, Epi::F32_BIAS, a, b, M, N, K, ep);
  c.finish();
}

// Row-chunked GEMM call.  With host A and host C the rows are split into chunks (~2 MB of
// A each, at most 8) and chunk i's H2D (copy-in stream), GEMM (call stream) and D2H of its C
// rows (copy-out stream) overlap with the neighbouring chunks', so a host-buffer call costs
// about its PCIe transfer time instead of copies + math in series.  Otherwise one launch.
// B (and the epilogue's column vectors in `ep`) must already be staged on the call stream.
static void gemm_rows(Call& c, GemmKind kind, Epi epi, const void* A, int M, int K, int elemA,
                      const Operand& b, int N, EpiParams ep, void* C, int elemC) {
  if (!c.ok()) return;
  const size_t pitchA = (size_t)K * elemA, crow = (size_t)N * elemC;
  const bool host_io = ptr_kind(A) == PtrKind::Host && ptr_kind(C) == PtrKind::Host;
  const size_t want = ((size_t)M * pitchA) >> 21;
  const int nch_want = (int)(want > 8 ? 8 : want);
  if (!host_io || nch_want < 2 || M < 256) {
    Operand a = tma_operand(c, A, M, K, elemA);
    void* dC = c.out(C, (size_t)M * crow);
    if (!c.ok()) return;
    ep.C = dC;
    ep.ldc = N;
    gemm_launch(c, kind, epi, a, b, M, N, K, ep);
    return;
  }
  const size_t ldp = align_up(pitchA, 16);
  uint8_t* dA = (uint8_t*)c.scratch((size_t)M * ldp);
  uint8_t* dC = (uint8_t*)c.scratch((size_t)M * crow);
  if (!dA || !dC) return;
  const int R = (int)align_up((size_t)((M + nch_want - 1) / nch_want), 128);
  const int nch = (M + R - 1) / R;
  const cudaStream_t cs = c.stream(), hs = c.copy_in(), ds = c.copy_out();
  c.note_host();
  // the copy streams start behind the work already queued on the call stream (an earlier
  // call may still read this scratch) ...
  if (!ACF_CUDA_OK(cudaEventRecord(c.event(0), cs)) ||
      !ACF_CUDA_OK(cudaStreamWaitEvent(hs, c.event(0))) ||
      !ACF_CUDA_OK(cudaStreamWaitEvent(ds, c.event(0)))) {
    c.fail();
    return;
  }
  bool ok = true;
  for (int i = 0; ok && i < nch; ++i) {
    const int r0 = i * R, rows = (M - r0 < R) ? M - r0 : R;
    ok = ACF_CUDA_OK(cudaMemcpy2DAsync(dA + (size_t)r0 * ldp, ldp,
                                       (const uint8_t*)A + (size_t)r0 * pitchA, pitchA, pitchA,
                                       rows, cudaMemcpyHostToDevice, hs)) &&
         ACF_CUDA_OK(cudaEventRecord(c.event(2 + i), hs));
  }
  for (int i = 0; ok && i < nch; ++i) {
    const int r0 = i * R, rows = (M - r0 < R) ? M - r0 : R;
    ok = ACF_CUDA_OK(cudaStreamWaitEvent(cs, c.event(2 + i)));
    Operand a;
    a.p = dA + (size_t)r0 * ldp;
    a.ld = (long long)(ldp / elemA);
    EpiParams e = ep;
    e.C = dC + (size_t)r0 * crow;
    e.ldc = N;
    ok = ok && gemm_launch(c, kind, epi, a, b, rows, N, K, e) &&
         ACF_CUDA_OK(cudaEventRecord(c.event(2 + nch + i), cs)) &&
         ACF_CUDA_OK(cudaStreamWaitEvent(ds, c.event(2 + nch + i))) &&
         ACF_CUDA_OK(cudaMemcpyAsync((uint8_t*)C + (size_t)r0 * crow, dC + (size_t)r0 * crow,
                                     (size_t)rows * crow, cudaMemcpyDeviceToHost, ds));
  }
  // ... and the call stream ends behind both copy streams, on every path, so finish()'s
  // synchronise covers every copy that touches caller memory
  cudaEventRecord(c.event(1), hs);
  cudaStreamWaitEvent(cs, c.event(1));
  cudaEventRecord(c.event(1), ds);
  cudaStreamWaitEvent(cs, c.event(1));
  if (!ok) c.fail();
}

extern "C" void acfun_gemm_int8(int M, int N, int K, const uint8_t* A, const int8_t* B,
                                int32_t* C) {
  if (M <= 0 || N <= 0 || K <= 0 || bad_ptrs("acfun_gemm_int8", A, B, C)) return;
  Call c("acfun_gemm_int8");
  if (!c.ok()) return;
  Operand b = tma_operand(c, B, K, N, 1);
  gemm_rows(c, GemmKind::I8U, Epi::S32, A, M, K, 1, b, N, EpiParams{}, C, 4);
  c.finish();
}

extern "C" void acfun_gemm_int8_epi(int M, int N, int K, const uint8_t* A, const int8_t* B,
                                    float* C, const float* alpha, const float* beta, int act) {
  if (M <= 0 || N <= 0 || K <= 0 || bad_ptrs("acfun_gemm_int8_epi", A, B, C)) return;
  if (!alpha || !beta) {
    set_error(kInvalid, "acfun_gemm_int8_epi: alpha/beta must not be NULL");
    return;
  }
  Call c("acfun_gemm_int8_epi");
  if (!c.ok()) return;
  Operand b = tma_operand(c, B, K, N, 1);
  EpiParams ep{};
  ep.f0 = (const float*)c.in(alpha, (size_t)N * 4);
  ep.f1 = (const float*)c.in(beta, (size_t)N * 4);
  ep.act = act ? 1 : 0;
  gemm_rows(c, GemmKind::I8U, Epi::F32_AB, A, M, K, 1, b, N, ep, C, 4);
  c.finish();
}

extern "C" void acfun_gemm_s8_requant(int M, int N, int K, const int8_t* A, const int8_t* B,
                                      const int32_t* bias, const float* scale, int8_t* C,
                                      int act) {
  if (M <= 0 || N <= 0 || K <= 0 || bad_ptrs("acfun_gemm_s8_requant", A, B, C)) return;
  if (!scale) {
    set_error(kInvalid, "acfun_gemm_s8_requant: scale must not be NULL");
    return;
  }
  Call c("acfun_gemm_s8_requant");
  if (!c.ok()) return;
  Operand b = tma_operand(c, B, K, N, 1);
  EpiParams ep{};
  ep.f0 = (const float*)c.in(scale, (size_t)N * 4);
  ep.i0 = bias ? (const int32_t*)c.in(bias, (size_t)N * 4) : nullptr;
  ep.act = act ? 1 : 0;
  gemm_rows(c, GemmKind::I8S, Epi::S8_REQ, A, M, K, 1, b, N, ep, C, 1);
  c.finish();
}

extern "C" int acfun_set_fp32_math(int mode) {
  if (mode < 0 || mode > 2) {
    set_error(kInvalid, "acfun_set_fp32_math: mode must be 0, 1 or 2");
    return kInvalid;
  }
  fp32_mode();
  g_fp32_mode.store(mode);
  return 0;
}
