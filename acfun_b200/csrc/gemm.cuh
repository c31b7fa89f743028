// gemm.cuh — host-side launch helpers around gemm_tc_kernel, shared by the GEMM, FC and
// convolution entry points.
#pragma once
#include "gemm_tc.cuh"
#include "runtime.cuh"

namespace acf {

// A device-resident GEMM operand: `rows x cols` elements with row stride `ld` (elements);
// for 3xTF32 operands a second (lo) copy lives `op_stride` elements after the first.
struct Operand {
  const void* p = nullptr;
  long long ld = 0;
  long long op_stride = 0;
};

// Make a byte / 16-bit / 32-bit matrix TMA-addressable: returns `src` when it is device
// memory with a 16-byte aligned base and a row pitch that is a multiple of 16 bytes,
// otherwise a zero-padded scratch copy (one 2D copy, host or device source).
Operand tma_operand(Call& c, const void* src, int rows, int cols, int elem);

// fp32 [rows][cols] (row stride lds) -> bf16 [rows][ldp], RNE as gemm_bf16_avx512.cpp:37-44.
Operand to_bf16(Call& c, const float* src_dev, int rows, int cols, long long lds);
// fp32 -> [2][rows][ldp] (hi = tf32-rounded, lo = tf32-rounded residual) for 3xTF32.
Operand to_tf32x2(Call& c, const float* src_dev, int rows, int cols, long long lds);

// fp32 [rows][cols] -> hi/lo pair at dst / dst + op_stride, row pitch ldp (multiple of 4),
// zero in the padding columns (defined in gemm.cu, used by to_tf32x2).
__global__ void k_to_tf32x2(const float* __restrict__ src, long long lds, int rows, int cols,
                            float* __restrict__ dst, long long ldp, long long op_stride);

enum class GemmKind { I8U, I8S, BF16, TF32X3, BF16X3 };

// fp32 math on tensor cores: 3xTF32 (tf32 hi/lo, ~2^-21 per product) or 3xBF16 (bf16 hi/lo on
// kind::f16: twice the MMA rate and half the operand bytes of 3xTF32, ~2^-17 per product).
// 3xBF16 is the default everywhere; ACFUN_FP32_MATH=tf32x3 (or acfun_set_fp32_math(1))
// selects 3xTF32.
enum class Fp32Math { TF32X3, BF16X3 };
enum class Fp32Use { GemmApi, Conv };
Fp32Math fp32_math(Fp32Use use);
// fp32 -> [2][rows][ldp] bf16 (hi, lo) for 3xBF16, ldp a multiple of 8; into scratch, or into
// `into` (bf16x2_bytes(rows, cols) bytes) when given, e.g. a model's cached weight split.
Operand to_bf16x2(Call& c, const float* src_dev, int rows, int cols, long long lds,
                  void* into = nullptr);
long long bf16x2_bytes(int rows, int cols);

// C-tile launch: chooses the tile width from the problem size and the SM count.
// With cg.enabled, A is a padded NHWC tensor [rows][cpad] and B the weights
// [taps][cpad][N] (implicit stride-1 convolution; K is then taps*cpad).
bool gemm_launch(Call& c, GemmKind kind, Epi epi, const Operand& A, const Operand& B, int M,
                 int N, int K, const EpiParams& ep, const ConvGeom& cg = ConvGeom{});
int gemm_bke(GemmKind kind);  // K elements per pipeline block (128 bytes)
// s8 x s8 -> requantised s8 on CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles, gemm_2sm.cu)
bool gemm_s8req_2sm(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                    const EpiParams& ep);
// the same 2-SM kernel for bf16 A [M][K] x bf16 B [K][N] with the fp32 bias / ReLU epilogue
bool gemm_bf16_2sm(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                   const EpiParams& ep);

// ---- tile table (acfun_autotune, tune.cu) ----
// Plain GEMMs (no implicit convolution, no remap / split / pool / maximum epilogue) of three
// families choose among several tile variants; the built-in choice is a size heuristic, and a
// table measured on this GPU by acfun_autotune overrides it per shape class (M, N, K rounded
// up to powers of two).
enum class TuneFamily : int { F32 = 0, BF16 = 1, I8 = 2 };
constexpr int kTuneVariants[3] = {6, 3, 2};
// F32 (3xBF16): 0 BN64 BKB128 | 1 BN64 BKB64 two sub-tiles | 2 BN128 BKB128 |
//               3 BN128 BKB64 two sub-tiles | 4 BN256 BKB64 | 5 split-K over 256x128 tiles
// BF16:         0 BN64 | 1 BN128 | 2 BN256
// I8:           0 BN128 | 1 BN256
bool tune_variant_valid(TuneFamily f, int v, int M, int N, int K);
// The table's variant for the shape class (or -1), or the variant the tuner forces on this
// thread while it measures.  The first lookup loads the table; with ACFUN_AUTOTUNE=1 and no
// table it measures one first, on the caller's stream.
int tune_variant(Call& c, TuneFamily f, int M, int N, int K);
void tune_force(int v);  // tuner only; -1 ends it

// u8 x s8 GEMM with a K-major B ([N][K] rows, ld = row pitch in bytes) and `bkb`-byte K
// blocks (64 or 128): tiles 64..256 wide, so narrow outputs (N <= 64) waste no MMA work.
// With cg.enabled, B is [N][taps*cpad] and cg.cblocks counts bkb-byte channel blocks.
// Epilogues: F32_AB, I8_WINO.
bool gemm_launch_i8k(Call& c, Epi epi, const Operand& A, const Operand& B, int M, int N, int K,
                     const EpiParams& ep, const ConvGeom& cg, int bkb);

// Narrow stride-1 int8 convolutions (conv_halo_i8.cu): A = the zero-point-padded u8 grid
// [N*Hp*Wp][64], wk = K-major s8 weights [Cout][KH*KW*64]; F32_AB or I8_WINO epilogue.
bool conv_halo_i8_ok(int Cpad, int KH, int KW, int Cout, int stride, int Wp);
bool conv_halo_i8_dev(Call& c, Epi epi, const uint8_t* A, const int8_t* wk, int N, int Hp, int Wp,
                      int KH, int KW, int OH, int OW, int Cout, const EpiParams& ep);
}  // namespace acf
