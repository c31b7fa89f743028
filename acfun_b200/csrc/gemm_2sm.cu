// gemm_2sm.cu — GEMMs on the 2-SM tensor-core MMA: a cluster of two CTAs on two SMs computes one
// 256 x 256 tile (tcgen05.mma.cta_group::2, M = 256, N = 256), each CTA staging its 128 rows of
// A and its 128 columns of B, so a pipeline stage is 32 KB per CTA instead of the 48 KB a 128 x
// 256 tile on one SM needs: six stages in flight instead of four, and half the B bytes per SM
// per MAC.  Two instances: s8 x s8 with the requantising epilogue
// (C[s8] = sat(rne(relu((acc + bias) * scale))), the bench headline) and bf16 x bf16 with the
// fp32 bias / ReLU epilogue (acfun_gemm_bf16).  A stage holds 128 bytes of K either way (128
// int8 or 64 bf16 elements); a CTA's 128 columns of B are one 128-byte swizzle atom wide for
// int8 and two for bf16.
//   warp 0      both CTAs: TMA producer for its own A rows / B columns; the copies complete
//               on the leader CTA's (rank 0) full barrier (cp.async.bulk.tensor.cta_group::2),
//               whose expect-tx covers both CTAs' bytes
//   warp 1      both CTAs: tensor-memory allocation (cta_group::2, same warp in each CTA);
//               leader lane 0: the MMA issuer; its commits arrive on the barrier of that name
//               in both CTAs (multicast), freeing both CTAs' stages / accumulators
//   warps 2..9  both CTAs: epilogue over the CTA's own 128 accumulator rows x 256 columns, the
//               arithmetic of gemm_tc_kernel's epilogue; each warp arrives on the leader's
//               accumulator-empty barrier when it has drained a buffer
// The pair walks 256 x 256 tiles persistently (grid = 2 x the number of SM pairs used).
// No load uses cluster multicast: each CTA fetches its own operand halves.  Every wait is
// bounded (ptx.cuh); on expiry the error word is flagged and both CTAs drain and exit.
#include <algorithm>

#include "api_export.cuh"
#include "gemm.cuh"

namespace acf {
namespace g2 {
constexpr int BM = 128;                 // A rows per CTA
constexpr int BN = 256;                 // accumulator columns (128 of B staged per CTA)
constexpr int BK = 128;                 // K bytes per stage
constexpr int STAGES = 6;
constexpr int A_STAGE = BM * BK;        // 16 KB
constexpr int B_STAGE = BK * (BN / 2);  // 16 KB: this CTA's 128 columns x 128 bytes of K
constexpr int STAGE = A_STAGE + B_STAGE;
constexpr int NBUF = 2;
constexpr int TMEM_COLS = NBUF * BN;    // 512
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int CHUNKS_PER_WARP = BN / 32 / 2;
// full[S], empty[S], tfull[2], tempty[2], drain
constexpr int BAR_BYTES = ((2 * STAGES + 2 * NBUF + 1) * 8 + 8 + 15) / 16 * 16;
constexpr int PARAM_BYTES = EPI_WARPS * CHUNKS_PER_WARP * (int)sizeof(ColSlice);
constexpr int SMEM = 1024 + STAGES * STAGE + BAR_BYTES + PARAM_BYTES;
static_assert(SMEM <= 232448, "shared memory");
// shared::cta address of a barrier with this bit cleared = the leader CTA's barrier at the same
// offset (the CTA-pair addressing of sm_100 clusters)
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;

// Per-kind stage geometry: K elements per stage, 128-byte B column chunks per CTA (MN-major
// B, one TMA box and one swizzle atom each) and the B descriptor advance per 32-byte K-step.
template <dev::MmaKind KIND>
struct Kind2 {
  static constexpr int ELEM = KIND == dev::MmaKind::I8 ? 1 : 2;
  static constexpr int KE = BK / ELEM;
  static constexpr int B_CHUNKS = (BN / 2) * ELEM / 128;
  static constexpr int B_CHUNK = KE * 128;
  static constexpr int CHUNK_COLS = 128 / ELEM;
  static constexpr int KSTEP_B = (32 / ELEM) * 128;
  static constexpr uint32_t C_FMT = KIND == dev::MmaKind::I8 ? 2u : 1u;  // s32 / f32 accumulator
  static constexpr uint32_t AB_FMT = 1u;                                  // s8 / bf16 operands
  static_assert(B_CHUNKS * B_CHUNK == B_STAGE, "stage layout");
};
}  // namespace g2

namespace dev2 {
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   dev::smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// TMA 2D load into this CTA's shared memory whose completion is counted on the leader's barrier
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint64_t* bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dev::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(dev::smem_u32(bar) & g2::kPeerBitMask), "r"(x), "r"(y)
      : "memory");
}
template <dev::MmaKind KIND>
__device__ __forceinline__ void umma2(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                      uint32_t accumulate) {
  if constexpr (KIND == dev::MmaKind::I8)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive (once) on `bar` in both CTAs of the pair when the issued MMAs are done
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          dev::smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// arrive (once) on the leader's `bar` when the issued MMAs are done
__device__ __forceinline__ void umma2_commit_leader(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   dev::smem_u32(bar))
               : "memory");
}
// arrive on the leader CTA's barrier at the offset of `bar`
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(dev::smem_u32(bar) & g2::kPeerBitMask)
               : "memory");
}
}  // namespace dev2

template <dev::MmaKind KIND, Epi EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(g2::THREADS, 1)
    gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    EpiParams ep, int M, int N, int K, unsigned* err) {
  using namespace g2;
  using KT = Kind2<KIND>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + NBUF;
  uint64_t* drain_bar = tempty_bar + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  ColSlice* col_slices = reinterpret_cast<ColSlice*>(smem + STAGES * STAGE + BAR_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = dev2::cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_m = (M + 2 * BM - 1) / (2 * BM), tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int nkb = (K + KT::KE - 1) / KT::KE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(&full_bar[s], 1);
      dev::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      dev::mbar_init(&tfull_bar[b], 1);
      dev::mbar_init(&tempty_bar[b], 2 * EPI_WARPS);  // both CTAs' epilogue warps
    }
    dev::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmA);
    dev::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    dev2::tmem_alloc2(tmem_slot, TMEM_COLS);
    dev2::tmem_relinquish2();
  }
  // launched as a programmatic dependent: nothing the previous kernel produced is read, and
  // nothing is written, before this
  dev::grid_dep_wait();
  dev::tc_fence_before();
  dev2::cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrive
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs)
    uint32_t it = 0, s = 0, ph = 0;
    bool stop = false;
    for (int t = pair; t < num_tiles && !stop; t += npairs) {
      const int m0 = (t / tiles_n) * 2 * BM + (int)rank * BM, n0 = (t % tiles_n) * BN + (int)rank * (BN / 2);
      for (int kb = 0; kb < nkb; ++kb) {
        if (*abort_flag || !dev::mbar_wait(&empty_bar[s], ph ^ 1, err)) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        uint8_t* st = smem + s * STAGE;
        if (rank == 0) dev::mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(2 * STAGE));
        dev2::tma_load_2d_pair(st, &tmA, &full_bar[s], kb * KT::KE, m0);
#pragma unroll
        for (int ch = 0; ch < KT::B_CHUNKS; ++ch)
          dev2::tma_load_2d_pair(st + A_STAGE + ch * KT::B_CHUNK, &tmB, &full_bar[s], n0 + ch * KT::CHUNK_COLS,
                                 kb * KT::KE);
        ++it;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- MMA issuer (leader only): M = 256 (128 rows from each CTA), N = 256
    constexpr uint32_t idesc = dev::umma_idesc(KT::C_FMT, KT::AB_FMT, KT::AB_FMT, 0u, 1u, 256u, (uint32_t)BN);
    const uint32_t base = dev::smem_u32(smem);
    const uint64_t a_desc0 = dev::umma_sdesc(base, 16, 8 * BK, dev::UMMA_SW128);
    // MN-major B: LBO = the stride between 128-byte column chunks, SBO = 8 K rows
    const uint64_t b_desc0 = dev::umma_sdesc(base + A_STAGE, KT::B_CHUNK, 1024, dev::UMMA_SW128);
    bool ok = true;
    uint32_t s = 0, ph = 0, local = 0;
    for (int t = pair; t < num_tiles && ok; t += npairs, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      if (*abort_flag || !dev::mbar_wait(&tempty_bar[buf], (use & 1) ^ 1, err)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      const uint32_t d_tmem = tmem + buf * BN;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!dev::mbar_wait(&full_bar[s], ph, err)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint64_t soff = (uint64_t)((s * (uint32_t)STAGE) >> 4);
#pragma unroll
        for (int ks = 0; ks < BK / 32; ++ks)
          dev2::umma2<KIND>(d_tmem, a_desc0 + soff + (uint64_t)((ks * 32) >> 4),
                            b_desc0 + soff + (uint64_t)((ks * KT::KSTEP_B) >> 4), idesc, (kb | ks) != 0);
        dev2::umma2_commit_both(&empty_bar[s]);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1;
        }
      }
      if (ok) dev2::umma2_commit_both(&tfull_bar[buf]);
    }
    if (!ok) {
      *abort_flag = 1;
      dev2::umma2_commit_leader(drain_bar);
      dev::mbar_wait(drain_bar, 0, nullptr, 200000000ull);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows x 256 columns
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;  // even / odd 32-column chunks
    ColSlice* my = col_slices + (warp - 2) * CHUNKS_PER_WARP;
    uint32_t local = 0;
    int staged_n0 = -1;
    for (int t = pair; t < num_tiles; t += npairs, ++local) {
      const uint32_t buf = local % NBUF, use = local / NBUF;
      const int m0 = (t / tiles_n) * 2 * BM + (int)rank * BM, n0 = (t % tiles_n) * BN;
      if (n0 != staged_n0) {
        __syncwarp();
#pragma unroll
        for (int k = 0; k < CHUNKS_PER_WARP; ++k)
          epi_stage_cols<EPI>(ep, n0 + h * 32 + 64 * k + lane, N, lane, my[k]);
        __syncwarp();
        staged_n0 = n0;
      }
      if (!dev::mbar_wait(&tfull_bar[buf], use & 1, err) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      dev::tc_fence_after();
      const int r = m0 + q * 32 + lane;
      float am = 0.0f;
#pragma unroll 1
      for (int k = 0; k < CHUNKS_PER_WARP; ++k) {
        const int c0 = h * 32 + 64 * k;
        if (n0 + c0 >= N) break;  // warp-uniform
        uint32_t v[32];
        dev::tmem_ld32(tmem + buf * BN + (uint32_t)c0 + ((uint32_t)(q * 32) << 16), v);
        dev::tmem_ld_wait();
        if (r < M) epi_store32<EPI>(ep, r, n0 + c0, N, v, my[k], false, 0.0f, am);
      }
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0) dev2::mbar_arrive_leader(&tempty_bar[buf]);
    }
  }

  dev::tc_fence_before();
  dev2::cluster_sync();  // neither CTA leaves while the pair's MMAs / arrivals may touch it
  if (warp == 1) {
    dev::tc_fence_after();
    dev2::tmem_dealloc2(tmem, TMEM_COLS);
  }
}

// Launches the 2-SM kernel on A [M][lda] (K-major) and B [K][ldb] (MN-major), device and
// TMA-aligned: s8 operands with the requantising epilogue, or bf16 with the fp32 one.
template <dev::MmaKind KIND, Epi EPI>
static bool gemm_2sm_launch(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                            const EpiParams& ep) {
  using namespace g2;
  using KT = Kind2<KIND>;
  const CUtensorMapDataType dt =
      KIND == dev::MmaKind::I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t E = KT::ELEM;
  CUtensorMap ta, tb;
  const uint64_t dA[2] = {(uint64_t)K, (uint64_t)M}, sA[1] = {(uint64_t)A.ld * E};
  const uint32_t bA[2] = {(uint32_t)KT::KE, (uint32_t)BM};
  const uint64_t dB[2] = {(uint64_t)N, (uint64_t)K}, sB[1] = {(uint64_t)B.ld * E};
  const uint32_t bB[2] = {(uint32_t)KT::CHUNK_COLS, (uint32_t)KT::KE};
  if (!encode_tmap(&ta, dt, 2, A.p, dA, sA, bA, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap(&tb, dt, 2, B.p, dB, sB, bB, CU_TENSOR_MAP_SWIZZLE_128B)) {
    c.fail();
    return false;
  }
  static bool attr_done[64] = {false};
  const int dv = current_device();
  if (dv >= 0 && dv < 64 && !attr_done[dv]) {
    if (!ACF_CUDA_OK(cudaFuncSetAttribute(gemm_2sm_kernel<KIND, EPI>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM))) {
      c.fail();
      return false;
    }
    attr_done[dv] = true;
  }
  const long long tiles = (long long)((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
  const int pairs = (int)std::min<long long>(tiles, c.sm_count() / 2);
  if (!ACF_CUDA_OK(launch_pdl(gemm_2sm_kernel<KIND, EPI>, dim3(2 * pairs), dim3(THREADS), (size_t)SMEM,
                              c.stream(), ta, tb, ep, M, N, K, c.err()))) {
    c.fail();
    return false;
  }
  return c.launched("gemm_2sm_kernel");
}

bool gemm_s8req_2sm(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                    const EpiParams& ep) {
  return gemm_2sm_launch<dev::MmaKind::I8, Epi::S8_REQ>(c, A, B, M, N, K, ep);
}

bool gemm_bf16_2sm(Call& c, const Operand& A, const Operand& B, int M, int N, int K,
                   const EpiParams& ep) {
  return gemm_2sm_launch<dev::MmaKind::F16, Epi::F32_BIAS>(c, A, B, M, N, K, ep);
}

}  // namespace acf
