// gemm_static.cu — acfun_gemm_epi_noalloc: the fp32 GEMM (+bias, +ReLU) of acfun_gemm_epi for
// callers that cannot allocate device memory.
//
// Who needs it: some callers cannot call cudaMalloc — processes that reserve all device
// memory up front in their own pool (a further cudaMalloc fails or fragments that pool),
// code running inside an out-of-memory handler or an allocator callback, and latency-
// critical loops in which cudaMalloc / cudaFree would synchronise the whole device.
// acfun_gemm_epi needs device scratch for the 3xTF32 hi/lo operand copies and takes it
// from a grow-only cudaMalloc'd workspace; this entry point instead uses one fixed
// file-scope device array and allocates nothing: no cudaMalloc, cudaFree, cudaHostAlloc or
// allocating library routine, and no staging of host memory.
//
// Contract:
//   * A, B, C (and bias, when given) must be device pointers; host pointers are rejected.
//   * The scratch holds 2*(M*Kp + K*Np) floats with Kp = K and Np = N rounded up to a
//     multiple of 4; larger problems are rejected (ACFUN_NOALLOC_SCRATCH_FLOATS below:
//     4 Mi floats = 16 MiB, e.g. any M = N = K <= 1024 problem).  Every GPU that loads the
//     library holds this array until the process exits.
//   * The first call on each device resolves the array's device address
//     (cudaGetSymbolAddress) with that device current.
//   * Every call waits for its stream (cudaStreamSynchronize) to read the device error word,
//     so it cannot be called while its stream is being captured into a CUDA graph.
//   * All calls share the one array and it keeps the last call's contents (the split
//     kernel rewrites every element a call reads, so nothing has to start at zero; the
//     device error word is cleared by every call).  Calls that overlap on the GPU — on two
//     streams, or from two threads — race on the array: serialise them.
//   * Work runs on the stream set with acfun_set_stream(); the call returns after that
//     stream has finished it.  Returns 0, or an acfun error code (also reported through
//     acfun_last_error()).
#include <mutex>

#include "api_export.cuh"
#include "gemm.cuh"

#define ACFUN_NOALLOC_SCRATCH_FLOATS (4u << 20)

namespace acf {

static __device__ __align__(256) float g_noalloc_scratch[ACFUN_NOALLOC_SCRATCH_FLOATS];
static __device__ unsigned g_noalloc_err;

struct NoAllocDevice {
  float* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  unsigned* err = nullptr;   // device address of g_noalloc_err
  int sms = 0;
  bool ready = false;
};
static NoAllocDevice g_na[64];
static std::mutex g_na_mu;

static NoAllocDevice* noalloc_setup(int device) {
  if (device < 0 || device >= 64) {
    set_error(kInvalid, "acfun_gemm_epi_noalloc: device index %d out of range", device);
    return nullptr;
  }
  NoAllocDevice* d = &g_na[device];
  std::lock_guard<std::mutex> g(g_na_mu);
  if (d->ready) return d;
  // with `device` current: host-side stand-ins are not device addresses
  if (!ACF_CUDA_OK(cudaGetSymbolAddress((void**)&d->scratch, g_noalloc_scratch))) return nullptr;
  if (!ACF_CUDA_OK(cudaGetSymbolAddress((void**)&d->err, g_noalloc_err))) return nullptr;
  int sms = 0;
  if (!ACF_CUDA_OK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)))
    return nullptr;
  d->sms = sms > 0 ? sms : 148;
  d->ready = true;
  return d;
}

template <int BN, int STAGES>
static int noalloc_launch(const NoAllocDevice* d, int device, cudaStream_t st, const float* a,
                          long long lda, long long a_op, const float* b, long long ldb,
                          long long b_op, int M, int N, int K, const EpiParams& ep) {
  using S = GemmShape<dev::MmaKind::TF32, BN, STAGES, 3>;
  CUtensorMap ta, tb;
  const uint64_t dA[3] = {(uint64_t)K, (uint64_t)M, 2}, sA[2] = {(uint64_t)lda * 4, (uint64_t)a_op * 4};
  const uint32_t bA[3] = {(uint32_t)S::BKE, 128u, 1u};
  const uint64_t dB[3] = {(uint64_t)N, (uint64_t)K, 2}, sB[2] = {(uint64_t)ldb * 4, (uint64_t)b_op * 4};
  const uint32_t bB[3] = {32u, (uint32_t)S::BKE, 1u};
  if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a, dA, sA, bA, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, b, dB, sB, bB,
                   CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return kCuda;
  auto kern = gemm_tc_kernel<dev::MmaKind::TF32, BN, STAGES, 3, Epi::F32_BIAS, false>;
  static bool attr_done[64] = {false};
  if (!attr_done[device]) {
    if (!ACF_CUDA_OK(
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM)))
      return kCuda;
    attr_done[device] = true;
  }
  const long long tiles = (long long)((M + 127) / 128) * ((N + BN - 1) / BN);
  const unsigned grid = (unsigned)(tiles < d->sms ? tiles : d->sms);
  kern<<<grid, S::THREADS, S::SMEM, st>>>(ta, tb, ep, ConvGeom{}, M, N, K, d->err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(kCuda, "acfun_gemm_epi_noalloc: launch failed: %s", cudaGetErrorString(e));
    return kCuda;
  }
  return 0;
}

// True when p is device (or managed) memory of `device`: a pointer into another GPU's memory
// would be read by the split kernel and written by the epilogue without peer access.
static bool on_device(const void* p, int device) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == device;
}

}  // namespace acf

using namespace acf;

extern "C" int acfun_gemm_epi_noalloc(int M, int N, int K, const float* A, const float* B,
                                      float* C, const float* bias, int act) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;  // nothing to do, like acfun_gemm_epi
  if (!A || !B || !C) {
    set_error(kInvalid, "acfun_gemm_epi_noalloc: NULL tensor argument");
    return kInvalid;
  }
  const int device = tctx().device;
  if (!on_device(A, device) || !on_device(B, device) || !on_device(C, device) ||
      (bias && !on_device(bias, device))) {
    set_error(kInvalid,
              "acfun_gemm_epi_noalloc: A, B, C and bias must be device pointers on the acfun "
              "device %d (host memory would need staging buffers)", device);
    return kInvalid;
  }
  const long long Kp = (K + 3) / 4 * 4, Np = (N + 3) / 4 * 4;
  const long long need = 2 * ((long long)M * Kp + (long long)K * Np);
  if (need > (long long)ACFUN_NOALLOC_SCRATCH_FLOATS) {
    set_error(kInvalid,
              "acfun_gemm_epi_noalloc: M=%d N=%d K=%d needs %lld scratch floats, the fixed "
              "maximum is %u (2*(M*K + K*N) with K, N rounded up to 4)",
              M, N, K, need, (unsigned)ACFUN_NOALLOC_SCRATCH_FLOATS);
    return kInvalid;
  }
  if (!ACF_CUDA_OK(cudaSetDevice(device))) return kCuda;
  NoAllocDevice* d = noalloc_setup(device);
  if (!d) return last_error_code() ? last_error_code() : kCuda;
  const cudaStream_t st = tctx().stream;
  if (!ACF_CUDA_OK(cudaMemsetAsync(d->err, 0, sizeof(unsigned), st))) return kCuda;
  float* a = d->scratch;                        // [2][M][Kp]
  float* b = d->scratch + 2 * (long long)M * Kp;  // [2][K][Np]
  const int blocks = d->sms * 8;
  k_to_tf32x2<<<blocks, 256, 0, st>>>(A, K, M, K, a, Kp, (long long)M * Kp);
  k_to_tf32x2<<<blocks, 256, 0, st>>>(B, N, K, N, b, Np, (long long)K * Np);
  if (cudaGetLastError() != cudaSuccess) {
    set_error(kCuda, "acfun_gemm_epi_noalloc: split kernel launch failed");
    return kCuda;
  }
  EpiParams ep{};
  ep.C = C;
  ep.ldc = N;
  ep.f0 = bias;
  ep.act = act ? 1 : 0;
  // same tile-width choice as acfun_gemm_epi (gemm.cu gemm_launch, TF32X3)
  const long long t128 = (long long)((M + 127) / 128) * ((N + 127) / 128);
  int rc;
  if (N > 64 && t128 >= d->sms)
    rc = noalloc_launch<128, 3>(d, device, st, a, Kp, (long long)M * Kp, b, Np, (long long)K * Np, M,
                                N, K, ep);
  else if (N > 32)
    rc = noalloc_launch<64, 4>(d, device, st, a, Kp, (long long)M * Kp, b, Np, (long long)K * Np, M,
                               N, K, ep);
  else
    rc = noalloc_launch<32, 5>(d, device, st, a, Kp, (long long)M * Kp, b, Np, (long long)K * Np, M,
                               N, K, ep);
  if (rc) return rc;
  // read the error word on the acfun stream only (no device-wide synchronisation)
  unsigned word = 0;
  if (!ACF_CUDA_OK(cudaMemcpyAsync(&word, d->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st)))
    return kCuda;
  if (!ACF_CUDA_OK(cudaStreamSynchronize(st))) return kCuda;
  if (word) {
    set_error(kTimeout, "acfun_gemm_epi_noalloc: device-side wait timed out (0x%x)", word);
    return kTimeout;
  }
  return 0;
}
