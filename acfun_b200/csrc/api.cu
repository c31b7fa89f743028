// api.cu — runtime-level entry points: backend identity, CPU-thread compatibility shims,
// device / stream selection, synchronisation and error reporting.
#include <stdio.h>
#include <stdlib.h>

#include "api_export.cuh"
#include "runtime.cuh"

namespace acf {
const char* last_error_msg();
}
using namespace acf;

static int g_rt_threads = 1;

// acfun.h:20 (gemm.cpp:38): the CPU thread count has no effect on the CUDA backend.
extern "C" void acfun_set_threads(int n) { (void)n; }
// acfun.h:23-24 (gemm.cpp:81-88)
extern "C" int acfun_backend(void) { return ACFUN_BACKEND_CUDA_SM100A; }
extern "C" const char* acfun_backend_name(void) { return "CUDA-sm100a"; }
// internal.h:111-115,225 (gemm.cpp:19-20,43-67,104-136)
extern "C" void acfun_set_num_threads_runtime(int n) { g_rt_threads = n > 0 ? n : 1; }
extern "C" int acfun_get_num_threads_runtime(void) { return g_rt_threads; }
extern "C" int acfun_pick_threads(int M, int N, int K) {
  (void)M; (void)N; (void)K;
  return 1;
}
// The analogue of "effective cores" on the GPU backend: SMs of the current device.
extern "C" int acfun_effective_cores(void) {
  DeviceState* d = device_state();
  return d ? d->sm_count : 1;
}

extern "C" void acfun_set_stream(void* stream) { tctx().stream = (cudaStream_t)stream; }
extern "C" void* acfun_get_stream(void) { return (void*)tctx().stream; }

extern "C" int acfun_set_device(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    set_error(kCuda, "acfun_set_device: no CUDA device");
    return kCuda;
  }
  if (device < 0 || device >= n) {
    set_error(kInvalid, "acfun_set_device: device %d out of range [0,%d)", device, n);
    return kInvalid;
  }
  tctx().device = device;
  return 0;
}

extern "C" int acfun_synchronize(void) {
  DeviceState* d = device_state();
  if (!d) return last_error_code();
  if (!ACF_CUDA_OK(cudaSetDevice(tctx().device))) return last_error_code();
  if (!ACF_CUDA_OK(cudaStreamSynchronize(tctx().stream))) return last_error_code();
  if (!check_device_error(d, tctx().stream)) return last_error_code();
  return 0;
}

extern "C" int acfun_last_error_code(void) { return last_error_code(); }
extern "C" const char* acfun_last_error(void) { return last_error_msg(); }
extern "C" void acfun_clear_error(void) { clear_error(); }
