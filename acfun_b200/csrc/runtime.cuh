// runtime.cuh — host runtime shared by every entry point of libacfun_b200.so.
//
//  * error state: thread-local code + message (acfun_last_error), set by ACF_* macros;
//  * device context: current device and stream per thread, one DeviceState per device
//    (device error word for bounded kernel waits, grow-only workspace, pinned mailbox);
//  * Call: the per-entry-point helper that resolves every tensor argument to a device
//    pointer (device / managed pointers used in place, host pointers staged through the
//    workspace), and on finish copies host outputs back, synchronises and surfaces any
//    device-side error;
//  * TMA tensor-map encoding through the driver entry point (no libcuda link dependency).
#pragma once
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>
#include <vector>

namespace acf {

enum ErrCode { kOk = 0, kInvalid = 1, kCuda = 2, kTimeout = 3, kNoMem = 4, kFormat = 5 };

void set_error(int code, const char* fmt, ...);
int last_error_code();
void clear_error();

#define ACF_CUDA_OK(expr)                                                                  \
  ([&]() -> bool {                                                                         \
    cudaError_t e__ = (expr);                                                              \
    if (e__ != cudaSuccess) {                                                              \
      ::acf::set_error(e__ == cudaErrorMemoryAllocation ? ::acf::kNoMem : ::acf::kCuda,   \
                       "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e__), __FILE__, \
                       __LINE__);                                                          \
      return false;                                                                        \
    }                                                                                      \
    return true;                                                                           \
  }())

// Grow-only device scratch.  Allocations of one call never move: when a request does not
// fit, a new chunk is added; the next call consolidates the chunks into one.
class Workspace {
 public:
  void* alloc(size_t bytes, cudaStream_t s);
  void reset(cudaStream_t s);
  size_t capacity() const { return total_; }
  void release_all(cudaStream_t s);

 private:
  struct Chunk {
    char* p;
    size_t n;
  };
  std::vector<Chunk> chunks_;
  size_t cur_ = 0, off_ = 0, total_ = 0;
};

struct DeviceState {
  int device = -1;
  unsigned* d_err = nullptr;      // device error word written by bounded waits
  unsigned* h_mailbox = nullptr;  // pinned host copy target
  Workspace ws;
  std::mutex mu;                  // one call at a time owns the workspace
  cudaStream_t ws_stream = nullptr;
  int sm_count = 148;
  // host-buffer calls overlap their H2D / D2H copies with the math on these streams
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  static constexpr int kEvents = 40;
  cudaEvent_t ev[kEvents] = {};
  bool ok = false;
};

struct ThreadCtx {
  int device = -1;
  cudaStream_t stream = nullptr;
};

ThreadCtx& tctx();
DeviceState* device_state();  // for the current thread's device (initialising it)
int current_device();

enum class PtrKind { Host, Device };
PtrKind ptr_kind(const void* p);

// Per-entry-point helper.  Typical use:
//   Call c("acfun_gemm"); if (!c.ok()) return;
//   const float* dA = c.in(A, bytes); float* dC = c.out(C, bytes);
//   launch(..., c.stream(), c.err()); c.finish();
class Call {
 public:
  explicit Call(const char* name);
  ~Call();
  bool ok() const { return ok_; }
  cudaStream_t stream() const { return stream_; }
  unsigned* err() const { return dev_ ? dev_->d_err : nullptr; }
  int sm_count() const { return dev_ ? dev_->sm_count : 148; }
  // Resolve an input: device pointers pass through, host data is copied into scratch.
  const void* in(const void* p, size_t bytes);
  // Resolve an output: host outputs get scratch that finish() copies back.
  void* out(void* p, size_t bytes);
  // In-place tensor (read and written).
  void* inout(void* p, size_t bytes);
  // Plain device scratch for intermediates (256-byte aligned).
  void* scratch(size_t bytes);
  bool any_host() const { return any_host_; }
  // Record that caller host memory takes part in this call (forces a final synchronise).
  void note_host() { any_host_ = true; }
  // Launch-error check after a kernel launch.
  bool launched(const char* what);
  // Copy host outputs back, synchronise when host memory was involved, check the device
  // error word.  Returns true on success.
  bool finish();
  const char* name() const { return name_; }
  void fail() { ok_ = false; }
  // Copy streams and a pool of timing-free events (indices < DeviceState::kEvents) for
  // calls that pipeline host copies; owned by the device, valid while the call holds it.
  cudaStream_t copy_in() const { return dev_->copy_in; }
  cudaStream_t copy_out() const { return dev_->copy_out; }
  cudaEvent_t event(int i) const { return dev_->ev[i]; }

 private:
  struct Pending {
    void* host;
    const void* dev;
    size_t bytes;
  };
  const char* name_;
  DeviceState* dev_ = nullptr;
  std::unique_lock<std::mutex> lock_;
  cudaStream_t stream_ = nullptr;
  std::vector<Pending> outs_;
  bool ok_ = false, any_host_ = false, finished_ = false;
};

// Device error word helpers (used by acfun_synchronize and Call::finish).
bool check_device_error(DeviceState* d, cudaStream_t s);

// TMA tensor map encoding (cuTensorMapEncodeTiled through the driver entry point).
bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swz);

// Launch `k` so that it may start while the previous kernel of `stream` finishes (programmatic
// stream serialisation); the kernel must call dev::grid_dep_wait() before it reads what that
// kernel produced or writes global memory.  ACFUN_PDL=0 launches normally.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace acf
