// runtime.cu — see runtime.cuh.
#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "runtime.cuh"

namespace acf {

// ------------------------------------------------------------------ errors
static thread_local int t_err_code = 0;
static thread_local char t_err_msg[512] = {0};

void set_error(int code, const char* fmt, ...) {
  t_err_code = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err_msg, sizeof(t_err_msg), fmt, ap);
  va_end(ap);
  if (getenv("ACFUN_VERBOSE")) fprintf(stderr, "[acfun] error %d: %s\n", code, t_err_msg);
}
int last_error_code() { return t_err_code; }
const char* last_error_msg() { return t_err_msg; }
void clear_error() {
  t_err_code = 0;
  t_err_msg[0] = 0;
}

// ------------------------------------------------------------------ workspace
void* Workspace::alloc(size_t bytes, cudaStream_t s) {
  (void)s;
  bytes = align_up(bytes ? bytes : 1, 256);
  if (!chunks_.empty() && off_ + bytes <= chunks_[cur_].n) {
    void* p = chunks_[cur_].p + off_;
    off_ += bytes;
    return p;
  }
  size_t n = bytes > total_ ? bytes : total_;
  if (n < (size_t(4) << 20)) n = size_t(4) << 20;
  char* p = nullptr;
  if (cudaMalloc(&p, n) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  chunks_.push_back({p, n});
  total_ += n;
  cur_ = chunks_.size() - 1;
  off_ = bytes;
  return p;
}

void Workspace::reset(cudaStream_t s) {
  if (chunks_.size() > 1) {
    cudaStreamSynchronize(s);
    size_t t = total_;
    for (auto& c : chunks_) cudaFree(c.p);
    chunks_.clear();
    total_ = 0;
    char* p = nullptr;
    if (cudaMalloc(&p, t) == cudaSuccess) {
      chunks_.push_back({p, t});
      total_ = t;
    } else {
      cudaGetLastError();
    }
  }
  cur_ = 0;
  off_ = 0;
}

void Workspace::release_all(cudaStream_t s) {
  cudaStreamSynchronize(s);
  for (auto& c : chunks_) cudaFree(c.p);
  chunks_.clear();
  total_ = 0;
  cur_ = off_ = 0;
}

// ------------------------------------------------------------------ devices
static std::mutex g_dev_mu;
static DeviceState g_devs[64];

ThreadCtx& tctx() {
  static thread_local ThreadCtx t;
  if (t.device < 0) {
    const char* e = getenv("ACFUN_DEVICE");
    t.device = e ? atoi(e) : 0;
    if (t.device < 0) t.device = 0;
  }
  return t;
}

int current_device() { return tctx().device; }

DeviceState* device_state() {
  int d = tctx().device;
  if (d < 0 || d >= 64) {
    set_error(kInvalid, "device index %d out of range", d);
    return nullptr;
  }
  DeviceState* s = &g_devs[d];
  if (s->ok) return s;
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (s->ok) return s;
  if (!ACF_CUDA_OK(cudaSetDevice(d))) return nullptr;
  if (!ACF_CUDA_OK(cudaMalloc(&s->d_err, sizeof(unsigned)))) return nullptr;
  if (!ACF_CUDA_OK(cudaMemset(s->d_err, 0, sizeof(unsigned)))) return nullptr;
  if (!ACF_CUDA_OK(cudaHostAlloc(&s->h_mailbox, 64, cudaHostAllocDefault))) return nullptr;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) == cudaSuccess && sms > 0)
    s->sm_count = sms;
  if (!ACF_CUDA_OK(cudaStreamCreateWithFlags(&s->copy_in, cudaStreamNonBlocking)) ||
      !ACF_CUDA_OK(cudaStreamCreateWithFlags(&s->copy_out, cudaStreamNonBlocking)))
    return nullptr;
  for (int i = 0; i < DeviceState::kEvents; ++i)
    if (!ACF_CUDA_OK(cudaEventCreateWithFlags(&s->ev[i], cudaEventDisableTiming))) return nullptr;
  s->device = d;
  s->ok = true;
  return s;
}

PtrKind ptr_kind(const void* p) {
  if (!p) return PtrKind::Host;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return PtrKind::Host;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return PtrKind::Device;
  return PtrKind::Host;
}

bool check_device_error(DeviceState* d, cudaStream_t s) {
  if (!d) return false;
  if (!ACF_CUDA_OK(cudaMemcpyAsync(d->h_mailbox, d->d_err, sizeof(unsigned),
                                   cudaMemcpyDeviceToHost, s)))
    return false;
  if (!ACF_CUDA_OK(cudaStreamSynchronize(s))) return false;
  unsigned v = d->h_mailbox[0];
  if (v) {
    cudaMemsetAsync(d->d_err, 0, sizeof(unsigned), s);
    cudaStreamSynchronize(s);
    if (v & 1u)
      set_error(kTimeout, "device-side wait timed out (error word 0x%x)", v);
    else
      set_error(kInvalid, "device-side argument check failed (error word 0x%x)", v);
    return false;
  }
  return true;
}

// ------------------------------------------------------------------ Call
Call::Call(const char* name) : name_(name) {
  ThreadCtx& t = tctx();
  dev_ = device_state();
  if (!dev_) return;
  if (!ACF_CUDA_OK(cudaSetDevice(t.device))) return;
  lock_ = std::unique_lock<std::mutex>(dev_->mu);
  stream_ = t.stream;
  if (dev_->ws_stream != stream_) {
    // scratch may still be in use by work queued on the previous stream
    cudaStreamSynchronize(dev_->ws_stream);
    dev_->ws_stream = stream_;
  }
  dev_->ws.reset(stream_);
  ok_ = true;
}

Call::~Call() {
  if (ok_ && !finished_) {
    // early exit after an error: never return while copies still read caller memory
    if (any_host_) cudaStreamSynchronize(stream_);
  }
}

void* Call::scratch(size_t bytes) {
  if (!ok_) return nullptr;
  void* p = dev_->ws.alloc(bytes, stream_);
  if (!p) {
    set_error(kNoMem, "%s: cannot allocate %zu bytes of device scratch", name_, bytes);
    ok_ = false;
  }
  return p;
}

const void* Call::in(const void* p, size_t bytes) {
  if (!ok_ || !p) return p;
  if (ptr_kind(p) == PtrKind::Device) return p;
  void* d = scratch(bytes);
  if (!d) return nullptr;
  any_host_ = true;
  if (bytes && !ACF_CUDA_OK(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, stream_))) {
    ok_ = false;
    return nullptr;
  }
  return d;
}

void* Call::out(void* p, size_t bytes) {
  if (!ok_ || !p) return p;
  if (ptr_kind(p) == PtrKind::Device) return p;
  void* d = scratch(bytes);
  if (!d) return nullptr;
  any_host_ = true;
  outs_.push_back({p, d, bytes});
  return d;
}

void* Call::inout(void* p, size_t bytes) {
  if (!ok_ || !p) return p;
  if (ptr_kind(p) == PtrKind::Device) return p;
  void* d = scratch(bytes);
  if (!d) return nullptr;
  any_host_ = true;
  if (bytes && !ACF_CUDA_OK(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, stream_))) {
    ok_ = false;
    return nullptr;
  }
  outs_.push_back({p, d, bytes});
  return d;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("ACFUN_PDL");
    return !(e && !strcmp(e, "0"));
  }();
  return on;
}

bool Call::launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(kCuda, "%s: launch of %s failed: %s", name_, what, cudaGetErrorString(e));
    ok_ = false;
    return false;
  }
  return true;
}

bool Call::finish() {
  if (finished_) return ok_;
  finished_ = true;
  if (!ok_) {
    if (any_host_) cudaStreamSynchronize(stream_);
    return false;
  }
  for (auto& o : outs_) {
    if (o.bytes &&
        !ACF_CUDA_OK(cudaMemcpyAsync(o.host, o.dev, o.bytes, cudaMemcpyDeviceToHost, stream_))) {
      ok_ = false;
    }
  }
  if (any_host_) {
    if (!ACF_CUDA_OK(cudaStreamSynchronize(stream_))) ok_ = false;
    if (ok_ && !check_device_error(dev_, stream_)) ok_ = false;
  }
  return ok_;
}

// ------------------------------------------------------------------ TMA encode
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swz) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    else
      cudaGetLastError();
  });
  if (!g_encode) {
    set_error(kCuda, "cuTensorMapEncodeTiled is unavailable");
    return false;
  }
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void*>(base),
                        reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(kCuda, "cuTensorMapEncodeTiled failed (CUresult %d, rank %d)", (int)r, rank);
    return false;
  }
  return true;
}

}  // namespace acf
