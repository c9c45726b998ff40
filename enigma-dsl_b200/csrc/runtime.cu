// runtime.cu — the C ABI declared in include/enigma_cuda.h.
//
// It plays the part of the reference's Swift runtime
// (enigma/runtime_dispatch/swift/libenigma_runtime.swift): device and queue
// creation, buffers, dispatch by kernel, timed dispatch and capability queries.
// Argument checks happen here, before anything is launched, and map to
// ENIGMA_ERR_BADARG with a message for enigma_last_error.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace enigma {

namespace {
thread_local char g_err[512] = {0};
std::mutex g_mu;
constexpr int kMaxDev = 64;
int g_sms[kMaxDev] = {0};
uint32_t* g_status[kMaxDev] = {nullptr};
cudaStream_t g_aux[kMaxDev] = {nullptr};

// Per-device state: the status word (bytes 0..255) and kWorkSlots pairs of work counters.
constexpr int kWorkSlots = 4096;
constexpr size_t kStateBytes = 256 + size_t(kWorkSlots) * 2 * sizeof(uint32_t);
std::atomic<uint32_t> g_work_next[kMaxDev];

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// Make sure the per-device state (SM count, status word) exists.
cudaError_t ensure_device_state(int dev) {
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status[dev] != nullptr) return cudaSuccess;
  int sms = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  uint32_t* st = nullptr;
  e = cudaMalloc(&st, kStateBytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(st, 0, kStateBytes);
  if (e != cudaSuccess) return e;
  g_sms[dev] = sms;
  g_status[dev] = st;
  return cudaSuccess;
}
}  // namespace

thread_local const char* g_last_kernel = "";

void note_kernel(const char* name) { g_last_kernel = name; }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int sm_count() {
  const int d = current_device();
  if (ensure_device_state(d) != cudaSuccess) return 148;
  return g_sms[d];
}

uint32_t* device_status() {
  const int d = current_device();
  if (ensure_device_state(d) != cudaSuccess) return nullptr;
  return g_status[d];
}

uint32_t* work_counters() {
  const int d = current_device();
  if (ensure_device_state(d) != cudaSuccess) return nullptr;
  const uint32_t slot = g_work_next[d].fetch_add(1, std::memory_order_relaxed) % kWorkSlots;
  return g_status[d] + 64 + 2 * slot;
}

uint32_t* device_status_if_exists() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_status[d];
}

// A library-owned non-blocking stream of the current device, for work a call overlaps with
// the caller's stream (created on first use, never destroyed).
cudaStream_t aux_stream() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_aux[d] == nullptr && cudaStreamCreateWithFlags(&g_aux[d], cudaStreamNonBlocking) != cudaSuccess)
    g_aux[d] = nullptr;
  return g_aux[d];
}

}  // namespace enigma

namespace {
// Self-test of the failure reporting: one thread waits on an mbarrier that nothing arrives
// on, gives up after `polls` polls exactly as the kernels' bounded waits do (flag the device
// status word, return), so the host side of a timeout can be exercised without hanging.
__global__ void timeout_probe_kernel(uint32_t* status, long long polls) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  enigma_sm100::mbar_init(&bar, 1);
  enigma_sm100::fence_barrier_init();
  for (long long i = 0; i < polls; ++i)
    if (enigma_sm100::mbar_try_wait(&bar, 0)) return;   // never completes: nothing arrives
  atomicExch(status, enigma_sm100::kDevTimeout);
}
}  // namespace

namespace enigma {
cudaError_t launch_timeout_probe(uint32_t* status, long long polls, cudaStream_t s) {
  timeout_probe_kernel<<<1, 32, 0, s>>>(status, polls);
  return cudaGetLastError();
}
}  // namespace enigma

using enigma::set_error;

namespace {

int32_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ENIGMA_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  // Errors raised at launch time are launch failures; sticky errors are execution errors.
  switch (e) {
    case cudaErrorInvalidValue:
    case cudaErrorInvalidConfiguration:
    case cudaErrorInvalidDeviceFunction:
    case cudaErrorLaunchOutOfResources:
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorMemoryAllocation:
      return ENIGMA_ERR_LAUNCH;
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice:
    case cudaErrorInsufficientDriver:
      return ENIGMA_ERR_DEVICE;
    default:
      return ENIGMA_ERR_EXEC;
  }
}

int32_t badarg(const char* msg) {
  set_error("bad argument: %s", msg);
  return ENIGMA_ERR_BADARG;
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int32_t check_ptr(const void* p, const char* name, size_t align) {
  if (p == nullptr) {
    set_error("bad argument: %s is NULL", name);
    return ENIGMA_ERR_BADARG;
  }
  if (reinterpret_cast<uintptr_t>(p) % align != 0) {
    set_error("bad argument: %s is not %zu-byte aligned", name, align);
    return ENIGMA_ERR_BADARG;
  }
  return ENIGMA_OK;
}

}  // namespace

extern "C" {

int32_t enigma_last_error(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return ENIGMA_ERR_BADARG;
  std::strncpy(buf, enigma::g_err, len - 1);
  buf[len - 1] = 0;
  return ENIGMA_OK;
}

int32_t enigma_last_kernel(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return ENIGMA_ERR_BADARG;
  snprintf(buf, len, "%s", enigma::g_last_kernel);
  return ENIGMA_OK;
}

int32_t enigma_device_count(int32_t* count) {
  if (count == nullptr) return badarg("count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_status(e, "cudaGetDeviceCount");
  }
  *count = n;
  return ENIGMA_OK;
}

int32_t enigma_init(int32_t device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    set_error("no CUDA device available (%s)", cudaGetErrorString(e));
    return ENIGMA_ERR_DEVICE;
  }
  if (device < 0 || device >= n) return badarg("device index out of range");
  cudaDeviceProp p;
  e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  if (p.major != 10) {
    set_error("device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
              p.major, p.minor);
    return ENIGMA_ERR_DEVICE;
  }
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  return cuda_status(enigma::ensure_device_state(device), "device state");
}

int32_t enigma_stream_create(void** stream) {
  if (stream == nullptr) return badarg("stream is NULL");
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  *stream = s;
  return cuda_status(e, "cudaStreamCreate");
}

int32_t enigma_stream_destroy(void* stream) {
  if (stream == nullptr) return ENIGMA_OK;
  return cuda_status(cudaStreamDestroy(as_stream(stream)), "cudaStreamDestroy");
}

int32_t enigma_take_device_status(int32_t* timeouts) {
  // Reads (and clears) the status words that exist on the current device: the library's
  // per-device word and the no-allocation decode entry's static word.  Neither is created
  // here, so this call allocates nothing.
  uint32_t v = 0;
  if (uint32_t* st = enigma::device_status_if_exists()) {
    cudaError_t e = cudaMemcpy(&v, st, sizeof(v), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_status(e, "read device status");
    if (v != 0) cudaMemset(st, 0, sizeof(uint32_t));
  }
  uint32_t w = 0;
  cudaError_t e = enigma::noalloc_take_status(&w);
  if (e != cudaSuccess) return cuda_status(e, "read no-allocation status");
  if (timeouts) *timeouts = static_cast<int32_t>(v + w);
  return ENIGMA_OK;
}

int32_t enigma_check_timeout_path(int64_t polls, void* stream) {
  if (polls < 0 || polls > (int64_t(1) << 24)) return badarg("polls must be in [0, 2^24]");
  uint32_t* st = enigma::device_status();
  if (st == nullptr) return cuda_status(cudaErrorNoDevice, "device status");
  return cuda_status(enigma::launch_timeout_probe(st, static_cast<long long>(polls),
                                                  as_stream(stream)),
                     "timeout probe");
}

int32_t enigma_synchronize(void* stream) {
  cudaError_t e = stream ? cudaStreamSynchronize(as_stream(stream)) : cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "synchronize");
  int32_t to = 0;
  int32_t rc = enigma_take_device_status(&to);
  if (rc != ENIGMA_OK) return rc;
  if (to != 0) {
    set_error("a device-side wait exceeded its limit and the kernel gave up");
    return ENIGMA_ERR_TIMEOUT;
  }
  return ENIGMA_OK;
}

int32_t enigma_device_name(int32_t device, char* buf, size_t len) {
  if (buf == nullptr || len == 0) return badarg("buffer is NULL");
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  std::strncpy(buf, p.name, len - 1);
  buf[len - 1] = 0;
  return ENIGMA_OK;
}

int32_t enigma_device_attrs(int32_t device, int64_t* sm_count, int64_t* max_smem_per_block,
                            int64_t* max_threads_per_block, int64_t* total_mem_bytes,
                            int32_t* cc_major, int32_t* cc_minor) {
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (max_smem_per_block) *max_smem_per_block = static_cast<int64_t>(p.sharedMemPerBlockOptin);
  if (max_threads_per_block) *max_threads_per_block = p.maxThreadsPerBlock;
  if (total_mem_bytes) *total_mem_bytes = static_cast<int64_t>(p.totalGlobalMem);
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  return ENIGMA_OK;
}

int32_t enigma_alloc(void** ptr, size_t bytes) {
  if (ptr == nullptr) return badarg("ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  return cuda_status(cudaMalloc(ptr, bytes), "cudaMalloc");
}
int32_t enigma_free(void* ptr) {
  if (ptr == nullptr) return ENIGMA_OK;
  return cuda_status(cudaFree(ptr), "cudaFree");
}
int32_t enigma_host_alloc(void** ptr, size_t bytes) {
  if (ptr == nullptr) return badarg("ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  return cuda_status(cudaMallocHost(ptr, bytes), "cudaMallocHost");
}
int32_t enigma_host_free(void* ptr) {
  if (ptr == nullptr) return ENIGMA_OK;
  return cuda_status(cudaFreeHost(ptr), "cudaFreeHost");
}
int32_t enigma_upload(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ENIGMA_OK;
  if (dst == nullptr || src == nullptr) return badarg("NULL pointer in upload");
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream)),
                     "upload");
}
int32_t enigma_download(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ENIGMA_OK;
  if (dst == nullptr || src == nullptr) return badarg("NULL pointer in download");
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)),
                     "download");
}
int32_t enigma_memset(void* dst, int32_t value, size_t bytes, void* stream) {
  if (bytes == 0) return ENIGMA_OK;
  if (dst == nullptr) return badarg("NULL pointer in memset");
  return cuda_status(cudaMemsetAsync(dst, value, bytes, as_stream(stream)), "memset");
}

}  // extern "C"
