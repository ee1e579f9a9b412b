// backend.cu -- device context, error state and the scratch pool.
//
// Replaces the reference's CLBackend singleton (src/cl_backend.{h,cc}): no
// platform probing, no runtime kernel compilation (kernels are compiled into
// this library for sm_100a), no global queue mutex.  Each device gets one
// lazily created DeviceInfo holding its SM count and a dedicated CUDA memory
// pool used as the caching, stream-ordered scratch allocator that the
// reference never had (docs/ARCHITECTURE.md:141-149).
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "b2_internal.cuh"

namespace b2 {

namespace {

thread_local std::string t_last_error;

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::once_flag g_device_once[kMaxDevices];
int g_device_status[kMaxDevices];
std::string g_device_error[kMaxDevices];
std::atomic<uint64_t> g_num_allocs[kMaxDevices];
std::atomic<uint64_t> g_launches{0};

// Bounded device-side waits: the limit kernels are launched with, and the
// host-mapped word they set when a wait expires (allocated with the first
// device's state, before any stream capture can be in progress).
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
std::once_flag g_expired_once;
unsigned int* g_expired_host = nullptr;  // host view
unsigned int* g_expired_dev = nullptr;   // device view of the same word

void alloc_expired_flag() {
  void* h = nullptr;
  if (cudaHostAlloc(&h, sizeof(unsigned int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(h);
    return;
  }
  *static_cast<volatile unsigned int*>(h) = 0u;
  g_expired_host = static_cast<unsigned int*>(h);
  g_expired_dev = static_cast<unsigned int*>(d);
}

bool wait_expired() {
  return g_expired_host != nullptr && *static_cast<volatile unsigned int*>(g_expired_host) != 0u;
}

bool env_flag(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
}

uint64_t pool_limit_bytes() {
  static const uint64_t limit = [] {
    const char* v = std::getenv("B2_POOL_LIMIT");
    return v ? std::strtoull(v, nullptr, 10) : 0ull;
  }();
  return limit;
}

void init_device(int dev) {
  DeviceInfo& d = g_devices[dev];
  d.device = dev;
  int st = B2_OK;
  std::string err;
  auto fail = [&](int code, const std::string& msg) {
    st = code;
    err = msg;
  };
  cudaError_t e;
  if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
          cudaSuccess) {
    fail(B2_ERR_NO_DEVICE, std::string("cannot query device: ") + cudaGetErrorString(e));
  } else if (d.cc_major != 10 || d.cc_minor != 0) {
    char buf[160];
    std::snprintf(buf, sizeof buf,
                  "device %d has compute capability %d.%d; this library is built for sm_100a (B200)", dev,
                  d.cc_major, d.cc_minor);
    fail(B2_ERR_NO_DEVICE, buf);
  } else {
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof props);
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    if ((e = cudaMemPoolCreate(&d.pool, &props)) != cudaSuccess) {
      fail(B2_ERR_INTERNAL, std::string("cudaMemPoolCreate: ") + cudaGetErrorString(e));
    } else {
      // Keep freed blocks cached in the pool instead of returning them to the
      // driver at every synchronisation point.
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
  }
  if (st == B2_OK) std::call_once(g_expired_once, alloc_expired_flag);
  g_device_status[dev] = st;
  g_device_error[dev] = err;
}

}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void clear_error() { t_last_error.clear(); }

int device_info(const DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(B2_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  std::call_once(g_device_once[dev], init_device, dev);
  if (g_device_status[dev] != B2_OK) return set_error(g_device_status[dev], "%s", g_device_error[dev].c_str());
  *out = &g_devices[dev];
  return B2_OK;
}

int check_launch(cudaStream_t s, const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(B2_ERR_INTERNAL, "launch of %s failed (cuda_err=%d: %s)", what, (int)e,
                     cudaGetErrorString(e));
  static const bool debug = env_flag("B2_DEBUG_CHECKS");
  if (debug) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusNone) {
      e = cudaStreamSynchronize(s);
      if (e != cudaSuccess)
        return set_error(B2_ERR_INTERNAL, "%s failed on the device (cuda_err=%d: %s)", what, (int)e,
                         cudaGetErrorString(e));
    }
  }
  if (wait_expired())
    return set_error(B2_ERR_TIMEOUT,
                     "a bounded device-side wait of an earlier kernel of this library expired (checked after "
                     "launching %s); results since then are invalid until b2_stream_status() reports and "
                     "clears it", what);
  return B2_OK;
}

std::atomic<int> g_reserved_sms{0};

int persistent_ctas(const DeviceInfo* d) {
  const int n = d->sm_count - g_reserved_sms.load(std::memory_order_relaxed);
  return n > 0 ? n : 1;
}

WaitParams wait_params() {
  return WaitParams{g_wait_limit_ns.load(std::memory_order_relaxed), g_expired_dev};
}

int SmemOptIn::ensure(const void* kernel, int device, int need) {
  if (device < 0 || device >= kDevices)
    return set_error(B2_ERR_NO_DEVICE, "device ordinal %d out of range", device);
  if (bytes[device].load(std::memory_order_acquire) >= need) return B2_OK;
  std::lock_guard<std::mutex> lock(mu);
  if (bytes[device].load(std::memory_order_relaxed) >= need) return B2_OK;
  B2_CUDA_OR_RETURN(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, need));
  bytes[device].store(need, std::memory_order_release);
  return B2_OK;
}

int scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
  *p = nullptr;
  if (bytes == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const uint64_t limit = pool_limit_bytes();
  if (limit) {
    uint64_t used = 0;
    cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrUsedMemCurrent, &used);
    if (used + bytes > limit)
      return set_error(B2_ERR_OUT_OF_MEMORY, "scratch request of %zu bytes exceeds B2_POOL_LIMIT=%llu (in use %llu)",
                       bytes, (unsigned long long)limit, (unsigned long long)used);
  }
  cudaError_t e = cudaMallocFromPoolAsync(p, bytes, d->pool, s);
  if (e != cudaSuccess) {
    *p = nullptr;
    return set_error(e == cudaErrorMemoryAllocation ? B2_ERR_OUT_OF_MEMORY : B2_ERR_INTERNAL,
                     "scratch allocation of %zu bytes failed (cuda_err=%d: %s)", bytes, (int)e,
                     cudaGetErrorString(e));
  }
  g_num_allocs[d->device].fetch_add(1, std::memory_order_relaxed);
  return B2_OK;
}

void scratch_free(void* p, cudaStream_t s) {
  if (p) cudaFreeAsync(p, s);
}

int parse_padding(const char* padding, bool* same) {
  if (padding && std::strcmp(padding, "SAME") == 0) {
    *same = true;
    return B2_OK;
  }
  if (padding && std::strcmp(padding, "VALID") == 0) {
    *same = false;
    return B2_OK;
  }
  return set_error(B2_ERR_INVALID_ARGUMENT, "padding must be 'SAME' or 'VALID', got '%s'",
                   padding ? padding : "(null)");
}

void resolve_padding(int64_t in, int64_t k, int64_t s, bool same, int64_t* out, int64_t* pad) {
  if (same) {
    *out = (in + s - 1) / s;
    int64_t total = (*out - 1) * s + k - in;
    if (total < 0) total = 0;
    *pad = total / 2;
  } else {
    *out = (in - k + s) / s;
    *pad = 0;
  }
}

int grid_for(int64_t work_items, int threads, int per_sm) {
  const DeviceInfo* d = nullptr;
  int sms = 148;
  if (device_info(&d) == B2_OK) sms = d->sm_count;
  int64_t need = ceil_div(work_items, threads);
  int64_t cap = (int64_t)sms * per_sm;
  if (need < 1) need = 1;
  return (int)(need < cap ? need : cap);
}

}  // namespace b2

// ====================================================================== ABI

using namespace b2;

extern "C" {

int b2_abi_version(void) { return B2_ABI_VERSION; }

const char* b2_last_error(void) { return t_last_error.c_str(); }

int b2_init(int device) {
  clear_error();
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess)
    return set_error(B2_ERR_NO_DEVICE, "cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(e));
  const DeviceInfo* d = nullptr;
  return device_info(&d);
}

int b2_resolve_padding(int64_t in_size, int64_t k, int64_t stride, const char* padding, int64_t* out_size,
                       int64_t* pad_before) {
  bool same = false;
  B2_RETURN_IF_ERROR(parse_padding(padding, &same));
  B2_REQUIRE(stride > 0, "strides must be positive");
  resolve_padding(in_size, k, stride, same, out_size, pad_before);
  return B2_OK;
}

int b2_pool_stats(b2_pool_stats_t* out) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  uint64_t v = 0;
  cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrUsedMemCurrent, &v);
  out->bytes_in_use = v;
  cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrReservedMemCurrent, &v);
  out->bytes_reserved = v;
  cudaMemPoolGetAttribute(d->pool, cudaMemPoolAttrUsedMemHigh, &v);
  out->peak_in_use = v;
  out->num_allocs = g_num_allocs[d->device].load(std::memory_order_relaxed);
  return B2_OK;
}

int b2_kernel_launch_count(uint64_t* count) {
  *count = g_launches.load(std::memory_order_relaxed);
  return B2_OK;
}

int b2_set_reserved_sms(int count) {
  clear_error();
  B2_REQUIRE(count >= 0, "the reserved SM count must be non-negative");
  g_reserved_sms.store(count, std::memory_order_relaxed);
  return B2_OK;
}

int b2_set_wait_limit_ns(uint64_t limit_ns) {
  clear_error();
  g_wait_limit_ns.store(limit_ns == 0 ? kDefaultWaitLimitNs : limit_ns, std::memory_order_relaxed);
  return B2_OK;
}

int b2_stream_status(b2_stream_t stream) {
  clear_error();
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  B2_CUDA_OR_RETURN(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  if (wait_expired()) {
    *static_cast<volatile unsigned int*>(g_expired_host) = 0u;
    return set_error(B2_ERR_TIMEOUT,
                     "a bounded device-side wait expired: the kernel gave up, so the outputs of the calls "
                     "enqueued before this check are invalid (state cleared)");
  }
  return B2_OK;
}

int b2_pool_trim(void) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  B2_CUDA_OR_RETURN(cudaDeviceSynchronize());
  B2_CUDA_OR_RETURN(cudaMemPoolTrimTo(d->pool, 0));
  return B2_OK;
}

}  // extern "C"
