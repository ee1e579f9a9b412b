// b2_internal.cuh -- shared helpers of the B200 backend (not part of the ABI).
//
// Error reporting, per-device state, the scratch pool and small numeric
// helpers used by every op file.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "b2_opencl_tf.h"

namespace b2 {

// ------------------------------------------------------------------ errors

// Records `fmt` as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

#define B2_REQUIRE(cond, ...)                                        \
  do {                                                               \
    if (!(cond)) return ::b2::set_error(B2_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define B2_CUDA_OR_RETURN(expr)                                                 \
  do {                                                                          \
    cudaError_t e_ = (expr);                                                    \
    if (e_ != cudaSuccess)                                                      \
      return ::b2::set_error(e_ == cudaErrorMemoryAllocation ? B2_ERR_OUT_OF_MEMORY \
                                                             : B2_ERR_INTERNAL, \
                             "%s failed (cuda_err=%d: %s)", #expr, (int)e_,     \
                             cudaGetErrorString(e_));                           \
  } while (0)

#define B2_RETURN_IF_ERROR(expr) \
  do {                           \
    int s_ = (expr);             \
    if (s_ != B2_OK) return s_;  \
  } while (0)

// Checks the last launch; with B2_DEBUG_CHECKS=1 in the environment it also
// synchronises the stream (outside graph capture) so a device fault is
// attributed to the op that caused it.  Returns B2_ERR_TIMEOUT while an
// expired device-side wait is pending (see WaitParams).
int check_launch(cudaStream_t s, const char* what);

// ------------------------------------------------------- bounded waits

// Every spin-wait in this library's kernels (the mbarrier waits of the
// tensor-core pipelines and of the staged depthwise filter gradient) gives up
// after limit_ns.  The kernel then counts the expiry on the device, stores 1
// into `expired` -- a word of host-mapped memory -- and tears its pipeline
// down cleanly (in-flight copies land, TMEM is freed).  check_launch() reads
// that word without synchronising, so every call made after the expiry became
// visible fails with B2_ERR_TIMEOUT until b2_stream_status() clears it.
struct WaitParams {
  uint64_t limit_ns;
  unsigned int* expired;  // host-mapped, device-visible; null if unavailable
};

constexpr uint64_t kDefaultWaitLimitNs = 10ull * 1000 * 1000 * 1000;  // 10 s

// The limit set by b2_set_wait_limit_ns (default 10 s) and the flag word.
WaitParams wait_params();

// Raises `kernel`'s dynamic shared-memory limit on the current device to at
// least `need` bytes before its first launch there.  The attribute belongs to the
// device's context, so it is tracked per device; concurrent first calls from
// several host threads are serialised.
struct SmemOptIn {
  static constexpr int kDevices = 64;
  std::atomic<int> bytes[kDevices] = {};
  std::mutex mu;
  int ensure(const void* kernel, int device, int need);
};

// ------------------------------------------------------------ device state

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  int max_smem_optin = 0;   // bytes of dynamic shared memory a CTA may opt into
  cudaMemPool_t pool = nullptr;
};

// Per-device state of the device current on the calling thread (created on
// first use; fails with B2_ERR_NO_DEVICE for anything but an sm_100 part).
int device_info(const DeviceInfo** out);

// CTAs of a persistent (one CTA per SM) kernel: the SM count less the SMs
// b2_set_reserved_sms keeps free for kernels that run beside this library's
// (NCCL's, during data-parallel training), at least 1.  Split-K GEMMs also
// size their splits to it (so no CTA takes a second slice), which changes
// the order of their additions: results stay deterministic for a given
// setting, and every rank of a data-parallel job uses the same one.
int persistent_ctas(const DeviceInfo* d);

// ---------------------------------------------------------------- scratch

// Stream-ordered scratch from the device's caching pool.  Legal inside CUDA
// graph capture (becomes a graph memory node there).
int scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

class Scratch {
 public:
  Scratch() = default;
  ~Scratch() { release(); }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  int alloc(size_t bytes, cudaStream_t s) {
    release();
    stream_ = s;
    return scratch_alloc(&ptr_, bytes, s);
  }
  template <class T>
  T* as() const { return static_cast<T*>(ptr_); }
  void release() {
    if (ptr_) scratch_free(ptr_, stream_);
    ptr_ = nullptr;
  }

 private:
  void* ptr_ = nullptr;
  cudaStream_t stream_ = nullptr;
};

// --------------------------------------------------------------- helpers

int parse_padding(const char* padding, bool* same);
// src/padding_utils.h:22-33
void resolve_padding(int64_t in, int64_t k, int64_t s, bool same, int64_t* out,
                     int64_t* pad);

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

constexpr int64_t kMaxInt32 = 2147483647LL;

// Grid size for a grid-stride kernel: enough CTAs to fill every SM
// `per_sm` times, never more than the work needs.
int grid_for(int64_t work_items, int threads, int per_sm);

}  // namespace b2
