// peer_exchange.cu -- averaging a small gradient across the GPUs of one node
// over NVLink peer memory, in one kernel per rank.
//
// The data-parallel step's last gradient (the first layer's weight, 12 KB at
// the README size) comes out of backward after every other one, so its
// exchange is always exposed; a ring all-reduce of a few KB is bound by the
// latency of its 2(N-1) steps.  Here every rank stores its copy directly into
// every rank's exchange block (P2P stores through NVSwitch), raises one flag
// per (rank, CTA) in every block, waits for the flags of all ranks and adds
// the N copies in rank order: one crossing of NVLink, and every rank computes
// the same bits.
//
// Exchange block of each rank (allocated by b2_peer_buffer_create, mapped in
// the other ranks' processes by b2_peer_buffer_open):
//   flags  [2][world][G] uint32   G = CTAs of the call (peer_ctas(n))
//   data   [2][world][n] float    (16-byte aligned)
// The half used by a call is its epoch's parity.  The epoch is a counter in
// the caller's device memory (counters[0]; counters[1] is a ticket), read at
// the start and advanced by the last CTA, so a captured call replays with
// increasing epochs.  A rank can be at most one call ahead of another (its
// next call waits for the other's flags of that call, raised only after the
// other finished the previous one), so the half it writes is never the half
// another rank is still reading.
//
// Every wait is bounded (WaitParams): on expiry the kernel leaves the data as
// it was, counts the expiry and sets the host-mapped expiry word, so the op
// calls that follow return B2_ERR_TIMEOUT.
#include <cstring>

#include "b2_internal.cuh"

namespace b2 {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kXThreads = 256;
constexpr int kMaxXCtas = 16;

struct PeerBases {
  uint8_t* base[kMaxRanks];
};

static __device__ unsigned int g_peer_timeouts = 0;

int peer_ctas(int64_t n) {
  const int64_t g = (n + 4095) / 4096;
  return (int)(g < 1 ? 1 : g > kMaxXCtas ? kMaxXCtas : g);
}

size_t flag_bytes(int world, int ctas) { return (size_t)ceil_div(2 * world * ctas * 4, 256) * 256; }

__device__ __forceinline__ void store_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kXThreads) peer_avg_kernel(float* __restrict__ data, int n, PeerBases pb,
                                                             int rank, int world, size_t fbytes,
                                                             unsigned int* __restrict__ counters,
                                                             WaitParams wp) {
  __shared__ unsigned int s_epoch;
  __shared__ int s_ok;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile unsigned int*>(counters) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned int e = s_epoch;
  const int par = (int)(e & 1u);
  const int per = (n + G - 1) / G;
  const int lo = c * per, hi = lo + per < n ? lo + per : n;

  // 1. this rank's slice into every rank's block (its own included)
  for (int r = 0; r < world; ++r) {
    float* dst = reinterpret_cast<float*>(pb.base[r] + fbytes) + ((size_t)par * world + rank) * n;
    for (int i = lo + tid; i < hi; i += kXThreads) dst[i] = data[i];
  }
  __syncthreads();
  // 2. one flag per rank: the stores above are visible before it
  if (tid == 0) {
    __threadfence_system();
    for (int r = 0; r < world; ++r) {
      unsigned int* f = reinterpret_cast<unsigned int*>(pb.base[r]) + ((size_t)par * world + rank) * G + c;
      store_release_sys(f, e);
    }
  }
  // 3. wait for every rank's slice c in this rank's block
  if (tid < world) {
    const unsigned int* f = reinterpret_cast<const unsigned int*>(pb.base[rank]) + ((size_t)par * world + tid) * G + c;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (load_acquire_sys(f) != e) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > wp.limit_ns) {
        atomicAdd(&g_peer_timeouts, 1u);
        if (wp.expired) {
          *reinterpret_cast<volatile unsigned int*>(wp.expired) = 1u;
          __threadfence_system();
        }
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  // 4. the average, ranks added in order (the same bits on every rank)
  if (s_ok) {
    const float* src = reinterpret_cast<const float*>(pb.base[rank] + fbytes) + (size_t)par * world * n;
    const float inv = 1.0f / (float)world;  // exact for 1, 2, 4, 8
    for (int i = lo + tid; i < hi; i += kXThreads) {
      float s = src[i];
      for (int r = 1; r < world; ++r) s = __fadd_rn(s, src[(size_t)r * n + i]);
      data[i] = __fmul_rn(s, inv);
    }
  }
  // 5. the last CTA advances the epoch (every CTA has read it by then)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(counters + 1, 1u) == (unsigned int)G - 1u) {
      counters[0] = e;
      counters[1] = 0u;
      __threadfence();
    }
  }
}

}  // namespace

unsigned int peer_timeouts() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_peer_timeouts, sizeof(v));
  return v;
}

}  // namespace b2

using namespace b2;

extern "C" {

size_t b2_peer_exchange_bytes(int64_t n, int world) {
  if (n <= 0 || world < 1 || world > kMaxRanks) return 0;
  return flag_bytes(world, peer_ctas(n)) + (size_t)ceil_div(2 * world * n * 4, 256) * 256;
}

int b2_peer_buffer_create(size_t bytes, void** ptr, unsigned char handle[64]) {
  clear_error();
  B2_REQUIRE(ptr != nullptr && handle != nullptr && bytes > 0, "peer buffer: bad arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  void* p = nullptr;
  B2_CUDA_OR_RETURN(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(B2_ERR_INTERNAL, "peer buffer: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, 64);
  *ptr = p;
  return B2_OK;
}

int b2_peer_buffer_open(const unsigned char handle[64], void** ptr) {
  clear_error();
  B2_REQUIRE(ptr != nullptr && handle != nullptr, "peer buffer: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  B2_CUDA_OR_RETURN(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return B2_OK;
}

int b2_peer_buffer_close(void* peer_ptr) {
  clear_error();
  B2_CUDA_OR_RETURN(cudaIpcCloseMemHandle(peer_ptr));
  return B2_OK;
}

int b2_peer_buffer_free(void* ptr) {
  clear_error();
  B2_CUDA_OR_RETURN(cudaFree(ptr));
  return B2_OK;
}

int b2_peer_allreduce_avg(b2_stream_t stream, float* data, int64_t n, int rank, int world,
                          void* const* peer_blocks, unsigned int* counters) {
  clear_error();
  B2_REQUIRE(world >= 1 && world <= kMaxRanks, "peer exchange: world must be 1 .. %d", kMaxRanks);
  B2_REQUIRE(rank >= 0 && rank < world, "peer exchange: rank out of range");
  B2_REQUIRE(n >= 0 && n <= kMaxInt32 / (2 * kMaxRanks), "peer exchange: too many elements");
  B2_REQUIRE(peer_blocks != nullptr && counters != nullptr, "peer exchange: missing buffers");
  if (n == 0) return B2_OK;
  B2_REQUIRE(data != nullptr, "peer exchange: missing data");
  PeerBases pb{};
  for (int r = 0; r < world; ++r) {
    B2_REQUIRE(peer_blocks[r] != nullptr && aligned16(peer_blocks[r]), "peer exchange: block %d missing or unaligned",
               r);
    pb.base[r] = static_cast<uint8_t*>(peer_blocks[r]);
  }
  const int G = peer_ctas(n);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  peer_avg_kernel<<<G, kXThreads, 0, s>>>(data, (int)n, pb, rank, world, flag_bytes(world, G), counters,
                                          wait_params());
  return check_launch(s, "peer_allreduce_avg");
}

}  // extern "C"
