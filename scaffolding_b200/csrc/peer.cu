// Copy-engine data exchange between the GPUs of one node, one process per
// GPU: device buffers shared through CUDA IPC handles, and 32-bit sequence
// flags that a one-thread kernel stores into a peer's memory (release, system
// scope) and a one-CTA kernel waits on (acquire, bounded by the global timer).
//
// The token-sharded DiT stack uses them for its per-layer K/V exchange
// (scaffolding_b200/dit.py): each rank's K/V rows are pushed into its peers'
// key buffers by cudaMemcpyAsync on side streams, so the copy runs on the
// copy engines over NVLink and takes no SMs from the attention running at
// the same time, in place of the all-gather kernel of the reference's
// DataParallel path (nn/parallel.py:229-267 gathers through the host).
//
// A wait never spins on work of the same GPU: the flags it waits on are
// stored by kernels of the other ranks' processes, each of which runs on its
// own GPU.  A wait that has not seen its value after the time limit records
// kDevTimeoutPeer in the device error word and returns.
#include <cuda_runtime.h>

#include <cstring>

#include "common.h"
#include "ptx.cuh"

namespace sf {
namespace {

constexpr int kMaxFlags = 8;

struct FlagList {
  int32_t* ptr[kMaxFlags];
};

__global__ void flag_store_kernel(FlagList f, int count, int32_t value) {
  const int i = threadIdx.x;
  if (i >= count) return;
  // Every earlier write of this stream's kernels and copies is complete
  // when this kernel starts; the release store orders the flag after them
  // for a reader on another GPU.
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f.ptr[i]), "r"(value) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread i waits until flags[i * stride] >= value (i != skip).
__global__ void flag_wait_kernel(const int32_t* flags, int count, int stride, int skip,
                                 int32_t value, unsigned long long limit_ns, int* err) {
  const int i = threadIdx.x;
  if (i < count && i != skip) {
    const int32_t* p = flags + static_cast<int64_t>(i) * stride;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_sys(p) < value) {
      if (global_timer_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, kDevTimeoutPeer);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncthreads();
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int32_t sf_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(SF_ERR_INVALID_ARGUMENT, "sf_ipc_alloc: null output or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  SF_CUDA_TRY(cudaMalloc(&p, bytes));
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return fail(SF_ERR_CUDA, "sf_ipc_alloc: %s", cudaGetErrorString(cudaGetLastError()));
  }
  SF_CUDA_TRY(cudaDeviceSynchronize());
  *ptr = p;
  return SF_OK;
}

int32_t sf_ipc_free(void* ptr) {
  if (!ptr) return SF_OK;
  SF_CUDA_TRY(cudaFree(ptr));
  return SF_OK;
}

int32_t sf_ipc_handle(void* ptr, uint8_t* handle) {
  if (!ptr || !handle) return fail(SF_ERR_INVALID_ARGUMENT, "sf_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  SF_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
  static_assert(sizeof(h) == SF_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return SF_OK;
}

int32_t sf_ipc_open(const uint8_t* handle, void** ptr) {
  if (!ptr || !handle) return fail(SF_ERR_INVALID_ARGUMENT, "sf_ipc_open: null argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  SF_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return SF_OK;
}

int32_t sf_ipc_close(void* ptr) {
  if (!ptr) return SF_OK;
  SF_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return SF_OK;
}

int32_t sf_flag_store(int32_t* const* flags, int32_t count, int32_t value, void* stream) {
  if (count < 0 || count > kMaxFlags) return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_store: %d flags (at most %d)", count, kMaxFlags);
  if (count == 0) return SF_OK;
  if (!flags) return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_store: null flag list");
  FlagList f{};
  for (int i = 0; i < count; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u))
      return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_store: flag %d null or misaligned", i);
    f.ptr[i] = flags[i];
  }
  flag_store_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, count, value);
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

int32_t sf_flag_wait(const int32_t* flags, int32_t count, int32_t stride, int32_t skip,
                     int32_t value, int64_t timeout_ns, void* stream) {
  if (count < 0 || count > 1024 || stride < 1) return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_wait: count %d stride %d", count, stride);
  if (count == 0) return SF_OK;
  if (!flags || (reinterpret_cast<uintptr_t>(flags) & 3u)) return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_wait: null or misaligned flags");
  if (timeout_ns < 0) return fail(SF_ERR_INVALID_ARGUMENT, "sf_flag_wait: negative time limit");
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  const unsigned long long limit = timeout_ns == 0 ? kWaitLimitNs : static_cast<unsigned long long>(timeout_ns);
  const int threads = (count + 31) / 32 * 32;
  flag_wait_kernel<<<1, threads, 0, static_cast<cudaStream_t>(stream)>>>(flags, count, stride, skip, value,
                                                                          limit, dev->err_word);
  SF_CUDA_TRY(cudaGetLastError());
  return SF_OK;
}

}  // extern "C"
