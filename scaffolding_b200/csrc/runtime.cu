// Runtime services of the engine's C ABI: error reporting, per-device state,
// the caching allocator, copies, streams, events and peer access.
//
// These replace the Cython runtime of the reference (_cuda_ops.pyx:307-685):
// the allocator keeps the reference's policy -- exact-size free lists per
// (device, rounded size), 256-byte rounding, a per-device cap on cached
// bytes above which freed blocks are returned to the driver
// (_cuda_ops.pyx:356-475) -- but lives in C++ behind a mutex so it can be
// called with the GIL released, and its cap defaults to 32 GiB instead of
// 2 GB because a B200 holds 180 GB and the attention score buffers of the
// DiT workload alone are several GB.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace sf {

static thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int32_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SF_OK;
  const int32_t code = (e == cudaErrorMemoryAllocation) ? SF_ERR_OUT_OF_MEMORY : SF_ERR_CUDA;
  return fail(code, "CUDA error %d (%s) in %s", static_cast<int>(e), cudaGetErrorString(e), what);
}

// ───────────────────────────── per-device state ─────────────────────────────

static std::mutex g_dev_mu;
static std::vector<DeviceInfo> g_devs;

int32_t current_device_info(DeviceInfo** out, int* device) {
  int dev = 0;
  SF_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_devs.empty()) {
    int n = 0;
    SF_CUDA_TRY(cudaGetDeviceCount(&n));
    g_devs.resize(std::max(n, 1));
  }
  if (dev < 0 || dev >= static_cast<int>(g_devs.size()))
    return fail(SF_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
  DeviceInfo& d = g_devs[dev];
  if (d.err_word == nullptr) {
    cudaDeviceProp prop;
    SF_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    d.sm_count = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.smem_optin = prop.sharedMemPerBlockOptin;
    int* w = nullptr;
    SF_CUDA_TRY(cudaMalloc(&w, 256));
    SF_CUDA_TRY(cudaMemset(w, 0, 256));
    d.err_word = w;
  }
  *out = &d;
  if (device) *device = dev;
  return SF_OK;
}

// ───────────────────────────── knobs ─────────────────────────────

static int g_fp32_mode = SF_FP32_ACCURATE;
static int g_kernel_override = SF_KERNEL_AUTO;
int fp32_mode() { return g_fp32_mode; }
int kernel_override() { return g_kernel_override; }

// ───────────────────────────── caching allocator ─────────────────────────────

namespace {
constexpr size_t kAlign = 256;
size_t round_up(size_t n) { return n == 0 ? kAlign : (n + kAlign - 1) & ~(kAlign - 1); }

struct Pool {
  std::unordered_map<size_t, std::vector<void*>> free_lists;  // rounded size -> blocks
  size_t cached = 0;     // bytes sitting in free lists
  size_t allocated = 0;  // bytes handed out and not yet returned
};
std::mutex g_pool_mu;
std::map<int, Pool> g_pools;
size_t g_pool_cap = static_cast<size_t>(32) << 30;

struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) {
      switched = cudaSetDevice(dev) == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};
}  // namespace

}  // namespace sf

using namespace sf;

extern "C" {

const char* sf_last_error(void) { return g_last_error.c_str(); }
const char* sf_version(void) { return "scaffolding-b200 engine 0.1 (sm_100a)"; }

int32_t sf_set_fp32_mode(int32_t mode) {
  if (mode != SF_FP32_ACCURATE && mode != SF_FP32_FFMA && mode != SF_FP32_TF32)
    return fail(SF_ERR_INVALID_ARGUMENT, "unknown fp32 mode %d", mode);
  g_fp32_mode = mode;
  return SF_OK;
}
int32_t sf_get_fp32_mode(int32_t* mode) {
  if (!mode) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  *mode = g_fp32_mode;
  return SF_OK;
}
int32_t sf_set_kernel_override(int32_t kernel) {
  if (kernel < SF_KERNEL_AUTO || kernel > SF_KERNEL_TCGEN05_1CTA)
    return fail(SF_ERR_INVALID_ARGUMENT, "unknown kernel override %d", kernel);
  g_kernel_override = kernel;
  return SF_OK;
}

int32_t sf_device_count(int32_t* count) {
  if (!count) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    *count = 0;
    return SF_OK;
  }
  SF_CUDA_TRY(e);
  *count = n;
  return SF_OK;
}

int32_t sf_set_device(int32_t device) {
  SF_CUDA_TRY(cudaSetDevice(device));
  return SF_OK;
}

int32_t sf_get_device(int32_t* device) {
  if (!device) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  int d = 0;
  SF_CUDA_TRY(cudaGetDevice(&d));
  *device = d;
  return SF_OK;
}

int32_t sf_device_synchronize(void) {
  SF_CUDA_TRY(cudaDeviceSynchronize());
  return SF_OK;
}

int32_t sf_device_properties(int32_t device, sf_device_props* out) {
  if (!out) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  cudaDeviceProp p;
  SF_CUDA_TRY(cudaGetDeviceProperties(&p, device));
  memset(out, 0, sizeof(*out));
  strncpy(out->name, p.name, sizeof(out->name) - 1);
  out->total_memory = p.totalGlobalMem;
  out->major = p.major;
  out->minor = p.minor;
  out->multi_processor_count = p.multiProcessorCount;
  out->max_threads_per_block = p.maxThreadsPerBlock;
  out->max_threads_per_mp = p.maxThreadsPerMultiProcessor;
  out->warp_size = p.warpSize;
  out->shared_mem_per_block = p.sharedMemPerBlock;
  out->shared_mem_per_block_optin = p.sharedMemPerBlockOptin;
  out->l2_cache_size = p.l2CacheSize;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrClockRate, device) == cudaSuccess) out->clock_rate_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMemoryClockRate, device) == cudaSuccess)
    out->memory_clock_rate_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrGlobalMemoryBusWidth, device) == cudaSuccess)
    out->memory_bus_width = v;
  return SF_OK;
}

int32_t sf_mem_info(size_t* free_bytes, size_t* total_bytes) {
  if (!free_bytes || !total_bytes) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  SF_CUDA_TRY(cudaMemGetInfo(free_bytes, total_bytes));
  return SF_OK;
}

int32_t sf_malloc(int32_t device, size_t bytes, void** ptr) {
  if (!ptr) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  const size_t sz = round_up(bytes);
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    Pool& pool = g_pools[device];
    auto it = pool.free_lists.find(sz);
    if (it != pool.free_lists.end() && !it->second.empty()) {
      *ptr = it->second.back();
      it->second.pop_back();
      pool.cached -= sz;
      pool.allocated += sz;
      return SF_OK;
    }
  }
  DeviceGuard g(device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, sz);
  if (e == cudaErrorMemoryAllocation) {
    // Out of memory: release cached blocks of this device and retry once.
    cudaGetLastError();
    sf_empty_cache(device);
    e = cudaMalloc(&p, sz);
  }
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
  std::lock_guard<std::mutex> lk(g_pool_mu);
  g_pools[device].allocated += sz;
  *ptr = p;
  return SF_OK;
}

int32_t sf_free(int32_t device, void* ptr, size_t bytes) {
  if (!ptr) return SF_OK;
  const size_t sz = round_up(bytes);
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    Pool& pool = g_pools[device];
    pool.allocated -= std::min(pool.allocated, sz);
    if (pool.cached + sz <= g_pool_cap) {
      pool.free_lists[sz].push_back(ptr);
      pool.cached += sz;
      return SF_OK;
    }
  }
  DeviceGuard g(device);
  SF_CUDA_TRY(cudaFree(ptr));
  return SF_OK;
}

int32_t sf_empty_cache(int32_t device) {
  std::vector<std::pair<int, void*>> victims;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    for (auto& kv : g_pools) {
      if (device >= 0 && kv.first != device) continue;
      for (auto& fl : kv.second.free_lists)
        for (void* p : fl.second) victims.emplace_back(kv.first, p);
      kv.second.free_lists.clear();
      kv.second.cached = 0;
    }
  }
  for (auto& v : victims) {
    DeviceGuard g(v.first);
    cudaFree(v.second);
  }
  return SF_OK;
}

int32_t sf_pool_stats(int32_t device, size_t* cached_bytes, size_t* allocated_bytes) {
  std::lock_guard<std::mutex> lk(g_pool_mu);
  Pool& pool = g_pools[device];
  if (cached_bytes) *cached_bytes = pool.cached;
  if (allocated_bytes) *allocated_bytes = pool.allocated;
  return SF_OK;
}

int32_t sf_set_pool_cap(size_t bytes_per_device) {
  std::lock_guard<std::mutex> lk(g_pool_mu);
  g_pool_cap = bytes_per_device;
  return SF_OK;
}

int32_t sf_host_alloc_pinned(size_t bytes, void** ptr) {
  if (!ptr) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  SF_CUDA_TRY(cudaHostAlloc(ptr, bytes ? bytes : 1, cudaHostAllocPortable));
  return SF_OK;
}

int32_t sf_host_free_pinned(void* ptr) {
  if (ptr) SF_CUDA_TRY(cudaFreeHost(ptr));
  return SF_OK;
}

int32_t sf_memcpy(void* dst, const void* src, size_t bytes, int32_t kind, void* stream) {
  if (bytes == 0) return SF_OK;
  if (!dst || !src) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer in sf_memcpy");
  cudaMemcpyKind k;
  switch (kind) {
    case 0: k = cudaMemcpyHostToDevice; break;
    case 1: k = cudaMemcpyDeviceToHost; break;
    case 2: k = cudaMemcpyDeviceToDevice; break;
    case 3: k = cudaMemcpyDefault; break;
    default: return fail(SF_ERR_INVALID_ARGUMENT, "unknown copy kind %d", kind);
  }
  SF_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_memcpy_peer(void* dst, int32_t dst_device, const void* src, int32_t src_device,
                       size_t bytes, void* stream) {
  if (bytes == 0) return SF_OK;
  if (!dst || !src) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer in sf_memcpy_peer");
  SF_CUDA_TRY(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, bytes,
                                  static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_memset(void* dst, int32_t value, size_t bytes, void* stream) {
  if (bytes == 0) return SF_OK;
  SF_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_stream_create(int32_t device, int32_t non_blocking, void** stream) {
  if (!stream) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  DeviceGuard g(device);
  cudaStream_t s;
  SF_CUDA_TRY(cudaStreamCreateWithFlags(&s, non_blocking ? cudaStreamNonBlocking : cudaStreamDefault));
  *stream = s;
  return SF_OK;
}

int32_t sf_stream_create_priority(int32_t device, int32_t non_blocking, int32_t high_priority,
                                  void** stream) {
  if (!stream) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  DeviceGuard g(device);
  int least = 0, greatest = 0;
  SF_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  cudaStream_t s;
  SF_CUDA_TRY(cudaStreamCreateWithPriority(
      &s, non_blocking ? cudaStreamNonBlocking : cudaStreamDefault,
      high_priority ? greatest : least));
  *stream = s;
  return SF_OK;
}

int32_t sf_stream_destroy(void* stream) {
  if (!stream) return SF_OK;
  attention_release_stream(stream);
  SF_CUDA_TRY(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_stream_synchronize(void* stream) {
  SF_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_stream_wait_event(void* stream, void* event) {
  SF_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
  return SF_OK;
}

int32_t sf_event_create(int32_t enable_timing, void** event) {
  if (!event) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  cudaEvent_t e;
  SF_CUDA_TRY(cudaEventCreateWithFlags(&e, enable_timing ? cudaEventDefault : cudaEventDisableTiming));
  *event = e;
  return SF_OK;
}

int32_t sf_event_destroy(void* event) {
  if (event) SF_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return SF_OK;
}

int32_t sf_event_record(void* event, void* stream) {
  SF_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_event_synchronize(void* event) {
  SF_CUDA_TRY(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
  return SF_OK;
}

int32_t sf_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!ms) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  SF_CUDA_TRY(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)));
  return SF_OK;
}

int32_t sf_graph_begin(void* stream) {
  if (!stream) return fail(SF_ERR_INVALID_ARGUMENT, "graph capture needs a non-default stream");
  SF_CUDA_TRY(cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeRelaxed));
  return SF_OK;
}

int32_t sf_graph_end(void* stream, void** exec) {
  if (!stream || !exec) return fail(SF_ERR_INVALID_ARGUMENT, "null argument");
  cudaGraph_t g = nullptr;
  SF_CUDA_TRY(cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &g));
  cudaGraphExec_t e = nullptr;
  cudaError_t err = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  if (err != cudaSuccess) return cuda_status(err, "cudaGraphInstantiate");
  *exec = e;
  return SF_OK;
}

int32_t sf_graph_launch(void* exec, void* stream) {
  if (!exec) return fail(SF_ERR_INVALID_ARGUMENT, "null graph");
  SF_CUDA_TRY(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), static_cast<cudaStream_t>(stream)));
  return SF_OK;
}

int32_t sf_graph_destroy(void* exec) {
  if (exec) SF_CUDA_TRY(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)));
  return SF_OK;
}

int32_t sf_can_access_peer(int32_t device, int32_t peer, int32_t* can) {
  if (!can) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  int c = 0;
  SF_CUDA_TRY(cudaDeviceCanAccessPeer(&c, device, peer));
  *can = c;
  return SF_OK;
}

int32_t sf_enable_peer_access_all(void) {
  int n = 0;
  SF_CUDA_TRY(cudaGetDeviceCount(&n));
  int prev = 0;
  SF_CUDA_TRY(cudaGetDevice(&prev));
  for (int i = 0; i < n; ++i) {
    SF_CUDA_TRY(cudaSetDevice(i));
    for (int j = 0; j < n; ++j) {
      if (i == j) continue;
      int c = 0;
      cudaDeviceCanAccessPeer(&c, i, j);
      if (c) {
        cudaError_t e = cudaDeviceEnablePeerAccess(j, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
        else if (e != cudaSuccess) {
          cudaSetDevice(prev);
          return cuda_status(e, "cudaDeviceEnablePeerAccess");
        }
      }
    }
  }
  SF_CUDA_TRY(cudaSetDevice(prev));
  return SF_OK;
}

int32_t sf_device_error_status(int32_t device, int32_t* code, int32_t clear) {
  if (!code) return fail(SF_ERR_INVALID_ARGUMENT, "null output");
  DeviceGuard g(device);
  DeviceInfo* info = nullptr;
  int32_t st = current_device_info(&info, nullptr);
  if (st != SF_OK) return st;
  int v = 0;
  SF_CUDA_TRY(cudaMemcpy(&v, info->err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) SF_CUDA_TRY(cudaMemset(info->err_word, 0, sizeof(int)));
  // The no-alloc linear records its timeouts in its own static word.
  int w = 0;
  st = noalloc_error_word(&w, clear != 0);
  if (st != SF_OK) return st;
  *code = v != 0 ? v : w;
  return SF_OK;
}

}  // extern "C"
