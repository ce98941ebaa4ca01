// Fused-attention entry points of the C ABI (sf_attention_fwd,
// sf_attention_fwd_partial, sf_attention_launch_count): argument checks,
// TMA descriptors, kernel choice, the stream-K tail of the last wave and
// its workspace.
//
// Kernel: attention_pp_kernel (attention_pp.cuh) with two 128-row query tiles
// per CTA and 64-key blocks (S and P in TMEM, O in a TMEM accumulator, integer
// row bases raised lazily), plus attention_merge_kernel for the parts of the
// units that the stream-K tail splits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

#include "attention.cuh"
#include "attention_pp.cuh"
#include "common.h"
#include "tma_host.h"

namespace sf {
namespace {

// Two 128-row query tiles per CTA, 64-key blocks, 4-stage K/V ring: 256 TMEM
// columns and ~96 KB of shared memory, two CTAs per SM.
using AttnCfg = AttnPpCfg<2, 64, 4>;

// `tail_ctas` stream-K tail CTAs (none when 0), then the whole units on
// `grid` (none when grid.x == 0).  The tail kernel triggers its dependents at
// once, so the whole units' kernel, launched with programmatic stream
// serialisation, starts on the slots the tail CTAs leave: the two run as one
// grid.  Neither reads what the other writes; work later in the stream waits
// for both.
template <bool BF16>
int32_t launch_attention(const dim3& grid, int tail_ctas, const CUtensorMap& mq,
                         const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a,
                         cudaStream_t s, int device) {
  static bool attr_set[64] = {false};
  if (device < 64 && !attr_set[device]) {
    SF_CUDA_TRY(cudaFuncSetAttribute(attention_pp_kernel<BF16, AttnCfg>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg::BYTES));
    SF_CUDA_TRY(cudaFuncSetAttribute(attention_pp_tail_kernel<BF16, AttnCfg>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg::BYTES));
    attr_set[device] = true;
  }
  if (tail_ctas > 0)
    attention_pp_tail_kernel<BF16, AttnCfg>
        <<<dim3(static_cast<unsigned>(tail_ctas)), AttnCfg::THREADS, AttnCfg::BYTES, s>>>(mq, mk, mv, a);
  if (grid.x > 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(AttnCfg::THREADS);
    cfg.dynamicSmemBytes = AttnCfg::BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = tail_ctas > 0 ? 1 : 0;
    SF_CUDA_TRY(cudaLaunchKernelEx(&cfg, attention_pp_kernel<BF16, AttnCfg>, mq, mk, mv, a));
  }
  return SF_OK;
}

// Key blocks of a unit over keys [0, kv_len) minus [skip_lo, skip_hi):
// *na blocks from key 0, then blocks from skip_hi; *ne in all.
void attn_key_blocks(int kv_len, int skip_lo, int skip_hi, int* na, int* ne) {
  const int kb = AttnCfg::KB;
  *na = skip_lo > 0 ? static_cast<int>(ceil_div(skip_lo, kb)) : 0;
  *ne = *na + (kv_len > skip_hi ? static_cast<int>(ceil_div(kv_len - skip_hi, kb)) : 0);
}

// Stream-K tail plan (see AttnArgs::split_first).  U units on P resident CTA
// slots run floor(U / P) full waves of whole units; the other R = U mod P
// units' ne key blocks each are shared by T = min(P, max(R, R ne /
// kTailMinBlocks)) tail CTAs.  Cost in block steps: the last wave of whole
// units takes ne; the tail takes ceil(R ne / T) plus about kTailCost for the
// second segment's pipeline restart, the parts' fp32 traffic and the merge
// launch (measured on B200: 70-block units lose with the tail, 139-block
// units gain 7 %).  The tail is used when it saves more than 3 %.
constexpr int kTailMinBlocks = 16;
constexpr double kTailCost = 16.0;
struct AttnTail {
  int split_first = -1, ctas = 0, units = 0;
};
AttnTail attn_tail_plan(int64_t units, int slots, int ne) {
  AttnTail tp;
  // Test hook: SF_ATTN_SPLIT=0 keeps the one-CTA-per-unit grid, 2 forces the
  // tail whenever the last wave is partial.
  const int hook = env_int("SF_ATTN_SPLIT", 1);
  if (hook == 0 || slots <= 0 || ne < 2) return tp;
  const int64_t full = units / slots, rem = units % slots;
  if (rem == 0) return tp;
  const int64_t ctas = std::min<int64_t>(slots, std::max<int64_t>(rem, rem * ne / kTailMinBlocks));
  if (hook != 2) {
    const double tail = static_cast<double>((rem * ne + ctas - 1) / ctas) + kTailCost;
    if (tail > 0.97 * ne - 0.03 * static_cast<double>(full) * ne) return tp;
  }
  tp.split_first = static_cast<int>(full * slots);
  tp.ctas = static_cast<int>(ctas);
  tp.units = static_cast<int>(rem);
  return tp;
}

// Workspace of the tail's parts, one per (device, stream) so that calls on
// different streams never share it; calls on one stream run in order.  The
// per-thread default stream (cudaStreamPerThread) is a different stream in
// every host thread, so its key also carries the thread.  A workspace grows
// on demand (to twice the size asked for) and is never shrunk.  A buffer
// that was handed to a launch while its stream was being captured may be
// referenced by a CUDA graph that outlives any later call, so it is never
// freed: when it is outgrown, or its stream is destroyed, it moves to a
// retired list kept until the process exits.  Other buffers are freed then
// (cudaFree waits for the work already queued on them).  A graph captured on
// stream S and replayed on another stream still uses S's workspace, so its
// replays must not overlap with direct calls on S.
struct AttnWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool captured = false;  // handed out during a stream capture
};
struct AttnWsKey {
  int device;
  void* stream;
  uint64_t thread;  // nonzero only for cudaStreamPerThread
  bool operator<(const AttnWsKey& o) const {
    if (device != o.device) return device < o.device;
    if (stream != o.stream) return stream < o.stream;
    return thread < o.thread;
  }
};
std::mutex g_attn_ws_mu;
std::map<AttnWsKey, AttnWorkspace> g_attn_ws;
std::vector<void*> g_attn_ws_retired;

uint64_t this_thread_tag() {
  static thread_local int tag;
  return static_cast<uint64_t>(reinterpret_cast<uintptr_t>(&tag));
}

// Drops a workspace buffer: retired if a capture may hold it, else freed.
// Called with g_attn_ws_mu held.
void attn_ws_drop(AttnWorkspace& ws) {
  if (ws.ptr) {
    if (ws.captured)
      g_attn_ws_retired.push_back(ws.ptr);
    else if (cudaFree(ws.ptr) != cudaSuccess)
      cudaGetLastError();
  }
  ws = AttnWorkspace{};
}

int32_t attention_impl(int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                       int32_t head_dim, const void* q, int64_t ldq, int64_t q_bstride,
                       const void* k, int64_t ldk, int64_t k_bstride, const void* v, int64_t ldv,
                       int64_t v_bstride, void* o, int64_t ldo, int64_t o_bstride, float scale,
                       int32_t dtype, int32_t skip_lo, int32_t skip_hi, float* part_o,
                       float* part_ml, int32_t part_mode, void* stream) {
  if (batch < 0 || heads < 0 || q_len < 0 || kv_len < 0)
    return fail(SF_ERR_INVALID_ARGUMENT, "negative size");
  if (batch == 0 || heads == 0 || q_len == 0) return SF_OK;
  if (kv_len == 0) return fail(SF_ERR_INVALID_ARGUMENT, "attention over zero keys");
  if (head_dim != kAttnD) return fail(SF_ERR_UNSUPPORTED, "fused attention needs head_dim 64 (got %d)", head_dim);
  if (dtype != kBF16 && dtype != kF16) return fail(SF_ERR_INVALID_ARGUMENT, "fused attention dtype %d", dtype);
  if (!(scale > 0.0f)) return fail(SF_ERR_INVALID_ARGUMENT, "attention scale must be positive");
  if (!q || !k || !v || !o) return fail(SF_ERR_INVALID_ARGUMENT, "null pointer");
  for (const void* ptr : {q, k, v, static_cast<const void*>(o)})
    if (!aligned16(ptr)) return fail(SF_ERR_INVALID_ARGUMENT, "attention operands must be 16-byte aligned");
  for (int64_t st : {ldq, ldk, ldv, ldo, q_bstride, k_bstride, v_bstride, o_bstride})
    if (!bytes16(st, 2) || st < 0) return fail(SF_ERR_INVALID_ARGUMENT, "attention strides must be 16-byte multiples");
  const int64_t row_min = static_cast<int64_t>(heads) * head_dim;
  if (ldq < row_min || ldk < row_min || ldv < row_min || ldo < row_min)
    return fail(SF_ERR_INVALID_ARGUMENT, "leading dimension < heads * head_dim");
  if (heads > 65535 || batch > 65535) return fail(SF_ERR_UNSUPPORTED, "attention grid");
  DeviceInfo* dev = nullptr;
  int device = 0;
  int32_t st = current_device_info(&dev, &device);
  if (st != SF_OK) return st;
  if (dev->cc_major != 10) return fail(SF_ERR_UNSUPPORTED, "fused attention needs sm_100");
  const CUtensorMapDataType dt = tma_dtype(dtype);
  const int rows = AttnCfg::ROWS;
  const uint32_t kb = static_cast<uint32_t>(AttnCfg::KB);
  CUtensorMap mq, mk, mv;
  MapSpec sq{q, 2, dt, static_cast<uint64_t>(head_dim), static_cast<uint64_t>(q_len),
             static_cast<uint64_t>(heads), static_cast<uint64_t>(batch), ldq, head_dim, q_bstride,
             static_cast<uint32_t>(head_dim), static_cast<uint32_t>(kAttnBlock)};
  MapSpec sk{k, 2, dt, static_cast<uint64_t>(head_dim), static_cast<uint64_t>(kv_len),
             static_cast<uint64_t>(heads), static_cast<uint64_t>(batch), ldk, head_dim, k_bstride,
             static_cast<uint32_t>(head_dim), kb};
  MapSpec sv{v, 2, dt, static_cast<uint64_t>(head_dim), static_cast<uint64_t>(kv_len),
             static_cast<uint64_t>(heads), static_cast<uint64_t>(batch), ldv, head_dim, v_bstride,
             static_cast<uint32_t>(head_dim), kb};
  if ((st = encode_map(&mq, sq)) != SF_OK) return st;
  if ((st = encode_map(&mk, sk)) != SF_OK) return st;
  if ((st = encode_map(&mv, sv)) != SF_OK) return st;
  AttnArgs a;
  a.q_len = q_len;
  a.kv_len = kv_len;
  a.heads = heads;
  a.batch = batch;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.o = o;
  a.out_dtype = dtype;
  a.ldo = ldo;
  a.o_bstride = o_bstride;
  a.err = dev->err_word;
  a.skip_lo = skip_lo;
  a.skip_hi = skip_hi;
  a.part_mode = part_mode;
  a.part_o = part_o;
  a.part_ml = part_ml;
  attn_key_blocks(kv_len, skip_lo, skip_hi, &a.nkb_a, &a.nkb_e);
  a.split_first = -1;
  a.tail_ctas = a.tail_units = 0;
  a.nqb = static_cast<int>(ceil_div(q_len, rows));
  a.ws_o = a.ws_ml = nullptr;
  dim3 grid(static_cast<unsigned>(a.nqb), static_cast<unsigned>(heads), static_cast<unsigned>(batch));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const AttnTail tp = attn_tail_plan(static_cast<int64_t>(a.nqb) * heads * batch,
                                     AttnCfg::MIN_BLOCKS * dev->sm_count, a.nkb_e);
  // Held until the launches are queued, so that no other thread's call on the
  // same stream regrows (frees) the workspace in between.
  std::unique_lock<std::mutex> ws_lock(g_attn_ws_mu, std::defer_lock);
  if (tp.split_first >= 0) {
    const size_t need = static_cast<size_t>(2 * tp.ctas) * rows * (kAttnD + 2) * sizeof(float);
    ws_lock.lock();
    const AttnWsKey key{device, stream, s == cudaStreamPerThread ? this_thread_tag() : 0};
    AttnWorkspace& ws = g_attn_ws[key];
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    SF_CUDA_TRY(cudaStreamIsCapturing(s, &cap));
    // No allocation while the stream is being captured: use the 3-D grid then.
    if (ws.bytes < need && cap == cudaStreamCaptureStatusNone) {
      attn_ws_drop(ws);
      SF_CUDA_TRY(cudaMalloc(&ws.ptr, 2 * need));
      ws.bytes = 2 * need;
    }
    if (ws.bytes >= need) {
      if (cap != cudaStreamCaptureStatusNone) ws.captured = true;
      a.split_first = tp.split_first;
      a.tail_ctas = tp.ctas;
      a.tail_units = tp.units;
      a.ws_o = static_cast<float*>(ws.ptr);
      a.ws_ml = a.ws_o + static_cast<size_t>(2 * tp.ctas) * rows * kAttnD;
      grid = dim3(static_cast<unsigned>(tp.split_first), 1, 1);
    }
  }
  st = dtype == kBF16 ? launch_attention<true>(grid, a.tail_ctas, mq, mk, mv, a, s, device)
                      : launch_attention<false>(grid, a.tail_ctas, mq, mk, mv, a, s, device);
  if (st != SF_OK) return st;
  SF_CUDA_TRY(cudaGetLastError());
  if (a.split_first >= 0) {
    const unsigned n_merge = static_cast<unsigned>(a.tail_units);
    if (dtype == kBF16)
      attention_merge_kernel<true, AttnCfg::ROWS><<<n_merge, AttnCfg::ROWS, 0, s>>>(a);
    else
      attention_merge_kernel<false, AttnCfg::ROWS><<<n_merge, AttnCfg::ROWS, 0, s>>>(a);
    SF_CUDA_TRY(cudaGetLastError());
  }
  return SF_OK;
}

}  // namespace

void attention_release_stream(void* stream) {
  std::lock_guard<std::mutex> lk(g_attn_ws_mu);
  for (auto it = g_attn_ws.begin(); it != g_attn_ws.end();) {
    if (it->first.stream == stream) {
      attn_ws_drop(it->second);
      it = g_attn_ws.erase(it);
    } else {
      ++it;
    }
  }
}

}  // namespace sf

using namespace sf;

// Number of kernel launches of sf_attention_fwd (part_mode 0, no skipped
// keys: skip_lo = skip_hi = kv_len) or sf_attention_fwd_partial for these
// sizes on the current device: 1; or, when the last wave runs as a stream-K
// tail, the tail kernel, the whole units' kernel and the merge kernel (3; 2
// when every unit is in the tail).
extern "C" int32_t sf_attention_launch_count(int32_t batch, int32_t heads, int32_t q_len,
                                             int32_t kv_len, int32_t skip_lo, int32_t skip_hi,
                                             int32_t* count) {
  if (!count) return fail(SF_ERR_INVALID_ARGUMENT, "null count");
  *count = 0;
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0) return SF_OK;
  if (skip_lo < 0 || skip_hi < skip_lo || skip_hi > kv_len)
    return fail(SF_ERR_INVALID_ARGUMENT, "skipped keys [%d, %d) outside [0, %d]", skip_lo, skip_hi, kv_len);
  DeviceInfo* dev = nullptr;
  int32_t st = current_device_info(&dev, nullptr);
  if (st != SF_OK) return st;
  int na = 0, ne = 0;
  attn_key_blocks(kv_len, skip_lo, skip_hi, &na, &ne);
  const int64_t units = ceil_div(q_len, AttnCfg::ROWS) * heads * batch;
  const AttnTail tp = attn_tail_plan(units, AttnCfg::MIN_BLOCKS * dev->sm_count, ne);
  *count = tp.split_first < 0 ? 1 : (tp.split_first > 0 ? 3 : 2);
  return SF_OK;
}

extern "C" int32_t sf_attention_fwd(int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                                    int32_t head_dim, const void* q, int64_t ldq,
                                    int64_t q_bstride, const void* k, int64_t ldk,
                                    int64_t k_bstride, const void* v, int64_t ldv,
                                    int64_t v_bstride, void* o, int64_t ldo, int64_t o_bstride,
                                    float scale, int32_t dtype, void* stream) {
  return attention_impl(batch, heads, q_len, kv_len, head_dim, q, ldq, q_bstride, k, ldk,
                        k_bstride, v, ldv, v_bstride, o, ldo, o_bstride, scale, dtype, kv_len,
                        kv_len, nullptr, nullptr, 0, stream);
}

extern "C" int32_t sf_attention_fwd_partial(int32_t batch, int32_t heads, int32_t q_len,
                                            int32_t kv_len, int32_t head_dim, const void* q,
                                            int64_t ldq, int64_t q_bstride, const void* k,
                                            int64_t ldk, int64_t k_bstride, const void* v,
                                            int64_t ldv, int64_t v_bstride, void* o, int64_t ldo,
                                            int64_t o_bstride, float scale, int32_t dtype,
                                            int32_t skip_lo, int32_t skip_hi, float* part_o,
                                            float* part_ml, int32_t part_mode, void* stream) {
  if (part_mode < 0 || part_mode > 2)
    return fail(SF_ERR_INVALID_ARGUMENT, "partial mode %d", part_mode);
  if (skip_lo < 0 || skip_hi < skip_lo || skip_hi > kv_len)
    return fail(SF_ERR_INVALID_ARGUMENT, "skipped keys [%d, %d) outside [0, %d]", skip_lo, skip_hi, kv_len);
  if (part_mode != 0 && (!part_o || !part_ml || !aligned16(part_o) || (reinterpret_cast<uintptr_t>(part_ml) & 7u)))
    return fail(SF_ERR_INVALID_ARGUMENT, "partial buffers missing or misaligned");
  if (part_mode != 2 && skip_hi - skip_lo == kv_len && kv_len > 0)
    return fail(SF_ERR_INVALID_ARGUMENT, "every key skipped");
  return attention_impl(batch, heads, q_len, kv_len, head_dim, q, ldq, q_bstride, k, ldk,
                        k_bstride, v, ldv, v_bstride, o, ldo, o_bstride, scale, dtype, skip_lo,
                        skip_hi, part_o, part_ml, part_mode, stream);
}
