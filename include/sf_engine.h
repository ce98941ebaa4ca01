/*
 * sf_engine.h -- C ABI of the B200 (sm_100a) matmul engine for Scaffolding.
 *
 * Replaces the hot-path part of the reference's C ABI
 * (_cuda_ops_decl.h, consumed by _cuda_ops.pyx) -- the cuBLAS SGEMM wrappers,
 * the bias-add, activation, scale and softmax launchers -- plus the runtime
 * services _cuda_ops.pyx implements in Cython around them (device
 * management, caching allocator, streams, events, peer access).  Citations
 * are file:line in the reference project (pictofeed/scaffolding).
 *
 * Conventions (all entry points):
 *   - Plain C types only; every function returns int32_t status
 *     (SF_OK == 0, negative = error).  sf_last_error() returns a
 *     thread-local description of the last failure on the calling thread.
 *   - Matrices are ROW-MAJOR, as in the reference's Python API; leading
 *     dimensions and batch strides are in ELEMENTS (int64_t).
 *   - Every launch takes an explicit stream (NULL = legacy default stream);
 *     nothing launches on a hidden stream (the reference's bias add always
 *     used the NULL stream, _cuda_ops.pyx:1298-1299).
 *   - Launches run on the CURRENT device; the engine never changes it.
 *   - The engine never allocates or frees caller tensors.  Paths that need
 *     scratch memory take a caller-owned workspace sized by
 *     sf_gemm_workspace_size().
 */
#ifndef SF_ENGINE_H_
#define SF_ENGINE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ───────────────────────────── status codes ───────────────────────────── */
#define SF_OK 0
#define SF_ERR_INVALID_ARGUMENT (-1)
#define SF_ERR_UNSUPPORTED (-2)
#define SF_ERR_CUDA (-3)
#define SF_ERR_OUT_OF_MEMORY (-4)
#define SF_ERR_WORKSPACE (-5)
#define SF_ERR_DEVICE_TIMEOUT (-6)
#define SF_ERR_NCCL (-7)

/* ───────────────────────────── enums ───────────────────────────── */
/* Storage types.  The reference treats every buffer as float*
 * (_cuda_ops.pyx:1095-1102) and cannot store bf16 at all (dtype.py:31). */
#define SF_DTYPE_F32 0
#define SF_DTYPE_F16 1
#define SF_DTYPE_BF16 2

/* Epilogue activations: SiLU (_cuda_kernels.cu:384, nn/functional.py:57-59),
 * GELU-tanh (_cuda_kernels.cu:428, nn/functional.py:79-82). */
#define SF_ACT_NONE 0
#define SF_ACT_SILU 1
#define SF_ACT_GELU_TANH 2

/* fp32 GEMM arithmetic.  ACCURATE (default) = 3xTF32 on tcgen05, the
 * replacement for non-TF32 cuBLAS SGEMM; FFMA = IEEE fp32 SIMT;
 * TF32 = single-pass TF32 (what backends.cuda.matmul.allow_tf32 = True
 * permits, backends/cuda.py:20-35 -> _cuda_kernels.cu:1928-1936). */
#define SF_FP32_ACCURATE 0
#define SF_FP32_FFMA 1
#define SF_FP32_TF32 2

/* Kernel selection override (tuning / tests only; AUTO in production). */
#define SF_KERNEL_AUTO 0
#define SF_KERNEL_TCGEN05 1      /* tensor-core kernels only (no GEMV) */
#define SF_KERNEL_SIMT 2
#define SF_KERNEL_TCGEN05_1CTA 3 /* tensor-core kernels without CTA pairs */

/* Fused epilogue:  D = act(alpha * (op(A) . op(B)) + bias) + beta * R.
 * Replaces the separate bias-add (cuda_bias_add_row_f32,
 * _cuda_kernels.cu:1490-1527), activation and scalar-mul launches. */
typedef struct sf_epilogue {
  float alpha;          /* 1.0 for a plain product */
  float beta;           /* residual weight; ignored when residual == NULL */
  const void* bias;     /* [N] or NULL */
  int32_t bias_dtype;   /* SF_DTYPE_* */
  int32_t activation;   /* SF_ACT_* */
  const void* residual; /* same shape as D, or NULL */
  int32_t residual_dtype;
  int32_t reserved;
  int64_t ldr;          /* residual leading dimension (elements) */
  int64_t r_stride0;    /* residual batch strides (batched calls) */
  int64_t r_stride1;
} sf_epilogue;

/* Two-level batch for strided-batched products, e.g. (heads, batch) of
 * attention.  Batch index z = b1 * count0 + b0; operand X of batch (b0, b1)
 * starts at X + b0 * x_stride0 + b1 * x_stride1 (elements). */
typedef struct sf_batch {
  int64_t count0, count1;
  int64_t a_stride0, a_stride1;
  int64_t b_stride0, b_stride1;
  int64_t c_stride0, c_stride1;
} sf_batch;

/* ───────────────────────────── GEMM ───────────────────────────── */

/* C[M,N] = epilogue( op(A)[M,K] . op(B)[K,N] ), row-major.
 *   trans_a = 0: A stored [M,K] (lda >= K);  1: A stored [K,M] (lda >= M)
 *   trans_b = 0: B stored [K,N] (ldb >= N);  1: B stored [N,K] (ldb >= K),
 *                the nn.Linear weight layout.
 * in_dtype applies to A and B; out_dtype to C.  fp32 inputs use the
 * arithmetic chosen by sf_set_fp32_mode().  workspace may be NULL when
 * sf_gemm_workspace_size() returns 0 for the same arguments.
 *
 * Replaces cuda_sgemm(handle, M, N, K, A, B, C, alpha, beta, transA, transB)
 * (_cuda_ops_decl.h:107-111, _cuda_kernels.cu:1175-1220) together with the
 * bias add that followed it in dev_linear_forward (_cuda_ops.pyx:1278-1302).
 */
int32_t sf_gemm(int64_t M, int64_t N, int64_t K,
                const void* A, int64_t lda, int32_t trans_a,
                const void* B, int64_t ldb, int32_t trans_b,
                void* C, int64_t ldc,
                int32_t in_dtype, int32_t out_dtype,
                const sf_epilogue* epi,
                void* workspace, size_t workspace_bytes,
                void* stream);

/* Strided-batched C[z] = epilogue( op(A[z]) . op(B[z]) ) over a two-level
 * batch.  Replaces cuda_sgemm_batched (_cuda_ops_decl.h:112-116,
 * _cuda_kernels.cu:1223-1243; NN only there) and the host loop of
 * per-batch cuda_sgemm calls behind dev_batched_matmul_nt
 * (_cuda_ops.pyx:1152-1190): one launch, NN and NT. */
int32_t sf_gemm_batched(const sf_batch* batch,
                        int64_t M, int64_t N, int64_t K,
                        const void* A, int64_t lda, int32_t trans_a,
                        const void* B, int64_t ldb, int32_t trans_b,
                        void* C, int64_t ldc,
                        int32_t in_dtype, int32_t out_dtype,
                        const sf_epilogue* epi,
                        void* workspace, size_t workspace_bytes,
                        void* stream);

/* Bytes of workspace sf_gemm / sf_gemm_batched need for these arguments
 * (batch == NULL for sf_gemm).  New; the reference had no workspace. */
int32_t sf_gemm_workspace_size(const sf_batch* batch, int64_t M, int64_t N, int64_t K,
                               int32_t trans_a, int32_t trans_b,
                               int32_t in_dtype, int32_t out_dtype, size_t* bytes);

/* y[M,N] = act(x[M,K] . W[N,K]^T + bias) for M <= 256 with bf16/fp16 x and W,
 * WITHOUT allocating: for callers that own all device memory themselves or
 * must not call cudaMalloc, and so cannot pass sf_gemm a workspace.  The
 * split-K partial sums live in a 4 MiB array compiled into the library
 * (M * N <= 1048576, larger sizes are rejected); calls on one device share
 * it, so calls that overlap on the GPU race.  The first call on a device
 * looks the array up (make it before any stream capture).  No counterpart
 * in the reference. */
int32_t sf_linear_skinny_noalloc(int64_t M, int64_t N, int64_t K,
                                 const void* x, int64_t ldx, const void* W, int64_t ldw,
                                 const void* bias, int32_t bias_dtype,
                                 void* y, int64_t ldy, int32_t in_dtype, int32_t out_dtype,
                                 int32_t activation, void* stream);

/* fp32 arithmetic mode (per process).  Replaces cuda_set_tf32
 * (_cuda_ops_decl.h:153, _cuda_kernels.cu:1928-1936). */
int32_t sf_set_fp32_mode(int32_t mode);
int32_t sf_get_fp32_mode(int32_t* mode);
/* Kernel override for tests/tuning (SF_KERNEL_*); AUTO by default. */
int32_t sf_set_kernel_override(int32_t kernel);

/* ───────────────────────────── row-wise ops ───────────────────────────── */

/* y[r,:] = softmax(scale * x[r,:]) for r < rows, fp32 arithmetic.
 * Replaces cuda_softmax_f32 (_cuda_ops_decl.h:83-84, _cuda_kernels.cu:604-640)
 * preceded by cuda_muls_f32 (_cuda_kernels.cu:237-277) in SDPA
 * (nn/functional.py:314-316). */
int32_t sf_softmax_rows(const void* x, int32_t x_dtype, int64_t ldx,
                        void* y, int32_t y_dtype, int64_t ldy,
                        int64_t rows, int64_t cols, float scale, void* stream);

/* Fused attention forward, head_dim 64, 16-bit Q/K/V/O (fp32 softmax):
 *   O[b, :, h] = softmax(scale * Q[b, :, h] K[b, :, h]^T) V[b, :, h]
 * Head h of batch b, row r of Q lives at q + b*q_bstride + r*ldq + h*64
 * (elements; likewise K, V, O), so the Q/K/V column blocks of a fused
 * [tokens, 3*C] projection are read in place.  Replaces the batched
 * matmul -> muls -> softmax -> batched matmul chain of
 * scaled_dot_product_attention (nn/functional.py:310-321, built from
 * _cuda_ops.pyx:1152-1190, :990-998, :1016-1034, :1122-1149) and the DiT
 * attention einsum (diffusion/models.py:529-536).  Pointers and strides
 * 16-byte aligned; kv_len >= 1. */
int32_t sf_attention_fwd(int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                         int32_t head_dim, const void* q, int64_t ldq, int64_t q_bstride,
                         const void* k, int64_t ldk, int64_t k_bstride, const void* v,
                         int64_t ldv, int64_t v_bstride, void* o, int64_t ldo, int64_t o_bstride,
                         float scale, int32_t dtype, void* stream);

/* sf_attention_fwd over part of the keys, for overlapping a key exchange
 * with attention (the token-sharded DiT stack: attention over a rank's own
 * keys while the other ranks' keys are gathered, then over the gathered
 * ones).  Keys [skip_lo, skip_hi) are left out (skip_lo = skip_hi = kv_len:
 * none).  part_mode 1 writes this pass's unnormalised fp32 output to part_o
 * ([batch][q_len][heads][64]) and each row's (integer exponent base, sum) to
 * part_ml ([batch][q_len][heads][2]) instead of o; part_mode 2 merges such
 * a partial result with this pass and writes the normalised o; part_mode 0
 * is sf_attention_fwd with the skip.  The split result equals the one-pass
 * result up to fp32 summation order (the merge scales by exact powers of
 * two).  Same DiT attention the entry above replaces
 * (diffusion/models.py:529-536; nn/parallel.py:45-290 is the reference's
 * multi-GPU wrapper, which gathers on the host instead). */
int32_t sf_attention_fwd_partial(int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                                 int32_t head_dim, const void* q, int64_t ldq,
                                 int64_t q_bstride, const void* k, int64_t ldk,
                                 int64_t k_bstride, const void* v, int64_t ldv,
                                 int64_t v_bstride, void* o, int64_t ldo, int64_t o_bstride,
                                 float scale, int32_t dtype, int32_t skip_lo, int32_t skip_hi,
                                 float* part_o, float* part_ml, int32_t part_mode, void* stream);

/* Kernel launches one sf_attention_fwd or sf_attention_fwd_partial call of
 * these sizes makes on the current device (keys [skip_lo, skip_hi) skipped;
 * skip_lo = skip_hi = kv_len for sf_attention_fwd): 1; or, when the last,
 * partial wave of query blocks runs as a stream-K tail (its key blocks shared
 * evenly by all CTA slots), 3 = the whole units' kernel, the tail kernel and
 * a merge kernel that combines the split units (2 when every unit is in the
 * tail); 0 for empty sizes.  Lets callers count their launches (no reference counterpart:
 * the reference's attention chain, nn/functional.py:310-321, launches a fixed
 * sequence). */
int32_t sf_attention_launch_count(int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                                  int32_t skip_lo, int32_t skip_hi, int32_t* count);

/* LayerNorm over the last dimension with an optional per-group adaptive
 * scale / shift (adaLN), for row r < rows, column c < cols:
 *   h = (x[r,c] - mean_r) / sqrt(var_r + eps) * gamma[c] + beta[c]
 *   y[r,c] = mod ? h * (1 + mod[g, c]) + mod[g, cols + c] : h,   g = r / group_rows
 * (population variance, fp32 arithmetic; gamma / beta fp32 [cols] or NULL;
 * mod [groups][ld_mod >= 2 * cols] in mod_dtype, e.g. the output of a DiT
 * block's modulation linear, one row per sample of group_rows tokens).
 * Replaces cuda_layer_norm_f32 (_cuda_ops_decl.h, _cuda_kernels.cu:1070-1093,
 * behind nn/layers.py:470-493) and the host modulation of AdaLayerNorm
 * (diffusion/models.py:478-487), as one bandwidth kernel before the QKV and
 * FFN-up GEMMs. */
int32_t sf_layernorm_modulate(int64_t rows, int64_t cols, const void* x, int32_t x_dtype,
                              int64_t ldx, const float* gamma, const float* beta, float eps,
                              const void* mod, int32_t mod_dtype, int64_t ld_mod,
                              int64_t group_rows, void* y, int32_t y_dtype, int64_t ldy,
                              void* stream);

/* y[i] = act(alpha * x[i]).  Replaces cuda_silu_f32 / cuda_gelu_f32 /
 * cuda_muls_f32 (_cuda_ops_decl.h:69, :74, :63; _cuda_kernels.cu:384, :428,
 * :237-277) for the standalone dev_silu / dev_gelu / dev_muls calls. */
int32_t sf_unary(const void* x, int32_t x_dtype, void* y, int32_t y_dtype,
                 int64_t n, float alpha, int32_t activation, void* stream);

/* ───────────────────────────── runtime ───────────────────────────── */
/* Replaces the device-management block of _cuda_ops.pyx:491-548. */
int32_t sf_device_count(int32_t* count);
int32_t sf_set_device(int32_t device);
int32_t sf_get_device(int32_t* device);
int32_t sf_device_synchronize(void);

typedef struct sf_device_props {
  char name[256];
  uint64_t total_memory;
  int32_t major, minor;
  int32_t multi_processor_count;
  int32_t max_threads_per_block;
  int32_t max_threads_per_mp;
  int32_t warp_size;
  uint64_t shared_mem_per_block;
  uint64_t shared_mem_per_block_optin;
  uint64_t l2_cache_size;
  int32_t clock_rate_khz;
  int32_t memory_clock_rate_khz;
  int32_t memory_bus_width;
  int32_t reserved;
} sf_device_props;
int32_t sf_device_properties(int32_t device, sf_device_props* out);
int32_t sf_mem_info(size_t* free_bytes, size_t* total_bytes);

/* Caching allocator: exact-size per-device free lists, 256-byte rounding,
 * per-device pool cap -- the policy of _make_buffer / _cache_pop /
 * _cache_return / empty_cache (_cuda_ops.pyx:356-475).  sf_malloc returns
 * memory on `device`, restoring the current device afterwards.  sf_free
 * must be given the size sf_malloc was asked for. */
int32_t sf_malloc(int32_t device, size_t bytes, void** ptr);
int32_t sf_free(int32_t device, void* ptr, size_t bytes);
int32_t sf_empty_cache(int32_t device); /* device < 0: all devices */
int32_t sf_pool_stats(int32_t device, size_t* cached_bytes, size_t* allocated_bytes);
int32_t sf_set_pool_cap(size_t bytes_per_device);
int32_t sf_host_alloc_pinned(size_t bytes, void** ptr);
int32_t sf_host_free_pinned(void* ptr);

/* Copies: kind 0 = host->device, 1 = device->host, 2 = device->device,
 * 3 = default (UVA-inferred).  Asynchronous on `stream`.  Replaces
 * gpu_memcpy_h2d / d2h / d2d (_cuda_ops.pyx:749-771). */
int32_t sf_memcpy(void* dst, const void* src, size_t bytes, int32_t kind, void* stream);
/* Cross-device copy.  Replaces the D2D copy in gputensor_to_device
 * (_cuda_ops.pyx:861-875) without its 4-byte element assumption. */
int32_t sf_memcpy_peer(void* dst, int32_t dst_device, const void* src, int32_t src_device,
                       size_t bytes, void* stream);
int32_t sf_memset(void* dst, int32_t value, size_t bytes, void* stream);

/* Streams and events (_cuda_ops.pyx:608-673). */
int32_t sf_stream_create(int32_t device, int32_t non_blocking, void** stream);
/* A stream whose kernels the scheduler prefers (high_priority != 0) or the
 * default priority: a collective issued on it gets SMs while a long kernel on
 * another stream is still filling the GPU (no counterpart in the reference,
 * whose streams are all default priority, _cuda_ops.pyx:608-640). */
int32_t sf_stream_create_priority(int32_t device, int32_t non_blocking, int32_t high_priority,
                                  void** stream);
int32_t sf_stream_destroy(void* stream);
int32_t sf_stream_synchronize(void* stream);
int32_t sf_stream_wait_event(void* stream, void* event);
int32_t sf_event_create(int32_t enable_timing, void** event);
int32_t sf_event_destroy(void* event);
int32_t sf_event_record(void* event, void* stream);
int32_t sf_event_synchronize(void* event);
int32_t sf_event_elapsed_ms(void* start, void* end, float* ms);

/* CUDA graphs: capture the launches issued on `stream` between begin and end
 * (relaxed capture mode) into an executable graph, then replay it.  For
 * launch-bound sequences such as skinny-M GEMMs.  New (the reference has no
 * graph support).  Workspaces must already be sized before capture. */
int32_t sf_graph_begin(void* stream);
int32_t sf_graph_end(void* stream, void** exec);
int32_t sf_graph_launch(void* exec, void* stream);
int32_t sf_graph_destroy(void* exec);

/* Peer access (_cuda_ops.pyx:550-587). */
int32_t sf_can_access_peer(int32_t device, int32_t peer, int32_t* can);
int32_t sf_enable_peer_access_all(void);

/* Device-side error word of `device`: kernels whose bounded waits expire
 * record a nonzero code here instead of hanging (no counterpart in the
 * reference, whose CUDA_CHECK only saw launch errors,
 * _cuda_kernels.cuh:303-319).  clear != 0 resets it to zero. */
int32_t sf_device_error_status(int32_t device, int32_t* code, int32_t clear);

/* Launches a kernel that waits, with limit `limit_ns`, on a barrier nothing
 * arrives on, and returns the device-side code it recorded (6 when the
 * bounded wait expired as designed).  Exercises the timeout path of the
 * engine's waits without faulting or hanging the GPU.  New (no counterpart
 * in the reference). */
int32_t sf_selftest_bounded_wait(int64_t limit_ns, int32_t* device_code, void* stream);

/* x[i] = mean + std * N(0,1) sample, i < n, from a counter-based generator
 * keyed by (seed, i): the same seed gives the same values on every device.
 * Synthetic weight/activation initialisation for benchmarks and tests (the
 * reference draws its inits on the host, nn/layers.py:66-74). */
int32_t sf_fill_normal(void* x, int32_t dtype, int64_t n, uint64_t seed, float mean, float std,
                       void* stream);

const char* sf_last_error(void);
const char* sf_version(void);

/* ───────────────────────────── collectives ───────────────────────────── */
/* New: the reference has no collective library (distributed/__init__.py
 * is a no-op stub; DataParallel gathers through host NumPy,
 * nn/parallel.py:229-267).  One communicator per process/GPU over NCCL
 * (NVLink/NVSwitch); NCCL is loaded at run time. */
int32_t sf_comm_unique_id(uint8_t id_out[128]);
int32_t sf_comm_init(void** comm, int32_t nranks, int32_t rank, const uint8_t id[128]);
/* Sub-communicator of the ranks passing the same `color`, ordered by `key`
 * (e.g. the ranks holding tokens of one sample, which exchange K/V). */
int32_t sf_comm_split(void* comm, int32_t color, int32_t key, void** out);
/* recv[r * bytes_per_rank ...] = send of rank r, for every rank r. */
int32_t sf_comm_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank,
                          void* stream);
/* In-place max / sum of `count` fp32 values across ranks (timing, checks). */
int32_t sf_comm_allreduce_f32(void* comm, float* buf, size_t count, int32_t op_max,
                              void* stream);
int32_t sf_comm_async_error(void* comm, int32_t* nccl_result);
int32_t sf_comm_abort(void* comm);
int32_t sf_comm_destroy(void* comm);

/* ──────────────────── peer buffers and flags (one node) ──────────────────── */
/* New (no counterpart in the reference, whose DataParallel moves rows
 * through the host, nn/parallel.py:111-147, :229-267).  Lets the ranks of a
 * node exchange device data with copy-engine copies (cudaMemcpyAsync into a
 * peer's buffer, no SMs used) and order them with sequence flags.
 *
 * sf_ipc_alloc: a zeroed device buffer of its own allocation on the current
 * device, shareable with sf_ipc_handle (64-byte handle, sent to the peers
 * over any channel) and mapped in a peer process with sf_ipc_open (peer
 * access enabled on demand); sf_ipc_close unmaps, sf_ipc_free frees (after
 * every peer has closed its mapping).
 *
 * sf_flag_store: after the stream's earlier work, stores `value` to each of
 * `count` (<= 8) int32 flags (local or peer-mapped; release, system scope).
 * sf_flag_wait: the stream's later work starts once flags[i * stride] >=
 * value for every i < count except i == skip (-1: none), read with acquire
 * loads.  The wait is bounded (timeout_ns, 0 = 2 s): when it expires the
 * device error word (sf_device_error_status) reads 7 and the stream goes on.
 * A wait must only depend on stores issued by other GPUs' streams, never on
 * later work of its own GPU. */
#define SF_IPC_HANDLE_BYTES 64
int32_t sf_ipc_alloc(size_t bytes, void** ptr);
int32_t sf_ipc_free(void* ptr);
int32_t sf_ipc_handle(void* ptr, uint8_t handle[SF_IPC_HANDLE_BYTES]);
int32_t sf_ipc_open(const uint8_t handle[SF_IPC_HANDLE_BYTES], void** ptr);
int32_t sf_ipc_close(void* ptr);
int32_t sf_flag_store(int32_t* const* flags, int32_t count, int32_t value, void* stream);
int32_t sf_flag_wait(const int32_t* flags, int32_t count, int32_t stride, int32_t skip,
                     int32_t value, int64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SF_ENGINE_H_ */
