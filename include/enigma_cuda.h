/* enigma_cuda.h — C ABI of libenigma_cuda.so, the B200 (sm_100a) backend of the
 * Enigma runtime.
 *
 * This library takes the place of the Swift/Metal runtime dylib
 * (enigma/runtime_dispatch/swift/libenigma_runtime.swift in the reference),
 * which Python binds with ctypes (enigma/runtime_dispatch/runtime.py:259-316).
 * Plain pointers and sizes only: device pointers are `void*` from
 * enigma_alloc (or any CUDA allocation), streams are `void*` holding a
 * cudaStream_t (NULL = the legacy default stream).
 *
 * Every function returns an int32 status:
 *    0  ENIGMA_OK
 *   -1  ENIGMA_ERR_LAUNCH   launch failed (the Swift runtime's "encoder" error)
 *   -2  ENIGMA_ERR_EXEC     execution error reported by the GPU
 *   -3  ENIGMA_ERR_TIMEOUT  a bounded device-side wait gave up
 *   -4  ENIGMA_ERR_BADARG   shape / pointer / alignment rejected before launch
 *   -5  ENIGMA_ERR_DEVICE   no usable sm_100 device
 * The message of the last failure on the calling thread is returned by
 * enigma_last_error.  -1 and -2 keep the Swift runtime's meaning
 * (libenigma_runtime.swift:146-175).
 */
#ifndef ENIGMA_CUDA_H
#define ENIGMA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ENIGMA_OK 0
#define ENIGMA_ERR_LAUNCH (-1)
#define ENIGMA_ERR_EXEC (-2)
#define ENIGMA_ERR_TIMEOUT (-3)
#define ENIGMA_ERR_BADARG (-4)
#define ENIGMA_ERR_DEVICE (-5)

/* Element types (storage); accumulation is always fp32. */
#define ENIGMA_DTYPE_F32 0
#define ENIGMA_DTYPE_BF16 1

/* Kernel ids for enigma_dispatch (the recognizer in enigma/compiler maps a
 * traced @enigma.kernel to one of these). */
#define ENIGMA_KERNEL_RMSNORM 1   /* bufs: x, w, y            ip: rows, hidden, dtype   fp: eps */
#define ENIGMA_KERNEL_GEMM 2      /* bufs: A, B, C            ip: M, N, K, dtype, accumulate */
#define ENIGMA_KERNEL_SDPA 3      /* bufs: Q, K, V, O         ip: B, Hq, Hkv, Sq, Skv, D, causal, dtype  fp: scale */

/* ---- device / queue: replaces enigma_create_device, enigma_create_queue
 *      (libenigma_runtime.swift:10, :19) ---- */
int32_t enigma_init(int32_t device);
int32_t enigma_device_count(int32_t* count);
int32_t enigma_stream_create(void** stream);
int32_t enigma_stream_destroy(void* stream);
int32_t enigma_synchronize(void* stream);
int32_t enigma_last_error(char* buf, size_t len);
/* Name of the device kernel the last operator call on this thread chose (e.g.
 * "gemm_bf16_pair_kernel", "sdpa_fwd_tc_kernel"); "" before any call.  No
 * counterpart in the reference, whose Swift runtime runs one named pipeline per
 * dispatch (libenigma_runtime.swift:132-214): here one operator picks between
 * tensor-core and CUDA-core kernels by shape and alignment. */
int32_t enigma_last_kernel(char* buf, size_t len);

/* ---- capability queries: replace enigma_device_name,
 *      enigma_device_max_threadgroup_memory,
 *      enigma_device_max_threads_per_threadgroup, enigma_device_supports_family
 *      (libenigma_runtime.swift:223-260) ---- */
int32_t enigma_device_name(int32_t device, char* buf, size_t len);
int32_t enigma_device_attrs(int32_t device, int64_t* sm_count, int64_t* max_smem_per_block,
                            int64_t* max_threads_per_block, int64_t* total_mem_bytes,
                            int32_t* cc_major, int32_t* cc_minor);

/* ---- buffers: replace enigma_create_buffer, enigma_create_buffer_empty,
 *      enigma_buffer_contents, enigma_release (libenigma_runtime.swift:91-124, :216).
 *      Device memory is not host-visible, so "contents" becomes explicit copies. ---- */
int32_t enigma_alloc(void** ptr, size_t bytes);
int32_t enigma_free(void* ptr);
int32_t enigma_host_alloc(void** ptr, size_t bytes); /* pinned host memory */
int32_t enigma_host_free(void* ptr);
int32_t enigma_upload(void* dst_dev, const void* src_host, size_t bytes, void* stream);
int32_t enigma_download(void* dst_host, const void* src_dev, size_t bytes, void* stream);
int32_t enigma_memset(void* dst_dev, int32_t value, size_t bytes, void* stream);

/* ---- the hot-path operators (asynchronous on `stream`) ---- */

/* y = x * rsqrt(mean(x^2) + eps) * w per row; x, y [rows, hidden] row-major, w [hidden].
 * Replaces the dispatch of rmsnorm_kernel (examples/benchmark_rmsnorm.py:31-84)
 * and of rmsnorm (examples/metal/rmsnorm_handwritten.metal:4-46). */
int32_t enigma_rmsnorm(int32_t dtype, const void* x, const void* w, void* y, int64_t rows,
                       int64_t hidden, float eps, void* stream);

/* C[M,N] = A[M,K] * B[K,N], all row-major bf16, fp32 accumulate, bf16 out.
 * Replaces the dispatch of gemm_async (examples/async_copy_gemm.py:32-79);
 * semantics of enigma.gemm (enigma/ops/gemm.py:51-167) with beta = 0. */
int32_t enigma_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                         void* stream);

/* O = softmax(scale * Q K^T [+ causal mask]) V per (batch, head); bf16 in and out,
 * Q/O [B, Hq, Sq, D], K/V [B, Hkv, Skv, D], GQA maps q-head h to kv-head h / (Hq/Hkv).
 * causal masks key j > query i + (Skv - Sq) (bottom-right aligned).
 * Replaces the dispatch of sdpa_enigma (examples/benchmark_sdpa.py:48-158),
 * fa_naive / fa_tv_kernel (examples/showcase_attention.py:31-125). */
int32_t enigma_sdpa_bf16(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                         int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                         int64_t head_dim, float scale, int32_t causal, void* stream);

/* C[i] = A[i] op B[i] for i < n; op 0 add, 1 sub, 2 mul, 3 max, 4 min; fp32 or bf16.
 * Replaces the dispatch of add_kernel (examples/vector_add_tv.py:13-55) and the
 * one-thread-per-element kernels of examples/vector_add.py.  Buffers 16-byte aligned
 * for the vector path (any alignment of the element size works, slower). */
int32_t enigma_elementwise(int32_t op, int32_t dtype, const void* A, const void* B, void* C,
                           int64_t n, void* stream);

/* fp32 reference-shape variants on CUDA cores (exact fp32 FMA accumulation):
 * C[M,N] (+)= A[M,K] * B[K,N] — replaces matmul_k4 / gemm_k4
 * (tests/metal/test_gemm_matmul_runtime.py:20-60); `accumulate` != 0 adds into C. */
int32_t enigma_gemm_f32(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                        int32_t accumulate, void* stream);
/* The same with either operand transposed: A is [K, M] when trans_a, B is [N, K] when
 * trans_b — replaces the tile op enigma.gemm(A_s, B_s, C, M, N, K, transpose_A,
 * transpose_B) (enigma/ops/gemm.py:51-167; C += A @ B, C starting from the zero-filled
 * register tile, tests/metal/test_new_features_runtime.py:25-56). */
int32_t enigma_gemm_f32_trans(const void* A, const void* B, void* C, int64_t M, int64_t N,
                              int64_t K, int32_t trans_a, int32_t trans_b, int32_t accumulate,
                              void* stream);
/* fp32 attention, same layout and masking as enigma_sdpa_bf16 (showcase_attention.py:31-125,
 * benchmark_sdpa.py:48-150 with the KV de-interleaved). */
int32_t enigma_sdpa_f32(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                        int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                        int64_t head_dim, float scale, int32_t causal, void* stream);

/* Attention over strided views (CUDA cores, any head_dim <= 256): strides12 holds the
 * element strides (batch, head, sequence) of Q, K, V and O in that order; head_dim is
 * contiguous.  Lets reference layouts run without copies, e.g. the token-major Q/O
 * [tokens, heads, D] and the interleaved [kv_head, token, K|V] buffer of
 * examples/benchmark_sdpa.py:188-194. */
int32_t enigma_sdpa_strided(int32_t dtype, const void* Q, const void* K, const void* V, void* O,
                            int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q,
                            int64_t seq_kv, int64_t head_dim, const int64_t* strides12,
                            float scale, int32_t causal, void* stream);
/* As enigma_sdpa_strided with an attention sink per query head (gpt-oss): sinks[h] is a
 * logit in the same units as scale * q.k that joins the softmax denominator only, i.e.
 * O = sum_j e^(s_j - M) v_j / (e^(sinks[h] - M) + sum_j e^(s_j - M)).  Replaces the
 * sink / running-max buffer `s` of examples/metal/sdpa_handwritten.metal:16-42 (m starts at
 * s[h], l at 1) and of sdpa_enigma (examples/benchmark_sdpa.py:64-72).  sinks may be NULL. */
int32_t enigma_sdpa_strided_sinks(int32_t dtype, const void* Q, const void* K, const void* V,
                                  void* O, int64_t batch, int64_t heads_q, int64_t heads_kv,
                                  int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                                  const int64_t* strides12, float scale, int32_t causal,
                                  const float* sinks, void* stream);

/* ---- RMSNorm of host-resident rows (the reference's execute() path: host arrays in, host
 *      bytes out, runtime.py:318-421, for the RMSNorm of examples/benchmark_rmsnorm.py) ----
 * x_host [rows, hidden] -> y_host, w_host [hidden]; dtype ENIGMA_DTYPE_F32 or _BF16.  Rows go
 * through the GPU in chunks of chunk_rows on two streams (the caller's and a library-owned
 * one): chunk c's upload, kernel and download run in order on stream c % 2, so uploads,
 * kernels and downloads of neighbouring chunks overlap (host<->device copies are full
 * duplex).  x_host / y_host should be page-locked (enigma_host_alloc) for the copies to
 * overlap.  workspace: device memory of enigma_rmsnorm_host_workspace_bytes() bytes, 256-byte
 * aligned (w and two chunk buffers each way).  Synchronous: returns when y_host is written. */
int32_t enigma_rmsnorm_host_workspace_bytes(int32_t dtype, int64_t hidden, int64_t chunk_rows,
                                            size_t* bytes);
int32_t enigma_rmsnorm_host(int32_t dtype, const void* x_host, const void* w_host, void* y_host,
                            int64_t rows, int64_t hidden, float eps, void* workspace,
                            size_t workspace_bytes, int64_t chunk_rows, void* stream);

/* ---- one decoder-layer decode step (Qwen-style; the reference's qwen_fused megakernel,
 *      examples/qwen_megakernel.py:228-269, at BASELINE config 5 shapes) ----
 * x, out: [batch, hidden] bf16.  Weights bf16, row-major [in, out]:
 *   w_qkv [hidden, (heads_q + 2 heads_kv) * head_dim]   (q heads | k heads | v heads)
 *   w_o [heads_q * head_dim, hidden], w_gate_up [hidden, 2 * intermediate] (gate | up),
 *   w_down [intermediate, hidden]; w_in_norm / w_post_norm [hidden].
 * rope_cos / rope_sin: fp32 [head_dim] rotate-half tables for `position`.
 * k_cache / v_cache: bf16 [batch, heads_kv, cache_capacity, head_dim]; the step writes
 * the new token's k, v at `position` and attends over position + 1 keys.
 * head_dim must be 64; heads_q / heads_kv <= 8; hidden <= 2048; batch <= 128.
 * workspace: caller-owned device memory of enigma_decode_workspace_bytes() bytes. */
typedef struct enigma_decode_layer_desc {
  int64_t batch, hidden, heads_q, heads_kv, head_dim, intermediate, cache_capacity, position;
  float eps, attn_scale;
  const void *w_in_norm, *w_qkv, *w_o, *w_post_norm, *w_gate_up, *w_down;
  const float *rope_cos, *rope_sin;
  void *k_cache, *v_cache;
} enigma_decode_layer_desc;
int32_t enigma_decode_workspace_bytes(const enigma_decode_layer_desc* desc, size_t* bytes);
int32_t enigma_decode_layer_bf16(const enigma_decode_layer_desc* desc, const void* x, void* out,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* The reference's own fp32 single-token layer (qwen_fused, examples/qwen_megakernel.py:
 * 228-269) with its buffer set: weights row-major [out, in] (y = W x); caches
 * [heads_kv, cache_total, head_dim] already holding the new token's k / v (as the
 * reference's host prepares them); norm_buf .. k_rope_buf are the reference's scratch
 * buffers and serve as the workspace.  fp32 throughout; head_dim even and <= 256. */
typedef struct enigma_qwen_decode_f32_desc {
  int64_t hidden, heads_q, heads_kv, head_dim, intermediate, cache_total;
  float eps, attn_scale;
  const float *x, *w_norm, *Wq, *Wk, *Wv, *w_q_norm, *w_k_norm, *cos_pos, *sin_pos;
  const float *k_cache, *v_cache, *Wo, *w_post, *Wg, *Wu, *Wd;
  float *norm_buf, *q_buf, *k_buf, *v_buf, *attn_buf, *mlp_buf, *post_buf, *q_rope_buf,
      *k_rope_buf, *out;
} enigma_qwen_decode_f32_desc;
int32_t enigma_qwen_decode_f32(const enigma_qwen_decode_f32_desc* desc, void* stream);

/* The same decode step without a caller-provided workspace, for callers that cannot
 * allocate device memory on this path: a serving loop that must never enter the
 * allocator, a plugin inside a host runtime that owns all device memory, code where an
 * allocation failure mid-step is not acceptable.  (No counterpart in the reference: its
 * Metal runtime always allocates buffers per call.)  The workspace is a fixed 16 MiB
 * device array inside this library, held on every GPU that loads it until the process
 * exits; a step that needs more (enigma_decode_workspace_bytes) is rejected with
 * ENIGMA_ERR_BADARG.  Its first call on a device looks up the array's device address once
 * (cudaGetSymbolAddress), so make that first call before any stream capture.  With lazy
 * module loading (CUDA's default) that first call is also when the driver loads this
 * library's device code on the device and commits the 16 MiB: it can fail for lack of
 * device memory, so make it during set-up.  Later calls allocate nothing.  A bounded wait
 * that runs out flags this entry's own static status word; enigma_synchronize and
 * enigma_take_device_status report it (ENIGMA_ERR_TIMEOUT) once and clear it.  All calls
 * share the array: calls that overlap on the GPU race, so serialize them on one stream. */
int32_t enigma_decode_layer_bf16_noalloc(const enigma_decode_layer_desc* desc, const void* x,
                                         void* out, void* stream);
/* Self-test of that reporting: the probe of enigma_check_timeout_path aimed at the
 * no-allocation entry's status word. */
int32_t enigma_decode_noalloc_check_timeout_path(int64_t polls, void* stream);

/* ---- generic dispatch by kernel id: replaces enigma_dispatch /
 *      enigma_dispatch_timed (libenigma_runtime.swift:132-214).
 *      grid / threads are Metal-style totals (threads per axis, not groups),
 *      accepted for interface parity and checked (no zero extent, at most 1024
 *      threads per threadgroup; NULL = not given); the kernels pick their own
 *      CTA shapes.
 *      dispatch_timed returns the device time of the launch in microseconds,
 *      measured with CUDA events on `stream`, and synchronizes. ---- */
int32_t enigma_dispatch(int32_t kernel_id, void* const* buffers, int32_t n_buffers,
                        const int64_t* iparams, int32_t n_iparams, const float* fparams,
                        int32_t n_fparams, const uint32_t* grid3, const uint32_t* threads3,
                        void* stream);
int32_t enigma_dispatch_timed(int32_t kernel_id, void* const* buffers, int32_t n_buffers,
                              const int64_t* iparams, int32_t n_iparams, const float* fparams,
                              int32_t n_fparams, const uint32_t* grid3, const uint32_t* threads3,
                              void* stream, double* elapsed_us);

/* ---- event timing (for benchmarks that time a sequence of launches) ---- */
int32_t enigma_event_create(void** ev);
int32_t enigma_event_destroy(void* ev);
int32_t enigma_event_record(void* ev, void* stream);
int32_t enigma_event_elapsed_ms(void* start, void* stop, float* ms);

/* Number of device-side timeouts flagged since the last call (and reset): the library's
 * per-device status word plus the no-allocation decode entry's word.  Allocates nothing. */
int32_t enigma_take_device_status(int32_t* timeouts);
/* Self-test of the timeout reporting: enqueues one CTA that waits on a barrier nothing
 * arrives on, gives up after `polls` polls (<= 2^24; microseconds) and flags the device status
 * word as the kernels' bounded waits do; the next enigma_synchronize then returns
 * ENIGMA_ERR_TIMEOUT and clears it, and the context stays usable. */
int32_t enigma_check_timeout_path(int64_t polls, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ENIGMA_CUDA_H */
