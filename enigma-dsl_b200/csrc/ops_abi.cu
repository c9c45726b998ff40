// ops_abi.cu — C-ABI operator entry points, generic dispatch by kernel id and
// event timing.  Validation happens here; kernels assume valid arguments.
#include <cstdio>

#include <algorithm>

#include "common.cuh"

using enigma::set_error;

namespace {

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int32_t launch_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ENIGMA_OK;
  set_error("%s launch failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  return ENIGMA_ERR_LAUNCH;
}

int32_t bad(const char* msg) {
  set_error("bad argument: %s", msg);
  return ENIGMA_ERR_BADARG;
}

bool aligned(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

}  // namespace

extern "C" {

int32_t enigma_rmsnorm(int32_t dtype, const void* x, const void* w, void* y, int64_t rows,
                       int64_t hidden, float eps, void* stream) {
  if (dtype != ENIGMA_DTYPE_F32 && dtype != ENIGMA_DTYPE_BF16) return bad("rmsnorm dtype");
  if (rows < 0 || hidden <= 0) return bad("rmsnorm needs rows >= 0 and hidden > 0");
  if (rows > 0 && (x == nullptr || w == nullptr || y == nullptr))
    return bad("rmsnorm: NULL buffer");
  const size_t es = dtype == ENIGMA_DTYPE_F32 ? 4 : 2;
  if (!aligned(x, es) || !aligned(w, es) || !aligned(y, es))
    return bad("rmsnorm: buffers must be aligned to the element size");
  if (!(eps >= 0.0f)) return bad("rmsnorm: eps must be >= 0");
  return launch_status(
      enigma::rmsnorm_launch(dtype, x, w, y, rows, hidden, eps, as_stream(stream)), "rmsnorm");
}

// ---- RMSNorm of host-resident rows with overlapped transfers ----------------------------
// Workspace: w, then two chunk sets (x chunk, y chunk), each 256-byte aligned.
static size_t rms_host_ws(size_t es, int64_t hidden, int64_t chunk_rows) {
  auto a256 = [](size_t v) { return (v + 255) & ~size_t(255); };
  return a256(size_t(hidden) * es) + 4 * a256(size_t(chunk_rows) * size_t(hidden) * es);
}

int32_t enigma_rmsnorm_host_workspace_bytes(int32_t dtype, int64_t hidden, int64_t chunk_rows,
                                            size_t* bytes) {
  if (dtype != ENIGMA_DTYPE_F32 && dtype != ENIGMA_DTYPE_BF16) return bad("rmsnorm dtype");
  if (hidden <= 0 || chunk_rows <= 0) return bad("rmsnorm_host: hidden and chunk_rows must be > 0");
  if (bytes == nullptr) return bad("rmsnorm_host: bytes is NULL");
  *bytes = rms_host_ws(dtype == ENIGMA_DTYPE_F32 ? 4 : 2, hidden, chunk_rows);
  return ENIGMA_OK;
}

int32_t enigma_rmsnorm_host(int32_t dtype, const void* x_host, const void* w_host, void* y_host,
                            int64_t rows, int64_t hidden, float eps, void* workspace,
                            size_t workspace_bytes, int64_t chunk_rows, void* stream) {
  if (dtype != ENIGMA_DTYPE_F32 && dtype != ENIGMA_DTYPE_BF16) return bad("rmsnorm dtype");
  if (rows < 0 || hidden <= 0 || chunk_rows <= 0)
    return bad("rmsnorm_host needs rows >= 0, hidden > 0, chunk_rows > 0");
  if (!(eps >= 0.0f)) return bad("rmsnorm: eps must be >= 0");
  if (rows == 0) return ENIGMA_OK;
  if (x_host == nullptr || w_host == nullptr || y_host == nullptr || workspace == nullptr)
    return bad("rmsnorm_host: NULL buffer");
  const size_t es = dtype == ENIGMA_DTYPE_F32 ? 4 : 2;
  if (!aligned(workspace, 256) || workspace_bytes < rms_host_ws(es, hidden, chunk_rows))
    return bad("rmsnorm_host: workspace must be 256-byte aligned and at least "
               "enigma_rmsnorm_host_workspace_bytes() bytes");
  auto a256 = [](size_t v) { return (v + 255) & ~size_t(255); };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* w_dev = ws;
  const size_t chunk_bytes = a256(size_t(chunk_rows) * size_t(hidden) * es);
  uint8_t* set0 = ws + a256(size_t(hidden) * es);
  cudaStream_t st[2] = {as_stream(stream), enigma::aux_stream()};
  if (st[1] == nullptr) return bad("rmsnorm_host: could not create the second stream");
  const uint8_t* xh = static_cast<const uint8_t*>(x_host);
  uint8_t* yh = static_cast<uint8_t*>(y_host);
  cudaEvent_t ready = nullptr, done = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
  // w once on the caller's stream; the second stream starts after it.
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w_dev, w_host, size_t(hidden) * es, cudaMemcpyHostToDevice, st[0]);
  if (e == cudaSuccess) e = cudaEventRecord(ready, st[0]);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st[1], ready, 0);
  // Chunk c on stream c % 2 with buffer set c % 2: upload, kernel, download in stream order,
  // so one stream's upload overlaps the other's kernel and download (PCIe is full duplex).
  for (int64_t r0 = 0, c = 0; e == cudaSuccess && r0 < rows; r0 += chunk_rows, ++c) {
    const int64_t n = std::min<int64_t>(chunk_rows, rows - r0);
    const size_t off = size_t(r0) * size_t(hidden) * es, nb = size_t(n) * size_t(hidden) * es;
    uint8_t* xd = set0 + (c & 1) * 2 * chunk_bytes;
    uint8_t* yd = xd + chunk_bytes;
    cudaStream_t sc = st[c & 1];
    e = cudaMemcpyAsync(xd, xh + off, nb, cudaMemcpyHostToDevice, sc);
    if (e == cudaSuccess) e = enigma::rmsnorm_launch(dtype, xd, w_dev, yd, n, hidden, eps, sc);
    if (e == cudaSuccess) e = cudaMemcpyAsync(yh + off, yd, nb, cudaMemcpyDeviceToHost, sc);
  }
  // The caller's stream ends after both; the call returns when everything is done.
  if (e == cudaSuccess) e = cudaEventRecord(done, st[1]);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st[0], done, 0);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st[0]);
  if (ready) cudaEventDestroy(ready);
  if (done) cudaEventDestroy(done);
  return launch_status(e, "rmsnorm_host");
}

int32_t enigma_elementwise(int32_t op, int32_t dtype, const void* A, const void* B, void* C,
                           int64_t n, void* stream) {
  if (op < 0 || op > 4) return bad("elementwise: op must be 0..4");
  if (dtype != ENIGMA_DTYPE_F32 && dtype != ENIGMA_DTYPE_BF16) return bad("elementwise: dtype");
  if (n < 0) return bad("elementwise: n < 0");
  if (n == 0) return ENIGMA_OK;
  if (A == nullptr || B == nullptr || C == nullptr) return bad("elementwise: NULL buffer");
  if (!aligned(A, 16) || !aligned(B, 16) || !aligned(C, 16))
    return bad("elementwise: buffers must be 16-byte aligned");
  return launch_status(enigma::elementwise_launch(op, dtype, A, B, C, n, as_stream(stream)),
                       "elementwise");
}

int32_t enigma_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                         void* stream) {
  if (M < 0 || N < 0 || K < 0) return bad("gemm: negative size");
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1)
    return bad("gemm: sizes must fit in int32");
  if (M == 0 || N == 0) return ENIGMA_OK;
  if (A == nullptr || B == nullptr || C == nullptr) return bad("gemm: NULL buffer");
  if (!aligned(A, 2) || !aligned(B, 2) || !aligned(C, 2)) return bad("gemm: misaligned buffer");
  return launch_status(enigma::gemm_bf16_launch(A, B, C, M, N, K, as_stream(stream)), "gemm");
}

int32_t enigma_sdpa_bf16(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                         int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                         int64_t head_dim, float scale, int32_t causal, void* stream) {
  if (batch < 0 || heads_q <= 0 || heads_kv <= 0 || seq_q < 0 || seq_kv < 0 || head_dim <= 0)
    return bad("sdpa: sizes must be positive");
  if (heads_q % heads_kv != 0) return bad("sdpa: heads_q must be a multiple of heads_kv");
  if (head_dim > 256) return bad("sdpa: head_dim must be <= 256");
  if (batch == 0 || seq_q == 0) return ENIGMA_OK;
  if (seq_kv == 0) return bad("sdpa: seq_kv must be > 0 when seq_q > 0");
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) return bad("sdpa: NULL buffer");
  if (!aligned(Q, 2) || !aligned(K, 2) || !aligned(V, 2) || !aligned(O, 2))
    return bad("sdpa: misaligned buffer");
  return launch_status(enigma::sdpa_bf16_launch(Q, K, V, O, batch, heads_q, heads_kv, seq_q,
                                                seq_kv, head_dim, scale, causal != 0,
                                                as_stream(stream)),
                       "sdpa");
}

int32_t enigma_gemm_f32(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                        int32_t accumulate, void* stream) {
  if (M < 0 || N < 0 || K < 0) return bad("gemm: negative size");
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1)
    return bad("gemm: sizes must fit in int32");
  if (M == 0 || N == 0) return ENIGMA_OK;
  if (A == nullptr || B == nullptr || C == nullptr) return bad("gemm: NULL buffer");
  if (!aligned(A, 4) || !aligned(B, 4) || !aligned(C, 4)) return bad("gemm: misaligned buffer");
  return launch_status(enigma::gemm_f32_launch(A, B, C, M, N, K, accumulate != 0,
                                               as_stream(stream)),
                       "gemm_f32");
}

int32_t enigma_gemm_f32_trans(const void* A, const void* B, void* C, int64_t M, int64_t N,
                              int64_t K, int32_t trans_a, int32_t trans_b, int32_t accumulate,
                              void* stream) {
  if (M < 0 || N < 0 || K < 0) return bad("gemm: negative size");
  if (M > (1ll << 31) - 1 || N > (1ll << 31) - 1 || K > (1ll << 31) - 1)
    return bad("gemm: sizes must fit in int32");
  if (M == 0 || N == 0) return ENIGMA_OK;
  if (A == nullptr || B == nullptr || C == nullptr) return bad("gemm: NULL buffer");
  if (!aligned(A, 4) || !aligned(B, 4) || !aligned(C, 4)) return bad("gemm: misaligned buffer");
  return launch_status(enigma::gemm_f32_trans_launch(A, B, C, M, N, K, trans_a != 0,
                                                     trans_b != 0, accumulate != 0,
                                                     as_stream(stream)),
                       "gemm_f32_trans");
}

int32_t enigma_sdpa_f32(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                        int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                        int64_t head_dim, float scale, int32_t causal, void* stream) {
  if (batch < 0 || heads_q <= 0 || heads_kv <= 0 || seq_q < 0 || seq_kv < 0 || head_dim <= 0)
    return bad("sdpa: sizes must be positive");
  if (heads_q % heads_kv != 0) return bad("sdpa: heads_q must be a multiple of heads_kv");
  if (head_dim > 256) return bad("sdpa: head_dim must be <= 256");
  if (batch == 0 || seq_q == 0) return ENIGMA_OK;
  if (seq_kv == 0) return bad("sdpa: seq_kv must be > 0 when seq_q > 0");
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) return bad("sdpa: NULL buffer");
  if (!aligned(Q, 4) || !aligned(K, 4) || !aligned(V, 4) || !aligned(O, 4))
    return bad("sdpa: misaligned buffer");
  return launch_status(enigma::sdpa_f32_launch(Q, K, V, O, batch, heads_q, heads_kv, seq_q, seq_kv,
                                               head_dim, scale, causal != 0, as_stream(stream)),
                       "sdpa_f32");
}

int32_t enigma_sdpa_strided_sinks(int32_t dtype, const void* Q, const void* K, const void* V,
                                  void* O, int64_t batch, int64_t heads_q, int64_t heads_kv,
                                  int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                                  const int64_t* strides12, float scale, int32_t causal,
                                  const float* sinks, void* stream) {
  if (dtype != ENIGMA_DTYPE_F32 && dtype != ENIGMA_DTYPE_BF16) return bad("sdpa: dtype");
  if (batch < 0 || heads_q <= 0 || heads_kv <= 0 || seq_q < 0 || seq_kv < 0 || head_dim <= 0)
    return bad("sdpa: sizes must be positive");
  if (heads_q % heads_kv != 0) return bad("sdpa: heads_q must be a multiple of heads_kv");
  if (head_dim > 256) return bad("sdpa: head_dim must be <= 256");
  if (strides12 == nullptr) return bad("sdpa: strides is NULL");
  for (int i = 0; i < 12; ++i)
    if (strides12[i] < 0) return bad("sdpa: negative stride");
  if (batch == 0 || seq_q == 0) return ENIGMA_OK;
  if (seq_kv == 0) return bad("sdpa: seq_kv must be > 0 when seq_q > 0");
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) return bad("sdpa: NULL buffer");
  if (sinks != nullptr && !aligned(sinks, 4)) return bad("sdpa: sinks must be 4-byte aligned");
  return launch_status(enigma::sdpa_strided_launch(dtype, Q, K, V, O, batch, heads_q, heads_kv,
                                                   seq_q, seq_kv, head_dim, strides12, scale,
                                                   causal != 0, sinks, as_stream(stream)),
                       "sdpa_strided");
}

int32_t enigma_sdpa_strided(int32_t dtype, const void* Q, const void* K, const void* V, void* O,
                            int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q,
                            int64_t seq_kv, int64_t head_dim, const int64_t* strides12,
                            float scale, int32_t causal, void* stream) {
  return enigma_sdpa_strided_sinks(dtype, Q, K, V, O, batch, heads_q, heads_kv, seq_q, seq_kv,
                                   head_dim, strides12, scale, causal, nullptr, stream);
}

}  // extern "C"

namespace enigma {
int32_t check_decode_desc(const enigma_decode_layer_desc* d) {
  if (d == nullptr) return bad("decode: desc is NULL");
  if (d->batch <= 0 || d->batch > 128) return bad("decode: batch must be in [1, 128]");
  if (d->head_dim != 64) return bad("decode: head_dim must be 64");
  if (d->heads_kv <= 0 || d->heads_q % d->heads_kv != 0 || d->heads_q / d->heads_kv > 8)
    return bad("decode: heads_q must be a multiple of heads_kv, at most 8 per kv head");
  if (d->hidden <= 0 || d->hidden > 2048 || d->hidden % 64 != 0)
    return bad("decode: hidden must be a multiple of 64, at most 2048");
  if (d->intermediate <= 0 || d->intermediate % 32 != 0)
    return bad("decode: intermediate must be a positive multiple of 32");
  if (((d->heads_q + 2 * d->heads_kv) * 64) % 64 != 0) return bad("decode: qkv width");
  if (d->position < 0 || d->position >= d->cache_capacity)
    return bad("decode: position must be in [0, cache_capacity)");
  const void* ptrs[] = {d->w_in_norm, d->w_qkv, d->w_o, d->w_post_norm, d->w_gate_up,
                        d->w_down, d->rope_cos, d->rope_sin, d->k_cache, d->v_cache};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned(p, 16)) return bad("decode: NULL or non-16-byte-aligned pointer");
  return ENIGMA_OK;
}
}  // namespace enigma

extern "C" {

int32_t enigma_decode_workspace_bytes(const enigma_decode_layer_desc* desc, size_t* bytes) {
  int32_t rc = enigma::check_decode_desc(desc);
  if (rc != ENIGMA_OK) return rc;
  if (bytes == nullptr) return bad("decode: bytes is NULL");
  *bytes = enigma::decode_workspace_bytes(*desc);
  return ENIGMA_OK;
}

int32_t enigma_decode_layer_bf16(const enigma_decode_layer_desc* desc, const void* x, void* out,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  int32_t rc = enigma::check_decode_desc(desc);
  if (rc != ENIGMA_OK) return rc;
  if (x == nullptr || out == nullptr || workspace == nullptr || !aligned(x, 16) ||
      !aligned(out, 16) || !aligned(workspace, 256))
    return bad("decode: x / out must be 16-byte aligned, workspace 256-byte aligned");
  if (workspace_bytes < enigma::decode_workspace_bytes(*desc))
    return bad("decode: workspace smaller than enigma_decode_workspace_bytes()");
  return launch_status(enigma::decode_layer_launch(*desc, x, out, workspace, as_stream(stream)),
                       "decode_layer");
}

int32_t enigma_qwen_decode_f32(const enigma_qwen_decode_f32_desc* d, void* stream) {
  if (d == nullptr) return bad("qwen decode: desc is NULL");
  if (d->hidden <= 0 || d->heads_q <= 0 || d->heads_kv <= 0 || d->heads_q % d->heads_kv != 0 ||
      d->head_dim <= 0 || d->head_dim > 256 || d->head_dim % 2 != 0 || d->intermediate <= 0 ||
      d->cache_total <= 0)
    return bad("qwen decode: sizes (head_dim even and <= 256, heads_q multiple of heads_kv)");
  const void* ptrs[] = {d->x, d->w_norm, d->Wq, d->Wk, d->Wv, d->w_q_norm, d->w_k_norm,
                        d->cos_pos, d->sin_pos, d->k_cache, d->v_cache, d->Wo, d->w_post,
                        d->Wg, d->Wu, d->Wd, d->norm_buf, d->q_buf, d->k_buf, d->v_buf,
                        d->attn_buf, d->mlp_buf, d->post_buf, d->q_rope_buf, d->k_rope_buf,
                        d->out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned(p, 16)) return bad("qwen decode: NULL or unaligned buffer");
  return launch_status(enigma::qwen_decode_f32_launch(*d, as_stream(stream)), "qwen_decode_f32");
}

int32_t enigma_dispatch(int32_t kernel_id, void* const* buffers, int32_t n_buffers,
                        const int64_t* ip, int32_t n_ip, const float* fp, int32_t n_fp,
                        const uint32_t* grid3, const uint32_t* threads3, void* stream) {
  // grid / threads are the Metal-style totals a caller of the reference passes; the
  // operators pick their own CTA shapes, so they are only checked (NULL means "not given").
  for (int i = 0; i < 3; ++i) {
    if (grid3 != nullptr && grid3[i] == 0) return bad("dispatch: grid has a zero extent");
    if (threads3 != nullptr && threads3[i] == 0) return bad("dispatch: threads has a zero extent");
  }
  if (threads3 != nullptr &&
      uint64_t(threads3[0]) * threads3[1] * threads3[2] > 1024)
    return bad("dispatch: threads per threadgroup exceed 1024");
  if (n_buffers > 0 && buffers == nullptr) return bad("dispatch: buffers is NULL");
  if (n_ip > 0 && ip == nullptr) return bad("dispatch: iparams is NULL");
  if (n_fp > 0 && fp == nullptr) return bad("dispatch: fparams is NULL");
  switch (kernel_id) {
    case ENIGMA_KERNEL_RMSNORM:
      if (n_buffers != 3 || n_ip != 3 || n_fp != 1)
        return bad("rmsnorm dispatch wants 3 buffers, 3 int params, 1 float param");
      return enigma_rmsnorm(static_cast<int32_t>(ip[2]), buffers[0], buffers[1], buffers[2], ip[0],
                            ip[1], fp[0], stream);
    case ENIGMA_KERNEL_GEMM:
      if (n_buffers != 3 || n_ip != 5)
        return bad("gemm dispatch wants 3 buffers, 5 int params (M, N, K, dtype, accumulate)");
      if (ip[3] == ENIGMA_DTYPE_F32)
        return enigma_gemm_f32(buffers[0], buffers[1], buffers[2], ip[0], ip[1], ip[2],
                               static_cast<int32_t>(ip[4]), stream);
      if (ip[4] != 0) return bad("gemm dispatch: accumulate is fp32-only");
      return enigma_gemm_bf16(buffers[0], buffers[1], buffers[2], ip[0], ip[1], ip[2], stream);
    case ENIGMA_KERNEL_SDPA:
      if (n_buffers != 4 || n_ip != 8 || n_fp != 1)
        return bad("sdpa dispatch wants 4 buffers, 8 int params, 1 float param");
      if (ip[7] == ENIGMA_DTYPE_F32)
        return enigma_sdpa_f32(buffers[0], buffers[1], buffers[2], buffers[3], ip[0], ip[1], ip[2],
                               ip[3], ip[4], ip[5], fp[0], static_cast<int32_t>(ip[6]), stream);
      return enigma_sdpa_bf16(buffers[0], buffers[1], buffers[2], buffers[3], ip[0], ip[1], ip[2],
                              ip[3], ip[4], ip[5], fp[0], static_cast<int32_t>(ip[6]), stream);
    default: {
      char msg[64];
      snprintf(msg, sizeof(msg), "unknown kernel id %d", kernel_id);
      return bad(msg);
    }
  }
}

int32_t enigma_dispatch_timed(int32_t kernel_id, void* const* buffers, int32_t n_buffers,
                              const int64_t* ip, int32_t n_ip, const float* fp, int32_t n_fp,
                              const uint32_t* grid3, const uint32_t* threads3, void* stream,
                              double* elapsed_us) {
  if (elapsed_us == nullptr) return bad("elapsed_us is NULL");
  cudaEvent_t a, b;
  if (cudaEventCreate(&a) != cudaSuccess) return launch_status(cudaGetLastError(), "event");
  if (cudaEventCreate(&b) != cudaSuccess) {
    cudaEventDestroy(a);
    return launch_status(cudaGetLastError(), "event");
  }
  cudaEventRecord(a, as_stream(stream));
  int32_t rc = enigma_dispatch(kernel_id, buffers, n_buffers, ip, n_ip, fp, n_fp, grid3, threads3,
                               stream);
  cudaEventRecord(b, as_stream(stream));
  if (rc == ENIGMA_OK) rc = enigma_synchronize(stream);
  if (rc == ENIGMA_OK) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    *elapsed_us = double(ms) * 1000.0;
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return rc;
}

int32_t enigma_event_create(void** ev) {
  if (ev == nullptr) return bad("ev is NULL");
  cudaEvent_t e = nullptr;
  cudaError_t r = cudaEventCreate(&e);
  *ev = e;
  return launch_status(r, "event create");
}
int32_t enigma_event_destroy(void* ev) {
  if (ev == nullptr) return ENIGMA_OK;
  return launch_status(cudaEventDestroy(static_cast<cudaEvent_t>(ev)), "event destroy");
}
int32_t enigma_event_record(void* ev, void* stream) {
  if (ev == nullptr) return bad("ev is NULL");
  return launch_status(cudaEventRecord(static_cast<cudaEvent_t>(ev), as_stream(stream)),
                       "event record");
}
int32_t enigma_event_elapsed_ms(void* start, void* stop, float* ms) {
  if (start == nullptr || stop == nullptr || ms == nullptr) return bad("event elapsed: NULL");
  cudaError_t e = cudaEventSynchronize(static_cast<cudaEvent_t>(stop));
  if (e != cudaSuccess) return launch_status(e, "event sync");
  return launch_status(
      cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)),
      "event elapsed");
}

}  // extern "C"
