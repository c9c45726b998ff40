// decode_f32.cu — the reference's fp32 single-layer decode megakernel, on sm_100a.
//
// examples/qwen_megakernel.py:228-269 (qwen_fused) runs, for one token:
//   norm1 = rmsnorm(x, w_norm); q, k, v = Wq norm1, Wk norm1, Wv norm1
//   q_rope = rope(rmsnorm_head(q, w_q_norm)); k_rope = rope(rmsnorm_head(k, w_k_norm))
//   attn[h] = softmax(K_cache[h/g] q_rope[h] * scale) V_cache[h/g]   (caches hold the new k, v)
//   oproj = Wo attn + x; post = rmsnorm(oproj, w_post)
//   out = Wd (silu(Wg post) * (Wu post)) + oproj
// with weights row-major [out, in] (y = W x).  Here each phase is its own kernel (fp32
// throughout, like the reference): warp-per-row GEMVs with 16-byte loads, a fused
// gate/up GEMV + SwiGLU, a per-head RMSNorm + RoPE kernel, the strided CUDA-core attention
// and the fp32 RMSNorm.  The reference's scratch buffers (norm_buf, q_buf, ...) are the
// workspace, so nothing is allocated.
#include "common.cuh"

namespace {

// out[n] = W[n, :] . x (+ res[n]); one warp per output row.
__global__ void __launch_bounds__(256)
gemv_f32_kernel(const float* __restrict__ W, const float* __restrict__ x,
                const float* __restrict__ res, float* __restrict__ out, int N, int K) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= N) return;
  const float* w = W + int64_t(row) * K;
  float acc = 0.f;
  if ((K & 3) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = lane; i < K / 4; i += 32) {
      const float4 a = __ldg(w4 + i), b = __ldg(x4 + i);
      acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
    }
  } else {
    for (int i = lane; i < K; i += 32) acc = fmaf(__ldg(w + i), __ldg(x + i), acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = res ? acc + res[row] : acc;
}

// out[n] = silu(Wg[n] . x) * (Wu[n] . x); one warp per row (qwen_megakernel.py:195-216).
__global__ void __launch_bounds__(256)
swiglu_gemv_f32_kernel(const float* __restrict__ Wg, const float* __restrict__ Wu,
                       const float* __restrict__ x, float* __restrict__ out, int N, int K) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= N) return;
  float g = 0.f, u = 0.f;
  for (int i = lane; i < K; i += 32) {
    const float xv = __ldg(x + i);
    g = fmaf(__ldg(Wg + int64_t(row) * K + i), xv, g);
    u = fmaf(__ldg(Wu + int64_t(row) * K + i), xv, u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    g += __shfl_xor_sync(0xffffffffu, g, o);
    u += __shfl_xor_sync(0xffffffffu, u, o);
  }
  if (lane == 0) out[row] = g / (1.0f + expf(-g)) * u;
}

// Per head h: y = rmsnorm(in[h, :]) * w, then rotate-half RoPE with full-length cos / sin
// tables (qwen_megakernel.py:86-107).  One CTA of D threads per head, D <= 256, D even.
__global__ void __launch_bounds__(256)
head_norm_rope_f32_kernel(const float* __restrict__ in, const float* __restrict__ w,
                          const float* __restrict__ cosv, const float* __restrict__ sinv,
                          float* __restrict__ out, int D, float eps) {
  __shared__ float y[256];
  __shared__ float red[8];
  const int h = blockIdx.x, d = threadIdx.x;
  const float v = in[int64_t(h) * D + d];
  float ss = v * v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((d & 31) == 0) red[d >> 5] = ss;
  __syncthreads();
  float total = 0.f;
  for (int i = 0; i < (D + 31) / 32; ++i) total += red[i];
  y[d] = v * (1.0f / sqrtf(total / float(D) + eps)) * w[d];
  __syncthreads();
  const int half = D / 2;
  float r;
  if (d < half) r = y[d] * cosv[d] - y[d + half] * sinv[d];
  else r = y[d] * cosv[d] + y[d - half] * sinv[d];
  out[int64_t(h) * D + d] = r;
}

}  // namespace

namespace enigma {

cudaError_t qwen_decode_f32_launch(const enigma_qwen_decode_f32_desc& q, cudaStream_t s) {
  const int H = int(q.hidden), D = int(q.head_dim), Hq = int(q.heads_q), Hkv = int(q.heads_kv);
  const int I = int(q.intermediate), CT = int(q.cache_total);
  const int QSZ = Hq * D, KVSZ = Hkv * D;
  auto gemv = [&](const float* W, const float* x, const float* res, float* out, int N, int K) {
    gemv_f32_kernel<<<(N + 7) / 8, 256, 0, s>>>(W, x, res, out, N, K);
    return cudaGetLastError();
  };
  cudaError_t e;
#define ENIGMA_TRY(expr)           \
  do {                             \
    e = (expr);                    \
    if (e != cudaSuccess) return e; \
  } while (0)
  ENIGMA_TRY(rmsnorm_launch(ENIGMA_DTYPE_F32, q.x, q.w_norm, q.norm_buf, 1, H, q.eps, s));
  ENIGMA_TRY(gemv(q.Wq, q.norm_buf, nullptr, q.q_buf, QSZ, H));
  ENIGMA_TRY(gemv(q.Wk, q.norm_buf, nullptr, q.k_buf, KVSZ, H));
  ENIGMA_TRY(gemv(q.Wv, q.norm_buf, nullptr, q.v_buf, KVSZ, H));
  head_norm_rope_f32_kernel<<<Hq, D, 0, s>>>(q.q_buf, q.w_q_norm, q.cos_pos, q.sin_pos,
                                              q.q_rope_buf, D, q.eps);
  ENIGMA_TRY(cudaGetLastError());
  head_norm_rope_f32_kernel<<<Hkv, D, 0, s>>>(q.k_buf, q.w_k_norm, q.cos_pos, q.sin_pos,
                                               q.k_rope_buf, D, q.eps);
  ENIGMA_TRY(cudaGetLastError());
  // Attention of each q head over the cache (one query per head): strided views
  // Q [1, Hq, 1, D], K/V [1, Hkv, CT, D], O [1, Hq, 1, D].
  const int64_t st[12] = {0, D, D, 0, int64_t(CT) * D, D, 0, int64_t(CT) * D, D, 0, D, D};
  ENIGMA_TRY(sdpa_strided_launch(ENIGMA_DTYPE_F32, q.q_rope_buf, q.k_cache, q.v_cache,
                                 q.attn_buf, 1, Hq, Hkv, 1, CT, D, st, q.attn_scale, false,
                                 nullptr, s));
  ENIGMA_TRY(gemv(q.Wo, q.attn_buf, q.x, q.norm_buf, H, QSZ));         // oproj (+ x)
  ENIGMA_TRY(rmsnorm_launch(ENIGMA_DTYPE_F32, q.norm_buf, q.w_post, q.post_buf, 1, H, q.eps, s));
  swiglu_gemv_f32_kernel<<<(I + 7) / 8, 256, 0, s>>>(q.Wg, q.Wu, q.post_buf, q.mlp_buf, I, H);
  ENIGMA_TRY(cudaGetLastError());
  ENIGMA_TRY(gemv(q.Wd, q.mlp_buf, q.norm_buf, q.out, H, I));          // down (+ oproj)
#undef ENIGMA_TRY
  return cudaSuccess;
}

}  // namespace enigma
