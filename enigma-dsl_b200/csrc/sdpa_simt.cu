// sdpa_simt.cu — scaled-dot-product attention on CUDA cores, any head_dim <= 256.
//
//   O[b,h,i,:] = sum_j softmax_j(scale * Q[b,h,i,:] . K[b,h/g,j,:]) V[b,h/g,j,:]
//
// Online (streaming) softmax over the key axis, one warp per query row, fp32
// accumulation.  This is the small-shape path: the reference's FlashAttention-1
// showcase (examples/showcase_attention.py:31-91, D = 4, with 1/sqrt(D) scale),
// its GQA decode kernel (examples/benchmark_sdpa.py:48-150, kv-head = q-head /
// QMUL, no scale), the fp32 variants, and any bf16 shape the tensor-core kernel
// does not take.  Causal masking keeps key j <= i + (Skv - Sq).
#include "common.cuh"

namespace {

template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void store_elem(T* p, float v);
template <> __device__ __forceinline__ void store_elem<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

constexpr int kMaxDPerLane = 8;  // head_dim <= 256

// Element strides (batch, head, sequence) of Q, K, V, O; head_dim is contiguous.
struct Strides {
  int64_t q[3], k[3], v[3], o[3];
};

template <typename T>
__global__ void __launch_bounds__(128)
sdpa_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
                 T* __restrict__ O, int64_t B, int Hq, int Hkv, int64_t Sq, int64_t Skv, int D,
                 float scale, int causal, Strides st, const float* __restrict__ sinks) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * 4 + warp;  // over B*Hq*Sq
  const int64_t total = B * Hq * Sq;
  if (row >= total) return;
  const int64_t i = row % Sq;
  const int64_t bh = row / Sq;
  const int h = int(bh % Hq);
  const int64_t b = bh / Hq;
  const int hk = h / (Hq / Hkv);
  const T* q = Q + b * st.q[0] + h * st.q[1] + i * st.q[2];
  const T* kb = K + b * st.k[0] + hk * st.k[1];
  const T* vb = V + b * st.v[0] + hk * st.v[1];
  const int64_t ks = st.k[2], vs = st.v[2];

  float qv[kMaxDPerLane], acc[kMaxDPerLane];
#pragma unroll
  for (int t = 0; t < kMaxDPerLane; ++t) {
    const int d = lane + 32 * t;
    qv[t] = d < D ? ld<T>(q + d) * scale : 0.f;
    acc[t] = 0.f;
  }
  const int64_t last = causal ? min(Skv - 1, i + (Skv - Sq)) : Skv - 1;
  float m = -INFINITY, l = 0.f;
  for (int64_t j = 0; j <= last; ++j) {
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < kMaxDPerLane; ++t) {
      const int d = lane + 32 * t;
      if (d < D) s = fmaf(qv[t], ld<T>(kb + j * ks + d), s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float m_new = fmaxf(m, s);
    const float corr = expf(m - m_new);
    const float p = expf(s - m_new);
    l = l * corr + p;
#pragma unroll
    for (int t = 0; t < kMaxDPerLane; ++t) {
      const int d = lane + 32 * t;
      if (d < D) acc[t] = fmaf(acc[t], corr, p * ld<T>(vb + j * vs + d));
    }
    m = m_new;
  }
  // An attention sink (gpt-oss; examples/metal/sdpa_handwritten.metal:39-42 start the
  // running max at s[h] with l = 1) adds exp(s_h - M) to the denominator only.
  if (sinks != nullptr) {
    const float sk = sinks[h];
    const float m_new = fmaxf(m, sk);
    const float corr = expf(m - m_new);
    l = l * corr + expf(sk - m_new);
#pragma unroll
    for (int t = 0; t < kMaxDPerLane; ++t) acc[t] *= corr;
  }
  // last < 0 only when causal with Sq > Skv: the row sees no key; it is defined as 0.
  const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
  for (int t = 0; t < kMaxDPerLane; ++t) {
    const int d = lane + 32 * t;
    if (d < D) store_elem<T>(O + b * st.o[0] + h * st.o[1] + i * st.o[2] + d, acc[t] * inv);
  }
}

Strides dense_strides(int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D) {
  Strides st;
  st.q[0] = st.o[0] = Hq * Sq * D;
  st.q[1] = st.o[1] = Sq * D;
  st.q[2] = st.o[2] = D;
  st.k[0] = st.v[0] = Hkv * Skv * D;
  st.k[1] = st.v[1] = Skv * D;
  st.k[2] = st.v[2] = D;
  return st;
}

template <typename T>
cudaError_t launch(const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t Hq,
                   int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, float scale, bool causal,
                   cudaStream_t s, const Strides& st, const float* sinks = nullptr) {
  const int64_t rows = B * Hq * Sq;
  const int64_t blocks = (rows + 3) / 4;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  sdpa_simt_kernel<T><<<unsigned(blocks), 128, 0, s>>>(
      static_cast<const T*>(Q), static_cast<const T*>(K), static_cast<const T*>(V),
      static_cast<T*>(O), B, int(Hq), int(Hkv), Sq, Skv, int(D), scale, causal ? 1 : 0, st, sinks);
  return cudaGetLastError();
}

}  // namespace

namespace enigma {
cudaError_t sdpa_simt_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                                  int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                                  float scale, bool causal, cudaStream_t s) {
  return launch<__nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s,
                               dense_strides(Hq, Hkv, Sq, Skv, D));
}
cudaError_t sdpa_f32_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                            int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                            float scale, bool causal, cudaStream_t s) {
  note_kernel("sdpa_simt_kernel");
  return launch<float>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s,
                       dense_strides(Hq, Hkv, Sq, Skv, D));
}

cudaError_t sdpa_strided_launch(int dtype, const void* Q, const void* K, const void* V, void* O,
                                int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv,
                                int64_t D, const int64_t* strides12, float scale, bool causal,
                                const float* sinks, cudaStream_t s) {
  Strides st;
  for (int i = 0; i < 3; ++i) {
    st.q[i] = strides12[i];
    st.k[i] = strides12[3 + i];
    st.v[i] = strides12[6 + i];
    st.o[i] = strides12[9 + i];
  }
  if (dtype == ENIGMA_DTYPE_F32)
    return launch<float>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s, st, sinks);
  return launch<__nv_bfloat16>(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s, st, sinks);
}
}  // namespace enigma
