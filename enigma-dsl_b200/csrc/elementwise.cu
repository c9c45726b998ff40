// elementwise.cu — C = A op B over n elements (the reference's TV-layout elementwise
// example, examples/vector_add_tv.py:13-55, and the one-thread-per-element form,
// examples/vector_add.py).  HBM-bound: 16-byte vector accesses, grid-stride loop over
// vectors, a scalar tail.  op: 0 add, 1 sub, 2 mul, 3 max, 4 min.
#include <algorithm>

#include "common.cuh"

namespace {

__device__ __forceinline__ float apply(int op, float a, float b) {
  switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    case 3: return fmaxf(a, b);
    default: return fminf(a, b);
  }
}

template <typename T> struct EW;
template <> struct EW<float> {
  static constexpr int kVec = 4;
  __device__ static float ld(const float* p) { return *p; }
  __device__ static void st(float* p, float v) { *p = v; }
};
template <> struct EW<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ static void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

template <typename T>
__global__ void __launch_bounds__(256)
elementwise_kernel(int op, const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c,
                   int64_t n) {
  constexpr int V = EW<T>::kVec;
  const int64_t nv = n / V;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const uint4* a4 = reinterpret_cast<const uint4*>(a);
  const uint4* b4 = reinterpret_cast<const uint4*>(b);
  uint4* c4 = reinterpret_cast<uint4*>(c);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    uint4 x = __ldg(a4 + i), y = __ldg(b4 + i), z;
    const T* xs = reinterpret_cast<const T*>(&x);
    const T* ys = reinterpret_cast<const T*>(&y);
    T* zs = reinterpret_cast<T*>(&z);
#pragma unroll
    for (int k = 0; k < V; ++k) EW<T>::st(zs + k, apply(op, EW<T>::ld(xs + k), EW<T>::ld(ys + k)));
    c4[i] = z;
  }
  for (int64_t i = nv * V + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    EW<T>::st(c + i, apply(op, EW<T>::ld(a + i), EW<T>::ld(b + i)));
}

template <typename T>
cudaError_t launch(int op, const void* a, const void* b, void* c, int64_t n, cudaStream_t s) {
  const int64_t vecs = n / EW<T>::kVec + 1;
  const int64_t cap = int64_t(enigma::sm_count()) * 8;
  const int grid = int(std::min<int64_t>(cap, (vecs + 255) / 256));
  elementwise_kernel<T><<<grid, 256, 0, s>>>(op, static_cast<const T*>(a), static_cast<const T*>(b),
                                             static_cast<T*>(c), n);
  return cudaGetLastError();
}

}  // namespace

namespace enigma {
cudaError_t elementwise_launch(int op, int dtype, const void* a, const void* b, void* c, int64_t n,
                               cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (dtype == ENIGMA_DTYPE_F32) return launch<float>(op, a, b, c, n, s);
  return launch<__nv_bfloat16>(op, a, b, c, n, s);
}
}  // namespace enigma
