// rmsnorm.cu — one-pass RMSNorm for sm_100a.
//
//   y[r, :] = x[r, :] * 1/sqrt(mean(x[r, :]^2) + eps) * w[:]
//
// Semantics follow the reference's numpy check
// (examples/benchmark_rmsnorm.py:117-118, `X / sqrt(mean(X**2) + eps) * W`) and
// the Qwen layer's `_rmsnorm` (examples/qwen_megakernel.py:308-310); the
// accumulation is fp32 for both fp32 and bf16 storage.
//
// Fast path: one CTA per row, the row held in registers between the reduction
// and the write, so HBM sees exactly one read of x and one write of y.  Every
// access is a 16-byte vector (128-bit coalesced), x is read with an
// L1::no_allocate streaming hint and y is written with .cs (evict-first): the
// only data worth caching is w, which every row re-reads.  The row reduction
// is a warp shuffle tree followed by one shared-memory exchange between warps.
//
// Generic path (any hidden size, any alignment): a grid-stride scalar kernel,
// two reads of the row.  It exists for ragged shapes and tests; the bench
// shapes never take it.
#include "common.cuh"

namespace {

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int kElems = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int kElems = 8; };

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w) : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack(const uint4& v, float* f);
template <>
__device__ __forceinline__ void unpack<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float* f);
template <>
__device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  using enigma_sm100::pack_bf16x2;
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// THREADS threads per row, NV 16-byte vectors per thread.  Without PRED the row is
// exactly THREADS*NV vectors; with PRED it has row_vecs <= THREADS*NV vectors and the
// vectors past the end are skipped (e.g. hidden 896 bf16 = 112 vectors on 128 threads).
// PDL: launched as a programmatic dependent (the decode step's first kernel, which in a
// layer stack follows the previous layer's last GEMM): the next kernel may start its
// prologue at once, and every read of x waits until the previous kernel has completed.
template <typename T, int THREADS, int NV, bool PRED = false, bool PDL = false>
__global__ void __launch_bounds__(THREADS)
rmsnorm_row_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                   int64_t rows, float inv_hidden, float eps, int row_vecs) {
  constexpr int VE = Vec<T>::kElems;
  constexpr int kWarps = THREADS / 32;
  const int64_t kRowVecs = PRED ? row_vecs : int64_t(THREADS) * NV;
  __shared__ float red[kWarps];
  if constexpr (PDL) {
    enigma_sm100::griddep_launch_dependents();
    enigma_sm100::griddep_wait();
  }

  const int tid = threadIdx.x;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint4* xv = reinterpret_cast<const uint4*>(x) + row * kRowVecs;
    uint4* yv = reinterpret_cast<uint4*>(y) + row * kRowVecs;

    uint4 raw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i)
      raw[i] = (!PRED || tid + i * THREADS < kRowVecs) ? ld_stream(xv + tid + i * THREADS)
                                                       : make_uint4(0u, 0u, 0u, 0u);

    float ss = 0.f;
    float f[NV][VE];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      unpack<T>(raw[i], f[i]);
#pragma unroll
      for (int j = 0; j < VE; ++j) ss = fmaf(f[i][j], f[i][j], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) total += red[i];
    __syncthreads();  // red[] is reused by the next row of this CTA

    const float scale = 1.0f / sqrtf(total * inv_hidden + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (PRED && tid + i * THREADS >= kRowVecs) continue;
      float wf[VE];
      unpack<T>(__ldg(wv + tid + i * THREADS), wf);
      float o[VE];
#pragma unroll
      for (int j = 0; j < VE; ++j) o[j] = f[i][j] * scale * wf[j];
      st_stream(yv + tid + i * THREADS, pack<T>(o));
    }
  }
}

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(256)
rmsnorm_generic_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                       int64_t rows, int64_t hidden, float eps) {
  __shared__ float red[8];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * hidden;
    T* yr = y + row * hidden;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < hidden; i += 256) {
      const float v = to_f<T>(xr[i]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) total += red[i];
    __syncthreads();
    const float scale = 1.0f / sqrtf(total / float(hidden) + eps);
    for (int64_t i = threadIdx.x; i < hidden; i += 256)
      yr[i] = from_f<T>(to_f<T>(xr[i]) * scale * to_f<T>(w[i]));
  }
}

template <typename T, int THREADS, int NV, bool PRED = false, bool PDL = false>
cudaError_t launch_row(const void* x, const void* w, void* y, int64_t rows, int64_t hidden,
                       float eps, int sms, cudaStream_t s) {
  // Enough CTAs to fill every SM several times over; each CTA strides over rows.
  const int64_t max_ctas = int64_t(sms) * (2048 / THREADS) * 8;
  const int grid = int(rows < max_ctas ? rows : max_ctas);
  enigma::note_kernel("rmsnorm_row_kernel");
  if constexpr (PDL) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rmsnorm_row_kernel<T, THREADS, NV, PRED, true>,
                              static_cast<const T*>(x), static_cast<const T*>(w),
                              static_cast<T*>(y), rows, 1.0f / float(hidden), eps,
                              int(hidden / Vec<T>::kElems));
  }
  rmsnorm_row_kernel<T, THREADS, NV, PRED><<<grid, THREADS, 0, s>>>(
      static_cast<const T*>(x), static_cast<const T*>(w), static_cast<T*>(y), rows,
      1.0f / float(hidden), eps, int(hidden / Vec<T>::kElems));
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch(const void* x, const void* w, void* y, int64_t rows, int64_t hidden,
                     float eps, int sms, cudaStream_t s) {
  constexpr int VE = Vec<T>::kElems;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(y) % 16 == 0) && (hidden % VE == 0);
  if (aligned) {
    const int64_t vecs = hidden / VE;  // 16-byte vectors per row
    // Pick (threads, vectors/thread) with threads <= 256 and at most 8 vectors held.
    switch (vecs) {
      case 32:   return launch_row<T, 32, 1>(x, w, y, rows, hidden, eps, sms, s);
      case 64:   return launch_row<T, 64, 1>(x, w, y, rows, hidden, eps, sms, s);
      case 128:  return launch_row<T, 128, 1>(x, w, y, rows, hidden, eps, sms, s);
      case 256:  return launch_row<T, 128, 2>(x, w, y, rows, hidden, eps, sms, s);
      case 512:  return launch_row<T, 128, 4>(x, w, y, rows, hidden, eps, sms, s);
      case 1024: return launch_row<T, 256, 4>(x, w, y, rows, hidden, eps, sms, s);
      case 2048: return launch_row<T, 256, 8>(x, w, y, rows, hidden, eps, sms, s);
      default:
        if (vecs <= 128) return launch_row<T, 128, 1, true>(x, w, y, rows, hidden, eps, sms, s);
        if (vecs <= 256) return launch_row<T, 128, 2, true>(x, w, y, rows, hidden, eps, sms, s);
        if (vecs <= 512) return launch_row<T, 128, 4, true>(x, w, y, rows, hidden, eps, sms, s);
        if (vecs <= 1024) return launch_row<T, 256, 4, true>(x, w, y, rows, hidden, eps, sms, s);
        if (vecs <= 2048) return launch_row<T, 256, 8, true>(x, w, y, rows, hidden, eps, sms, s);
        break;
    }
  }
  const int64_t max_ctas = int64_t(sms) * 16;
  const int grid = int(rows < max_ctas ? rows : max_ctas);
  enigma::note_kernel("rmsnorm_generic_kernel");
  rmsnorm_generic_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(x),
                                                 static_cast<const T*>(w), static_cast<T*>(y),
                                                 rows, hidden, eps);
  return cudaGetLastError();
}

}  // namespace

namespace enigma {
cudaError_t rmsnorm_launch_sms(int dtype, const void* x, const void* w, void* y, int64_t rows,
                               int64_t hidden, float eps, int sms, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (dtype == ENIGMA_DTYPE_F32) return dispatch<float>(x, w, y, rows, hidden, eps, sms, s);
  return dispatch<__nv_bfloat16>(x, w, y, rows, hidden, eps, sms, s);
}

cudaError_t rmsnorm_launch_pdl_bf16(const void* x, const void* w, void* y, int64_t rows,
                                    int64_t hidden, float eps, int sms, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  using T = __nv_bfloat16;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(y) % 16 == 0) && (hidden % 8 == 0);
  const int64_t vecs = hidden / 8;
  if (aligned && vecs == 128) return launch_row<T, 128, 1, false, true>(x, w, y, rows, hidden, eps, sms, s);
  if (aligned && vecs < 128) return launch_row<T, 128, 1, true, true>(x, w, y, rows, hidden, eps, sms, s);
  return dispatch<T>(x, w, y, rows, hidden, eps, sms, s);
}

cudaError_t rmsnorm_launch(int dtype, const void* x, const void* w, void* y, int64_t rows,
                           int64_t hidden, float eps, cudaStream_t s) {
  return rmsnorm_launch_sms(dtype, x, w, y, rows, hidden, eps, sm_count(), s);
}
}  // namespace enigma
