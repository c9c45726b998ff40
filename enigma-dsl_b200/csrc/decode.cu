// decode.cu — one decoder-layer decode step (Qwen-style) on sm_100a.
//
// The reference runs the layer as one threadgroup-wide Metal megakernel
// (examples/qwen_megakernel.py:228-269: RMSNorm -> Q/K/V matvec -> RoPE ->
// SDPA over the KV cache -> O-proj + residual -> RMSNorm -> SwiGLU -> down-proj
// + residual).  At batch 64 every GEMM is skinny (M = 64) and the step is bound
// by HBM: ~30 MB of weights and ~67 MB of KV cache per step.  So:
//
//   * GEMMs are split-K tcgen05 kernels: grid (N/64 tiles, K splits) fills the
//     148 SMs even for N = 896; each CTA streams its K range of B through a TMA
//     ring and writes an fp32 128x64 partial tile to a workspace.
//   * The split reduction is fused with what follows each GEMM: RoPE + KV-cache
//     append (QKV), residual add + RMSNorm (O-proj), SwiGLU (gate/up), residual
//     add (down-proj).
//   * Attention is split-KV ("flash decoding") in one persistent kernel: CTAs stream
//     balanced ranges of (sequence x kv head, 128-key chunk) pairs through a TMA ring,
//     and the CTA that finishes a (sequence, kv head) merges its partials.
//
// Workspace (caller-owned, enigma_decode_workspace_bytes) holds every partial
// and intermediate, so a step makes no allocation.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <utility>
#include <mutex>

#include "common.cuh"
#include "decode_common.cuh"

namespace {

using namespace enigma_sm100;
using namespace enigma_decode;

constexpr int SK_THREADS = 192;
constexpr int SK_SMEM = SK_RING + 1024;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// One split-K item per CTA: blockIdx = (N tile, split).
__global__ void __launch_bounds__(SK_THREADS)
gemm_splitk_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      float* __restrict__ partial, int M, int N, int K, int kb_per_split,
                      int a_rows, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[2 * SK_STAGES + 2];
  __shared__ uint32_t tmem_slot;
  const SkRing r{align1024(smem_raw), bars, bars + SK_STAGES, bars + 2 * SK_STAGES,
                 bars + 2 * SK_STAGES + 1};
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const SkItem w = sk_item(blockIdx.y * gridDim.x + blockIdx.x, gridDim.x, kb_per_split,
                           (K + SK_BK - 1) / SK_BK);
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    sk_ring_init(r);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, SK_BN);
    tmem_relinquish();
  }
  sk_zero_pad(r, a_rows, threadIdx.x, SK_THREADS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // The first stages' weight tiles go to shared memory and the rest of this CTA's slice to
  // L2 before waiting on the predecessor, so the weight stream overlaps its tail.
  int pre = 0;
  if (warp == 0 && lane == 0) {
    pre = sk_produce_pre(r, &tmB, w, a_rows, 0, status);
    for (int kb = w.kb0 + pre; kb < w.kb1; ++kb) tma_prefetch_l2_2d(&tmB, w.nb * SK_BN, kb * SK_BK);
  }
  griddep_wait();  // A (the previous kernel's output) and the partial buffer are ready / free
  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      sk_produce_rest(r, &tmA, &tmB, w, a_rows, pre, it, status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, acc = 0;
      sk_mma(r, tmem, w, it, acc, status);
    }
    __syncwarp();
  } else {
    uint32_t acc = 0;
    sk_store(r, tmem, w, partial, M, N, warp & 3, lane, acc, status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SK_BN);
  }
}

// Grid (M, Hq + 2 Hkv), 32 threads: one (row, head) per CTA.
__global__ void __launch_bounds__(32)
qkv_finalize_kernel(const float* __restrict__ part, int splits, int M, int N, int Hq, int Hkv,
                    const float* __restrict__ cosv, const float* __restrict__ sinv,
                    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kc,
                    __nv_bfloat16* __restrict__ vc, int s_cap, int pos,
                    uint32_t* __restrict__ attn_counters) {
  griddep_launch_dependents();
  griddep_wait();
  qkv_finalize_item(part, splits, M, N, Hq, Hkv, cosv, sinv, q_out, kc, vc, s_cap, pos,
                    attn_counters, blockIdx.x, blockIdx.y, threadIdx.x);
}

// One row per CTA of 256 threads.
__global__ void __launch_bounds__(256)
reduce_residual_norm_kernel(const float* __restrict__ part, int splits, int M, int N,
                            const __nv_bfloat16* __restrict__ residual,
                            __nv_bfloat16* __restrict__ h_out, const __nv_bfloat16* __restrict__ w,
                            __nv_bfloat16* __restrict__ y_out, float eps) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ float red[8];
  reduce_residual_norm_row(part, splits, M, N, residual, h_out, w, y_out, eps, blockIdx.x,
                           threadIdx.x, red);
}

// One float4 group (four columns) per thread.
__global__ void __launch_bounds__(256)
swiglu_kernel(const float* __restrict__ part, int splits, int M, int I,
              __nv_bfloat16* __restrict__ act) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t q = int64_t(blockIdx.x) * 256 + threadIdx.x;
  if (q * 4 < int64_t(M) * I) swiglu_group(part, splits, M, I, act, q);
}

// Persistent split-KV attention: one producer + DA_WARPS consumer warps per CTA, CTA c of
// gridDim.x takes chunk range c (see AttnCtx).
__global__ void __launch_bounds__(DA_THREADS)
decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __nv_bfloat16* __restrict__ q, float* __restrict__ opart,
                   float* __restrict__ mlpart, uint32_t* __restrict__ counters,
                   __nv_bfloat16* __restrict__ out, int Hq, int Hkv, int cap, int L, int S,
                   int units, float scale_log2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[DA_NST], empty[DA_NST];
  __shared__ float s_m[DA_WARPS][8], s_l[DA_WARPS][8];
  __shared__ uint32_t s_last;
  const AttnCtx cx{&tmK, &tmV, q, opart, mlpart, counters, out, Hq, Hkv, cap, L, S, units,
                   scale_log2, status, int(blockIdx.x), int(gridDim.x), align1024(smem_raw),
                   full, empty, s_m, s_l, &s_last};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    attn_init(cx);
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch_dependents();
  if (warp == DA_WARPS) {
    if (lane == 0) {
      int64_t ci;
      int i;
      attn_produce_pre(cx, ci, i);
      griddep_wait();
      attn_produce_rest(cx, ci, i);
    }
    return;
  }
  griddep_wait();   // q, the appended K / V rows and the counters are ready
  attn_consumers<1>(cx, warp, lane, threadIdx.x);
}

}  // namespace

namespace enigma {

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint64_t row_pitch_elems, uint32_t box_cols, uint32_t box_rows);

namespace {

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Launch with programmatic stream serialization: the kernel may start while its
// predecessor drains; every decode kernel waits (griddep_wait) before touching memory
// the predecessor writes or reads.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Split-K factor: about one (tile, split) CTA per SM, at least 2 k-blocks per split.
int pick_splits(int64_t N, int64_t K, int sms) {
  const int64_t tiles = (N + SK_BN - 1) / SK_BN;
  const int64_t kbs = (K + SK_BK - 1) / SK_BK;
  int64_t s = (int64_t(sms) + tiles - 1) / tiles;
  s = std::min<int64_t>(s, std::max<int64_t>(1, kbs / 2));
  return int(std::max<int64_t>(1, s));
}

struct Layout {
  size_t partial, xn, q, attn, h1, h1n, act, opart, mlpart, counters, total;
  int attn_splits;
};

Layout plan(const enigma_decode_layer_desc& d, int sms) {
  const int64_t B = d.batch, H = d.hidden, D = d.head_dim, Hq = d.heads_q, Hkv = d.heads_kv;
  const int64_t I = d.intermediate, Nqkv = (Hq + 2 * Hkv) * D;
  const int64_t L = d.position + 1;
  const int64_t gemms[4][2] = {{Nqkv, H}, {H, Hq * D}, {2 * I, H}, {H, I}};
  int64_t part = 0;
  for (auto& g : gemms) part = std::max(part, pick_splits(g[0], g[1], sms) * B * g[0]);
  Layout l;
  // Attention CTAs take 128-key chunks of one (sequence, kv head); the partial buffers
  // are sized for the cache capacity, so one workspace serves every position.
  const int64_t smax = (d.cache_capacity + DA_KEYS - 1) / DA_KEYS;
  l.attn_splits = int((L + DA_KEYS - 1) / DA_KEYS);
  const int64_t G = Hq / Hkv;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align256(off + bytes); return o; };
  l.partial = take(size_t(part) * 4);
  l.xn = take(size_t(B * H) * 2);
  l.q = take(size_t(B * Hq * D) * 2);
  l.attn = take(size_t(B * Hq * D) * 2);
  l.h1 = take(size_t(B * H) * 2);
  l.h1n = take(size_t(B * H) * 2);
  l.act = take(size_t(B * I) * 2);
  l.opart = take(size_t(B * Hkv * smax * G * D) * 4);
  l.mlpart = take(size_t(B * Hkv * smax * G * 2) * 4);
  l.counters = take(size_t(B * Hkv) * 4);
  l.total = off;
  return l;
}

cudaError_t splitk_gemm(const void* A, const void* Bw, float* partial, int64_t M, int64_t N,
                        int64_t K, int splits, uint32_t* status, cudaStream_t s) {
  CUtensorMap ta, tb;
  const int a_rows = int(std::min<int64_t>(SK_BM, (M + 7) / 8 * 8));
  if (!make_tmap_bf16_2d(&ta, A, M, K, K, SK_BK, uint32_t(a_rows)) ||
      !make_tmap_bf16_2d(&tb, Bw, K, N, N, SK_BN, SK_BK))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(gemm_splitk_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM);
  if (e != cudaSuccess) return e;
  const int kbs = int((K + SK_BK - 1) / SK_BK);
  const int per = (kbs + splits - 1) / splits;
  dim3 grid(unsigned((N + SK_BN - 1) / SK_BN), unsigned(splits));
  return launch_pdl(gemm_splitk_tc_kernel, grid, dim3(SK_THREADS), SK_SMEM, s, ta, tb, partial,
                    int(M), int(N), int(K), per, a_rows, status);
}

}  // namespace

// The whole step with an explicit SM count and status word (no per-device state used).
cudaError_t decode_layer_run(const enigma_decode_layer_desc& d, const void* x, void* out,
                             void* ws, int sms, uint32_t* status, cudaStream_t s) {
  const Layout l = plan(d, sms);
  uint8_t* w = static_cast<uint8_t*>(ws);
  float* part = reinterpret_cast<float*>(w + l.partial);
  auto bfp = [&](size_t o) { return reinterpret_cast<__nv_bfloat16*>(w + o); };
  const int B = int(d.batch), H = int(d.hidden), D = int(d.head_dim);
  const int Hq = int(d.heads_q), Hkv = int(d.heads_kv), I = int(d.intermediate);
  const int Nqkv = (Hq + 2 * Hkv) * D;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  cudaError_t e;
#define ENIGMA_TRY(expr)           \
  do {                             \
    e = (expr);                    \
    if (e != cudaSuccess) return e; \
  } while (0)
  // 1. input RMSNorm
  ENIGMA_TRY(rmsnorm_launch_sms(ENIGMA_DTYPE_BF16, x, d.w_in_norm, bfp(l.xn), B, H, d.eps, sms, s));
  // 2-3. QKV projection, RoPE, KV-cache append at `position`
  int sp = pick_splits(Nqkv, H, sms);
  ENIGMA_TRY(splitk_gemm(bfp(l.xn), d.w_qkv, part, B, Nqkv, H, sp, status, s));
  ENIGMA_TRY(launch_pdl(qkv_finalize_kernel, dim3(B, Hq + 2 * Hkv), dim3(32), 0, s,
                        static_cast<const float*>(part), sp, B, Nqkv, Hq, Hkv, d.rope_cos,
                        d.rope_sin, bfp(l.q), static_cast<__nv_bfloat16*>(d.k_cache),
                        static_cast<__nv_bfloat16*>(d.v_cache), int(d.cache_capacity),
                        int(d.position), reinterpret_cast<uint32_t*>(w + l.counters)));
  // 4. attention over position + 1 keys (split-KV, combined by each unit's last CTA)
  {
    CUtensorMap tk, tv;
    const uint64_t rows = uint64_t(B) * Hkv * uint64_t(d.cache_capacity);
    if (!make_tmap_bf16_2d(&tk, d.k_cache, rows, DA_D, DA_D, DA_D, DA_KEYS) ||
        !make_tmap_bf16_2d(&tv, d.v_cache, rows, DA_D, DA_D, DA_D, DA_KEYS))
      return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DA_SMEM);   // per device, cheap: set on every call
    if (e != cudaSuccess) return e;
    const int64_t chunks = int64_t(B) * Hkv * l.attn_splits;
    const int ctas = int(std::min<int64_t>(chunks, int64_t(sms) * DA_CTAS_PER_SM));
    ENIGMA_TRY(launch_pdl(decode_attn_kernel, dim3(ctas), dim3(DA_THREADS), DA_SMEM, s, tk, tv, static_cast<const __nv_bfloat16*>(bfp(l.q)),
                          reinterpret_cast<float*>(w + l.opart),
                          reinterpret_cast<float*>(w + l.mlpart),
                          reinterpret_cast<uint32_t*>(w + l.counters), bfp(l.attn), Hq, Hkv,
                          int(d.cache_capacity), int(d.position + 1), l.attn_splits, B * Hkv,
                          d.attn_scale * 1.4426950408889634f, status));
  }
  // 6-7. O projection + residual(x) -> h1, post-attention RMSNorm -> h1n
  sp = pick_splits(H, Hq * D, sms);
  ENIGMA_TRY(splitk_gemm(bfp(l.attn), d.w_o, part, B, H, Hq * D, sp, status, s));
  ENIGMA_TRY(launch_pdl(reduce_residual_norm_kernel, dim3(B), dim3(256), 0, s,
                        static_cast<const float*>(part), sp, B, H, xb, bfp(l.h1),
                        static_cast<const __nv_bfloat16*>(d.w_post_norm), bfp(l.h1n), d.eps));
  // 8-9. gate|up projection, SwiGLU
  sp = pick_splits(2 * I, H, sms);
  ENIGMA_TRY(splitk_gemm(bfp(l.h1n), d.w_gate_up, part, B, 2 * I, H, sp, status, s));
  ENIGMA_TRY(launch_pdl(swiglu_kernel, dim3(unsigned((int64_t(B) * I / 4 + 255) / 256)),
                        dim3(256), 0, s, static_cast<const float*>(part), sp, B, I, bfp(l.act)));
  // 10-11. down projection + residual(h1) -> out
  sp = pick_splits(H, I, sms);
  ENIGMA_TRY(splitk_gemm(bfp(l.act), d.w_down, part, B, H, I, sp, status, s));
  ENIGMA_TRY(launch_pdl(reduce_residual_norm_kernel, dim3(B), dim3(256), 0, s,
                        static_cast<const float*>(part), sp, B, H,
                        static_cast<const __nv_bfloat16*>(bfp(l.h1)),
                        static_cast<__nv_bfloat16*>(out),
                        static_cast<const __nv_bfloat16*>(nullptr),
                        static_cast<__nv_bfloat16*>(nullptr), 0.f));
#undef ENIGMA_TRY
  return cudaSuccess;
}

size_t decode_workspace_bytes(const enigma_decode_layer_desc& d) {
  return plan(d, sm_count()).total;
}

cudaError_t decode_layer_launch(const enigma_decode_layer_desc& d, const void* x, void* out,
                                void* ws, cudaStream_t s) {
  return decode_layer_run(d, x, out, ws, sm_count(), device_status(), s);
}

}  // namespace enigma

// ============================================================================ no-allocation entry
// Some callers cannot call cudaMalloc on the path that runs a decode step: a real-time
// serving loop that must not enter the allocator (which can synchronize or stall), a
// plugin inside another runtime that owns all device memory, or code running where an
// allocation failure is not allowed to happen mid-step.  enigma_decode_layer_bf16_noalloc
// serves them: it runs the same kernels as enigma_decode_layer_bf16, with the workspace
// in a fixed device array compiled into this library instead of caller memory.
//
// The array costs kNoAllocScratchBytes on every GPU that loads the library, until the
// process exits.  All calls share it and it keeps the previous call's contents: every
// byte a step reads from it is written earlier in the same step, so nothing needs
// clearing except the status word, which is zeroed at the start of each call.  Calls
// that overlap on the GPU (different streams, or different host threads on one device)
// race on the array; serialize them on one stream.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) uint32_t g_noalloc_status[64];

struct NoAllocDevice {
  bool ready = false;
  uint8_t* scratch = nullptr;   // device address of g_noalloc_scratch on this device
  uint32_t* status = nullptr;   // device address of g_noalloc_status on this device
  int sms = 0;
};
constexpr int kNoAllocMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: resolve the arrays' device addresses.  In
// host code the array names are host-side stand-ins, not device addresses; only the
// addresses returned by cudaGetSymbolAddress may be given to a kernel.
int32_t noalloc_setup(NoAllocDevice** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    enigma::set_error("decode noalloc: no current CUDA device (%s)", cudaGetErrorString(e));
    return ENIGMA_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      enigma::set_error("decode noalloc: cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
      return ENIGMA_ERR_DEVICE;
    }
    void* st = nullptr;
    e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess) {
      enigma::set_error("decode noalloc: cudaGetSymbolAddress(status) failed: %s", cudaGetErrorString(e));
      return ENIGMA_ERR_DEVICE;
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || sms <= 0) {
      enigma::set_error("decode noalloc: SM count query failed: %s", cudaGetErrorString(e));
      return ENIGMA_ERR_DEVICE;
    }
    d.scratch = static_cast<uint8_t*>(p);
    d.status = static_cast<uint32_t*>(st);
    d.sms = sms;
    d.ready = true;
  }
  *out = &d;
  return ENIGMA_OK;
}

}  // namespace

extern "C" int32_t enigma_decode_layer_bf16_noalloc(const enigma_decode_layer_desc* desc,
                                                    const void* x, void* out, void* stream) {
  int32_t rc = enigma::check_decode_desc(desc);
  if (rc != ENIGMA_OK) return rc;
  if (x == nullptr || out == nullptr || reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0) {
    enigma::set_error("bad argument: decode noalloc: x / out must be non-NULL and 16-byte aligned");
    return ENIGMA_ERR_BADARG;
  }
  NoAllocDevice* dev = nullptr;
  rc = noalloc_setup(&dev);
  if (rc != ENIGMA_OK) return rc;
  const size_t need = enigma::plan(*desc, dev->sms).total;
  if (need > kNoAllocScratchBytes) {
    enigma::set_error("bad argument: decode noalloc: this step needs %zu bytes of scratch, more than "
              "the fixed %zu-byte array of the no-allocation entry point; use "
              "enigma_decode_layer_bf16 with a caller-provided workspace",
              need, kNoAllocScratchBytes);
    return ENIGMA_ERR_BADARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(dev->status, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess)
    e = enigma::decode_layer_run(*desc, x, out, dev->scratch, dev->sms, dev->status, s);
  if (e != cudaSuccess) {
    enigma::set_error("decode noalloc launch failed: %s (%s)", cudaGetErrorName(e), cudaGetErrorString(e));
    return ENIGMA_ERR_LAUNCH;
  }
  return ENIGMA_OK;
}
