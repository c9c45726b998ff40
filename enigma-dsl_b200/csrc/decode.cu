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

namespace {

using namespace enigma_sm100;

// ============================================================================ split-K GEMM
constexpr int SK_BM = 128;
constexpr int SK_BN = 64;
constexpr int SK_BK = 64;
constexpr int SK_STAGES = 4;
constexpr int SK_A_BYTES = SK_BM * SK_BK * 2;   // 16 KB
constexpr int SK_B_BYTES = SK_BK * SK_BN * 2;   // 8 KB
constexpr int SK_STAGE = SK_A_BYTES + SK_B_BYTES;
constexpr int SK_SMEM = SK_STAGES * SK_STAGE + 1024 + 256;
constexpr int SK_THREADS = 192;

// partial[split][m][n] (fp32) = A[m, kslice] * B[kslice, n] for one 128 x 64 tile.
// M <= 128 (rows past M are zero-filled by TMA and not stored).
__global__ void __launch_bounds__(SK_THREADS)
gemm_splitk_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      float* __restrict__ partial, int M, int N, int K, int kb_per_split,
                      int a_rows, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + SK_STAGES * SK_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SK_STAGES * SK_STAGE);
  uint64_t* empty = full + SK_STAGES;
  uint64_t* acc_full = empty + SK_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = blockIdx.x, split = blockIdx.y;
  const int num_kb = (K + SK_BK - 1) / SK_BK;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(num_kb, kb0 + kb_per_split);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < SK_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, SK_BN);
    tmem_relinquish();
  }
  // The TMA box covers the a_rows (= M rounded up to 8) real rows of A; the MMA reads 128.
  // Rows a_rows..127 of every A stage are zeroed once here (128-byte rows, swizzle only
  // permutes 16-byte chunks within a row, so whole rows stay zero) and never written again.
  if (a_rows < SK_BM) {
    for (int i = threadIdx.x; i < SK_STAGES * (SK_BM - a_rows) * 8; i += SK_THREADS) {
      const int st = i / ((SK_BM - a_rows) * 8), rem = i % ((SK_BM - a_rows) * 8);
      reinterpret_cast<uint4*>(sA + st * SK_A_BYTES + a_rows * 128)[rem] = make_uint4(0, 0, 0, 0);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // B (weights) never depends on the previous kernel: the first stages' B tiles go to
  // shared memory and the rest of this CTA's slice to L2 before waiting on the
  // predecessor, so the weight stream overlaps its tail.
  const int pre = min(SK_STAGES, max(0, kb1 - kb0));
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], a_rows * SK_BK * 2 + SK_B_BYTES);
      tma_load_2d(sB + i * SK_B_BYTES, &tmB, &full[i], nb * SK_BN, (kb0 + i) * SK_BK);
    }
    for (int kb = kb0 + pre; kb < kb1; ++kb) tma_prefetch_l2_2d(&tmB, nb * SK_BN, kb * SK_BK);
  }
  griddep_wait();  // A (the previous kernel's output) and the partial buffer are ready / free

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sA + i * SK_A_BYTES, &tmA, &full[i], (kb0 + i) * SK_BK, 0);
      for (int kb = kb0 + pre, i = pre; kb < kb1; ++kb, ++i) {
        const int s = i % SK_STAGES;
        if (!mbar_wait(&empty[s], ((i / SK_STAGES) & 1) ^ 1, status)) break;
        mbar_arrive_expect_tx(&full[s], a_rows * SK_BK * 2 + SK_B_BYTES);
        tma_load_2d(sA + s * SK_A_BYTES, &tmA, &full[s], kb * SK_BK, 0);
        tma_load_2d(sB + s * SK_B_BYTES, &tmB, &full[s], nb * SK_BN, kb * SK_BK);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(SK_BM, SK_BN, false, true);
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      bool ok = true;
      for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
        const int s = i % SK_STAGES;
        if (!mbar_wait(&full[s], (i / SK_STAGES) & 1, status)) { ok = false; break; }
        tc_fence_after();
        const uint64_t da = smem_desc_sw128(a0 + s * SK_A_BYTES, 16, 1024);
        const uint64_t db = smem_desc_sw128(b0 + s * SK_B_BYTES, SK_B_BYTES, 1024);
#pragma unroll
        for (int kk = 0; kk < SK_BK / 16; ++kk)
          mma_bf16_ss(tmem, da + uint64_t((kk * 32) >> 4), db + uint64_t((kk * 2048) >> 4), idesc,
                      (i | kk) != 0 ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(acc_full);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool have = kb1 > kb0;
    if (!have || mbar_wait(acc_full, 0, status)) {
      tc_fence_after();
      float* dst = partial + (int64_t(split) * M + row) * N + nb * SK_BN;
      const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < SK_BN; c += 16) {
        uint32_t r[16];
        if (have) {
          tmem_ld16(taddr + c, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) r[t] = 0u;
        }
        if (row < M && nb * SK_BN + c < N) {
          float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SK_BN);
  }
}

// ============================================================================ reductions
// q / k / v = sum over splits of the QKV partials; RoPE on the q and k heads
// (rotate-half pairing d <-> d + D/2 with full-length cos / sin tables, as in
// examples/qwen_megakernel.py:90-107); q to q_out [M, Hq, D], k and v appended
// at position `pos` of the caches [M, Hkv, S_cap, D].  One warp per (row, head),
// lane d owns dims d and d + 32 (D = 64).
__global__ void __launch_bounds__(32)
qkv_finalize_kernel(const float* __restrict__ part, int splits, int M, int N, int Hq, int Hkv,
                    const float* __restrict__ cosv, const float* __restrict__ sinv,
                    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kc,
                    __nv_bfloat16* __restrict__ vc, int s_cap, int pos,
                    uint32_t* __restrict__ attn_counters) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int D = 64, H2 = 32;
  const int m = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  // The attention kernel's per-(sequence, kv head) completion counters start at zero.
  if (head >= Hq && head < Hq + Hkv && d == 0) attn_counters[m * Hkv + head - Hq] = 0u;
  const int c = head * D + d;
  float lo = 0.f, hi = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float* p = part + (int64_t(s) * M + m) * N;
    lo += p[c];
    hi += p[c + H2];
  }
  if (head < Hq + Hkv) {
    const float l2 = lo * cosv[d] - hi * sinv[d];
    const float h2 = hi * cosv[d + H2] + lo * sinv[d + H2];
    lo = l2;
    hi = h2;
  }
  __nv_bfloat16* dst;
  if (head < Hq) {
    dst = q_out + (int64_t(m) * Hq + head) * D;
  } else {
    const int kvh = head < Hq + Hkv ? head - Hq : head - Hq - Hkv;
    __nv_bfloat16* cache = head < Hq + Hkv ? kc : vc;
    dst = cache + ((int64_t(m) * Hkv + kvh) * s_cap + pos) * D;
  }
  dst[d] = __float2bfloat16_rn(lo);
  dst[d + H2] = __float2bfloat16_rn(hi);
}

// h = sum_s partial + residual (fp32), written as bf16 to h_out when given; then
// y = rmsnorm(h) * w when y_out is given.  One CTA (256 threads) per row, each thread
// four adjacent columns (float4 partial loads, all splits in flight); N % 4 == 0, N <= 2048.
__global__ void __launch_bounds__(256)
reduce_residual_norm_kernel(const float* __restrict__ part, int splits, int M, int N,
                            const __nv_bfloat16* __restrict__ residual,
                            __nv_bfloat16* __restrict__ h_out, const __nv_bfloat16* __restrict__ w,
                            __nv_bfloat16* __restrict__ y_out, float eps) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int kPer = 2;  // float4 groups per thread: 256 * 2 * 4 = 2048 columns
  __shared__ float red[8];
  const int m = blockIdx.x;
  float4 h[kPer];
  float ss = 0.f;
#pragma unroll
  for (int t = 0; t < kPer; ++t) {
    const int n = (threadIdx.x + t * 256) * 4;
    h[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n < N) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (residual) {
        const uint2 r = *reinterpret_cast<const uint2*>(residual + int64_t(m) * N + n);
        acc = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u),
                          __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xFFFF0000u));
      }
#pragma unroll 4
      for (int s = 0; s < splits; ++s) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(part + (int64_t(s) * M + m) * N + n));
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      h[t] = acc;
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      if (h_out)
        *reinterpret_cast<uint2*>(h_out + int64_t(m) * N + n) =
            make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
    }
  }
  if (y_out == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += red[i];
  const float r = 1.0f / sqrtf(total / float(N) + eps);
#pragma unroll
  for (int t = 0; t < kPer; ++t) {
    const int n = (threadIdx.x + t * 256) * 4;
    if (n < N) {
      const uint2 wv = *reinterpret_cast<const uint2*>(w + n);
      *reinterpret_cast<uint2*>(y_out + int64_t(m) * N + n) = make_uint2(
          pack_bf16x2(h[t].x * r * __uint_as_float(wv.x << 16),
                      h[t].y * r * __uint_as_float(wv.x & 0xFFFF0000u)),
          pack_bf16x2(h[t].z * r * __uint_as_float(wv.y << 16),
                      h[t].w * r * __uint_as_float(wv.y & 0xFFFF0000u)));
    }
  }
}

// act[m, j] = silu(g) * u with g = column j and u = column j + I of the summed
// gate|up partials (N = 2 I); silu(g) = g / (1 + e^-g) (qwen_megakernel.py:212-216).
// Four columns per thread; I % 4 == 0.
__global__ void __launch_bounds__(256)
swiglu_kernel(const float* __restrict__ part, int splits, int M, int I,
              __nv_bfloat16* __restrict__ act) {
  griddep_launch_dependents();
  griddep_wait();
  const int64_t q = int64_t(blockIdx.x) * 256 + threadIdx.x;  // float4 group index
  if (q * 4 >= int64_t(M) * I) return;
  const int m = int(q * 4 / I), j = int(q * 4 % I);
  float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
  for (int s = 0; s < splits; ++s) {
    const float* p = part + (int64_t(s) * M + m) * (2 * I);
    const float4 a = __ldg(reinterpret_cast<const float4*>(p + j));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p + j + I));
    g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
    u.x += b.x; u.y += b.y; u.z += b.z; u.w += b.w;
  }
  auto sw = [](float gg, float uu) { return gg / (1.0f + __expf(-gg)) * uu; };
  *reinterpret_cast<uint2*>(act + q * 4) = make_uint2(pack_bf16x2(sw(g.x, u.x), sw(g.y, u.y)),
                                                     pack_bf16x2(sw(g.z, u.z), sw(g.w, u.w)));
}

// ============================================================================ decode attention
constexpr int DA_D = 64;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Split-KV decode attention on the tensor cores (mma.sync m16n8k16, bf16 -> fp32), as a
// persistent kernel.  The work is the flattened list of (unit = sequence b x kv head,
// 128-key chunk) pairs; CTA c of P takes the contiguous range [c T / P, (c + 1) T / P),
// so every SM streams the same number of chunks whatever the batch and head counts.
//   * Warp 4 is the producer: one TMA box of K and one of V per chunk (128 rows x 128 B,
//     128-byte swizzle) into a DA_NST-stage ring.  The first chunks, if they do not hold
//     the key appended by the predecessor, are requested before the programmatic wait.
//   * Warps 0..3 each take 32 keys of every chunk:
//       S = Q K^T  (Q = the group's G <= 8 heads as the 16-row A operand, rows >= G zero;
//                  K from shared memory by ldmatrix),
//       online softmax in the log2 domain over the chunks of one unit,
//       O += P V   (V by ldmatrix.trans).
//   * At the end of a unit's run of chunks (a "segment") the warps merge in shared memory
//     into one (m, l, O) partial stored in the slot of the segment's first chunk; the other
//     slots of the segment are marked empty (m = -inf).  A device-scope counter per unit
//     (zeroed by the QKV finalize kernel of the same step) counts finished chunks; the CTA
//     that completes the count merges the unit's partials and writes the bf16 output.
//   q [B, Hq, D] bf16 (RoPE applied); K / V cache maps over [B*Hkv*cap, D] bf16; L keys
//   opart [B*Hkv, S, G, D] fp32, mlpart [B*Hkv, S, G, 2] (max in log2 units, sum)
//   out [B, Hq, D] bf16
constexpr int DA_KEYS = 128;
constexpr int DA_WARPS = 4;                        // consumer warps
constexpr int DA_THREADS = (DA_WARPS + 1) * 32;    // + the producer warp
constexpr int DA_NST = 3;
constexpr int DA_TILE = DA_KEYS * DA_D * 2;        // 16 KB: one of K or V
constexpr int DA_STAGE = 2 * DA_TILE;
constexpr int DA_MERGE = DA_WARPS * 8 * DA_D * 4;  // 8 KB: warp partials, then the weights
constexpr int DA_SMEM = DA_NST * DA_STAGE + DA_MERGE + 1024;
constexpr int DA_CTAS_PER_SM = 2;

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a2,
                                               uint32_t b0, uint32_t b1) {
  // A rows 8..15 (registers a1, a3) are zero: the group has at most 8 query heads.
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile (1024-aligned base).
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Named barrier over the consumer warps only (the producer never joins it).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(DA_WARPS * 32) : "memory");
}

__global__ void __launch_bounds__(DA_THREADS)
decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __nv_bfloat16* __restrict__ q, float* __restrict__ opart,
                   float* __restrict__ mlpart, uint32_t* __restrict__ counters,
                   __nv_bfloat16* __restrict__ out, int Hq, int Hkv, int cap, int L, int S,
                   int units, float scale_log2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_o = reinterpret_cast<float*>(stages + DA_NST * DA_STAGE);   // [warp][8][D]
  __shared__ uint64_t full[DA_NST], empty[DA_NST];
  __shared__ float s_m[DA_WARPS][8], s_l[DA_WARPS][8];
  __shared__ uint32_t s_last;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_chunks = int64_t(S) * units;
  const int64_t c_begin = n_chunks * blockIdx.x / gridDim.x;
  const int64_t c_end = n_chunks * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int s = 0; s < DA_NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], DA_WARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == DA_WARPS) {                       // ---------------- producer
    if (lane == 0) {
      auto issue = [&](int64_t ci, int st) {
        const int32_t row = int32_t((ci / S) * cap + (ci % S) * DA_KEYS);
        uint8_t* dst = stages + st * DA_STAGE;
        mbar_arrive_expect_tx(&full[st], DA_STAGE);
        tma_load_2d(dst, &tmK, &full[st], 0, row);
        tma_load_2d(dst + DA_TILE, &tmV, &full[st], 0, row);
      };
      // Before the wait: the first stages, stopping at the first chunk that holds an
      // appended key (the last of a unit).  (An L2 prefetch of the rest of the range was
      // measured 1.7 us slower: it queues the ring's demand loads behind 67 MB of prefetch.)
      int64_t ci = c_begin;
      int i = 0;
      for (; ci < c_end && i < DA_NST && ci % S != S - 1; ++ci, ++i) issue(ci, i);
      griddep_wait();
      for (; ci < c_end; ++ci, ++i) {
        const int st = i % DA_NST;
        if (!mbar_wait(&empty[st], ((i / DA_NST) & 1) ^ 1, status)) break;
        issue(ci, st);
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  griddep_wait();   // q, the appended K / V rows and the counters are ready
  const int g = lane >> 2, t = lane & 3, kw = warp * 32;
  const uint32_t stage0 = smem_u32(stages);
  uint32_t qa[4][2];
  float o[8][4];
  float m_run = -INFINITY, l_run = 0.f;
  int64_t cur_unit = -1;
  int seg_first = 0;
  for (int64_t ci = c_begin, i = 0; ci < c_end; ++ci, ++i) {
    const int64_t unit = ci / S;
    const int j = int(ci % S);
    if (unit != cur_unit) {
      // Q fragments: a0 = dims 16 ks + 2t, +1 and a2 = dims 16 ks + 8 + 2t, +1 of head g.
      const bool live = g < G;
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          q + ((unit / Hkv) * Hq + (unit % Hkv) * G + (live ? g : 0)) * DA_D);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qa[ks][0] = live ? qrow[8 * ks + t] : 0u;
        qa[ks][1] = live ? qrow[8 * ks + 4 + t] : 0u;
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m_run = -INFINITY;
      l_run = 0.f;
      cur_unit = unit;
      seg_first = j;
    }
    const int st = int(i % DA_NST);
    if (!mbar_wait(&full[st], uint32_t((i / DA_NST) & 1), status)) return;
    const uint32_t kaddr = stage0 + st * DA_STAGE, vaddr = kaddr + DA_TILE;
    const int nk = min(DA_KEYS, L - j * DA_KEYS);
    const bool ragged = nk < kw + 32;
    if (ragged) {
      // Rows past the last key may hold anything (other units, unwritten cache slots):
      // zero this warp's V rows there so that P = 0 never meets a NaN.
      uint8_t* vt = stages + st * DA_STAGE + DA_TILE;
      for (int idx = lane; idx < 32 * 8; idx += 32) {
        const int r = kw + (idx >> 3);
        if (r >= nk) reinterpret_cast<uint4*>(vt + r * 128)[idx & 7] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // S for the warp's 4 blocks of 8 keys.
    float sacc[4][4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
      const int r = kw + nb * 8 + (lane & 7);
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {     // k-steps 2 kp and 2 kp + 1
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kaddr + sw128(r, 4 * kp + (lane >> 3)), b0, b1, b2, b3);
        mma_bf16_16816(sacc[nb], qa[2 * kp][0], qa[2 * kp][1], b0, b1);
        mma_bf16_16816(sacc[nb], qa[2 * kp + 1][0], qa[2 * kp + 1][1], b2, b3);
      }
    }
    // Online softmax of row g (lane holds keys kw + 8 nb + 2t + e).
    float mx = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = kw + nb * 8 + 2 * t + e < nk;
        sacc[nb][e] = ok ? sacc[nb][e] * scale_log2 : -INFINITY;
        mx = fmaxf(mx, sacc[nb][e]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float mref = m_new == -INFINITY ? 0.f : m_new;   // nothing seen yet: all p = 0
    const float corr = ex2f(m_run - mref);                  // 0 while m_run = -inf
    m_run = m_new;
    float psum = 0.f;
    uint32_t pa[4];
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const float p0 = ex2f(sacc[nb][0] - mref), p1 = ex2f(sacc[nb][1] - mref);
      psum += p0 + p1;
      pa[nb] = pack_bf16x2(p0, p1);
    }
    l_run = fmaf(l_run, corr, psum);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] *= corr;
      o[n][1] *= corr;
    }
    // O += P V over the warp's 32 keys (k-steps of 16), 8 blocks of 8 dims.
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int mi = lane >> 3, r = kw + 16 * kk + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int nb2 = 0; nb2 < 4; ++nb2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(vaddr + sw128(r, 2 * nb2 + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * nb2], pa[2 * kk], pa[2 * kk + 1], b0, b1);
        mma_bf16_16816(o[2 * nb2 + 1], pa[2 * kk], pa[2 * kk + 1], b2, b3);
      }
    }
    // Release the stage (the zeroing writes were generic-proxy: order them before the
    // next TMA write into the same bytes).
    if (ragged) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);

    if (ci + 1 != c_end && j + 1 != S) continue;
    // ------------------------------------------------ end of this unit's segment
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (g < G) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
        *reinterpret_cast<float2*>(s_o + (warp * 8 + g) * DA_D + 8 * n + 2 * t) =
            make_float2(o[n][0], o[n][1]);
      if (t == 0) {
        s_m[warp][g] = m_run;
        s_l[warp][g] = l_run;
      }
    }
    consumers_sync();
    const int64_t pbase = (unit * S + seg_first) * G;
    for (int idx = threadIdx.x; idx < G * (DA_D / 4); idx += DA_WARPS * 32) {
      const int gg = idx / (DA_D / 4), d = (idx % (DA_D / 4)) * 4;
      float M = s_m[0][gg];                      // warp 0 always holds a valid key
#pragma unroll
      for (int w = 1; w < DA_WARPS; ++w) M = fmaxf(M, s_m[w][gg]);
      float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
      float den = 0.f;
#pragma unroll
      for (int w = 0; w < DA_WARPS; ++w) {
        const float wt = s_m[w][gg] == -INFINITY ? 0.f : ex2f(s_m[w][gg] - M);
        const float4 v = *reinterpret_cast<const float4*>(s_o + (w * 8 + gg) * DA_D + d);
        num.x = fmaf(wt, v.x, num.x);
        num.y = fmaf(wt, v.y, num.y);
        num.z = fmaf(wt, v.z, num.z);
        num.w = fmaf(wt, v.w, num.w);
        den = fmaf(wt, s_l[w][gg], den);
      }
      *reinterpret_cast<float4*>(opart + (pbase + gg) * DA_D + d) = num;
      if (d == 0) *reinterpret_cast<float2*>(mlpart + (pbase + gg) * 2) = make_float2(M, den);
    }
    __threadfence();
    consumers_sync();
    if (threadIdx.x == 0) {
      const uint32_t n = uint32_t(j - seg_first + 1);
      s_last = atomicAdd(&counters[unit], n) + n == uint32_t(S) ? 1u : 0u;
    }
    consumers_sync();
    if (s_last) {
      // This CTA completed the unit.  Its partials sit in the slots of its segments' first
      // chunks: chunk 0 of the unit and every CTA range start inside the unit.
      __threadfence();
      const int64_t u0 = unit * S, P = gridDim.x;
      int64_t c0 = u0 * P / n_chunks;            // the CTA whose range holds chunk u0
      while (c0 + 1 < P && n_chunks * (c0 + 1) / P <= u0) ++c0;
      while (c0 > 0 && n_chunks * c0 / P > u0) --c0;
      const int64_t b = unit / Hkv, kvh = unit % Hkv;
      for (int idx = threadIdx.x; idx < G * (DA_D / 4); idx += DA_WARPS * 32) {
        const int gg = idx / (DA_D / 4), d = (idx % (DA_D / 4)) * 4;
        float M = -INFINITY, den = 0.f;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t c = c0; c < P; c += 4) {
          // Up to 4 segments per batch, all loads in flight, then an online merge.
          float2 ml[4];
          float4 ov[4];
          bool live[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int64_t start = c + k == c0 ? u0 : n_chunks * (c + k) / P;
            live[k] = c + k < P && start < u0 + S && start >= u0;
            const int64_t i = (live[k] ? start : u0) * G + gg;
            ml[k] = __ldcg(reinterpret_cast<const float2*>(mlpart + i * 2));
            ov[k] = __ldcg(reinterpret_cast<const float4*>(opart + i * DA_D + d));
          }
          float Mb = M;
#pragma unroll
          for (int k = 0; k < 4; ++k) if (live[k]) Mb = fmaxf(Mb, ml[k].x);
          const float corr = ex2f(M - Mb);        // 0 on the first batch (M = -inf)
          num.x *= corr; num.y *= corr; num.z *= corr; num.w *= corr;
          den *= corr;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (!live[k]) continue;
            const float w = ex2f(ml[k].x - Mb);
            num.x = fmaf(w, ov[k].x, num.x);
            num.y = fmaf(w, ov[k].y, num.y);
            num.z = fmaf(w, ov[k].z, num.z);
            num.w = fmaf(w, ov[k].w, num.w);
            den = fmaf(w, ml[k].y, den);
          }
          M = Mb;
          if (!live[3]) break;
        }
        const float inv = 1.0f / den;
        *reinterpret_cast<uint2*>(out + (b * Hq + kvh * G + gg) * DA_D + d) =
            make_uint2(pack_bf16x2(num.x * inv, num.y * inv), pack_bf16x2(num.z * inv, num.w * inv));
      }
    }
    consumers_sync();   // the merge area is free again
  }
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
