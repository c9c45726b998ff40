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
//   * Attention is split-KV ("flash decoding"): CTAs of (sequence, kv head,
//     key chunk) write (max, sum, o) partials for the group's query heads; a
//     combine kernel merges the chunks.
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
__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// q / k / v = sum over splits of the QKV partials; RoPE on the q and k heads
// (rotate-half pairing d <-> d + D/2 with full-length cos / sin tables, as in
// examples/qwen_megakernel.py:90-107); q to q_out [M, Hq, D], k and v appended
// at position `pos` of the caches [M, Hkv, S_cap, D].  One warp per (row, head),
// lane d owns dims d and d + 32 (D = 64).
__global__ void __launch_bounds__(32)
qkv_finalize_kernel(const float* __restrict__ part, int splits, int M, int N, int Hq, int Hkv,
                    const float* __restrict__ cosv, const float* __restrict__ sinv,
                    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kc,
                    __nv_bfloat16* __restrict__ vc, int s_cap, int pos) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int D = 64, H2 = 32;
  const int m = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
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

// d = a * b + c on two fp32 lanes at once (sm_100 packed FMA).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Split-KV decode attention on the tensor cores (mma.sync m16n8k16, bf16 -> fp32).
// CTA = (sequence b, kv head, key chunk); each of its 4 warps owns a contiguous quarter
// of the chunk and writes its own unnormalised partial (max, sum, o) for the G <= 8
// query heads of the group; the combine kernel merges all partials.
//
// Per 64-key block a warp computes S = Q K^T (Q = the group's heads as the 16-row A
// operand, rows >= G zero; K as the B operand straight from global memory), an online
// softmax in the log2 domain, and O += P V with P taken from the S accumulators and V
// staged through shared memory (cp.async, XOR-swizzled rows) and read by ldmatrix.trans.
// The head dimension is consumed in a permuted order: for k-step ks, lane quad t holds
// fragment columns {2t, 2t+1, 2t+8, 2t+9} = physical dims 16t + 4ks + {0..3}, applied to
// both Q and K (a dot product is order-free), so each lane reads its K row slice as two
// contiguous 16-byte loads.
//   q [B, Hq, D] bf16 (RoPE applied); kc / vc [B, Hkv, cap, D] bf16; L keys valid
//   opart [B*Hkv, parts, G, D] fp32, mlpart [B*Hkv, parts, G, 2] (max in log2 units, sum)
constexpr int DA_WARPS = 4;
constexpr int DA_BLOCK = 64;       // keys per inner step

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem), "l"(gmem) : "memory");
}

__global__ void __launch_bounds__(DA_WARPS * 32)
decode_attn_split_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                         const __nv_bfloat16* __restrict__ vc, float* __restrict__ opart,
                         float* __restrict__ mlpart, int Hq, int Hkv, int cap, int L, int chunk,
                         float scale_log2) {
  griddep_launch_dependents();
  __shared__ __align__(128) uint8_t sv[DA_WARPS][DA_BLOCK * DA_D * 2];   // 8 KB per warp
  const int G = Hq / Hkv;
  const int bhk = blockIdx.x, split = blockIdx.y;
  // The cached keys before the appended one are not written by the predecessor: pull
  // this CTA's K and V rows into L2 while it finishes (the new row is read after the wait).
  if (threadIdx.x == 0) {
    const int c0 = split * chunk, c1 = min(L - 1, c0 + chunk);
    if (c1 > c0) {
      const int64_t off = (int64_t(bhk) * cap + c0) * DA_D;
      bulk_prefetch_l2(kc + off, uint32_t(c1 - c0) * DA_D * 2);
      bulk_prefetch_l2(vc + off, uint32_t(c1 - c0) * DA_D * 2);
    }
  }
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int parts = gridDim.y * DA_WARPS, part = split * DA_WARPS + warp;
  const int b = bhk / Hkv, kvh = bhk % Hkv;
  const int g = lane >> 2, t = lane & 3;
  const int per_warp = (chunk + DA_WARPS - 1) / DA_WARPS;
  const int k0 = split * chunk + warp * per_warp;
  const int k1 = min(L, min(split * chunk + chunk, k0 + per_warp));

  // Q fragments (A operand): row g = head g of the group (rows >= G and rows 8..15 zero).
  uint32_t qa[4][4];
  {
    const bool live = g < G;
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        q + (int64_t(b) * Hq + kvh * G + (live ? g : 0)) * DA_D + 16 * t);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qa[ks][0] = live ? qrow[2 * ks] : 0u;
      qa[ks][2] = live ? qrow[2 * ks + 1] : 0u;
      qa[ks][1] = 0u;
      qa[ks][3] = 0u;
    }
  }
  const __nv_bfloat16* kbase = kc + int64_t(bhk) * cap * DA_D;
  const __nv_bfloat16* vbase = vc + int64_t(bhk) * cap * DA_D;
  const uint32_t sv_addr = smem_u32(sv[warp]);

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;   // row g, log2 units

  for (int kb = k0; kb < k1; kb += DA_BLOCK) {
    const int nk = min(DA_BLOCK, k1 - kb);
    // V block -> shared memory: row r (key), 16-byte chunk c stored at chunk c ^ (r & 7).
    __syncwarp();
#pragma unroll
    for (int i = 0; i < (DA_BLOCK * 8) / 32; ++i) {
      const int idx = i * 32 + lane, r = idx >> 3, c = idx & 7;
      const int key = kb + min(r, nk - 1);
      cp_async16(sv_addr + r * 128 + ((c ^ (r & 7)) << 4), vbase + int64_t(key) * DA_D + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");

    // S = Q K^T for 8 blocks of 8 keys; lane (g, t) loads key kb + 8 nb + g, dims 16t..16t+15.
    float sacc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int key = kb + min(nb * 8 + g, nk - 1);
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + int64_t(key) * DA_D + 16 * t);
      const uint4 lo = __ldg(kr), hi = __ldg(kr + 1);
      const uint32_t kw[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) mma_bf16_16816(sacc[nb], qa[ks], kw[2 * ks], kw[2 * ks + 1]);
    }
    // Online softmax on row g (columns 2t, 2t+1 of each 8-key block).
    float mx = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = nb * 8 + 2 * t + e < nk;
        sacc[nb][e] = ok ? sacc[nb][e] * scale_log2 : -INFINITY;
        mx = fmaxf(mx, sacc[nb][e]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float corr = ex2f(m_run - m_new);   // 0 on the first block (m_run = -inf)
    m_run = m_new;
    float psum = 0.f;
    uint32_t pa[8];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const float p0 = ex2f(sacc[nb][0] - m_new), p1 = ex2f(sacc[nb][1] - m_new);
      psum += p0 + p1;
      pa[nb] = pack_bf16x2(p0, p1);
    }
    l_run = l_run * corr + psum;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= corr;
      o[i][1] *= corr;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    // O += P V: k-step kk covers keys 16 kk .. 16 kk + 15 (S blocks 2 kk and 2 kk + 1).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pa[2 * kk], 0u, pa[2 * kk + 1], 0u};
#pragma unroll
      for (int nb2 = 0; nb2 < 4; ++nb2) {   // dims 16 nb2 .. 16 nb2 + 15 (two n-blocks)
        const int mi = lane >> 3, r = 16 * kk + (mi & 1) * 8 + (lane & 7);
        const int c = 2 * nb2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(sv_addr + r * 128 + ((c ^ (r & 7)) << 4), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * nb2], a, b0, b1);
        mma_bf16_16816(o[2 * nb2 + 1], a, b2, b3);
      }
    }
  }
  // Row sums: each lane holds 16 of the block's 64 columns per step.
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (g < G) {
    const int64_t base = (int64_t(bhk) * parts + part) * G + g;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<float2*>(opart + base * DA_D + 8 * i + 2 * t) = make_float2(o[i][0], o[i][1]);
    if (t == 0) {
      mlpart[base * 2] = m_run;
      mlpart[base * 2 + 1] = l_run;
    }
  }
}

// out[b, h*D + d] = sum_s 2^(m_s - M) o_s[d] / sum_s 2^(m_s - M) l_s  (bf16).
// One CTA of 64 threads per (b, h): the first warp reduces the partials' maxima and sums
// (lane s owns partial s, parts <= 64), the weights go to shared memory, then every
// thread sums its dim over the partials with independent loads.
__global__ void __launch_bounds__(DA_D)
decode_attn_combine_kernel(const float* __restrict__ opart, const float* __restrict__ mlpart,
                           __nv_bfloat16* __restrict__ out, int Hq, int Hkv, int nparts) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ float wgt[64];
  __shared__ float inv_den;
  const int G = Hq / Hkv;
  const int bh = blockIdx.x;            // b * Hq + h
  const int b = bh / Hq, h = bh % Hq;
  const int bhk = b * Hkv + h / G, g = h % G;
  const int tid = threadIdx.x;
  if (tid < 32) {
    float m[2], l[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int s = tid + 32 * k;
      const int64_t i = (int64_t(bhk) * nparts + s) * G + g;
      m[k] = s < nparts ? mlpart[i * 2] : -INFINITY;
      l[k] = s < nparts ? mlpart[i * 2 + 1] : 0.f;
    }
    float M = fmaxf(m[0], m[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float den = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float w = (m[k] == -INFINITY) ? 0.f : ex2f(m[k] - M);
      wgt[tid + 32 * k] = w;
      den = fmaf(w, l[k], den);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (tid == 0) inv_den = den > 0.f ? 1.0f / den : 0.f;
  }
  __syncthreads();
  const float* op = opart + (int64_t(bhk) * nparts * G + g) * DA_D + tid;
  float num = 0.f;
#pragma unroll 4
  for (int s = 0; s < nparts; ++s) num = fmaf(wgt[s], __ldg(op + int64_t(s) * G * DA_D), num);
  out[int64_t(bh) * DA_D + tid] = __float2bfloat16_rn(num * inv_den);
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
  size_t partial, xn, q, attn, h1, h1n, act, opart, mlpart, total;
  int attn_splits, attn_chunk;
};

Layout plan(const enigma_decode_layer_desc& d, int sms) {
  const int64_t B = d.batch, H = d.hidden, D = d.head_dim, Hq = d.heads_q, Hkv = d.heads_kv;
  const int64_t I = d.intermediate, Nqkv = (Hq + 2 * Hkv) * D;
  const int64_t L = d.position + 1;
  const int64_t gemms[4][2] = {{Nqkv, H}, {H, Hq * D}, {2 * I, H}, {H, I}};
  int64_t part = 0;
  for (auto& g : gemms) part = std::max(part, pick_splits(g[0], g[1], sms) * B * g[0]);
  Layout l;
  // Split the keys so (sequence, kv head, chunk) CTAs cover ~4 per SM, at most 16 chunks
  // (4 warp partials each; the combine kernel takes up to 64 partials).  The workspace is
  // sized for that maximum, so one workspace serves every position.
  const int64_t splits = std::min<int64_t>(
      16, std::max<int64_t>(1, (4 * int64_t(sms) + B * Hkv - 1) / (B * Hkv)));
  const int64_t chunk = (L + splits - 1) / splits;
  l.attn_splits = int((L + chunk - 1) / chunk);
  l.attn_chunk = int(chunk);
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
  l.opart = take(size_t(B * Hkv * splits * DA_WARPS * G * D) * 4);
  l.mlpart = take(size_t(B * Hkv * splits * DA_WARPS * G * 2) * 4);
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
                        int(d.position)));
  // 4-5. attention over position + 1 keys, split-KV then combine
  ENIGMA_TRY(launch_pdl(decode_attn_split_kernel, dim3(B * Hkv, l.attn_splits),
                        dim3(DA_WARPS * 32), 0, s, static_cast<const __nv_bfloat16*>(bfp(l.q)),
                        static_cast<const __nv_bfloat16*>(d.k_cache),
                        static_cast<const __nv_bfloat16*>(d.v_cache),
                        reinterpret_cast<float*>(w + l.opart),
                        reinterpret_cast<float*>(w + l.mlpart), Hq, Hkv, int(d.cache_capacity),
                        int(d.position + 1), l.attn_chunk, d.attn_scale * 1.4426950408889634f));
  ENIGMA_TRY(launch_pdl(decode_attn_combine_kernel, dim3(B * Hq), dim3(DA_D), 0, s,
                        static_cast<const float*>(reinterpret_cast<float*>(w + l.opart)),
                        static_cast<const float*>(reinterpret_cast<float*>(w + l.mlpart)),
                        bfp(l.attn), Hq, Hkv, l.attn_splits * DA_WARPS));
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
