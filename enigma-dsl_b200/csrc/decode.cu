// decode.cu — one decoder-layer decode step (Qwen-style) on sm_100a.
//
// The reference runs the layer as one threadgroup-wide Metal megakernel
// (examples/qwen_megakernel.py:228-269: RMSNorm -> Q/K/V matvec -> RoPE ->
// SDPA over the KV cache -> O-proj + residual -> RMSNorm -> SwiGLU -> down-proj
// + residual).  At batch 64 every GEMM is skinny (M = 64) and the step is bound
// by HBM: ~30 MB of weights and ~67 MB of KV cache per step.  So:
//
//   * Each GEMM is one cluster launch: grid (N/64 tiles, cs) with cluster (1, cs), the
//     cs CTAs of a cluster split the tile's k-blocks, accumulate in TMEM and sum their
//     partial tiles over distributed shared memory, so the whole grid fills the 148 SMs
//     even for N = 896 and no partial goes through global memory.
//   * What follows each GEMM runs in its epilogue: RoPE + KV-cache append (QKV),
//     residual add + the post-attention RMSNorm's weight and row sums of squares
//     (O-proj), the RMSNorm factor + SwiGLU (gate/up), residual add (down-proj).
//   * Attention is split-KV ("flash decoding") in one persistent kernel: CTAs stream
//     balanced ranges of (sequence x kv head, 128-key chunk) pairs through a TMA ring,
//     and the CTA that finishes a (sequence, kv head) merges its partials.
//
// Workspace (caller-owned, enigma_decode_workspace_bytes) holds every intermediate and the
// attention partials, so a step makes no allocation.
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

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ============================================================================ cluster split-K
// One GEMM of the step with its epilogue in a single launch.  Grid (tiles, cs) with cluster
// dims (1, cs, 1): the cs CTAs of a cluster share one output tile (64 columns, or 64 gate +
// 64 up columns) and split its k-blocks evenly.  Each CTA accumulates its K range in TMEM,
// drains it into its own shared memory (the drained ring), and after a cluster barrier CTA r
// sums rows [r R, (r + 1) R) of all cs partials over distributed shared memory, in rank
// order (deterministic), and applies the epilogue to them.  No partials go through global
// memory and no separate reduction kernel runs.
enum : int { EPI_QKV = 0, EPI_OPROJ = 1, EPI_GATEUP = 2, EPI_DOWN = 3 };

struct EpiArgs {
  int M;                                // rows (batch)
  // EPI_QKV: RoPE on q / k heads, q to q_out, k / v appended at `pos`, counters zeroed
  int Hq, Hkv, s_cap, pos;
  const float* cosv;
  const float* sinv;
  __nv_bfloat16* q_out;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  uint32_t* counters;
  // EPI_OPROJ: h = acc + residual -> h_out; h * w_norm -> hw_out; row sums of h^2 of this
  // tile -> ssq[tile][m].  EPI_DOWN: acc + residual -> h_out.
  int ld;                               // row pitch of residual / h_out / hw_out (hidden)
  const __nv_bfloat16* residual;
  __nv_bfloat16* h_out;
  const __nv_bfloat16* w_norm;
  __nv_bfloat16* hw_out;
  float* ssq;                           // [tiles][128]
  // EPI_GATEUP: r = 1 / sqrt(sum_t ssq[t][m] / ld + eps) (s_rs); act = silu(r g) * (r u)
  int I, ssq_tiles;
  float eps;
  __nv_bfloat16* act;
};

constexpr int CK_THREADS = 192;
constexpr int CK_MAX_CLUSTER = 16;   // non-portable cluster size (opted in at launch)

// Shared memory: `stages` A slots of AR rows (AR = 64 when M <= 64, else 128), `stages` B
// slots, then the receive area.  The MMA always reads 128 A rows; with AR = 64 rows 64..127
// of a slot are the next slot's (or B slot 0's) bytes, which only feed accumulator rows
// >= M, never stored.  So a 64-row slot halves the A bytes per stage.
// The receive area holds, for this CTA's R = ceil(M / cs) rows of the tile, the partial of
// every CTA of the cluster: [cs][R][PSTRIDE] fp32.
constexpr int CK_MAX_STAGES = 12;

template <int NB, int AR>
struct CkShape {
  static constexpr int A_BYTES = AR * SK_BK * 2;                     // 8 or 16 KB
  static constexpr int B_BYTES = NB * SK_BK * 64 * 2;                // 8 KB per 64 columns
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int PSTRIDE = NB * 64 + 4;                        // floats per partial row
  static_assert(AR == 128 || B_BYTES >= 8192, "rows 64..127 of the last A slot must be in the ring");
};

// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to a (possibly remote)
// CTA's shared memory of the cluster, counted on that CTA's mbarrier `mbar` when it lands.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst, uint32_t src, uint32_t bytes,
                                                     uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "r"(src), "r"(bytes), "r"(mbar) : "memory");
}
__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float a, float b, float c, float d) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
}

// Global inputs of one item's epilogue, loaded before the accumulator is complete.
struct EpiIn {
  float4 c0, c1, s0, s1;     // QKV: cos / sin at d.. and d + 32..
  uint2 r, w;                // O-proj / down: residual; O-proj: norm weight
};

template <int EPI>
__device__ __forceinline__ EpiIn ck_prefetch(const EpiArgs& e, int tile, int m, int g, bool valid) {
  EpiIn in;
  if constexpr (EPI == EPI_QKV) {
    if (valid && g < 8 && tile < e.Hq + e.Hkv) {
      const int d = 4 * g;
      in.c0 = *reinterpret_cast<const float4*>(e.cosv + d);
      in.c1 = *reinterpret_cast<const float4*>(e.cosv + d + 32);
      in.s0 = *reinterpret_cast<const float4*>(e.sinv + d);
      in.s1 = *reinterpret_cast<const float4*>(e.sinv + d + 32);
    }
  } else if constexpr (EPI == EPI_OPROJ || EPI == EPI_DOWN) {
    if (valid) {
      const int col = tile * 64 + 4 * g;
      in.r = *reinterpret_cast<const uint2*>(e.residual + int64_t(m) * e.ld + col);
      if constexpr (EPI == EPI_OPROJ) in.w = *reinterpret_cast<const uint2*>(e.w_norm + col);
    }
  }
  return in;
}

__device__ __forceinline__ float4 bf16x4_u2(uint2 r) {
  return make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
}

// The epilogue of one item: row m, four columns 4 g.. of the tile (a0), and the matching
// four of the second 64 columns (gate|up: the up half) or, for QKV, columns 4 g + 32.. (a1).
// All threads call it (shuffles); `valid` marks a real item.
template <int EPI>
__device__ __forceinline__ void ck_epilogue(const EpiArgs& e, int tile, int m, int g, bool valid,
                                            float4 a0, float4 a1, const EpiIn& in,
                                            const float* s_rs) {
  if constexpr (EPI == EPI_QKV) {
    constexpr int D = 64, H2 = 32;
    if (!valid || g >= 8) return;
    const int head = tile, d = 4 * g;
    if (head >= e.Hq && head < e.Hq + e.Hkv && g == 0) e.counters[m * e.Hkv + head - e.Hq] = 0u;
    float lo[4] = {a0.x, a0.y, a0.z, a0.w}, hi[4] = {a1.x, a1.y, a1.z, a1.w};
    if (head < e.Hq + e.Hkv) {   // RoPE, rotate-half pairing d <-> d + 32
      const float c0[4] = {in.c0.x, in.c0.y, in.c0.z, in.c0.w};
      const float c1[4] = {in.c1.x, in.c1.y, in.c1.z, in.c1.w};
      const float s0[4] = {in.s0.x, in.s0.y, in.s0.z, in.s0.w};
      const float s1[4] = {in.s1.x, in.s1.y, in.s1.z, in.s1.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float l2 = lo[t] * c0[t] - hi[t] * s0[t];
        const float h2 = hi[t] * c1[t] + lo[t] * s1[t];
        lo[t] = l2;
        hi[t] = h2;
      }
    }
    __nv_bfloat16* dst;
    if (head < e.Hq) {
      dst = e.q_out + (int64_t(m) * e.Hq + head) * D;
    } else {
      const int kvh = head < e.Hq + e.Hkv ? head - e.Hq : head - e.Hq - e.Hkv;
      __nv_bfloat16* cache = head < e.Hq + e.Hkv ? e.kc : e.vc;
      dst = cache + ((int64_t(m) * e.Hkv + kvh) * e.s_cap + e.pos) * D;
    }
    st_bf16x4(dst + d, lo[0], lo[1], lo[2], lo[3]);
    st_bf16x4(dst + d + H2, hi[0], hi[1], hi[2], hi[3]);
  } else if constexpr (EPI == EPI_OPROJ) {
    const int col = tile * 64 + 4 * g;
    float ss = 0.f;
    if (valid) {
      const int64_t o = int64_t(m) * e.ld + col;
      const float4 h = f4add(a0, bf16x4_u2(in.r));
      st_bf16x4(e.h_out + o, h.x, h.y, h.z, h.w);
      const float4 w = bf16x4_u2(in.w);
      st_bf16x4(e.hw_out + o, h.x * w.x, h.y * w.y, h.z * w.z, h.w * w.w);
      ss = h.x * h.x + h.y * h.y + h.z * h.z + h.w * h.w;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (valid && g == 0) e.ssq[tile * 128 + m] = ss;
  } else if constexpr (EPI == EPI_GATEUP) {
    const int j = tile * 64 + 4 * g;
    if (!valid || j >= e.I) return;
    const float r = s_rs[m];
    auto sw = [r](float gg, float uu) {
      gg *= r;
      return __fdividef(gg, 1.0f + __expf(-gg)) * (uu * r);   // no IEEE-division subroutine
    };
    st_bf16x4(e.act + int64_t(m) * e.I + j, sw(a0.x, a1.x), sw(a0.y, a1.y), sw(a0.z, a1.z),
              sw(a0.w, a1.w));
  } else {
    if (!valid) return;
    const int64_t o = int64_t(m) * e.ld + tile * 64 + 4 * g;
    const float4 h = f4add(a0, bf16x4_u2(in.r));
    st_bf16x4(e.h_out + o, h.x, h.y, h.z, h.w);
  }
}

// Warp roles: warp 0 producer (one thread), warp 1 TMEM owner + MMA issuer (one thread),
// warps 2..5 drain TMEM lanes 32 (warp % 4).. (lane = tile row) and push each CTA's rows to
// it; then all six warps reduce and apply the epilogue.
template <int EPI, int NB, int AR>
__global__ void __launch_bounds__(CK_THREADS)
gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const EpiArgs ea, int num_kb, int a_rows, int b_col2, int stages,
                    uint32_t* status) {
  using S = CkShape<NB, AR>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[CK_MAX_STAGES], empty[CK_MAX_STAGES], acc_full, recv_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ float s_rs[SK_BM];           // EPI_GATEUP: RMSNorm factor of each row
  uint8_t* ring = align1024(smem_raw);
  auto a_slot = [&](int s) { return ring + s * S::A_BYTES; };
  auto b_slot = [&](int s) { return ring + stages * S::A_BYTES + s * S::B_BYTES; };
  float* recv = reinterpret_cast<float*>(ring + stages * S::STAGE);
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int cs = int(gridDim.y), rank = int(cluster_ctarank());
  const int kb0 = rank * num_kb / cs, kb1 = (rank + 1) * num_kb / cs, nkb = kb1 - kb0;
  const int R = (ea.M + cs - 1) / cs;                  // rows owned per CTA
  const int r0 = rank * R;
  const int rows_own = max(0, min(ea.M, r0 + R) - r0);
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&recv_bar, 1);
    mbar_arrive_expect_tx(&recv_bar, uint32_t(cs * rows_own * S::PSTRIDE * 4));
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, NB * 64);
    tmem_relinquish();
  }
  // A rows >= M are whatever the slot holds: accumulator rows are independent, and rows
  // >= M are never stored.
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync();   // every CTA's receive barrier is initialised before any row is pushed
  const uint32_t tmem = tmem_slot;
  const uint32_t tx = uint32_t(a_rows * SK_BK * 2 + S::B_BYTES);
  auto load_b = [&](int s, int kb) {
    tma_load_2d(b_slot(s), &tmB, &full[s], tile * 64, kb * SK_BK);
    if constexpr (NB == 2) tma_load_2d(b_slot(s) + 8192, &tmB, &full[s], b_col2 + tile * 64, kb * SK_BK);
  };
  // Weights never depend on the previous kernel: the first stages' tiles and an L2 prefetch
  // of the rest of the slice are issued before waiting on it.
  const int pre = nkb < stages ? nkb : stages;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], tx);
      load_b(i, kb0 + i);
    }
    for (int kb = kb0 + pre; kb < kb1; ++kb) {
      tma_prefetch_l2_2d(&tmB, tile * 64, kb * SK_BK);
      if constexpr (NB == 2) tma_prefetch_l2_2d(&tmB, b_col2 + tile * 64, kb * SK_BK);
    }
  }
  griddep_wait();   // A (the previous kernel's output) is ready
  // This thread's first reduction item; its epilogue inputs are loaded now, while the
  // MMAs run.
  const EpiIn in0 = ck_prefetch<EPI>(ea, tile, r0 + int(threadIdx.x) / 16, int(threadIdx.x) % 16,
                                     int(threadIdx.x) < rows_own * 16);
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) tma_load_2d(a_slot(i), &tmA, &full[i], (kb0 + i) * SK_BK, 0);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&empty[s], ((i / stages) & 1) ^ 1, status)) break;
        mbar_arrive_expect_tx(&full[s], tx);
        tma_load_2d(a_slot(s), &tmA, &full[s], (kb0 + i) * SK_BK, 0);
        load_b(s, kb0 + i);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {
      // M = 64 when the batch fits (AR = 64): no accumulator rows beyond the batch are
      // computed (the instruction costs the same as M = 128 on the tensor pipe).
      constexpr uint32_t idesc = idesc_bf16_f32(AR == 64 ? 64 : SK_BM, NB * 64, false, true);
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&full[s], (i / stages) & 1, status)) { ok = false; break; }
        tc_fence_after();
        const uint64_t da = smem_desc_sw128(smem_u32(a_slot(s)), 16, 1024);
        const uint64_t db = smem_desc_sw128(smem_u32(b_slot(s)), 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < SK_BK / 16; ++kk)
          mma_bf16_ss(tmem, da + uint64_t((kk * 32) >> 4), db + uint64_t((kk * 2048) >> 4),
                      idesc, (i | kk) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(&acc_full);
    }
    __syncwarp();
  } else {
    // Drain row `row` of the accumulator into this CTA's idle ring ([M][PSTRIDE] fp32), then
    // push rows [q R, (q + 1) R) to CTA q of the cluster, into slot [rank] of its receive
    // area, with one bulk copy per CTA.
    // Accumulator row of this thread's TMEM lane (q * 32 + lane).  M = 128: row = lane.  M = 64:
    // rows 16 q .. 16 q + 15 sit in the first 16 lanes of lane quarter q; the other 16 lanes
    // of each quarter hold no row (kNoRow).
    constexpr int kNoRow = 1 << 20;
    const int q = warp & 3;
    const int row = AR == 64 ? (lane < 16 ? q * 16 + lane : kNoRow) : q * 32 + lane;
    if constexpr (EPI == EPI_GATEUP) {   // while the MMAs run
      float t4[4] = {0.f, 0.f, 0.f, 0.f};
      if (row < ea.M) {
#pragma unroll 4
        for (int t = 0; t < ea.ssq_tiles; ++t) t4[t & 3] += ea.ssq[t * 128 + row];
      }
      if (row < SK_BM)
        s_rs[row] = 1.0f / sqrtf(((t4[0] + t4[1]) + (t4[2] + t4[3])) / float(ea.ld) + ea.eps);
    }
    const bool ok = nkb == 0 || mbar_wait(&acc_full, 0, status);
    tc_fence_after();
    float* prow = reinterpret_cast<float*>(ring) + row * S::PSTRIDE;
    const uint32_t taddr = tmem + (uint32_t(q * 32) << 16);
#pragma unroll 1
    // 32 accumulator columns per TMEM round trip (one load, one wait).
    for (int c = 0; c < NB * 64; c += 32) {
      uint32_t v[32];
      if (nkb > 0 && ok) {
        tmem_ld32(taddr + c, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = 0u;
      }
      if (row < ea.M) {
#pragma unroll
        for (int t = 0; t < 8; ++t)
          reinterpret_cast<float4*>(prow + c)[t] =
              make_float4(__uint_as_float(v[4 * t]), __uint_as_float(v[4 * t + 1]),
                          __uint_as_float(v[4 * t + 2]), __uint_as_float(v[4 * t + 3]));
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the copies
    asm volatile("bar.sync 1, 128;" ::: "memory");                   // the four drain warps
    if (warp == 2 && lane < cs) {
      const int o = lane, n = max(0, min(ea.M, (o + 1) * R) - o * R);
      if (n > 0)
        bulk_copy_to_cluster(
            mapa_shared(smem_u32(recv + rank * R * S::PSTRIDE), uint32_t(o)),
            smem_u32(reinterpret_cast<float*>(ring) + o * R * S::PSTRIDE),
            uint32_t(n * S::PSTRIDE * 4), mapa_shared(smem_u32(&recv_bar), uint32_t(o)));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NB * 64);
  }
  // Every CTA's rows have arrived here; once all CTAs have arrived on the cluster barrier,
  // no copy to or from any CTA is in flight, so the wait before exit keeps every ring and
  // receive area alive as long as it is read or written.
  mbar_wait(&recv_bar, 0, status);
  __syncwarp();   // the .aligned cluster barrier needs converged warps
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  const int iters = (R * 16 + CK_THREADS - 1) / CK_THREADS;
  for (int itn = 0; itn < iters; ++itn) {
    const int idx = itn * CK_THREADS + int(threadIdx.x);
    const int rl = idx / 16, g = idx % 16, m = r0 + rl;
    const bool valid = rl < rows_own;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    if (valid) {
      const bool second = NB == 2 || (EPI == EPI_QKV && g < 8);
      const float* src = recv + rl * S::PSTRIDE + 4 * g;
      for (int p = 0; p < cs; ++p) {
        const float* sp = src + p * R * S::PSTRIDE;
        a0 = f4add(a0, *reinterpret_cast<const float4*>(sp));
        if (second) a1 = f4add(a1, *reinterpret_cast<const float4*>(sp + (NB == 2 ? 64 : 32)));
      }
    }
    ck_epilogue<EPI>(ea, tile, m, g, valid, a0, a1,
                     itn == 0 ? in0 : ck_prefetch<EPI>(ea, tile, m, g, valid), s_rs);
  }
  __syncwarp();
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Split-KV attention: one producer + DA_WARPS consumer warps per CTA.  Flat mode (cl = 0):
// persistent, CTA c of gridDim.x takes chunk range c of all units' chunks, partials merged
// through global memory by each unit's last CTA.  Cluster mode (cl > 0, grid units x cl,
// clusters of cl): the cl CTAs of a cluster split one unit's chunks and merge over
// distributed shared memory.
__global__ void __launch_bounds__(DA_THREADS)
decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __nv_bfloat16* __restrict__ q, float* __restrict__ opart,
                   float* __restrict__ mlpart, uint32_t* __restrict__ counters,
                   __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ kcache,
                   const __nv_bfloat16* __restrict__ vcache, int Hq, int Hkv, int cap, int L,
                   int S, int units, float scale_log2, int cl, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[DA_NST], empty[DA_NST], recv_bar;
  __shared__ float s_m[DA_WARPS][8], s_l[DA_WARPS][8];
  __shared__ uint32_t s_last;
  __shared__ int64_t s_seg_unit[DA_MAX_SEGS];
  __shared__ uint32_t s_seg_n[DA_MAX_SEGS];
  const int rank = cl > 0 ? int(cluster_ctarank()) : 0;
  int64_t cb, ce;
  if (cl > 0) {
    // The chunks cover the L - 1 cached keys; the appended key joins in rank 0's merge, so
    // the ranks split whole chunks evenly and no chunk is loaded for that one key.
    const int64_t unit = blockIdx.x / cl;
    const int sc = (L - 1 + DA_KEYS - 1) / DA_KEYS;
    cb = unit * S + int64_t(rank) * sc / cl;
    ce = unit * S + int64_t(rank + 1) * sc / cl;
    L -= 1;
  } else {
    cb = range_start(int64_t(S) * units, blockIdx.x, gridDim.x);
    ce = range_start(int64_t(S) * units, blockIdx.x + 1, gridDim.x);
  }
  const AttnCtx cx{&tmK, &tmV, q, opart, mlpart, counters, out, kcache, vcache, Hq, Hkv, cap, L, S, units,
                   scale_log2, status, int(blockIdx.x), int(gridDim.x), cl, rank, cb, ce,
                   align1024(smem_raw), &recv_bar, full, empty, s_m, s_l, &s_last, s_seg_unit,
                   s_seg_n};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    attn_init(cx);
    mbar_init(&recv_bar, 1);
    if (cl > 0 && rank == 0) mbar_arrive_expect_tx(&recv_bar, uint32_t((cl - 1) * DA_PART));
    fence_barrier_init();
  }
  __syncthreads();
  if (cl > 0) cluster_sync();   // rank 0's receive barrier is initialised before any copy
  griddep_launch_dependents();
  if (warp == DA_WARPS) {
    if (lane == 0) {
      int64_t ci;
      int i;
      attn_produce_pre(cx, ci, i);
      griddep_wait();
      attn_produce_rest(cx, ci, i);
    }
    __syncwarp();
  } else {
    griddep_wait();   // q, the appended K / V rows and the counters are ready
    attn_consumers<1>(cx, warp, lane, threadIdx.x);
  }
  // Cluster mode: rank 0 arrives once every copy into it has landed, so after the wait no
  // copy out of any CTA's ring is still reading it.
  if (cl > 0) {
    __syncwarp();   // the .aligned cluster barrier needs converged warps
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
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

// Cluster size of a GEMM: double it (up to CK_MAX_CLUSTER, and at most one k-block per CTA) while the
// tiles x cluster CTAs do not yet cover the SMs.
int pick_cluster(int64_t tiles, int64_t kbs, int sms) {
  int cs = 1;
  while (cs * 2 <= CK_MAX_CLUSTER && cs * 2 <= kbs && tiles * cs < sms) cs *= 2;
  return cs;
}

struct Layout {
  size_t xn, q, attn, h1, h1w, act, ssq, opart, mlpart, counters, total;
  int attn_splits;
};

Layout plan(const enigma_decode_layer_desc& d) {
  const int64_t B = d.batch, H = d.hidden, D = d.head_dim, Hq = d.heads_q, Hkv = d.heads_kv;
  const int64_t I = d.intermediate;
  const int64_t L = d.position + 1;
  Layout l;
  // Attention CTAs take 128-key chunks of one (sequence, kv head); the partial buffers
  // are sized for the cache capacity, so one workspace serves every position.
  const int64_t smax = (d.cache_capacity + DA_KEYS - 1) / DA_KEYS;
  l.attn_splits = int((L + DA_KEYS - 1) / DA_KEYS);
  const int64_t G = Hq / Hkv;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align256(off + bytes); return o; };
  l.xn = take(size_t(B * H) * 2);
  l.q = take(size_t(B * Hq * D) * 2);
  l.attn = take(size_t(B * Hq * D) * 2);
  l.h1 = take(size_t(B * H) * 2);
  l.h1w = take(size_t(B * H) * 2);
  l.act = take(size_t(B * I) * 2);
  l.ssq = take(size_t(H / 64) * 128 * 4);
  l.opart = take(size_t(B * Hkv * smax * G * D) * 4);
  l.mlpart = take(size_t(B * Hkv * smax * G * 2) * 4);
  l.counters = take(size_t(B * Hkv) * 4);
  l.total = off;
  return l;
}

// C-tile columns [tile * 64, +64) of A [M, K] x Bw [K, n_cols] (and, NB = 2, columns
// b_col2 + tile * 64 ..) with epilogue EPI, as one cluster launch.
// Shared memory per CTA when two CTAs must share an SM (more CTAs than SMs), else one.
constexpr int kCkSmemTwoPerSm = 112 * 1024;
constexpr int kCkSmemOnePerSm = 200 * 1024;

template <int EPI, int NB, int AR>
cudaError_t cluster_gemm_ar(const void* A, const void* Bw, int64_t M, int64_t n_cols, int64_t K,
                            int64_t tiles, int b_col2, const EpiArgs& ea, int sms,
                            uint32_t* status, cudaStream_t s) {
  using S = CkShape<NB, AR>;
  CUtensorMap ta, tb;
  const int a_rows = int(std::min<int64_t>(SK_BM, (M + 7) / 8 * 8));
  if (!make_tmap_bf16_2d(&ta, A, M, K, K, SK_BK, uint32_t(a_rows)) ||
      !make_tmap_bf16_2d(&tb, Bw, K, n_cols, n_cols, 64, SK_BK))
    return cudaErrorInvalidValue;
  const int64_t kbs = (K + SK_BK - 1) / SK_BK;
  const int cs = pick_cluster(tiles, kbs, sms);
  const int64_t R = (M + cs - 1) / cs;
  const int recv = int(cs * R * S::PSTRIDE * 4);
  int budget = tiles * cs > sms ? kCkSmemTwoPerSm : kCkSmemOnePerSm;
  int stages = (budget - 1024 - recv) / S::STAGE;
  if (stages < 2) stages = (227 * 1024 - 1024 - recv) / S::STAGE;
  // No more stages than the CTA has k-blocks: all of its weight tiles are then requested
  // before the wait, and the CTA leaves room for the next kernel's CTAs.
  stages = std::min<int>(stages, std::max<int64_t>(2, (kbs + cs - 1) / cs));
  // The drained ring stages the whole partial tile.
  stages = std::max<int>(stages, int((M * S::PSTRIDE * 4 + S::STAGE - 1) / S::STAGE));
  stages = std::min(stages, CK_MAX_STAGES);
  if (stages < 2) return cudaErrorInvalidValue;
  const int smem = 1024 + stages * S::STAGE + recv;
  auto kern = gemm_cluster_kernel<EPI, NB, AR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && cs > 8)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(tiles), unsigned(cs));
  cfg.blockDim = dim3(CK_THREADS);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = unsigned(cs);
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, ea, int(kbs), a_rows, b_col2, stages, status);
}

template <int EPI, int NB>
cudaError_t cluster_gemm(const void* A, const void* Bw, int64_t M, int64_t n_cols, int64_t K,
                         int64_t tiles, int b_col2, const EpiArgs& ea, int sms, uint32_t* status,
                         cudaStream_t s) {
  return M <= 64 ? cluster_gemm_ar<EPI, NB, 64>(A, Bw, M, n_cols, K, tiles, b_col2, ea, sms, status, s)
                 : cluster_gemm_ar<EPI, NB, 128>(A, Bw, M, n_cols, K, tiles, b_col2, ea, sms, status, s);
}

}  // namespace

// The whole step with an explicit SM count and status word (no per-device state used).
cudaError_t decode_layer_run(const enigma_decode_layer_desc& d, const void* x, void* out,
                             void* ws, int sms, uint32_t* status, cudaStream_t s) {
  const Layout l = plan(d);
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto bfp = [&](size_t o) { return reinterpret_cast<__nv_bfloat16*>(w + o); };
  const int B = int(d.batch), H = int(d.hidden), D = int(d.head_dim);
  const int Hq = int(d.heads_q), Hkv = int(d.heads_kv), I = int(d.intermediate);
  const int Nqkv = (Hq + 2 * Hkv) * D;
  cudaError_t e;
#define ENIGMA_TRY(expr)           \
  do {                             \
    e = (expr);                    \
    if (e != cudaSuccess) return e; \
  } while (0)
  EpiArgs ea = {};
  ea.M = B;
  // 1. input RMSNorm
  ENIGMA_TRY(rmsnorm_launch_pdl_bf16(x, d.w_in_norm, bfp(l.xn), B, H, d.eps, sms, s));
  // 2. QKV projection + RoPE + KV-cache append at `position` (+ attention counters zeroed)
  ea.Hq = Hq;
  ea.Hkv = Hkv;
  ea.s_cap = int(d.cache_capacity);
  ea.pos = int(d.position);
  ea.cosv = d.rope_cos;
  ea.sinv = d.rope_sin;
  ea.q_out = bfp(l.q);
  ea.kc = static_cast<__nv_bfloat16*>(d.k_cache);
  ea.vc = static_cast<__nv_bfloat16*>(d.v_cache);
  ea.counters = reinterpret_cast<uint32_t*>(w + l.counters);
  ENIGMA_TRY((cluster_gemm<EPI_QKV, 1>(bfp(l.xn), d.w_qkv, B, Nqkv, H, Nqkv / 64, 0, ea, sms,
                                      status, s)));
  // 3. attention over position + 1 keys (split-KV: the CTAs of a unit merge over distributed
  //    shared memory, or, flat ranges, through global memory by the unit's last CTA)
  {
    CUtensorMap tk, tv;
    const uint64_t rows = uint64_t(B) * Hkv * uint64_t(d.cache_capacity);
    if (!make_tmap_bf16_2d(&tk, d.k_cache, rows, DA_D, DA_D, DA_D, DA_KEYS) ||
        !make_tmap_bf16_2d(&tv, d.v_cache, rows, DA_D, DA_D, DA_D, DA_KEYS))
      return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DA_SMEM);   // per device, cheap: set on every call
    if (e != cudaSuccess) return e;
    // Cluster mode when the units can fill the SMs with k <= DA_CL_MAX CTAs each in one
    // wave (k = the smallest power of two with units x k >= SMs); else flat ranges.
    const int64_t units = int64_t(B) * Hkv;
    int cl = 1;
    while (cl < DA_CL_MAX && units * cl < sms) cl *= 2;
    const int cached_chunks = int((d.position + DA_KEYS - 1) / DA_KEYS);
    if (units * cl < sms || units * cl > int64_t(sms) * DA_CTAS_PER_SM || cl > cached_chunks)
      cl = 0;
    const int64_t chunks = units * l.attn_splits;
    const int ctas = cl > 0 ? int(units * cl)
                            : int(std::min<int64_t>(chunks, int64_t(sms) * DA_CTAS_PER_SM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(ctas));
    cfg.blockDim = dim3(DA_THREADS);
    cfg.dynamicSmemBytes = DA_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(cl > 0 ? cl : 1);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    ENIGMA_TRY(cudaLaunchKernelEx(&cfg, decode_attn_kernel, tk, tv,
                                  static_cast<const __nv_bfloat16*>(bfp(l.q)),
                                  reinterpret_cast<float*>(w + l.opart),
                                  reinterpret_cast<float*>(w + l.mlpart),
                                  reinterpret_cast<uint32_t*>(w + l.counters), bfp(l.attn),
                                  static_cast<const __nv_bfloat16*>(d.k_cache),
                                  static_cast<const __nv_bfloat16*>(d.v_cache), Hq,
                                  Hkv, int(d.cache_capacity), int(d.position + 1), l.attn_splits,
                                  B * Hkv, d.attn_scale * 1.4426950408889634f, cl, status));
  }
  // 4. O projection + residual(x) -> h1; h1 * w_post_norm -> h1w; row sums of h1^2 per tile
  ea.ld = H;
  ea.residual = static_cast<const __nv_bfloat16*>(x);
  ea.h_out = bfp(l.h1);
  ea.w_norm = static_cast<const __nv_bfloat16*>(d.w_post_norm);
  ea.hw_out = bfp(l.h1w);
  ea.ssq = reinterpret_cast<float*>(w + l.ssq);
  ENIGMA_TRY((cluster_gemm<EPI_OPROJ, 1>(bfp(l.attn), d.w_o, B, H, int64_t(Hq) * D, H / 64, 0, ea,
                                        sms, status, s)));
  // 5. gate|up projection of h1w, scaled by the post-attention RMSNorm factor, SwiGLU -> act
  //    (rmsnorm(h) w W = r (h w) W with r = 1 / sqrt(mean(h^2) + eps) per row)
  ea.I = I;
  ea.ssq_tiles = H / 64;
  ea.eps = d.eps;
  ea.act = bfp(l.act);
  ENIGMA_TRY((cluster_gemm<EPI_GATEUP, 2>(bfp(l.h1w), d.w_gate_up, B, 2 * int64_t(I), H,
                                         (I + 63) / 64, I, ea, sms, status, s)));
  // 6. down projection + residual(h1) -> out
  ea.residual = bfp(l.h1);
  ea.h_out = static_cast<__nv_bfloat16*>(out);
  ENIGMA_TRY((cluster_gemm<EPI_DOWN, 1>(bfp(l.act), d.w_down, B, H, I, H / 64, 0, ea, sms,
                                       status, s)));
#undef ENIGMA_TRY
  return cudaSuccess;
}

size_t decode_workspace_bytes(const enigma_decode_layer_desc& d) {
  return plan(d).total;
}

cudaError_t decode_layer_launch(const enigma_decode_layer_desc& d, const void* x, void* out,
                                void* ws, cudaStream_t s) {
  uint32_t* status = device_status();
  if (status == nullptr) return cudaErrorMemoryAllocation;   // the kernels' waits need it
  return decode_layer_run(d, x, out, ws, sm_count(), status, s);
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
// clearing.  The entry has its own status word, also a static device array: a bounded
// wait that runs out flags it, and enigma_synchronize / enigma_take_device_status report
// it once (ENIGMA_ERR_TIMEOUT) and clear it, like the library's per-device word.  Calls
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
  const size_t need = enigma::plan(*desc).total;
  if (need > kNoAllocScratchBytes) {
    enigma::set_error("bad argument: decode noalloc: this step needs %zu bytes of scratch, more than "
              "the fixed %zu-byte array of the no-allocation entry point; use "
              "enigma_decode_layer_bf16 with a caller-provided workspace",
              need, kNoAllocScratchBytes);
    return ENIGMA_ERR_BADARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = enigma::decode_layer_run(*desc, x, out, dev->scratch, dev->sms, dev->status, s);
  if (e != cudaSuccess) {
    enigma::set_error("decode noalloc launch failed: %s (%s)", cudaGetErrorName(e), cudaGetErrorString(e));
    return ENIGMA_ERR_LAUNCH;
  }
  return ENIGMA_OK;
}

namespace enigma {
cudaError_t noalloc_take_status(uint32_t* value) {
  *value = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return e;
  uint32_t* st = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_dev[dev].ready) st = g_noalloc_dev[dev].status;
  }
  if (st == nullptr) return cudaSuccess;
  e = cudaMemcpy(value, st, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && *value != 0) e = cudaMemset(st, 0, sizeof(uint32_t));
  return e;
}
}  // namespace enigma

// Self-test of the no-allocation entry's timeout reporting: the same probe as
// enigma_check_timeout_path, aimed at this entry's static status word.
extern "C" int32_t enigma_decode_noalloc_check_timeout_path(int64_t polls, void* stream) {
  if (polls < 0 || polls > (int64_t(1) << 24)) {
    enigma::set_error("bad argument: polls must be in [0, 2^24]");
    return ENIGMA_ERR_BADARG;
  }
  NoAllocDevice* dev = nullptr;
  int32_t rc = noalloc_setup(&dev);
  if (rc != ENIGMA_OK) return rc;
  cudaError_t e = enigma::launch_timeout_probe(dev->status, static_cast<long long>(polls),
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    enigma::set_error("timeout probe: %s", cudaGetErrorString(e));
    return ENIGMA_ERR_LAUNCH;
  }
  return ENIGMA_OK;
}
