// decode_common.cuh — device building blocks of the decode step: the
// split-K GEMM roles, the reductions that follow each GEMM and the split-KV attention.
// decode.cu wraps each in a kernel (one launch per stage, programmatic dependent launches).
//
// Every block takes its work item and its pipeline state explicitly, so a CTA can run one
// item or a sequence of items (the GEMM ring and accumulator counters carry across items).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace enigma_decode {

using namespace enigma_sm100;

// ============================================================================ split-K GEMM
// partial[split][m][n] (fp32) = A[m, kslice] * B[kslice, n] for one 128 x 64 tile (M <= 128;
// accumulator rows past M are not stored).  Warp roles inside a CTA: one producer thread
// (TMA), one MMA thread, four epilogue warps (TMEM lanes 32 (warp % 4) ..).
constexpr int SK_BM = 128;
constexpr int SK_BN = 64;
constexpr int SK_BK = 64;
constexpr int SK_STAGES = 4;
constexpr int SK_A_BYTES = SK_BM * SK_BK * 2;   // 16 KB
constexpr int SK_B_BYTES = SK_BK * SK_BN * 2;   // 8 KB
constexpr int SK_RING = SK_STAGES * (SK_A_BYTES + SK_B_BYTES);   // 96 KB

struct SkItem {
  int nb, split, kb0, kb1;                      // N tile, split index, k-block range
};

__host__ __device__ inline SkItem sk_item(int item, int tiles, int kb_per_split, int num_kb) {
  SkItem it;
  it.nb = item % tiles;
  it.split = item / tiles;
  it.kb0 = it.split * kb_per_split;
  it.kb1 = it.kb0 + kb_per_split < num_kb ? it.kb0 + kb_per_split : num_kb;
  if (it.kb1 < it.kb0) it.kb1 = it.kb0;
  return it;
}

// The ring: A slots [SK_STAGES][16 KB] then B slots [SK_STAGES][8 KB] (1024-aligned base),
// full/empty barriers per stage, one TMEM accumulator (64 columns) with full/empty barriers.
struct SkRing {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;
  uint64_t* acc_empty;
  __device__ uint8_t* a(int s) const { return base + s * SK_A_BYTES; }
  __device__ uint8_t* b(int s) const { return base + SK_STAGES * SK_A_BYTES + s * SK_B_BYTES; }
};

__device__ inline void sk_ring_init(const SkRing& r) {
  for (int s = 0; s < SK_STAGES; ++s) {
    mbar_init(&r.full[s], 1);
    mbar_init(&r.empty[s], 1);
  }
  mbar_init(r.acc_full, 1);
  mbar_init(r.acc_empty, 128);
}

// The TMA box covers the a_rows (= M rounded up to 8) real rows of A; the MMA reads 128.
// Rows a_rows..127 of every A slot are zeroed (128-byte rows: swizzling permutes 16-byte
// chunks within a row, so whole rows stay zero); TMA never writes them.  Callers order this
// before the first MMA (a CTA barrier after it).
__device__ inline void sk_zero_pad(const SkRing& r, int a_rows, int tid, int nthreads) {
  if (a_rows >= SK_BM) return;
  const int per = (SK_BM - a_rows) * 8;
  for (int i = tid; i < SK_STAGES * per; i += nthreads)
    reinterpret_cast<uint4*>(r.a(i / per) + a_rows * 128)[i % per] = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
}

// Producer, first part: the weight (B) tiles of the item's first stages, which never depend
// on earlier stages of the step, so they can be requested before waiting for them.  `it` is
// the producer's running k-block count over all items; returns how many stages it started.
__device__ inline int sk_produce_pre(const SkRing& r, const CUtensorMap* tmB, const SkItem& w,
                                     int a_rows, uint32_t it, uint32_t* status) {
  const int n = w.kb1 - w.kb0;
  const int pre = n < SK_STAGES ? n : SK_STAGES;
  for (int i = 0; i < pre; ++i) {
    const uint32_t k = it + i, s = k % SK_STAGES;
    if (!mbar_wait(&r.empty[s], ((k / SK_STAGES) & 1) ^ 1, status)) return i;
    mbar_arrive_expect_tx(&r.full[s], a_rows * SK_BK * 2 + SK_B_BYTES);
    tma_load_2d(r.b(s), tmB, &r.full[s], w.nb * SK_BN, (w.kb0 + i) * SK_BK);
  }
  return pre;
}

// Producer, second part (after the wait): A for the pre-started stages, then both operands
// for the rest.  Advances `it` by the item's k-block count.
__device__ inline void sk_produce_rest(const SkRing& r, const CUtensorMap* tmA,
                                       const CUtensorMap* tmB, const SkItem& w, int a_rows,
                                       int pre, uint32_t& it, uint32_t* status) {
  for (int i = 0; i < pre; ++i)
    tma_load_2d(r.a((it + i) % SK_STAGES), tmA, &r.full[(it + i) % SK_STAGES], (w.kb0 + i) * SK_BK, 0);
  for (int kb = w.kb0 + pre; kb < w.kb1; ++kb) {
    const uint32_t k = it + uint32_t(kb - w.kb0), s = k % SK_STAGES;
    if (!mbar_wait(&r.empty[s], ((k / SK_STAGES) & 1) ^ 1, status)) break;
    mbar_arrive_expect_tx(&r.full[s], a_rows * SK_BK * 2 + SK_B_BYTES);
    tma_load_2d(r.a(s), tmA, &r.full[s], kb * SK_BK, 0);
    tma_load_2d(r.b(s), tmB, &r.full[s], w.nb * SK_BN, kb * SK_BK);
  }
  it += uint32_t(w.kb1 - w.kb0);
}

// MMA thread: accumulate the item into the TMEM accumulator.  `it` = running k-block count,
// `acc` = running count of accumulator uses (items with at least one k-block).
__device__ inline void sk_mma(const SkRing& r, uint32_t tmem, const SkItem& w, uint32_t& it,
                              uint32_t& acc, uint32_t* status) {
  if (w.kb1 <= w.kb0) return;
  if (acc > 0 && !mbar_wait(r.acc_empty, (acc - 1) & 1, status)) return;
  tc_fence_after();
  constexpr uint32_t idesc = idesc_bf16_f32(SK_BM, SK_BN, false, true);
  bool ok = true;
  for (int kb = w.kb0; kb < w.kb1; ++kb) {
    const uint32_t k = it + uint32_t(kb - w.kb0), s = k % SK_STAGES;
    if (!mbar_wait(&r.full[s], (k / SK_STAGES) & 1, status)) { ok = false; break; }
    tc_fence_after();
    const uint64_t da = smem_desc_sw128(smem_u32(r.a(s)), 16, 1024);
    const uint64_t db = smem_desc_sw128(smem_u32(r.b(s)), SK_B_BYTES, 1024);
#pragma unroll
    for (int kk = 0; kk < SK_BK / 16; ++kk)
      mma_bf16_ss(tmem, da + uint64_t((kk * 32) >> 4), db + uint64_t((kk * 2048) >> 4), idesc,
                  (kb != w.kb0 || kk != 0) ? 1u : 0u);
    mma_commit(&r.empty[s]);
  }
  if (ok) mma_commit(r.acc_full);
  it += uint32_t(w.kb1 - w.kb0);
  ++acc;
}

// Epilogue warps (quarter = warp % 4): drain the accumulator into partial[split][m][n]
// (zeros for an item without k-blocks) and hand the accumulator back.
__device__ inline void sk_store(const SkRing& r, uint32_t tmem, const SkItem& w, float* partial,
                                int M, int N, int quarter, int lane, uint32_t& acc,
                                uint32_t* status) {
  const int row = quarter * 32 + lane;
  const bool have = w.kb1 > w.kb0;
  if (have && !mbar_wait(r.acc_full, acc & 1, status)) return;
  tc_fence_after();
  float* dst = partial + (int64_t(w.split) * M + row) * N + w.nb * SK_BN;
  const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
  for (int c = 0; c < SK_BN; c += 16) {
    uint32_t v[16];
    if (have) {
      tmem_ld16(taddr + c, v);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int t = 0; t < 16; ++t) v[t] = 0u;
    }
    if (row < M && w.nb * SK_BN + c < N) {
      float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        d4[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                            __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
    }
  }
  if (have) {
    tc_fence_before();
    mbar_arrive(r.acc_empty);
    ++acc;
  }
}

// ============================================================================ reductions
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// q / k / v = sum over splits of the QKV partials; RoPE on the q and k heads
// (rotate-half pairing d <-> d + D/2 with full-length cos / sin tables, as in
// examples/qwen_megakernel.py:90-107); q to q_out [M, Hq, D], k and v appended at position
// `pos` of the caches [M, Hkv, S_cap, D].  One warp per (row m, head), lane d owns dims d and
// d + 32 (D = 64).  The warp of each (m, k head) also zeroes the attention's completion
// counter of that (sequence, kv head).
__device__ inline void qkv_finalize_item(const float* __restrict__ part, int splits, int M, int N,
                                         int Hq, int Hkv, const float* __restrict__ cosv,
                                         const float* __restrict__ sinv,
                                         __nv_bfloat16* __restrict__ q_out,
                                         __nv_bfloat16* __restrict__ kc,
                                         __nv_bfloat16* __restrict__ vc, int s_cap, int pos,
                                         uint32_t* __restrict__ attn_counters, int m, int head,
                                         int d) {
  constexpr int D = 64, H2 = 32;
  if (head >= Hq && head < Hq + Hkv && d == 0) attn_counters[m * Hkv + head - Hq] = 0u;
  const int c = head * D + d;
  float lo = 0.f, hi = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float* p = part + (int64_t(s) * M + m) * N;
    lo += __ldcg(p + c);
    hi += __ldcg(p + c + H2);
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
// y = rmsnorm(h) * w when y_out is given.  One row m per call on 256 threads (tid < 256),
// each thread four adjacent columns (float4 partial loads, all splits in flight); N % 4 == 0,
// N <= 2048.  `red` is 8 floats of shared memory; the caller's 256 threads all call this.
__device__ inline void reduce_residual_norm_row(const float* __restrict__ part, int splits, int M,
                                                int N, const __nv_bfloat16* __restrict__ residual,
                                                __nv_bfloat16* __restrict__ h_out,
                                                const __nv_bfloat16* __restrict__ w,
                                                __nv_bfloat16* __restrict__ y_out, float eps,
                                                int m, int tid, float* red) {
  constexpr int kPer = 2;  // float4 groups per thread: 256 * 2 * 4 = 2048 columns
  float4 h[kPer];
  float ss = 0.f;
#pragma unroll
  for (int t = 0; t < kPer; ++t) {
    const int n = (tid + t * 256) * 4;
    h[t] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n < N) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (residual) {
        const uint2 r = *reinterpret_cast<const uint2*>(residual + int64_t(m) * N + n);
        acc = make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
      }
#pragma unroll 4
      for (int s = 0; s < splits; ++s) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(part + (int64_t(s) * M + m) * N + n));
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
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  asm volatile("bar.sync 2, 256;" ::: "memory");
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += red[i];
  asm volatile("bar.sync 2, 256;" ::: "memory");   // red is free again for the next row
  const float r = 1.0f / sqrtf(total / float(N) + eps);
#pragma unroll
  for (int t = 0; t < kPer; ++t) {
    const int n = (tid + t * 256) * 4;
    if (n < N) {
      const uint2 wv = *reinterpret_cast<const uint2*>(w + n);
      *reinterpret_cast<uint2*>(y_out + int64_t(m) * N + n) = make_uint2(
          pack_bf16x2(h[t].x * r * bf16_lo(wv.x), h[t].y * r * bf16_hi(wv.x)),
          pack_bf16x2(h[t].z * r * bf16_lo(wv.y), h[t].w * r * bf16_hi(wv.y)));
    }
  }
}

// act[m, j] = silu(g) * u with g = column j and u = column j + I of the summed gate|up
// partials (N = 2 I); silu(g) = g / (1 + e^-g) (qwen_megakernel.py:212-216).  Float4 group
// q = four columns; I % 4 == 0.
__device__ inline void swiglu_group(const float* __restrict__ part, int splits, int M, int I,
                                    __nv_bfloat16* __restrict__ act, int64_t q) {
  const int m = int(q * 4 / I), j = int(q * 4 % I);
  float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
  for (int s = 0; s < splits; ++s) {
    const float* p = part + (int64_t(s) * M + m) * (2 * I);
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p + j));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + j + I));
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

// Named barrier BAR over the DA_WARPS consumer warps only (the producer never joins it).
template <int BAR>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(DA_WARPS * 32) : "memory");
}

// One attention "group": a producer warp and DA_WARPS consumer warps working through the
// chunk range of virtual CTA vc of nvc (one group per CTA; nvc <= the number of chunks, so
// every range is non-empty, as the merge's range arithmetic requires).
struct AttnCtx {
  const CUtensorMap* tmK;
  const CUtensorMap* tmV;
  const __nv_bfloat16* q;
  float* opart;
  float* mlpart;
  uint32_t* counters;
  __nv_bfloat16* out;
  int Hq, Hkv, cap, L, S, units;
  float scale_log2;
  uint32_t* status;
  int vc, nvc;
  uint8_t* stages;          // DA_NST stages, then the DA_MERGE merge area; 1024-aligned
  uint64_t* full;           // [DA_NST]
  uint64_t* empty;          // [DA_NST]
  float (*s_m)[8];          // [DA_WARPS][8]
  float (*s_l)[8];
  uint32_t* s_last;
  __device__ int64_t c_begin() const { return int64_t(S) * units * vc / nvc; }
  __device__ int64_t c_end() const { return int64_t(S) * units * (vc + 1) / nvc; }
};

__device__ inline void attn_init(const AttnCtx& c) {
  for (int s = 0; s < DA_NST; ++s) {
    mbar_init(&c.full[s], 1);
    mbar_init(&c.empty[s], DA_WARPS);
  }
}

__device__ inline void attn_issue(const AttnCtx& c, int64_t ci, int st) {
  const int32_t row = int32_t((ci / c.S) * c.cap + (ci % c.S) * DA_KEYS);
  uint8_t* dst = c.stages + st * DA_STAGE;
  mbar_arrive_expect_tx(&c.full[st], DA_STAGE);
  tma_load_2d(dst, c.tmK, &c.full[st], 0, row);
  tma_load_2d(dst + DA_TILE, c.tmV, &c.full[st], 0, row);
}

// Producer thread, before the wait for the step's earlier stages: the first chunks of the
// range, stopping at the first chunk that holds the appended key (the last of a unit).  (An
// L2 prefetch of the whole range was measured 1.7 us slower: it queues the ring's demand
// loads behind 67 MB of prefetch.)  `ci` / `i` carry the position to attn_produce_rest.
__device__ inline void attn_produce_pre(const AttnCtx& c, int64_t& ci, int& i) {
  ci = c.c_begin();
  i = 0;
  const int64_t ce = c.c_end();
  for (; ci < ce && i < DA_NST && ci % c.S != c.S - 1; ++ci, ++i) attn_issue(c, ci, i);
}

__device__ inline void attn_produce_rest(const AttnCtx& c, int64_t ci, int i) {
  const int64_t ce = c.c_end();
  for (; ci < ce; ++ci, ++i) {
    const int st = i % DA_NST;
    if (!mbar_wait(&c.empty[st], ((i / DA_NST) & 1) ^ 1, c.status)) break;
    attn_issue(c, ci, st);
  }
}


// The DA_WARPS consumer warps of a group (warp 0..3 within the group, tid 0..127); BAR is
// the group's named barrier.
template <int BAR>
__device__ inline void attn_consumers(const AttnCtx& cx, int warp, int lane, int tid) {
  float* s_o = reinterpret_cast<float*>(cx.stages + DA_NST * DA_STAGE);   // [warp][8][D]
  const int G = cx.Hq / cx.Hkv;
  const int64_t n_chunks = int64_t(cx.S) * cx.units;
  const int64_t cb = cx.c_begin(), ce = cx.c_end();
  const int g = lane >> 2, t = lane & 3, kw = warp * 32;
  const uint32_t stage0 = smem_u32(cx.stages);
  uint32_t qa[4][2];
  float o[8][4];
  float m_run = -INFINITY, l_run = 0.f;
  int64_t cur_unit = -1;
  int seg_first = 0;
  for (int64_t ci = cb, i = 0; ci < ce; ++ci, ++i) {
    const int64_t unit = ci / cx.S;
    const int j = int(ci % cx.S);
    if (unit != cur_unit) {
      // Q fragments: a0 = dims 16 ks + 2t, +1 and a2 = dims 16 ks + 8 + 2t, +1 of head g.
      const bool live = g < G;
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          cx.q + ((unit / cx.Hkv) * cx.Hq + (unit % cx.Hkv) * G + (live ? g : 0)) * DA_D);
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
    if (!mbar_wait(&cx.full[st], uint32_t((i / DA_NST) & 1), cx.status)) return;
    const uint32_t kaddr = stage0 + st * DA_STAGE, vaddr = kaddr + DA_TILE;
    const int nk = min(DA_KEYS, cx.L - j * DA_KEYS);
    const bool ragged = nk < kw + 32;
    if (ragged) {
      // Rows past the last key may hold anything (other units, unwritten cache slots):
      // zero this warp's V rows there so that P = 0 never meets a NaN.
      uint8_t* vt = cx.stages + st * DA_STAGE + DA_TILE;
      for (int idx = lane; idx < 32 * 8; idx += 32) {
        const int r = kw + (idx >> 3);
        if (r >= nk) reinterpret_cast<uint4*>(vt + r * 128)[idx & 7] = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // cx.S for the warp's 4 blocks of 8 keys.
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
        sacc[nb][e] = ok ? sacc[nb][e] * cx.scale_log2 : -INFINITY;
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
    if (lane == 0) mbar_arrive(&cx.empty[st]);

    if (ci + 1 != ce && j + 1 != cx.S) continue;
    // ------------------------------------------------ end of this unit's segment
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (g < G) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
        *reinterpret_cast<float2*>(s_o + (warp * 8 + g) * DA_D + 8 * n + 2 * t) =
            make_float2(o[n][0], o[n][1]);
      if (t == 0) {
        cx.s_m[warp][g] = m_run;
        cx.s_l[warp][g] = l_run;
      }
    }
    consumers_sync<BAR>();
    const int64_t pbase = (unit * cx.S + seg_first) * G;
    for (int idx = tid; idx < G * (DA_D / 4); idx += DA_WARPS * 32) {
      const int gg = idx / (DA_D / 4), d = (idx % (DA_D / 4)) * 4;
      float M = cx.s_m[0][gg];                      // warp 0 always holds a valid key
#pragma unroll
      for (int w = 1; w < DA_WARPS; ++w) M = fmaxf(M, cx.s_m[w][gg]);
      float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
      float den = 0.f;
#pragma unroll
      for (int w = 0; w < DA_WARPS; ++w) {
        const float wt = cx.s_m[w][gg] == -INFINITY ? 0.f : ex2f(cx.s_m[w][gg] - M);
        const float4 v = *reinterpret_cast<const float4*>(s_o + (w * 8 + gg) * DA_D + d);
        num.x = fmaf(wt, v.x, num.x);
        num.y = fmaf(wt, v.y, num.y);
        num.z = fmaf(wt, v.z, num.z);
        num.w = fmaf(wt, v.w, num.w);
        den = fmaf(wt, cx.s_l[w][gg], den);
      }
      *reinterpret_cast<float4*>(cx.opart + (pbase + gg) * DA_D + d) = num;
      if (d == 0) *reinterpret_cast<float2*>(cx.mlpart + (pbase + gg) * 2) = make_float2(M, den);
    }
    __threadfence();
    consumers_sync<BAR>();
    if (tid == 0) {
      const uint32_t n = uint32_t(j - seg_first + 1);
      (*cx.s_last) = atomicAdd(&cx.counters[unit], n) + n == uint32_t(cx.S) ? 1u : 0u;
    }
    consumers_sync<BAR>();
    if ((*cx.s_last)) {
      // This CTA completed the unit.  Its partials sit in the slots of its segments' first
      // chunks: chunk 0 of the unit and every CTA range start inside the unit.
      __threadfence();
      const int64_t u0 = unit * cx.S, P = cx.nvc;
      int64_t c0 = u0 * P / n_chunks;            // the CTA whose range holds chunk u0
      while (c0 + 1 < P && n_chunks * (c0 + 1) / P <= u0) ++c0;
      while (c0 > 0 && n_chunks * c0 / P > u0) --c0;
      const int64_t b = unit / cx.Hkv, kvh = unit % cx.Hkv;
      for (int idx = tid; idx < G * (DA_D / 4); idx += DA_WARPS * 32) {
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
            live[k] = c + k < P && start < u0 + cx.S && start >= u0;
            const int64_t i = (live[k] ? start : u0) * G + gg;
            ml[k] = __ldcg(reinterpret_cast<const float2*>(cx.mlpart + i * 2));
            ov[k] = __ldcg(reinterpret_cast<const float4*>(cx.opart + i * DA_D + d));
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
        *reinterpret_cast<uint2*>(cx.out + (b * cx.Hq + kvh * G + gg) * DA_D + d) =
            make_uint2(pack_bf16x2(num.x * inv, num.y * inv), pack_bf16x2(num.z * inv, num.w * inv));
      }
    }
    consumers_sync<BAR>();   // the merge area is free again
  }
}

}  // namespace enigma_decode
