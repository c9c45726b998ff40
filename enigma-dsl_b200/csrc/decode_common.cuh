// decode_common.cuh — device building blocks of the decode step: the
// GEMM tile constants, bf16 helpers and the split-KV attention (producer and consumer roles,
// each taking its chunk range and pipeline state explicitly).  decode.cu wraps them in
// kernels (one launch per stage, programmatic dependent launches).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace enigma_decode {

using namespace enigma_sm100;

// ============================================================================ GEMM tiles
// The decode GEMMs (decode.cu) compute 128-row (M <= 128) x 64-column tiles over 64-deep
// k-blocks.
constexpr int SK_BM = 128;
constexpr int SK_BK = 64;

// ============================================================================ bf16 helpers
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

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
// Cluster mode: a unit's k <= DA_CL_MAX CTAs merge over distributed shared memory; each
// sends rank 0 one partial of DA_PART bytes ([8][D] fp32 O, then [8] (m, l) pairs).
constexpr int DA_CL_MAX = 4;
constexpr int DA_PART = 8 * DA_D * 4 + 8 * 2 * 4;
constexpr int DA_RECV = (DA_CL_MAX - 1) * DA_PART;
constexpr int DA_SMEM = DA_NST * DA_STAGE + DA_MERGE + DA_RECV + 1024;
constexpr int DA_CTAS_PER_SM = 2;
constexpr int DA_MAX_SEGS = 8;

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

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Named barrier BAR over the DA_WARPS consumer warps only (the producer never joins it).
template <int BAR>
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(DA_WARPS * 32) : "memory");
}

// floor(n c / P) (n c < 2^53) without a 64-bit division, which the GPU runs as a long
// software sequence: a double quotient, then corrected by at most one either way.
__device__ __forceinline__ int64_t range_start(int64_t n, int64_t c, int64_t P) {
  const int64_t x = n * c;
  int64_t q = int64_t(double(x) / double(P));
  if ((q + 1) * P <= x) ++q;
  if (q * P > x) --q;
  return q;
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
  const __nv_bfloat16* kcache;   // [units, cap, D] (cluster mode: the appended key's row)
  const __nv_bfloat16* vcache;
  int Hq, Hkv, cap;
  int L;                    // keys the chunks cover (cluster mode: the cached ones, pos)
  int S, units;             // S: chunk stride per unit
  float scale_log2;
  uint32_t* status;
  int vc, nvc;              // flat mode: range vc of nvc over all units' chunks
  int cl, cl_rank;          // cluster mode (cl > 0): rank cl_rank of the unit's cl CTAs
  int64_t cb, ce;           // this CTA's chunk range [cb, ce)
  uint8_t* stages;          // DA_NST stages, the DA_MERGE merge area, the DA_RECV receive
                            // area (cluster rank 0); 1024-aligned
  uint64_t* recv_bar;       // cluster mode: rank 0's receive barrier
  uint64_t* full;           // [DA_NST]
  uint64_t* empty;          // [DA_NST]
  float (*s_m)[8];          // [DA_WARPS][8]
  float (*s_l)[8];
  uint32_t* s_last;         // bit k: this CTA completed recorded segment k's unit
  int64_t* s_seg_unit;      // [DA_MAX_SEGS] segments written, not yet counted
  uint32_t* s_seg_n;        // [DA_MAX_SEGS] their chunk counts
  __device__ int64_t c_begin() const { return cb; }
  __device__ int64_t c_end() const { return ce; }
};

__device__ inline void attn_init(const AttnCtx& c) {
  for (int s = 0; s < DA_NST; ++s) {
    mbar_init(&c.full[s], 1);
    mbar_init(&c.empty[s], DA_WARPS);
  }
}

// Chunk j of unit `unit` into stage st.
__device__ inline void attn_issue(const AttnCtx& c, int unit, int j, int st) {
  const int32_t row = int32_t(int64_t(unit) * c.cap + j * DA_KEYS);
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
  int unit = int(ci / c.S), j = int(ci % c.S);
  for (; ci < ce && i < DA_NST && j != c.S - 1; ++ci, ++i) {
    attn_issue(c, unit, j, i);
    if (++j == c.S) { j = 0; ++unit; }
  }
}

__device__ inline void attn_produce_rest(const AttnCtx& c, int64_t ci, int i) {
  const int64_t ce = c.c_end();
  int unit = int(ci / c.S), j = int(ci % c.S);
  for (; ci < ce; ++ci, ++i) {
    const int st = i % DA_NST;
    if (!mbar_wait(&c.empty[st], ((i / DA_NST) & 1) ^ 1, c.status)) break;
    attn_issue(c, unit, j, st);
    if (++j == c.S) { j = 0; ++unit; }
  }
}


// Cluster mode, end of the CTA's range (one unit's cached keys): the warps' partials (s_o,
// s_m, s_l) are merged into this CTA's (m, l, O); ranks > 0 send theirs to rank 0 with one
// bulk copy (from the idle ring), rank 0 waits for the cl - 1 copies on its receive barrier,
// merges them in rank order with the appended key and writes the bf16 output.
// G * D / 4 <= 128 items: one per thread.
template <int BAR>
__device__ inline void attn_cluster_merge(const AttnCtx& cx, int64_t unit, int G, int tid,
                                          const float* s_o) {
  const int gg = tid / (DA_D / 4), d = (tid % (DA_D / 4)) * 4;
  const bool has = tid < G * (DA_D / 4);
  float M = -INFINITY, den = 0.f;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  if (has) {
    M = cx.s_m[0][gg];                      // warp 0 always holds a valid key
#pragma unroll
    for (int w = 1; w < DA_WARPS; ++w) M = fmaxf(M, cx.s_m[w][gg]);
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
  }
  float* recv = reinterpret_cast<float*>(cx.stages + DA_NST * DA_STAGE + DA_MERGE);
  if (cx.cl_rank > 0) {
    float* part = reinterpret_cast<float*>(cx.stages);   // the ring is idle
    if (has) {
      *reinterpret_cast<float4*>(part + gg * DA_D + d) = num;
      if (d == 0) *reinterpret_cast<float2*>(part + 8 * DA_D + gg * 2) = make_float2(M, den);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the copy
    consumers_sync<BAR>();
    if (tid == 0) {
      const uint32_t dst = mapa_shared(smem_u32(recv + (cx.cl_rank - 1) * (DA_PART / 4)), 0u);
      const uint32_t bar = mapa_shared(smem_u32(cx.recv_bar), 0u);
      asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"(dst), "r"(smem_u32(part)), "r"(uint32_t(DA_PART)), "r"(bar) : "memory");
    }
    return;
  }
  // Warp-uniform outcome: the shuffles below need every lane of the warp.
  if (!__all_sync(0xffffffffu, mbar_wait(cx.recv_bar, 0, cx.status))) {
    // A peer's partial never arrived (the status word is flagged).  Skip the merge and the
    // store, and give copies still landing in this CTA's shared memory one more bounded
    // wait before the CTA moves on to the final cluster barrier and exits.
    mbar_wait(cx.recv_bar, 0, cx.status);
    return;
  }
  // The appended key (cache row cx.L of the unit) is one more partial: m = q.k in log2
  // units, l = 1, O = v.  The 16 threads of head gg hold 4 dimensions each of the product.
  const int64_t b = int(unit) / cx.Hkv, kvh = int(unit) % cx.Hkv;
  float sn = 0.f;
  float4 vn = make_float4(0.f, 0.f, 0.f, 0.f);
  if (has) {
    const int64_t row = (unit * cx.cap + cx.L) * DA_D + d;
    const uint2 qv = *reinterpret_cast<const uint2*>(cx.q + (b * cx.Hq + kvh * G + gg) * DA_D + d);
    const uint2 kv = *reinterpret_cast<const uint2*>(cx.kcache + row);
    const uint2 vv = *reinterpret_cast<const uint2*>(cx.vcache + row);
    sn = bf16_lo(qv.x) * bf16_lo(kv.x) + bf16_hi(qv.x) * bf16_hi(kv.x) +
         bf16_lo(qv.y) * bf16_lo(kv.y) + bf16_hi(qv.y) * bf16_hi(kv.y);
    vn = make_float4(bf16_lo(vv.x), bf16_hi(vv.x), bf16_lo(vv.y), bf16_hi(vv.y));
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sn += __shfl_xor_sync(0xffffffffu, sn, o);
  sn *= cx.scale_log2;
  if (!has) return;
  float Mx = fmaxf(M, sn);
  for (int p = 0; p < cx.cl - 1; ++p) Mx = fmaxf(Mx, recv[p * (DA_PART / 4) + 8 * DA_D + gg * 2]);
  const float c0 = ex2f(M - Mx);
  num.x *= c0; num.y *= c0; num.z *= c0; num.w *= c0;
  den *= c0;
  for (int p = 0; p < cx.cl - 1; ++p) {
    const float* pp = recv + p * (DA_PART / 4);
    const float2 ml = *reinterpret_cast<const float2*>(pp + 8 * DA_D + gg * 2);
    const float4 v = *reinterpret_cast<const float4*>(pp + gg * DA_D + d);
    const float w = ex2f(ml.x - Mx);
    num.x = fmaf(w, v.x, num.x);
    num.y = fmaf(w, v.y, num.y);
    num.z = fmaf(w, v.z, num.z);
    num.w = fmaf(w, v.w, num.w);
    den = fmaf(w, ml.y, den);
  }
  {
    const float w = ex2f(sn - Mx);
    num.x = fmaf(w, vn.x, num.x);
    num.y = fmaf(w, vn.y, num.y);
    num.z = fmaf(w, vn.z, num.z);
    num.w = fmaf(w, vn.w, num.w);
    den += w;
  }
  const float inv = 1.0f / den;
  *reinterpret_cast<uint2*>(cx.out + (b * cx.Hq + kvh * G + gg) * DA_D + d) =
      make_uint2(pack_bf16x2(num.x * inv, num.y * inv), pack_bf16x2(num.z * inv, num.w * inv));
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
  int nseg = 0;
  int64_t unit = cb / cx.S;
  int j = int(cb % cx.S) - 1;
  int i = -1;
  for (int64_t ci = cb; ci < ce; ++ci) {
    ++i;
    if (++j == cx.S) { j = 0; ++unit; }
    if (unit != cur_unit) {
      // Q fragments: a0 = dims 16 ks + 2t, +1 and a2 = dims 16 ks + 8 + 2t, +1 of head g.
      const bool live = g < G;
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          cx.q + (int64_t(int(unit) / cx.Hkv) * cx.Hq + (int(unit) % cx.Hkv) * G + (live ? g : 0)) * DA_D);
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
    const int st = i % DA_NST;
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
    if (cx.cl > 0) {   // one segment per CTA: merge over the cluster, then done
      attn_cluster_merge<BAR>(cx, unit, G, tid, s_o);
      return;
    }
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
    // Count the segment later: the fence and the counter round trip would stall the ring
    // in the middle of the range.  The recorded segments are counted (one fence) at the end
    // of the range, or when the list is full.
    if (tid == 0) {
      cx.s_seg_unit[nseg] = unit;
      cx.s_seg_n[nseg] = uint32_t(j - seg_first + 1);
    }
    ++nseg;
    if (ci + 1 != ce && nseg < DA_MAX_SEGS) {
      consumers_sync<BAR>();   // the merge area is free again
      continue;
    }
    // The partial stores of all consumer threads happen before the barrier, and the barrier
    // before thread 0's acq_rel counter updates: the release covers them (cumulativity), and
    // the acquire of the update that completes a unit covers every other CTA's partials for
    // the threads that read them after the next barrier.
    consumers_sync<BAR>();
    if (tid == 0) {
      uint32_t bits = 0;
      for (int k = 0; k < nseg; ++k) {
        const uint32_t n = cx.s_seg_n[k];
        if (atom_add_acq_rel_gpu(&cx.counters[cx.s_seg_unit[k]], n) + n == uint32_t(cx.S))
          bits |= 1u << k;
      }
      *cx.s_last = bits;
    }
    consumers_sync<BAR>();
    const uint32_t bits = *cx.s_last;
    for (int sk = 0; sk < nseg; ++sk) {
      if (!((bits >> sk) & 1u)) continue;
      // This CTA completed the unit.  Its partials sit in the slots of its segments' first
      // chunks: chunk 0 of the unit and every CTA range start inside the unit.
      const int64_t mu = cx.s_seg_unit[sk];
      const int64_t u0 = mu * cx.S, P = cx.nvc;
      int64_t c0 = range_start(u0, P, n_chunks);   // the CTA whose range holds chunk u0
      while (c0 + 1 < P && range_start(n_chunks, c0 + 1, P) <= u0) ++c0;
      while (c0 > 0 && range_start(n_chunks, c0, P) > u0) --c0;
      const int64_t b = int(mu) / cx.Hkv, kvh = int(mu) % cx.Hkv;
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
            const int64_t start = c + k == c0 ? u0 : range_start(n_chunks, c + k, P);
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
    nseg = 0;
    consumers_sync<BAR>();   // the merge area is free again
  }
}

}  // namespace enigma_decode
