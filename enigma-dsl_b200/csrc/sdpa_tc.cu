// sdpa_tc.cu — FlashAttention-style forward on the sm_100a tensor cores.
//
//   O[b,h] = softmax(scale * Q[b,h] K[b,h/g]^T [+ causal mask]) V[b,h/g]
//
// The reference computes the same thing with an online softmax over KV tiles
// on Apple SIMD groups (examples/benchmark_sdpa.py:48-150,
// examples/showcase_attention.py:31-91, check at :150-153).
//
// A work item is two 128-row Q tiles (Q0, Q1) of one (batch, head); the kernel is
// persistent (at most one CTA per SM, items taken in a fixed order, see item_coords) and
// streams 128-key K/V tiles past both tiles of each item:
//
//   warp 0      TMA: Q0, Q1 once per item; K and V tiles into 2-stage rings (128B swizzle,
//               3-D tensor maps [D, S, B*H]: ragged S zero-fills and never reads
//               the next head).  Each CTA loads its own tiles.
//   warp 1      one lane issues tcgen05.mma (fp32 accumulators in TMEM):
//                 S_i = Q_i K_j^T   (SS, M128 N128)          i = 0, 1
//                 O_i += P_i V_j    (TS: P read from TMEM over S_i's columns)
//               in the order S0_0 S1_0 | PV0_0 S0_1 PV1_0 S1_1 | PV0_1 S0_2 ...
//               so the tensor core works on one tile's S / PV while the other
//               tile's softmax runs (ping-pong).  Because tcgen05.commit tracks
//               every earlier MMA of the issuing thread, "S_i(j) done" also means
//               "PV_i(j-1) done": the softmax may touch O_i after that wait.
//   warps 2-5   softmax of Q0, warps 6-9 softmax of Q1; one thread per row:
//               tcgen05.ld the S row, row max (3-input max), s*c - m*c with packed
//               f32x2 FMAs, p = 2^() with the fp32 MUFU exponential, one packed bf16x2
//               convert per key pair for the P operand of the PV MMA, row sum of the
//               fp32 p with packed adds, P stored with tcgen05.st over the first half of
//               S's columns.  The softmax is issue-bound: 5 instructions per key pair.
//               O is rescaled only when a row max grows by more than 2^8 (exact: the
//               numerator and denominator share the stale max; P < 2^8 is far inside
//               bf16's range).  The exponent argument stays fp32: a bf16 argument (the bf16x2
//               MUFU form) loses up to 2^-9 |argument| in log2 units, and with a stale
//               max the largest keys of a row have arguments up to +8 — a peaked
//               softmax (Q scaled x8) then missed a 2e-2 bound.
// All mbarrier waits are bounded (sm100.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace {

using namespace enigma_sm100;

constexpr int BM = 128;            // rows per Q tile (two tiles per CTA)
constexpr int BN = 128;            // keys per KV tile
constexpr int KV_STAGES = 2;
constexpr int THREADS = 384;       // warpgroup 0: TMA warp, MMA warp, 2 idle; WG 1, 2: softmax
// Register split (setmaxnreg): the kernel launches with LAUNCH_REGS per thread
// (384 x 168 = 64512 of the SM's 65536); warpgroup 0 gives back down to WG0_REGS and
// the two softmax warpgroups grow to SOFTMAX_REGS.  128*104 + 256*200 = 64512: the sum
// equals the launch budget exactly (the host refuses to launch if the compiled kernel
// has fewer registers than LAUNCH_REGS, since the increase could then never be granted).
constexpr int LAUNCH_REGS = 168;
constexpr int WG0_REGS = 104;
constexpr int SOFTMAX_REGS = 200;
static_assert(128 * WG0_REGS + 256 * SOFTMAX_REGS <= THREADS * LAUNCH_REGS, "register split");
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays below 2^8

template <int D>
struct Cfg {
  static constexpr int Q_BYTES = BM * D * 2;     // one Q tile
  static constexpr int KV_BYTES = BN * D * 2;    // one K tile == one V tile
  static constexpr int KATOMS = D / 64;          // 128-byte swizzle atoms along D
  static constexpr int SMEM = 2 * Q_BYTES + 2 * KV_STAGES * KV_BYTES + 1024 + 512;  // + barriers
  static constexpr uint32_t TMEM_COLS = 512;     // S0 | S1 | O0 | O1
  static constexpr uint32_t O_COL = 2 * BN;
};

struct Params {
  __nv_bfloat16* O;
  int Sq, Sk, Hq, Hkv, num_ctas_q, nbh;
  float scale_log2;
  int causal;
  uint32_t* status;
  uint32_t* work;   // dynamic work queue counter (zeroed before the launch), or nullptr
  int head_group;   // (batch, head) pairs per group of the item order
};

// ------------------------------------------------------------------ packed fp32 math
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 f2add(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

#ifndef SDPA_HEAD_GROUP
#define SDPA_HEAD_GROUP 8
#endif
constexpr int kHeadGroup = SDPA_HEAD_GROUP;
constexpr int kItemSlots = 4;   // depth of the in-CTA ring of item ids (dynamic schedule)

// Work item t (0 .. items-1) -> (b * Hq + h, query-tile pair).  Groups of kHeadGroup
// (batch, head) pairs; inside a group the heaviest query pairs (late, for causal) of all
// its heads first.  CTAs running at the same time then share a few heads' K / V in L2, and
// the last items are light ones.
__device__ __forceinline__ void item_coords(int t, int nq, int nbh, int hg, int& bh, int& pair) {
  const int grp = t / (hg * nq);
  const int in_grp = t - grp * hg * nq;
  const int gsz = min(hg, nbh - grp * hg);
  pair = nq - 1 - in_grp / gsz;
  bh = grp * hg + in_grp % gsz;
}

// KV tiles query tile i (0, 1) of the pair starting at row q0 needs.
__device__ __forceinline__ int kv_tiles(const Params& p, int q0, int i) {
  int end = p.Sk;                                                  // exclusive
  if (p.causal) end = min(p.Sk, q0 + i * BM + BM - 1 + (p.Sk - p.Sq) + 1);
  if (q0 + i * BM >= p.Sq) end = 0;                                // tile entirely past Sq
  return end > 0 ? (end + BN - 1) / BN : 0;
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1)
sdpa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // Q0 | Q1
  uint8_t* sK = sQ + 2 * C::Q_BYTES;
  uint8_t* sV = sK + KV_STAGES * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KV_STAGES * C::KV_BYTES);
  uint64_t* q_full = bars;                   // [1]
  uint64_t* q_empty = q_full + 1;            // [1] the item's last S MMA has read Q
  uint64_t* k_full = q_empty + 1;            // [KV_STAGES]
  uint64_t* k_empty = k_full + KV_STAGES;
  uint64_t* v_full = k_empty + KV_STAGES;
  uint64_t* v_empty = v_full + KV_STAGES;
  uint64_t* s_full = v_empty + KV_STAGES;    // [2] one per Q tile
  uint64_t* p_full = s_full + 2;             // [2 tiles][2 halves of the keys]
  uint64_t* o_done = p_full + 4;             // [2]
  uint64_t* o_free = o_done + 2;             // [2] the epilogue has read O_i
  uint64_t* item_full = o_free + 2;          // [kItemSlots] an item id was published
  uint64_t* item_empty = item_full + kItemSlots;   // [kItemSlots] every role has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + kItemSlots);
  volatile int* s_item = reinterpret_cast<volatile int*>(tmem_slot + 1);   // [kItemSlots]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Items (one (batch, head) and one pair of 128-row query tiles each) are taken in the
  // order item_coords gives, CTA c taking items c, c + gridDim.x, ...  With one item per
  // CTA (grid = items) this is the plain one-CTA-per-pair launch; with fewer CTAs the
  // kernel is persistent and each CTA's next item overlaps the current one's tail: its Q
  // loads once the last S MMA has read Q, its S MMAs start while the epilogue drains O,
  // and its first PV waits only for that drain (o_free).
  const int nq = p.num_ctas_q, nbh = p.nbh, items = nq * nbh;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[2 * i], 128);
      mbar_init(&p_full[2 * i + 1], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 128);
    }
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 1 + 256);    // the MMA thread and the 256 softmax threads
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The k-th item of this CTA.  Static: blockIdx.x + k * gridDim.x.  Dynamic (p.work set):
  // the producer takes the next item from the device-wide counter and publishes it in a
  // small ring; the MMA thread and the softmax threads read it from there, in order.  An id
  // >= items ends the CTA's loop.
  auto fetch_item = [&](int k) -> int {     // producer
    if (p.work == nullptr) return int(blockIdx.x) + k * int(gridDim.x);
    const int slot = k % kItemSlots;
    if (!mbar_wait(&item_empty[slot], ((k / kItemSlots) & 1) ^ 1, p.status)) return items;
    const int t = int(atomicAdd(p.work, 1u));
    s_item[slot] = t;
    mbar_arrive(&item_full[slot]);
    return t;
  };
  auto take_item = [&](int k) -> int {      // MMA thread, softmax threads
    if (p.work == nullptr) return int(blockIdx.x) + k * int(gridDim.x);
    const int slot = k % kItemSlots;
    if (!mbar_wait(&item_full[slot], (k / kItemSlots) & 1, p.status)) return items;
    const int t = s_item[slot];
    mbar_arrive(&item_empty[slot]);
    return t;
  };

  if (warp < 4) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(WG0_REGS));
   if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int jg = 0, it = 0;                    // KV tiles loaded so far; items with work
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = fetch_item(k);
        if (t >= items) break;
        int bh, pair;
        item_coords(t, nq, nbh, p.head_group, bh, pair);
        const int q0 = pair * 2 * BM;
        const int n_all = max(kv_tiles(p, q0, 0), kv_tiles(p, q0, 1));
        if (n_all == 0) continue;
        const int b = bh / p.Hq, h = bh % p.Hq;
        const int bhk = b * p.Hkv + h / (p.Hq / p.Hkv);
        // The previous item's last S MMA has read Q.
        if (it > 0 && !mbar_wait(q_empty, (it - 1) & 1, p.status)) break;
        mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int a = 0; a < C::KATOMS; ++a)
            tma_load_3d(sQ + i * C::Q_BYTES + a * BM * 128, &tmQ, q_full, a * 64, q0 + i * BM, bh);
        for (int j = 0; j < n_all; ++j, ++jg) {
          const int s = jg % KV_STAGES;
          const uint32_t ph = (jg / KV_STAGES) & 1;
          if (!mbar_wait(&k_empty[s], ph ^ 1, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
          for (int a = 0; a < C::KATOMS; ++a)
            tma_load_3d(sK + s * C::KV_BYTES + a * BN * 128, &tmK, &k_full[s], a * 64, j * BN, bhk);
          if (!mbar_wait(&v_empty[s], ph ^ 1, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
          for (int a = 0; a < C::KATOMS; ++a)
            tma_load_3d(sV + s * C::KV_BYTES + a * BN * 128, &tmV, &v_full[s], a * 64, j * BN, bhk);
        }
        ++it;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BM, D, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      // Running counts across items (barrier phases): KV tiles consumed, items with work,
      // PV tiles issued per Q tile, and items whose O_i accumulated per Q tile.
      int jg = 0, it = 0;
      int pv_g[2] = {0, 0}, acc_items[2] = {0, 0};
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = take_item(k);
        if (t >= items) break;
        int bh, pair;
        item_coords(t, nq, nbh, p.head_group, bh, pair);
        const int q0 = pair * 2 * BM;
        const int n_kv[2] = {kv_tiles(p, q0, 0), kv_tiles(p, q0, 1)};
        const int n_all = max(n_kv[0], n_kv[1]);
        if (n_all == 0) continue;
        if (!mbar_wait(q_full, it & 1, p.status)) break;
        // S_i(j) = Q_i K_j^T into S buffer i.
        auto issue_s = [&](int i, int jgl) {
          const int s = jgl % KV_STAGES;
          const uint32_t s_tmem = tmem + uint32_t(i * BN);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t offq = i * C::Q_BYTES + (kk / 4) * (BM * 128) + (kk % 4) * 32;
            const uint32_t offk = s * C::KV_BYTES + (kk / 4) * (BN * 128) + (kk % 4) * 32;
            mma_bf16_ss(s_tmem, smem_desc_sw128(q_addr + offq, 16, 1024),
                        smem_desc_sw128(k_addr + offk, 16, 1024), idesc_s, kk != 0 ? 1u : 0u);
          }
          mma_commit(&s_full[i]);
        };
        // O_i += P_i(j) V_j, P_i(j) read from TMEM over S buffer i.  P arrives in two halves
        // (keys 0-63, 64-127) so the first half's MMAs start while the softmax finishes the
        // second.  The item's first PV overwrites O_i, so it waits until the previous
        // item's epilogue has read O_i.
        auto issue_pv = [&](int i, int j, int jgl) -> bool {
          const int s = jgl % KV_STAGES;
          if (!mbar_wait(&v_full[s], (jgl / KV_STAGES) & 1, p.status)) return false;
          if (j == 0 && acc_items[i] > 0 &&
              !mbar_wait(&o_free[i], (acc_items[i] - 1) & 1, p.status))
            return false;
          const uint32_t p_tmem = tmem + uint32_t(i * BN);
          const uint64_t dv = smem_desc_sw128(v_addr + s * C::KV_BYTES, BN * 128, 1024);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            if (!mbar_wait(&p_full[2 * i + half], pv_g[i] & 1, p.status)) return false;
            tc_fence_after();
#pragma unroll
            for (int kk = half * 4; kk < half * 4 + 4; ++kk)
              mma_bf16_ts(tmem + C::O_COL + i * D, p_tmem + kk * 8,
                          dv + uint64_t((kk * 2048) >> 4), idesc_o, (j | kk) != 0 ? 1u : 0u);
          }
          ++pv_g[i];
          return true;
        };
        for (int j = 0; j <= n_all && ok; ++j) {
          const bool have_k = j < n_all;
          if (have_k) {
            if (!mbar_wait(&k_full[(jg + j) % KV_STAGES], ((jg + j) / KV_STAGES) & 1, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
#pragma unroll
          for (int i = 0; i < 2 && ok; ++i) {
            if (j >= 1 && j - 1 < n_kv[i]) {
              ok = issue_pv(i, j - 1, jg + j - 1);
              if (ok && j == n_kv[i]) {
                mma_commit(&o_done[i]);
                ++acc_items[i];
              }
            }
            if (ok && have_k && j < n_kv[i]) issue_s(i, jg + j);
          }
          if (!ok) break;
          if (have_k) mma_commit(&k_empty[(jg + j) % KV_STAGES]);
          if (j == n_all - 1) mma_commit(q_empty);    // the item's last S MMA was just issued
          if (j >= 1) mma_commit(&v_empty[(jg + j - 1) % KV_STAGES]);
        }
        jg += n_all;
        ++it;
      }
    }
    __syncwarp();
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(SOFTMAX_REGS));
    // ------------------------------------------------------------ softmax / epilogue
    const int ti = (warp - 4) >> 2;           // Q tile of this warpgroup
    const int quarter = warp & 3;             // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;        // row of the tile owned by this thread
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + uint32_t(ti * BN);
    const uint32_t o_addr = tmem + lane_off + C::O_COL + uint32_t(ti * D);
    const float c = p.scale_log2;
    int sg = 0, acc_items = 0;                // S tiles seen, items whose O accumulated
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int t = take_item(k);
      if (t >= items) break;
      int bh, pair;
      item_coords(t, nq, nbh, p.head_group, bh, pair);
      const int q0 = pair * 2 * BM;
      const int n_my = kv_tiles(p, q0, ti);
      if (max(kv_tiles(p, q0, 0), kv_tiles(p, q0, 1)) == 0) continue;
      const int qi = q0 + ti * BM + r;        // query index
      float m_used = -INFINITY, l = 0.f;      // m in raw score units
      for (int j = 0; j < n_my && ok; ++j, ++sg) {
        if (!mbar_wait(&s_full[ti], sg & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        float x[BN];
#pragma unroll
        for (int k = 0; k < BN; k += 32) tmem_ld32(s_addr + k, reinterpret_cast<uint32_t*>(&x[k]));
        tmem_wait_ld();
        // Keys past the sequence end and, for causal, past this row's diagonal are masked.
        const int k0 = j * BN;
        int lim = p.Sk - k0;
        if (p.causal) lim = min(lim, qi + (p.Sk - p.Sq) - k0 + 1);
        // Warp-uniform: the exp loop below holds warp-collective tcgen05.st.
        const bool masked = __any_sync(0xffffffffu, lim < BN);
        if (masked) {
#pragma unroll
          for (int k = 0; k < BN; ++k) x[k] = (k < lim) ? x[k] : -INFINITY;
        }
        // Row max: four independent 3-input-max chains, then combined.
        float mq[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
        for (int k = 4; k + 8 <= BN; k += 8) {   // x[4 .. BN - 5]
#pragma unroll
          for (int u = 0; u < 4; ++u) mq[u] = max3f(mq[u], x[k + u], x[k + 4 + u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) mq[u] = fmaxf(mq[u], x[BN - 4 + u]);   // x[BN - 4 .. BN - 1]
        const float mx = max3f(mq[0], mq[1], fmaxf(mq[2], mq[3]));
        const float m_new = fmaxf(m_used, mx);
        // tcgen05.ld/st are warp-collective: the lazy-rescale decision is taken per warp.
        const bool need = (j > 0) && ((m_new - m_used) * c > kRescaleThreshold);
        if (j == 0) {
          m_used = m_new;
        } else if (__any_sync(0xffffffffu, need)) {
          // "S_i(j) done" implies PV_i(j-1) done (commit order), so O is complete here.
          const float f = need ? ex2((m_used - m_new) * c) : 1.0f;   // m_used = -inf: f = 0
          l *= f;
#pragma unroll 1
          for (int k = 0; k < D; k += 16) {
            uint32_t o[16];
            tmem_ld16(o_addr + k, o);
            tmem_wait_ld();
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int t2 = 0; t2 < 8; ++t2) {
              lo[t2] = __float_as_uint(__uint_as_float(o[t2]) * f);
              hi[t2] = __float_as_uint(__uint_as_float(o[8 + t2]) * f);
            }
            tmem_st8(o_addr + k, lo);
            tmem_st8(o_addr + k + 8, hi);
          }
          tmem_wait_st();
          if (need) m_used = m_new;
        }
        const float mc = (m_used == -INFINITY) ? 0.f : m_used * c;
        const float2 cc = make_float2(c, c), nmc = make_float2(-mc, -mc);
        float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};    // four independent accumulation chains
        // exp, row sum, P store: p = 2^(s c - m c) in fp32, summed in fp32, stored as bf16
        // pairs (the PV MMA weights V with p rounded to bf16; the sum differs from the sum of
        // the rounded values by at most 2^-9 relative).
#pragma unroll
        for (int k = 0; k < BN; k += 16) {
          uint32_t pk[8];
#pragma unroll
          for (int t2 = 0; t2 < 8; ++t2) {
            const float2 y = f2fma(make_float2(x[k + 2 * t2], x[k + 2 * t2 + 1]), cc, nmc);
            const float2 e = make_float2(ex2(y.x), ex2(y.y));
            sum2[t2 & 3] = f2add(sum2[t2 & 3], e);
            pk[t2] = pack_bf16x2(e.x, e.y);
          }
          tmem_st8(s_addr + k / 2, pk);        // P (bf16 pairs) over S's first 64 columns
          if (k == BN / 2 - 16 || k == BN - 16) {  // a half of the keys is done: release it
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[2 * ti + (k == BN - 16 ? 1 : 0)]);
          }
        }
        const float2 s01 = f2add(sum2[0], sum2[1]), s23 = f2add(sum2[2], sum2[3]);
        l += (s01.x + s23.x) + (s01.y + s23.y);
      }
      if (!ok) break;
      // Epilogue: O / l, bf16, straight to global (each thread one 2*D-byte row).
      if (n_my > 0) {
        ok = mbar_wait(&o_done[ti], acc_items & 1, p.status);
        if (!ok) break;
        tc_fence_after();
      }
      const bool live = qi < p.Sq;
      const float inv = (n_my > 0 && l > 0.f) ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = p.O + (int64_t(bh) * p.Sq + (live ? qi : 0)) * D;
#pragma unroll 1
      for (int k = 0; k < D; k += 16) {
        uint32_t o[16];
        if (n_my > 0) {  // warp-uniform: the collective load runs on every lane
          tmem_ld16(o_addr + k, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int t2 = 0; t2 < 16; ++t2) o[t2] = 0u;
        }
        uint4 w0, w1;
        w0.x = pack_bf16x2(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv);
        w0.y = pack_bf16x2(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv);
        w0.z = pack_bf16x2(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv);
        w0.w = pack_bf16x2(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv);
        w1.x = pack_bf16x2(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv);
        w1.y = pack_bf16x2(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv);
        w1.z = pack_bf16x2(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv);
        w1.w = pack_bf16x2(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv);
        if (live) {
          reinterpret_cast<uint4*>(orow + k)[0] = w0;
          reinterpret_cast<uint4*>(orow + k)[1] = w1;
        }
      }
      if (n_my > 0) {
        // O_i has been read: the next item's first PV may overwrite it.
        tc_fence_before();
        mbar_arrive(&o_free[ti]);
        ++acc_items;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [D, S, BH] bf16 view of a contiguous [BH, S, D] tensor; 64 x box_rows x 1 boxes.
bool make_map_3d(CUtensorMap* m, const void* base, int64_t D, int64_t S, int64_t BH,
                 uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(S), cuuint64_t(BH)};
  cuuint64_t strides[2] = {cuuint64_t(D * 2), cuuint64_t(S * D * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
cudaError_t launch_tc(const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t Hq,
                      int64_t Hkv, int64_t Sq, int64_t Sk, float scale, bool causal,
                      cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  // Q boxes are BM rows (one Q tile), K / V boxes BN rows (one KV tile): the byte counts
  // the producer expects (Q_BYTES, KV_BYTES) are exactly what these boxes deliver.
  if (!make_map_3d(&mq, Q, D, Sq, B * Hq, BM) || !make_map_3d(&mk, K, D, Sk, B * Hkv, BN) ||
      !make_map_3d(&mv, V, D, Sk, B * Hkv, BN))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sdpa_fwd_tc_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM);
  if (e != cudaSuccess) return e;
  static int regs[2] = {-1, -1};
  int& nreg = regs[D == 128 ? 1 : 0];
  if (nreg < 0) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, sdpa_fwd_tc_kernel<D>);
    if (e != cudaSuccess) return e;
    nreg = fa.numRegs;
  }
  if (nreg < LAUNCH_REGS) return cudaErrorInvalidConfiguration;  // split could not be granted
  Params p;
  p.O = static_cast<__nv_bfloat16*>(O);
  p.Sq = int(Sq);
  p.Sk = int(Sk);
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.num_ctas_q = int((Sq + 2 * BM - 1) / (2 * BM));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.nbh = int(B * Hq);
  p.status = enigma::device_status();
  if (p.status == nullptr) return cudaErrorMemoryAllocation;   // the bounded waits need it
  // Persistent: at most one CTA per SM walking the items, so the per-CTA start-up
  // (barriers, TMEM, the first Q / K round trip) and tail are paid once per SM and the next
  // item overlaps the current one's tail.  Measured against one CTA per item: +24 % causal /
  // +15 % non-causal at S = 1024, +10 % / +8 % at 2048, +1-3 % at 4096, even at 8192.
  const int64_t items = int64_t(p.num_ctas_q) * B * Hq;
  const int64_t ctas = std::min<int64_t>(items, enigma::sm_count());
  // Causal items differ in cost (late query pairs see more keys): CTAs take items from a
  // device-wide counter in the item order instead of a fixed stride, so the SMs finish
  // together; the counter pair is zeroed on the stream before the launch.  Up to S = 2048
  // the order groups 32 heads (K/V of 32 heads still fit L2 comfortably, and the heavy items
  // of more heads start first), from 4096 on 8.  Measured (same box): S = 2048 874 -> 911
  // TFLOP/s, 4096 1023 -> 1048, 8192 +0-4 %, 1024 unchanged; non-causal items are equal and
  // keep the fixed stride.
  p.work = nullptr;
  p.head_group = Sq <= 2048 ? 32 : kHeadGroup;
  const bool dyn = causal;
  if (dyn && items > ctas) {
    p.work = enigma::work_counters();
    if (p.work == nullptr) return cudaErrorMemoryAllocation;
    e = cudaMemsetAsync(p.work, 0, 2 * sizeof(uint32_t), s);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid(static_cast<unsigned>(ctas));
  sdpa_fwd_tc_kernel<D><<<grid, THREADS, Cfg<D>::SMEM, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace

namespace enigma {
// True when the tensor-core kernel takes this shape.
bool sdpa_tc_supported(const void* Q, const void* K, const void* V, const void* O, int64_t B,
                       int64_t Hq, int64_t Sq, int64_t Sk, int64_t D) {
  auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return (D == 64 || D == 128) && a16(Q) && a16(K) && a16(V) && a16(O) && B * Hq <= 65535 &&
         Sq < (1ll << 31) && Sk < (1ll << 31);
}

cudaError_t sdpa_tc_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                                float scale, bool causal, cudaStream_t s) {
  if (D == 128) return launch_tc<128>(Q, K, V, O, B, Hq, Hkv, Sq, Sk, scale, causal, s);
  return launch_tc<64>(Q, K, V, O, B, Hq, Hkv, Sq, Sk, scale, causal, s);
}
}  // namespace enigma
