// sdpa_tc.cu — FlashAttention-style forward on the sm_100a tensor cores.
//
//   O[b,h] = softmax(scale * Q[b,h] K[b,h/g]^T [+ causal mask]) V[b,h/g]
//
// The reference computes the same thing with an online softmax over KV tiles
// on Apple SIMD groups (examples/benchmark_sdpa.py:48-150,
// examples/showcase_attention.py:31-91, check at :150-153).  Here each CTA owns
// one 128-row Q tile of one (batch, head) and streams 128-key K/V tiles:
//
//   warp 0     TMA: Q once; K and V tiles into 2-stage rings (128B swizzle,
//              3-D tensor maps [D, S, B*H] so ragged S edges zero-fill and
//              never read the next head).  No multicast.
//   warp 1     one lane issues tcgen05.mma:
//                S_j = Q K_j^T      (SS, M128 N128, fp32 in TMEM, 2 buffers)
//                O  += P_j V_j      (TS: P read from TMEM, V MN-major from smem)
//              in the order S_0, S_1, PV_0, S_2, PV_1, ... so the tensor core
//              computes S_{j+1} and PV_{j-1} while the softmax works on S_j.
//   warps 2-5  softmax, one thread per Q row: tcgen05.ld the S row, mask,
//              running max in the log2 domain, p = 2^(x - m) with ex2.approx,
//              row sum, P packed to bf16 and stored with tcgen05.st over the
//              first half of S's own columns.  O is rescaled only when the
//              running max grows by more than 8 (a factor 256), which keeps the
//              result exact (numerator and denominator share the stale max)
//              and makes the TMEM read-modify-write of O rare.
// All mbarrier waits are bounded (sm100.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace {

using namespace enigma_sm100;

constexpr int BM = 128;            // query rows per CTA
constexpr int BN = 128;            // keys per KV tile
constexpr int KV_STAGES = 2;
constexpr int THREADS = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
struct Cfg {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;   // one K tile == one V tile
  static constexpr int KATOMS = D / 64;          // 128-byte swizzle atoms along D
  static constexpr int SMEM = Q_BYTES + 2 * KV_STAGES * KV_BYTES + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 512;     // S0 | S1 | O (| unused)
  static constexpr uint32_t O_COL = 2 * BN;
};

struct Params {
  __nv_bfloat16* O;
  int Sq, Sk, Hq, Hkv, num_q_tiles;
  float scale_log2;
  int causal;
  uint32_t* status;
};

template <int D>
__global__ void __launch_bounds__(THREADS, 1)
sdpa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;
  uint8_t* sV = sK + KV_STAGES * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KV_STAGES * C::KV_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + KV_STAGES;
  uint64_t* v_full = k_empty + KV_STAGES;
  uint64_t* v_empty = v_full + KV_STAGES;
  uint64_t* s_full = v_empty + KV_STAGES;   // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_done = p_full + 2;            // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Heavy (late, for causal) query tiles first.
  const int qb = p.num_q_tiles - 1 - int(blockIdx.x);
  const int bh = int(blockIdx.y);             // b * Hq + h
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int bhk = b * p.Hkv + h / (p.Hq / p.Hkv);
  const int q0 = qb * BM;
  const int diag = p.Sk - p.Sq;               // key j visible to query i iff j <= i + diag
  int kv_end = p.Sk;                          // exclusive
  if (p.causal) kv_end = min(p.Sk, q0 + BM - 1 + diag + 1);
  const int n_kv = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
    }
    mbar_init(o_done, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one() && n_kv > 0) {
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int a = 0; a < C::KATOMS; ++a)
        tma_load_3d(sQ + a * BM * 128, &tmQ, q_full, a * 64, q0, bh);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        if (!mbar_wait(&k_empty[s], ph ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < C::KATOMS; ++a)
          tma_load_3d(sK + s * C::KV_BYTES + a * BN * 128, &tmK, &k_full[s], a * 64, j * BN, bhk);
        if (!mbar_wait(&v_empty[s], ph ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < C::KATOMS; ++a)
          tma_load_3d(sV + s * C::KV_BYTES + a * BN * 128, &tmV, &v_full[s], a * 64, j * BN, bhk);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BM, D, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(q_full, 0, p.status);
      auto issue_pv = [&](int i) -> bool {
        const int s = i % KV_STAGES;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, p.status)) return false;
        if (!mbar_wait(&v_full[s], (i / KV_STAGES) & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + uint32_t((i & 1) * BN);
        const uint64_t dv = smem_desc_sw128(v_addr + s * C::KV_BYTES, BN * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_bf16_ts(tmem + C::O_COL, p_tmem + kk * 8, dv + uint64_t((kk * 2048) >> 4), idesc_o,
                      (i | kk) != 0 ? 1u : 0u);
        mma_commit(&v_empty[s]);
        mma_commit(o_done);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % KV_STAGES;
        if (!mbar_wait(&k_full[s], (j / KV_STAGES) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t s_tmem = tmem + uint32_t((j & 1) * BN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * (BM * 128) + (kk % 4) * 32;
          const uint32_t offk = (kk / 4) * (BN * 128) + (kk % 4) * 32;
          mma_bf16_ss(s_tmem, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + s * C::KV_BYTES + offk, 16, 1024), idesc_s,
                      kk != 0 ? 1u : 0u);
        }
        mma_commit(&k_empty[s]);
        mma_commit(&s_full[j & 1]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n_kv - 1);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // row of the Q tile owned by this thread
    const int qi = q0 + r;                    // query index
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_off + uint32_t((j & 1) * BN);
      float x[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 16) tmem_ld16(s_addr + c, *reinterpret_cast<uint32_t(*)[16]>(&x[c]));
      tmem_wait_ld();
      // Mask keys past the sequence end and, for causal, past this row's diagonal.
      const int k0 = j * BN;
      int lim = p.Sk - k0;                                // keys [k0, k0+lim) are valid
      if (p.causal) lim = min(lim, qi + (p.Sk - p.Sq) - k0 + 1);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        x[c] = (c < lim) ? x[c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      const float m_new = fmaxf(m_used, mx);
      // tcgen05.ld/st are warp-collective, so the rescale decision is taken per warp:
      // if any row of the warp needs it, every lane rewrites its O row (factor 1
      // for rows that keep their max).
      const bool need = (j > 0) && (m_new > m_used + kRescaleThreshold);
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, need)) {
        // O holds PV_0..PV_{j-1}; wait for PV_{j-1} before rewriting it.
        if (!mbar_wait(o_done, (j - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const float f = need ? ex2(m_used - m_new) : 1.0f;  // m_used may be -inf: f = 0
        l *= f;
        const uint32_t o_addr = tmem + lane_off + C::O_COL;
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          uint32_t o[16];
          tmem_ld16(o_addr + c, o);
          tmem_wait_ld();
          uint32_t lo[8], hi[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            lo[t] = __float_as_uint(__uint_as_float(o[t]) * f);
            hi[t] = __float_as_uint(__uint_as_float(o[8 + t]) * f);
          }
          tmem_st8(o_addr + c, lo);
          tmem_st8(o_addr + c + 8, hi);
        }
        tmem_wait_st();
        if (need) m_used = m_new;
      }
      const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
      float sum = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float a = ex2(x[c] - m_eff), bb = ex2(x[c + 1] - m_eff);
        sum += a + bb;
        pk[c / 2] = pack_bf16x2(a, bb);
      }
      l += sum;
#pragma unroll
      for (int c = 0; c < BN / 2; c += 8)
        tmem_st8(s_addr + c, *reinterpret_cast<const uint32_t(*)[8]>(&pk[c]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    // Epilogue: O / l, bf16, straight to global (each thread one 2*D-byte row).
    if (ok && n_kv > 0) ok = mbar_wait(o_done, (n_kv - 1) & 1, p.status);
    if (ok) {
      tc_fence_after();
      const bool live = qi < p.Sq;
      const float inv = (n_kv > 0 && l > 0.f) ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = p.O + (int64_t(bh) * p.Sq + (live ? qi : 0)) * D;
      const uint32_t o_addr = tmem + lane_off + C::O_COL;
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        uint32_t o[16];
        if (n_kv > 0) {  // CTA-uniform: the warp-collective load runs on every lane
          tmem_ld16(o_addr + c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = 0u;
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
          reinterpret_cast<uint4*>(orow + c)[0] = w0;
          reinterpret_cast<uint4*>(orow + c)[1] = w1;
        }
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

// [D, S, BH] bf16 view of a contiguous [BH, S, D] tensor; 64 x 128 x 1 boxes.
bool make_map_3d(CUtensorMap* m, const void* base, int64_t D, int64_t S, int64_t BH) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(S), cuuint64_t(BH)};
  cuuint64_t strides[2] = {cuuint64_t(D * 2), cuuint64_t(S * D * 2)};
  cuuint32_t box[3] = {64, 128, 1};
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
  if (!make_map_3d(&mq, Q, D, Sq, B * Hq) || !make_map_3d(&mk, K, D, Sk, B * Hkv) ||
      !make_map_3d(&mv, V, D, Sk, B * Hkv))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sdpa_fwd_tc_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM);
  if (e != cudaSuccess) return e;
  Params p;
  p.O = static_cast<__nv_bfloat16*>(O);
  p.Sq = int(Sq);
  p.Sk = int(Sk);
  p.Hq = int(Hq);
  p.Hkv = int(Hkv);
  p.num_q_tiles = int((Sq + BM - 1) / BM);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.status = enigma::device_status();
  dim3 grid(unsigned(p.num_q_tiles), unsigned(B * Hq));
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
