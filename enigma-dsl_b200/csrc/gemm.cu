// gemm.cu — C[M,N] = A[M,K] * B[K,N] on the sm_100a tensor cores.
//
// A, B, C row-major bf16, fp32 accumulation in TMEM, bf16 output.  This is the
// kernel behind the reference's tiled-GEMM example (examples/async_copy_gemm.py:
// 32-79: async copies of A/B tiles into on-chip memory feeding a tile MMA) and
// the enigma.gemm tile op semantics C = A @ B (enigma/ops/gemm.py:144-167).
//
// Design (one persistent CTA per SM, warp-specialised):
//   warp 0      TMA producer: A tile 128x64 (K-major, 128B swizzle) and B tile
//               64x256 (N-major, four 64x64 boxes, 128B swizzle) per stage,
//               into a 4-stage shared-memory ring guarded by full/empty mbarriers.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and
//               one elected lane issues tcgen05.mma 128x256x16; each stage is
//               released by tcgen05.commit -> empty[stage].
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, convert to bf16,
//               16-byte stores; then release the accumulator so the MMA warp
//               can start the tile after next.  The epilogue of tile i overlaps
//               the main loop of tile i+1.
// Tiles are walked in groups of 8 M-blocks so that consecutive CTAs share B
// columns in L2.  Ragged M/N/K edges are zero-filled by TMA and masked on store.
// Each CTA issues its own TMA loads.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"

namespace {

using namespace enigma_sm100;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;         // 16 KB
constexpr int B_STAGE_BYTES = BK * BN * 2;         // 32 KB
constexpr int B_BOX_BYTES = BK * 64 * 2;           // 8 KB: one 64(N) x 64(K) box
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 2 * BN;                  // double-buffered accumulator
constexpr int GROUP_M = 8;
constexpr int EPI_THREADS = 128;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

struct TileSched {
  int num_m, num_n;
  __device__ __forceinline__ void coords(int t, int& mb, int& nb) const {
    const int per_group = GROUP_M * num_n;
    const int g = t / per_group;
    const int first_m = g * GROUP_M;
    const int gm = min(GROUP_M, num_m - first_m);
    const int r = t - g * per_group;
    mb = first_m + r % gm;
    nb = r / gm;
  }
};

__global__ void __launch_bounds__(THREADS, 1)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, __nv_bfloat16* __restrict__ C,
                    int M, int N, int K, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], EPI_THREADS);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const TileSched sched{(M + BM - 1) / BM, (N + BN - 1) / BN};
  const int num_tiles = sched.num_m * sched.num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (warp == 0) {
    // ---------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        sched.coords(t, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_STAGE_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
          uint8_t* b = sB + stage * B_STAGE_BYTES;
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(b + j * B_BOX_BYTES, &tmB, &full[stage], nb * BN + j * 64, kb * BK);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every stage this thread filled must have landed before the CTA
      // can exit (the MMA warp consumes them; its commits free the slots).
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, /*a_mn=*/false, /*b_mn=*/true);
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, status)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status)) { ok = false; break; }
          tc_fence_after();
          // A: K-major, 128B swizzle atoms of 8 rows x 128 B -> SBO 1024 B; LBO unused.
          // B: N-major, atoms of 8 K-rows x 64 N; next 64-wide N box is 8 KB away (LBO),
          //    next 8 K-rows 1 KB away (SBO).
          const uint64_t da = smem_desc_sw128(a0 + stage * A_STAGE_BYTES, 16, 1024);
          const uint64_t db = smem_desc_sw128(b0 + stage * B_STAGE_BYTES, B_BOX_BYTES, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 B along K inside the swizzled A row; +16 K-rows (2 KB) for B.
            mma_bf16_ss(d, da + uint64_t((kk * 32) >> 4), db + uint64_t((kk * 2048) >> 4), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        mma_commit(&acc_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5 -> TMEM lane quarters 2,3,0,1)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      sched.coords(t, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, status)) break;
      tc_fence_after();
      const int row = mb * BM + row_in_tile;
      const int col0 = nb * BN;
      __nv_bfloat16* crow = C + int64_t(row) * N;
      const uint32_t taddr = tmem_base + acc * BN + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld16(taddr + c, r0);
        tmem_ld16(taddr + c + 16, r1);
        tmem_wait_ld();
        if (row < M && col0 + c < N) {
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            p[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
            p[8 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
          }
          __nv_bfloat16* dst = crow + col0 + c;
          if (col0 + c + 32 <= N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
          } else {
            const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(p);
            for (int i = 0; i < 32 && col0 + c + i < N; ++i) dst[i] = pb[i];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ============================================================================ 2-SM variant
// A cluster of two CTAs (a "CTA pair" on neighbouring SMs) owns one 256x256 tile:
// tcgen05.mma.cta_group::2 (M = 256, N = 256) is issued by the pair's leader (rank 0)
// and reads A rows 0-127 / B columns 0-127 from the leader's shared memory and A rows
// 128-255 / B columns 128-255 from the peer's; each CTA's TMEM holds its own 128 rows
// of the 256-wide accumulator.  Per SM this moves 32 KB of operands per 64-deep K step
// instead of 48 KB for the same FLOPs, easing shared-memory bandwidth.
//   both CTAs, warp 0   TMA of the CTA's A half and B half; completion bytes counted on
//                       the leader's full[stage] barrier (cta_group::2 form of the load)
//   leader, warp 1      MMA issue; releases a stage / publishes an accumulator by
//                       committing to the barrier in both CTAs
//   both CTAs, warps 2-5 epilogue of the CTA's 128 rows (32 per warp, through a
//                       swizzled shared-memory box and a TMA tile store per 64 columns);
//                       arrive on the leader's acc_empty (256 arrivals per accumulator)
constexpr int P_BM = 256;                              // tile rows per pair
constexpr int P_BN = 256;                              // tile columns per pair
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = (P_BM / 2) * BK * 2;         // 16 KB: this CTA's 128 rows
constexpr int P_B_BYTES = BK * (P_BN / 2) * 2;         // 16 KB: this CTA's 128 columns
constexpr int P_STAGE = P_A_BYTES + P_B_BYTES;
// Epilogue staging: per epilogue warp two 32-row x 64-column bf16 boxes (4 KB each, 128-byte
// swizzle) that TMA stores to C while the warp fills the other one.
constexpr int P_C_BOX_BYTES = 32 * 64 * 2;
constexpr int P_C_BYTES = (EPI_THREADS / 32) * 2 * P_C_BOX_BYTES;
constexpr int P_SMEM = P_STAGES * P_STAGE + P_C_BYTES + 1024 + 256;
static_assert(P_SMEM <= 232448, "pair GEMM shared memory");

// HALF: every 256 x 256 tile runs as two 256 x 128 halves (MMA N = 128, one 64-column B box
// per CTA), for problems with fewer tiles than CTA pairs: twice the pairs get work (1024^3:
// 16 tiles -> 32 halves on 32 pairs).  The full-tile instance is used otherwise.
template <bool HALF>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
                      uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * P_A_BYTES;
  uint8_t* sC = smem + P_STAGES * P_STAGE;                 // epilogue staging (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + P_C_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* acc_full = empty + P_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * EPI_THREADS);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated, before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const TileSched sched{(M + P_BM - 1) / P_BM, (N + P_BN - 1) / P_BN};
  constexpr int UW = HALF ? P_BN / 2 : P_BN;            // unit width (columns)
  constexpr int BOXES = UW / 128;                        // 64-column B boxes per CTA
  const int num_tiles = sched.num_m * sched.num_n * (HALF ? 2 : 1);   // work units
  const int num_kb = (K + BK - 1) / BK;
  const int pair_id = int(blockIdx.x) >> 1, num_pairs = int(gridDim.x) >> 1;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (elect_one()) {
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs) {
        int mb, nb;
        sched.coords(HALF ? t >> 1 : t, mb, nb);
        const int n0 = nb * P_BN + (HALF ? (t & 1) * UW : 0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, status)) { ok = false; break; }
          const uint32_t fb = full_leader0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (P_A_BYTES + BOXES * B_BOX_BYTES));
          tma_load_2d_pair(sA + stage * P_A_BYTES, &tmA, fb, kb * BK, mb * P_BM + int(rank) * 128);
          uint8_t* b = sB + stage * P_B_BYTES;
#pragma unroll
          for (int j = 0; j < BOXES; ++j)
            tma_load_2d_pair(b + j * B_BOX_BYTES, &tmB, fb, n0 + int(rank) * (UW / 2) + j * 64,
                             kb * BK);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(P_BM, UW, /*a_mn=*/false, /*b_mn=*/true);
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      const uint32_t empty0_self = smem_u32(&empty[0]), empty0_peer = mapa_shared(empty0_self, peer);
      const uint32_t accf0_self = smem_u32(&acc_full[0]), accf0_peer = mapa_shared(accf0_self, peer);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += num_pairs) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, status)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * P_BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(a0 + stage * P_A_BYTES, 16, 1024);
          const uint64_t db = smem_desc_sw128(b0 + stage * P_B_BYTES, B_BOX_BYTES, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16_ss_pair(d, da + uint64_t((kk * 32) >> 4), db + uint64_t((kk * 2048) >> 4),
                             idesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit_pair(empty0_self + stage * 8);
          mma_commit_pair(empty0_peer + stage * 8);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit_pair(accf0_self + acc * 8);
        mma_commit_pair(accf0_peer + acc * 8);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of each 256-row tile, 32 per
    // warp.  Per 64-column chunk: tcgen05.ld -> bf16 -> a 128-byte-swizzled 32 x 64 box in
    // this warp's staging buffer -> one TMA tile store (clipped at ragged edges), while the
    // warp fills its other buffer.  The accumulator is released once its last chunk is in
    // registers, before the stores complete.
    const int quarter = warp & 3;
    const int row_in_tile = int(rank) * 128 + quarter * 32;    // first row of this warp
    uint8_t* stg = sC + (warp - 2) * 2 * P_C_BOX_BYTES;
    const uint32_t sw = uint32_t(lane & 7);
    const uint32_t acce0_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    int acc = 0, buf = 0;
    uint32_t acc_phase = 0;
    for (int t = pair_id; t < num_tiles; t += num_pairs) {
      int mb, nb;
      sched.coords(HALF ? t >> 1 : t, mb, nb);
      if (!mbar_wait(&acc_full[acc], acc_phase, status)) break;
      tc_fence_after();
      const int row0 = mb * P_BM + row_in_tile;
      const int col0 = nb * P_BN + (HALF ? (t & 1) * UW : 0);
      const uint32_t taddr = tmem_base + acc * P_BN + (uint32_t(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < UW; c += 64) {
        uint32_t r[64];
        tmem_ld32(taddr + c, r);
        tmem_ld32(taddr + c + 32, r + 32);
        tmem_wait_ld();
        if (c + 64 >= UW) {           // every TMEM read of this accumulator is done
          tc_fence_before();
          mbar_arrive_cluster(acce0_leader + acc * 8);
        }
        if (lane == 0) bulk_wait_group_read<1>();   // the store two chunks back has read buf
        __syncwarp();
        uint8_t* box = stg + buf * P_C_BOX_BYTES + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
          v.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
          v.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
          v.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
          *reinterpret_cast<uint4*>(box + ((uint32_t(j) ^ sw) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < M && col0 + c < N) tma_store_2d(&tmC, stg + buf * P_C_BOX_BYTES, col0 + c, row0);
          bulk_commit_group();        // (an empty group when the box lies past M or N)
        }
        buf ^= 1;
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// CUDA-core GEMM for shapes the TMA path cannot describe (row pitch not a
// multiple of 16 bytes, e.g. K = 4).  16x16 output tile per CTA, fp32 accumulate.
template <typename T>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, int M,
                 int N, int K, int accumulate, int trans_a = 0, int trans_b = 0) {
  __shared__ float sa[16][17];
  __shared__ float sb[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    // A is [M, K] row-major, or [K, M] when trans_a; B is [K, N], or [N, K] when trans_b.
    const int64_t ia = trans_a ? int64_t(k0 + tx) * M + row : int64_t(row) * K + k0 + tx;
    const int64_t ib = trans_b ? int64_t(col) * K + k0 + ty : int64_t(k0 + ty) * N + col;
    sa[ty][tx] = (row < M && k0 + tx < K) ? float(A[ia]) : 0.f;
    sb[ty][tx] = (k0 + ty < K && col < N) ? float(B[ib]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(sa[ty][k], sb[k][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) {
    T* dst = C + int64_t(row) * N + col;
    *dst = T(accumulate ? float(*dst) + acc : acc);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

namespace enigma {

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with 128-byte swizzle.
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint64_t row_pitch_elems, uint32_t box_cols, uint32_t box_rows) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t gemm_bf16_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, cudaStream_t s) {
  if (K == 0) return cudaMemsetAsync(C, 0, size_t(M) * size_t(N) * 2, s);
  const bool tma_ok = (K % 8 == 0) && (N % 8 == 0) &&
                      (reinterpret_cast<uintptr_t>(A) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(B) % 16 == 0);
  if (tma_ok) {
    uint32_t* status = device_status();
    if (status == nullptr) return cudaErrorMemoryAllocation;   // the bounded waits need it
    CUtensorMap ta, tb;
    if (!make_tmap_bf16_2d(&ta, A, M, K, K, BK, BM) || !make_tmap_bf16_2d(&tb, B, K, N, N, 64, BK))
      return cudaErrorInvalidValue;
    // Set on every call: the attribute is per device, and the call is cheap.
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    CUtensorMap tc;
    if (M >= 256 && N >= 256 && reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
        make_tmap_bf16_2d(&tc, C, M, N, N, 64, 32)) {
      // CTA-pair kernel: B boxes of the pair's two N halves, A boxes of 128 rows.
      const int64_t ptiles = ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN);
      const bool half = 2 * ptiles <= sm_count() / 2;
      auto kern = half ? gemm_bf16_pair_kernel<true> : gemm_bf16_pair_kernel<false>;
      note_kernel("gemm_bf16_pair_kernel");
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
      if (e != cudaSuccess) return e;
      const int pairs = int(std::min<int64_t>(half ? 2 * ptiles : ptiles, sm_count() / 2));
      kern<<<2 * pairs, THREADS, P_SMEM, s>>>(ta, tb, tc, int(M), int(N), int(K), status);
      return cudaGetLastError();
    }
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = int(tiles < sm_count() ? tiles : sm_count());
    note_kernel("gemm_bf16_tc_kernel");
    gemm_bf16_tc_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(
        ta, tb, static_cast<__nv_bfloat16*>(C), int(M), int(N), int(K), status);
    return cudaGetLastError();
  }
  dim3 grid(unsigned((N + 15) / 16), unsigned((M + 15) / 16));
  note_kernel("gemm_simt_kernel");
  gemm_simt_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B),
      static_cast<__nv_bfloat16*>(C), int(M), int(N), int(K), 0);
  return cudaGetLastError();
}

cudaError_t gemm_f32_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                            int64_t K, bool accumulate, cudaStream_t s) {
  dim3 grid(unsigned((N + 15) / 16), unsigned((M + 15) / 16));
  note_kernel("gemm_simt_kernel");
  gemm_simt_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(A),
                                               static_cast<const float*>(B),
                                               static_cast<float*>(C), int(M), int(N), int(K),
                                               accumulate ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t gemm_f32_trans_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                  int64_t K, bool trans_a, bool trans_b, bool accumulate,
                                  cudaStream_t s) {
  dim3 grid(unsigned((N + 15) / 16), unsigned((M + 15) / 16));
  note_kernel("gemm_simt_kernel");
  gemm_simt_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(A),
                                               static_cast<const float*>(B),
                                               static_cast<float*>(C), int(M), int(N), int(K),
                                               accumulate ? 1 : 0, trans_a ? 1 : 0,
                                               trans_b ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace enigma
