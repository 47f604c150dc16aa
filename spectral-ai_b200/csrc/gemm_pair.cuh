// gemm_pair.cuh — tcgen05 GEMM on CTA pairs (cta_group::2) with the fused
// per-row epilogue of gemm_tc.cuh:  C[m, n] = epi(sum_k A[m, k] * B[n, k]).
//
// A cluster of two CTAs computes a 256 x 256 tile: CTA r loads rows
// m0 + 128 r .. +127 of A and rows n0 + 128 r .. +127 of B (TMA, 128-byte
// swizzle, no multicast; both CTAs' loads complete on the rank-0 CTA's
// barrier), and the rank-0 CTA issues 8 MMAs of M=256, N=256, K=16 per 128-K
// block for both SMs.  Each SM keeps its 128 rows x 256 columns in TMEM (two
// buffers, so the epilogue of one tile overlaps the next tile's MMAs).
//
// Against one CTA per 128 x 256 tile (gemm_tc.cuh): each CTA loads half of B,
// and one barrier wait of the MMA issuer covers 8 MMAs of 128 cycles instead
// of 4 — the issuing thread's waits cost a few hundred cycles each, which the
// longer block hides.
//
// Optional tail n-tile (TAIL): one more tile of TAIL_N = 16 columns per m-tile
// against a second B operand (tmB2, an 8-row box per CTA), handed to
// Epi::tail() — the router's 3-D position.
//
//   warp 0      : TMA producer (each CTA)
//   warp 1      : MMA issuer (rank-0 CTA)
//   warp 2      : TMEM allocator (both CTAs, cta_group::2)
//   warps 4..7  : epilogue, one row per thread (warp w: TMEM lanes 32*(w%4)..)
#pragma once

#include "gemm_tc.cuh"
#include "sm100_pair.cuh"

namespace sb {

constexpr int GP_BM = 256;                         // rows per pair tile (128 per CTA)
constexpr int GP_BN = 256;                         // columns per pair tile (B rows: 128 per CTA)
constexpr int GP_KB = 128;                         // K per block (two 64-wide swizzle atoms)
constexpr int GP_STAGES = 3;
constexpr int GP_ATOM = 128 * 128;                 // 16 KB: 128 rows x 64 K
constexpr int GP_A_BYTES = 2 * GP_ATOM;            // 32 KB per CTA per stage
constexpr int GP_B_BYTES = 2 * GP_ATOM;
constexpr int GP_TAIL_ATOM = 8 * 128;              // tail B: 8 rows per CTA
constexpr int GP_STAGE_BYTES = GP_A_BYTES + GP_B_BYTES;
constexpr int GP_BAR_BYTES = (2 * GP_STAGES + 4) * 8 + 16;
constexpr int GP_SMEM_BYTES = GP_STAGES * GP_STAGE_BYTES + GP_BAR_BYTES + 1024;
constexpr int GP_THREADS = 256;
static_assert(GP_SMEM_BYTES <= 227 * 1024, "shared memory budget");

// D[tmem] (+)= A[smem] * B[smem]^T over the pair: M = 256 (128 rows per SM).
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <class Epi, bool TAIL>
__global__ void __launch_bounds__(GP_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmB2, int M, int N, int K, uint32_t idesc,
                     uint32_t idesc_tail, Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GP_STAGES * GP_STAGE_BYTES);  // rank 0: both CTAs' loads
  uint64_t* empty = full + GP_STAGES;                                                // stage's MMAs completed
  uint64_t* tfull = empty + GP_STAGES;                                               // [2]
  uint64_t* tempty = tfull + 2;                                                      // [2] rank 0: 8 warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (M + GP_BM - 1) / GP_BM;
  const int n_main = (N + GP_BN - 1) / GP_BN;
  const int n_tiles = n_main + (TAIL ? 1 : 0);
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + GP_KB - 1) / GP_KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GP_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // 4 epilogue warps x 2 CTAs
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (each CTA)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if (TAIL) tma_prefetch_desc(&tmB2);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < num_tiles; tile += npairs) {
        const int m0 = (tile / n_tiles) * GP_BM + (int)rank * 128;
        const int nt = tile % n_tiles;
        const bool is_tail = TAIL && nt == n_main;
        const int n0 = nt * GP_BN + (int)rank * 128;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, ST_TIMEOUT_PRODUCER)) goto done;
          uint8_t* st = smem + stage * GP_STAGE_BYTES;
          if (rank == 0)
            mbar_arrive_expect_tx(&full[stage], 2 * (GP_A_BYTES + (is_tail ? 2 * GP_TAIL_ATOM : GP_B_BYTES)));
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(st, &tmA, fb, kb * GP_KB, m0);
          tma_load_2d_pair(st + GP_ATOM, &tmA, fb, kb * GP_KB + 64, m0);
          if (is_tail) {
            tma_load_2d_pair(st + GP_A_BYTES, &tmB2, fb, kb * GP_KB, (int)rank * 8);
            tma_load_2d_pair(st + GP_A_BYTES + GP_TAIL_ATOM, &tmB2, fb, kb * GP_KB + 64, (int)rank * 8);
          } else {
            tma_load_2d_pair(st + GP_A_BYTES, &tmB, fb, kb * GP_KB, n0);
            tma_load_2d_pair(st + GP_A_BYTES + GP_ATOM, &tmB, fb, kb * GP_KB + 64, n0);
          }
          if (++stage == GP_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
        const int acc = local & 1;
        const bool is_tail = TAIL && tile % n_tiles == n_main;
        const uint32_t id = is_tail ? idesc_tail : idesc;
        const uint32_t b_atom = (uint32_t)((is_tail ? GP_TAIL_ATOM : GP_ATOM) >> 4);
        if (!mbar_wait_cluster(&tempty[acc], ((uint32_t)(local >> 1) & 1u) ^ 1u, ST_TIMEOUT_MMA)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * GP_BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, ST_TIMEOUT_MMA)) goto done;
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(smem_u32(smem + stage * GP_STAGE_BYTES));
          const uint64_t bdesc = sdesc_sw128(smem_u32(smem + stage * GP_STAGE_BYTES + GP_A_BYTES));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // K 16k..16k+15: the first or second 64-K atom of each operand
            const uint64_t ak = adesc + (k < 4 ? 2u * k : (uint32_t)(GP_ATOM >> 4) + 2u * (k - 4));
            const uint64_t bk = bdesc + (k < 4 ? 2u * k : b_atom + 2u * (k - 4));
            umma_ss_pair(d_tmem, ak, bk, id, (kb | k) != 0);
          }
          umma_commit_pair(&empty[stage]);
          if (++stage == GP_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit_pair(&tfull[acc]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (each CTA)
    const int q = warp & 3;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
      const int m0 = (tile / n_tiles) * GP_BM + (int)rank * 128;
      const int nt = tile % n_tiles;
      const int n0 = nt * GP_BN;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, ST_TIMEOUT_EPILOGUE)) goto done;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * GP_BN);
      if (TAIL && nt == n_main) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl, r);
        tmem_ld_wait();
        if (row < M) epi.tail(row, r);
      } else {
#pragma unroll 1
        for (int c = 0; c < GP_BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tl + (uint32_t)(c * 32), r);
          tmem_ld_wait();
          const int col0 = n0 + c * 32;
          if (row < M && col0 < N) epi.apply(row, col0, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + (uint32_t)(acc * 8));
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrive or MMA still targets this CTA
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace sb
