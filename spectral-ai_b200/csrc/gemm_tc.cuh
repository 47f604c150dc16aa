// gemm_tc.cuh — persistent, warp-specialised tcgen05 GEMM for sm_100a with a
// fused per-row epilogue:  C[m, n] = epi(sum_k A[m, k] * B[n, k]).
//
//   A [M, K], B [N, K]: 16-bit (bf16 or fp16), row-major with K contiguous
//   (the nn.Linear weight layout), both loaded by TMA (no multicast) into
//   128-byte-swizzled K-major tiles.  Accumulators live in TMEM (fp32), two
//   buffers of BN columns so the epilogue of tile i overlaps the MMAs of i+1.
//
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : MMA issuer   (one elected lane)
//   warp 2      : TMEM allocator
//   warps 4..7  : epilogue, warp w reads TMEM lanes 32*(w%4) .. +31 (one row per thread)
#pragma once

#include "sm100.cuh"

#include <type_traits>

namespace sb {

// An epilogue that needs whole rows (one n-tile covers N) declares
// `static constexpr bool kWholeRow = true` and `apply_row(taddr, row, valid)`,
// which reads the row's BN accumulator columns from TMEM itself (every lane of
// the warp calls it; `valid` says whether the row exists).
template <class E, class = void>
struct EpiWholeRow {
  static constexpr bool value = false;
};
template <class E>
struct EpiWholeRow<E, std::void_t<decltype(E::kWholeRow)>> {
  static constexpr bool value = E::kWholeRow;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int GEMM_THREADS = 256;

constexpr uint32_t pow2_at_least(uint32_t v) {
  uint32_t p = 32;
  while (p < v) p <<= 1;
  return p;
}

// Optional tail n-tile: after the ceil(N/BN) regular n-tiles of every m-tile
// the kernel runs one more tile of TAIL_N columns against a second B operand
// (tmB2, a TAIL_N-row box) and hands it to Epi::tail().  The router uses it to
// compute the 3-D position from the same A rows as the encoder GEMM.
constexpr int TAIL_N = 16;

template <int BN, int STAGES>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int TAIL_B_BYTES = TAIL_N * GEMM_BK * 2;
  static constexpr int TILE_BYTES = STAGES * (A_BYTES + B_BYTES);
  static constexpr int BAR_BYTES = (2 * STAGES + 4) * 8 + 16;
  static constexpr int SMEM_BYTES = TILE_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = pow2_at_least(2 * BN);
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(TMEM_COLS <= 512, "TMEM columns");
  static_assert(B_BYTES % 1024 == 0, "B tile must keep 1024-byte alignment");
};

// Warp-uniform bounded wait: every lane polls (sleeping between polls), the
// decision is made together.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, unsigned code) {
  const uint32_t a = smem_u32(bar);
  if (__all_sync(0xffffffffu, mbar_try_wait(a, parity))) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    const bool ok = mbar_try_wait_sleep(a, parity, SB_WAIT_SLEEP_NS);
    if (__all_sync(0xffffffffu, ok)) return true;
    const bool late = globaltimer() - t0 > SB_WAIT_LIMIT_NS;
    if (__any_sync(0xffffffffu, late)) {
      if ((threadIdx.x & 31) == 0) set_status(code);
      return false;
    }
  }
}

template <int BN, int STAGES, class Epi, bool TAIL = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmB2, int M, int N, int K, uint32_t idesc,
                   uint32_t idesc_tail, Epi epi) {
  using C = GemmCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + GEMM_BM - 1) / GEMM_BM;
  const int n_main = (N + BN - 1) / BN;
  const int n_tiles = n_main + (TAIL ? 1 : 0);
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + GEMM_BK - 1) / GEMM_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      if (TAIL) tma_prefetch_desc(&tmB2);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * GEMM_BM;
        const int nt = tile % n_tiles;
        const bool is_tail = TAIL && nt == n_main;
        const int n0 = nt * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, ST_TIMEOUT_PRODUCER)) goto done;
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES + (is_tail ? C::TAIL_B_BYTES : C::B_BYTES));
          tma_load_2d(a_tiles + stage * C::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, m0);
          if (is_tail)
            tma_load_2d(b_tiles + stage * C::B_BYTES, &tmB2, &full[stage], kb * GEMM_BK, 0);
          else
            tma_load_2d(b_tiles + stage * C::B_BYTES, &tmB, &full[stage], kb * GEMM_BK, n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
        const uint32_t id = (TAIL && tile % n_tiles == n_main) ? idesc_tail : idesc;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, ST_TIMEOUT_MMA)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, ST_TIMEOUT_MMA)) goto done;
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128(smem_u32(a_tiles + stage * C::A_BYTES));
          const uint64_t bdesc = sdesc_sw128(smem_u32(b_tiles + stage * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k)
            umma_f16(d_tmem, adesc + 2u * k, bdesc + 2u * k, id, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
      const int m0 = (tile / n_tiles) * GEMM_BM;
      const int nt = tile % n_tiles;
      const int n0 = nt * BN;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, ST_TIMEOUT_EPILOGUE)) goto done;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      if (TAIL && nt == n_main) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN), r);
        tmem_ld_wait();
        if (row < M) epi.tail(row, r);
      } else if constexpr (EpiWholeRow<Epi>::value) {
        epi.apply_row(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN), row, row < M);
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32),
                             r);
          tmem_ld_wait();
          const int col0 = n0 + c * 32;
          if (row < M && col0 < N) epi.apply(row, col0, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace sb
