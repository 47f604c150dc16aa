// ternary_gemm.cuh — grouped tcgen05 GEMM whose B operand is ternary {-1,0,+1}
// weights stored 2 bits per weight (split-plane words, see ternary.cu).
//
// C[row, n] = epi( sum_k A[row, k] * T[e][n, k] ) for the rows of one expert e.
//
//   A  : 16-bit activations [R, K] (bf16 or fp16), rows grouped by expert,
//        TMA-loaded into 128-byte-swizzled K-major tiles (no multicast).
//   T  : packed words [E*N, KW] uint32; a 128- or 256-row x 16-byte box per
//        64-wide K step is TMA-loaded into a staging buffer, then four unpack
//        warps expand each word to sixteen 16-bit +-1/0 values and write them
//        in the same swizzled K-major layout the MMA reads.
//   MMA: tcgen05.mma kind::f16, M = 128, N = 256, fp32 accumulators in TMEM
//        (two buffers so the epilogue of one tile overlaps the next).
//
// Roles (384 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// allocator, warps 4..7 epilogue, warps 8..11 unpack.
//
// Tiles: the host does not know how many rows each expert received, so the
// kernel reads the m-tile table (expert, first row, row count) and its length
// from device memory; n-tiles are the fastest-varying index.
#pragma once

#include "sm100.cuh"

namespace sb {

struct MTile {
  int expert;
  int row0;
  int rows;
  int pad;
};

enum { TG_GATEUP = 0, TG_DOWN = 1, TG_LINEAR = 2 };

struct TernGemmParams {
  const MTile* mtiles;
  const int* num_mtiles;
  int n_ntiles;   // n-tiles per m-tile
  int N;          // valid output columns per expert
  int K;          // reduction length
  int b_rows;     // packed rows per expert in the B maps
  const float* s0;     // GATEUP: gate scale [E*N]; DOWN: down scale [E*N]; LINEAR: scale [N]
  const float* s1;     // GATEUP: up scale [E*N]
  const float* bias;   // LINEAR: bias [N] or null
  const float* row_w;  // DOWN: routing weight of each row
  void* out;
  int64_t ldo;
  // Split activations (pair engine): K runs over two halves that share the
  // weights — the packed weights' K-block index wraps after kb_wrap blocks —
  // so [x_hi | x_lo] against [T | T] sums T x_hi + T x_lo.  0 = no wrap.
  int kb_wrap;
  // GATEUP (pair engine): 0 = h stored as fp16; > 0 = h stored as two bf16
  // terms, hi = bf16(h) at column c and lo = bf16(h - hi) at c + h_lo_col.
  int h_lo_col;
};

constexpr int TG_THREADS = 384;
constexpr int TG_STAGES = 4;
constexpr int TG_A_BYTES = 128 * 64 * 2;   // 16 KB
constexpr int TG_BU_BYTES = 256 * 64 * 2;  // 32 KB unpacked B
constexpr int TG_BP_BYTES = 256 * 16;      // 4 KB packed B
constexpr int TG_STAGE_BYTES = TG_A_BYTES + TG_BU_BYTES + TG_BP_BYTES;  // 52 KB (1024-multiple)
constexpr int TG_BAR_BYTES = (3 * TG_STAGES + 4) * 8 + 16;
constexpr int TG_SMEM_BYTES = TG_STAGES * TG_STAGE_BYTES + TG_BAR_BYTES + 1024;
constexpr uint32_t TG_TMEM_COLS = 512;
static_assert(TG_STAGE_BYTES % 1024 == 0, "stage alignment");

// Two ternary weights (elements 2j, 2j+1 of a word) as two 16-bit floats.
//   FMT 1: bf16, FMT 0: fp16.  The biased codes c in {0,1,2} are placed in the
//   mantissa of b = 128 (bf16) / 1024 (fp16), whose last place is 1, and b + 1
//   is subtracted: (b + c) - (b + 1) = c - 1, exact in both formats.
// Bit position, in each 16-bit half of a layout word, of pair j (elements
// 2j and 2j+1 of the word's 16 K; the second element sits 16 bits above the
// first).  The order puts six pairs (bf16) or seven (fp16) where the format's
// mantissa can take the code in place (below).
__host__ __device__ constexpr int tern_pos(int j) { return j < 3 ? 2 * j : j < 6 ? 2 * j + 2 : j == 6 ? 6 : 14; }

// The codes at bit P of each half as 16-bit floats: OR-ing in the exponent
// that makes bit P the mantissa's unit turns code c into base + c exactly, and
// one packed subtraction of base + 1 leaves c - 1, the weight.  P must leave
// both code bits inside the mantissa: at most 4 for bf16 (7 mantissa bits),
// 8 for fp16 (10 bits).  base is 2^(7-P) (bf16) or 2^(10-P) (fp16).
template <int FMT, int P>
__device__ __forceinline__ uint32_t tern_decode_at(uint32_t w) {
  static_assert(P >= 0 && P <= (FMT ? 4 : 8), "both code bits must lie inside the mantissa");
  constexpr uint32_t base = FMT ? ((134u - P) << 7) : ((25u - P) << 10);
  constexpr uint32_t one = base + (1u << P);
  const uint32_t t = (w & (0x00030003u << P)) | (base | (base << 16));
  uint32_t r;
  if constexpr (FMT)
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(one | (one << 16)));
  else
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(one | (one << 16)));
  return r;
}

// Pair J of word w (J known at compile time): in place where the mantissa
// allows, else from w >> 8 (shared by the pairs that use it), else shifted down.
template <int FMT, int J>
__device__ __forceinline__ uint32_t tern_pair_c(uint32_t w) {
  constexpr int P = tern_pos(J);
  constexpr int LIM = FMT ? 4 : 8;
  if constexpr (P <= LIM)
    return tern_decode_at<FMT, P>(w);
  else if constexpr (P >= 8 && P - 8 <= LIM)
    return tern_decode_at<FMT, P - 8>(w >> 8);
  else
    return tern_decode_at<FMT, 0>(w >> P);
}

// The word's eight pairs: out[j] holds elements 2j, 2j+1 (K order).
template <int FMT>
__device__ __forceinline__ void tern_word(uint32_t w, uint32_t* out) {
  out[0] = tern_pair_c<FMT, 0>(w);
  out[1] = tern_pair_c<FMT, 1>(w);
  out[2] = tern_pair_c<FMT, 2>(w);
  out[3] = tern_pair_c<FMT, 3>(w);
  out[4] = tern_pair_c<FMT, 4>(w);
  out[5] = tern_pair_c<FMT, 5>(w);
  out[6] = tern_pair_c<FMT, 6>(w);
  out[7] = tern_pair_c<FMT, 7>(w);
}

// Pair j of word w for a j known only at run time (the few-token kernels).
template <int FMT>
__device__ __forceinline__ uint32_t tern_pair(uint32_t w, int j) {
  return tern_decode_at<FMT, 0>(w >> ((0xE6CA8420u >> (4 * j)) & 15u));
}

// Bounded wait by a whole warp (the lanes leave together); sleeps while waiting.
__device__ __forceinline__ bool mbar_wait_warp_t(uint64_t* bar, uint32_t parity, unsigned code) {
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

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <int MODE, int FMT>
__global__ void __launch_bounds__(TG_THREADS, 1)
    ternary_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB0,
                        const __grid_constant__ CUtensorMap tmB1, TernGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* full_tma = reinterpret_cast<uint64_t*>(smem + TG_STAGES * TG_STAGE_BYTES);
  uint64_t* full_b = full_tma + TG_STAGES;
  uint64_t* empty = full_b + TG_STAGES;
  uint64_t* tfull = empty + TG_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mt = *p.num_mtiles;
  const int num_tiles = n_mt * p.n_ntiles;
  const int kblocks = (p.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TG_STAGES; ++s) {
      mbar_init(&full_tma[s], 1);
      mbar_init(&full_b[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TG_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB0);
      if (MODE == TG_GATEUP) tma_prefetch_desc(&tmB1);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const MTile mt = p.mtiles[tile / p.n_ntiles];
        const int nt = tile % p.n_ntiles;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, ST_TIMEOUT_PRODUCER)) goto done;
          uint8_t* st = smem + stage * TG_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_tma[stage], TG_A_BYTES + TG_BP_BYTES);
          tma_load_2d(st, &tmA, &full_tma[stage], kb * 64, mt.row0);
          uint8_t* bp = st + TG_A_BYTES + TG_BU_BYTES;
          if (MODE == TG_GATEUP) {
            const int brow = mt.expert * p.b_rows + nt * 128;
            tma_load_2d(bp, &tmB0, &full_tma[stage], kb * 4, brow);
            tma_load_2d(bp + TG_BP_BYTES / 2, &tmB1, &full_tma[stage], kb * 4, brow);
          } else {
            const int brow = mt.expert * p.b_rows + nt * 256;
            tma_load_2d(bp, &tmB0, &full_tma[stage], kb * 4, brow);
          }
          if (++stage == TG_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(FMT, 128, 256);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, ST_TIMEOUT_MMA)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full_tma[stage], phase, ST_TIMEOUT_MMA)) goto done;
          if (!mbar_wait(&full_b[stage], phase, ST_TIMEOUT_MMA)) goto done;
          tc_fence_after();
          uint8_t* st = smem + stage * TG_STAGE_BYTES;
          const uint64_t adesc = sdesc_sw128(smem_u32(st));
          const uint64_t bdesc = sdesc_sw128(smem_u32(st + TG_A_BYTES));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == TG_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ unpack warps
    const int ut = threadIdx.x - 256;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_warp_t(&full_tma[stage], phase, ST_TIMEOUT_UNPACK)) goto done;
        uint8_t* st = smem + stage * TG_STAGE_BYTES;
        uint8_t* bu = st + TG_A_BYTES;
        const uint8_t* bp = st + TG_A_BYTES + TG_BU_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = ut + 128 * h;  // B row (output channel within the n-tile)
          const uint4 wv = *reinterpret_cast<const uint4*>(bp + r * 16);
          const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t w = words[q];
            uint4 lo, hi;
            uint32_t pr[8];
            tern_word<FMT>(w, pr);
            lo = make_uint4(pr[0], pr[1], pr[2], pr[3]);
            hi = make_uint4(pr[4], pr[5], pr[6], pr[7]);
            *reinterpret_cast<uint4*>(bu + sw128_offset(r, 2 * q)) = lo;
            *reinterpret_cast<uint4*>(bu + sw128_offset(r, 2 * q + 1)) = hi;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_b[stage]);
        if (++stage == TG_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
      const MTile mt = p.mtiles[tile / p.n_ntiles];
      const int nt = tile % p.n_ntiles;
      if (!mbar_wait_warp_t(&tfull[acc], acc_phase, ST_TIMEOUT_EPILOGUE)) goto done;
      tc_fence_after();
      const int lr = q * 32 + lane;
      const bool row_ok = lr < mt.rows;
      const int64_t row = (int64_t)mt.row0 + lr;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256);
      if (MODE == TG_GATEUP) {
        __half* out = static_cast<__half*>(p.out);
        const float* sg = p.s0 + (int64_t)mt.expert * p.N;
        const float* su = p.s1 + (int64_t)mt.expert * p.N;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tbase + c * 32, rg);
          tmem_ld_32x32b_x32(tbase + 128 + c * 32, ru);
          tmem_ld_wait();
          const int col0 = nt * 128 + c * 32;
          if (row_ok) {
            __half* dst = out + row * p.ldo + col0;
            if (col0 + 32 <= p.N && (p.ldo & 7) == 0) {
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float g0 = __uint_as_float(rg[2 * j]) * __ldg(sg + col0 + 2 * j);
                const float g1 = __uint_as_float(rg[2 * j + 1]) * __ldg(sg + col0 + 2 * j + 1);
                const float u0 = __uint_as_float(ru[2 * j]) * __ldg(su + col0 + 2 * j);
                const float u1 = __uint_as_float(ru[2 * j + 1]) * __ldg(su + col0 + 2 * j + 1);
                __half2 hv = __floats2half2_rn(silu_f(g0) * u0, silu_f(g1) * u1);
                pk[j] = *reinterpret_cast<uint32_t*>(&hv);
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j) d4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) {
                  const float g = __uint_as_float(rg[j]) * __ldg(sg + col0 + j);
                  const float u = __uint_as_float(ru[j]) * __ldg(su + col0 + j);
                  dst[j] = __float2half_rn(silu_f(g) * u);
                }
            }
          }
        }
      } else {
        float* out = static_cast<float*>(p.out);
        const float* sc = (MODE == TG_DOWN) ? p.s0 + (int64_t)mt.expert * p.N : p.s0;
        const float rw = (MODE == TG_DOWN && row_ok) ? __ldg(p.row_w + row) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          const int col0 = nt * 256 + c * 32;
          if (row_ok) {
            float* dst = out + row * p.ldo + col0;
            if (col0 + 32 <= p.N && (p.ldo & 3) == 0) {
              float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int cc = col0 + 4 * j + u;
                  float y = __uint_as_float(r[4 * j + u]) * __ldg(sc + cc);
                  if (MODE == TG_DOWN) y *= rw;
                  if (MODE == TG_LINEAR && p.bias) y += __ldg(p.bias + cc);
                  v[u] = y;
                }
                d4[j] = make_float4(v[0], v[1], v[2], v[3]);
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) {
                  float y = __uint_as_float(r[j]) * __ldg(sc + col0 + j);
                  if (MODE == TG_DOWN) y *= rw;
                  if (MODE == TG_LINEAR && p.bias) y += __ldg(p.bias + col0 + j);
                  dst[j] = y;
                }
            }
          }
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
    tmem_dealloc(tmem_base, TG_TMEM_COLS);
  }
}

}  // namespace sb
