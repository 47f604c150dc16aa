// ternary_ts.cuh — grouped ternary GEMM with the weights as the TMEM operand.
//
//   D^T[c, t] = sum_k W[e][c, k] * X[t, k]     (c: output channel, t: token row)
//
// The ternary weights are the A operand and live in tensor memory: unpack
// warps read the 2-bit split-plane words of the tile's channels for one 64-K
// block (TMA'd into a 4 KB staging buffer), expand them in registers to 16-bit
// +-1/0 and write them straight into TMEM with tcgen05.st (lane = channel, two
// K values per 32-bit column).  Shared memory carries only the 128-token x
// 64-K activation tile (TMA, 128-byte swizzle, no multicast) that is the B
// operand, so the unpack does not compete with the MMA for shared memory.
//
// A tile covers 256 output channels with two accumulators that share every
// activation tile (8 MMAs of M=128, N=128, K=16 per 64-K block): GATEUP puts
// gate channels c0..c0+127 in accumulator 0 and the up channels c0..c0+127 in
// accumulator 1, so lane r holds the gate and up value of channel c0+r and
// the SwiGLU needs no exchange; DOWN/LINEAR cover channels c0..c0+255.
//
//   tcgen05.mma.cta_group::1.kind::f16 [D], [A_tmem], B_smem_desc, idesc
//
// Pipelines.  One K-block's MMAs take 512 cycles, while a shared-memory slot
// is held from its TMA issue through the load latency, the unpack and the
// MMAs queued ahead of it: a few microseconds.  So the shared-memory ring is
// deep (TS_STAGES slots of activation tile + packed words, nearly all of
// shared memory) and the packed words have their own barrier, so the unpack
// of a K-block starts as soon as its 4 KB have landed.  The unpacked weights
// go through a separate ring of TS_A_STAGES TMEM stages, which only has to
// cover the unpack latency.
//
// TMEM (512 columns): accumulators at [0,128) and [128,256), then the A ring
// of 64-column stages (two 128x64 weight blocks each).  The accumulators are
// single-buffered; the epilogue reads them 32 tokens at a time, releases TMEM
// after its last load and writes straight from registers (lane = channel, so
// a warp's store covers 32 consecutive channels of one token row).
//
// Roles (512 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// allocator, warps 4..7 epilogue, warps 8..15 unpack in two groups of four
// that take alternate K-blocks (warp w owns TMEM lanes 32*(w%4)..+31).
#pragma once

#include "sm100.cuh"
#include "ternary_gemm.cuh"

namespace sb {

constexpr int TS_UNPACK_GROUPS = 2;
constexpr int TS_THREADS = 256 + 128 * TS_UNPACK_GROUPS;
constexpr int TS_STAGES = 10;                      // shared-memory ring (activations + packed words)
constexpr int TS_A_STAGES = 4;                     // TMEM ring of unpacked weights
constexpr int TS_N = 128;                          // tokens per tile
constexpr int TS_CH = 256;                         // channels per tile (two accumulators)
constexpr int TS_X_BYTES = TS_N * 64 * 2;          // 16 KB activation tile
constexpr int TS_P_BYTES = TS_CH * 16;             // 4 KB packed weights
constexpr int TS_STAGE_BYTES = TS_X_BYTES + TS_P_BYTES;  // 20 KB (1024-multiple)
constexpr int TS_BAR_BYTES = (3 * TS_STAGES + 2 * TS_A_STAGES + 2) * 8 + 16;
constexpr int TS_SMEM_BYTES = TS_STAGES * TS_STAGE_BYTES + TS_BAR_BYTES + 1024;
constexpr uint32_t TS_TMEM_COLS = 512;
constexpr uint32_t TS_D_COLS = 2 * TS_N;           // accumulators at columns [0, 256)
constexpr uint32_t TS_A_COLS = 64;                 // per A stage: two 128 x 64 weight blocks
static_assert(TS_STAGE_BYTES % 1024 == 0, "stage alignment");
static_assert(TS_D_COLS + TS_A_COLS * TS_A_STAGES <= TS_TMEM_COLS, "TMEM budget");
static_assert(TS_A_STAGES % TS_UNPACK_GROUPS == 0, "groups must own whole A stages");
static_assert(TS_SMEM_BYTES <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16.
__device__ __forceinline__ void umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Expands the four packed words of one row (64 K) into 32 TMEM columns.
template <int FMT>
__device__ __forceinline__ void unpack_row_to_tmem(const uint4 wv, uint32_t taddr) {
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t a[32];
#pragma unroll
  for (int w = 0; w < 4; ++w) tern_word<FMT>(words[w], a + 8 * w);
  tmem_st_32x32b_x32(taddr, a);
}

template <int MODE, int FMT>
__global__ void __launch_bounds__(TS_THREADS, 1)
    ternary_ts_kernel(const __grid_constant__ CUtensorMap tmX,
                      const __grid_constant__ CUtensorMap tmW0,
                      const __grid_constant__ CUtensorMap tmW1, TernGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + TS_STAGES * TS_STAGE_BYTES);
  uint64_t* full_p = full_x + TS_STAGES;     // the slot's packed words landed
  uint64_t* xp_empty = full_p + TS_STAGES;   // the slot's MMAs completed
  uint64_t* full_a = xp_empty + TS_STAGES;   // A stage written (4 unpack warps)
  uint64_t* a_empty = full_a + TS_A_STAGES;  // A stage's MMAs completed
  uint64_t* tfull = a_empty + TS_A_STAGES;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mt = *p.num_mtiles;
  const int num_tiles = n_mt * p.n_ntiles;
  const int kblocks = (p.K + 63) / 64;
  // first channel of accumulator 0 (GATEUP: gate and up channels c0..c0+127)
  constexpr int CSTEP = (MODE == TG_GATEUP) ? 128 : 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TS_STAGES; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_p[s], 1);
      mbar_init(&xp_empty[s], 1);
    }
    for (int s = 0; s < TS_A_STAGES; ++s) {
      mbar_init(&full_a[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 4);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TS_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmW0);
      if (MODE == TG_GATEUP) tma_prefetch_desc(&tmW1);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const MTile mt = p.mtiles[tile / p.n_ntiles];
        const int c0 = (tile % p.n_ntiles) * CSTEP;
        const int wrow = mt.expert * p.b_rows + c0;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&xp_empty[stage], phase ^ 1u, ST_TIMEOUT_PRODUCER)) goto done;
          uint8_t* st = smem + stage * TS_STAGE_BYTES;
          // packed words first: the unpack waits only for them
          mbar_arrive_expect_tx(&full_p[stage], TS_P_BYTES);
          if (MODE == TG_GATEUP) {
            tma_load_2d(st + TS_X_BYTES, &tmW0, &full_p[stage], kb * 4, wrow);
            tma_load_2d(st + TS_X_BYTES + TS_P_BYTES / 2, &tmW1, &full_p[stage], kb * 4, wrow);
          } else {
            tma_load_2d(st + TS_X_BYTES, &tmW0, &full_p[stage], kb * 4, wrow);
          }
          mbar_arrive_expect_tx(&full_x[stage], TS_X_BYTES);
          tma_load_2d(st, &tmX, &full_x[stage], kb * 64, mt.row0);
          if (++stage == TS_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(FMT, 128, TS_N);
      int stage = 0, astage = 0;
      uint32_t phase = 0, aphase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        if (!mbar_wait(tempty, ((uint32_t)local & 1u) ^ 1u, ST_TIMEOUT_MMA)) goto done;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full_a[astage], aphase, ST_TIMEOUT_MMA)) goto done;
          if (!mbar_wait(&full_x[stage], phase, ST_TIMEOUT_MMA)) goto done;
          tc_fence_after();
          const uint64_t bdesc = sdesc_sw128(smem_u32(smem + stage * TS_STAGE_BYTES));
          const uint32_t a_tmem = tmem_base + TS_D_COLS + (uint32_t)(astage * TS_A_COLS);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_ts_f16(tmem_base, a_tmem + 8u * k, bdesc + 2u * k, idesc, (kb | k) != 0);
            umma_ts_f16(tmem_base + TS_N, a_tmem + 32u + 8u * k, bdesc + 2u * k, idesc, (kb | k) != 0);
          }
          umma_commit(&xp_empty[stage]);
          umma_commit(&a_empty[astage]);
          if (++stage == TS_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (++astage == TS_A_STAGES) {
            astage = 0;
            aphase ^= 1u;
          }
        }
        umma_commit(tfull);
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ unpack warps
    const int q = warp & 3;
    const int grp = (warp - 8) >> 2;
    const int r = q * 32 + lane;  // TMEM lane; packed rows r and 128 + r
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + TS_D_COLS;
    int it = 0;  // K-block counter over this CTA's whole tile sequence
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        if (it % TS_UNPACK_GROUPS != grp) continue;
        const int stage = it % TS_STAGES;
        const uint32_t phase = (uint32_t)(it / TS_STAGES) & 1u;
        const int astage = it % TS_A_STAGES;
        const uint32_t aphase = (uint32_t)(it / TS_A_STAGES) & 1u;
        if (!mbar_wait_warp_t(&full_p[stage], phase, ST_TIMEOUT_UNPACK)) goto done;
        const uint8_t* bp = smem + stage * TS_STAGE_BYTES + TS_X_BYTES;
        const uint4 w0 = *reinterpret_cast<const uint4*>(bp + r * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(bp + (128 + r) * 16);
        if (!mbar_wait_warp_t(&a_empty[astage], aphase ^ 1u, ST_TIMEOUT_UNPACK)) goto done;
        tc_fence_after();
        const uint32_t col = lane_base + (uint32_t)(astage * TS_A_COLS);
        unpack_row_to_tmem<FMT>(w0, col);
        unpack_row_to_tmem<FMT>(w1, col + 32u);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[astage]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;  // accumulator row = channel within the accumulator
    const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16);
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const uint32_t ph = (uint32_t)local & 1u;
      const MTile mt = p.mtiles[tile / p.n_ntiles];
      const int c0 = (tile % p.n_ntiles) * CSTEP;
      const int nch = (mt.rows + 31) / 32;  // 32-token chunks holding valid tokens
      float sc[2], bi[2];
      int col[2];
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const float* sv;
        if (MODE == TG_GATEUP) {
          col[a] = c0 + r;
          sv = (a == 0 ? p.s0 : p.s1) + (int64_t)mt.expert * p.N;
        } else {
          col[a] = c0 + 128 * a + r;
          sv = (MODE == TG_DOWN) ? p.s0 + (int64_t)mt.expert * p.N : p.s0;
        }
        const bool ok = col[a] < p.N;
        sc[a] = ok ? __ldg(sv + col[a]) : 0.f;
        bi[a] = (MODE == TG_LINEAR && p.bias && ok) ? __ldg(p.bias + col[a]) : 0.f;
      }
      if (!mbar_wait_warp_t(tfull, ph, ST_TIMEOUT_EPILOGUE)) goto done;
      tc_fence_after();
      if (nch == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty);
        continue;
      }
      if (MODE == TG_GATEUP) {
        const bool ok = col[0] < p.N;
        __half* out = static_cast<__half*>(p.out) + col[0];
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), g);
          tmem_ld_32x32b_x32(tbase + (uint32_t)(TS_N + c * 32), u);
          tmem_ld_wait();
          if (c == nch - 1) {  // accumulators free for the next tile
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);
          }
          const int t0 = c * 32;
          const int nt = min(32, mt.rows - t0);
          if (ok) {
            __half* o = out + (int64_t)(mt.row0 + t0) * p.ldo;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nt)
                o[(int64_t)j * p.ldo] = __float2half_rn(silu_f(__uint_as_float(g[j]) * sc[0]) *
                                                        (__uint_as_float(u[j]) * sc[1]));
          }
        }
      } else {
        float* out = static_cast<float*>(p.out);
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          const bool ok = col[a] < p.N;
#pragma unroll 1
          for (int c = 0; c < nch; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tbase + (uint32_t)(a * TS_N + c * 32), v);
            tmem_ld_wait();
            if (a == 1 && c == nch - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(tempty);
            }
            const int t0 = c * 32;
            const int nt = min(32, mt.rows - t0);
            // token t0+lane's routing weight, handed round the warp
            const float rwl = (MODE == TG_DOWN && lane < nt) ? __ldg(p.row_w + mt.row0 + t0 + lane) : 1.0f;
            float* o = out + (int64_t)(mt.row0 + t0) * p.ldo + col[a];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float rw = __shfl_sync(0xffffffffu, rwl, j);
              if (ok && j < nt) o[(int64_t)j * p.ldo] = fmaf(__uint_as_float(v[j]), sc[a], bi[a]) * rw;
            }
          }
        }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TS_TMEM_COLS);
  }
}

}  // namespace sb
