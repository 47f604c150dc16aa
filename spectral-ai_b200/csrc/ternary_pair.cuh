// ternary_pair.cuh — grouped ternary GEMM on CTA pairs (tcgen05 cta_group::2).
//
//   D^T[c, t] = sum_k W[e][c, k] * X[t, k]     (c: output channel, t: token row)
//
// A pair of CTAs on two SMs computes one tile of 256 output channels x up to
// 192 tokens of one expert.  The ternary weights are the A operand and live in
// tensor memory: each CTA unpacks its 128 channels for one 128-K block (2-bit
// biased codes, TMA'd into a 4 KB buffer) into 16-bit +-1/0 and writes them
// into its TMEM with tcgen05.st (lane = channel).  Each CTA loads its half of
// the token tile (96 rows x 128 K as two 64-K boxes, 128-byte swizzle) into
// its own shared memory.  The rank-0 CTA issues 8 MMAs of M=256, N=tile
// tokens, K=16 per K-block for both SMs; each SM keeps its 128 channels x N
// tokens of D.
//
// Why 128-K blocks: once MMAs are in flight, any wait of the issuing thread
// (an mbarrier poll, even a plain shared-memory load) costs a few hundred
// cycles before the next MMA can issue, so each wait has to cover as much MMA
// work as possible (768 cycles at N = 192).
//
// Compared with one CTA per tile (256 channels x 128 tokens), every unpacked
// weight meets 192 tokens, so the unpack work per FLOP drops by a third, and
// one issued MMA covers three times the FLOPs.
//
// GATEUP: a CTA's 128 TMEM lanes hold 64 gate and 64 up channels; in warp q,
// lane i < 16 is gate channel c0+16q+i and lane i+16 the up channel of the
// same index, so each SwiGLU pair sits in one warp (one shuffle apart).
// DOWN: lane r is output channel c0+r.
//
// Tokens: expert segments are padded to 32 rows, and a tile covers `pad` rows
// (a multiple of 32, at most 192), so the epilogue writes whole 32-row boxes
// with TMA stores and never touches another expert's rows.
//
// TMEM per CTA (512 columns): two accumulators at [0, 192) and [192, 384)
// (lane = channel, column = token) that alternate between tiles, so the
// epilogue of one tile overlaps the MMAs of the next; then TP_A_STAGES A
// stages of 64 columns (128 channels x 128 K) at [384, 512).
//
// Pipelines (each CTA):  shared-memory ring of TP_STAGES slots (token half +
// packed words); the token halves of both CTAs complete on the rank-0 CTA's
// full_x barrier; the packed words on the local full_p.  The MMA commits
// arrive on the same barrier offset in both CTAs.  Unpack and epilogue warps of
// both CTAs arrive on the rank-0 CTA's full_a / tempty barriers; the rank-0
// unpack warps arrive only after full_x, so full_a alone gates an MMA K-block.
//
// Roles (384 threads per CTA): warp 0 TMA producer, warp 1 MMA issuer (rank 0
// only), warp 2 TMEM allocator, warps 4..7 epilogue (TMEM -> registers ->
// shared tile -> TMA store), warps 8..11 unpack.  Warp w may only touch TMEM
// lanes 32*(w%4)..+31.  The MMA issuer's scheduler is shared with one epilogue
// and one unpack warp only: the tensor pipe queues one or two MMAs, so every
// instruction the issuing thread waits for is idle tensor time.
#pragma once

#include "sm100_pair.cuh"
#include "ternary_gemm.cuh"

namespace sb {

constexpr int TP_EPI_WARPS = 4;
constexpr int TP_EPI_SETS = TP_EPI_WARPS / 4;        // epilogue warps per TMEM lane quarter
constexpr int TP_UNPACK_WARPS = 4;                   // 4, or 8: two per TMEM lane quarter, one 64-K half each
constexpr int TP_UNPACK_WARP0 = 4 + TP_EPI_WARPS;
constexpr int TP_THREADS = 32 * (TP_UNPACK_WARP0 + TP_UNPACK_WARPS);
constexpr int TP_STAGES = 4;
constexpr int TP_A_STAGES = 2;
constexpr int TP_KB = 128;                           // K per block
constexpr int TP_TILE_ROWS = 192;                    // tokens per tile (both CTAs)
constexpr int TP_HALF_ROWS = TP_TILE_ROWS / 2;       // token rows loaded by each CTA
constexpr int TP_QROWS = TP_HALF_ROWS / 2;           // rows per activation box (two boxes per CTA)
constexpr int TP_XATOM_BYTES = TP_HALF_ROWS * 128;   // 12 KB: 96 token rows x 64 K
constexpr int TP_X_BYTES = 2 * TP_XATOM_BYTES;       // 24 KB: 96 token rows x 128 K
constexpr int TP_P_BYTES = 128 * 32;                 // 4 KB: 128 channels x 128 K at 2 bits
constexpr int TP_STAGE_BYTES = TP_X_BYTES + TP_P_BYTES;  // 28 KB (1024-multiple)
constexpr int TP_EBUF_BYTES = 4096;                  // one 32-token x 32-channel fp32 tile
constexpr int TP_EPI_BYTES = TP_EPI_WARPS * 2 * TP_EBUF_BYTES;  // double-buffered per warp
constexpr int TP_BAR_BYTES = (3 * TP_STAGES + TP_A_STAGES + 4) * 8 + 16;
constexpr int TP_SMEM_BYTES = TP_STAGES * TP_STAGE_BYTES + TP_EPI_BYTES + TP_BAR_BYTES + 1024;
constexpr uint32_t TP_TMEM_COLS = 512;
constexpr uint32_t TP_D_COLS = TP_TILE_ROWS;         // one accumulator
constexpr uint32_t TP_A_BASE = 2 * TP_D_COLS;        // A ring after both accumulators
constexpr uint32_t TP_A_COLS = 64;
static_assert(TP_STAGE_BYTES % 1024 == 0, "stage alignment");
static_assert(TP_HALF_ROWS % 8 == 0, "whole 8-row swizzle atoms per CTA");
static_assert(TP_A_BASE + TP_A_COLS * TP_A_STAGES <= TP_TMEM_COLS, "TMEM budget");
static_assert(TP_SMEM_BYTES <= 227 * 1024, "shared memory budget");

// silu with the fast exponential and division (relative error near 1e-6)
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ void tmem_st_32x32b_x32_p(uint32_t taddr, const uint32_t (&r)[32]) {
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

// STREAMS = 2: a tile of P tokens, P a multiple of 64, is computed by two MMA
// streams of N = P/2, each issued by its own thread (warps 1 and 3 of the even CTA) into
// its half of the accumulator.  Each CTA holds stream 0's quarter of the
// tokens in shared-memory rows 0.. and stream 1's in rows TP_QROWS.., so each
// stream's B operand is a contiguous run of rows and the accumulator columns
// stay in token order.  While one issuer waits on a barrier (a few hundred
// cycles once its MMAs are queued), the other keeps the tensor pipe fed.
template <int MODE, int FMT, int STREAMS>
__global__ void __launch_bounds__(TP_THREADS, 1)
    ternary_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW0,
                        const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmOut,
                        TernGemmParams p) {
  static_assert(MODE == TG_GATEUP || MODE == TG_DOWN, "pair kernel: GATEUP or DOWN");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* epi = smem + TP_STAGES * TP_STAGE_BYTES;
  uint64_t* full_x = reinterpret_cast<uint64_t*>(epi + TP_EPI_BYTES);  // rank 0: both token halves landed
  uint64_t* full_p = full_x + TP_STAGES;                               // local packed words landed
  uint64_t* xp_empty = full_p + TP_STAGES;                             // slot's MMAs completed
  uint64_t* full_a = xp_empty + TP_STAGES;                             // rank 0: A stage + token tile ready
  uint64_t* tfull = full_a + TP_A_STAGES;                              // [2] accumulator's MMAs completed
  uint64_t* tempty = tfull + 2;                                        // [2] rank 0: epilogue warps done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int n_mt = *p.num_mtiles;
  const int num_tiles = n_mt * p.n_ntiles;
  const int kblocks = (p.K + TP_KB - 1) / TP_KB;
  constexpr int CPAIR = (MODE == TG_GATEUP) ? 128 : 256;  // output channels of a pair tile
  constexpr int CCTA = CPAIR / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TP_STAGES; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_p[s], 1);
      mbar_init(&xp_empty[s], STREAMS);  // one commit per MMA stream
    }
    for (int s = 0; s < TP_A_STAGES; ++s) mbar_init(&full_a[s], 2 * TP_UNPACK_WARPS);  // unpack warps x 2 CTAs
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], STREAMS);
      mbar_init(&tempty[b], 2 * TP_EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, TP_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
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
      for (int tile = pair; tile < num_tiles; tile += npairs) {
        const MTile mt = p.mtiles[tile / p.n_ntiles];
        const int c0 = (tile % p.n_ntiles) * CPAIR + (int)rank * CCTA;
        const int wrow = mt.expert * p.b_rows + c0;
        // this CTA's tokens: stream 0's quarter (rows 0..) and stream 1's
        // (rows TP_QROWS..); one stream per CTA half when the tile is small
        const bool two = STREAMS == 2 && (mt.pad & 63) == 0;  // stream N = pad/2, a multiple of 32
        const int q = two ? mt.pad >> 2 : mt.pad >> 1;
        const int xrow0 = mt.row0 + (int)rank * q;
        const int xrow1 = mt.row0 + (mt.pad >> 1) + (int)rank * q;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&xp_empty[stage], phase ^ 1u, ST_TIMEOUT_PRODUCER)) goto done;
          uint8_t* st = smem + stage * TP_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_p[stage], TP_P_BYTES);
          const int wkb = (p.kb_wrap > 0 && kb >= p.kb_wrap) ? kb - p.kb_wrap : kb;  // weight K-block
          if (MODE == TG_GATEUP) {
            tma_load_2d(st + TP_X_BYTES, &tmW0, &full_p[stage], wkb * 8, wrow);
            tma_load_2d(st + TP_X_BYTES + TP_P_BYTES / 2, &tmW1, &full_p[stage], wkb * 8, wrow);
          } else {
            tma_load_2d(st + TP_X_BYTES, &tmW0, &full_p[stage], wkb * 8, wrow);
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_x[stage], 2 * TP_X_BYTES);
          const uint32_t fx = mapa_shared(smem_u32(&full_x[stage]), 0);
          if (STREAMS == 2) {
            // 48-row boxes: rows 0..47 and 48..95 of each 64-K atom
            const int h = TP_QROWS * 128;
            tma_load_2d_pair(st, &tmX, fx, kb * TP_KB, xrow0);
            tma_load_2d_pair(st + h, &tmX, fx, kb * TP_KB, two ? xrow1 : xrow0 + TP_QROWS);
            tma_load_2d_pair(st + TP_XATOM_BYTES, &tmX, fx, kb * TP_KB + 64, xrow0);
            tma_load_2d_pair(st + TP_XATOM_BYTES + h, &tmX, fx, kb * TP_KB + 64, two ? xrow1 : xrow0 + TP_QROWS);
          } else {
            tma_load_2d_pair(st, &tmX, fx, kb * TP_KB, xrow0);
            tma_load_2d_pair(st + TP_XATOM_BYTES, &tmX, fx, kb * TP_KB + 64, xrow0);
          }
          if (++stage == TP_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1 || (STREAMS == 2 && warp == 3)) {
    // ------------------------------------------------------------ MMA issuers (rank 0)
    const int sid = warp == 1 ? 0 : 1;  // this thread's MMA stream
    if (lane == 0 && rank == 0) {
      int stage = 0, astage = 0;
      uint32_t phase = 0, aphase = 0;
      int local = 0;
      for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
        const MTile mt = p.mtiles[tile / p.n_ntiles];
        const bool two = STREAMS == 2 && (mt.pad & 63) == 0;  // stream N = pad/2, a multiple of 32
        const int n = two ? mt.pad >> 1 : mt.pad;  // this stream's tokens
        const bool active = two || sid == 0;       // stream 1 idles on small tiles (commits only)
        const uint32_t idesc = idesc_f16(FMT, 256, (uint32_t)n);
        const int buf = local & 1;
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * TP_D_COLS) + (uint32_t)(sid * n);
        const uint32_t b_off = (uint32_t)(sid * TP_QROWS * 128) >> 4;  // stream's rows in the slot
        if (!mbar_wait_cluster(&tempty[buf], ((uint32_t)(local >> 1) & 1u) ^ 1u, ST_TIMEOUT_MMA)) goto done;
        tc_fence_after();
        bool ready = false;  // this K-block's full_a was seen complete by the previous peek
        for (int kb = 0; kb < kblocks; ++kb) {
          // one wait per K-block: full_a completes only after the rank-0 unpack
          // warps have also seen this slot's token halves land (full_x)
          if (!ready && !mbar_wait_cluster(&full_a[astage], aphase, ST_TIMEOUT_MMA)) goto done;
          tc_fence_after();
          // peek at the next K-block's barrier now: the poll's latency overlaps
          // the MMA issue below, and the result is only used in the next pass
          const int nastage = astage + 1 == TP_A_STAGES ? 0 : astage + 1;
          const uint32_t naphase = nastage == 0 ? aphase ^ 1u : aphase;
          const bool peek = kb + 1 < kblocks && mbar_test_wait(smem_u32(&full_a[nastage]), naphase);
          const uint64_t bdesc = sdesc_sw128(smem_u32(smem + stage * TP_STAGE_BYTES));
          const uint32_t a_tmem = tmem_base + TP_A_BASE + (uint32_t)(astage * TP_A_COLS);
          if (active) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              // K 16k..16k+15: A columns 8k..; B in the first or second 64-K atom
              const uint64_t bk =
                  bdesc + b_off + (k < 4 ? 2u * k : (uint32_t)(TP_XATOM_BYTES >> 4) + 2u * (k - 4));
              umma_ts_pair(d_tmem, a_tmem + 8u * k, bk, idesc, (kb | k) != 0);
            }
          }
          // frees the slot's token tile and packed words, and the A stage this
          // K-block read (the unpack warps wait on this barrier for both)
          umma_commit_pair(&xp_empty[stage]);
          ready = peek;
          if (++stage == TP_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          astage = nastage;
          aphase = naphase;
        }
        umma_commit_pair(&tfull[buf]);
      }
    }
  } else if (warp >= TP_UNPACK_WARP0) {
    // ------------------------------------------------------------ unpack warps
    const int q = warp & 3;
    [[maybe_unused]] const int uh = (warp - TP_UNPACK_WARP0) >> 2;  // 8 unpack warps: this warp's 64-K half
    // the packed row this lane expands (TMEM lane 32q + lane)
    int prow;
    if (MODE == TG_GATEUP)
      prow = lane < 16 ? 16 * q + lane : 64 + 16 * q + (lane - 16);
    else
      prow = 32 * q + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + TP_A_BASE;
    int it = 0;  // K-block counter over this pair's whole tile sequence
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int stage = it % TP_STAGES;
        const uint32_t phase = (uint32_t)(it / TP_STAGES) & 1u;
        const int astage = it % TP_A_STAGES;
        if (!mbar_wait_warp_t(&full_p[stage], phase, ST_TIMEOUT_UNPACK)) goto done;
        // expand the row's eight words (128 K) into registers first: only the
        // stores into TMEM have to wait for the A stage to drain
        const uint8_t* pw = smem + stage * TP_STAGE_BYTES + TP_X_BYTES + prow * 32;
        uint32_t a0[32];
        [[maybe_unused]] uint32_t a1[TP_UNPACK_WARPS == 4 ? 32 : 1];
        if constexpr (TP_UNPACK_WARPS == 4) {
          const uint4 w0 = *reinterpret_cast<const uint4*>(pw);
          const uint4 w1 = *reinterpret_cast<const uint4*>(pw + 16);
          const uint32_t words0[4] = {w0.x, w0.y, w0.z, w0.w};
          const uint32_t words1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            tern_word<FMT>(words0[w], a0 + 8 * w);
            tern_word<FMT>(words1[w], a1 + 8 * w);
          }
        } else {
          const uint4 w0 = *reinterpret_cast<const uint4*>(pw + 16 * uh);
          const uint32_t words0[4] = {w0.x, w0.y, w0.z, w0.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) tern_word<FMT>(words0[w], a0 + 8 * w);
        }
        // The A stage is free once the MMAs of K-block it - TP_A_STAGES have
        // completed, which the commit on that block's slot barrier signals.
        // That barrier is then in the phase of that block or one past it (the
        // block before it completed before this warp's previous pass, and the
        // next use of the slot needs this very pass), so the parity is exact.
        if (it >= TP_A_STAGES) {
          const int pj = it - TP_A_STAGES;
          if (!mbar_wait_warp_t(&xp_empty[pj % TP_STAGES], (uint32_t)(pj / TP_STAGES) & 1u, ST_TIMEOUT_UNPACK))
            goto done;
        }
        tc_fence_after();
        const uint32_t col = lane_base + (uint32_t)(astage * TP_A_COLS);
        if constexpr (TP_UNPACK_WARPS == 4) {
          tmem_st_32x32b_x32_p(col, a0);
          tmem_st_32x32b_x32_p(col + 32u, a1);
        } else {
          tmem_st_32x32b_x32_p(col + 32u * (uint32_t)uh, a0);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        // rank 0 also waits for both token halves of this slot, so that the MMA
        // issuer needs a single barrier per K-block
        if (rank == 0 && !mbar_wait_warp_t(&full_x[stage], phase, ST_TIMEOUT_UNPACK)) goto done;
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&full_a[astage]), 0));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 4) >> 2;  // this warp takes chunks half, half + TP_EPI_SETS, ...
    const uint32_t tlanes = tmem_base + ((uint32_t)(q * 32) << 16);
    uint8_t* ebuf = epi + (warp - 4) * 2 * TP_EBUF_BYTES;
    int local = 0, nbuf = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
      const int buf = local & 1;
      const uint32_t ph = (uint32_t)(local >> 1) & 1u;
      const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[buf]), 0);
      const MTile mt = p.mtiles[tile / p.n_ntiles];
      const int c0 = (tile % p.n_ntiles) * CPAIR + (int)rank * CCTA;
      const int nch = mt.pad >> 5;
      // this lane's channel and scales
      int ch;
      float s_a, s_b = 0.f;
      if (MODE == TG_GATEUP) {
        ch = c0 + 16 * q + (lane & 15);
        const bool ok = ch < p.N;
        s_a = ok ? __ldg(p.s0 + (int64_t)mt.expert * p.N + ch) : 0.f;
        s_b = ok ? __ldg(p.s1 + (int64_t)mt.expert * p.N + ch) : 0.f;
      } else {
        ch = c0 + 32 * q + lane;
        s_a = ch < p.N ? __ldg(p.s0 + (int64_t)mt.expert * p.N + ch) : 0.f;
      }
      const int xcol = (MODE == TG_GATEUP) ? c0 + 16 * q : c0 + 32 * q;  // box column
      const bool store = xcol < p.N;
      if (!mbar_wait_warp_t(&tfull[buf], ph, ST_TIMEOUT_EPILOGUE)) goto done;
      tc_fence_after();
      const uint32_t tbase = tlanes + (uint32_t)(buf * TP_D_COLS);
      // this warp's last chunk (or none): the accumulator is released after its load
      const int last = (nch - 1 - half) >= 0 ? half + ((nch - 1 - half) / TP_EPI_SETS) * TP_EPI_SETS : -1;
      if (last < 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader);
      }
#pragma unroll 1
      for (int c = half; c < nch; c += TP_EPI_SETS) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        tmem_ld_wait();
        if (c == last) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader);
        }
        uint8_t* sb = ebuf + nbuf * TP_EBUF_BYTES;
        // the store that last read this buffer (two chunks ago) has finished reading
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        const int t0 = mt.row0 + c * 32;
        if (MODE == TG_GATEUP) {
          const bool gate = lane < 16;
          const int ci = lane & 15;
          if (p.h_lo_col > 0) {
            // two bf16 terms: hi [32 tokens][16 channels] at sb, lo at sb + 1 KB
            __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(sb);
            __nv_bfloat16* lo = hi + 32 * 16;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float mine = __uint_as_float(gate ? v[j] : v[16 + j]);
              const float other = __shfl_xor_sync(0xffffffffu, __uint_as_float(gate ? v[16 + j] : v[j]), 16);
              const float g = (gate ? mine : other) * s_a;
              const float u = (gate ? other : mine) * s_b;
              const float h = silu_fast(g) * u;
              const __nv_bfloat16 hh = __float2bfloat16_rn(h);
              hi[(gate ? j : 16 + j) * 16 + ci] = hh;
              lo[(gate ? j : 16 + j) * 16 + ci] = __float2bfloat16_rn(h - __bfloat162float(hh));
            }
          } else {
            // fp16 h: a value past 65504 becomes inf here and a non-finite
            // output, which the combine reports through the status word
            __half* hb = reinterpret_cast<__half*>(sb);  // [32 tokens][16 channels]
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float mine = __uint_as_float(gate ? v[j] : v[16 + j]);
              const float other = __shfl_xor_sync(0xffffffffu, __uint_as_float(gate ? v[16 + j] : v[j]), 16);
              // gate lane: token j (own gate, partner's up); up lane: token 16+j
              const float g = (gate ? mine : other) * s_a;
              const float u = (gate ? other : mine) * s_b;
              hb[(gate ? j : 16 + j) * 16 + ci] = __float2half_rn(silu_fast(g) * u);
            }
          }
        } else {
          float* fb = reinterpret_cast<float*>(sb);  // [32 tokens][32 channels]
          const float rwl = __ldg(p.row_w + t0 + lane);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float rw = __shfl_sync(0xffffffffu, rwl, j);
            fb[j * 32 + lane] = __uint_as_float(v[j]) * s_a * rw;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && store) {
          tma_store_2d(&tmOut, sb, xcol, t0);
          if (MODE == TG_GATEUP && p.h_lo_col > 0) tma_store_2d(&tmOut, sb + 32 * 16 * 2, xcol + p.h_lo_col, t0);
          bulk_commit_group();
        }
        nbuf ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }
done:
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrive or MMA still targets this CTA
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TP_TMEM_COLS);
  }
}

}  // namespace sb
