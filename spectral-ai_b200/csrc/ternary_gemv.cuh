// ternary_gemv.cuh — ternary_gated_mlp for a handful of tokens (one expert).
//
// With at most GEMV_ROWS tokens the expert is a weight stream, not a GEMM:
// its 2-bit weights (1.57 MB at the OLMoE shape) are read once and each decoded
// weight meets one to a few tokens.  The tile kernels spend a fixed pipeline of
// TMA loads, unpacking into tensor memory and MMA rounds on each 256-channel
// tile, on 16 SMs for one expert, whatever the token count; here the rows are
// cut into 512-K chunks and every (row, chunk) is one warp's task, so one
// expert's stream spreads over the whole GPU.  The arithmetic is fp32
// throughout (tokens as given, fp32 or bf16; the hidden state kept in fp32),
// like the reference kernel's (cuda/v5/ternary_torch_ext.cu:123-191, one
// token per CTA).
//
//   gate/up:  h[r, c] = silu(s_g[c] * (T_g[c,:] . x_r)) * (s_u[c] * (T_u[c,:] . x_r))   -> fp32 scratch
//   down:     y[r, o] = s_d[o] * (T_d[o,:] . h_r)                                         -> fp32 output
//
// A warp's task: lane l loads word l of the chunk (32 words = 512 K, one
// 128-byte line per warp) and its tokens' values at K = 64s + 2l, +1 for the
// chunk's eight steps s, all before any arithmetic; at step s it takes the
// word it needs from lane 4s + l/8 by a shuffle, decodes its pair of weights
// and accumulates in fp32; a butterfly sums the lanes.  The chunk sums of a row
// meet in shared memory and are added in chunk order, so the result does not
// depend on the launch shape.
#pragma once

#include "ternary_gemm.cuh"

namespace sb {

constexpr int GEMV_ROWS = 4;      // tokens at most
constexpr int GEMV_WARPS = 8;     // warps per block
constexpr int GEMV_CHUNK = 512;   // K per task
constexpr int GEMV_MAX_CHUNKS = 16;

// The pair of weights (elements 2j, 2j+1 of word w) as two floats, from the
// bf16 pair tern_pair<1> makes (exact +-1/0; j known at run time).
__device__ __forceinline__ float2 tern_pair_f2(uint32_t w, int j) {
  const uint32_t p = tern_pair<1>(w, j);
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}

template <typename TX>
__device__ __forceinline__ float2 load_pair(const TX* p) {
  if constexpr (std::is_same<TX, float>::value) {
    return __ldg(reinterpret_cast<const float2*>(p));
  } else {
    const uint32_t v = __ldg(reinterpret_cast<const unsigned int*>(p));
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  }
}

// Sum over one chunk [k0, k0 + 512) of row `prow` (K/16 packed words) against
// token rows r < m <= N of x (row stride ldx; rows past m count as zero); K is
// a multiple of 64.
template <int N, typename TX>
__device__ __forceinline__ void gemv_chunk(const uint32_t* __restrict__ prow, const TX* __restrict__ x,
                                           int64_t ldx, int K, int k0, int m, float (&acc)[N]) {
  const int lane = threadIdx.x & 31;
  const int nw = min(GEMV_CHUNK, K - k0) / 16;  // words in this chunk, a multiple of 4
  const uint32_t word = lane < nw ? __ldg(prow + k0 / 16 + lane) : 0u;
  float2 xv[8][N];
#pragma unroll
  for (int s = 0; s < 8; ++s)
#pragma unroll
    for (int r = 0; r < N; ++r)
      xv[s][r] = (4 * s < nw && r < m) ? load_pair(x + (int64_t)r * ldx + k0 + 64 * s + 2 * lane)
                                       : make_float2(0.f, 0.f);
  float part[N];
#pragma unroll
  for (int r = 0; r < N; ++r) part[r] = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint32_t wd = __shfl_sync(0xffffffffu, word, 4 * s + (lane >> 3));
    const float2 t = tern_pair_f2(wd, lane & 7);
#pragma unroll
    for (int r = 0; r < N; ++r) part[r] = fmaf(t.x, xv[s][r].x, fmaf(t.y, xv[s][r].y, part[r]));
  }
#pragma unroll
  for (int r = 0; r < N; ++r) {
    float v = part[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    acc[r] = v;
  }
}

// gate/up: a block takes `cpb` channels (2 rows each, gate then up); its
// tasks are (row, chunk) pairs, warp w taking tasks w, w + 8, ...
template <int N, typename TX>
__global__ void __launch_bounds__(GEMV_WARPS * 32) ternary_gemv_gateup_kernel(
    const TX* __restrict__ x, const uint32_t* __restrict__ gate, const uint32_t* __restrict__ up,
    const float* __restrict__ gs, const float* __restrict__ us, int H, int I, int cpb, int m,
    float* __restrict__ h) {
  __shared__ float part[GEMV_WARPS * 4][GEMV_MAX_CHUNKS][N];  // [row of the block][chunk][token]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (H + GEMV_CHUNK - 1) / GEMV_CHUNK;
  const int c0 = blockIdx.x * cpb;
  const int tasks = 2 * cpb * chunks;
  for (int t = warp; t < tasks; t += GEMV_WARPS) {
    const int rb = t / chunks, ch = t % chunks;  // row of the block (2c gate, 2c+1 up), chunk
    const int c = c0 + (rb >> 1);
    float acc[N];
    if (c < I) {
      const uint32_t* prow = ((rb & 1) ? up : gate) + (int64_t)c * (H / 16);
      gemv_chunk<N>(prow, x, H, H, ch * GEMV_CHUNK, m, acc);
    } else {
#pragma unroll
      for (int r = 0; r < N; ++r) acc[r] = 0.f;
    }
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < N; ++r) part[rb][ch][r] = acc[r];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < cpb * N; i += blockDim.x) {
    const int cl = i / N, r = i % N, c = c0 + cl;
    if (c >= I || r >= m) continue;
    float g = 0.f, u = 0.f;
    for (int ch = 0; ch < chunks; ++ch) {
      g += part[2 * cl][ch][r];
      u += part[2 * cl + 1][ch][r];
    }
    h[(int64_t)r * I + c] = silu_fast(g * __ldg(gs + c)) * (u * __ldg(us + c));
  }
}

// down: a block takes `opb` output channels; tasks (row, chunk) as above.
template <int N>
__global__ void __launch_bounds__(GEMV_WARPS * 32) ternary_gemv_down_kernel(
    const float* __restrict__ h, const uint32_t* __restrict__ down, const float* __restrict__ ds, int H, int I,
    int opb, int m, float* __restrict__ y) {
  __shared__ float part[GEMV_WARPS * 4][GEMV_MAX_CHUNKS][N];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (I + GEMV_CHUNK - 1) / GEMV_CHUNK;
  const int o0 = blockIdx.x * opb;
  const int tasks = opb * chunks;
  for (int t = warp; t < tasks; t += GEMV_WARPS) {
    const int rb = t / chunks, ch = t % chunks;
    const int o = o0 + rb;
    float acc[N];
    if (o < H) {
      gemv_chunk<N>(down + (int64_t)o * (I / 16), h, I, I, ch * GEMV_CHUNK, m, acc);
    } else {
#pragma unroll
      for (int r = 0; r < N; ++r) acc[r] = 0.f;
    }
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < N; ++r) part[rb][ch][r] = acc[r];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < opb * N; i += blockDim.x) {
    const int ol = i / N, r = i % N, o = o0 + ol;
    if (o >= H || r >= m) continue;
    float acc = 0.f;
    for (int ch = 0; ch < chunks; ++ch) acc += part[ol][ch][r];
    y[(int64_t)r * H + o] = acc * __ldg(ds + o);
  }
}

}  // namespace sb
