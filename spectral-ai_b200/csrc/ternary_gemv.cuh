// ternary_gemv.cuh — ternary_gated_mlp for a handful of tokens (one expert).
//
// With at most GEMV_ROWS tokens the expert is a weight stream, not a GEMM:
// its 2-bit weights (1.57 MB at the OLMoE shape) are read once and each decoded
// weight meets one to a few tokens.  The tile kernels spend a fixed pipeline of
// TMA loads, unpacking into tensor memory and MMA rounds on each 256-channel
// tile, on 16 SMs for one expert, whatever the token count; here every output
// channel is one warp's dot products, so the expert's rows spread over the
// whole GPU and the time is the weight stream's.  The arithmetic is fp32
// throughout (tokens as given, fp32 or bf16; the hidden state kept in fp32),
// like the reference kernel's (cuda/v5/ternary_torch_ext.cu:123-191, one
// token per CTA).
//
//   gate/up:  h[r, c] = silu(s_g[c] * (T_g[c,:] . x_r)) * (s_u[c] * (T_u[c,:] . x_r))   -> fp32 scratch
//   down:     y[r, o] = s_d[o] * (T_d[o,:] . h_r)                                         -> fp32 output
//
// A block (8 warps) stages the tokens in shared memory as fp32 (n x K x 4
// bytes) and each warp takes one output channel.  A lane loads 16 bytes of the
// packed row per 512 K, all of the row's loads before any arithmetic; the
// pairs of weights are handed out by shuffles so that lane l works on
// K = 64s + 2l, 2l+1 and its shared-memory reads are consecutive 8-byte words
// (no bank conflicts).  Products accumulate in fp32 in the lane, then a warp
// sum.
#pragma once

#include "ternary_gemm.cuh"

namespace sb {

constexpr int GEMV_ROWS = 8;          // tokens at most
constexpr int GEMV_THREADS = 256;     // 8 warps = 8 channels per block
constexpr int GEMV_MAX_K = 4096;      // K <= 8 rounds of 512

// The pair of weights (elements 2j, 2j+1 of word w) as two floats, from the
// bf16 pair tern_pair<1> makes (exact +-1/0).
__device__ __forceinline__ float2 tern_pair_f2(uint32_t w, int j) {
  const uint32_t p = tern_pair<1>(w, j);
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}

// acc[r] = T[row, :] . xs[r, :] over K (a multiple of 64, at most GEMV_MAX_K)
// for r < n; the packed row has K/16 words.  Every lane gets the sums.
template <int R>
__device__ __forceinline__ void gemv_row(const uint32_t* __restrict__ prow, const float* __restrict__ xs, int K,
                                         int n, float (&acc)[R]) {
  const int lane = threadIdx.x & 31;
  const int words = K / 16;
  uint4 q[GEMV_MAX_K / 512];
#pragma unroll
  for (int i = 0; i < GEMV_MAX_K / 512; ++i)
    q[i] = (i * 32 + 4 * lane < words) ? __ldg(reinterpret_cast<const uint4*>(prow) + i * 8 + lane)
                                       : make_uint4(0, 0, 0, 0);
  float part[R];
#pragma unroll
  for (int r = 0; r < R; ++r) part[r] = 0.f;
#pragma unroll
  for (int i = 0; i < GEMV_MAX_K / 512; ++i) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {  // 64 K per step: lane l takes K = 512i + 64s + 2l, +1
      if (i * 32 + 4 * s >= words) break;
      const int src = s * 4 + (lane >> 3);  // word 4s + lane/8 of the round: lane src/4, component src%4
      const uint32_t a = __shfl_sync(0xffffffffu, q[i].x, src >> 2), b = __shfl_sync(0xffffffffu, q[i].y, src >> 2);
      const uint32_t c = __shfl_sync(0xffffffffu, q[i].z, src >> 2), d = __shfl_sync(0xffffffffu, q[i].w, src >> 2);
      const uint32_t word = (src & 3) == 0 ? a : (src & 3) == 1 ? b : (src & 3) == 2 ? c : d;
      const float2 t = tern_pair_f2(word, lane & 7);
      const int kk = 512 * i + 64 * s + 2 * lane;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r < n) {
          const float2 x = *reinterpret_cast<const float2*>(xs + (size_t)r * K + kk);
          part[r] = fmaf(t.x, x.x, fmaf(t.y, x.y, part[r]));
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = part[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    acc[r] = v;
  }
}

// Stages n rows of [*, K] (fp32 or bf16, row stride ld) as fp32 in shared memory.
template <typename TX>
__device__ __forceinline__ void gemv_stage(const TX* __restrict__ src, int64_t ld, int n, int K,
                                           float* __restrict__ xs) {
  for (int i = threadIdx.x; i < n * K; i += blockDim.x) {
    const int r = i / K, c = i % K;
    if constexpr (std::is_same<TX, float>::value)
      xs[i] = __ldg(src + (int64_t)r * ld + c);
    else
      xs[i] = __bfloat162float(src[(int64_t)r * ld + c]);
  }
  __syncthreads();
}

// grid ceil(I / 8): warp w of block b takes channel 8b + w.
template <typename TX>
__global__ void __launch_bounds__(GEMV_THREADS) ternary_gemv_gateup_kernel(
    const TX* __restrict__ x, int n, const uint32_t* __restrict__ gate, const uint32_t* __restrict__ up,
    const float* __restrict__ gs, const float* __restrict__ us, int H, int I, float* __restrict__ h) {
  extern __shared__ float xs[];  // [n, H]
  gemv_stage(x, H, n, H, xs);
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (GEMV_THREADS / 32) + (threadIdx.x >> 5);
  if (c >= I) return;
  float g[GEMV_ROWS], u[GEMV_ROWS];
  gemv_row<GEMV_ROWS>(gate + (int64_t)c * (H / 16), xs, H, n, g);
  gemv_row<GEMV_ROWS>(up + (int64_t)c * (H / 16), xs, H, n, u);
  const float sg = __ldg(gs + c), su = __ldg(us + c);
#pragma unroll
  for (int r = 0; r < GEMV_ROWS; ++r)
    if (r < n && lane == r) h[(int64_t)r * I + c] = silu_fast(g[r] * sg) * (u[r] * su);
}

// grid ceil(H / 8): warp w of block b takes output channel 8b + w.
__global__ void __launch_bounds__(GEMV_THREADS) ternary_gemv_down_kernel(
    const float* __restrict__ h, int n, const uint32_t* __restrict__ down, const float* __restrict__ ds, int H,
    int I, float* __restrict__ y) {
  extern __shared__ float hs[];  // [n, I]
  gemv_stage(h, I, n, I, hs);
  const int lane = threadIdx.x & 31;
  const int o = blockIdx.x * (GEMV_THREADS / 32) + (threadIdx.x >> 5);
  if (o >= H) return;
  float acc[GEMV_ROWS];
  gemv_row<GEMV_ROWS>(down + (int64_t)o * (I / 16), hs, I, n, acc);
  const float sd = __ldg(ds + o);
#pragma unroll
  for (int r = 0; r < GEMV_ROWS; ++r)
    if (r < n && lane == r) y[(int64_t)r * H + o] = acc[r] * sd;
}

}  // namespace sb
