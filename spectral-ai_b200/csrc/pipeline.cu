// pipeline.cu — the MoE pipeline's stage kernels around the expert GEMMs:
// calibration + softmax + top-k, scatter of tokens by expert, and the weighted
// combine of the top-k expert outputs.
//
// Reference: cuda/async_pipeline.cu:79-230 (scatter_by_expert_kernel,
// weighted_combine_kernel, apply_calibration_kernel, softmax_topk_kernel) and
// the stage functions of python/async_pipeline_bridge.py:89-150.
//
// B200 shapes of the same steps:
//   * softmax / top-k / calibration: one warp per token (the reference runs
//     one thread per token for the softmax and the top-k scan); values stay in
//     registers, reductions are warp shuffles; the calibration matrix sits
//     transposed in shared memory, loaded once per CTA of a grid-stride loop.
//   * scatter: a stable stream compaction per expert (one CTA per expert, 4096
//     entries per pass, block-wide exclusive scan) instead of atomicAdd slots,
//     so each expert's list is in token order and the result is deterministic.
//   * combine: float4 over the hidden dimension, fused multiply-add over the k
//     slots in slot order (the reference kernel's order).
#include "common.cuh"

namespace sb {

constexpr int PIPE_THREADS = 256;
constexpr int PIPE_CAL_MAX = 128;       // calibration size held in shared memory
constexpr int SCATTER_THREADS = 1024;
constexpr int SCATTER_PER_THREAD = 4;

__device__ __forceinline__ float pipe_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float pipe_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// calibrated[e] = b[e] + sum_j W[e][j] raw[j], j ascending, one fused
// multiply-add per term (apply_calibration_kernel, async_pipeline.cu:150-170).
// Wt is W transposed in shared memory ([j][e], row stride E): lane e reads
// consecutive words.  raw values come from their lanes by shuffle.
template <int PER>
__device__ __forceinline__ void pipe_calibrate(float (&v)[PER], int E, const float* Wt, const float* __restrict__ b,
                                               int lane) {
  float acc[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int e = lane + 32 * u;
    acc[u] = e < E ? __ldg(b + e) : 0.f;
  }
#pragma unroll
  for (int u2 = 0; u2 < PER; ++u2) {
    if (32 * u2 >= E) break;
    for (int s = 0; s < 32; ++s) {
      const int j = 32 * u2 + s;
      if (j >= E) break;
      const float rj = __shfl_sync(0xffffffffu, v[u2], s);
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = lane + 32 * u;
        if (e < E) acc[u] = fmaf(Wt[j * E + e], rj, acc[u]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < PER; ++u) v[u] = acc[u];
}

// One warp per token: [calibration] -> [softmax over E] -> top-k by value,
// larger first, the lower expert index first among equal values (the
// reference's first-maximum scan, async_pipeline.cu:211-224).
template <int PER>
__global__ void __launch_bounds__(PIPE_THREADS) pipe_softmax_topk_kernel(
    const float* __restrict__ logits, int64_t B, int E, int k, const float* __restrict__ cal_w,
    const float* __restrict__ cal_b, int apply_softmax, int only_calibrate, float* __restrict__ probs,
    uint32_t* __restrict__ ids, float* __restrict__ wts) {
  extern __shared__ float wt_s[];  // [E][E] transposed calibration (when cal_w)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (cal_w) {
    for (int i = threadIdx.x; i < E * E; i += blockDim.x) {
      const int e = i / E, j = i % E;  // W[e][j] -> Wt[j][e]
      wt_s[j * E + e] = __ldg(cal_w + i);
    }
    __syncthreads();
  }
  const int64_t wstride = (int64_t)gridDim.x * (PIPE_THREADS / 32);
  for (int64_t t = (int64_t)blockIdx.x * (PIPE_THREADS / 32) + warp; t < B; t += wstride) {
    const float* row = logits + t * E;
    float v[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = lane + 32 * u;
      v[u] = e < E ? __ldg(row + e) : 0.f;
    }
    if (cal_w) pipe_calibrate<PER>(v, E, wt_s, cal_b, lane);
    if (only_calibrate) {
#pragma unroll
      for (int u = 0; u < PER; ++u)
        if (lane + 32 * u < E) probs[t * E + lane + 32 * u] = v[u];
      continue;
    }
    if (apply_softmax) {
      float m = -INFINITY;
#pragma unroll
      for (int u = 0; u < PER; ++u)
        if (lane + 32 * u < E) m = fmaxf(m, v[u]);
      m = pipe_warp_max(m);
      float s = 0.f;
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        if (lane + 32 * u < E) {
          v[u] = expf(v[u] - m);
          s += v[u];
        }
      }
      s = pipe_warp_sum(s);
#pragma unroll
      for (int u = 0; u < PER; ++u) v[u] = v[u] / s;
    }
    if (probs) {
#pragma unroll
      for (int u = 0; u < PER; ++u)
        if (lane + 32 * u < E) probs[t * E + lane + 32 * u] = v[u];
    }
    // top-k by repeated warp argmax; a chosen entry drops out (by a mask, so
    // -inf inputs are still picked once each)
    float sel_v = 0.f;
    uint32_t sel_i = 0;
    unsigned taken = 0;
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = lane + 32 * u;
        if (e < E && !((taken >> u) & 1u) && (v[u] > bv || (v[u] == bv && e < bi))) {
          bv = v[u];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == r) {
        sel_v = bv;
        sel_i = (uint32_t)bi;
      }
#pragma unroll
      for (int u = 0; u < PER; ++u)
        if (lane + 32 * u == bi) taken |= 1u << u;
    }
    if (lane < k) {
      ids[t * k + lane] = sel_i;
      if (wts) wts[t * k + lane] = sel_v;
    }
  }
}

// Stable compaction of one expert's entries (one CTA per expert, grid-stride
// over experts): entry r = t*k + j of ids with ids[r] == e lands at the next
// slot of e in ascending r.  counts[e] is the full count; only slots below
// max_per are stored (scatter_by_expert_kernel, async_pipeline.cu:79-101,
// keeps the same count/limit contract with atomic slots).
__global__ void __launch_bounds__(SCATTER_THREADS) pipe_scatter_kernel(const uint32_t* __restrict__ ids, int64_t R,
                                                                       int k, int E, int max_per, int store_entry,
                                                                       int32_t* __restrict__ disp,
                                                                       int32_t* __restrict__ counts) {
  __shared__ int warp_sum_s[SCATTER_THREADS / 32];
  __shared__ int base_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int CHUNK = SCATTER_THREADS * SCATTER_PER_THREAD;
  for (int e = blockIdx.x; e < E; e += gridDim.x) {
    if (threadIdx.x == 0) base_s = 0;
    __syncthreads();
    for (int64_t r0 = 0; r0 < R; r0 += CHUNK) {
      // thread handles SCATTER_PER_THREAD consecutive entries
      const int64_t rb = r0 + (int64_t)threadIdx.x * SCATTER_PER_THREAD;
      unsigned hit = 0;
#pragma unroll
      for (int q = 0; q < SCATTER_PER_THREAD; ++q)
        if (rb + q < R && __ldg(ids + rb + q) == (uint32_t)e) hit |= 1u << q;
      const int mine = __popc(hit);
      // exclusive scan of `mine` over the block: warp scan + warp totals
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) warp_sum_s[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        const int wv = lane < SCATTER_THREADS / 32 ? warp_sum_s[lane] : 0;
        int wi = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, wi, o);
          if (lane >= o) wi += y;
        }
        if (lane < SCATTER_THREADS / 32) warp_sum_s[lane] = wi - wv;  // exclusive warp offsets
      }
      __syncthreads();
      int slot = base_s + warp_sum_s[warp] + (incl - mine);
#pragma unroll
      for (int q = 0; q < SCATTER_PER_THREAD; ++q) {
        if (hit & (1u << q)) {
          const int64_t r = rb + q;
          if (slot < max_per) disp[(int64_t)e * max_per + slot] = store_entry ? (int32_t)r : (int32_t)(r / k);
          ++slot;
        }
      }
      __syncthreads();
      if (threadIdx.x == SCATTER_THREADS - 1) base_s += warp_sum_s[SCATTER_THREADS / 32 - 1] + incl;
      __syncthreads();
    }
    if (threadIdx.x == 0) counts[e] = base_s;
    __syncthreads();
  }
}

// out[t][d] = sum_j w[t][j] * eo[(t*k + j)][d], j ascending, one fused
// multiply-add per term from 0 (weighted_combine_kernel, async_pipeline.cu:112-132).
__global__ void __launch_bounds__(PIPE_THREADS) pipe_combine_vec4_kernel(const float4* __restrict__ eo,
                                                                         const float* __restrict__ w, int64_t B,
                                                                         int H4, int k, float4* __restrict__ out) {
  const int64_t n = B * H4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H4;
    const int d = (int)(i % H4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const float wj = __ldg(w + t * k + j);
      const float4 v = __ldg(eo + (t * k + j) * H4 + d);
      acc.x = fmaf(wj, v.x, acc.x);
      acc.y = fmaf(wj, v.y, acc.y);
      acc.z = fmaf(wj, v.z, acc.z);
      acc.w = fmaf(wj, v.w, acc.w);
    }
    out[i] = acc;
  }
}

__global__ void __launch_bounds__(PIPE_THREADS) pipe_combine_kernel(const float* __restrict__ eo,
                                                                    const float* __restrict__ w, int64_t B, int H,
                                                                    int k, float* __restrict__ out) {
  const int64_t n = B * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H;
    const int d = (int)(i % H);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc = fmaf(__ldg(w + t * k + j), __ldg(eo + (t * k + j) * H + d), acc);
    out[i] = acc;
  }
}

namespace {

int pipe_launch_softmax_topk(const float* logits, int64_t B, int E, int k, const float* cal_w, const float* cal_b,
                             int apply_softmax, int only_calibrate, float* probs, uint32_t* ids, float* wts,
                             cudaStream_t stream, const char* name) {
  const size_t smem = cal_w ? (size_t)E * E * sizeof(float) : 0;
  int64_t blocks = (B + PIPE_THREADS / 32 - 1) / (PIPE_THREADS / 32);
  const int64_t cap = (int64_t)num_sms() * (cal_w ? 4 : 16);  // calibration: amortise the matrix load
  if (blocks > cap) blocks = cap;
  ProfScope prof(name, stream);
#define SB_PIPE_LAUNCH(P)                                                                                     \
  do {                                                                                                        \
    if (smem > 48 * 1024)                                                                                     \
      SB_CUDA_TRY(cudaFuncSetAttribute(pipe_softmax_topk_kernel<P>,                                           \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));              \
    pipe_softmax_topk_kernel<P><<<(unsigned)blocks, PIPE_THREADS, smem, stream>>>(                           \
        logits, B, E, k, cal_w, cal_b, apply_softmax, only_calibrate, probs, ids, wts);                      \
  } while (0)
  if (E <= 32) SB_PIPE_LAUNCH(1);
  else if (E <= 64) SB_PIPE_LAUNCH(2);
  else if (E <= 128) SB_PIPE_LAUNCH(4);
  else if (E <= 256) SB_PIPE_LAUNCH(8);
  else if (E <= 512) SB_PIPE_LAUNCH(16);
  else SB_PIPE_LAUNCH(32);
#undef SB_PIPE_LAUNCH
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

}  // namespace
}  // namespace sb

extern "C" int sb_softmax_topk(const float* logits, int64_t batch, int n_experts, int top_k, const float* cal_w,
                               const float* cal_b, int apply_softmax, float* probs, uint32_t* topk_ids,
                               float* topk_weights, void* stream) {
  using namespace sb;
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  SB_REQUIRE(n_experts >= 1 && n_experts <= 1024, "n_experts=%d must be in [1, 1024]", n_experts);
  SB_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= n_experts, "top_k=%d must be in [1, min(32, %d)]", top_k,
             n_experts);
  SB_REQUIRE(!cal_w || n_experts <= PIPE_CAL_MAX, "calibration supports n_experts <= %d", PIPE_CAL_MAX);
  SB_REQUIRE(!cal_b || cal_w, "cal_b needs cal_w");
  if (batch == 0) return SB_OK;
  SB_REQUIRE(logits && topk_ids, "logits and topk_ids are required");
  return pipe_launch_softmax_topk(logits, batch, n_experts, top_k, cal_w, cal_b, apply_softmax ? 1 : 0, 0, probs,
                                  topk_ids, topk_weights, reinterpret_cast<cudaStream_t>(stream),
                                  cal_w ? "pipe_cal_softmax_topk" : "pipe_softmax_topk");
}

extern "C" int sb_apply_calibration(const float* raw, int64_t batch, int n_experts, const float* cal_w,
                                    const float* cal_b, float* out, void* stream) {
  using namespace sb;
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  SB_REQUIRE(n_experts >= 1 && n_experts <= PIPE_CAL_MAX, "n_experts=%d must be in [1, %d]", n_experts,
             PIPE_CAL_MAX);
  if (batch == 0) return SB_OK;
  SB_REQUIRE(raw && cal_w && cal_b && out, "raw, cal_w, cal_b and out are required");
  return pipe_launch_softmax_topk(raw, batch, n_experts, 1, cal_w, cal_b, 0, 1, out, nullptr, nullptr,
                                  reinterpret_cast<cudaStream_t>(stream), "pipe_calibration");
}

extern "C" int sb_scatter_by_expert(const uint32_t* expert_ids, int64_t batch, int top_k, int n_experts,
                                    int max_tokens_per_expert, int store_entry, int32_t* dispatch_indices,
                                    int32_t* expert_counts, void* stream) {
  using namespace sb;
  SB_REQUIRE(batch >= 0 && top_k >= 1, "batch=%lld, top_k=%d", (long long)batch, top_k);
  SB_REQUIRE(n_experts >= 1, "n_experts=%d must be >= 1", n_experts);
  SB_REQUIRE(max_tokens_per_expert >= 0, "max_tokens_per_expert=%d must be >= 0", max_tokens_per_expert);
  SB_REQUIRE(batch * top_k <= (int64_t)INT32_MAX, "batch * top_k too large");
  SB_REQUIRE(expert_counts && (dispatch_indices || max_tokens_per_expert == 0),
             "expert_counts and dispatch_indices are required");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (batch == 0) {
    SB_CUDA_TRY(cudaMemsetAsync(expert_counts, 0, (size_t)n_experts * sizeof(int32_t), st));
    return SB_OK;
  }
  SB_REQUIRE(expert_ids != nullptr, "expert_ids is null");
  const int grid = n_experts < 65535 ? n_experts : 65535;
  ProfScope prof("pipe_scatter_by_expert", st);
  pipe_scatter_kernel<<<grid, SCATTER_THREADS, 0, st>>>(expert_ids, batch * top_k, top_k, n_experts,
                                                       max_tokens_per_expert, store_entry ? 1 : 0,
                                                       dispatch_indices, expert_counts);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

extern "C" int sb_weighted_combine(const float* expert_outputs, const float* weights, int64_t batch, int hidden,
                                   int top_k, float* output, void* stream) {
  using namespace sb;
  SB_REQUIRE(batch >= 0 && hidden >= 1 && top_k >= 1, "batch=%lld, hidden=%d, top_k=%d", (long long)batch, hidden,
             top_k);
  if (batch == 0) return SB_OK;
  SB_REQUIRE(expert_outputs && weights && output, "expert_outputs, weights and output are required");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = hidden % 4 == 0 && (reinterpret_cast<uintptr_t>(expert_outputs) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(output) & 15u) == 0;
  const int64_t n = batch * (vec ? hidden / 4 : hidden);
  int64_t blocks = (n + PIPE_THREADS - 1) / PIPE_THREADS;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (blocks > cap) blocks = cap;
  ProfScope prof("pipe_weighted_combine", st);
  if (vec)
    pipe_combine_vec4_kernel<<<(unsigned)blocks, PIPE_THREADS, 0, st>>>(
        reinterpret_cast<const float4*>(expert_outputs), weights, batch, hidden / 4, top_k,
        reinterpret_cast<float4*>(output));
  else
    pipe_combine_kernel<<<(unsigned)blocks, PIPE_THREADS, 0, st>>>(expert_outputs, weights, batch, hidden, top_k,
                                                                  output);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}
