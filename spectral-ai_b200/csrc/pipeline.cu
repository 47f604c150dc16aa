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
//   * scatter: stable lists instead of atomicAdd slots, so each expert's list
//     is in entry order and the result is deterministic.  Up to 512 experts,
//     every warp owns a contiguous segment of the entries (a histogram row per
//     segment, a scan over the segments, then each warp places its segment);
//     above that, a stream compaction per expert (one CTA per expert).
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
    // -inf inputs are still picked once each); NaN ranks as -inf, as in the
    // thread-per-token kernel, so every chosen id is a valid expert
#pragma unroll
    for (int u = 0; u < PER; ++u)
      if (v[u] != v[u]) v[u] = -INFINITY;
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

// ---------------------------------------------------------------------------
// Thread-per-token form for E <= 64 (the reference's shape): a CTA stages 128
// tokens' rows through shared memory (coalesced), each thread keeps its row in
// registers, the calibration reads W as shared-memory broadcasts, and the
// softmax sums in ascending expert order like the reference kernel.
// ---------------------------------------------------------------------------
constexpr int PIPE_TOK = 128;

// Two fp32 lanes in a 64-bit register; d = a * b + c per lane, each rounded
// once like fmaf.
__device__ __forceinline__ uint64_t pipe_pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void pipe_unpack2(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t pipe_ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

template <int EP>
__global__ void __launch_bounds__(PIPE_TOK, 3) pipe_topk_thread_kernel(
    const float* __restrict__ logits, int64_t B, int E, int k, const float* __restrict__ cal_w,
    const float* __restrict__ cal_b, int apply_softmax, int only_calibrate, float* __restrict__ probs,
    uint32_t* __restrict__ ids, float* __restrict__ wts) {
  // tile rows of EP + 4 floats: 16-byte aligned, and a quarter-warp's float4
  // reads of eight consecutive rows fall in distinct banks
  constexpr int LD = EP + 4;
  extern __shared__ __align__(16) float pipe_dsm[];
  float* wt_s = pipe_dsm;             // [EP][EP] W transposed: wt_s[j*EP + e] = W[e][j]
  float* b_s = wt_s + EP * EP;        // [EP]
  float* tile = b_s + EP;             // [PIPE_TOK][LD] token rows, zero past E
  const int tid = threadIdx.x;
  if (cal_w) {
    for (int i = tid; i < EP * EP; i += PIPE_TOK) {
      const int e = i / EP, j = i % EP;
      wt_s[j * EP + e] = (e < E && j < E) ? __ldg(cal_w + e * E + j) : 0.f;
    }
    for (int e = tid; e < EP; e += PIPE_TOK) b_s[e] = (e < E && cal_b) ? __ldg(cal_b + e) : 0.f;
  }
  const bool vec = E == EP && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  const int E4 = (E + 3) >> 2;  // row length in float4 (zero padded)
  for (int64_t t0 = (int64_t)blockIdx.x * PIPE_TOK; t0 < B; t0 += (int64_t)gridDim.x * PIPE_TOK) {
    const int ntok = (int)((B - t0) < PIPE_TOK ? (B - t0) : PIPE_TOK);
    __syncthreads();
    if (vec) {
      // the tile's rows as float4, all of a thread's loads in flight before
      // the first store to shared memory
      constexpr int Q = EP / 4;  // float4 per row; PIPE_TOK rows, so Q per thread
      const float4* src = reinterpret_cast<const float4*>(logits + t0 * EP);
      float4 r4[Q];
#pragma unroll
      for (int u = 0; u < Q; ++u) {
        const int i = tid + u * PIPE_TOK;
        if (i < ntok * Q) r4[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < Q; ++u) {
        const int i = tid + u * PIPE_TOK;
        if (i < ntok * Q) *reinterpret_cast<float4*>(tile + (i / Q) * LD + (i % Q) * 4) = r4[u];
      }
    } else {
      for (int i = tid; i < ntok * E4 * 4; i += PIPE_TOK) {
        const int r = i / (E4 * 4), c = i % (E4 * 4);
        tile[r * LD + c] = c < E ? __ldg(logits + (t0 + r) * E + c) : 0.f;
      }
    }
    __syncthreads();
    const float* myrow = tile + tid * LD;
    float v[EP];
    if (cal_w) {
      // c[e] = b[e] + sum_j W[e][j] raw[j], j ascending: raw[j..j+3] as one
      // float4 of this thread's row, W's row j as float4 broadcasts; the loop
      // stays rolled (a fully unrolled E x E body overflows the instruction cache)
      // two experts per instruction (fma.rn.f32x2: each lane one fmaf)
      uint64_t vp[EP / 2];
#pragma unroll
      for (int q = 0; q < EP / 2; ++q) vp[q] = *reinterpret_cast<const uint64_t*>(b_s + 2 * q);
#pragma unroll 1
      for (int j4 = 0; j4 < E4; ++j4) {
        const float4 r4 = tid < ntok ? *reinterpret_cast<const float4*>(myrow + 4 * j4) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint64_t r2 = pipe_pack2(rr[jj], rr[jj]);
          const ulonglong2* wr = reinterpret_cast<const ulonglong2*>(wt_s + (4 * j4 + jj) * EP);
#pragma unroll
          for (int q = 0; q < EP / 4; ++q) {
            const ulonglong2 w4 = wr[q];
            vp[2 * q + 0] = pipe_ffma2(w4.x, r2, vp[2 * q + 0]);
            vp[2 * q + 1] = pipe_ffma2(w4.y, r2, vp[2 * q + 1]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < EP / 2; ++q) pipe_unpack2(vp[q], v[2 * q], v[2 * q + 1]);
    } else {
#pragma unroll
      for (int e = 0; e < EP; ++e) v[e] = (e < E && tid < ntok) ? myrow[e] : 0.f;
    }
    if (!only_calibrate && apply_softmax) {
      float m = -INFINITY;
#pragma unroll
      for (int e = 0; e < EP; ++e)
        if (e < E) m = fmaxf(m, v[e]);
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < EP; ++e)
        if (e < E) {
          v[e] = expf(v[e] - m);
          s += v[e];
        }
#pragma unroll
      for (int e = 0; e < EP; ++e) v[e] = v[e] / s;
    }
    if (probs) {  // through the tile for coalesced stores
      __syncthreads();
#pragma unroll
      for (int e = 0; e < EP; ++e)
        if (e < E) tile[tid * LD + e] = v[e];
      __syncthreads();
      for (int i = tid; i < ntok * E; i += PIPE_TOK) probs[t0 * E + i] = tile[(i / E) * LD + i % E];
    }
    if (only_calibrate || tid >= ntok) continue;
    const int64_t t = t0 + tid;
    // experts still to choose from (k <= E, so never empty)
    unsigned long long avail = E >= 64 ? ~0ull : (1ull << E) - 1ull;
    for (int r = 0; r < k; ++r) {
      // the first largest remaining value (NaN ranks as -inf)
      float bv = -INFINITY;
      int bi = -1;
#pragma unroll
      for (int e = 0; e < EP; ++e)
        if (((avail >> e) & 1ull) && v[e] > bv) {
          bv = v[e];
          bi = e;
        }
      if (bi < 0) bi = __ffsll((long long)avail) - 1;  // only -inf left: the lowest remaining expert
      avail &= ~(1ull << bi);
      ids[t * k + r] = (uint32_t)bi;
      if (wts) wts[t * k + r] = bv;
    }
  }
}

// ---------------------------------------------------------------------------
// Scatter for E <= 512 over all SMs, three passes.  Every warp owns one
// contiguous segment of the entries (CTA b, warp w: segment 32 b + w), so the
// segments in row order are the entries in ascending order:
//   hist:    each warp counts its segment per expert (shared-memory atomics
//            into its own row) -> hist[e][segment]
//   offsets: per expert, exclusive sum over the segments (and the totals)
//   place:   each warp walks its segment 32 entries at a time; an entry's slot
//            is its segment's next slot for the expert + its rank among equal
//            ids in the 32 (the equal-id lanes from one ballot per id bit),
//            so slots follow ascending entry order.  No block-wide barrier.
// ---------------------------------------------------------------------------
constexpr int SC_TILE = 1024;
constexpr int SC_WARPS = SC_TILE / 32;
constexpr int SC_MAX_E = 512;

__global__ void __launch_bounds__(SC_TILE) pipe_scatter_hist_kernel(const uint32_t* __restrict__ ids, int64_t R,
                                                                    int64_t seg, int E, int nseg,
                                                                    int32_t* __restrict__ hist) {
  extern __shared__ int h_s[];  // [SC_WARPS][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* h = h_s + warp * E;
  for (int e = lane; e < E; e += 32) h[e] = 0;
  __syncwarp();
  const int s = blockIdx.x * SC_WARPS + warp;
  const int64_t r0 = (int64_t)s * seg, r1 = r0 + seg < R ? r0 + seg : R;
  for (int64_t rb = r0; rb < r1; rb += 8 * 32) {  // eight ids a lane in flight
    uint32_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t r = rb + u * 32 + lane;
      v[u] = r < r1 ? __ldg(ids + r) : 0xffffffffu;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (v[u] < (uint32_t)E) atomicAdd(&h[v[u]], 1);
  }
  __syncwarp();
  for (int e = lane; e < E; e += 32) hist[(int64_t)e * nseg + s] = h[e];
}

// One CTA per expert: exclusive scan of the expert's row of segment counts,
// in place.  The row is staged in shared memory (coalesced), each thread sums
// a run of consecutive segments there, one block-wide scan of the run sums,
// each thread writes its run's prefixes, and the row goes back (coalesced);
// counts[e] = the total.
__global__ void __launch_bounds__(SC_TILE) pipe_scatter_offsets_kernel(int32_t* __restrict__ hist, int nseg, int E,
                                                                       int32_t* __restrict__ counts) {
  __shared__ int wsum[SC_WARPS];
  extern __shared__ int row_s[];  // [nseg]
  const int e = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* grow = hist + (int64_t)e * nseg;
  for (int i = threadIdx.x; i < nseg; i += SC_TILE) row_s[i] = grow[i];
  __syncthreads();
  int* row = row_s;
  const int per = (nseg + SC_TILE - 1) / SC_TILE;
  const int i0 = threadIdx.x * per, i1 = i0 + per < nseg ? i0 + per : nseg;
  int sum = 0;
  for (int i = i0; i < i1; ++i) sum += row[i];
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = wsum[lane];
    int wi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    wsum[lane] = wi - v;
    if (lane == 31) counts[e] = wi;
  }
  __syncthreads();
  int run = wsum[warp] + incl - sum;
  for (int i = i0; i < i1; ++i) {
    const int c = row[i];
    row[i] = run;
    run += c;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nseg; i += SC_TILE) grow[i] = row_s[i];
}

// Lanes of this warp whose key equals this lane's: one ballot per key bit
// (keys below 2^nbits).
__device__ __forceinline__ unsigned pipe_same_key(uint32_t key, int nbits) {
  unsigned same = 0xffffffffu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1u;
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    same &= bit ? bal : ~bal;
  }
  return same;
}

__global__ void __launch_bounds__(SC_TILE) pipe_scatter_place_kernel(const uint32_t* __restrict__ ids, int64_t R,
                                                                     int64_t seg, int k, int E, int nseg, int max_per,
                                                                     int store_entry, const int32_t* __restrict__ offs,
                                                                     int32_t* __restrict__ disp) {
  extern __shared__ int sm[];  // [SC_WARPS][E] next slot of each expert for each warp's segment
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* base = sm + warp * E;
  const int nbits = 32 - __clz(E);  // keys 0..E (E: no expert)
  const int s = blockIdx.x * SC_WARPS + warp;
  for (int e = lane; e < E; e += 32) base[e] = offs[(int64_t)e * nseg + s];
  __syncwarp();
  const int64_t r0 = (int64_t)s * seg, r1 = r0 + seg < R ? r0 + seg : R;
  for (int64_t t0 = r0; t0 < r1; t0 += 8 * 32) {  // warp-uniform trip count
    uint32_t v[8];  // eight steps of ids in flight before the first is placed
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t r = t0 + 32 * u + lane;
      v[u] = r < r1 ? __ldg(ids + r) : 0xffffffffu;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t r = t0 + 32 * u + lane;
      const uint32_t id = v[u];
      const bool valid = id < (uint32_t)E;
      const unsigned same = pipe_same_key(valid ? id : (uint32_t)E, nbits);
      const int rank = __popc(same & ((1u << lane) - 1u));
      if (valid) {
        const int slot = base[id] + rank;
        if (slot < max_per) disp[(int64_t)id * max_per + slot] = store_entry ? (int32_t)r : (int32_t)(r / k);
      }
      __syncwarp();
      if (valid && rank == 0) base[id] += __popc(same);
      __syncwarp();
    }
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
  if (E <= 64 && k <= E) {  // thread per token
    int64_t tb = (B + PIPE_TOK - 1) / PIPE_TOK;
    const int64_t tcap = (int64_t)num_sms() * 8;
    if (tb > tcap) tb = tcap;
    ProfScope prof(name, stream);
    if (E <= 32) {
      const size_t sm = (size_t)(32 * 32 + 32 + PIPE_TOK * 36) * sizeof(float);
      pipe_topk_thread_kernel<32><<<(unsigned)tb, PIPE_TOK, sm, stream>>>(logits, B, E, k, cal_w, cal_b,
                                                                          apply_softmax, only_calibrate, probs, ids,
                                                                          wts);
    } else {
      const size_t sm = (size_t)(64 * 64 + 64 + PIPE_TOK * 68) * sizeof(float);
      static PerDevice attr;
      int dev = 0, rc;
      SB_CUDA_TRY(cudaGetDevice(&dev));
      if ((rc = attr.once(dev, [&]() -> int {
             SB_CUDA_TRY(cudaFuncSetAttribute(pipe_topk_thread_kernel<64>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
             return SB_OK;
           })))
        return rc;
      pipe_topk_thread_kernel<64><<<(unsigned)tb, PIPE_TOK, sm, stream>>>(logits, B, E, k, cal_w, cal_b,
                                                                          apply_softmax, only_calibrate, probs, ids,
                                                                          wts);
    }
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
  }
  ProfScope prof(name, stream);
  int dev = 0;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  SB_REQUIRE(dev < 64, "device ordinal %d out of range", dev);
  // opt-in shared memory (a calibration of up to PIPE_CAL_MAX experts), once per device and kernel
#define SB_PIPE_LAUNCH(P)                                                                                     \
  do {                                                                                                        \
    static PerDevice attr_p;                                                                                  \
    if (smem > 48 * 1024) {                                                                                   \
      const int arc = attr_p.once(dev, [&]() -> int {                                                                  \
        SB_CUDA_TRY(cudaFuncSetAttribute(pipe_softmax_topk_kernel<P>,                                         \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,                         \
                                         PIPE_CAL_MAX * PIPE_CAL_MAX * (int)sizeof(float)));                  \
        return SB_OK;                                                                                         \
      });                                                                                                     \
      if (arc) return arc;                                                                                    \
    }                                                                                                         \
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
  const int64_t R = batch * top_k;
  if (n_experts <= SC_MAX_E && R > SC_TILE) {
    // all SMs: one histogram row per warp segment in stream-ordered scratch
    // from the device's memory pool (concurrent scatters on other streams get
    // their own)
    int64_t nb = (R + 8 * SC_TILE - 1) / (8 * SC_TILE);
    const int64_t cap = (int64_t)num_sms() * 4;
    if (nb > cap) nb = cap;
    int64_t chunk = (R + nb - 1) / nb;
    chunk = (chunk + SC_TILE - 1) / SC_TILE * SC_TILE;  // whole 32-entry steps per warp
    nb = (R + chunk - 1) / chunk;
    const int64_t seg = chunk / SC_WARPS;
    const int nseg = (int)(nb * SC_WARPS);
    const size_t sm_rows = (size_t)SC_WARPS * n_experts * sizeof(int);
    const size_t sm_seg = (size_t)nseg * sizeof(int);  // one expert's row of segment counts
    SB_REQUIRE(sm_seg <= 200 * 1024, "too many scatter segments (%d) for one CTA's shared memory", nseg);
    // opt-in shared memory: the kernels' caps are raised to 200 KB once per device
    static PerDevice attr;
    int dev = 0, arc;
    SB_CUDA_TRY(cudaGetDevice(&dev));
    if ((sm_seg > 48 * 1024 || sm_rows > 48 * 1024) &&
        (arc = attr.once(dev, []() -> int {
           SB_CUDA_TRY(cudaFuncSetAttribute(pipe_scatter_offsets_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
           SB_CUDA_TRY(cudaFuncSetAttribute(pipe_scatter_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
           SB_CUDA_TRY(cudaFuncSetAttribute(pipe_scatter_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024));
           return SB_OK;
         })))
      return arc;
    int32_t* hist = nullptr;
    SB_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&hist), (size_t)nseg * n_experts * sizeof(int32_t), st));
    ProfScope prof("pipe_scatter_by_expert", st);
    pipe_scatter_hist_kernel<<<(unsigned)nb, SC_TILE, sm_rows, st>>>(expert_ids, R, seg, n_experts, nseg, hist);
    pipe_scatter_offsets_kernel<<<n_experts, SC_TILE, sm_seg, st>>>(hist, nseg, n_experts, expert_counts);
    pipe_scatter_place_kernel<<<(unsigned)nb, SC_TILE, sm_rows, st>>>(expert_ids, R, seg, top_k, n_experts, nseg,
                                                                     max_tokens_per_expert, store_entry ? 1 : 0,
                                                                     hist, dispatch_indices);
    SB_CUDA_TRY(cudaGetLastError());
    SB_CUDA_TRY(cudaFreeAsync(hist, st));
    return SB_OK;
  }
  const int grid = n_experts < 65535 ? n_experts : 65535;
  ProfScope prof("pipe_scatter_by_expert", st);
  pipe_scatter_kernel<<<grid, SCATTER_THREADS, 0, st>>>(expert_ids, R, top_k, n_experts, max_tokens_per_expert,
                                                       store_entry ? 1 : 0, dispatch_indices, expert_counts);
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
