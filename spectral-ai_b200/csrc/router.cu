// router.cu — BVH router forward for B200 (sm_100a).
//
// Restates BVHRouter.forward (python/bvh_router.py:269-329) in eval mode as
// four kernels (FAST engine; the EXACT engine swaps 1-3 for fp32 FFMA kernels):
//   1. G = GELU_erf(x W1^T + b1) (bf16) and, in an extra 16-column tail tile of
//      the same tcgen05 GEMM over the same x tiles, pos = x W3^T + b3 with W3
//      split into three bf16 terms so the positions keep fp32 accuracy
//      (SpectralEncoder :84-97, to_3d :232, :285).
//   2. spec = tanh(G W2^T + b2)                      tcgen05 GEMM, bf16 out
//   3. n = sigmoid(spec Wr^T + br) for every node    tcgen05 GEMM (PrismaticRefraction :117-125)
//   4. the level chain of RouterLevel.forward (:156-204): d^2 to every node of
//      the level, logits -d^2 / (2T^2 + 1e-8) plus the parent log-mask
//      log(p_parent + 1e-10), argmax (HARD, :190-193) or softmax(logits/tau)
//      (SOFT, :200-202 without the Gumbel noise), p = p*n / (sum + 1e-8)
//      (:291-311), portals (:100-114), then the MoE top-k + softmax
//      (python/olmoe_extract.py:105-118).  HARD runs one thread per token,
//      SOFT one warp per token.
#include "common.cuh"
#include "gemm_pair.cuh"
#include "gemm_tc.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include <new>
#include <vector>

namespace sb {

// ---------------------------------------------------------------------------
// GEMM epilogues
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
}
__device__ __forceinline__ float sigmoidf_(float z) { return 1.0f / (1.0f + expf(-z)); }

// G = GELU(acc + b1) as bf16; tail tile: pos[row] = hi + (mid + lo) + b3.
struct EpiGeluBf16 {
  const float* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  int N;
  const float* b3d;  // [3]
  float* pos;        // [B, 4]
  __device__ __forceinline__ void apply(int64_t row, int col0, const uint32_t (&r)[32]) const {
    __nv_bfloat16* dst = out + row * ldo + col0;
    if (col0 + 32 <= N && (ldo & 7) == 0) {
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = gelu_erf(__uint_as_float(r[2 * j]) + __ldg(bias + col0 + 2 * j));
        const float b = gelu_erf(__uint_as_float(r[2 * j + 1]) + __ldg(bias + col0 + 2 * j + 1));
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N)
          dst[j] = __float2bfloat16_rn(gelu_erf(__uint_as_float(r[j]) + __ldg(bias + col0 + j)));
    }
  }
  __device__ __forceinline__ void tail(int64_t row, const uint32_t (&r)[32]) const {
    float4 v;
    v.x = __uint_as_float(r[0]) + (__uint_as_float(r[3]) + __uint_as_float(r[6])) + __ldg(b3d + 0);
    v.y = __uint_as_float(r[1]) + (__uint_as_float(r[4]) + __uint_as_float(r[7])) + __ldg(b3d + 1);
    v.z = __uint_as_float(r[2]) + (__uint_as_float(r[5]) + __uint_as_float(r[8])) + __ldg(b3d + 2);
    v.w = 0.f;
    reinterpret_cast<float4*>(pos)[row] = v;
  }
};

// spec = tanh(acc + b2) as bf16 (the A operand of the refraction GEMM).
// C = acc + bias, fp32, row-major [M, ldo].
struct EpiBiasF32 {
  const float* bias;
  float* out;
  int64_t ldo;
  int N;
  __device__ __forceinline__ void apply(int64_t row, int col0, const uint32_t (&r)[32]) const {
    float* dst = out + row * ldo + col0;
    if (col0 + 32 <= N && (ldo & 3) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + j) =
            make_float4(__uint_as_float(r[j]) + __ldg(bias + col0 + j), __uint_as_float(r[j + 1]) + __ldg(bias + col0 + j + 1),
                        __uint_as_float(r[j + 2]) + __ldg(bias + col0 + j + 2),
                        __uint_as_float(r[j + 3]) + __ldg(bias + col0 + j + 3));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = __uint_as_float(r[j]) + __ldg(bias + col0 + j);
    }
  }
  __device__ __forceinline__ void tail(int64_t, const uint32_t (&)[32]) const {}
};

struct EpiTanhBf16 {
  const float* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  int N;
  __device__ __forceinline__ void apply(int64_t row, int col0, const uint32_t (&r)[32]) const {
    __nv_bfloat16* dst = out + row * ldo + col0;
    if (col0 + 32 <= N && (ldo & 7) == 0) {
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = tanhf(__uint_as_float(r[2 * j]) + __ldg(bias + col0 + 2 * j));
        const float b = tanhf(__uint_as_float(r[2 * j + 1]) + __ldg(bias + col0 + 2 * j + 1));
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = __float2bfloat16_rn(tanhf(__uint_as_float(r[j]) + __ldg(bias + col0 + j)));
    }
  }
  __device__ __forceinline__ void tail(int64_t, const uint32_t (&)[32]) const {}
};

// n = sigmoid(acc + br) in fp32, row-major [B, ldn] (SOFT) or node-major
// [nodes, ldn] (HARD, one thread per token reads its own column coalesced).
struct EpiSigmoidN {
  const float* bias;
  float* out;
  int64_t ldn;
  int N;
  int node_major;
  __device__ __forceinline__ void apply(int64_t row, int col0, const uint32_t (&r)[32]) const {
    if (node_major) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) out[(int64_t)(col0 + j) * ldn + row] = sigmoidf_(__uint_as_float(r[j]) + __ldg(bias + col0 + j));
    } else {
      float* dst = out + row * ldn + col0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = sigmoidf_(__uint_as_float(r[j]) + __ldg(bias + col0 + j));
    }
  }
  __device__ __forceinline__ void tail(int64_t, const uint32_t (&)[32]) const {}
};

// ---------------------------------------------------------------------------
// EXACT engine: fp32 FFMA GEMM, C = act(A B^T + bias), A [M,K] fp32|bf16, B [N,K] fp32.
// 128x128 tile, K-step 8, 256 threads, 8x8 outputs per thread.
// ---------------------------------------------------------------------------
enum { ACT_GELU = 0, ACT_TANH = 1, ACT_SIGMOID = 2, ACT_NONE = 3 };

template <typename TA>
__device__ __forceinline__ float to_f32(TA v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// C element (m, n) is stored at C[m * ldc + n], or at C[n * ldc + m] when transposed.
template <typename TA, int ACT>
__global__ void __launch_bounds__(256) sgemm_nt_kernel(const TA* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       const float* __restrict__ bias,
                                                       float* __restrict__ C, int M, int N, int K,
                                                       int64_t ldc, int transposed) {
  __shared__ float As[8][128 + 4];
  __shared__ float Bs[8][128 + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
  const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 8x8 each
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  // loader mapping: 256 threads load 128 rows x 8 k -> 4 elements each
  const int lrow = tid / 2, lk = (tid % 2) * 4;
  for (int k0 = 0; k0 < K; k0 += 8) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + lk + u;
      const int ma = m0 + lrow, nb = n0 + lrow;
      As[lk + u][lrow] = (ma < M && k < K) ? to_f32<TA>(A[(int64_t)ma * K + k]) : 0.f;
      Bs[lk + u][lrow] = (nb < N && k < K) ? B[(int64_t)nb * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[kk][tr * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tc * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + tr * 8 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tc * 8 + j;
      if (n >= N) continue;
      const float v = acc[i][j] + bias[n];
      const float y = ACT == ACT_GELU   ? gelu_erf(v)
                      : ACT == ACT_TANH ? tanhf(v)
                      : ACT == ACT_NONE ? v
                                        : sigmoidf_(v);
      if (transposed)
        C[(int64_t)n * ldc + m] = y;
      else
        C[(int64_t)m * ldc + n] = y;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// (value, index) argmax, ties -> lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}

// EXACT engine: pos = x W3^T + b3 in fp32, one warp per token.
template <typename TX>
__global__ void __launch_bounds__(256) pos_f32_kernel(const TX* __restrict__ x, const float* __restrict__ w3d,
                                                      const float* __restrict__ b3d, int64_t B, int H,
                                                      float* __restrict__ pos) {
  const int lane = threadIdx.x & 31;
  for (int64_t tok = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; tok < B;
       tok += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    const TX* xr = x + tok * (int64_t)H;
    for (int i = lane * 4; i < H; i += 128) {
      float v[4];
      load4(xr + i, v);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a0 = fmaf(v[u], __ldg(w3d + i + u), a0);
        a1 = fmaf(v[u], __ldg(w3d + H + i + u), a1);
        a2 = fmaf(v[u], __ldg(w3d + 2 * H + i + u), a2);
      }
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    a2 = warp_sum(a2);
    if (lane == 0)
      reinterpret_cast<float4*>(pos)[tok] =
          make_float4(a0 + __ldg(b3d + 0), a1 + __ldg(b3d + 1), a2 + __ldg(b3d + 2), 0.f);
  }
}

// ---------------------------------------------------------------------------
// Descent
// ---------------------------------------------------------------------------
struct TreeDev {
  int L;
  int branching[SB_MAX_LEVELS];
  int nodes[SB_MAX_LEVELS];   // N_l
  int offset[SB_MAX_LEVELS];  // first node of level l in the flat arrays
  int total_nodes;
  int max_nodes;
  float denom;  // 2 T^2 + 1e-8 in fp32
  float tau;    // clamp(T, 0.01)
  const float* centers;  // [total,3]
  const float* portals;  // [total,12]
  float bbox[SB_MAX_LEVELS][6];  // per level: min x,y,z then max x,y,z of the centers
  int S;
  const float* refb;     // [total]
  const void* refw;      // [total,S], bf16 (FAST) or fp32 (EXACT)
  int stage;             // 1: the kernel copies centers and portals into shared memory first
};

// Trees up to this many nodes are staged in shared memory by the descent
// kernels (centers and portals, 60 bytes a node): one round of loads at the
// block's start instead of dependent global loads level after level, which is
// what a small batch waits on.
constexpr int STAGE_MAX_NODES = 512;

// Copies the tree's centers [total*3] and portals [total*12] into `sm` (when
// t.stage) and returns the pointers the descent reads them from.
__device__ __forceinline__ void stage_tree(const TreeDev& t, float* sm, const float*& cen, const float*& por) {
  cen = t.centers;
  por = t.portals;
  if (!t.stage) return;
  const int nc = t.total_nodes * 3, np = t.total_nodes * 12;
  for (int i = threadIdx.x; i < nc; i += blockDim.x) sm[i] = __ldg(t.centers + i);
  for (int i = threadIdx.x; i < np; i += blockDim.x) sm[nc + i] = __ldg(t.portals + i);
  __syncthreads();
  cen = sm;
  por = sm + nc;
}

struct DescentOut {
  int32_t* topk_ids;
  float* topk_w;
  int64_t* expert_id;
  float* expert_probs;
  int64_t* route_path;
  float* confidence;
  int k;
};

// HARD: a group of G lanes per token (G = 8 for large batches, 32 when the
// batch is too small to fill the GPU otherwise).  Only the chosen node of a
// level carries probability, so the parent mask is log(p_c + 1e-10) inside the
// chosen parent and log(1e-10) elsewhere, and only the chosen node's refraction
// n = sigmoid(Wr[c] . spec + br[c]) is needed: the group computes it from the
// token's spectral row (bf16 for FAST, fp32 for EXACT), one coalesced row read
// per level.
//
// Exact pruning: after the chosen parent's children are scored, every other
// node of the level has logit <= -dmin^2/denom + log(1e-10), where dmin is the
// distance from the position to the bounding box of the level's centers.  When
// the best in-parent logit beats that bound (with a margin for fp32 rounding),
// no other node can win and the scan over the rest of the level is skipped.
// When any group of the warp cannot prove that, every group of the warp scans
// its whole level (the full scan is always the exact answer), which keeps all
// shuffles warp-uniform.  Either scan is spread over the group's lanes and
// reduced with the first-index rule of torch.argmax.
constexpr int HARD_WARPS = 8;

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;  // butterfly: every lane of the group holds the same bits
}
template <int G>
__device__ __forceinline__ void group_argmax(float& v, int& i) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  // the group's first lane's pair for all of it: with NaN logits the lanes'
  // pairs could differ
  v = __shfl_sync(0xffffffffu, v, 0, G);
  i = __shfl_sync(0xffffffffu, i, 0, G);
}

template <int G>
__device__ __forceinline__ float dot_spec_group(const __nv_bfloat16* sp, const __nv_bfloat16* wp, int S,
                                                int sub) {
  float a0 = 0.f, a1 = 0.f;
  for (int i = sub * 8; i < S; i += 8 * G) {
    const uint4 u = *reinterpret_cast<const uint4*>(sp + i);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(wp + i));
    const __nv_bfloat162* hu = reinterpret_cast<const __nv_bfloat162*>(&u);
    const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __bfloat1622float2(hu[e]), y = __bfloat1622float2(hv[e]);
      a0 = fmaf(x.x, y.x, a0);
      a1 = fmaf(x.y, y.y, a1);
    }
  }
  return group_sum<G>(a0 + a1);
}
template <int G>
__device__ __forceinline__ float dot_spec_group(const float* sp, const float* wp, int S, int sub) {
  float a0 = 0.f, a1 = 0.f;
  for (int i = sub * 4; i < S; i += 4 * G) {
    const float4 u = *reinterpret_cast<const float4*>(sp + i);
    const float4 v = __ldg(reinterpret_cast<const float4*>(wp + i));
    a0 = fmaf(u.x, v.x, fmaf(u.z, v.z, a0));
    a1 = fmaf(u.y, v.y, fmaf(u.w, v.w, a1));
  }
  return group_sum<G>(a0 + a1);
}

template <typename TS, int G>
__global__ void __launch_bounds__(HARD_WARPS * 32) descent_hard_kernel(const float* __restrict__ pos,
                                                                       const TS* __restrict__ spec,
                                                                       int64_t B, TreeDev t, DescentOut o) {
  constexpr int TPW = 32 / G;  // tokens per warp
  extern __shared__ float hsm[];
  const float* cen_all;
  const float* por_all;
  stage_tree(t, hsm, cen_all, por_all);
  const float m_out = logf(0.0f + 1e-10f);
  const TS* __restrict__ wr = static_cast<const TS*>(t.refw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / G, sub = lane % G;
  // the loop runs over whole warps so that every lane takes every shuffle;
  // a group past the end works on the last token and writes nothing
  for (int64_t base = ((int64_t)blockIdx.x * HARD_WARPS + warp) * TPW; base < B;
       base += (int64_t)gridDim.x * HARD_WARPS * TPW) {
    const bool valid = base + grp < B;
    const int64_t tok = valid ? base + grp : B - 1;
    const float4 p4 = reinterpret_cast<const float4*>(pos)[tok];
    float cx = p4.x, cy = p4.y, cz = p4.z;
    const TS* srow = spec + tok * (int64_t)t.S;
    int prev = 0;
    float pc = 1.f;
    int choice = 0;
    for (int l = 0; l < t.L; ++l) {
      const int Nl = t.nodes[l], off = t.offset[l], nb = t.branching[l];
      const float m_in = logf(pc + 1e-10f);
      const int lo = l > 0 ? prev * nb : 0, hi = l > 0 ? lo + nb : Nl;
      const float* cen = cen_all + (size_t)off * 3;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      // a warp-uniform trip count (groups have the same nb; level 0 is whole)
      for (int j0 = 0; j0 < hi - lo; j0 += G) {
        const int j = lo + j0 + sub;
        if (j < hi) {
          const float dx = cx - cen[3 * j], dy = cy - cen[3 * j + 1],
                      dz = cz - cen[3 * j + 2];
          const float d2 = (dx * dx + dy * dy) + dz * dz;
          float lg = -d2 / t.denom;
          if (l > 0) lg = lg + m_in;
          if (lg > best) {  // strided scan: a lane's first maximum is its lowest index
            best = lg;
            bi = j;
          }
        }
      }
      group_argmax<G>(best, bi);
      if (l > 0) {
        const float* bb = t.bbox[l];
        const float ex = fmaxf(fmaxf(bb[0] - cx, cx - bb[3]), 0.f);
        const float ey = fmaxf(fmaxf(bb[1] - cy, cy - bb[4]), 0.f);
        const float ez = fmaxf(fmaxf(bb[2] - cz, cz - bb[5]), 0.f);
        const float bound = -((ex * ex + ey * ey) + ez * ez) / t.denom + m_out;
        const float margin = 1e-4f + 1e-5f * (fabsf(best) + fabsf(bound));
        if (__any_sync(0xffffffffu, !(best > bound + margin))) {
          best = -INFINITY;
          bi = 0x7fffffff;
          for (int j0 = 0; j0 < Nl; j0 += G) {
            const int j = j0 + sub;
            if (j < Nl) {
              const float dx = cx - cen[3 * j], dy = cy - cen[3 * j + 1],
                          dz = cz - cen[3 * j + 2];
              const float d2 = (dx * dx + dy * dy) + dz * dz;
              const float lg = -d2 / t.denom + ((j >= lo && j < hi) ? m_in : m_out);
              if (lg > best) {
                best = lg;
                bi = j;
              }
            }
          }
          group_argmax<G>(best, bi);
        }
      }
      // every logit NaN: torch.argmax would report the first NaN, the scan's first index
      choice = bi == 0x7fffffff ? lo : bi;
      const int node = off + choice;
      const float nv = sigmoidf_(dot_spec_group<G>(srow, wr + (size_t)node * t.S, t.S, sub) + __ldg(t.refb + node));
      pc = nv / (nv + 1e-8f);
      if (o.route_path && valid && sub == 0) o.route_path[tok * t.L + l] = choice;
      if (l < t.L - 1) {
        const float* a = por_all + (size_t)node * 12;
        const float lx = fmaf(a[0], cx, fmaf(a[1], cy, fmaf(a[2], cz, a[3])));
        const float ly = fmaf(a[4], cx, fmaf(a[5], cy, fmaf(a[6], cz, a[7])));
        const float lz = fmaf(a[8], cx, fmaf(a[9], cy, fmaf(a[10], cz, a[11])));
        cx = lx * pc;
        cy = ly * pc;
        cz = lz * pc;
      }
      prev = choice;
    }
    if (!valid) continue;
    const int NL = t.nodes[t.L - 1];
    const bool live = pc > 0.f;  // an all-zero row: argmax returns index 0
    if (o.expert_id && sub == 0) o.expert_id[tok] = live ? choice : 0;
    if (o.confidence && sub == 0) o.confidence[tok] = live ? pc : 0.f;
    if (o.expert_probs) {
      float* row = o.expert_probs + tok * NL;
      for (int j = sub; j < NL; j += G) row[j] = (j == choice) ? pc : 0.f;
    }
    if (o.topk_ids) {
      // top-k of a one-hot row: the chosen expert, then the lowest other ids
      const int k = o.k;
      const float v0 = live ? pc : 0.f;
      const float e0 = 1.f, ez = expf(0.f - v0);
      const float den = live ? e0 + (float)(k - 1) * ez : (float)k;
      for (int i = sub; i < k; i += G) {
        int id;
        float w;
        if (live) {
          id = (i == 0) ? choice : ((i - 1 < choice) ? i - 1 : i);
          w = (i == 0 ? e0 : ez) / den;
        } else {
          id = i;
          w = 1.f / den;
        }
        o.topk_ids[tok * k + i] = id;
        if (o.topk_w) o.topk_w[tok * k + i] = w;
      }
    }
  }
}

constexpr int SOFT_WARPS = 8;

// SOFT: one warp per token.  n is row-major: n[tok * total + node].
// Shared memory: two probability buffers of max_nodes floats per warp.
__global__ void __launch_bounds__(SOFT_WARPS * 32)
    descent_soft_kernel(const float* __restrict__ pos, const float* __restrict__ n, int64_t B, TreeDev t,
                        DescentOut o) {
  extern __shared__ float dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* const pa0 = dsm + (size_t)warp * 2 * t.max_nodes;
  float* const pb0 = pa0 + t.max_nodes;
  const float* cen_all;
  const float* por_all;
  stage_tree(t, dsm + (size_t)SOFT_WARPS * 2 * t.max_nodes, cen_all, por_all);
  for (int64_t tok = (int64_t)blockIdx.x * SOFT_WARPS + warp; tok < B; tok += (int64_t)gridDim.x * SOFT_WARPS) {
    const float4 p4 = reinterpret_cast<const float4*>(pos)[tok];
    float cx = p4.x, cy = p4.y, cz = p4.z;
    const float* nrow = n + tok * (int64_t)t.total_nodes;
    float* pa = pa0;
    float* pb = pb0;
    for (int l = 0; l < t.L; ++l) {
      const int Nl = t.nodes[l], off = t.offset[l], nb = t.branching[l];
      const float* cen = cen_all + (size_t)off * 3;
      float mx = -INFINITY;
      for (int j = lane; j < Nl; j += 32) {
        const float dx = cx - cen[3 * j], dy = cy - cen[3 * j + 1],
                    dz = cz - cen[3 * j + 2];
        const float d2 = (dx * dx + dy * dy) + dz * dz;
        float lg = -d2 / t.denom;
        if (l > 0) lg = lg + logf(pa[j / nb] + 1e-10f);
        lg = lg / t.tau;
        pb[j] = lg;
        mx = fmaxf(mx, lg);
      }
      mx = warp_max(mx);
      float sum = 0.f;
      for (int j = lane; j < Nl; j += 32) {
        const float e = expf(pb[j] - mx);
        pb[j] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      float best = -INFINITY;
      int bi = 0x7fffffff;
      float tot = 0.f;
      for (int j = lane; j < Nl; j += 32) {
        const float pr = pb[j] / sum;
        if (pr > best || (pr == best && j < bi)) {
          best = pr;
          bi = j;
        }
        const float v = pr * __ldg(nrow + off + j);
        pb[j] = v;
        tot += v;
      }
      warp_argmax(best, bi);
      tot = warp_sum(tot);
      const float den = tot + 1e-8f;
      for (int j = lane; j < Nl; j += 32) pb[j] = pb[j] / den;
      __syncwarp();
      // route_path holds the level-global node index (bvh_router.py:322)
      if (o.route_path && lane == 0) o.route_path[tok * t.L + l] = bi;
      if (l < t.L - 1) {
        const float* A = por_all + (size_t)off * 12;
        float sx = 0.f, sy = 0.f, sz = 0.f;
        for (int j = lane; j < Nl; j += 32) {
          const float* a = A + (size_t)j * 12;
          const float pj = pb[j];
          sx += pj * fmaf(a[0], cx, fmaf(a[1], cy, fmaf(a[2], cz, a[3])));
          sy += pj * fmaf(a[4], cx, fmaf(a[5], cy, fmaf(a[6], cz, a[7])));
          sz += pj * fmaf(a[8], cx, fmaf(a[9], cy, fmaf(a[10], cz, a[11])));
        }
        cx = warp_sum(sx);
        cy = warp_sum(sy);
        cz = warp_sum(sz);
      }
      float* tmp = pa;
      pa = pb;
      pb = tmp;
    }
    // last level probabilities are in pa
    const int NL = t.nodes[t.L - 1];
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < NL; j += 32) {
      const float v = pa[j];
      if (o.expert_probs) o.expert_probs[tok * NL + j] = v;
      if (v > best || (v == best && j < bi)) {
        best = v;
        bi = j;
      }
    }
    warp_argmax(best, bi);
    if (o.topk_ids) {
      const int k = o.k;
      float top0 = best, wsum = 0.f, myv = 0.f;
      int myid = 0;
      for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bj = 0x7fffffff;
        for (int j = lane; j < NL; j += 32) {
          const float v = pa[j];
          if (v > bv || (v == bv && j < bj)) {
            bv = v;
            bj = j;
          }
        }
        warp_argmax(bv, bj);
        if (r == 0) top0 = bv;
        const float e = expf(bv - top0);
        wsum += e;
        if (lane == r) {
          myv = e;
          myid = bj;
        }
        __syncwarp();
        if (lane == (bj & 31)) pa[bj] = -INFINITY;
        __syncwarp();
      }
      if (lane < k) {
        o.topk_ids[tok * k + lane] = myid;
        if (o.topk_w) o.topk_w[tok * k + lane] = myv / wsum;
      }
    }
    if (lane == 0) {
      if (o.expert_id) o.expert_id[tok] = bi;
      if (o.confidence) o.confidence[tok] = best;
    }
    __syncwarp();
  }
}

}  // namespace sb

// ===========================================================================
// Host side: handle, upload, forward
// ===========================================================================
struct sb_router {
  int device = 0;
  sb_router_desc desc{};
  int total_nodes = 0;
  int nodes[SB_MAX_LEVELS] = {};
  int offset[SB_MAX_LEVELS] = {};
  int max_nodes = 0;
  int bn_ref = 32;  // tile width of the refraction GEMM
  float temperature = 1.f;
  bool uploaded = false;
  // device-resident parameters
  __nv_bfloat16* w1_bf16 = nullptr;  // [H,H]
  __nv_bfloat16* w2_bf16 = nullptr;  // [S,H]
  __nv_bfloat16* w3s_bf16 = nullptr; // [16,H]: to_3d weights split hi, mid, lo (rows 0-8)
  __nv_bfloat16* wr_bf16 = nullptr;  // [total,S] refraction weights
  float* w1_f32 = nullptr;           // [H,H]
  float* w2_f32 = nullptr;           // [S,H]
  float* b1 = nullptr;               // [H]
  float* b2 = nullptr;               // [S]
  float* w3d = nullptr;              // [3,H]
  float* b3d = nullptr;              // [3]
  float* centers = nullptr;          // [total,3]
  float* refw = nullptr;             // [total,S]
  float* refb = nullptr;             // [total]
  float* portals = nullptr;          // [total,12]
  CUtensorMap tm_w1{}, tm_w2{}, tm_w3s{}, tm_wr{};
  // narrower boxes for small batches, where the wide tiles leave SMs idle
  CUtensorMap tm_w1_128{}, tm_w2_64{}, tm_wr_32{};
  // 32-row boxes for batches of a few row blocks: the weights (W1 is 8 MB at
  // hidden 2048) are then streamed by many SMs instead of a handful
  CUtensorMap tm_w1_32{}, tm_w2_32{};
  // the position rows split over a CTA pair: 8 of the 16 rows per CTA; W2 in
  // 128-row boxes for the pair GEMM
  CUtensorMap tm_w3s_8{}, tm_w2_128{};
  float bbox[SB_MAX_LEVELS][6] = {};  // per level: min x,y,z, max x,y,z of the centers
};

namespace sb {
namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

void free_router_buffers(sb_router* h) {
  void* ptrs[] = {h->w1_bf16, h->w2_bf16, h->w3s_bf16, h->wr_bf16, h->w1_f32, h->w2_f32, h->b1,
                  h->b2,      h->w3d,     h->b3d,      h->centers, h->refw,   h->refb,   h->portals};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  h->w1_bf16 = h->w2_bf16 = h->w3s_bf16 = h->wr_bf16 = nullptr;
  h->w1_f32 = h->w2_f32 = h->b1 = h->b2 = h->w3d = h->b3d = nullptr;
  h->centers = h->refw = h->refb = h->portals = nullptr;
}

template <typename T>
int dev_alloc(T** p, size_t count) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16);
  if (e != cudaSuccess) return fail(SB_ERR_NOMEM, "cudaMalloc(%zu) failed: %s", count * sizeof(T), cudaGetErrorString(e));
  return SB_OK;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

// w [3,H] fp32 -> out [16,H] bf16 with rows c, 3+c, 6+c = hi, mid, lo of row c
// (w = hi + mid + lo to within 2^-24 relative); rows 9..15 are zero.
__global__ void split3_bf16_kernel(const float* __restrict__ w, int H, __nv_bfloat16* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 16 * H; i += gridDim.x * blockDim.x) {
    const int r = i / H, col = i % H;
    __nv_bfloat16 v = __float2bfloat16_rn(0.f);
    if (r < 9) {
      const int c = r % 3, part = r / 3;
      const float x = w[c * H + col];
      const __nv_bfloat16 hi = __float2bfloat16_rn(x);
      const float r1 = x - __bfloat162float(hi);
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      const float r2 = r1 - __bfloat162float(mid);
      v = part == 0 ? hi : (part == 1 ? mid : __float2bfloat16_rn(r2));
    }
    out[i] = v;
  }
}

int upload_f32(float* dst, const float* src, size_t count, float fill_if_null) {
  if (src) {
    SB_CUDA_TRY(cudaMemcpy(dst, src, count * sizeof(float), cudaMemcpyHostToDevice));
  } else {
    std::vector<float> tmp(count, fill_if_null);
    SB_CUDA_TRY(cudaMemcpy(dst, tmp.data(), count * sizeof(float), cudaMemcpyHostToDevice));
  }
  return SB_OK;
}

}  // namespace
}  // namespace sb

extern "C" int sb_router_create(const sb_router_desc* desc, int device, sb_router** out) {
  SB_REQUIRE(desc && out, "sb_router_create: null argument");
  *out = nullptr;
  SB_REQUIRE(desc->hidden > 0 && desc->hidden % 8 == 0,
             "hidden=%d must be a positive multiple of 8", desc->hidden);
  SB_REQUIRE(desc->spectral > 0 && desc->spectral % 8 == 0 && desc->spectral <= 4096,
             "spectral=%d must be a positive multiple of 8 (at most 4096)", desc->spectral);
  SB_REQUIRE(desc->n_levels >= 1 && desc->n_levels <= SB_MAX_LEVELS, "n_levels=%d must be in [1,%d]",
             desc->n_levels, SB_MAX_LEVELS);
  sb_router* h = new (std::nothrow) sb_router();
  if (!h) return sb::fail(SB_ERR_NOMEM, "out of host memory");
  h->device = device;
  h->desc = *desc;
  int n = 1, total = 0;
  for (int l = 0; l < desc->n_levels; ++l) {
    if (desc->branching[l] < 1) {
      delete h;
      return sb::fail(SB_ERR_INVALID, "branching[%d]=%d must be >= 1", l, desc->branching[l]);
    }
    n *= desc->branching[l];
    if (n > (1 << 16)) {
      delete h;
      return sb::fail(SB_ERR_INVALID, "level %d has %d nodes (max 65536)", l, n);
    }
    h->nodes[l] = n;
    h->offset[l] = total;
    total += n;
    if (n > h->max_nodes) h->max_nodes = n;
  }
  h->total_nodes = total;
  h->bn_ref = total >= 256 ? 256 : (total + 31) / 32 * 32;
  *out = h;
  return SB_OK;
}

extern "C" int sb_router_destroy(sb_router* h) {
  if (!h) return SB_OK;
  {
    sb::DeviceGuard g(h->device);
    sb::free_router_buffers(h);
  }
  delete h;
  return SB_OK;
}

extern "C" int sb_router_upload(sb_router* h, const sb_router_weights* w) {
  using namespace sb;
  SB_REQUIRE(h && w, "sb_router_upload: null argument");
  SB_REQUIRE(w->to3d_w && w->enc1_w && w->enc2_w, "to3d_w, enc1_w and enc2_w are required");
  const int H = h->desc.hidden, S = h->desc.spectral, L = h->desc.n_levels;
  for (int l = 0; l < L; ++l) {
    SB_REQUIRE(w->centers[l] && w->refract_w[l], "level %d: centers and refract_w are required", l);
    if (l < L - 1) SB_REQUIRE(w->portals[l], "level %d: portals are required", l);
  }
  DeviceGuard g(h->device);
  free_router_buffers(h);
  h->uploaded = false;
  int rc;
  const size_t HH = (size_t)H * H, SH = (size_t)S * H, T = (size_t)h->total_nodes;
  if ((rc = dev_alloc(&h->w1_f32, HH)) || (rc = dev_alloc(&h->w2_f32, SH)) ||
      (rc = dev_alloc(&h->w1_bf16, HH)) || (rc = dev_alloc(&h->w2_bf16, SH)) ||
      (rc = dev_alloc(&h->w3s_bf16, (size_t)16 * H)) || (rc = dev_alloc(&h->wr_bf16, T * S)) ||
      (rc = dev_alloc(&h->b1, (size_t)H)) || (rc = dev_alloc(&h->b2, (size_t)S)) ||
      (rc = dev_alloc(&h->w3d, (size_t)3 * H)) || (rc = dev_alloc(&h->b3d, (size_t)3)) ||
      (rc = dev_alloc(&h->centers, T * 3)) || (rc = dev_alloc(&h->refw, T * S)) ||
      (rc = dev_alloc(&h->refb, T)) || (rc = dev_alloc(&h->portals, T * 12))) {
    free_router_buffers(h);
    return rc;
  }
  if ((rc = upload_f32(h->w1_f32, w->enc1_w, HH, 0.f)) || (rc = upload_f32(h->w2_f32, w->enc2_w, SH, 0.f)) ||
      (rc = upload_f32(h->b1, w->enc1_b, H, 0.f)) || (rc = upload_f32(h->b2, w->enc2_b, S, 0.f)) ||
      (rc = upload_f32(h->w3d, w->to3d_w, (size_t)3 * H, 0.f)) || (rc = upload_f32(h->b3d, w->to3d_b, 3, 0.f))) {
    free_router_buffers(h);
    return rc;
  }
  for (int l = 0; l < L; ++l) {
    const size_t off = h->offset[l], n = h->nodes[l];
    for (int a = 0; a < 3; ++a) {
      float mn = INFINITY, mx = -INFINITY;
      for (size_t j = 0; j < n; ++j) {
        const float v = w->centers[l][j * 3 + a];
        mn = v < mn ? v : mn;
        mx = v > mx ? v : mx;
      }
      h->bbox[l][a] = mn;
      h->bbox[l][3 + a] = mx;
    }
    if ((rc = upload_f32(h->centers + off * 3, w->centers[l], n * 3, 0.f)) ||
        (rc = upload_f32(h->refw + off * S, w->refract_w[l], n * S, 0.f)) ||
        (rc = upload_f32(h->refb + off, w->refract_b[l], n, 0.f))) {
      free_router_buffers(h);
      return rc;
    }
    if (l < L - 1) {
      if ((rc = upload_f32(h->portals + off * 12, w->portals[l], n * 12, 0.f))) {
        free_router_buffers(h);
        return rc;
      }
    } else {
      SB_CUDA_TRY(cudaMemset(h->portals + off * 12, 0, n * 12 * sizeof(float)));
    }
  }
  f32_to_bf16_kernel<<<1024, 256>>>(h->w1_f32, h->w1_bf16, (int64_t)HH);
  f32_to_bf16_kernel<<<256, 256>>>(h->w2_f32, h->w2_bf16, (int64_t)SH);
  f32_to_bf16_kernel<<<256, 256>>>(h->refw, h->wr_bf16, (int64_t)(T * S));
  split3_bf16_kernel<<<64, 256>>>(h->w3d, H, h->w3s_bf16);
  SB_CUDA_TRY(cudaGetLastError());
  SB_CUDA_TRY(cudaDeviceSynchronize());
  if ((rc = make_tmap_2d(&h->tm_w1, h->w1_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, H, H,
                         GEMM_BK, 256, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, S, H, H,
                         GEMM_BK, S <= 128 ? 128 : 256, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w3s, h->w3s_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 16, H, H,
                         GEMM_BK, TAIL_N, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_wr, h->wr_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, S, S,
                         GEMM_BK, (uint32_t)h->bn_ref, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w1_128, h->w1_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, H, H,
                         GEMM_BK, 128, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2_64, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, S, H, H,
                         GEMM_BK, 64, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_wr_32, h->wr_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, S, S,
                         GEMM_BK, 32, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w3s_8, h->w3s_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 16, H, H,
                         GEMM_BK, 8, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2_128, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, S, H, H,
                         GEMM_BK, S < 128 ? S : 128, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w1_32, h->w1_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, H, H,
                         GEMM_BK, 32, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2_32, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, S, H, H,
                         GEMM_BK, 32, CU_TENSOR_MAP_SWIZZLE_128B))) {
    free_router_buffers(h);
    return rc;
  }
  h->temperature = w->temperature;
  h->uploaded = true;
  return SB_OK;
}

namespace sb {
namespace {

struct RouterWs {
  size_t g, spec, pos, n, total;
};

RouterWs router_ws(const sb_router* h, int64_t B, int precision) {
  RouterWs w{};
  const size_t el = precision == SB_PREC_FAST ? 2 : 4;
  w.g = 0;
  w.spec = align_up((size_t)B * h->desc.hidden * el, 1024);
  w.pos = w.spec + align_up((size_t)B * h->desc.spectral * el, 1024);
  w.n = w.pos + align_up((size_t)B * 16, 1024);
  w.total = w.n + align_up((size_t)B * h->total_nodes * 4, 1024);
  return w;
}

template <int BN, int STAGES, class Epi, bool TAIL = false>
int launch_gemm_tc(const char* name, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2,
                   int M, int N, int K, Epi epi, cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, Epi, TAIL>;
  static PerDevice attr;
  int dev = 0, rc;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  if ((rc = attr.once(dev, [&]() -> int {
         SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
         return SB_OK;
       })))
    return rc;
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN + (TAIL ? 1 : 0));
  const int grid = tiles < num_sms() ? tiles : num_sms();
  ProfScope prof(name, stream);
  kern<<<grid, GEMM_THREADS, C::SMEM_BYTES, stream>>>(ta, tb, tb2, M, N, K, idesc_f16(1, GEMM_BM, BN),
                                                      idesc_f16(1, GEMM_BM, TAIL_N), epi);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

// The CTA-pair GEMM (256 x 256 tiles) as a persistent grid of one pair per
// two SMs (as many as fit: one CTA per SM).
template <class Epi, bool TAIL>
int launch_gemm_pair(const char* name, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2,
                     int M, int N, int K, Epi epi, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<Epi, TAIL>;
  static PerDevice pairs;
  int dev = 0, rc;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(GP_THREADS);
  cfg.dynamicSmemBytes = GP_SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if ((rc = pairs.once(dev, [&]() -> int {
         SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GP_SMEM_BYTES));
         cfg.gridDim = dim3(2 * (num_sms() / 2));
         int n = 0;
         SB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
         if (n < 1) return fail(SB_ERR_CUDA, "no CTA pair of the GEMM fits on this GPU");
         pairs.value[dev] = n;
         return SB_OK;
       })))
    return rc;
  const int tiles = ((M + GP_BM - 1) / GP_BM) * ((N + GP_BN - 1) / GP_BN + (TAIL ? 1 : 0));
  cfg.gridDim = dim3(2 * (tiles < pairs.value[dev] ? tiles : pairs.value[dev]));
  ProfScope prof(name, stream);
  SB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, tb2, M, N, K, idesc_f16(1, GP_BM, GP_BN),
                                 idesc_f16(1, GP_BM, TAIL_N), epi));
  return SB_OK;
}

// SB_ROUTER_GEMM=single keeps the single-CTA GEMM for the wide encoder layer.
bool router_pair_gemm_enabled() {
  static const bool on = [] {
    const char* e = getenv("SB_ROUTER_GEMM");
    return !(e && strcmp(e, "single") == 0);
  }();
  return on;
}

}  // namespace
}  // namespace sb

extern "C" size_t sb_router_workspace_bytes(const sb_router* h, int64_t batch, int precision) {
  if (!h || batch < 0) return 0;
  return sb::router_ws(h, batch, precision).total;
}

extern "C" int sb_router_forward(sb_router* h, const void* x, int x_dtype, int64_t batch,
                                 int precision, int select, int top_k, const sb_router_outputs* out,
                                 void* workspace, size_t workspace_bytes, void* stream_) {
  using namespace sb;
  SB_REQUIRE(h && out, "sb_router_forward: null argument");
  SB_REQUIRE(h->uploaded, "sb_router_forward: weights were not uploaded");
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  SB_REQUIRE(x_dtype == SB_F32 || x_dtype == SB_BF16, "x dtype %d must be SB_F32 or SB_BF16", x_dtype);
  SB_REQUIRE(precision == SB_PREC_FAST || precision == SB_PREC_EXACT, "unknown precision %d", precision);
  SB_REQUIRE(select == SB_SELECT_HARD || select == SB_SELECT_SOFT, "unknown select mode %d", select);
  SB_REQUIRE(precision != SB_PREC_FAST || x_dtype == SB_BF16,
             "FAST precision needs bf16 input (use EXACT for fp32 input)");
  const int L = h->desc.n_levels, NL = h->nodes[L - 1];
  if (out->topk_ids || out->topk_weights) {
    SB_REQUIRE(out->topk_ids, "topk_weights requires topk_ids");
    SB_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= NL, "top_k=%d must be in [1, min(32, %d)]", top_k, NL);
  }
  if (batch == 0) return SB_OK;
  SB_REQUIRE(x != nullptr, "x is null");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0, "x must be 16-byte aligned");
  const RouterWs W = router_ws(h, batch, precision);
  if (!workspace || workspace_bytes < W.total)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, W.total);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  SB_REQUIRE(batch <= (int64_t)INT32_MAX / 2, "batch=%lld too large", (long long)batch);
  const size_t dsm_soft = (size_t)SOFT_WARPS * 2 * h->max_nodes * sizeof(float);
  SB_REQUIRE(select != SB_SELECT_SOFT || dsm_soft <= 227 * 1024,
             "SOFT selection with %d nodes per level exceeds shared memory", h->max_nodes);
  DeviceGuard g(h->device);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int H = h->desc.hidden, S = h->desc.spectral, T = h->total_nodes;
  const int M = (int)batch;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* G = ws + W.g;
  void* spec = ws + W.spec;
  float* pos = reinterpret_cast<float*>(ws + W.pos);
  float* nbuf = reinterpret_cast<float*>(ws + W.n);
  const int node_major = select == SB_SELECT_HARD;
  const int64_t ldn = node_major ? batch : T;
  int rc;
  if (precision == SB_PREC_FAST) {
    CUtensorMap ta, tg, ts;
    if ((rc = make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, H, H, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = make_tmap_2d(&tg, G, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, H, H, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = make_tmap_2d(&ts, spec, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, S, S, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    // Tile widths: the widest tile that still gives every SM work.  A batch of
    // a few thousand tokens has only ceil(M/128) row blocks, so the output
    // columns are split finer there.
    const int64_t mblocks = (M + GEMM_BM - 1) / GEMM_BM;
    const int64_t sms = num_sms();
    EpiGeluBf16 e1{h->b1, static_cast<__nv_bfloat16*>(G), H, H, h->b3d, pos};
    const int64_t pair_tiles = ((M + GP_BM - 1) / GP_BM) * ((H + GP_BN - 1) / GP_BN + 1);
    if (router_pair_gemm_enabled() && pair_tiles >= 2 * (sms / 2))
      // enough 256 x 256 tiles for two rounds over the pairs: the pair GEMM
      rc = launch_gemm_pair<EpiGeluBf16, true>("router_enc1_gelu_tc", ta, h->tm_w1_128, h->tm_w3s_8, M, H, H,
                                               e1, stream);
    else if (mblocks * ((H + 255) / 256 + 1) >= sms)
      rc = launch_gemm_tc<256, 4, EpiGeluBf16, true>("router_enc1_gelu_tc", ta, h->tm_w1, h->tm_w3s, M, H, H,
                                                      e1, stream);
    else if (mblocks * ((H + 127) / 128 + 1) * 2 <= sms)
      // 128-wide tiles would leave half the SMs idle: 32-wide tiles and a
      // deeper ring, so the weight stream is spread over the GPU
      rc = launch_gemm_tc<32, 8, EpiGeluBf16, true>("router_enc1_gelu_tc", ta, h->tm_w1_32, h->tm_w3s, M, H, H,
                                                     e1, stream);
    else
      rc = launch_gemm_tc<128, 4, EpiGeluBf16, true>("router_enc1_gelu_tc", ta, h->tm_w1_128, h->tm_w3s, M, H,
                                                      H, e1, stream);
    if (rc) return rc;
    EpiTanhBf16 e2{h->b2, static_cast<__nv_bfloat16*>(spec), S, S};
    const int64_t pair_tiles2 = ((M + GP_BM - 1) / GP_BM) * ((S + GP_BN - 1) / GP_BN);
    if (router_pair_gemm_enabled() && S % 256 == 0 && pair_tiles2 >= 2 * (sms / 2)) {
      // tm_w1_128's twin for W2: a 128-row box per CTA of the pair
      if ((rc = launch_gemm_pair<EpiTanhBf16, false>("router_enc2_tanh_tc", tg, h->tm_w2_128, h->tm_w2_128, M, S, H,
                                                     e2, stream)))
        return rc;
    } else if (mblocks * ((S + 63) / 64) * 2 <= sms) {
      if ((rc = launch_gemm_tc<32, 8>("router_enc2_tanh_tc", tg, h->tm_w2_32, h->tm_w2_32, M, S, H, e2, stream)))
        return rc;
    } else if (S > 64 && mblocks * ((S + 127) / 128) < sms) {
      if ((rc = launch_gemm_tc<64, 4>("router_enc2_tanh_tc", tg, h->tm_w2_64, h->tm_w2_64, M, S, H, e2, stream)))
        return rc;
    } else if (S <= 128) {  // tm_w2's box height matches this tile width (set at upload)
      if ((rc = launch_gemm_tc<128, 4>("router_enc2_tanh_tc", tg, h->tm_w2, h->tm_w2, M, S, H, e2, stream)))
        return rc;
    } else {
      if ((rc = launch_gemm_tc<256, 4>("router_enc2_tanh_tc", tg, h->tm_w2, h->tm_w2, M, S, H, e2, stream)))
        return rc;
    }
    EpiSigmoidN e3{h->refb, nbuf, ldn, T, node_major};
    if (select == SB_SELECT_HARD) rc = SB_OK;  // HARD evaluates the chosen nodes in the descent
    else if (h->bn_ref > 32 && mblocks * ((T + h->bn_ref - 1) / h->bn_ref) < sms)
      rc = launch_gemm_tc<32, 4>("router_refract_tc", ts, h->tm_wr_32, h->tm_wr_32, M, T, S, e3, stream);
    else switch (h->bn_ref) {  // tm_wr's box height matches this tile width (set at create)
      case 32: rc = launch_gemm_tc<32, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 64: rc = launch_gemm_tc<64, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 96: rc = launch_gemm_tc<96, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 128: rc = launch_gemm_tc<128, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 160: rc = launch_gemm_tc<160, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 192: rc = launch_gemm_tc<192, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      case 224: rc = launch_gemm_tc<224, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
      default: rc = launch_gemm_tc<256, 4>("router_refract_tc", ts, h->tm_wr, h->tm_wr, M, T, S, e3, stream); break;
    }
    if (rc) return rc;
  } else {
    dim3 grid1((H + 127) / 128, (M + 127) / 128), grid2((S + 127) / 128, (M + 127) / 128),
        grid3((T + 127) / 128, (M + 127) / 128);
    float* G32 = static_cast<float*>(G);
    float* S32 = static_cast<float*>(spec);
    {
      ProfScope prof1("router_enc1_gelu_f32", stream);
      if (x_dtype == SB_BF16)
        sgemm_nt_kernel<__nv_bfloat16, ACT_GELU><<<grid1, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), h->w1_f32, h->b1, G32, M, H, H, H, 0);
      else
        sgemm_nt_kernel<float, ACT_GELU><<<grid1, 256, 0, stream>>>(static_cast<const float*>(x), h->w1_f32,
                                                                   h->b1, G32, M, H, H, H, 0);
      SB_CUDA_TRY(cudaGetLastError());
    }
    {
      ProfScope prof2("router_enc2_tanh_f32", stream);
      sgemm_nt_kernel<float, ACT_TANH><<<grid2, 256, 0, stream>>>(G32, h->w2_f32, h->b2, S32, M, S, H, S, 0);
      SB_CUDA_TRY(cudaGetLastError());
    }
    if (select == SB_SELECT_SOFT) {
      ProfScope prof3("router_refract_f32", stream);
      sgemm_nt_kernel<float, ACT_SIGMOID><<<grid3, 256, 0, stream>>>(S32, h->refw, h->refb, nbuf, M, T, S,
                                                                     ldn, node_major);
      SB_CUDA_TRY(cudaGetLastError());
    }
    {
      ProfScope prof4("router_pos_f32", stream);
      int64_t blocks = (batch * 32 + 255) / 256;
      if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
      if (x_dtype == SB_BF16)
        pos_f32_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), h->w3d, h->b3d, batch, H, pos);
      else
        pos_f32_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const float*>(x), h->w3d,
                                                                    h->b3d, batch, H, pos);
      SB_CUDA_TRY(cudaGetLastError());
    }
  }
  TreeDev t{};
  t.L = L;
  for (int l = 0; l < L; ++l) {
    t.branching[l] = h->desc.branching[l];
    t.nodes[l] = h->nodes[l];
    t.offset[l] = h->offset[l];
  }
  t.total_nodes = T;
  t.max_nodes = h->max_nodes;
  const float Tm = h->temperature;
  t.denom = 2.0f * (Tm * Tm) + 1e-8f;
  t.tau = Tm < 0.01f ? 0.01f : Tm;
  t.centers = h->centers;
  t.portals = h->portals;
  for (int l = 0; l < L; ++l)
    for (int a = 0; a < 6; ++a) t.bbox[l][a] = h->bbox[l][a];
  t.S = S;
  t.refb = h->refb;
  t.refw = precision == SB_PREC_FAST ? static_cast<const void*>(h->wr_bf16) : static_cast<const void*>(h->refw);
  t.stage = h->total_nodes <= STAGE_MAX_NODES ? 1 : 0;
  const size_t stage_bytes = t.stage ? (size_t)h->total_nodes * 15 * sizeof(float) : 0;
  DescentOut o{out->topk_ids, out->topk_weights, out->expert_id, out->expert_probs,
               out->route_path, out->confidence, top_k};
  ProfScope prof("router_descent", stream);
  if (select == SB_SELECT_HARD) {
    // 8 lanes per token once the batch fills every warp slot of the GPU that
    // way; otherwise a whole warp per token for parallelism
    const bool wide = batch < (int64_t)num_sms() * 64 * 4;
    const int tpw = wide ? 1 : 4;
    int64_t blocks = (batch + (int64_t)HARD_WARPS * tpw - 1) / ((int64_t)HARD_WARPS * tpw);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    const dim3 grid((unsigned)blocks), block(HARD_WARPS * 32);
    if (precision == SB_PREC_FAST) {
      const __nv_bfloat16* sp = static_cast<const __nv_bfloat16*>(spec);
      if (wide) descent_hard_kernel<__nv_bfloat16, 32><<<grid, block, stage_bytes, stream>>>(pos, sp, batch, t, o);
      else descent_hard_kernel<__nv_bfloat16, 8><<<grid, block, stage_bytes, stream>>>(pos, sp, batch, t, o);
    } else {
      const float* sp = static_cast<const float*>(spec);
      if (wide) descent_hard_kernel<float, 32><<<grid, block, stage_bytes, stream>>>(pos, sp, batch, t, o);
      else descent_hard_kernel<float, 8><<<grid, block, stage_bytes, stream>>>(pos, sp, batch, t, o);
    }
  } else {
    if (dsm_soft + stage_bytes > 48 * 1024) {
      // the opt-in limit is per device: set it once on each
      static PerDevice attr;
      int dev = 0, arc;
      SB_CUDA_TRY(cudaGetDevice(&dev));
      if ((arc = attr.once(dev, []() -> int {
             SB_CUDA_TRY(cudaFuncSetAttribute(descent_soft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              227 * 1024));
             return SB_OK;
           })))
        return arc;
    }
    int64_t blocks = (batch + SOFT_WARPS - 1) / SOFT_WARPS;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    descent_soft_kernel<<<(unsigned)blocks, SOFT_WARPS * 32, dsm_soft + stage_bytes, stream>>>(pos, nbuf, batch, t,
                                                                                              o);
  }
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

// ===========================================================================
// Allocation-free router forward
// ===========================================================================
// Some callers cannot allocate device memory at the point where they route a
// batch: a serving process that reserved all of HBM for its own pool at
// start-up (the router then runs inside a request with no allocator to turn
// to), or a host that binds this C ABI from a language runtime that has no
// device allocator at all.  For them sb_router_forward_noalloc takes its
// scratch (the GELU activations and the spectral rows) from this fixed array
// instead of a caller-provided workspace.  Every GPU that loads the library
// holds the array until the process exits.
static __device__ __align__(256) unsigned char g_router_noalloc_scratch[SB_ROUTER_NOALLOC_SCRATCH_BYTES];

namespace sb {
namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};  // device address of the array, per device ordinal
}  // namespace
}  // namespace sb

extern "C" int sb_router_forward_noalloc(sb_router* h, const void* x, int x_dtype, int64_t batch,
                                         int precision, int select, int top_k,
                                         const sb_router_outputs* out, void* stream) {
  using namespace sb;
  SB_REQUIRE(h != nullptr, "sb_router_forward_noalloc: null handle");
  SB_REQUIRE(h->device >= 0 && h->device < 64, "device ordinal %d out of range", h->device);
  DeviceGuard g(h->device);
  void* base = nullptr;
  {
    // In host code the array's name is only a host-side stand-in; the device
    // address comes from the runtime, once per device, with that device current.
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[h->device]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_router_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr)
        return fail(SB_ERR_CUDA, "cudaGetSymbolAddress of the router scratch failed: %s",
                    cudaGetErrorString(e));
      g_noalloc_ptr[h->device] = p;
    }
    base = g_noalloc_ptr[h->device];
  }
  // the forward wants 1024-byte-aligned scratch; the array is 256-byte aligned
  const uintptr_t b = reinterpret_cast<uintptr_t>(base);
  const uintptr_t aligned = (b + 1023u) & ~static_cast<uintptr_t>(1023u);
  const size_t usable = SB_ROUTER_NOALLOC_SCRATCH_BYTES - (size_t)(aligned - b);
  if (batch < 0) return fail(SB_ERR_INVALID, "batch=%lld must be >= 0", (long long)batch);
  const size_t need = sb_router_workspace_bytes(h, batch, precision);
  if (need > usable)
    return fail(SB_ERR_INVALID,
                "sb_router_forward_noalloc: batch %lld needs %zu bytes of scratch, more than the "
                "%zu bytes of its fixed array (split the batch or use sb_router_forward)",
                (long long)batch, need, usable);
  return sb_router_forward(h, x, x_dtype, batch, precision, select, top_k, out,
                           reinterpret_cast<void*>(aligned), usable, stream);
}
