// router.cu — BVH router forward for B200 (sm_100a).
//
// Restates BVHRouter.forward (python/bvh_router.py:269-329) in eval mode as
// three kernels:
//   1. G    = GELU_erf(x W1^T + b1)        tcgen05 bf16 GEMM (FAST) or fp32 FFMA (EXACT)
//   2. spec = tanh(G W2^T + b2)            same engines          (SpectralEncoder, :84-97)
//   3. per token, one warp: pos = x W3^T + b3 (fp32), then the level chain of
//      RouterLevel.forward (:156-204) with the parent log-mask over all nodes of
//      each level, refraction sigmoid(W_l spec + b_l) (:117-125), portals
//      (:100-114), normalisation p = p*n/(sum+1e-8) (:291-311), and the MoE
//      top-k + softmax (python/olmoe_extract.py:105-118).
// In HARD mode only the chosen node of each level has non-zero probability,
// so only its refraction row is evaluated (the others multiply a zero).
#include "common.cuh"
#include "gemm_tc.cuh"

#include <math.h>
#include <mutex>
#include <new>

namespace sb {

// ---------------------------------------------------------------------------
// GEMM epilogues
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
}

struct EpiGeluBf16 {
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
};

struct EpiTanhF32 {
  const float* bias;
  float* out;
  int64_t ldo;
  int N;
  __device__ __forceinline__ void apply(int64_t row, int col0, const uint32_t (&r)[32]) const {
    float* dst = out + row * ldo + col0;
    if (col0 + 32 <= N && (ldo & 3) == 0) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 v;
        v.x = tanhf(__uint_as_float(r[4 * j + 0]) + __ldg(bias + col0 + 4 * j + 0));
        v.y = tanhf(__uint_as_float(r[4 * j + 1]) + __ldg(bias + col0 + 4 * j + 1));
        v.z = tanhf(__uint_as_float(r[4 * j + 2]) + __ldg(bias + col0 + 4 * j + 2));
        v.w = tanhf(__uint_as_float(r[4 * j + 3]) + __ldg(bias + col0 + 4 * j + 3));
        d4[j] = v;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) dst[j] = tanhf(__uint_as_float(r[j]) + __ldg(bias + col0 + j));
    }
  }
};

// ---------------------------------------------------------------------------
// EXACT engine: fp32 FFMA GEMM, C = act(A B^T + bias), A [M,K] fp32|bf16, B [N,K] fp32.
// 128x128 tile, K-step 8, 256 threads, 8x8 outputs per thread.
// ---------------------------------------------------------------------------
enum { ACT_GELU = 0, ACT_TANH = 1 };

template <typename TA>
__device__ __forceinline__ float to_f32(TA v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename TA, int ACT>
__global__ void __launch_bounds__(256) sgemm_nt_kernel(const TA* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       const float* __restrict__ bias,
                                                       float* __restrict__ C, int M, int N, int K) {
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
      C[(int64_t)m * N + n] = ACT == ACT_GELU ? gelu_erf(v) : tanhf(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Descent: one warp per token.
// ---------------------------------------------------------------------------
struct TreeDev {
  int L;
  int S;
  int H;
  int branching[SB_MAX_LEVELS];
  int nodes[SB_MAX_LEVELS];   // N_l
  int offset[SB_MAX_LEVELS];  // first node of level l in the flat arrays
  int max_nodes;
  float denom;  // 2 T^2 + 1e-8 in fp32
  float tau;    // clamp(T, 0.01)
  const float* w3d;      // [3,H]
  const float* b3d;      // [3]
  const float* centers;  // [total,3]
  const float* refw;     // [total,S]
  const float* refwT;    // [S,total]
  int total_nodes;
  const float* refb;     // [total]
  const float* portals;  // [total,12]
};

struct DescentOut {
  int32_t* topk_ids;
  float* topk_w;
  int64_t* expert_id;
  float* expert_probs;
  int64_t* route_path;
  float* confidence;
  int k;
};

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

__device__ __forceinline__ float sigmoidf_(float z) { return 1.0f / (1.0f + expf(-z)); }

// dot(spec, refw[node]) over S with spec distributed as spec_r[j] = spec[lane + 32 j]
template <int SPL>
__device__ __forceinline__ float refract_dot(const float* __restrict__ w, const float (&spec_r)[SPL],
                                             int S, int lane) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < SPL; ++j) {
    const int s = lane + 32 * j;
    if (s < S) acc = fmaf(spec_r[j], __ldg(w + s), acc);
  }
  return warp_sum(acc);
}

// Loads 8 consecutive input features as fp32.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

constexpr int DESC_WARPS = 8;
constexpr int SPL_MAX = 8;  // spectral dims per lane: S <= 256

// Loads 4 consecutive input features as fp32 (8-byte / 16-byte aligned).
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

constexpr int DESC_TPW = 4;  // tokens per warp iteration sharing the to_3d weight reads

// Shared memory: to_3d weights [3][H] fp32, then (soft mode) two probability
// buffers of max_nodes floats per warp.
template <typename TX>
__global__ void __launch_bounds__(DESC_WARPS * 32)
    descent_kernel(const TX* __restrict__ x, const float* __restrict__ spec, int64_t B, TreeDev t,
                   int soft, DescentOut o) {
  extern __shared__ float dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = t.H, S = t.S, L = t.L;
  float* w3 = dsm;
  for (int i = threadIdx.x; i < 3 * H; i += blockDim.x) w3[i] = t.w3d[i];
  __syncthreads();
  float* pa0 = dsm + 3 * H + (size_t)warp * (2 * t.max_nodes + t.S);  // previous level probs (soft)
  float* pb0 = pa0 + t.max_nodes;                                      // current level probs (soft)
  float* spec_s = pb0 + t.max_nodes;                                   // this token's spectral row (soft)
  const float b3x = __ldg(t.b3d + 0), b3y = __ldg(t.b3d + 1), b3z = __ldg(t.b3d + 2);
  for (int64_t tok0 = ((int64_t)blockIdx.x * DESC_WARPS + warp) * DESC_TPW; tok0 < B;
       tok0 += (int64_t)gridDim.x * DESC_WARPS * DESC_TPW) {
    // ---- pos = to_3d(x) in fp32 for DESC_TPW tokens (bvh_router.py:285)
    float acc[DESC_TPW][3];
#pragma unroll
    for (int u = 0; u < DESC_TPW; ++u) acc[u][0] = acc[u][1] = acc[u][2] = 0.f;
    // four 128-wide chunks per iteration keep 4 x DESC_TPW independent loads in flight
#pragma unroll 4
    for (int i = lane * 4; i < H; i += 128) {
      const float4 wa = *reinterpret_cast<const float4*>(w3 + i);
      const float4 wb = *reinterpret_cast<const float4*>(w3 + H + i);
      const float4 wc = *reinterpret_cast<const float4*>(w3 + 2 * H + i);
      float v[DESC_TPW][4];
#pragma unroll
      for (int u = 0; u < DESC_TPW; ++u) {
        if (tok0 + u < B) {
          load4(x + (tok0 + u) * (int64_t)H + i, v[u]);
        } else {
          v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < DESC_TPW; ++u) {
        acc[u][0] = fmaf(v[u][0], wa.x, fmaf(v[u][1], wa.y, fmaf(v[u][2], wa.z, fmaf(v[u][3], wa.w, acc[u][0]))));
        acc[u][1] = fmaf(v[u][0], wb.x, fmaf(v[u][1], wb.y, fmaf(v[u][2], wb.z, fmaf(v[u][3], wb.w, acc[u][1]))));
        acc[u][2] = fmaf(v[u][0], wc.x, fmaf(v[u][1], wc.y, fmaf(v[u][2], wc.z, fmaf(v[u][3], wc.w, acc[u][2]))));
      }
    }
#pragma unroll
    for (int u = 0; u < DESC_TPW; ++u) {
      acc[u][0] = warp_sum(acc[u][0]);
      acc[u][1] = warp_sum(acc[u][1]);
      acc[u][2] = warp_sum(acc[u][2]);
    }
#pragma unroll 1
    for (int u = 0; u < DESC_TPW; ++u) {
    const int64_t tok = tok0 + u;
    if (tok >= B) break;
    float* pa = pa0;
    float* pb = pb0;
    float cx = acc[0][0] + b3x, cy = acc[0][1] + b3y, cz = acc[0][2] + b3z;
    // select this token's sums without dynamic register indexing
#pragma unroll
    for (int v = 1; v < DESC_TPW; ++v)
      if (u == v) {
        cx = acc[v][0] + b3x;
        cy = acc[v][1] + b3y;
        cz = acc[v][2] + b3z;
      }

    float spec_r[SPL_MAX];
#pragma unroll
    for (int j = 0; j < SPL_MAX; ++j) {
      const int s = lane + 32 * j;
      spec_r[j] = (s < S) ? spec[tok * (int64_t)S + s] : 0.f;
      if (soft && s < S) spec_s[s] = spec_r[j];
    }
    if (soft) __syncwarp();

    int prev_choice = 0;
    float prev_pc = 1.f;  // HARD: probability of the chosen parent
    int choice = 0;
    float pc = 0.f;
    for (int l = 0; l < L; ++l) {
      const int Nl = t.nodes[l], off = t.offset[l], nb = t.branching[l];
      const float* cen = t.centers + (size_t)off * 3;
      if (!soft) {
        // argmax over all Nl logits with the parent log-mask (bvh_router.py:176-192)
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (int j = lane; j < Nl; j += 32) {
          const float dx = cx - __ldg(cen + 3 * j), dy = cy - __ldg(cen + 3 * j + 1),
                      dz = cz - __ldg(cen + 3 * j + 2);
          const float d2 = (dx * dx + dy * dy) + dz * dz;
          float lg = -d2 / t.denom;
          if (l > 0) {
            const float parent = (j / nb == prev_choice) ? prev_pc : 0.f;
            lg = lg + logf(parent + 1e-10f);
          }
          if (lg > best || (lg == best && j < bi)) {
            best = lg;
            bi = j;
          }
        }
        warp_argmax(best, bi);
        choice = bi;
        const float n = sigmoidf_(refract_dot<SPL_MAX>(t.refw + (size_t)(off + choice) * S, spec_r, S, lane) +
                                  __ldg(t.refb + off + choice));
        pc = n / (n + 1e-8f);
      } else {
        // logits, softmax(logits / tau), refraction of every node, normalisation
        float mx = -INFINITY;
        for (int j = lane; j < Nl; j += 32) {
          const float dx = cx - __ldg(cen + 3 * j), dy = cy - __ldg(cen + 3 * j + 1),
                      dz = cz - __ldg(cen + 3 * j + 2);
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
        for (int j = lane; j < Nl; j += 32) {
          const float pr = pb[j] / sum;
          if (pr > best || (pr == best && j < bi)) {
            best = pr;
            bi = j;
          }
          pb[j] = pr;
        }
        warp_argmax(best, bi);
        choice = bi;
        __syncwarp();
        // p_j = probs_j * n_j with n_j = sigmoid(W_j . spec + b_j): one node per lane,
        // refraction weights read transposed ([S][nodes]) so a warp's loads coalesce
        float tot = 0.f;
        for (int j = lane; j < Nl; j += 32) {
          const float* wt = t.refwT + off + j;
          float d0 = 0.f, d1 = 0.f;
          int s = 0;
          for (; s + 1 < S; s += 2) {
            d0 = fmaf(spec_s[s], __ldg(wt + (size_t)s * t.total_nodes), d0);
            d1 = fmaf(spec_s[s + 1], __ldg(wt + (size_t)(s + 1) * t.total_nodes), d1);
          }
          if (s < S) d0 = fmaf(spec_s[s], __ldg(wt + (size_t)s * t.total_nodes), d0);
          const float n = sigmoidf_((d0 + d1) + __ldg(t.refb + off + j));
          const float v = pb[j] * n;
          pb[j] = v;
          tot += v;
        }
        tot = warp_sum(tot);
        __syncwarp();
        const float inv_den = tot + 1e-8f;
        for (int j = lane; j < Nl; j += 32) pb[j] = pb[j] / inv_den;
        __syncwarp();
      }
      // route_path holds the level-global node index (bvh_router.py:322)
      if (o.route_path && lane == 0) o.route_path[tok * L + l] = choice;
      if (l < L - 1) {
        const float* A = t.portals + (size_t)off * 12;
        if (!soft) {
          const float* a = A + (size_t)choice * 12;
          const float lx = fmaf(__ldg(a + 0), cx, fmaf(__ldg(a + 1), cy, fmaf(__ldg(a + 2), cz, __ldg(a + 3))));
          const float ly = fmaf(__ldg(a + 4), cx, fmaf(__ldg(a + 5), cy, fmaf(__ldg(a + 6), cz, __ldg(a + 7))));
          const float lz = fmaf(__ldg(a + 8), cx, fmaf(__ldg(a + 9), cy, fmaf(__ldg(a + 10), cz, __ldg(a + 11))));
          cx = lx * pc;
          cy = ly * pc;
          cz = lz * pc;
        } else {
          float sx = 0.f, sy = 0.f, sz = 0.f;
          for (int j = lane; j < Nl; j += 32) {
            const float* a = A + (size_t)j * 12;
            const float pj = pb[j];
            sx += pj * fmaf(__ldg(a + 0), cx, fmaf(__ldg(a + 1), cy, fmaf(__ldg(a + 2), cz, __ldg(a + 3))));
            sy += pj * fmaf(__ldg(a + 4), cx, fmaf(__ldg(a + 5), cy, fmaf(__ldg(a + 6), cz, __ldg(a + 7))));
            sz += pj * fmaf(__ldg(a + 8), cx, fmaf(__ldg(a + 9), cy, fmaf(__ldg(a + 10), cz, __ldg(a + 11))));
          }
          cx = warp_sum(sx);
          cy = warp_sum(sy);
          cz = warp_sum(sz);
        }
      }
      prev_choice = choice;
      prev_pc = pc;
      if (soft) {
        float* tmp = pa;
        pa = pb;
        pb = tmp;
      }
    }
    // ---- outputs of the last level
    const int NL = t.nodes[L - 1];
    float conf;
    int eid;
    if (!soft) {
      conf = pc;
      eid = choice;
      if (!(pc > 0.f)) {  // all-zero (or NaN) row: argmax returns the first index
        eid = 0;
        conf = pc > 0.f ? pc : 0.f;
      }
      if (o.expert_probs)
        for (int j = lane; j < NL; j += 32) o.expert_probs[tok * NL + j] = (j == choice) ? pc : 0.f;
      if (o.topk_ids) {
        // top-k of a one-hot row: the chosen expert, then the lowest other ids
        const int k = o.k;
        if (lane < k) {
          int id;
          float v;
          if (pc > 0.f) {
            if (lane == 0) {
              id = choice;
              v = pc;
            } else {
              id = (lane - 1 < choice) ? lane - 1 : lane;
              v = 0.f;
            }
          } else {
            id = lane;
            v = pc > 0.f ? pc : 0.f;
          }
          const float v0 = (pc > 0.f) ? pc : 0.f;
          const float e = expf(v - v0);
          const float denom = (pc > 0.f) ? 1.f + (float)(k - 1) * expf(-v0) : (float)k;
          o.topk_ids[tok * k + lane] = id;
          if (o.topk_w) o.topk_w[tok * k + lane] = e / denom;
        }
      }
    } else {
      // expert_probs = pa (swapped above)
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
      eid = bi;
      conf = best;
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
      __syncwarp();
    }
    if (lane == 0) {
      if (o.expert_id) o.expert_id[tok] = eid;
      if (o.confidence) o.confidence[tok] = conf;
    }
    }  // tokens of the group
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
  float temperature = 1.f;
  bool uploaded = false;
  // device-resident parameters
  __nv_bfloat16* w1_bf16 = nullptr;  // [H,H]
  __nv_bfloat16* w2_bf16 = nullptr;  // [S,H]
  float* w1_f32 = nullptr;           // [H,H]
  float* w2_f32 = nullptr;           // [S,H]
  float* b1 = nullptr;               // [H]
  float* b2 = nullptr;               // [S]
  float* w3d = nullptr;              // [3,H]
  float* b3d = nullptr;              // [3]
  float* centers = nullptr;          // [total,3]
  float* refw = nullptr;             // [total,S]
  float* refwT = nullptr;            // [S,total] (soft-mode layout)
  float* refb = nullptr;             // [total]
  float* portals = nullptr;          // [total,12]
  CUtensorMap tm_w1{}, tm_w2{};
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
  void* ptrs[] = {h->w1_bf16, h->w2_bf16, h->w1_f32, h->w2_f32, h->b1,   h->b2,
                  h->w3d,     h->b3d,     h->centers, h->refw,  h->refb, h->portals, h->refwT};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  h->w1_bf16 = h->w2_bf16 = nullptr;
  h->w1_f32 = h->w2_f32 = h->b1 = h->b2 = h->w3d = h->b3d = nullptr;
  h->centers = h->refw = h->refb = h->portals = h->refwT = nullptr;
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

// out[c, r] = in[r, c] for a rows x cols matrix
__global__ void transpose_f32_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t rows,
                                     int64_t cols) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * cols;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    out[c * rows + r] = in[i];
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
  SB_REQUIRE(desc->spectral > 0 && desc->spectral <= 32 * sb::SPL_MAX,
             "spectral=%d must be in [1, %d]", desc->spectral, 32 * sb::SPL_MAX);
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
    if (n > (1 << 20)) {
      delete h;
      return sb::fail(SB_ERR_INVALID, "level %d has %d nodes (max 1048576)", l, n);
    }
    h->nodes[l] = n;
    h->offset[l] = total;
    total += n;
    if (n > h->max_nodes) h->max_nodes = n;
  }
  h->total_nodes = total;
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
      (rc = dev_alloc(&h->b1, (size_t)H)) || (rc = dev_alloc(&h->b2, (size_t)S)) ||
      (rc = dev_alloc(&h->w3d, (size_t)3 * H)) || (rc = dev_alloc(&h->b3d, (size_t)3)) ||
      (rc = dev_alloc(&h->centers, T * 3)) || (rc = dev_alloc(&h->refw, T * S)) ||
      (rc = dev_alloc(&h->refwT, T * S)) ||
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
  transpose_f32_kernel<<<256, 256>>>(h->refw, h->refwT, (int64_t)T, (int64_t)S);
  f32_to_bf16_kernel<<<1024, 256>>>(h->w1_f32, h->w1_bf16, (int64_t)HH);
  f32_to_bf16_kernel<<<256, 256>>>(h->w2_f32, h->w2_bf16, (int64_t)SH);
  SB_CUDA_TRY(cudaGetLastError());
  SB_CUDA_TRY(cudaDeviceSynchronize());
  if ((rc = make_tmap_2d(&h->tm_w1, h->w1_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, H, H,
                         GEMM_BK, 256, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, S, H, H,
                         GEMM_BK, S <= 128 ? 128 : 256, CU_TENSOR_MAP_SWIZZLE_128B))) {
    free_router_buffers(h);
    return rc;
  }
  h->temperature = w->temperature;
  h->uploaded = true;
  return SB_OK;
}

namespace sb {
namespace {
size_t ws_g_bytes(const sb_router* h, int64_t B, int precision) {
  const size_t el = precision == SB_PREC_FAST ? 2 : 4;
  return align_up((size_t)B * h->desc.hidden * el, 1024);
}
size_t ws_spec_bytes(const sb_router* h, int64_t B) {
  return align_up((size_t)B * h->desc.spectral * 4, 1024);
}

template <int BN, int STAGES, class Epi>
int launch_gemm_tc(const char* name, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
                   int K, Epi epi, cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, Epi>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_done[dev] = true;
  }
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  ProfScope prof(name, stream);
  kern<<<grid, GEMM_THREADS, C::SMEM_BYTES, stream>>>(ta, tb, M, N, K, idesc_f16(1, GEMM_BM, BN), epi);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}
}  // namespace
}  // namespace sb

extern "C" size_t sb_router_workspace_bytes(const sb_router* h, int64_t batch, int precision) {
  if (!h || batch < 0) return 0;
  return sb::ws_g_bytes(h, batch, precision) + sb::ws_spec_bytes(h, batch);
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
  const size_t need = sb_router_workspace_bytes(h, batch, precision);
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  SB_REQUIRE(batch <= (int64_t)INT32_MAX / 2, "batch=%lld too large", (long long)batch);
  DeviceGuard g(h->device);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int H = h->desc.hidden, S = h->desc.spectral;
  const int M = (int)batch;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* G = ws;
  float* spec = reinterpret_cast<float*>(ws + ws_g_bytes(h, batch, precision));
  int rc;
  if (precision == SB_PREC_FAST) {
    CUtensorMap ta, tg;
    if ((rc = make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, H, H, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if ((rc = make_tmap_2d(&tg, G, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, H, H, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    EpiGeluBf16 e1{h->b1, static_cast<__nv_bfloat16*>(G), H, H};
    if ((rc = launch_gemm_tc<256, 4>("router_enc1_gelu_tc", ta, h->tm_w1, M, H, H, e1, stream))) return rc;
    EpiTanhF32 e2{h->b2, spec, S, S};
    if (S <= 128) {  // tm_w2's box height matches this tile width (set at upload)
      if ((rc = launch_gemm_tc<128, 4>("router_enc2_tanh_tc", tg, h->tm_w2, M, S, H, e2, stream))) return rc;
    } else {
      if ((rc = launch_gemm_tc<256, 4>("router_enc2_tanh_tc", tg, h->tm_w2, M, S, H, e2, stream))) return rc;
    }
  } else {
    dim3 grid1((H + 127) / 128, (M + 127) / 128), grid2((S + 127) / 128, (M + 127) / 128);
    float* G32 = static_cast<float*>(G);
    {
      ProfScope prof1("router_enc1_gelu_f32", stream);
      if (x_dtype == SB_BF16)
        sgemm_nt_kernel<__nv_bfloat16, ACT_GELU><<<grid1, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), h->w1_f32, h->b1, G32, M, H, H);
      else
        sgemm_nt_kernel<float, ACT_GELU><<<grid1, 256, 0, stream>>>(static_cast<const float*>(x),
                                                                   h->w1_f32, h->b1, G32, M, H, H);
      SB_CUDA_TRY(cudaGetLastError());
    }
    {
      ProfScope prof2("router_enc2_tanh_f32", stream);
      sgemm_nt_kernel<float, ACT_TANH><<<grid2, 256, 0, stream>>>(G32, h->w2_f32, h->b2, spec, M, S, H);
      SB_CUDA_TRY(cudaGetLastError());
    }
  }
  TreeDev t{};
  t.L = L;
  t.S = S;
  t.H = H;
  for (int l = 0; l < L; ++l) {
    t.branching[l] = h->desc.branching[l];
    t.nodes[l] = h->nodes[l];
    t.offset[l] = h->offset[l];
  }
  t.max_nodes = h->max_nodes;
  const float T = h->temperature;
  t.denom = 2.0f * (T * T) + 1e-8f;
  t.tau = T < 0.01f ? 0.01f : T;
  t.w3d = h->w3d;
  t.b3d = h->b3d;
  t.centers = h->centers;
  t.refw = h->refw;
  t.refwT = h->refwT;
  t.total_nodes = h->total_nodes;
  t.refb = h->refb;
  t.portals = h->portals;
  DescentOut o{out->topk_ids, out->topk_weights, out->expert_id, out->expert_probs,
               out->route_path, out->confidence, top_k};
  const size_t dsm = (size_t)3 * H * sizeof(float) +
                     (select == SB_SELECT_SOFT ? (size_t)DESC_WARPS * (2 * h->max_nodes + S) * sizeof(float) : 0);
  if (dsm > 48 * 1024) {
    static bool attr[2] = {false, false};
    auto k0 = descent_kernel<float>;
    auto k1 = descent_kernel<__nv_bfloat16>;
    SB_REQUIRE(dsm <= 227 * 1024, "soft mode with %d nodes per level exceeds shared memory", h->max_nodes);
    if (!attr[0]) { SB_CUDA_TRY(cudaFuncSetAttribute(k0, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)); attr[0] = true; }
    if (!attr[1]) { SB_CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)); attr[1] = true; }
  }
  int64_t blocks = (batch + DESC_WARPS * DESC_TPW - 1) / (DESC_WARPS * DESC_TPW);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  ProfScope prof("router_descent", stream);
  if (x_dtype == SB_BF16)
    descent_kernel<__nv_bfloat16><<<(unsigned)blocks, DESC_WARPS * 32, dsm, stream>>>(
        static_cast<const __nv_bfloat16*>(x), spec, batch, t, select == SB_SELECT_SOFT, o);
  else
    descent_kernel<float><<<(unsigned)blocks, DESC_WARPS * 32, dsm, stream>>>(
        static_cast<const float*>(x), spec, batch, t, select == SB_SELECT_SOFT, o);
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
