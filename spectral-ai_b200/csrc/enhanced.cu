// enhanced.cu — EnhancedBVHRouter eval forward + BVHGateWrapper top-k on B200.
//
// Reference: python/olmoe_bvh_distill.py:324-632 (HierarchicalLevel,
// EnhancedBVHRouter, spectral_mode off, n_rays = 1) and the "softmax" /
// "topk_softmax" weight modes of BVHGateWrapper.forward, python/olmoe_e2e_eval.py:316-971.
//
// Work per token at hidden 2048 (feature 128, 4x4x4): input_proj.0 2048 -> 512
// is 1.05 M MAC (86 % of the router); input_proj.2 512 -> 256 is 0.13 M; the
// three levels and the expert head are 0.17 M MAC of small layers.
//
//   1. G = GELU(x W0^T + b0)       [B,512]  tcgen05 GEMM (bf16, FAST) or fp32 FFMA GEMM (EXACT)
//   2. P = G W2^T + b2             [B,256]  fp32 out, same two engines
//   3. enh_tail_kernel, 32 tokens per CTA, fp32 CUDA cores:
//      LayerNorm(P) -> level 1 -> level 2 -> level 3 -> expert head -> logits,
//      softmax(logits / max(T, 0.1)), argmax, leaf distances, branch bonus,
//      and the gate's softmax / top-k.  The layer weights are stored transposed
//      ([in][out]) so a warp reads 32 consecutive outputs of one input row;
//      activations sit in shared memory and are read as broadcasts.
#include "common.cuh"

#include <stdlib.h>
#include <string.h>
#include <vector>

namespace sb {

constexpr int ENH_TOK = 32;        // tokens per CTA of the tail kernel
constexpr int ENH_THREADS = 256;
constexpr int ENH_LD = 260;        // activation row stride (256 + pad), floats
constexpr int ENH_LDF = 160;       // feature/concat row stride: F + 3 or F + n1 + n2 + n3
constexpr int ENH_MAXK = 32;       // children per level

// Device copy of the tail weights.  Transposed matrices are [in][out].
struct EnhTail {
  int F, E, n[3];
  float tau_geo;    // 2 T^2 + 1e-8
  float tau_soft;   // max(T, 0.1)
  const float* ln_w;
  const float* ln_b;
  // per level
  const float* centers[3];  // [K,3]
  const float* t3w[3];      // [3][in]   (row-major, a warp reduces over in)
  const float* t3b[3];
  const float* f0t[3];      // [in][F]
  const float* f0b[3];
  const float* f2t[3];      // [F][F]
  const float* f2b[3];
  const float* rhw[3];      // [K][F+3] (row-major)
  const float* rhb[3];
  const float* e0t;         // [F+n1+n2+n3][256]
  const float* e0b;
  const float* e2t;         // [256][E]
  const float* e2b;
};

struct EnhOut {
  float* logits;
  float* probs;
  int64_t* ids;
  float* geo;
  float* bonus;
  float* rprobs;
  float* topw;
  int32_t* topi;
  int k;
  int mode;        // SB_GATE_*
  int norm;        // norm_topk_prob
  int round_bf16;  // logits.to(bfloat16) before the gate
  // SB_GATE_HYBRID: the dense gate's raw logits [B,E] (fp32 accumulate) and
  // the number of BVH candidates
  const float* dense;
  int n_cand;
};

__device__ __forceinline__ float enh_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float enh_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// (value, index) maximum over the warp, equal values toward the lower index
__device__ __forceinline__ void enh_warp_argmax(float& v, int& i) {
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

// out[t][o] = act(b[o] + sum_i in[t][i] Wt[i][o]) for the CTA's 32 tokens.
// Thread (g, o): group g of 256 / Opad threads takes tokens g*TPG .. +TPG-1.
// The sum runs over i in order with one FMA per term.
template <int TPG, bool GELU>
__device__ __forceinline__ void enh_dense(const float* in, int ldi, int I, const float* __restrict__ Wt,
                                          const float* __restrict__ b, int O, int Opad, float* out, int ldo) {
  const int o = threadIdx.x % Opad, g = threadIdx.x / Opad;
  const int t0 = g * TPG;
  if (o >= O || t0 >= ENH_TOK) return;
  float acc[TPG];
  const float bo = __ldg(b + o);
#pragma unroll
  for (int j = 0; j < TPG; ++j) acc[j] = 0.f;
  int i = 0;
#pragma unroll 4
  for (; i + 4 <= I; i += 4) {
    const float w0 = __ldg(Wt + (int64_t)(i + 0) * O + o), w1 = __ldg(Wt + (int64_t)(i + 1) * O + o);
    const float w2 = __ldg(Wt + (int64_t)(i + 2) * O + o), w3 = __ldg(Wt + (int64_t)(i + 3) * O + o);
#pragma unroll
    for (int j = 0; j < TPG; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(in + (t0 + j) * ldi + i);
      acc[j] = fmaf(a.x, w0, acc[j]);
      acc[j] = fmaf(a.y, w1, acc[j]);
      acc[j] = fmaf(a.z, w2, acc[j]);
      acc[j] = fmaf(a.w, w3, acc[j]);
    }
  }
  for (; i < I; ++i) {
    const float w = __ldg(Wt + (int64_t)i * O + o);
#pragma unroll
    for (int j = 0; j < TPG; ++j) acc[j] = fmaf(in[(t0 + j) * ldi + i], w, acc[j]);
  }
#pragma unroll
  for (int j = 0; j < TPG; ++j) {
    const float v = acc[j] + bo;
    out[(t0 + j) * ldo + o] = GELU ? gelu_erf(v) : v;
  }
}

template <bool GELU>
__device__ __forceinline__ void enh_dense_any(const float* in, int ldi, int I, const float* __restrict__ Wt,
                                              const float* __restrict__ b, int O, float* out, int ldo) {
  const int Opad = (O + 31) & ~31;  // O <= 256
  const int groups = ENH_THREADS / Opad;
  if (groups >= 8)
    enh_dense<ENH_TOK / 8, GELU>(in, ldi, I, Wt, b, O, Opad, out, ldo);
  else if (groups >= 4)
    enh_dense<ENH_TOK / 4, GELU>(in, ldi, I, Wt, b, O, Opad, out, ldo);
  else if (groups >= 2)
    enh_dense<ENH_TOK / 2, GELU>(in, ldi, I, Wt, b, O, Opad, out, ldo);
  else
    enh_dense<ENH_TOK, GELU>(in, ldi, I, Wt, b, O, Opad, out, ldo);
}

// One dot product per (token, output) for narrow layers (to_3d, route_head):
// warp w takes tokens w, w+8, ...; lanes split the input and reduce.
__device__ __forceinline__ float enh_dot(const float* in, const float* __restrict__ w, int I, int lane) {
  float a = 0.f;
  for (int i = lane; i < I; i += 32) a = fmaf(in[i], __ldg(w + i), a);
  return enh_warp_sum(a);
}

__device__ __forceinline__ float enh_round(float v, int bf16) {
  return bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// The gate for one token (one warp): logits rounded to the hidden dtype, then
//   SOFTMAX:      router_probs = softmax(lg); top-k of router_probs (renormalised
//                 when norm_topk_prob)
//   TOPK_SOFTMAX: top-k of lg; weights = softmax of those k; router_probs = the
//                 k weights scattered into zeros
// Top-k: largest first, equal values toward the lower index.
__device__ void enh_gate_token(const float* lg, int E, const EnhOut& o, int64_t tok, int lane) {
  constexpr int PER = 8;  // E <= 256
  float v[PER];
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int e = lane + 32 * u;
    v[u] = e < E ? enh_round(lg[e], o.round_bf16) : -INFINITY;
    m = fmaxf(m, v[u]);
  }
  m = enh_warp_max(m);
  float sum = 0.f;
  if (o.mode == SB_GATE_SOFTMAX) {
#pragma unroll
    for (int u = 0; u < PER; ++u) sum += lane + 32 * u < E ? expf(v[u] - m) : 0.f;
    sum = enh_warp_sum(sum);
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = lane + 32 * u;
      if (e < E) {
        v[u] = expf(v[u] - m) / sum;  // router_probs
        if (o.rprobs) o.rprobs[tok * E + e] = v[u];
      }
    }
  } else if (o.rprobs) {
#pragma unroll
    for (int u = 0; u < PER; ++u)
      if (lane + 32 * u < E) o.rprobs[tok * E + lane + 32 * u] = 0.f;
  }
  // top-k by repeated warp argmax; the chosen entry drops to -inf
  float sel_v = 0.f;  // lane j keeps the j-th value
  int sel_i = 0;
  for (int r = 0; r < o.k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = lane + 32 * u;
      if (e < E && (v[u] > bv || (v[u] == bv && e < bi))) {
        bv = v[u];
        bi = e;
      }
    }
    enh_warp_argmax(bv, bi);
    if (lane == r) {
      sel_v = bv;
      sel_i = bi;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u)
      if (lane + 32 * u == bi) v[u] = -INFINITY;
  }
  float w = sel_v;
  if (o.mode == SB_GATE_SOFTMAX) {
    if (o.norm) {
      const float s = enh_warp_sum(lane < o.k ? sel_v : 0.f);
      w = sel_v / s;
    }
  } else {
    const float mk = enh_warp_max(lane < o.k ? sel_v : -INFINITY);
    const float ek = lane < o.k ? expf(sel_v - mk) : 0.f;
    w = ek / enh_warp_sum(ek);
  }
  if (lane < o.k) {
    o.topi[tok * o.k + lane] = sel_i;
    if (o.topw) o.topw[tok * o.k + lane] = w;
    if (o.mode != SB_GATE_SOFTMAX && o.rprobs) o.rprobs[tok * E + sel_i] = w;
  }
}

// Hybrid pre-filter gate of one token (one warp), olmoe_e2e_eval.py:1264-1296:
//   candidates   = topk(expert_probs, n_cand)            (BVH, fp32)
//   router_probs = softmax(round(x W_gate^T), fp32)      (all E experts)
//   top-k of router_probs over the candidates, renormalised when norm.
// expert_probs are recomputed here with the same operations and order as the
// values the tail writes to o.probs, so the candidate set follows those bits.
__device__ void enh_gate_hybrid(const float* lg, int E, float tau, const EnhOut& o, int64_t tok, int lane) {
  constexpr int PER = 8;  // E <= 256
  float pb[PER];
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int e = lane + 32 * u;
    pb[u] = e < E ? lg[e] / tau : -INFINITY;
    m = fmaxf(m, pb[u]);
  }
  m = enh_warp_max(m);
  float sum = 0.f;
#pragma unroll
  for (int u = 0; u < PER; ++u) sum += lane + 32 * u < E ? expf(pb[u] - m) : 0.f;
  sum = enh_warp_sum(sum);
#pragma unroll
  for (int u = 0; u < PER; ++u) pb[u] = lane + 32 * u < E ? expf(pb[u] - m) / sum : -INFINITY;
  // rank of each expert by BVH probability: larger first, lower index first on ties
  int rank[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) rank[u] = 0;
#pragma unroll
  for (int u2 = 0; u2 < PER; ++u2) {
    if (32 * u2 >= E) break;
    for (int s2 = 0; s2 < 32; ++s2) {
      const float pj = __shfl_sync(0xffffffffu, pb[u2], s2);
      const int j = 32 * u2 + s2;
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int e = lane + 32 * u;
        rank[u] += (pj > pb[u] || (pj == pb[u] && j < e)) ? 1 : 0;
      }
    }
  }
  // the dense gate's softmax over all experts
  float d[PER];
  float m2 = -INFINITY;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int e = lane + 32 * u;
    d[u] = e < E ? enh_round(o.dense[tok * E + e], o.round_bf16) : -INFINITY;
    m2 = fmaxf(m2, d[u]);
  }
  m2 = enh_warp_max(m2);
  float s2 = 0.f;
#pragma unroll
  for (int u = 0; u < PER; ++u) s2 += lane + 32 * u < E ? expf(d[u] - m2) : 0.f;
  s2 = enh_warp_sum(s2);
  float v[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int e = lane + 32 * u;
    if (e < E) {
      d[u] = expf(d[u] - m2) / s2;
      if (o.rprobs) o.rprobs[tok * E + e] = d[u];
    }
    v[u] = (e < E && rank[u] < o.n_cand) ? d[u] : -INFINITY;
  }
  // top-k over the candidates by repeated warp argmax
  float sel_v = 0.f;
  int sel_i = 0;
  for (int r = 0; r < o.k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = lane + 32 * u;
      if (e < E && (v[u] > bv || (v[u] == bv && e < bi))) {
        bv = v[u];
        bi = e;
      }
    }
    enh_warp_argmax(bv, bi);
    if (lane == r) {
      sel_v = bv;
      sel_i = bi;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u)
      if (lane + 32 * u == bi) v[u] = -INFINITY;
  }
  float w = sel_v;
  if (o.norm) w = sel_v / enh_warp_sum(lane < o.k ? sel_v : 0.f);
  if (lane < o.k) {
    o.topi[tok * o.k + lane] = sel_i;
    if (o.topw) o.topw[tok * o.k + lane] = w;
  }
}

// Shared memory of the tail kernel, floats.
constexpr int ENH_SMEM_FLOATS = 2 * ENH_TOK * ENH_LD       // X, Z
                                + ENH_TOK * ENH_LDF         // Fb: features | pos | level probs
                                + 3 * ENH_TOK * 4           // positions per level
                                + 3 * ENH_TOK * ENH_MAXK    // leaf distances per level
                                + 3 * ENH_TOK * ENH_MAXK;   // level probabilities
constexpr int ENH_SMEM_BYTES = ENH_SMEM_FLOATS * 4 + 3 * ENH_TOK * 4;  // + level argmaxes

__global__ void __launch_bounds__(ENH_THREADS) enh_tail_kernel(const float* __restrict__ P, int64_t B, EnhTail t,
                                                               EnhOut o) {
  extern __shared__ __align__(16) float esm[];
  float* X = esm;
  float* Z = X + ENH_TOK * ENH_LD;
  float* Fb = Z + ENH_TOK * ENH_LD;
  float* posl = Fb + ENH_TOK * ENH_LDF;           // [3][TOK][4]
  float* distl = posl + 3 * ENH_TOK * 4;          // [3][TOK][MAXK]
  float* probl = distl + 3 * ENH_TOK * ENH_MAXK;  // [3][TOK][MAXK]
  int* amax = reinterpret_cast<int*>(probl + 3 * ENH_TOK * ENH_MAXK);  // [3][TOK]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int F = t.F, E = t.E;

  for (int64_t tb = (int64_t)blockIdx.x * ENH_TOK; tb < B; tb += (int64_t)gridDim.x * ENH_TOK) {
    const int ntok = (int)((B - tb) < ENH_TOK ? (B - tb) : ENH_TOK);
    // ---- LayerNorm(P) -> X (rows past the batch are zero)
    for (int tt = warp; tt < ENH_TOK; tt += ENH_THREADS / 32) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = tt < ntok ? P[(tb + tt) * 256 + lane + 32 * u] : 0.f;
      float s1 = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) s1 += v[u];
      const float mean = enh_warp_sum(s1) / 256.f;
      float s2 = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) s2 = fmaf(v[u] - mean, v[u] - mean, s2);
      const float var = enh_warp_sum(s2) / 256.f;
      const float den = sqrtf(var + 1e-5f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = lane + 32 * u;
        X[tt * ENH_LD + c] = (v[u] - mean) / den * __ldg(t.ln_w + c) + __ldg(t.ln_b + c);
      }
    }
    __syncthreads();
    // ---- three hierarchical levels
    for (int l = 0; l < 3; ++l) {
      const float* in = l == 0 ? X : Fb;
      const int ldi = l == 0 ? ENH_LD : ENH_LDF;
      const int I = l == 0 ? 256 : F;
      const int K = t.n[l];
      // pos = to_3d(in): warp per token
      for (int tt = warp; tt < ENH_TOK; tt += ENH_THREADS / 32) {
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          const float v = enh_dot(in + tt * ldi, t.t3w[l] + a * I, I, lane) + __ldg(t.t3b[l] + a);
          if (lane == 0) posl[(l * ENH_TOK + tt) * 4 + a] = v;
        }
      }
      // Z = GELU(feature_net.0(in))
      enh_dense_any<true>(in, ldi, I, t.f0t[l], t.f0b[l], F, Z, ENH_LD);
      __syncthreads();
      // Fb[:, :F] = feature_net.2(Z); Fb[:, F:F+3] = pos
      enh_dense_any<false>(Z, ENH_LD, F, t.f2t[l], t.f2b[l], F, Fb, ENH_LDF);
      for (int i = threadIdx.x; i < ENH_TOK * 3; i += ENH_THREADS) {
        const int tt = i / 3, a = i % 3;
        Fb[tt * ENH_LDF + F + a] = posl[(l * ENH_TOK + tt) * 4 + a];
      }
      __syncthreads();
      // logits = route_head([f, pos]) + 0.5 geo; probs = softmax(logits / max(T, 0.1))
      for (int tt = warp; tt < ENH_TOK; tt += ENH_THREADS / 32) {
        const float* pp = posl + (l * ENH_TOK + tt) * 4;
        float lg = -INFINITY;
        for (int kk = 0; kk < K; ++kk) {
          const float v = enh_dot(Fb + tt * ENH_LDF, t.rhw[l] + kk * (F + 3), F + 3, lane) + __ldg(t.rhb[l] + kk);
          if (lane == kk) {
            const float* c = t.centers[l] + 3 * kk;
            const float dx = pp[0] - __ldg(c), dy = pp[1] - __ldg(c + 1), dz = pp[2] - __ldg(c + 2);
            const float d2 = (dx * dx + dy * dy) + dz * dz;
            lg = v + 0.5f * (-d2 / t.tau_geo);
            distl[(l * ENH_TOK + tt) * ENH_MAXK + kk] = sqrtf(d2 + 1e-8f);
          }
        }
        const float z = lane < K ? lg / t.tau_soft : -INFINITY;
        const float m = enh_warp_max(z);
        const float ex = lane < K ? expf(z - m) : 0.f;
        const float pr = ex / enh_warp_sum(ex);
        if (lane < K) probl[(l * ENH_TOK + tt) * ENH_MAXK + lane] = pr;
        float bv = lane < K ? pr : -INFINITY;
        int bi = lane < K ? lane : 0x7fffffff;
        enh_warp_argmax(bv, bi);
        if (lane == 0) amax[l * ENH_TOK + tt] = bi;
      }
      __syncthreads();
    }
    // ---- expert head: [f3 | p1 | p2 | p3] -> 256 (GELU) -> E
    const int n1 = t.n[0], n2 = t.n[1], n3 = t.n[2];
    for (int i = threadIdx.x; i < ENH_TOK * (n1 + n2 + n3); i += ENH_THREADS) {
      const int tt = i / (n1 + n2 + n3), c = i % (n1 + n2 + n3);
      const int l = c < n1 ? 0 : (c < n1 + n2 ? 1 : 2);
      const int kk = c - (l == 0 ? 0 : (l == 1 ? n1 : n1 + n2));
      Fb[tt * ENH_LDF + F + c] = probl[(l * ENH_TOK + tt) * ENH_MAXK + kk];
    }
    __syncthreads();
    enh_dense_any<true>(Fb, ENH_LDF, F + n1 + n2 + n3, t.e0t, t.e0b, 256, Z, ENH_LD);
    __syncthreads();
    enh_dense_any<false>(Z, ENH_LD, 256, t.e2t, t.e2b, E, X, ENH_LD);
    __syncthreads();
    // ---- per token outputs (warp per token)
    for (int tt = warp; tt < ntok; tt += ENH_THREADS / 32) {
      const int64_t tok = tb + tt;
      const float* lg = X + tt * ENH_LD;
      // expert_probs = softmax(logits / max(T, 0.1)); ids = argmax
      float m = -INFINITY;
      for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e] / t.tau_soft);
      m = enh_warp_max(m);
      float sum = 0.f;
      for (int e = lane; e < E; e += 32) sum += expf(lg[e] / t.tau_soft - m);
      sum = enh_warp_sum(sum);
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        const float pr = expf(lg[e] / t.tau_soft - m) / sum;
        if (o.logits) o.logits[tok * E + e] = lg[e];
        if (o.probs) o.probs[tok * E + e] = pr;
        if (pr > bv) {
          bv = pr;
          bi = e;
        }
      }
      enh_warp_argmax(bv, bi);
      if (o.ids && lane == 0) o.ids[tok] = bi;
      // leaf distances and branch bonus, expert e = i*n2*n3 + j*n3 + k
      if (o.geo || o.bonus) {
        const int a1 = amax[tt], a2 = amax[ENH_TOK + tt];
        for (int e = lane; e < E; e += 32) {
          const int i = e / (n2 * n3), j = (e % (n2 * n3)) / n3, k = e % n3;
          if (o.geo)
            o.geo[tok * E + e] = (distl[tt * ENH_MAXK + i] + distl[(ENH_TOK + tt) * ENH_MAXK + j]) +
                                 distl[(2 * ENH_TOK + tt) * ENH_MAXK + k];
          if (o.bonus) o.bonus[tok * E + e] = (1.0f + 0.2f * (float)(i == a1)) + 0.1f * (float)(j == a2);
        }
      }
      if (o.topi) {
        if (o.mode == SB_GATE_HYBRID)
          enh_gate_hybrid(lg, E, t.tau_soft, o, tok, lane);
        else
          enh_gate_token(lg, E, o, tok, lane);
      }
    }
    __syncthreads();
  }
}

}  // namespace sb

#include "enhanced_tc.cuh"

namespace sb {

// input_proj.2 + LayerNorm as the GEMM's epilogue (FAST engine with the
// tensor-core tail): X = LN(acc + b2) * ln_w + ln_b over the 256 columns of a
// row, in bf16 [M, 256] — three passes over the row's accumulators in TMEM
// (mean, biased variance, normalise), eps 1e-5 (olmoe_bvh_distill.py:465).
struct EpiLayerNormBf16 {
  static constexpr bool kWholeRow = true;
  const float* bias;
  const float* ln_w;
  const float* ln_b;
  __nv_bfloat16* out;
  __device__ __forceinline__ void apply_row(uint32_t taddr, int64_t row, bool valid) const {
    const float4* b4 = reinterpret_cast<const float4*>(bias);
    float s1 = 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = __ldg(b4 + c * 8 + q);
        s1 += ((__uint_as_float(r[4 * q]) + bb.x) + (__uint_as_float(r[4 * q + 1]) + bb.y)) +
              ((__uint_as_float(r[4 * q + 2]) + bb.z) + (__uint_as_float(r[4 * q + 3]) + bb.w));
      }
    }
    const float mean = s1 / 256.f;
    float s2 = 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = __ldg(b4 + c * 8 + q);
        const float d0 = __uint_as_float(r[4 * q]) + bb.x - mean, d1 = __uint_as_float(r[4 * q + 1]) + bb.y - mean;
        const float d2 = __uint_as_float(r[4 * q + 2]) + bb.z - mean, d3 = __uint_as_float(r[4 * q + 3]) + bb.w - mean;
        s2 = fmaf(d0, d0, s2);
        s2 = fmaf(d1, d1, s2);
        s2 = fmaf(d2, d2, s2);
        s2 = fmaf(d3, d3, s2);
      }
    }
    const float inv = 1.f / sqrtf(s2 / 256.f + 1e-5f);
    const float4* w4 = reinterpret_cast<const float4*>(ln_w);
    const float4* l4 = reinterpret_cast<const float4*>(ln_b);
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), r);
      tmem_ld_wait();
      uint32_t packed[16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = __ldg(b4 + c * 8 + q), ww = __ldg(w4 + c * 8 + q), ll = __ldg(l4 + c * 8 + q);
        const float x0 = (__uint_as_float(r[4 * q]) + bb.x - mean) * inv * ww.x + ll.x;
        const float x1 = (__uint_as_float(r[4 * q + 1]) + bb.y - mean) * inv * ww.y + ll.y;
        const float x2 = (__uint_as_float(r[4 * q + 2]) + bb.z - mean) * inv * ww.z + ll.z;
        const float x3 = (__uint_as_float(r[4 * q + 3]) + bb.w - mean) * inv * ww.w + ll.w;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(x0, x1), h1 = __floats2bfloat162_rn(x2, x3);
        packed[2 * q] = *reinterpret_cast<uint32_t*>(&h0);
        packed[2 * q + 1] = *reinterpret_cast<uint32_t*>(&h1);
      }
      if (valid) {
        uint4* d4 = reinterpret_cast<uint4*>(out + row * 256 + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
      }
    }
  }
  __device__ __forceinline__ void tail(int64_t, const uint32_t (&)[32]) const {}
};

}  // namespace sb

// ===========================================================================
// Host side
// ===========================================================================
struct sb_enh {
  int device = 0;
  int H = 0, F = 0, n[3] = {0, 0, 0}, E = 0;
  bool uploaded = false;
  float temperature = 1.f;
  // input_proj
  __nv_bfloat16* w0_bf16 = nullptr;  // [512,H]
  __nv_bfloat16* w2_bf16 = nullptr;  // [256,512]
  float* w0_f32 = nullptr;
  float* w2_f32 = nullptr;
  float* b0 = nullptr;
  float* b2 = nullptr;
  // tail: one device block holding every small tensor
  float* tail = nullptr;
  size_t tail_floats = 0;
  sb::EnhTail t{};
  CUtensorMap tm_w0{}, tm_w2{};
  // the layer's dense gate for the hybrid pre-filter (sb_enh_set_dense_gate)
  __nv_bfloat16* wg_bf16 = nullptr;  // [E,H]
  float* wg_f32 = nullptr;           // [E,H]
  float* zero_e = nullptr;           // [E] zero bias of the dense gate GEMM
  CUtensorMap tm_wg{};
  // the tail's dense layers as bf16 [N][Kp] blocks for the tensor-core tail
  // (feature 128, <= 64 experts, <= 8 children per level)
  uint16_t* tcw = nullptr;
  sb::EnhTC tc{};
  bool tc_ok = false;
};

namespace sb {
namespace {

struct EnhWs {
  size_t g, p, d, total;
};

EnhWs enh_ws(const sb_enh* h, int64_t B, int precision) {
  EnhWs w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 1024);
    return at;
  };
  w.g = take((size_t)B * 512 * (precision == SB_PREC_FAST ? 2 : 4));
  w.p = take((size_t)B * 256 * 4);
  w.d = take((size_t)B * h->E * 4);  // dense gate logits (hybrid gate only)
  w.total = o;
  return w;
}

void enh_free(sb_enh* h) {
  cudaFree(h->w0_bf16);
  cudaFree(h->w2_bf16);
  cudaFree(h->w0_f32);
  cudaFree(h->w2_f32);
  cudaFree(h->b0);
  cudaFree(h->b2);
  cudaFree(h->tail);
  cudaFree(h->tcw);
  h->w0_bf16 = h->w2_bf16 = nullptr;
  h->w0_f32 = h->w2_f32 = h->b0 = h->b2 = h->tail = nullptr;
  h->tcw = nullptr;
  h->tc_ok = false;
}

uint16_t enh_bf16_bits(float f) {  // round to nearest even
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// The tensor-core tail's weights: each MMA's matrix as bf16 [N][Kp] (rows =
// output features in nn.Linear layout, K zero-padded to 64, N to 16), one
// 1024-byte-aligned block per MMA.  A matrix is a stack of row segments: a
// wide layer plus the narrow layers reading the same input (to_3d rows, the
// feature part of a route head), in the order enhanced_tc.cuh documents.
int enh_build_tc(sb_enh* h, const sb_enh_weights* w) {
  const int F = h->F, E = h->E, n1 = h->n[0], n2 = h->n[1], n3 = h->n[2], nsum = n1 + n2 + n3;
  h->tc_ok = false;
  if (F != ETC_F || E > ETC_MAXE || n1 > ETC_MAXN || n2 > ETC_MAXN || n3 > ETC_MAXN || F + nsum > 192)
    return SB_OK;  // the FFMA tail serves this shape
  struct Seg { const float* src; int rows, ld; };  // rows x K taken from src (row stride ld)
  struct M { Seg seg[3]; int nseg, K; const float* bias; };
  const sb_enh_level* L = w->level;
  const M mats[ETC_LAYERS] = {
      {{{L[0].feat0_w, F, 256}, {L[0].to3d_w, 3, 256}}, 2, 256, h->t.f0b[0]},
      {{{L[0].feat2_w, F, F}}, 1, F, h->t.f2b[0]},
      {{{L[1].feat0_w, F, F}, {L[0].head_w, n1, F + 3}, {L[1].to3d_w, 3, F}}, 3, F, h->t.f0b[1]},
      {{{L[1].feat2_w, F, F}}, 1, F, h->t.f2b[1]},
      {{{L[2].feat0_w, F, F}, {L[1].head_w, n2, F + 3}, {L[2].to3d_w, 3, F}}, 3, F, h->t.f0b[2]},
      {{{L[2].feat2_w, F, F}}, 1, F, h->t.f2b[2]},
      {{{L[2].head_w, n3, F + 3}}, 1, F, h->t.rhb[2]},
      {{{w->eh0_w, 256, F + nsum}}, 1, F + nsum, h->t.e0b},
      {{{w->eh2_w, E, 256}}, 1, 256, h->t.e2b}};
  size_t off[ETC_LAYERS], total = 0;
  int Np[ETC_LAYERS], Kp[ETC_LAYERS];
  for (int l = 0; l < ETC_LAYERS; ++l) {
    int rows = 0;
    for (int g = 0; g < mats[l].nseg; ++g) rows += mats[l].seg[g].rows;
    Np[l] = (rows + 15) / 16 * 16;
    Kp[l] = (mats[l].K + 63) / 64 * 64;
    off[l] = total;
    total += ((size_t)Np[l] * Kp[l] * 2 + 1023) / 1024 * 1024;
  }
  std::vector<uint16_t> blk(total / 2, 0);
  for (int l = 0; l < ETC_LAYERS; ++l) {
    uint16_t* d = blk.data() + off[l] / 2;
    int row = 0;
    for (int g = 0; g < mats[l].nseg; ++g) {
      const Seg& sg = mats[l].seg[g];
      if (!sg.src) return fail(SB_ERR_INVALID, "sb_enh_upload: a tail weight is missing");
      for (int r = 0; r < sg.rows; ++r, ++row)
        for (int k = 0; k < mats[l].K; ++k) d[(size_t)row * Kp[l] + k] = enh_bf16_bits(sg.src[(size_t)r * sg.ld + k]);
    }
  }
  SB_CUDA_TRY(cudaMalloc(&h->tcw, total));
  SB_CUDA_TRY(cudaMemcpy(h->tcw, blk.data(), total, cudaMemcpyHostToDevice));
  for (int l = 0; l < ETC_LAYERS; ++l) {
    int rc = make_tmap_2d(&h->tc.tm[l], h->tcw + off[l] / 2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Np[l], Kp[l], Kp[l],
                          64, (uint32_t)Np[l], CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    h->tc.N[l] = Np[l];
    h->tc.Kp[l] = Kp[l];
    h->tc.bias[l] = mats[l].bias;
  }
  h->tc_ok = true;
  return SB_OK;
}

// SB_ENH_TAIL=simt keeps the FFMA tail for the FAST engine too.
bool enh_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("SB_ENH_TAIL");
    return !(e && strcmp(e, "simt") == 0);
  }();
  return on;
}

void enh_free_gate(sb_enh* h) {
  cudaFree(h->wg_bf16);
  cudaFree(h->wg_f32);
  cudaFree(h->zero_e);
  h->wg_bf16 = nullptr;
  h->wg_f32 = h->zero_e = nullptr;
}

__global__ void enh_gate_convert_kernel(const void* in, int bf16_in, float* f32, __nv_bfloat16* bf, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = bf16_in ? __bfloat162float(static_cast<const __nv_bfloat16*>(in)[i]) : static_cast<const float*>(in)[i];
    f32[i] = v;
    bf[i] = __float2bfloat16_rn(v);
  }
}

__global__ void enh_f32_to_bf16_kernel(const float* in, __nv_bfloat16* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

}  // namespace
}  // namespace sb

extern "C" int sb_enh_create(const sb_enh_desc* desc, int device, sb_enh** out) {
  using namespace sb;
  SB_REQUIRE(desc && out, "sb_enh_create: null argument");
  *out = nullptr;
  SB_REQUIRE(desc->hidden > 0 && desc->hidden % 8 == 0, "hidden=%d must be a positive multiple of 8",
             desc->hidden);
  SB_REQUIRE(desc->feature == 32 || desc->feature == 64 || desc->feature == 128,
             "feature=%d must be 32, 64 or 128", desc->feature);
  int E = 1, sum = 0;
  for (int l = 0; l < 3; ++l) {
    SB_REQUIRE(desc->branching[l] >= 1 && desc->branching[l] <= ENH_MAXK, "branching[%d]=%d must be in [1,%d]",
               l, desc->branching[l], ENH_MAXK);
    E *= desc->branching[l];
    sum += desc->branching[l];
  }
  SB_REQUIRE(E <= 256, "n_level1*n_level2*n_level3=%d must be at most 256", E);
  SB_REQUIRE(desc->feature + sum <= ENH_LDF, "feature + n_level1 + n_level2 + n_level3 = %d exceeds %d",
             desc->feature + sum, ENH_LDF);
  int ndev = 0;
  SB_CUDA_TRY(cudaGetDeviceCount(&ndev));
  SB_REQUIRE(device >= 0 && device < ndev, "device %d out of range", device);
  sb_enh* h = new sb_enh();
  h->device = device;
  h->H = desc->hidden;
  h->F = desc->feature;
  for (int l = 0; l < 3; ++l) h->n[l] = desc->branching[l];
  h->E = E;
  *out = h;
  return SB_OK;
}

extern "C" int sb_enh_upload(sb_enh* h, const sb_enh_weights* w) {
  using namespace sb;
  SB_REQUIRE(h && w, "sb_enh_upload: null argument");
  SB_REQUIRE(w->in0_w && w->in2_w && w->eh0_w && w->eh2_w, "missing weight matrix");
  for (int l = 0; l < 3; ++l)
    SB_REQUIRE(w->level[l].centers && w->level[l].to3d_w && w->level[l].feat0_w && w->level[l].feat2_w &&
                   w->level[l].head_w,
               "missing level %d weights", l + 1);
  DeviceGuard g(h->device);
  enh_free(h);
  h->uploaded = false;
  const int H = h->H, F = h->F, E = h->E;
  const int nsum = h->n[0] + h->n[1] + h->n[2];
  // host staging of the tail block: [ln_w, ln_b, per level ..., head ...]
  std::vector<float> blk;
  std::vector<size_t> off;
  auto put = [&](const float* src, size_t count, float fill) {
    off.push_back(blk.size());
    for (size_t i = 0; i < count; ++i) blk.push_back(src ? src[i] : fill);
    while (blk.size() % 4) blk.push_back(0.f);  // keep 16-byte alignment
  };
  auto put_t = [&](const float* src, int rows, int cols) {  // [rows][cols] -> [cols][rows]
    off.push_back(blk.size());
    for (int c = 0; c < cols; ++c)
      for (int r = 0; r < rows; ++r) blk.push_back(src[(size_t)r * cols + c]);
    while (blk.size() % 4) blk.push_back(0.f);
  };
  put(w->ln_w, 256, 1.f);
  put(w->ln_b, 256, 0.f);
  for (int l = 0; l < 3; ++l) {
    const sb_enh_level& L = w->level[l];
    const int in = l == 0 ? 256 : F, K = h->n[l];
    put(L.centers, (size_t)K * 3, 0.f);
    put(L.to3d_w, (size_t)3 * in, 0.f);
    put(L.to3d_b, 3, 0.f);
    put_t(L.feat0_w, F, in);
    put(L.feat0_b, F, 0.f);
    put_t(L.feat2_w, F, F);
    put(L.feat2_b, F, 0.f);
    put(L.head_w, (size_t)K * (F + 3), 0.f);
    put(L.head_b, K, 0.f);
  }
  put_t(w->eh0_w, 256, F + nsum);
  put(w->eh0_b, 256, 0.f);
  put_t(w->eh2_w, E, 256);
  put(w->eh2_b, E, 0.f);
  SB_CUDA_TRY(cudaMalloc(&h->tail, blk.size() * sizeof(float)));
  SB_CUDA_TRY(cudaMemcpy(h->tail, blk.data(), blk.size() * sizeof(float), cudaMemcpyHostToDevice));
  h->tail_floats = blk.size();
  size_t i = 0;
  EnhTail& t = h->t;
  t.F = F;
  t.E = E;
  for (int l = 0; l < 3; ++l) t.n[l] = h->n[l];
  t.ln_w = h->tail + off[i++];
  t.ln_b = h->tail + off[i++];
  for (int l = 0; l < 3; ++l) {
    t.centers[l] = h->tail + off[i++];
    t.t3w[l] = h->tail + off[i++];
    t.t3b[l] = h->tail + off[i++];
    t.f0t[l] = h->tail + off[i++];
    t.f0b[l] = h->tail + off[i++];
    t.f2t[l] = h->tail + off[i++];
    t.f2b[l] = h->tail + off[i++];
    t.rhw[l] = h->tail + off[i++];
    t.rhb[l] = h->tail + off[i++];
  }
  t.e0t = h->tail + off[i++];
  t.e0b = h->tail + off[i++];
  t.e2t = h->tail + off[i++];
  t.e2b = h->tail + off[i++];
  const float T = w->temperature;
  t.tau_geo = 2.0f * (T * T) + 1e-8f;
  t.tau_soft = T > 0.1f ? T : 0.1f;
  h->temperature = T;
  // input_proj: fp32 copies for EXACT, bf16 copies for the tensor cores
  const size_t n0 = (size_t)512 * H, n2 = (size_t)256 * 512;
  SB_CUDA_TRY(cudaMalloc(&h->w0_f32, n0 * 4));
  SB_CUDA_TRY(cudaMalloc(&h->w2_f32, n2 * 4));
  SB_CUDA_TRY(cudaMalloc(&h->w0_bf16, n0 * 2));
  SB_CUDA_TRY(cudaMalloc(&h->w2_bf16, n2 * 2));
  SB_CUDA_TRY(cudaMalloc(&h->b0, 512 * 4));
  SB_CUDA_TRY(cudaMalloc(&h->b2, 256 * 4));
  int rc;
  if ((rc = upload_f32(h->w0_f32, w->in0_w, n0, 0.f)) || (rc = upload_f32(h->w2_f32, w->in2_w, n2, 0.f)) ||
      (rc = upload_f32(h->b0, w->in0_b, 512, 0.f)) || (rc = upload_f32(h->b2, w->in2_b, 256, 0.f))) {
    enh_free(h);
    return rc;
  }
  enh_f32_to_bf16_kernel<<<512, 256>>>(h->w0_f32, h->w0_bf16, (int64_t)n0);
  enh_f32_to_bf16_kernel<<<256, 256>>>(h->w2_f32, h->w2_bf16, (int64_t)n2);
  SB_CUDA_TRY(cudaGetLastError());
  SB_CUDA_TRY(cudaDeviceSynchronize());
  if ((rc = make_tmap_2d(&h->tm_w0, h->w0_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 512, H, H, GEMM_BK, 256,
                         CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&h->tm_w2, h->w2_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 256, 512, 512, GEMM_BK, 256,
                         CU_TENSOR_MAP_SWIZZLE_128B))) {
    enh_free(h);
    return rc;
  }
  if ((rc = enh_build_tc(h, w))) {
    enh_free(h);
    return rc;
  }
  h->uploaded = true;
  return SB_OK;
}

extern "C" size_t sb_enh_workspace_bytes(const sb_enh* h, int64_t batch, int precision) {
  if (!h || batch < 0) return 0;
  return sb::enh_ws(h, batch, precision).total;
}

namespace sb {
namespace {

int enh_forward(sb_enh* h, const void* x, int x_dtype, int64_t batch, int precision, int gate_mode, int n_cand,
                int norm_topk_prob, int round_dtype, int top_k, const sb_enh_outputs* out, void* workspace,
                size_t workspace_bytes, void* stream_) {
  SB_REQUIRE(h && out, "sb_enh_forward: null argument");
  SB_REQUIRE(h->uploaded, "sb_enh_forward: weights were not uploaded");
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  SB_REQUIRE(x_dtype == SB_F32 || x_dtype == SB_BF16, "x dtype %d must be SB_F32 or SB_BF16", x_dtype);
  SB_REQUIRE(precision == SB_PREC_FAST || precision == SB_PREC_EXACT, "unknown precision %d", precision);
  SB_REQUIRE(precision != SB_PREC_FAST || x_dtype == SB_BF16,
             "FAST precision needs bf16 input (use EXACT for fp32 input)");
  SB_REQUIRE(gate_mode == SB_GATE_SOFTMAX || gate_mode == SB_GATE_TOPK_SOFTMAX || gate_mode == SB_GATE_HYBRID,
             "unknown gate mode %d", gate_mode);
  if (gate_mode == SB_GATE_HYBRID) {
    SB_REQUIRE(h->wg_f32 != nullptr, "the hybrid gate needs the dense gate weight (sb_enh_set_dense_gate)");
    SB_REQUIRE(out->topk_ids, "the hybrid gate needs topk_ids");
    SB_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= h->E, "top_k=%d must be in [1, min(32, %d)]", top_k, h->E);
    SB_REQUIRE(n_cand >= top_k && n_cand <= h->E, "n_candidates=%d must be in [top_k=%d, %d]", n_cand, top_k,
               h->E);
  }
  SB_REQUIRE(round_dtype == SB_F32 || round_dtype == SB_BF16, "round dtype %d must be SB_F32 or SB_BF16",
             round_dtype);
  if (out->topk_ids || out->topk_weights || out->router_probs) {
    SB_REQUIRE(out->topk_ids, "the gate outputs need topk_ids");
    SB_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= h->E, "top_k=%d must be in [1, min(32, %d)]", top_k, h->E);
  }
  if (batch == 0) return SB_OK;
  SB_REQUIRE(x != nullptr, "x is null");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0, "x must be 16-byte aligned");
  SB_REQUIRE(batch <= (int64_t)INT32_MAX / 2, "batch=%lld too large", (long long)batch);
  const EnhWs W = enh_ws(h, batch, precision);
  if (!workspace || workspace_bytes < W.total)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, W.total);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  DeviceGuard g(h->device);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* G = ws + W.g;
  float* P = reinterpret_cast<float*>(ws + W.p);
  float* D = reinterpret_cast<float*>(ws + W.d);
  const int H = h->H, M = (int)batch, E = h->E;
  const bool hybrid = gate_mode == SB_GATE_HYBRID;
  const bool use_tc = precision == SB_PREC_FAST && h->tc_ok && enh_tc_enabled();
  int rc;
  if (precision == SB_PREC_FAST) {
    CUtensorMap ta, tg;
    if ((rc = make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, H, H, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = make_tmap_2d(&tg, G, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, 512, 512, GEMM_BK, GEMM_BM,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    EpiGeluBf16 e0{h->b0, static_cast<__nv_bfloat16*>(G), 512, 512, nullptr, nullptr};
    if ((rc = launch_gemm_tc<256, 4, EpiGeluBf16, false>("enh_proj0_gelu_tc", ta, h->tm_w0, h->tm_w0, M, 512, H,
                                                          e0, stream)))
      return rc;
    if (use_tc) {  // input_proj.2 + LayerNorm -> X bf16 (the tensor-core tail's input)
      EpiLayerNormBf16 e2{h->b2, h->t.ln_w, h->t.ln_b, reinterpret_cast<__nv_bfloat16*>(P)};
      if ((rc = launch_gemm_tc<256, 4, EpiLayerNormBf16, false>("enh_proj2_ln_tc", tg, h->tm_w2, h->tm_w2, M, 256,
                                                                512, e2, stream)))
        return rc;
    } else {
      EpiBiasF32 e2{h->b2, P, 256, 256};
      if ((rc = launch_gemm_tc<256, 4, EpiBiasF32, false>("enh_proj2_tc", tg, h->tm_w2, h->tm_w2, M, 256, 512, e2,
                                                           stream)))
        return rc;
    }
    if (hybrid) {  // full_logits = x W_gate^T (fp32 accumulate; rounded to the hidden dtype in the tail)
      EpiBiasF32 ed{h->zero_e, D, E, E};
      if ((rc = launch_gemm_tc<64, 4, EpiBiasF32, false>("enh_dense_gate_tc", ta, h->tm_wg, h->tm_wg, M, E, H, ed,
                                                          stream)))
        return rc;
    }
  } else {
    float* G32 = static_cast<float*>(G);
    {
      ProfScope prof("enh_proj0_gelu_f32", stream);
      const dim3 grid(512 / 128, (M + 127) / 128);
      if (x_dtype == SB_BF16)
        sgemm_nt_kernel<__nv_bfloat16, ACT_GELU><<<grid, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), h->w0_f32, h->b0, G32, M, 512, H, 512, 0);
      else
        sgemm_nt_kernel<float, ACT_GELU><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), h->w0_f32, h->b0,
                                                                   G32, M, 512, H, 512, 0);
      SB_CUDA_TRY(cudaGetLastError());
    }
    {
      ProfScope prof("enh_proj2_f32", stream);
      const dim3 grid(256 / 128, (M + 127) / 128);
      sgemm_nt_kernel<float, ACT_NONE><<<grid, 256, 0, stream>>>(G32, h->w2_f32, h->b2, P, M, 256, 512, 256, 0);
      SB_CUDA_TRY(cudaGetLastError());
    }
    if (hybrid) {
      ProfScope prof("enh_dense_gate_f32", stream);
      const dim3 grid((E + 127) / 128, (M + 127) / 128);
      if (x_dtype == SB_BF16)
        sgemm_nt_kernel<__nv_bfloat16, ACT_NONE><<<grid, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), h->wg_f32, h->zero_e, D, M, E, H, E, 0);
      else
        sgemm_nt_kernel<float, ACT_NONE><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), h->wg_f32,
                                                                   h->zero_e, D, M, E, H, E, 0);
      SB_CUDA_TRY(cudaGetLastError());
    }
  }
  EnhOut o{out->logits, out->expert_probs, out->expert_ids, out->geo_dist, out->branch_bonus,
           out->router_probs, out->topk_weights, out->topk_ids, top_k, gate_mode, norm_topk_prob ? 1 : 0,
           round_dtype == SB_BF16 ? 1 : 0, hybrid ? D : nullptr, n_cand};
  if (use_tc) {
    CUtensorMap tmx;
    if ((rc = make_tmap_2d(&tmx, P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, 256, 256, 64, ETC_TOK,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    static PerDevice attr_tc;
    if ((rc = attr_tc.once(h->device, []() -> int {
           SB_CUDA_TRY(cudaFuncSetAttribute(enh_tail_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            ETC_SMEM_BYTES));
           SB_CUDA_TRY(cudaFuncSetAttribute(enh_tail_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            ETC_SMEM_BYTES));
           return SB_OK;
         })))
      return rc;
    ProfScope prof("enh_tail_tc", stream);
    int64_t blocks = (batch + ETC_TOK - 1) / ETC_TOK;
    if (blocks > num_sms()) blocks = num_sms();
    if (h->E <= 32)
      enh_tail_tc_kernel<32><<<(unsigned)blocks, ETC_THREADS, ETC_SMEM_BYTES, stream>>>(tmx, batch, h->t, o, h->tc);
    else
      enh_tail_tc_kernel<64><<<(unsigned)blocks, ETC_THREADS, ETC_SMEM_BYTES, stream>>>(tmx, batch, h->t, o, h->tc);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
  }
  {
    static PerDevice attr;
    if ((rc = attr.once(h->device, []() -> int {
           SB_CUDA_TRY(cudaFuncSetAttribute(enh_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            ENH_SMEM_BYTES));
           return SB_OK;
         })))
      return rc;
    ProfScope prof("enh_tail", stream);
    int64_t blocks = (batch + ENH_TOK - 1) / ENH_TOK;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    enh_tail_kernel<<<(unsigned)blocks, ENH_THREADS, ENH_SMEM_BYTES, stream>>>(P, batch, h->t, o);
    SB_CUDA_TRY(cudaGetLastError());
  }
  return SB_OK;
}

}  // namespace
}  // namespace sb

extern "C" int sb_enh_forward(sb_enh* h, const void* x, int x_dtype, int64_t batch, int precision, int gate_mode,
                              int norm_topk_prob, int round_dtype, int top_k, const sb_enh_outputs* out,
                              void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sb;
  SB_REQUIRE(gate_mode != SB_GATE_HYBRID, "the hybrid gate runs through sb_enh_forward_hybrid");
  return enh_forward(h, x, x_dtype, batch, precision, gate_mode, 0, norm_topk_prob, round_dtype, top_k, out,
                     workspace, workspace_bytes, stream);
}

extern "C" int sb_enh_forward_hybrid(sb_enh* h, const void* x, int x_dtype, int64_t batch, int precision,
                                     int n_candidates, int norm_topk_prob, int round_dtype, int top_k,
                                     const sb_enh_outputs* out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  return sb::enh_forward(h, x, x_dtype, batch, precision, SB_GATE_HYBRID, n_candidates, norm_topk_prob, round_dtype,
                         top_k, out, workspace, workspace_bytes, stream);
}

extern "C" int sb_enh_set_dense_gate(sb_enh* h, const void* w_gate, int w_dtype, int rows, int cols) {
  using namespace sb;
  SB_REQUIRE(h && w_gate, "sb_enh_set_dense_gate: null argument");
  SB_REQUIRE(w_dtype == SB_F32 || w_dtype == SB_BF16, "gate dtype %d must be SB_F32 or SB_BF16", w_dtype);
  SB_REQUIRE(rows == h->E && cols == h->H, "gate weight [%d,%d] must be [n_experts=%d, hidden=%d]", rows, cols,
             h->E, h->H);
  DeviceGuard g(h->device);
  enh_free_gate(h);
  const size_t n = (size_t)rows * cols, el = w_dtype == SB_BF16 ? 2 : 4;
  void* staging = nullptr;
  SB_CUDA_TRY(cudaMalloc(&staging, n * el));
  int rc = SB_OK;
  if (cudaMemcpy(staging, w_gate, n * el, cudaMemcpyDefault) != cudaSuccess ||
      cudaMalloc(&h->wg_f32, n * 4) != cudaSuccess || cudaMalloc(&h->wg_bf16, n * 2) != cudaSuccess ||
      cudaMalloc(&h->zero_e, (size_t)rows * 4) != cudaSuccess ||
      cudaMemset(h->zero_e, 0, (size_t)rows * 4) != cudaSuccess) {
    rc = fail(SB_ERR_CUDA, "dense gate upload: %s", cudaGetErrorString(cudaGetLastError()));
  } else {
    enh_gate_convert_kernel<<<256, 256>>>(staging, w_dtype == SB_BF16, h->wg_f32, h->wg_bf16, (int64_t)n);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      rc = fail(SB_ERR_CUDA, "dense gate conversion failed");
  }
  cudaFree(staging);
  if (!rc)
    rc = make_tmap_2d(&h->tm_wg, h->wg_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, cols, GEMM_BK, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) enh_free_gate(h);
  return rc;
}

extern "C" int sb_enh_destroy(sb_enh* h) {
  if (!h) return SB_OK;
  {
    sb::DeviceGuard g(h->device);
    sb::enh_free(h);
    sb::enh_free_gate(h);
  }
  delete h;
  return SB_OK;
}
