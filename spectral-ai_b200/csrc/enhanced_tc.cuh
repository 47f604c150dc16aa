// enhanced_tc.cuh — the EnhancedBVHRouter tail on tcgen05 tensor cores (FAST engine).
//
// Same computation as enh_tail_kernel (enhanced.cu), reorganised for sm_100a:
// a CTA of 128 threads owns a tile of 128 tokens (one TMEM lane and one thread
// per token).  The dense layers run as M=128 bf16 MMAs with fp32 accumulators
// in TMEM; the narrow layers that read the same input ride along as extra
// rows of the wide layer's weight matrix (columns 128.. of its accumulator):
//   MMA 0  level-1 feature_net.0 | level-1 to_3d            X      -> 128 GELU | 3
//   MMA 1  level-1 feature_net.2                            Z      -> 128      (f1)
//   MMA 2  level-2 feature_net.0 | level-1 route head (f part) | level-2 to_3d
//                                                           f1     -> 128 GELU | n1 | 3
//   MMA 3  level-2 feature_net.2                            Z      -> 128      (f2)
//   MMA 4  level-3 feature_net.0 | level-2 route head | level-3 to_3d
//   MMA 5  level-3 feature_net.2                            Z      -> 128      (f3)
//   MMA 6  level-3 route head (f part)                      f3     -> n3
//   MMA 7  expert_head.0   [f3 | p1 | p2 | p3] (K 140 -> 192) -> 256 GELU
//   MMA 8  expert_head.2   [256]                            -> E (<= 64) logits
// Activations are bf16 in shared memory in the 128-byte-swizzled K-major
// layout the MMA reads; a layer's input is dead once its MMA completes, so
// each epilogue writes its output over it (two buffers: XA 64 KB, FA 48 KB).
// Weights stream per layer by TMA into one 96 KB buffer; the next layer's
// load is issued as soon as the current MMA completes and overlaps the
// epilogue.  On the CUDA cores, in fp32 and thread per token: LayerNorm, the
// route heads' position terms, the geometry, softmaxes, argmaxes, leaf
// distances, branch bonus and the gate.
#pragma once

#include "sm100.cuh"

namespace sb {

constexpr int ETC_TOK = 128;
constexpr int ETC_THREADS = 256;  // two warps per 32 tokens: each takes half the columns
constexpr int ETC_F = 128;         // feature_dim served by this engine
constexpr int ETC_MAXN = 8;        // children per level
constexpr int ETC_MAXE = 64;       // experts
constexpr int ETC_LAYERS = 9;
constexpr int ETC_ATOM = ETC_TOK * 128;      // 16 KB: 128 rows x 64 bf16
constexpr int ETC_XA_BYTES = 4 * ETC_ATOM;   // K up to 256
constexpr int ETC_FA_BYTES = 3 * ETC_ATOM;   // K up to 192
constexpr int ETC_WB_BYTES = 96 * 1024;      // N x K bf16 of the largest layer (256 x 192)
constexpr int ETC_SMEM_BYTES = ETC_XA_BYTES + ETC_FA_BYTES + ETC_WB_BYTES + 64 + 1024;
static_assert(ETC_SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct EnhTC {
  CUtensorMap tm[ETC_LAYERS];  // bf16 [N][Kp] weights, box {64, N}
  int N[ETC_LAYERS];           // MMA N (rows of the weight matrix, multiple of 16)
  int Kp[ETC_LAYERS];          // K padded to 64
  const float* bias[ETC_LAYERS];
};

__device__ __forceinline__ float etc_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Writes 8 fp32 values as bf16 to columns [c0, c0+8) of row r of a K-major
// SW128 activation buffer (c0 a multiple of 8).
__device__ __forceinline__ void etc_store8(uint8_t* buf, int r, int c0, const float* v) {
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]), h3 = __floats2bfloat162_rn(v[6], v[7]);
  uint4 u;
  u.x = *reinterpret_cast<uint32_t*>(&h0);
  u.y = *reinterpret_cast<uint32_t*>(&h1);
  u.z = *reinterpret_cast<uint32_t*>(&h2);
  u.w = *reinterpret_cast<uint32_t*>(&h3);
  uint8_t* atom = buf + (c0 >> 6) * ETC_ATOM;
  *reinterpret_cast<uint4*>(atom + sw128_offset((uint32_t)r, (uint32_t)((c0 & 63) >> 3))) = u;
}

// One bf16 at column c of row r of a K-major SW128 activation buffer.
__device__ __forceinline__ void etc_store1(uint8_t* buf, int r, int c, float v) {
  uint8_t* atom = buf + (c >> 6) * ETC_ATOM;
  *reinterpret_cast<__nv_bfloat16*>(atom + sw128_offset((uint32_t)r, (uint32_t)((c & 63) >> 3)) + (c & 7) * 2) =
      __float2bfloat16_rn(v);
}

// Bounded wait by every thread of the CTA; false when it gave up (status set).
__device__ __forceinline__ bool etc_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait(bar, parity, ST_TIMEOUT_EPILOGUE);
}

// One layer's MMAs (thread 0): D[128 x N] = A[128 x Kp] W[N x Kp]^T.
__device__ __forceinline__ void etc_mma(uint32_t d_tmem, const uint8_t* a, const uint8_t* w, int N, int Kp) {
  const uint32_t idesc = idesc_f16(1, ETC_TOK, (uint32_t)N);
  const uint32_t w_atom = (uint32_t)(N * 128);
  for (int kb = 0; kb < Kp / 64; ++kb) {
    const uint64_t ad = sdesc_sw128(smem_u32(a + kb * ETC_ATOM));
    const uint64_t bd = sdesc_sw128(smem_u32(w + kb * w_atom));
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_f16(d_tmem, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0);
  }
}

// One token's E values to a row-major [B, E] output: float4 stores when every
// row starts on a 16-byte boundary (E a multiple of 4, aligned base), scalar
// stores otherwise.
template <int EP>
__device__ __forceinline__ void etc_store_row(float* out, int64_t tok, int E, const float (&v)[EP]) {
  float* row = out + tok * E;
  if ((E & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
#pragma unroll
    for (int e = 0; e < EP; e += 4)
      if (e < E) *reinterpret_cast<float4*>(row + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
  } else {
#pragma unroll
    for (int e = 0; e < EP; ++e)
      if (e < E) row[e] = v[e];
  }
}

// The per-token outputs after the expert head (thread = token): logits,
// expert_probs / expert_ids, leaf distances, branch bonus and the gate.
// sd: this tile's leaf distances in shared memory, [3 * ETC_MAXN][ETC_TOK].
template <int EP>
__device__ __forceinline__ void etc_outputs(float (&lg)[EP], int64_t tok, int tid, const EnhTail& t, const EnhOut& o,
                                            const float* sd, const int (&amx)[3]) {
  const int E = t.E, n2 = t.n[1], n3 = t.n[2];
  if (o.logits) etc_store_row<EP>(o.logits, tok, E, lg);
  // expert_probs = softmax(logits / max(T, 0.1)); ids = first argmax (only
  // when an output or the hybrid gate's candidate ranking reads them).  v
  // holds them, then the gate's values (two arrays of EP live, not three).
  float v[EP];
  const bool hybrid = o.topi && o.mode == SB_GATE_HYBRID;
  unsigned long long cand = ~0ull;  // experts the top-k may choose from
  if (o.probs || o.ids || hybrid) {
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < EP; ++e)
      if (e < E) m = fmaxf(m, lg[e] / t.tau_soft);
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      v[e] = e < E ? expf(lg[e] / t.tau_soft - m) : 0.f;
      sum += v[e];
    }
    float bv = -INFINITY;
    int bi = 0;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      v[e] = v[e] / sum;
      if (e < E && v[e] > bv) {
        bv = v[e];
        bi = e;
      }
    }
    if (o.probs) etc_store_row<EP>(o.probs, tok, E, v);
    if (o.ids) o.ids[tok] = bi;
    if (hybrid) {
      // BVH candidates: the n_cand first experts in the order (expert_probs
      // descending, index ascending) — by n_cand passes adding the largest
      // remaining, or, when fewer passes, by removing the smallest remaining
      // (the last in that order: the higher index among equal values)
      const unsigned long long all = E < 64 ? (1ull << E) - 1ull : ~0ull;
      if (2 * o.n_cand <= E) {
        cand = 0ull;
        for (int r = 0; r < o.n_cand; ++r) {
          float best = -INFINITY;
          int b = -1;
#pragma unroll
          for (int e = 0; e < EP; ++e)
            if (((all & ~cand) >> e) & 1ull)
              if (b < 0 || v[e] > best) {
                best = v[e];
                b = e;
              }
          cand |= 1ull << b;
        }
      } else {
        cand = all;
        for (int r = 0; r < E - o.n_cand; ++r) {
          float worst = INFINITY;
          int b = -1;
#pragma unroll
          for (int e = 0; e < EP; ++e)
            if ((cand >> e) & 1ull)
              if (b < 0 || v[e] <= worst) {
                worst = v[e];
                b = e;
              }
          cand &= ~(1ull << b);
        }
      }
    }
  }
  if (o.geo || o.bonus) {
    for (int e = 0; e < E; ++e) {
      const int i = e / (n2 * n3), j = (e % (n2 * n3)) / n3, k = e % n3;
      if (o.geo)
        o.geo[tok * E + e] = (sd[i * ETC_TOK + tid] + sd[(ETC_MAXN + j) * ETC_TOK + tid]) +
                             sd[(2 * ETC_MAXN + k) * ETC_TOK + tid];
      if (o.bonus) o.bonus[tok * E + e] = (1.0f + 0.2f * (float)(i == amx[0])) + 0.1f * (float)(j == amx[1]);
    }
  }
  if (!o.topi) return;
  const int K = o.k;
  if (hybrid) {
    float m2 = -INFINITY;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      v[e] = e < E ? (o.round_bf16 ? etc_bf(o.dense[tok * E + e]) : o.dense[tok * E + e]) : -INFINITY;
      m2 = fmaxf(m2, v[e]);
    }
    float s2 = 0.f;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      v[e] = e < E ? expf(v[e] - m2) : 0.f;
      s2 += v[e];
    }
#pragma unroll
    for (int e = 0; e < EP; ++e) v[e] = v[e] / s2;
    if (o.rprobs) etc_store_row<EP>(o.rprobs, tok, E, v);
  } else {
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      v[e] = e < E ? (o.round_bf16 ? etc_bf(lg[e]) : lg[e]) : -INFINITY;
      mx = fmaxf(mx, v[e]);
    }
    if (o.mode == SB_GATE_SOFTMAX) {
      float s2 = 0.f;
#pragma unroll
      for (int e = 0; e < EP; ++e) {
        v[e] = e < E ? expf(v[e] - mx) : 0.f;
        s2 += v[e];
      }
#pragma unroll
      for (int e = 0; e < EP; ++e) v[e] = v[e] / s2;
      if (o.rprobs) etc_store_row<EP>(o.rprobs, tok, E, v);
    } else if (o.rprobs) {
      for (int e = 0; e < E; ++e) o.rprobs[tok * E + e] = 0.f;
    }
  }
  if (E < 64) cand &= (1ull << E) - 1ull;
  // top-k by k passes, larger first, lower index first among equal values
  float sel_v[32];
  int sel_i[32];
  unsigned long long taken = 0ull;
  float tot = 0.f;
  for (int r = 0; r < K; ++r) {
    float best = -INFINITY;
    int b = -1;
#pragma unroll
    for (int e = 0; e < EP; ++e) {
      const bool ok = ((cand & ~taken) >> e) & 1ull;
      if (ok && (b < 0 || v[e] > best)) {
        best = v[e];
        b = e;
      }
    }
    taken |= 1ull << b;
    sel_v[r & 31] = best;
    sel_i[r & 31] = b;
    tot += best;
  }
  float wmax = -INFINITY, esum = 0.f;
  if (o.mode == SB_GATE_TOPK_SOFTMAX) {
    for (int r = 0; r < K; ++r) wmax = fmaxf(wmax, sel_v[r]);
    for (int r = 0; r < K; ++r) esum += expf(sel_v[r] - wmax);
  }
  for (int r = 0; r < K; ++r) {
    float w = sel_v[r];
    if (o.mode == SB_GATE_TOPK_SOFTMAX) w = expf(sel_v[r] - wmax) / esum;
    else if (o.norm) w = sel_v[r] / tot;
    o.topi[tok * K + r] = sel_i[r];
    if (o.topw) o.topw[tok * K + r] = w;
    if (o.mode == SB_GATE_TOPK_SOFTMAX && o.rprobs) o.rprobs[tok * E + sel_i[r]] = w;
  }
}

// Route of level LV (thread = token): logits = rh + W_pos . pos + b + 0.5 *
// geometric logit, softmax(logits / max(T, 0.1)), first argmax, leaf
// distances; the probabilities go to the expert-head input columns of FA.
// rh: the route head's feature part, computed by the tensor cores.
template <int LV>
__device__ __forceinline__ void etc_route(const uint32_t (&rh)[32], int rh0, uint8_t* FA, int tid, const EnhTail& t,
                                          const float (&pos)[3], float* sd, int (&amx)[3]) {
  constexpr int F = ETC_F;
  const int K = t.n[LV];
  const float* rhw = t.rhw[LV];
  float lg[ETC_MAXN];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < ETC_MAXN; ++k) {
    lg[k] = -INFINITY;
    if (k >= K) continue;
    float v = __uint_as_float(rh[rh0 + k]);
    v = fmaf(pos[0], __ldg(rhw + k * (F + 3) + F), v);
    v = fmaf(pos[1], __ldg(rhw + k * (F + 3) + F + 1), v);
    v = fmaf(pos[2], __ldg(rhw + k * (F + 3) + F + 2), v);
    v += __ldg(t.rhb[LV] + k);
    const float* cc = t.centers[LV] + 3 * k;
    const float dx = pos[0] - __ldg(cc), dy = pos[1] - __ldg(cc + 1), dz = pos[2] - __ldg(cc + 2);
    const float d2 = (dx * dx + dy * dy) + dz * dz;
    lg[k] = (v + 0.5f * (-d2 / t.tau_geo)) / t.tau_soft;
    sd[(LV * ETC_MAXN + k) * ETC_TOK + tid] = sqrtf(d2 + 1e-8f);
    m = fmaxf(m, lg[k]);
  }
  float pr[ETC_MAXN];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < ETC_MAXN; ++k) {
    pr[k] = k < K ? expf(lg[k] - m) : 0.f;
    sum += pr[k];
  }
  float bv = -INFINITY;
  int bi = 0;
  const int off = F + (LV > 0 ? t.n[0] : 0) + (LV > 1 ? t.n[1] : 0);
#pragma unroll
  for (int k = 0; k < ETC_MAXN; ++k) {
    if (k >= K) continue;
    pr[k] = pr[k] / sum;
    if (pr[k] > bv) {
      bv = pr[k];
      bi = k;
    }
    etc_store1(FA, tid, off + k, pr[k]);
  }
  amx[LV] = bi;
}

__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// act(acc + b) over columns [c0, c1) of this warp's 32 rows into an activation
// buffer, 8 columns per step (a short loop the whole CTA reuses).
// GELU in its tanh form (Hendrycks & Gimpel, 2016) on the hardware tanh: it
// departs from the erf form by about 1e-3 at most, below the bf16 rounding the
// FAST engine applies to the same activation right after.
__device__ __forceinline__ float etc_gelu(float x) {
  const float u = 0.7978845608f * fmaf(0.044715f * x, x * x, x);
  float th;
  asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(u));
  return 0.5f * x * (1.f + th);
}

template <bool GELU>
__device__ __noinline__ void etc_act_epilogue(uint32_t tl, uint8_t* dst, int row, const float* __restrict__ b, int c0,
                                              int c1) {
#pragma unroll 1
  for (int c = c0; c < c1; c += 8) {
    uint32_t r[8];
    tmem_ld_32x32b_x8(tl + (uint32_t)c, r);
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(b + c)), b1 = __ldg(reinterpret_cast<const float4*>(b + c + 4));
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    tmem_ld_wait();
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = __uint_as_float(r[j]) + bb[j];
      v[j] = GELU ? etc_gelu(a) : a;
    }
    etc_store8(dst, row, c, v);
  }
}

template <int EP>
__global__ void __launch_bounds__(ETC_THREADS, 1)
    enh_tail_tc_kernel(const __grid_constant__ CUtensorMap tmx, int64_t B, const EnhTail t, const EnhOut o,
                       const __grid_constant__ EnhTC p) {
  extern __shared__ uint8_t etc_smem_raw[];
  const uint32_t raw = smem_u32(etc_smem_raw);
  uint8_t* XA = etc_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* FA = XA + ETC_XA_BYTES;
  uint8_t* WB = FA + ETC_FA_BYTES;
  uint64_t* wbar = reinterpret_cast<uint64_t*>(WB + ETC_WB_BYTES);
  uint64_t* mbar = wbar + 1;
  uint64_t* xbar = mbar + 1;  // the tile's LayerNorm output X arrived in XA
  uint32_t* tslot = reinterpret_cast<uint32_t*>(xbar + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tslot + 1);
  __shared__ float sd[3 * ETC_MAXN * ETC_TOK];  // leaf distances of this tile
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (ETC_TOK - 1);  // token of this thread (TMEM lane)
  const int half = tid >> 7;            // which half of each layer's columns

  if (tid == 0) {
    mbar_init(wbar, 1);
    mbar_init(mbar, 1);
    mbar_init(xbar, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const int64_t tile_stride = (int64_t)gridDim.x * ETC_TOK;
  uint32_t wcount = 0, mcount = 0, xcount = 0;  // completed weight loads / MMA batches / X tiles
  bool w_pending = false, x_pending = false;     // thread 0: a load is in flight

  auto load_w = [&](int l) {
    const int N = p.N[l], Kp = p.Kp[l];
    mbar_arrive_expect_tx(wbar, (uint32_t)(Kp / 64) * (uint32_t)N * 128u);
    for (int kb = 0; kb < Kp / 64; ++kb) tma_load_2d(WB + kb * N * 128, &p.tm[l], wbar, kb * 64, 0);
    w_pending = true;
  };
  // X rows t0 .. t0+127 (bf16, 4 boxes of 64 columns) into XA; rows past the
  // batch arrive as zeros
  auto load_x = [&](int64_t t0) {
    mbar_arrive_expect_tx(xbar, 4u * ETC_ATOM);
    for (int kb = 0; kb < 4; ++kb) tma_load_2d(XA + kb * ETC_ATOM, &tmx, xbar, kb * 64, (int32_t)t0);
    x_pending = true;
  };
  if (tid == 0 && (int64_t)blockIdx.x * ETC_TOK < B) {
    for (int l = 0; l < ETC_LAYERS; ++l) tma_prefetch_desc(&p.tm[l]);
    tma_prefetch_desc(&tmx);
    load_x((int64_t)blockIdx.x * ETC_TOK);
    load_w(0);
  }

  for (int64_t t0 = (int64_t)blockIdx.x * ETC_TOK; t0 < B; t0 += tile_stride) {
    const int64_t tok = t0 + row;
    const bool live = tok < B;
    const bool last_tile = t0 + tile_stride >= B;
    float pos[3] = {0.f, 0.f, 0.f};
    {
      // expert-head input columns F .. 191 start at zero; each level writes its
      // probabilities there ([p1 | p2 | p3 | 0...], read only by MMA 7)
      const float z8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int g = 0; g < 4; ++g) etc_store8(FA, row, ETC_F + (half * 4 + g) * 8, z8);
    }
    int amx[3] = {0, 0, 0};
    float lg[EP];
#pragma unroll
    for (int l = 0; l < ETC_LAYERS; ++l) {
      // this layer's input (written above by every thread) -> the MMA's async proxy
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (*s_abort) break;
      if (tid == 0) {
        bool ok = etc_wait(wbar, wcount & 1u);
        ++wcount;
        if (ok) w_pending = false;
        if (ok && l == 0) {
          ok = etc_wait(xbar, xcount & 1u);
          ++xcount;
          if (ok) x_pending = false;
        }
        if (!ok) {
          *s_abort = 1;
        } else {
          tc_fence_after();
          etc_mma(tmem, (l == 0 || l == 8) ? XA : FA, WB, p.N[l], p.Kp[l]);
          umma_commit(mbar);
        }
      }
      __syncthreads();
      if (*s_abort) break;
      if (!etc_wait(mbar, mcount & 1u)) *s_abort = 1;
      ++mcount;
      tc_fence_after();
      // the MMA that read WB is complete: fetch the next layer's weights
      if (tid == 0 && !*s_abort && !(last_tile && l == ETC_LAYERS - 1)) load_w((l + 1) % ETC_LAYERS);
      // MMA 8 has read XA: the next tile's X may land there now
      if (tid == 0 && !*s_abort && !last_tile && l == ETC_LAYERS - 1) load_x(t0 + tile_stride);
      if (l == 0 || l == 2 || l == 4) {
        // feature_net.0 (GELU) and the rows riding along: [route head of the
        // previous level (n) | this level's to_3d (3)]
        etc_act_epilogue<true>(tl, FA, row, p.bias[l], half * 64, half * 64 + 64);
        if (half == 0) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tl + (uint32_t)ETC_F, r);
          tmem_ld_wait();
          const int lv = l / 2;  // the level this feature_net belongs to
          const int nprev = lv > 0 ? t.n[lv - 1] : 0;
          if (l == 2) etc_route<0>(r, 0, FA, row, t, pos, sd, amx);
          if (l == 4) etc_route<1>(r, 0, FA, row, t, pos, sd, amx);
#pragma unroll
          for (int d = 0; d < 3; ++d) {
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (q == nprev + d) v = __uint_as_float(r[q]);
            pos[d] = v + __ldg(t.t3b[lv] + d);
          }
        }
      } else if (l == 1 || l == 3 || l == 5) {
        etc_act_epilogue<false>(tl, FA, row, p.bias[l], half * 64, half * 64 + 64);
      } else if (l == 6) {
        if (half == 0) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tl, r);
          tmem_ld_wait();
          etc_route<2>(r, 0, FA, row, t, pos, sd, amx);
        }
      } else if (l == 7) {
        etc_act_epilogue<true>(tl, XA, row, p.bias[l], half * 128, half * 128 + 128);
      } else if (half == 0) {
        const int E = t.E;
#pragma unroll
        for (int c = 0; c < EP / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tl + (uint32_t)(c * 32), r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int e = c * 32 + j;
            lg[e] = e < E ? __uint_as_float(r[j]) + __ldg(p.bias[l] + e) : 0.f;
          }
        }
      }
      tc_fence_before();
    }
    if (*s_abort) break;
    if (live && half == 0) etc_outputs<EP>(lg, tok, row, t, o, sd, amx);
  }
  // unwind: no TMA may still write this CTA's shared memory, no MMA its TMEM
  __syncthreads();
  if (tid == 0 && w_pending) etc_wait(wbar, (wcount - (*s_abort ? 1u : 0u)) & 1u);
  if (tid == 0 && x_pending) etc_wait(xbar, (xcount - (*s_abort ? 1u : 0u)) & 1u);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace sb
