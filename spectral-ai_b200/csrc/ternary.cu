// ternary.cu — ternary {-1,0,+1} weights: reference-layout packer and the
// repack into the B200 device layout.
//
// Reference layout (cuda/v5/ternary_torch_ext.cu:197-231): int32 [ceil(K/16), N],
// 2-bit codes 00 = 0, 01 = +1, 10 = -1, bit pair i of word [p, c] holds
// row p*16+i (K index), column c (output channel).  Decode rule
// (ternary_torch_ext.cu:38-53): sign = (code == 1) - (code >> 1).
//
// Device layout: uint32 [N, KW] with KW = ceil(K/64)*4 words per output row
// (row n holds K contiguous, padded to a multiple of 64 with zeros).  Word w of
// row n covers K indices 16w .. 16w+15; element 16w+2j+e (e = 0,1; j = 0..7)
// is stored as the biased code value+1 in {0,1,2} at bits 16e+p_j .. 16e+p_j+1
// with p_j = tern_pos(j) = 0, 2, 4, 8, 10, 12, 6, 14 (padding holds code 1,
// value 0).  A pair (2j, 2j+1) becomes two packed 16-bit floats with one and-or
// and one packed subtraction: with E the exponent that makes bit p the
// mantissa's unit (bf16: p <= 4, fp16: p <= 8),
//   (w & (0x00030003 << p)) | E  is the pair  (b + code_2j, b + code_2j+1)
// for b = 2^(7-p) (bf16) or 2^(10-p) (fp16), and subtracting b + 1 leaves
// code - 1 = value exactly.  Pairs past the mantissa are first shifted down
// (by 8, shared by three pairs, or to bit 0): 19 instructions per word of 16
// weights in bf16 and 17 in fp16, against 24 with a shift for every pair.
#include "common.cuh"
#include "ternary_gemm.cuh"
#include "ternary_ts.cuh"
#include "ternary_pair.cuh"
#include "tree_sum.cuh"
#include "ternary_gemv.cuh"

#include <cstdlib>
#include <cstring>
#include <type_traits>

namespace sb {

__host__ __device__ __forceinline__ int ternary_code_to_sign(uint32_t code) {
  return (int)(code == 1u) - (int)(code >> 1);
}

__host__ __device__ __forceinline__ int64_t ternary_row_words(int64_t K) {
  return (K + 63) / 64 * 4;
}

// One thread per output word of the device layout.
__global__ void ternary_repack_kernel(const uint32_t* __restrict__ ref, int64_t K, int64_t N,
                                      uint32_t* __restrict__ dst) {
  const int64_t KW = ternary_row_words(K);
  const int64_t P = (K + 15) / 16;  // reference packed rows
  const int64_t total = N * KW;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / KW, w = i % KW;
    uint32_t out = 0x55555555u;  // every element code 1 (value 0)
    if (w < P) {
      const uint32_t codes = ref[w * N + n];  // 16 codes of K rows 16w..16w+15, column n
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int64_t k = w * 16 + t;
        if (k >= K) break;
        const int s = ternary_code_to_sign((codes >> (2 * t)) & 3u);
        const int e = t & 1, j = t >> 1;
        const int sh = 16 * e + tern_pos(j);
        out = (out & ~(3u << sh)) | ((uint32_t)(s + 1) << sh);
      }
    }
    dst[i] = out;
  }
}

}  // namespace sb

extern "C" int sb_ternary_pack_ref(const int8_t* w, int64_t K, int64_t N, int32_t* packed) {
  SB_REQUIRE(w && packed, "sb_ternary_pack_ref: null argument");
  SB_REQUIRE(K >= 0 && N >= 0, "negative shape");
  const int64_t P = (K + 15) / 16;
  for (int64_t p = 0; p < P; ++p)
    for (int64_t c = 0; c < N; ++c) {
      uint32_t word = 0;
      for (int i = 0; i < 16; ++i) {
        const int64_t r = p * 16 + i;
        if (r >= K) break;
        const int8_t v = w[r * N + c];
        const uint32_t code = v > 0 ? 1u : (v < 0 ? 2u : 0u);
        word |= code << (2 * i);
      }
      packed[p * N + c] = (int32_t)word;
    }
  return SB_OK;
}

extern "C" size_t sb_ternary_matrix_bytes(int64_t K, int64_t N) {
  if (K <= 0 || N <= 0) return 0;
  return (size_t)(N * sb::ternary_row_words(K) * 4);
}

extern "C" int sb_ternary_repack(const int32_t* packed_ref, int64_t K, int64_t N, uint32_t* dst,
                                 void* stream) {
  SB_REQUIRE(packed_ref && dst, "sb_ternary_repack: null argument");
  SB_REQUIRE(K > 0 && N > 0, "shape must be positive (K=%lld N=%lld)", (long long)K, (long long)N);
  const int64_t total = N * sb::ternary_row_words(K);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  sb::ternary_repack_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed_ref), K, N, dst);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

// ===========================================================================
// MoE dispatch / combine and the host entry points
// ===========================================================================
namespace sb {

// expert histogram of the (token, slot) pairs; out-of-range ids are reported
// through the status word and dropped
__global__ void moe_hist_kernel(const int32_t* __restrict__ ids, int64_t R, int E,
                                int* __restrict__ counts) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < R;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E)
      atomicAdd(&counts[e], 1);
    else
      set_status(ST_BAD_ARGUMENT);
  }
}

constexpr int PLAN_THREADS = 1024;

// Expert offsets (exclusive scan of the counts rounded up to 32), zeroed
// scatter cursors and the m-tile table, by one block of PLAN_THREADS threads;
// `count(e)` gives expert e's rows (with `write_counts` they are also stored).
// Expert segments start on 32-row boundaries (segment = count rounded up to
// 32); m-tiles of `tile_rows` rows cover them, `rows` valid and `pad` rows up
// to the segment end (a multiple of 32).
template <typename CountFn>
__device__ __forceinline__ void plan_segments(int E, CountFn count, bool write_counts, int* __restrict__ counts,
                                              int* __restrict__ offsets, int* __restrict__ cursor,
                                              MTile* __restrict__ mtiles, int* __restrict__ num_mtiles,
                                              int max_mtiles, int tile_rows) {
  __shared__ int warp_rows[32], warp_tiles[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // each thread owns a run of consecutive experts
  const int per = (E + PLAN_THREADS - 1) / PLAN_THREADS;
  const int e0 = tid * per < E ? tid * per : E, e1 = e0 + per < E ? e0 + per : E;
  int my_rows = 0, my_tiles = 0;
  for (int e = e0; e < e1; ++e) {
    const int cp = (count(e) + 31) & ~31;
    my_rows += cp;
    my_tiles += (cp + tile_rows - 1) / tile_rows;
  }
  // block-wide exclusive scan of (rows, tiles)
  int r_inc = my_rows, t_inc = my_tiles;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int rv = __shfl_up_sync(0xffffffffu, r_inc, o), tv = __shfl_up_sync(0xffffffffu, t_inc, o);
    if (lane >= o) {
      r_inc += rv;
      t_inc += tv;
    }
  }
  if (lane == 31) {
    warp_rows[warp] = r_inc;
    warp_tiles[warp] = t_inc;
  }
  __syncthreads();
  if (warp == 0) {
    int rw = warp_rows[lane], tw = warp_tiles[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int rv = __shfl_up_sync(0xffffffffu, rw, o), tv = __shfl_up_sync(0xffffffffu, tw, o);
      if (lane >= o) {
        rw += rv;
        tw += tv;
      }
    }
    warp_rows[lane] = rw;  // inclusive over warps
    warp_tiles[lane] = tw;
  }
  __syncthreads();
  int off = r_inc - my_rows + (warp > 0 ? warp_rows[warp - 1] : 0);
  int nt = t_inc - my_tiles + (warp > 0 ? warp_tiles[warp - 1] : 0);
  for (int e = e0; e < e1; ++e) {
    const int c = count(e);
    const int cp = (c + 31) & ~31;
    if (write_counts) counts[e] = c;
    offsets[e] = off;
    cursor[e] = 0;
    for (int r = 0; r < cp; r += tile_rows, ++nt) {
      if (nt >= max_mtiles) continue;
      MTile t;
      t.expert = e;
      t.row0 = off + r;
      t.rows = (c - r) < tile_rows ? (c - r) : tile_rows;
      t.pad = (cp - r) < tile_rows ? (cp - r) : tile_rows;
      mtiles[nt] = t;
    }
    off += cp;
  }
  if (tid == PLAN_THREADS - 1) *num_mtiles = nt < max_mtiles ? nt : max_mtiles;
}

// The plan of one batch in one block: with `hist` set the block also counts
// the ids itself (shared-memory histogram; small batches), otherwise it reads
// `counts` from moe_hist_kernel.
__global__ void __launch_bounds__(PLAN_THREADS) moe_plan_kernel(const int32_t* __restrict__ ids, int64_t R, int E,
                                                               int hist, int* __restrict__ counts,
                                                               int* __restrict__ offsets, int* __restrict__ cursor,
                                                               MTile* __restrict__ mtiles, int* __restrict__ num_mtiles,
                                                               int max_mtiles, int tile_rows) {
  extern __shared__ int sh_count[];  // [E] when hist
  const int tid = threadIdx.x;
  if (hist) {
    for (int e = tid; e < E; e += PLAN_THREADS) sh_count[e] = 0;
    __syncthreads();
    auto count = [&](int e) {
      if (e >= 0 && e < E)
        atomicAdd(&sh_count[e], 1);
      else
        set_status(ST_BAD_ARGUMENT);
    };
    int64_t i0 = 0;
    if ((reinterpret_cast<uintptr_t>(ids) & 15u) == 0) {
      // 16-byte words, eight a thread loaded before any is counted: one
      // memory round trip per 32 Ki ids instead of one per 1 Ki
      const int4* ids4 = reinterpret_cast<const int4*>(ids);
      const int64_t R4 = R >> 2;
      for (int64_t b = 0; b < R4; b += 8 * PLAN_THREADS) {
        int4 w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int64_t j = b + u * PLAN_THREADS + tid;
          if (j < R4) w[u] = __ldg(ids4 + j);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (b + u * PLAN_THREADS + tid < R4) {
            count(w[u].x);
            count(w[u].y);
            count(w[u].z);
            count(w[u].w);
          }
        }
      }
      i0 = R4 << 2;
    }
    for (int64_t i = i0 + tid; i < R; i += PLAN_THREADS) count(ids[i]);
    __syncthreads();
  }
  plan_segments(E, [&](int e) { return hist ? sh_count[e] : counts[e]; }, hist != 0, counts, offsets, cursor,
                mtiles, num_mtiles, max_mtiles, tile_rows);
}

// Histogram + plan for one batch: one fused block for small batches, else a
// grid-wide histogram first.
int moe_plan(const int32_t* ids, int64_t R, int E, int* counts, int* offsets, int* cursor, MTile* mtiles, int* nmt,
             int max_mt, int tile_rows, cudaStream_t stream) {
  const bool fused = R <= (int64_t)1 << 17 && E <= 8192;
  if (!fused) {
    SB_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int) * E, stream));
    int64_t blocks = (R + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    moe_hist_kernel<<<(unsigned)blocks, 256, 0, stream>>>(ids, R, E, counts);
  }
  moe_plan_kernel<<<1, PLAN_THREADS, fused ? sizeof(int) * E : 0, stream>>>(
      ids, R, E, fused ? 1 : 0, counts, offsets, cursor, mtiles, nmt, max_mt, tile_rows);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

template <typename TX, typename TA>
__device__ __forceinline__ TA cvt_act(TX v);
template <> __device__ __forceinline__ __nv_bfloat16 cvt_act<float, __nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half cvt_act<float, __half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_act<__nv_bfloat16, __nv_bfloat16>(__nv_bfloat16 v) { return v; }
template <> __device__ __forceinline__ __half cvt_act<__nv_bfloat16, __half>(__nv_bfloat16 v) { return __float2half_rn(__bfloat162float(v)); }

constexpr int SCATTER_REG_ROW = 8 * 32 * 8;  // bf16 row width held in a warp's registers

// One warp per (token, slot) pair: claim a row of the expert's segment, record
// the routing weight and the inverse map, and copy the token's activations.
// 16-byte vector row copies (bf16 -> bf16: 8 values per lane step; fp32 -> fp16: 4)
__device__ __forceinline__ void copy_row_vec(const __nv_bfloat16* src, __nv_bfloat16* dst, int H, int lane) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int c = lane; c < H / 8; c += 32) d4[c] = __ldg(s4 + c);
}
__device__ __forceinline__ void copy_row_vec(const float* src, __half* dst, int H, int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  uint2* d2 = reinterpret_cast<uint2*>(dst);
  for (int c = lane; c < H / 4; c += 32) {
    const float4 v = __ldg(s4 + c);
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    d2[c] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  }
}

template <typename TX, typename TA>
__global__ void moe_scatter_kernel(const TX* __restrict__ x, const int32_t* __restrict__ ids,
                                   const float* __restrict__ wts, int64_t B, int k, int H, int E,
                                   const int* __restrict__ offsets, int* __restrict__ cursor,
                                   TA* __restrict__ xp, int64_t ldx, float* __restrict__ row_w,
                                   int* __restrict__ inv, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t R = B * k;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < R;
       i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int e = ids[i];
    if constexpr (std::is_same<TX, __nv_bfloat16>::value && std::is_same<TA, __nv_bfloat16>::value) {
      if (vec && H <= SCATTER_REG_ROW) {
        // The whole row (up to 2048 bf16: eight 16-byte words a lane) is
        // loaded into registers before the slot is claimed, so its loads are
        // in flight during the claim's atomic round trip.
        const uint4* s4 = reinterpret_cast<const uint4*>(x + (i / k) * (int64_t)H);
        const int n = H >> 3;
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (lane + 32 * u < n) v[u] = __ldg(s4 + lane + 32 * u);
        int pos = -1;
        if (lane == 0 && e >= 0 && e < E) pos = offsets[e] + atomicAdd(&cursor[e], 1);
        pos = __shfl_sync(0xffffffffu, pos, 0);
        if (lane == 0) inv[i] = pos;
        if (pos < 0) continue;
        if (lane == 0) row_w[pos] = wts ? wts[i] : 1.0f;
        uint4* d4 = reinterpret_cast<uint4*>(xp + (int64_t)pos * ldx);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (lane + 32 * u < n) d4[lane + 32 * u] = v[u];
        continue;
      }
    }
    int pos = -1;
    if (lane == 0 && e >= 0 && e < E) pos = offsets[e] + atomicAdd(&cursor[e], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (lane == 0) inv[i] = pos;
    if (pos < 0) continue;
    if (lane == 0) row_w[pos] = wts ? wts[i] : 1.0f;
    const TX* src = x + (i / k) * (int64_t)H;
    TA* dst = xp + (int64_t)pos * ldx;
    if (vec) {
      copy_row_vec(src, dst, H, lane);
    } else {
      for (int c = lane; c < H; c += 32) dst[c] = cvt_act<TX, TA>(src[c]);
    }
  }
}

// The fp32-faithful dispatch: each fp32 row becomes two bf16 rows side by
// side, hi = bf16(x) in columns [0, H) and lo = bf16(x - hi) in [H, 2H), so that
// the GEMM over the doubled K sums T x_hi + T x_lo = T x to 2^-16 relative
// (bf16 keeps fp32's exponent range).  H % 4 == 0 and 16-byte aligned rows.
__global__ void moe_scatter_split_kernel(const float* __restrict__ x, const int32_t* __restrict__ ids,
                                         const float* __restrict__ wts, int64_t B, int k, int H, int E,
                                         const int* __restrict__ offsets, int* __restrict__ cursor,
                                         __nv_bfloat16* __restrict__ xp, int64_t ldx, float* __restrict__ row_w,
                                         int* __restrict__ inv) {
  const int lane = threadIdx.x & 31;
  const int64_t R = B * k;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < R;
       i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int e = ids[i];
    int pos = -1;
    if (lane == 0 && e >= 0 && e < E) pos = offsets[e] + atomicAdd(&cursor[e], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (lane == 0) inv[i] = pos;
    if (pos < 0) continue;
    if (lane == 0) row_w[pos] = wts ? wts[i] : 1.0f;
    const float4* s4 = reinterpret_cast<const float4*>(x + (i / k) * (int64_t)H);
    __nv_bfloat16* dst = xp + (int64_t)pos * ldx;
    for (int c = lane; c < H / 4; c += 32) {
      const float4 v = __ldg(s4 + c);
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
      const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
      const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
      *reinterpret_cast<uint2*>(dst + 4 * c) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
      *reinterpret_cast<uint2*>(dst + H + 4 * c) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
    }
  }
}

template <typename TO>
__device__ __forceinline__ TO cvt_out(float v);
template <> __device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename TO>
__device__ __forceinline__ void store4(TO* p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

// out[t] = the tree sum (tree_sum.cuh) of y[inv[t*k + j]] over the token's
// slots j whose expert is in range, the positions being the expert ids, so the
// single-GPU layer and the expert-parallel layer add the same values in the
// same grouping.  One warp per token: the warp ranks the token's entries, then
// each lane sums its columns (16-byte groups when H % 4 == 0) with the KC
// values of one column group in registers (KC >= k).
template <typename TO, int KC>
__global__ void moe_combine_kernel(const float* __restrict__ y, const int* __restrict__ inv,
                                   const int32_t* __restrict__ ids, int64_t B, int k, int H,
                                   TO* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const bool vec = (H & 3) == 0;
  const int ncol = vec ? H >> 2 : H;
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < B;
       t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    int pos = -1, e = 0;
    if (lane < k) {
      pos = __ldg(inv + t * k + lane);
      e = __ldg(ids + t * k + lane);
    }
    const unsigned vm = __ballot_sync(0xffffffffu, lane < k && pos >= 0);
    const int n = __popc(vm);
    // entry `lane` of the compacted list (lanes < n)
    int from = 0;
    if (lane < n) {
      unsigned m = vm;
      for (int i = 0; i < lane; ++i) m &= m - 1u;
      from = __ffs(m) - 1;
    }
    const int cp = __shfl_sync(0xffffffffu, e, from), crow = __shfl_sync(0xffffffffu, pos, from);
    const WarpTree wt = warp_tree(cp, n);
    int64_t row[KC];
#pragma unroll
    for (int r = 0; r < KC; ++r) row[r] = (int64_t)__shfl_sync(0xffffffffu, crow, r < n ? tree_order(wt, r) : 0);
    constexpr int CW = 2;  // column groups per pass of the schedule
    // the loop bound is warp-uniform (lanes past the row's end load zeros and
    // store nothing), so every lane reaches the warp vote below
    for (int cb = 0; cb < ncol; cb += 32 * CW) {
      const int c0 = cb + lane;
      float4 v[KC][CW];
#pragma unroll
      for (int r = 0; r < KC; ++r)
#pragma unroll
        for (int w = 0; w < CW; ++w) {
          const int c = c0 + 32 * w;
          if (r < n && c < ncol)
            v[r][w] = vec ? __ldg(reinterpret_cast<const float4*>(y + row[r] * H) + c)
                          : make_float4(__ldg(y + row[r] * H + c), 0.f, 0.f, 0.f);
          else
            v[r][w] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      tree_apply<KC, CW>(v, wt.sched);
      // a non-finite output (non-finite input, or an fp16 hidden value past
      // 65504 on the bf16 path) is reported through the status word
      bool bad = false;
#pragma unroll
      for (int w = 0; w < CW; ++w)
        bad |= !(isfinite(v[0][w].x) && isfinite(v[0][w].y) && isfinite(v[0][w].z) && isfinite(v[0][w].w));
      if (__any_sync(0xffffffffu, bad) && lane == 0) set_status(ST_RANGE);
#pragma unroll
      for (int w = 0; w < CW; ++w) {
        const int c = c0 + 32 * w;
        if (c < ncol) {
          if (vec)
            store4<TO>(out + t * H + 4 * c, v[0][w]);
          else
            out[t * H + c] = cvt_out<TO>(v[0][w].x);
        }
      }
    }
  }
}

// Slot-order sum for k > TREE_MAX (outside the tree's range).
template <typename TO>
__global__ void moe_combine_slots_kernel(const float* __restrict__ y, const int* __restrict__ inv, int64_t B,
                                         int k, int H, TO* __restrict__ out) {
  const int64_t total = B * (int64_t)H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H;
    const int c = (int)(i % H);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int pos = inv[t * k + j];
      if (pos >= 0) acc += y[(int64_t)pos * H + c];
    }
    out[i] = cvt_out<TO>(acc);
  }
}

template <typename TX, typename TA>
__global__ void rows_convert_kernel(const TX* __restrict__ x, int64_t M, int K, TA* __restrict__ xp,
                                    int64_t ldx) {
  const int64_t total = M * (int64_t)K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / K;
    const int c = (int)(i % K);
    xp[r * ldx + c] = cvt_act<TX, TA>(x[i]);
  }
}

__global__ void fill_i32_kernel(int32_t* p, int64_t n, int32_t v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

namespace {

inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

struct MoeLayout {
  int64_t R, Rp, ldx, ldh, max_mt;  // Rp: rows with every expert segment padded to 32
  size_t off_counts, off_offsets, off_cursor, off_nmt, off_mtiles, off_roww, off_inv, off_ids, off_xp,
      off_hp, off_yp, total;
};

// split: the fp32-faithful form's rows, [hi | lo] (twice as wide)
MoeLayout moe_layout(int64_t B, int64_t H, int64_t I, int32_t E, int32_t k, bool split = false) {
  MoeLayout L{};
  L.R = B * k;
  L.Rp = L.R + 32 * (int64_t)E;
  L.ldx = split ? 2 * H : round_up(H, 64);
  L.ldh = split ? 2 * I : round_up(I, 64);
  L.max_mt = L.Rp / 128 + E + 1;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 1024);
    return at;
  };
  L.off_counts = take(sizeof(int) * E);
  L.off_offsets = take(sizeof(int) * E);
  L.off_cursor = take(sizeof(int) * E);
  L.off_nmt = take(sizeof(int));
  L.off_mtiles = take(sizeof(MTile) * L.max_mt);
  L.off_roww = take(sizeof(float) * L.Rp);
  L.off_inv = take(sizeof(int) * L.R);
  L.off_ids = take(sizeof(int) * L.R);
  L.off_xp = take((size_t)L.Rp * L.ldx * 2);
  L.off_hp = take((size_t)L.Rp * L.ldh * 2);
  L.off_yp = take((size_t)L.Rp * H * 4);
  L.total = o;
  return L;
}

template <int MODE, int FMT>
int launch_tgemm(const char* name, const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1,
                 const TernGemmParams& p, cudaStream_t stream) {
  auto kern = ternary_gemm_kernel<MODE, FMT>;
  static PerDevice attr;
  int dev = 0, rc;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  if ((rc = attr.once(dev, [&]() -> int {
         SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TG_SMEM_BYTES));
         return SB_OK;
       })))
    return rc;
  ProfScope prof(name, stream);
  kern<<<num_sms(), TG_THREADS, TG_SMEM_BYTES, stream>>>(ta, tb0, tb1, p);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

template <int MODE, int FMT>
int launch_ts(const char* name, const CUtensorMap& tx, const CUtensorMap& tw0, const CUtensorMap& tw1,
              const TernGemmParams& p, cudaStream_t stream) {
  auto kern = ternary_ts_kernel<MODE, FMT>;
  static PerDevice attr;
  int dev = 0, rc;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  if ((rc = attr.once(dev, [&]() -> int {
         SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TS_SMEM_BYTES));
         return SB_OK;
       })))
    return rc;
  ProfScope prof(name, stream);
  kern<<<num_sms(), TS_THREADS, TS_SMEM_BYTES, stream>>>(tx, tw0, tw1, p);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

// Which grouped ternary GEMM runs, from SB_TERNARY_ENGINE: "pair" (CTA pairs,
// cta_group::2; the default), "ts" (one CTA per tile, weights in TMEM) or
// "ss" (one CTA per tile, weights unpacked into shared memory).
enum { ENGINE_PAIR = 0, ENGINE_TS = 1, ENGINE_SS = 2 };
int ternary_engine() {
  const char* e = getenv("SB_TERNARY_ENGINE");
  if (e && strcmp(e, "ss") == 0) return ENGINE_SS;
  if (e && strcmp(e, "ts") == 0) return ENGINE_TS;
  return ENGINE_PAIR;
}
bool use_ts_engine() { return ternary_engine() != ENGINE_SS; }

// MMA streams per pair tile.  One issuing thread is the default: two streams
// (SB_PAIR_STREAMS=2) measured 3 % slower on the OLMoE layer (gate/up 0.263 vs
// 0.255 ms), so the issuer's per-block stall is not hidden by a second issuer.
int pair_streams() {
  static const int n = [] {
    const char* e = getenv("SB_PAIR_STREAMS");
    return (e && strcmp(e, "2") == 0) ? 2 : 1;
  }();
  return n;
}

// CTA pairs (clusters of two) as many as fit at once, one persistent pair per two SMs.
template <int MODE, int FMT, int STREAMS>
int launch_pair_s(const char* name, const CUtensorMap& tx, const CUtensorMap& tw0, const CUtensorMap& tw1,
                  const CUtensorMap& tout, const TernGemmParams& p, cudaStream_t stream) {
  auto kern = ternary_pair_kernel<MODE, FMT, STREAMS>;
  static PerDevice pairs;
  int dev = 0, rc;
  SB_CUDA_TRY(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(TP_THREADS);
  cfg.dynamicSmemBytes = TP_SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if ((rc = pairs.once(dev, [&]() -> int {
         SB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TP_SMEM_BYTES));
         cfg.gridDim = dim3(2 * (num_sms() / 2));
         int n = 0;
         SB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
         if (n < 1) return fail(SB_ERR_CUDA, "no CTA pair of the ternary kernel fits on this GPU");
         pairs.value[dev] = n;
         return SB_OK;
       })))
    return rc;
  cfg.gridDim = dim3(2 * pairs.value[dev]);
  ProfScope prof(name, stream);
  SB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tx, tw0, tw1, tout, p));
  return SB_OK;
}

template <int MODE, int FMT>
int launch_pair(const char* name, const CUtensorMap& tx, const CUtensorMap& tw0, const CUtensorMap& tw1,
                const CUtensorMap& tout, const TernGemmParams& p, cudaStream_t stream) {
  return pair_streams() == 2 ? launch_pair_s<MODE, FMT, 2>(name, tx, tw0, tw1, tout, p, stream)
                             : launch_pair_s<MODE, FMT, 1>(name, tx, tw0, tw1, tout, p, stream);
}

bool split_form_fits(int64_t H, int64_t I, int engine) {
  return engine == ENGINE_PAIR && H % TP_KB == 0 && I % TP_KB == 0;
}

int check_ternary_shapes(int64_t H, int64_t I) {
  SB_REQUIRE(H > 0 && I > 0, "hidden=%lld and intermediate=%lld must be positive", (long long)H, (long long)I);
  SB_REQUIRE(H <= (1 << 20) && I <= (1 << 20), "dimensions too large");
  return SB_OK;
}

template <typename TO>
int launch_combine(const float* yp, const int* inv, const int32_t* ids, int64_t B, int k, int64_t H, TO* out,
                   cudaStream_t stream) {
  if (k > TREE_MAX) {
    int64_t blocks = (B * H + 255) / 256;
    if (blocks > (int64_t)num_sms() * 32) blocks = (int64_t)num_sms() * 32;
    moe_combine_slots_kernel<TO><<<(unsigned)blocks, 256, 0, stream>>>(yp, inv, B, k, (int)H, out);
  } else {
    int64_t blocks = (B + 7) / 8;  // 8 tokens (warps) per block
    if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
    if (k <= 8)
      moe_combine_kernel<TO, 8><<<(unsigned)blocks, 256, 0, stream>>>(yp, inv, ids, B, k, (int)H, out);
    else
      moe_combine_kernel<TO, 16><<<(unsigned)blocks, 256, 0, stream>>>(yp, inv, ids, B, k, (int)H, out);
  }
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

// The k per-slot outputs of each token summed into out (tree order).
int moe_combine(const float* yp, const int* inv, const int32_t* ids, int64_t B, int k, int64_t H, void* out,
                int out_dtype, cudaStream_t stream) {
  ProfScope prof("moe_combine", stream);
  if (out_dtype == SB_F32) return launch_combine(yp, inv, ids, B, k, H, static_cast<float*>(out), stream);
  return launch_combine(yp, inv, ids, B, k, H, static_cast<__nv_bfloat16*>(out), stream);
}

// The two grouped GEMMs of the SwiGLU over rows grouped by expert (the m-tile
// table in device memory): h = silu(s_g * (x T_g^T)) * (s_u * (x T_u^T)) into
// hp (fp16), then y = w * s_d * (h T_d^T) into yp (fp32, one row per slot).
struct GroupedSwiGLU {
  const void* xp;
  __half* hp;
  float* yp;
  int64_t Rp, ldx, ldh, H, I;
  int32_t E;
  const MTile* mtiles;
  const int* nmt;
  const float* row_w;
  const uint32_t *gate, *up, *down;
  const float *gs, *us, *ds;
  int fmt_gu;  // 1: bf16 activations, 0: fp16
  int engine;
  // 1: fp32-faithful form (pair engine, H and I multiples of 128): the rows of
  // xp are [x_hi | x_lo] (bf16, 2H wide), h is stored as [h_hi | h_lo] (bf16,
  // 2I wide), and both GEMMs run over the doubled K with the weights read twice
  int split = 0;
};

int grouped_swiglu(const GroupedSwiGLU& g, cudaStream_t stream) {
  int rc;
  const int64_t H = g.H, I = g.I;
  const int32_t E = g.E;
  const int engine = g.engine, fmt_gu = g.fmt_gu;
  const void* xp = g.xp;
  __half* hp = g.hp;
  float* yp = g.yp;
  const uint32_t *gate = g.gate, *up = g.up, *down = g.down;
  const float *gs = g.gs, *us = g.us, *ds = g.ds;
  const MTile* mtiles = g.mtiles;
  const int* nmt = g.nmt;
  const float* row_w = g.row_w;
  // tensor maps: activations (SW128, 64 x 128 box) and packed weights (16 B x rows box)
  CUtensorMap tmx, tmg, tmu, tmh, tmd;
  const CUtensorMapDataType adt = fmt_gu ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapDataType hdt = g.split ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t xk = g.split ? 2 * H : H, hk = g.split ? 2 * I : I;  // activation columns the GEMMs run over
  const int64_t KWh = ternary_row_words(H), KWi = ternary_row_words(I);
  const bool pair = engine == ENGINE_PAIR;
  const uint32_t gu_box = pair ? 64 : 128, d_box = pair ? 128 : 256;
  const uint32_t p_words = pair ? TP_KB / 16 : 4;  // packed words per row in one weight box
  // token rows per activation box: two 48-row boxes per CTA with two MMA streams
  const uint32_t x_rows = pair ? (pair_streams() == 2 ? TP_QROWS : TP_HALF_ROWS) : 128;
  if ((rc = make_tmap_2d(&tmx, xp, adt, 2, g.Rp, xk, g.ldx, 64, x_rows, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&tmg, gate, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)E * I, KWh, KWh, p_words, gu_box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)) ||
      (rc = make_tmap_2d(&tmu, up, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)E * I, KWh, KWh, p_words, gu_box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)) ||
      (rc = make_tmap_2d(&tmh, hp, hdt, 2, g.Rp, hk, g.ldh, 64, x_rows, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&tmd, down, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)E * H, KWi, KWi, p_words, d_box,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  CUtensorMap tmh_out{}, tmy_out{};
  if (pair && ((rc = make_tmap_2d(&tmh_out, hp, hdt, 2, g.Rp, hk, g.ldh, 16, 32, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
               (rc = make_tmap_2d(&tmy_out, yp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.Rp, H, H, 32, 32,
                                  CU_TENSOR_MAP_SWIZZLE_NONE))))
    return rc;

  TernGemmParams pg{};
  pg.mtiles = mtiles;
  pg.num_mtiles = nmt;
  pg.n_ntiles = (int)((I + 127) / 128);
  pg.N = (int)I;
  pg.K = (int)xk;
  pg.b_rows = (int)I;
  if (g.split) {
    pg.kb_wrap = (int)(H / TP_KB);
    pg.h_lo_col = (int)I;
  }
  pg.s0 = gs;
  pg.s1 = us;
  pg.out = hp;
  pg.ldo = g.ldh;
  if (engine == ENGINE_PAIR)
    rc = fmt_gu ? launch_pair<TG_GATEUP, 1>("ternary_gateup_tc", tmx, tmg, tmu, tmh_out, pg, stream)
                : launch_pair<TG_GATEUP, 0>("ternary_gateup_tc", tmx, tmg, tmu, tmh_out, pg, stream);
  else if (engine == ENGINE_TS)
    rc = fmt_gu ? launch_ts<TG_GATEUP, 1>("ternary_gateup_tc", tmx, tmg, tmu, pg, stream)
                : launch_ts<TG_GATEUP, 0>("ternary_gateup_tc", tmx, tmg, tmu, pg, stream);
  else
    rc = fmt_gu ? launch_tgemm<TG_GATEUP, 1>("ternary_gateup_tc", tmx, tmg, tmu, pg, stream)
                : launch_tgemm<TG_GATEUP, 0>("ternary_gateup_tc", tmx, tmg, tmu, pg, stream);
  if (rc) return rc;
  TernGemmParams pd{};
  pd.mtiles = mtiles;
  pd.num_mtiles = nmt;
  pd.n_ntiles = (int)((H + 255) / 256);
  pd.N = (int)H;
  pd.K = (int)hk;
  pd.b_rows = (int)H;
  if (g.split) pd.kb_wrap = (int)(I / TP_KB);
  pd.s0 = ds;
  pd.row_w = row_w;
  pd.out = yp;
  pd.ldo = H;
  if (engine == ENGINE_PAIR)
    rc = g.split ? launch_pair<TG_DOWN, 1>("ternary_down_tc", tmh, tmd, tmd, tmy_out, pd, stream)
                 : launch_pair<TG_DOWN, 0>("ternary_down_tc", tmh, tmd, tmd, tmy_out, pd, stream);
  else if (engine == ENGINE_TS)
    rc = launch_ts<TG_DOWN, 0>("ternary_down_tc", tmh, tmd, tmd, pd, stream);
  else
    rc = launch_tgemm<TG_DOWN, 0>("ternary_down_tc", tmh, tmd, tmd, pd, stream);
  if (rc) return rc;

  return SB_OK;
}

// The grouped SwiGLU pipeline shared by the MoE layer and the single-expert API.
int moe_forward(const void* x, int x_dtype, int64_t B, int64_t H, int64_t I, int32_t E, int32_t k,
                const int32_t* ids, const float* weights, const uint32_t* gate, const uint32_t* up,
                const uint32_t* down, const float* gs, const float* us, const float* ds, void* out,
                int out_dtype, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int rc;
  if ((rc = check_ternary_shapes(H, I))) return rc;
  SB_REQUIRE(E >= 1 && E <= 65536, "n_experts=%d out of range", E);
  SB_REQUIRE(k >= 1 && k <= 64, "top_k=%d out of range", k);
  SB_REQUIRE(x_dtype == SB_F32 || x_dtype == SB_BF16, "x dtype must be SB_F32 or SB_BF16");
  SB_REQUIRE(out_dtype == SB_F32 || out_dtype == SB_BF16, "out dtype must be SB_F32 or SB_BF16");
  if (B == 0) return SB_OK;
  SB_REQUIRE(x && ids && gate && up && down && gs && us && ds && out, "null pointer argument");
  SB_REQUIRE(B * k <= (int64_t)INT32_MAX / 2, "too many (token, slot) pairs");
  // the pair engine stores y rows with TMA: its row pitch (H floats) must be a 16-byte multiple
  int engine = ternary_engine();
  if (engine == ENGINE_PAIR && (H % 4) != 0) engine = ENGINE_TS;
  const bool x16 = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  // fp32 inputs take the fp32-faithful split form where its shapes allow
  // (otherwise they are rounded to fp16, as bf16 inputs' hidden state is)
  const bool split = x_dtype == SB_F32 && split_form_fits(H, I, engine) && x16;
  const MoeLayout L = moe_layout(B, H, I, E, k, split);
  if (!workspace || workspace_bytes < L.total)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, L.total);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(gate) & 15u) == 0 && (reinterpret_cast<uintptr_t>(up) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(down) & 15u) == 0,
             "packed weights must be 16-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + L.off_counts);
  int* offsets = reinterpret_cast<int*>(ws + L.off_offsets);
  int* cursor = reinterpret_cast<int*>(ws + L.off_cursor);
  int* nmt = reinterpret_cast<int*>(ws + L.off_nmt);
  MTile* mtiles = reinterpret_cast<MTile*>(ws + L.off_mtiles);
  float* row_w = reinterpret_cast<float*>(ws + L.off_roww);
  int* inv = reinterpret_cast<int*>(ws + L.off_inv);
  void* xp = ws + L.off_xp;
  __half* hp = reinterpret_cast<__half*>(ws + L.off_hp);
  float* yp = reinterpret_cast<float*>(ws + L.off_yp);
  // bf16 inputs stay bf16; fp32 inputs become bf16 hi/lo pairs (split) or fp16
  const int fmt_gu = (x_dtype == SB_BF16 || split) ? 1 : 0;

  {
    const int64_t R = L.R;
    {
      ProfScope prof_plan("moe_plan", stream);
      if ((rc = moe_plan(ids, R, E, counts, offsets, cursor, mtiles, nmt, (int)L.max_mt,
                         engine == ENGINE_PAIR ? TP_TILE_ROWS : 128, stream)))
        return rc;
    }
    ProfScope prof("moe_dispatch", stream);
    int64_t wblocks = (R * 32 + 255) / 256;
    if (wblocks > (int64_t)num_sms() * 16) wblocks = (int64_t)num_sms() * 16;
    if (split)
      moe_scatter_split_kernel<<<(unsigned)wblocks, 256, 0, stream>>>(
          static_cast<const float*>(x), ids, weights, B, k, (int)H, E, offsets, cursor,
          static_cast<__nv_bfloat16*>(xp), L.ldx, row_w, inv);
    else if (x_dtype == SB_BF16)
      moe_scatter_kernel<__nv_bfloat16, __nv_bfloat16><<<(unsigned)wblocks, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), ids, weights, B, k, (int)H, E, offsets, cursor,
          static_cast<__nv_bfloat16*>(xp), L.ldx, row_w, inv, x16 && (H % 8) == 0);
    else
      moe_scatter_kernel<float, __half><<<(unsigned)wblocks, 256, 0, stream>>>(
          static_cast<const float*>(x), ids, weights, B, k, (int)H, E, offsets, cursor,
          static_cast<__half*>(xp), L.ldx, row_w, inv, x16 && (H % 4) == 0);
    SB_CUDA_TRY(cudaGetLastError());
  }

  GroupedSwiGLU g{xp, hp, yp, L.Rp, L.ldx, L.ldh, H, I, E, mtiles, nmt, row_w,
                  gate, up, down, gs, us, ds, fmt_gu, engine, split ? 1 : 0};
  if ((rc = grouped_swiglu(g, stream))) return rc;
  return moe_combine(yp, inv, ids, B, k, H, out, out_dtype, stream);
}

}  // namespace
}  // namespace sb

extern "C" size_t sb_ternary_moe_workspace_bytes(int64_t B, int64_t H, int64_t I, int32_t E, int32_t k) {
  if (B < 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0) return 0;
  // sized for the fp32-faithful form when the shapes allow it (it is the larger)
  return sb::moe_layout(B, H, I, E, k, sb::split_form_fits(H, I, sb::ENGINE_PAIR)).total;
}

extern "C" int sb_ternary_moe_swiglu(const void* x, int x_dtype, int64_t B, int64_t H, int64_t I,
                                     int32_t n_experts, int32_t top_k, const int32_t* ids,
                                     const float* weights, const uint32_t* gate, const uint32_t* up,
                                     const uint32_t* down, const float* gate_scale, const float* up_scale,
                                     const float* down_scale, void* out, int out_dtype, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  SB_REQUIRE(weights != nullptr || B == 0, "weights is null");
  return sb::moe_forward(x, x_dtype, B, H, I, n_experts, top_k, ids, weights, gate, up, down, gate_scale,
                         up_scale, down_scale, out, out_dtype, workspace, workspace_bytes,
                         reinterpret_cast<cudaStream_t>(stream));
}

namespace sb {
// The few-token path fits: K multiples of 64, at most GEMV_MAX_CHUNKS chunks.
inline bool gemv_fits(int64_t H, int64_t I) {
  return H % 64 == 0 && I % 64 == 0 && H <= GEMV_CHUNK * GEMV_MAX_CHUNKS && I <= GEMV_CHUNK * GEMV_MAX_CHUNKS;
}

template <int N>
int launch_gemv_n(const void* x, int x_dtype, int M, int H, int I, const uint32_t* gate, const uint32_t* up,
                  const uint32_t* down, const float* gs, const float* us, const float* ds, float* h, float* y,
                  cudaStream_t stream) {
  const int hch = (H + GEMV_CHUNK - 1) / GEMV_CHUNK, ich = (I + GEMV_CHUNK - 1) / GEMV_CHUNK;
  const int cpb = GEMV_WARPS / (2 * hch) > 0 ? GEMV_WARPS / (2 * hch) : 1;  // channels per block
  const int opb = GEMV_WARPS / ich > 0 ? GEMV_WARPS / ich : 1;              // output channels per block
  {
    ProfScope prof("ternary_gateup_gemv", stream);
    const unsigned blocks = (unsigned)((I + cpb - 1) / cpb);
    if (x_dtype == SB_F32)
      ternary_gemv_gateup_kernel<N, float><<<blocks, GEMV_WARPS * 32, 0, stream>>>(
          static_cast<const float*>(x), gate, up, gs, us, H, I, cpb, M, h);
    else
      ternary_gemv_gateup_kernel<N, __nv_bfloat16><<<blocks, GEMV_WARPS * 32, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), gate, up, gs, us, H, I, cpb, M, h);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ternary_down_gemv", stream);
    const unsigned blocks = (unsigned)((H + opb - 1) / opb);
    ternary_gemv_down_kernel<N><<<blocks, GEMV_WARPS * 32, 0, stream>>>(h, down, ds, H, I, opb, M, y);
    SB_CUDA_TRY(cudaGetLastError());
  }
  return SB_OK;
}

// One expert over every row (the drop-in ternary_gated_mlp past the few-token
// sizes): the m-tile table of rows [0, M) — tiles of up to tile_rows rows from
// row 0, the last padded to 32 — and a routing weight of 1 for every padded row.
// The rows need no dispatch copy and the single slot no combine: the GEMMs read
// the rows where they are (TMA fills rows past M with zeros and clips the
// stores there), and the down GEMM stores y itself.
__global__ void single_plan_kernel(int64_t M, int tile_rows, int max_mt, MTile* __restrict__ mtiles,
                                   int* __restrict__ nmt, float* __restrict__ row_w) {
  const int64_t cp = (M + 31) & ~(int64_t)31;
  const int64_t nt = (cp + tile_rows - 1) / tile_rows;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  if (i == 0) *nmt = (int)(nt < max_mt ? nt : max_mt);
  for (int64_t t = i; t < nt && t < max_mt; t += stride) {
    MTile m;
    m.expert = 0;
    m.row0 = (int)(t * tile_rows);
    m.rows = (int)(M - m.row0 < tile_rows ? M - m.row0 : tile_rows);
    m.pad = (int)(cp - m.row0 < tile_rows ? cp - m.row0 : tile_rows);
    mtiles[t] = m;
  }
  for (int64_t r = i; r < cp; r += stride) row_w[r] = 1.0f;
}

// The fp32-faithful rows of the single-expert form: row r of x becomes
// [bf16(x) | bf16(x - bf16(x))] in place r of xs (the arithmetic of
// moe_scatter_split_kernel).  A warp per row; H % 4 == 0, 16-byte rows.
__global__ void split_rows_kernel(const float* __restrict__ x, int64_t M, int H, __nv_bfloat16* __restrict__ xs,
                                  int64_t ldx) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < M;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const float4* s4 = reinterpret_cast<const float4*>(x + r * (int64_t)H);
    __nv_bfloat16* dst = xs + r * ldx;
    for (int c = lane; c < H / 4; c += 32) {
      const float4 v = __ldg(s4 + c);
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
      const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
      const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
      *reinterpret_cast<uint2*>(dst + 4 * c) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
      *reinterpret_cast<uint2*>(dst + H + 4 * c) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
    }
  }
}

// The single-expert form applies: the pair engine (its stores are TMA stores,
// clipped at row M), y and the rows 16-byte aligned with 16-byte row pitches;
// bf16 rows are read in place, fp32 rows take the fp32-faithful form.
bool single_form_fits(const void* x, int x_dtype, int64_t H, int64_t I, const float* y) {
  const bool a16 = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  if (ternary_engine() != ENGINE_PAIR || !a16 || (H % 4) != 0) return false;
  if (x_dtype == SB_BF16) return (H % 8) == 0;
  return x_dtype == SB_F32 && split_form_fits(H, I, ENGINE_PAIR);
}

int single_expert_forward(const void* x, int x_dtype, int64_t M, int64_t H, int64_t I, const uint32_t* gate,
                          const uint32_t* up, const uint32_t* down, const float* gs, const float* us,
                          const float* ds, float* y, void* workspace, cudaStream_t stream) {
  const bool split = x_dtype == SB_F32;
  const MoeLayout L = moe_layout(M, H, I, 1, 1, split);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* nmt = reinterpret_cast<int*>(ws + L.off_nmt);
  MTile* mtiles = reinterpret_cast<MTile*>(ws + L.off_mtiles);
  float* row_w = reinterpret_cast<float*>(ws + L.off_roww);
  const void* xp = x;
  int64_t ldx = H;
  {
    ProfScope prof("moe_plan", stream);
    int64_t blocks = ((M + 31) / 32 + 255) / 256 * 32;
    if (blocks < 1) blocks = 1;
    if (blocks > (int64_t)num_sms() * 4) blocks = (int64_t)num_sms() * 4;
    single_plan_kernel<<<(unsigned)blocks, 256, 0, stream>>>(M, TP_TILE_ROWS, (int)L.max_mt, mtiles, nmt, row_w);
    SB_CUDA_TRY(cudaGetLastError());
  }
  if (split) {
    ProfScope prof("moe_dispatch", stream);
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ws + L.off_xp);
    int64_t blocks = (M * 32 + 255) / 256;
    if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
    split_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const float*>(x), M, (int)H, xs, L.ldx);
    SB_CUDA_TRY(cudaGetLastError());
    xp = xs;
    ldx = L.ldx;
  }
  GroupedSwiGLU g{xp, reinterpret_cast<__half*>(ws + L.off_hp), y, M, ldx, L.ldh, H, I, 1, mtiles, nmt, row_w,
                  gate, up, down, gs, us, ds, 1, ENGINE_PAIR, split ? 1 : 0};
  return grouped_swiglu(g, stream);
}

int launch_gemv(const void* x, int x_dtype, int M, int H, int I, const uint32_t* gate, const uint32_t* up,
                const uint32_t* down, const float* gs, const float* us, const float* ds, float* h, float* y,
                cudaStream_t stream) {
  if (M <= 1) return launch_gemv_n<1>(x, x_dtype, M, H, I, gate, up, down, gs, us, ds, h, y, stream);
  if (M <= 2) return launch_gemv_n<2>(x, x_dtype, M, H, I, gate, up, down, gs, us, ds, h, y, stream);
  return launch_gemv_n<4>(x, x_dtype, M, H, I, gate, up, down, gs, us, ds, h, y, stream);
}
}  // namespace sb

// Single expert = the grouped path with one expert and one slot per token;
// the slot ids live at the end of the workspace.
extern "C" size_t sb_ternary_gated_mlp_workspace_bytes(int64_t M, int64_t H, int64_t I) {
  if (M < 0 || H <= 0 || I <= 0) return 0;
  return sb::moe_layout(M, H, I, 1, 1, sb::split_form_fits(H, I, sb::ENGINE_PAIR)).total +
         sb::align_up(sizeof(int32_t) * (size_t)(M > 0 ? M : 1), 1024);
}

extern "C" int sb_ternary_gated_mlp(const void* x, int x_dtype, int64_t M, int64_t H, int64_t I,
                                    const uint32_t* gate, const uint32_t* up, const uint32_t* down,
                                    const float* gate_scale, const float* up_scale, const float* down_scale,
                                    float* y, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sb;
  int rc;
  if ((rc = check_ternary_shapes(H, I))) return rc;
  if (M == 0) return SB_OK;
  const size_t need = sb_ternary_gated_mlp_workspace_bytes(M, H, I);
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
  const size_t base = moe_layout(M, H, I, 1, 1, split_form_fits(H, I, ENGINE_PAIR)).total;
  int32_t* ids = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + base);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (M <= GEMV_ROWS && gemv_fits(H, I) && (reinterpret_cast<uintptr_t>(x) & 7u) == 0) {
    // a handful of tokens: the weight stream over all SMs (ternary_gemv.cuh),
    // the hidden state in fp32 in the workspace
    SB_REQUIRE(gate && up && down && gate_scale && up_scale && down_scale && x && y, "null pointer argument");
    float* h = reinterpret_cast<float*>(workspace);
    return launch_gemv(x, x_dtype, (int)M, (int)H, (int)I, gate, up, down, gate_scale, up_scale, down_scale, h, y,
                       st);
  }
  SB_REQUIRE(gate && up && down && gate_scale && up_scale && down_scale && x && y, "null pointer argument");
  if (single_form_fits(x, x_dtype, H, I, y)) {
    SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
    SB_REQUIRE((reinterpret_cast<uintptr_t>(gate) & 15u) == 0 && (reinterpret_cast<uintptr_t>(up) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(down) & 15u) == 0,
               "packed weights must be 16-byte aligned");
    return single_expert_forward(x, x_dtype, M, H, I, gate, up, down, gate_scale, up_scale, down_scale, y,
                                 workspace, st);
  }
  int64_t blocks = (M + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  fill_i32_kernel<<<(unsigned)blocks, 256, 0, st>>>(ids, M, 0);
  SB_CUDA_TRY(cudaGetLastError());
  return moe_forward(x, x_dtype, M, H, I, 1, 1, ids, nullptr, gate, up, down, gate_scale, up_scale,
                     down_scale, y, SB_F32, workspace, base, st);
}

// y = scale * (x @ T) + bias: the dispatch copies x into the activation layout
// (one expert, identity rows), then one grouped GEMM with the linear epilogue.
extern "C" size_t sb_ternary_linear_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M < 0 || K <= 0 || N <= 0) return 0;
  return sb::moe_layout(M, K, 64, 1, 1).total + sb::align_up(sizeof(int32_t) * (size_t)(M > 0 ? M : 1), 1024);
}

extern "C" int sb_ternary_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                                 const uint32_t* w, const float* scale, const float* bias, float* y,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sb;
  SB_REQUIRE(K > 0 && N > 0, "shape must be positive");
  SB_REQUIRE(x_dtype == SB_F32 || x_dtype == SB_BF16, "x dtype must be SB_F32 or SB_BF16");
  if (M == 0) return SB_OK;
  SB_REQUIRE(x && w && scale && y, "null pointer argument");
  const size_t need = sb_ternary_linear_workspace_bytes(M, K, N);
  if (!workspace || workspace_bytes < need)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  const MoeLayout L = moe_layout(M, K, 64, 1, 1);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + L.off_counts);
  int* offsets = reinterpret_cast<int*>(ws + L.off_offsets);
  int* cursor = reinterpret_cast<int*>(ws + L.off_cursor);
  int* nmt = reinterpret_cast<int*>(ws + L.off_nmt);
  MTile* mtiles = reinterpret_cast<MTile*>(ws + L.off_mtiles);
  void* xp = ws + L.off_xp;
  int32_t* ids = reinterpret_cast<int32_t*>(ws + L.total);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int fmt = (x_dtype == SB_BF16) ? 1 : 0;
  // one expert holding every row in token order: the m-tile table comes from
  // the histogram + scan of all-zero ids, and x is converted row for row
  int64_t blocks = (M + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  fill_i32_kernel<<<(unsigned)blocks, 256, 0, st>>>(ids, M, 0);
  int rc;
  if ((rc = moe_plan(ids, M, 1, counts, offsets, cursor, mtiles, nmt, (int)L.max_mt, 128, st))) return rc;
  {
    int64_t cb = (M * K + 255) / 256;
    if (cb > (int64_t)num_sms() * 32) cb = (int64_t)num_sms() * 32;
    if (fmt)
      rows_convert_kernel<__nv_bfloat16, __nv_bfloat16><<<(unsigned)cb, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(x), M, (int)K, static_cast<__nv_bfloat16*>(xp), L.ldx);
    else
      rows_convert_kernel<float, __half><<<(unsigned)cb, 256, 0, st>>>(static_cast<const float*>(x), M, (int)K,
                                                                         static_cast<__half*>(xp), L.ldx);
    SB_CUDA_TRY(cudaGetLastError());
  }
  CUtensorMap tmx, tmw;
  const int64_t KW = ternary_row_words(K);
  if ((rc = make_tmap_2d(&tmx, xp, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, M,
                         K, L.ldx, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = make_tmap_2d(&tmw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)N, KW, KW, 4, 256,
                         CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  TernGemmParams pl{};
  pl.mtiles = mtiles;
  pl.num_mtiles = nmt;
  pl.n_ntiles = (int)((N + 255) / 256);
  pl.N = (int)N;
  pl.K = (int)K;
  pl.b_rows = (int)N;
  pl.s0 = scale;
  pl.bias = bias;
  pl.out = y;
  pl.ldo = N;
  if (use_ts_engine()) {
    if (fmt) return launch_ts<TG_LINEAR, 1>("ternary_linear_tc", tmx, tmw, tmw, pl, st);
    return launch_ts<TG_LINEAR, 0>("ternary_linear_tc", tmx, tmw, tmw, pl, st);
  }
  if (fmt) return launch_tgemm<TG_LINEAR, 1>("ternary_linear_tc", tmx, tmw, tmw, pl, st);
  return launch_tgemm<TG_LINEAR, 0>("ternary_linear_tc", tmx, tmw, tmw, pl, st);
}
