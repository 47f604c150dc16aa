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
// has its non-zero flag at bit 16e+j and its sign flag at bit 16e+8+j.  A pair
// (2j, 2j+1) expands to two packed 16-bit floats with
//   ((w & (0x00010001 << j)) * (M << (P - j))) | ((w & (0x01000100 << j)) << (7 - j))
// where M << P is the magnitude pattern of 1.0 (bf16: 0x7F << 7, fp16: 0xF << 10).
#include "common.cuh"

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
    uint32_t out = 0;
    if (w < P) {
      const uint32_t codes = ref[w * N + n];  // 16 codes of K rows 16w..16w+15, column n
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int64_t k = w * 16 + t;
        if (k >= K) break;
        const int s = ternary_code_to_sign((codes >> (2 * t)) & 3u);
        if (s == 0) continue;
        const int e = t & 1, j = t >> 1;
        out |= 1u << (16 * e + j);
        if (s < 0) out |= 1u << (16 * e + 8 + j);
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

extern "C" size_t sb_ternary_gated_mlp_workspace_bytes(int64_t M, int64_t H, int64_t I) {
  (void)M; (void)H; (void)I;
  return 0;
}
extern "C" int sb_ternary_gated_mlp(const void*, int, int64_t, int64_t, int64_t, const uint32_t*,
                                    const uint32_t*, const uint32_t*, const float*, const float*,
                                    const float*, float*, void*, size_t, void*) {
  return sb::fail(SB_ERR_UNSUPPORTED, "sb_ternary_gated_mlp: not built yet");
}
extern "C" size_t sb_ternary_linear_workspace_bytes(int64_t, int64_t, int64_t) { return 0; }
extern "C" int sb_ternary_linear(const void*, int, int64_t, int64_t, int64_t, const uint32_t*,
                                 const float*, const float*, float*, void*, size_t, void*) {
  return sb::fail(SB_ERR_UNSUPPORTED, "sb_ternary_linear: not built yet");
}
extern "C" size_t sb_ternary_moe_workspace_bytes(int64_t, int64_t, int64_t, int32_t, int32_t) {
  return 0;
}
extern "C" int sb_ternary_moe_swiglu(const void*, int, int64_t, int64_t, int64_t, int32_t, int32_t,
                                     const int32_t*, const float*, const uint32_t*,
                                     const uint32_t*, const uint32_t*, const float*, const float*,
                                     const float*, void*, int, void*, size_t, void*) {
  return sb::fail(SB_ERR_UNSUPPORTED, "sb_ternary_moe_swiglu: not built yet");
}
