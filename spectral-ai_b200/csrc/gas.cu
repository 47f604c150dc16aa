// gas.cu — the OptiX router's routing, served by CUDA kernels (no RT cores or
// OptiX on this path).
//
// Reference: cuda/v5/optix_training_ext.cu:182-263 (route, route_topk), the
// device programs cuda/optix_router_raygen.cu:57-186 (one ray, or a fan of k
// rays on a golden-angle spiral inside a 0.5-rad cone) and
// cuda/optix_router_hitgroup.cu (closest hit -> expert id, hit distance; miss ->
// 0xFFFFFFFF, 1e30), and the acceleration-structure builders of
// cuda/optix_router_host.cpp:372-600:
//   * triangles (the mode BVHGateWrapper builds): per expert an octahedron with
//     vertices c +- r e_x, c +- r e_y, c +- r e_z and 8 faces; expert = the
//     closest hit triangle's index / 8; the distance is its ray parameter t;
//   * AABBs: per expert the box c +- r.  The reference's intersection program
//     reports every box at the ray's tmin, which leaves the choice to the RT
//     traversal order; here a box is hit at its entry point max(t_entry,
//     tmin), as that program's comment describes, and the closest box wins.
// Rays live in [tmin, tmax] = [0.001, 1000] (optix_router_host.cpp:719-720);
// equal distances go to the lower expert index.
//
// B200 shape: one thread per ray; the experts' centers and radii sit in shared
// memory; a ray first tests the expert's bounding sphere (the octahedron and
// the box lie inside / around it) and skips the 8 triangles or the slab test
// when it misses.
#include "common.cuh"

namespace sb {

constexpr int GAS_THREADS = 128;
constexpr int GAS_MAX_EXPERTS = 4096;
constexpr float GAS_TMIN = 0.001f, GAS_TMAX = 1000.0f;

__device__ __forceinline__ float3 gas_cross(float3 a, float3 b) {
  return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
__device__ __forceinline__ float gas_dot(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float3 gas_sub(float3 a, float3 b) { return make_float3(a.x - b.x, a.y - b.y, a.z - b.z); }

// Ray-triangle (two-sided) ray parameter t, or INFINITY.
__device__ __forceinline__ float gas_tri(float3 o, float3 d, float3 v0, float3 v1, float3 v2) {
  const float3 e1 = gas_sub(v1, v0), e2 = gas_sub(v2, v0);
  const float3 p = gas_cross(d, e2);
  const float det = gas_dot(e1, p);
  if (fabsf(det) < 1e-12f) return INFINITY;
  const float inv = 1.0f / det;
  const float3 s = gas_sub(o, v0);
  const float u = gas_dot(s, p) * inv;
  if (u < 0.f || u > 1.f) return INFINITY;
  const float3 q = gas_cross(s, e1);
  const float v = gas_dot(d, q) * inv;
  if (v < 0.f || u + v > 1.f) return INFINITY;
  return gas_dot(e2, q) * inv;
}

// Closest hit of one ray: (expert or -1, distance or 1e30).
__device__ __forceinline__ void gas_trace(float3 o, float3 d, const float4* sph, int n, bool tris, int& id,
                                          float& dist) {
  const float dd = gas_dot(d, d);
  float best = INFINITY;
  int bi = -1;
  for (int e = 0; e < n; ++e) {
    const float4 c = sph[e];
    const float3 cc = make_float3(c.x, c.y, c.z);
    // bounding sphere of radius r * sqrt(3) (covers the box's corners too)
    const float3 oc = gas_sub(cc, o);
    const float tc = gas_dot(oc, d) / dd;
    const float3 pc = make_float3(o.x + tc * d.x - cc.x, o.y + tc * d.y - cc.y, o.z + tc * d.z - cc.z);
    if (gas_dot(pc, pc) > 3.0f * c.w * c.w * 1.0001f) continue;
    float t = INFINITY;
    if (tris) {
      const float r = c.w;
      const float3 vx[6] = {make_float3(cc.x + r, cc.y, cc.z), make_float3(cc.x - r, cc.y, cc.z),
                            make_float3(cc.x, cc.y + r, cc.z), make_float3(cc.x, cc.y - r, cc.z),
                            make_float3(cc.x, cc.y, cc.z + r), make_float3(cc.x, cc.y, cc.z - r)};
      const int f[8][3] = {{0, 2, 4}, {0, 4, 3}, {0, 3, 5}, {0, 5, 2}, {1, 4, 2}, {1, 3, 4}, {1, 5, 3}, {1, 2, 5}};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float tk = gas_tri(o, d, vx[f[k][0]], vx[f[k][1]], vx[f[k][2]]);
        if (tk >= GAS_TMIN && tk <= GAS_TMAX && tk < t) t = tk;
      }
    } else {
      float t0 = -INFINITY, t1 = INFINITY;
      const float oo[3] = {o.x, o.y, o.z}, dv[3] = {d.x, d.y, d.z}, cv[3] = {cc.x, cc.y, cc.z};
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const float lo = cv[a] - c.w, hi = cv[a] + c.w;
        if (dv[a] == 0.f) {
          if (oo[a] < lo || oo[a] > hi) t0 = INFINITY;
        } else {
          float ta = (lo - oo[a]) / dv[a], tb = (hi - oo[a]) / dv[a];
          if (ta > tb) {
            const float tmp = ta;
            ta = tb;
            tb = tmp;
          }
          t0 = fmaxf(t0, ta);
          t1 = fminf(t1, tb);
        }
      }
      const float te = fmaxf(t0, GAS_TMIN);
      if (t0 <= t1 && t1 >= GAS_TMIN && te <= GAS_TMAX) t = te;
    }
    if (t < best) {
      best = t;
      bi = e;
    }
  }
  id = bi;
  dist = bi < 0 ? 1e30f : best;
}

__global__ void __launch_bounds__(GAS_THREADS) gas_route_kernel(const float4* __restrict__ spheres, int n, int tris,
                                                                const float* __restrict__ pos,
                                                                const float* __restrict__ dir, int64_t B, int k,
                                                                int32_t* __restrict__ ids, float* __restrict__ dists,
                                                                int32_t* __restrict__ tids,
                                                                float* __restrict__ tdists) {
  extern __shared__ float4 gas_sph[];
  for (int i = threadIdx.x; i < n; i += GAS_THREADS) gas_sph[i] = spheres[i];
  __syncthreads();
  for (int64_t b = (int64_t)blockIdx.x * GAS_THREADS + threadIdx.x; b < B; b += (int64_t)gridDim.x * GAS_THREADS) {
    const float3 o = make_float3(pos[3 * b], pos[3 * b + 1], pos[3 * b + 2]);
    const float3 d = make_float3(dir[3 * b], dir[3 * b + 1], dir[3 * b + 2]);
    if (k <= 1) {
      int id;
      float t;
      gas_trace(o, d, gas_sph, n, tris != 0, id, t);
      ids[b] = id;
      dists[b] = t;
      continue;
    }
    // fan of k rays around d (optix_router_raygen.cu:103-170)
    float3 u;
    {
      const float3 tmp = fabsf(d.x) < 0.9f ? make_float3(1.f, 0.f, 0.f) : make_float3(0.f, 1.f, 0.f);
      u = gas_cross(d, tmp);
      const float len = sqrtf(u.x * u.x + u.y * u.y + u.z * u.z);
      if (len > 1e-6f) u = make_float3(u.x / len, u.y / len, u.z / len);
    }
    const float3 v = gas_cross(d, u);
    for (int i = 0; i < k; ++i) {
      const float t = (float)i / (float)k;
      const float phi = 2.0f * 3.14159265f * t * 1.6180339887f;
      const float r = 0.5f * sqrtf(t);
      const float cp = cosf(phi), sp = sinf(phi);
      float3 di = make_float3(d.x + r * (cp * u.x + sp * v.x), d.y + r * (cp * u.y + sp * v.y),
                              d.z + r * (cp * u.z + sp * v.z));
      const float len = sqrtf(di.x * di.x + di.y * di.y + di.z * di.z);
      if (len > 1e-6f) di = make_float3(di.x / len, di.y / len, di.z / len);
      int id;
      float th;
      gas_trace(o, di, gas_sph, n, tris != 0, id, th);
      if (tids) tids[b * k + i] = id;
      if (tdists) tdists[b * k + i] = th;
      if (i == 0) {
        ids[b] = id;
        dists[b] = th;
      }
    }
  }
}

}  // namespace sb

struct sb_gas {
  int device = 0;
  float4* spheres = nullptr;  // [n] center xyz, radius
  int n = 0;
  int tris = 1;
};

extern "C" int sb_gas_create(int device, sb_gas** out) {
  using namespace sb;
  SB_REQUIRE(out, "sb_gas_create: null out");
  *out = nullptr;
  int nd = 0;
  SB_CUDA_TRY(cudaGetDeviceCount(&nd));
  SB_REQUIRE(device >= 0 && device < nd, "device %d out of range (%d devices)", device, nd);
  sb_gas* h = new (std::nothrow) sb_gas;
  if (!h) return fail(SB_ERR_NOMEM, "sb_gas_create: host allocation failed");
  h->device = device;
  *out = h;
  return SB_OK;
}

extern "C" int sb_gas_build(sb_gas* h, const float* centers, const float* radii, int n_experts, int use_triangles) {
  using namespace sb;
  SB_REQUIRE(h && centers && radii, "sb_gas_build: null argument");
  SB_REQUIRE(n_experts >= 1 && n_experts <= GAS_MAX_EXPERTS, "n_experts=%d must be in [1, %d]", n_experts,
             GAS_MAX_EXPERTS);
  std::vector<float4> sph((size_t)n_experts);
  for (int e = 0; e < n_experts; ++e)
    sph[e] = make_float4(centers[3 * e], centers[3 * e + 1], centers[3 * e + 2], radii[e]);
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  SB_CUDA_TRY(cudaSetDevice(h->device));
  if (h->spheres) cudaFree(h->spheres);
  h->spheres = nullptr;
  h->n = 0;
  cudaError_t e = cudaMalloc(&h->spheres, sph.size() * sizeof(float4));
  if (e == cudaSuccess) e = cudaMemcpy(h->spheres, sph.data(), sph.size() * sizeof(float4), cudaMemcpyHostToDevice);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "sb_gas_build: %s", cudaGetErrorString(e));
  h->n = n_experts;
  h->tris = use_triangles ? 1 : 0;
  return SB_OK;
}

extern "C" int sb_gas_route(sb_gas* h, const float* positions, const float* directions, int64_t batch, int top_k,
                            int32_t* expert_ids, float* distances, int32_t* topk_ids, float* topk_dists,
                            void* stream) {
  using namespace sb;
  SB_REQUIRE(h && h->n > 0, "sb_gas_route: build the geometry first");
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  SB_REQUIRE(top_k >= 1 && top_k <= 1024, "top_k=%d must be in [1, 1024]", top_k);
  if (batch == 0) return SB_OK;
  SB_REQUIRE(positions && directions && expert_ids && distances, "positions, directions and outputs are required");
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  if (prev != h->device) SB_CUDA_TRY(cudaSetDevice(h->device));
  int64_t blocks = (batch + GAS_THREADS - 1) / GAS_THREADS;
  if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)h->n * sizeof(float4);
  cudaError_t e = cudaSuccess;
  // opt-in shared memory: the kernel's cap is raised to 227 KB once per device
  static PerDevice attr;
  if (smem > 48 * 1024 &&
      attr.once(h->device, [&]() -> int {
        e = cudaFuncSetAttribute(gas_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        return e == cudaSuccess ? SB_OK : SB_ERR_CUDA;
      }) != SB_OK && e == cudaSuccess)
    e = cudaErrorInvalidDevice;
  if (e == cudaSuccess) {
    ProfScope prof("gas_route", st);
    gas_route_kernel<<<(unsigned)blocks, GAS_THREADS, smem, st>>>(h->spheres, h->n, h->tris, positions, directions,
                                                                 batch, top_k, expert_ids, distances, topk_ids,
                                                                 topk_dists);
    e = cudaGetLastError();
  }
  if (prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "sb_gas_route: %s", cudaGetErrorString(e));
  return SB_OK;
}

extern "C" int sb_gas_destroy(sb_gas* h) {
  if (!h) return SB_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  if (h->spheres) cudaFree(h->spheres);
  cudaSetDevice(prev);
  delete h;
  return SB_OK;
}
