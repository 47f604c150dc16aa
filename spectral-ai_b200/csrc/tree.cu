// tree.cu — the legacy ray-sphere tree router on B200, and the reference's
// ctypes C ABI around it.
//
// Reference: cuda/v5/bvh_router_kernel.cu (bvh_router_fused_kernel_v2 :244-371,
// host API :378-717) and cuda/v5/bvh_torch_ext.cu:270-371 (same kernel behind
// the torch extension).  A fixed 85-node tree (root, 4, 16, 64 leaves = experts):
//   per level: d_k = |o + t d - c_k|^2 - r_k^2 with t = (c_k - o).d for the 4
//   children; the first minimum wins; the ray passes the child's 3x4 portal
//   (origin affine, direction linear then renormalised); confidence *= exp(-d_min);
//   scores[leaf] = exp(-|o + t d - c_leaf|^2) with the original ray.
// The reference also updates a 64-wide spectral vector at every node (Snell
// dispersion, :180-229); no output reads that vector, so it is not computed
// here and the spectral input is not read.  Arithmetic follows the
// reference's fused multiply-add order and intrinsics, so results match it to
// the last bit wherever the compiler's contraction of the reference agrees.
//
// B200 shape: one thread per ray (the reference spends a 32-thread warp per
// ray on 3 levels of 4 distances); the tree (85 x 16 floats) sits in shared
// memory; the 64 scores per ray are written by (ray, leaf)-mapped threads so
// the stores are coalesced.  The ctypes API keeps pinned staging buffers and
// replays one CUDA graph (copy in, kernel, copy out) per batch size.
#include "common.cuh"

#include <mutex>

namespace sb {

constexpr int TREE_NODES = 85, TREE_LEAVES = 64, TREE_LEAF0 = 21, TREE_LEVELS = 3, TREE_SPEC = 64;
constexpr int TREE_TOK = 128;  // rays per CTA
constexpr int TREE_NODE_F = 16;  // per node: cx, cy, cz, r, portal[12]

__device__ __forceinline__ float tree_ray_dist2(float ox, float oy, float oz, float dx, float dy, float dz, float cx,
                                                float cy, float cz) {
  const float ocx = cx - ox, ocy = cy - oy, ocz = cz - oz;
  const float t = __fmaf_rn(ocx, dx, __fmaf_rn(ocy, dy, ocz * dz));
  const float px = __fmaf_rn(t, dx, ox) - cx;
  const float py = __fmaf_rn(t, dy, oy) - cy;
  const float pz = __fmaf_rn(t, dz, oz) - cz;
  return __fmaf_rn(px, px, __fmaf_rn(py, py, pz * pz));
}

__global__ void __launch_bounds__(TREE_TOK) tree_route_kernel(const float* __restrict__ tree, const float* __restrict__ ro,
                                                              const float* __restrict__ rd, int64_t B,
                                                              int32_t* __restrict__ expert, float* __restrict__ scores,
                                                              int32_t* __restrict__ path, float* __restrict__ conf) {
  __shared__ float nd[TREE_NODES * TREE_NODE_F];
  __shared__ float ray[TREE_TOK][7];
  for (int i = threadIdx.x; i < TREE_NODES * TREE_NODE_F; i += TREE_TOK) nd[i] = __ldg(tree + i);
  for (int64_t b0 = (int64_t)blockIdx.x * TREE_TOK; b0 < B; b0 += (int64_t)gridDim.x * TREE_TOK) {
    __syncthreads();
    const int64_t s = b0 + threadIdx.x;
    if (s < B) {
      float ox = __ldg(ro + 3 * s), oy = __ldg(ro + 3 * s + 1), oz = __ldg(ro + 3 * s + 2);
      float dx = __ldg(rd + 3 * s), dy = __ldg(rd + 3 * s + 1), dz = __ldg(rd + 3 * s + 2);
      float* rr = ray[threadIdx.x];
      rr[0] = ox, rr[1] = oy, rr[2] = oz, rr[3] = dx, rr[4] = dy, rr[5] = dz;
      int node = 0;
      float c = 1.0f;
#pragma unroll
      for (int l = 0; l < TREE_LEVELS; ++l) {
        const int first = node * 4 + 1;
        float d[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* n = nd + (first + q) * TREE_NODE_F;
          d[q] = __fmaf_rn(-n[3], n[3], tree_ray_dist2(ox, oy, oz, dx, dy, dz, n[0], n[1], n[2]));
        }
        // first minimum of (d0, d1) vs (d2, d3), as a two-stage tournament
        const float ab = d[0] <= d[1] ? d[0] : d[1];
        const int abi = d[0] <= d[1] ? 0 : 1;
        const float cd = d[2] <= d[3] ? d[2] : d[3];
        const int cdi = d[2] <= d[3] ? 2 : 3;
        const float best = ab <= cd ? ab : cd;
        const int child = first + (ab <= cd ? abi : cdi);
        if (path) path[s * TREE_LEVELS + l] = child;
        // portal of the chosen child: origin affine, direction linear, renormalised
        const float* p = nd + child * TREE_NODE_F + 4;
        const float nox = __fmaf_rn(p[0], ox, __fmaf_rn(p[1], oy, __fmaf_rn(p[2], oz, p[3])));
        const float noy = __fmaf_rn(p[4], ox, __fmaf_rn(p[5], oy, __fmaf_rn(p[6], oz, p[7])));
        const float noz = __fmaf_rn(p[8], ox, __fmaf_rn(p[9], oy, __fmaf_rn(p[10], oz, p[11])));
        float ndx = __fmaf_rn(p[0], dx, __fmaf_rn(p[1], dy, p[2] * dz));
        float ndy = __fmaf_rn(p[4], dx, __fmaf_rn(p[5], dy, p[6] * dz));
        float ndz = __fmaf_rn(p[8], dx, __fmaf_rn(p[9], dy, p[10] * dz));
        const float inv = rsqrtf(__fmaf_rn(ndx, ndx, __fmaf_rn(ndy, ndy, ndz * ndz)) + 1e-12f);
        ox = nox, oy = noy, oz = noz;
        dx = ndx * inv, dy = ndy * inv, dz = ndz * inv;
        c *= __expf(-best);
        node = child;
      }
      if (expert) expert[s] = node - TREE_LEAF0;
      if (conf) conf[s] = c;
    }
    __syncthreads();
    if (scores) {
      const int ntok = (int)(B - b0 < TREE_TOK ? B - b0 : TREE_TOK);
      for (int i = threadIdx.x; i < ntok * TREE_LEAVES; i += TREE_TOK) {
        const int t = i / TREE_LEAVES, leaf = i % TREE_LEAVES;
        const float* rr = ray[t];
        const float* n = nd + (TREE_LEAF0 + leaf) * TREE_NODE_F;
        const float d2 = tree_ray_dist2(rr[0], rr[1], rr[2], rr[3], rr[4], rr[5], n[0], n[1], n[2]);
        scores[(b0 + t) * TREE_LEAVES + leaf] = __expf(-d2);
      }
    }
  }
}

int tree_launch(const float* tree, const float* ro, const float* rd, int64_t B, int32_t* expert, float* scores,
                int32_t* path, float* conf, cudaStream_t st, bool timed = true) {
  int64_t blocks = (B + TREE_TOK - 1) / TREE_TOK;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (!timed) {  // inside a stream capture: no profiling events
    tree_route_kernel<<<(unsigned)blocks, TREE_TOK, 0, st>>>(tree, ro, rd, B, expert, scores, path, conf);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
  }
  ProfScope prof("tree_route", st);
  tree_route_kernel<<<(unsigned)blocks, TREE_TOK, 0, st>>>(tree, ro, rd, B, expert, scores, path, conf);
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

}  // namespace sb

struct sb_tree {
  int device = 0;
  float* d_tree = nullptr;  // [85][16]
  bool uploaded = false;
};

extern "C" int sb_tree_create(int device, sb_tree** out) {
  using namespace sb;
  SB_REQUIRE(out, "sb_tree_create: null out");
  *out = nullptr;
  int n = 0;
  SB_CUDA_TRY(cudaGetDeviceCount(&n));
  SB_REQUIRE(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  SB_CUDA_TRY(cudaSetDevice(device));
  sb_tree* h = new (std::nothrow) sb_tree;
  if (!h) {
    cudaSetDevice(prev);
    return fail(SB_ERR_NOMEM, "sb_tree_create: host allocation failed");
  }
  h->device = device;
  const cudaError_t e = cudaMalloc(&h->d_tree, TREE_NODES * TREE_NODE_F * sizeof(float));
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    delete h;
    return fail(SB_ERR_NOMEM, "sb_tree_create: %s", cudaGetErrorString(e));
  }
  *out = h;
  return SB_OK;
}

extern "C" int sb_tree_upload(sb_tree* h, const float* centers, const float* radii, const float* portals,
                              const float* snell_w, const float* snell_b) {
  using namespace sb;
  SB_REQUIRE(h && centers && radii && portals, "sb_tree_upload: centers, radii and portals are required");
  (void)snell_w;  // the dispersion parameters change no output (see the file comment)
  (void)snell_b;
  float blk[TREE_NODES * TREE_NODE_F];
  for (int n = 0; n < TREE_NODES; ++n) {
    float* b = blk + n * TREE_NODE_F;
    b[0] = centers[3 * n], b[1] = centers[3 * n + 1], b[2] = centers[3 * n + 2], b[3] = radii[n];
    for (int i = 0; i < 12; ++i) b[4 + i] = portals[12 * n + i];
  }
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  SB_CUDA_TRY(cudaSetDevice(h->device));
  const cudaError_t e = cudaMemcpy(h->d_tree, blk, sizeof(blk), cudaMemcpyHostToDevice);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "sb_tree_upload: %s", cudaGetErrorString(e));
  h->uploaded = true;
  return SB_OK;
}

extern "C" int sb_tree_route(sb_tree* h, const float* origins, const float* directions, int64_t batch,
                             int32_t* expert, float* scores, int32_t* path, float* confidence, void* stream) {
  using namespace sb;
  SB_REQUIRE(h, "sb_tree_route: null handle");
  SB_REQUIRE(h->uploaded, "sb_tree_route: tree was not uploaded");
  SB_REQUIRE(batch >= 0, "batch=%lld must be >= 0", (long long)batch);
  if (batch == 0) return SB_OK;
  SB_REQUIRE(origins && directions, "origins and directions are required");
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  if (prev != h->device) SB_CUDA_TRY(cudaSetDevice(h->device));
  const int rc = tree_launch(h->d_tree, origins, directions, batch, expert, scores, path, confidence,
                             reinterpret_cast<cudaStream_t>(stream));
  if (prev != h->device) cudaSetDevice(prev);
  return rc;
}

extern "C" int sb_tree_destroy(sb_tree* h) {
  if (!h) return SB_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  cudaFree(h->d_tree);
  cudaSetDevice(prev);
  delete h;
  return SB_OK;
}

// ===========================================================================
// The reference's ctypes C ABI (cuda/v5/bvh_router_kernel.cu:378-717), same
// names and signatures, process-global like the reference: one tree on the
// device current at bvh_upload_tree, device buffers and pinned staging sized
// by bvh_alloc_buffers, and bvh_route_batch synchronous on host buffers with
// optional CUDA-graph replay.  The graph copies through the pinned staging
// buffers, so a replay is correct for any caller buffers (the reference's
// graph keeps the host pointers of the call that captured it).  The spectral
// input is accepted and not read.  Status: 0 ok, -1 failure (message on
// stderr and in sb_last_error).
// ===========================================================================
namespace {

struct LegacyTree {
  std::mutex mu;
  sb_tree* tree = nullptr;
  int cap = 0;
  float *d_o = nullptr, *d_d = nullptr, *d_s = nullptr, *d_c = nullptr;
  int32_t *d_e = nullptr, *d_p = nullptr;
  float *h_o = nullptr, *h_d = nullptr, *h_s = nullptr, *h_c = nullptr;
  int32_t *h_e = nullptr, *h_p = nullptr;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t exec = nullptr;
  int graph_batch = 0;

  void drop_graph() {
    if (exec) cudaGraphExecDestroy(exec);
    exec = nullptr;
    graph_batch = 0;
  }
  void free_buffers() {
    drop_graph();
    for (void* p : {(void*)d_o, (void*)d_d, (void*)d_s, (void*)d_c, (void*)d_e, (void*)d_p})
      if (p) cudaFree(p);
    for (void* p : {(void*)h_o, (void*)h_d, (void*)h_s, (void*)h_c, (void*)h_e, (void*)h_p})
      if (p) cudaFreeHost(p);
    d_o = d_d = d_s = d_c = h_o = h_d = h_s = h_c = nullptr;
    d_e = d_p = h_e = h_p = nullptr;
    cap = 0;
  }
};

LegacyTree g_legacy;

int legacy_fail(const char* where, const char* msg) {
  fprintf(stderr, "[%s] %s\n", where, msg);
  sb::fail(SB_ERR_INVALID, "%s: %s", where, msg);
  return -1;
}

}  // namespace

extern "C" int bvh_upload_tree(const float* centers, const float* radii, const float* portals, const float* snell_w,
                               const float* snell_b) {
  std::lock_guard<std::mutex> lk(g_legacy.mu);
  if (!g_legacy.tree) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || sb_tree_create(dev, &g_legacy.tree) != SB_OK)
      return legacy_fail("bvh_upload_tree", "cannot create the device tree");
  }
  if (sb_tree_upload(g_legacy.tree, centers, radii, portals, snell_w, snell_b) != SB_OK)
    return legacy_fail("bvh_upload_tree", "upload failed");
  return 0;
}

extern "C" int bvh_alloc_buffers(int batch_size) {
  std::lock_guard<std::mutex> lk(g_legacy.mu);
  if (batch_size <= 0) return legacy_fail("bvh_alloc_buffers", "batch_size must be >= 1");
  if (batch_size <= g_legacy.cap) return 0;
  g_legacy.free_buffers();
  const size_t B = (size_t)batch_size;
  bool ok = cudaMalloc(&g_legacy.d_o, B * 3 * 4) == cudaSuccess && cudaMalloc(&g_legacy.d_d, B * 3 * 4) == cudaSuccess &&
            cudaMalloc(&g_legacy.d_s, B * sb::TREE_LEAVES * 4) == cudaSuccess &&
            cudaMalloc(&g_legacy.d_c, B * 4) == cudaSuccess && cudaMalloc(&g_legacy.d_e, B * 4) == cudaSuccess &&
            cudaMalloc(&g_legacy.d_p, B * sb::TREE_LEVELS * 4) == cudaSuccess &&
            cudaMallocHost(&g_legacy.h_o, B * 3 * 4) == cudaSuccess &&
            cudaMallocHost(&g_legacy.h_d, B * 3 * 4) == cudaSuccess &&
            cudaMallocHost(&g_legacy.h_s, B * sb::TREE_LEAVES * 4) == cudaSuccess &&
            cudaMallocHost(&g_legacy.h_c, B * 4) == cudaSuccess && cudaMallocHost(&g_legacy.h_e, B * 4) == cudaSuccess &&
            cudaMallocHost(&g_legacy.h_p, B * sb::TREE_LEVELS * 4) == cudaSuccess;
  if (ok && !g_legacy.stream) ok = cudaStreamCreateWithFlags(&g_legacy.stream, cudaStreamNonBlocking) == cudaSuccess;
  if (!ok) {
    g_legacy.free_buffers();
    return legacy_fail("bvh_alloc_buffers", cudaGetErrorString(cudaGetLastError()));
  }
  g_legacy.cap = batch_size;
  return 0;
}

extern "C" void bvh_free_buffers(void) {
  std::lock_guard<std::mutex> lk(g_legacy.mu);
  g_legacy.free_buffers();
  if (g_legacy.stream) cudaStreamDestroy(g_legacy.stream);
  g_legacy.stream = nullptr;
}

extern "C" int bvh_route_batch(const float* h_origins, const float* h_directions, const float* h_spectral,
                               int* h_expert, float* h_scores, int* h_path, float* h_confidence, int batch_size,
                               int use_graph) {
  (void)h_spectral;
  std::lock_guard<std::mutex> lk(g_legacy.mu);
  LegacyTree& L = g_legacy;
  if (!L.tree || !L.tree->uploaded) return legacy_fail("bvh_route_batch", "call bvh_upload_tree first");
  if (batch_size <= 0 || batch_size > L.cap) {
    char m[96];
    snprintf(m, sizeof(m), "batch_size=%d but buffer capacity=%d", batch_size, L.cap);
    return legacy_fail("bvh_route_batch", m);
  }
  if (!h_origins || !h_directions) return legacy_fail("bvh_route_batch", "origins and directions are required");
  const size_t B = (size_t)batch_size;
  memcpy(L.h_o, h_origins, B * 3 * 4);
  memcpy(L.h_d, h_directions, B * 3 * 4);
  cudaStream_t st = L.stream;
  auto enqueue = [&](bool timed) -> bool {
    return cudaMemcpyAsync(L.d_o, L.h_o, B * 3 * 4, cudaMemcpyHostToDevice, st) == cudaSuccess &&
           cudaMemcpyAsync(L.d_d, L.h_d, B * 3 * 4, cudaMemcpyHostToDevice, st) == cudaSuccess &&
           sb::tree_launch(L.tree->d_tree, L.d_o, L.d_d, (int64_t)B, L.d_e, L.d_s, L.d_p, L.d_c, st, timed) ==
               SB_OK &&
           cudaMemcpyAsync(L.h_e, L.d_e, B * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
           cudaMemcpyAsync(L.h_s, L.d_s, B * sb::TREE_LEAVES * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
           cudaMemcpyAsync(L.h_p, L.d_p, B * sb::TREE_LEVELS * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
           cudaMemcpyAsync(L.h_c, L.d_c, B * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
  };
  bool ok;
  if (use_graph) {
    if (L.graph_batch != batch_size || !L.exec) {
      L.drop_graph();
      cudaGraph_t g = nullptr;
      ok = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
      const bool enq = ok && enqueue(false);
      ok = cudaStreamEndCapture(st, &g) == cudaSuccess && enq && g != nullptr;
      if (ok) ok = cudaGraphInstantiate(&L.exec, g, 0) == cudaSuccess;
      if (g) cudaGraphDestroy(g);
      if (!ok) {
        L.drop_graph();
        return legacy_fail("bvh_route_batch", "graph capture failed");
      }
      L.graph_batch = batch_size;
    }
    ok = cudaGraphLaunch(L.exec, st) == cudaSuccess;
  } else {
    ok = enqueue(true);
  }
  if (!ok || cudaStreamSynchronize(st) != cudaSuccess)
    return legacy_fail("bvh_route_batch", cudaGetErrorString(cudaGetLastError()));
  if (h_expert) memcpy(h_expert, L.h_e, B * 4);
  if (h_scores) memcpy(h_scores, L.h_s, B * sb::TREE_LEAVES * 4);
  if (h_path) memcpy(h_path, L.h_p, B * sb::TREE_LEVELS * 4);
  if (h_confidence) memcpy(h_confidence, L.h_c, B * 4);
  return 0;
}

extern "C" int bvh_get_batch_capacity(void) { return g_legacy.cap; }
extern "C" int bvh_get_num_nodes(void) { return sb::TREE_NODES; }
extern "C" int bvh_get_num_experts(void) { return sb::TREE_LEAVES; }
extern "C" int bvh_get_spec_dim(void) { return sb::TREE_SPEC; }
