// ep.cu — the MoE layer expert-parallel over the GPUs of one node, with the
// token exchange done by the layer's own kernels through peer memory (NVLink /
// NVSwitch): no host round trip, no library collective on the data path.
//
// W ranks (one process per GPU), E experts, rank r holds the experts at
// positions [r*El, (r+1)*El), El = E / W; an expert's position is its id, or
// perm[id] after sb_ep_set_placement (spreading the busy experts over the
// ranks).  One forward on every rank (all ranks call it the same number of
// times; it is collective):
//
//   ep_send         a warp per token: the ranks its k expert ids live on, a
//                   row claimed in each of those ranks' receive segment for
//                   this rank (an atomic counter per destination), the token's
//                   row (bf16, loaded once) and its metadata — the
//                   destination's local expert ids of the token, ascending, and
//                   their routing weights — stored straight into the
//                   destination's receive buffer; a token goes once to each
//                   rank holding any of its experts, however many live there
//                   (the reference sends one copy per slot through its Python
//                   loop, python/olmoe_extract.py:146-155).  The last block
//                   stores the row counts and raises this rank's dispatch flag
//                   at every destination.
//   ep_wait         one block waits (bounded) for every source's flag;
//   ep_recv_plan    histograms the received (row, expert) entries, plans expert
//                   segments and m-tiles as the single-GPU layer does.
//   ep_recv_scatter copies each received row into its experts' segments.
//   grouped GEMMs   the same tcgen05 kernels as the single-GPU layer
//                   (gate/up + SwiGLU, down + routing weight, fp32 per entry).
//   ep_return       per received row, the tree sum (tree_sum.cuh) of its
//                   entries' outputs — the subtree of this rank's experts —
//                   stored (fp32) into the source's return buffer; the last
//                   block raises this rank's return flag at every source.
//   ep_wait         one block waits for every destination's return flag;
//   ep_combine      per token, the tree sum of its destinations' partial sums -> out.
//
// Because the partial sums follow the same tree as the single-GPU combine,
// the layer's output equals the single-GPU layer's bit for bit whenever E/W is
// a power of two.  The reference has no multi-GPU code; this replaces its
// per-slot dispatch loop and the atomic scatter / weighted combine kernels of
// cuda/async_pipeline.cu:79-133 when the experts are spread over GPUs.
//
// Ordering: a source's rows are plain stores into peer memory; each block
// orders them before its done count with a GPU-scope fence, and the last block,
// having seen every count, fences at system scope before its st.release.sys of
// the flag; a waiting thread reads the flag with ld.acquire.sys.  Flags carry
// the forward's epoch (a counter in device memory, bumped by ep_send), so they
// never need resetting and the
// forward can be replayed from a CUDA graph.  Buffer reuse across forwards is
// ordered by the protocol itself: a source writes forward t+1's rows only after
// its combine of forward t saw every destination's return flag, which each
// destination raises after its last read of forward t's rows.
//
// Waits are bounded (the handle's timeout) and happen in a one-block kernel
// only (the heavy kernels never spin, so they never hold SMs that another
// stream's kernels need); one that runs out records an error in the handle's
// control word (sb_ep_status) and the kernels after it finish with what they
// have.  Every wait is on a flag another rank's kernel raises without waiting
// itself, so no wait depends on a kernel of the same GPU.
//
// No TMA or bulk copy touches peer memory: peer rows move with 16-byte
// loads and stores from the SMs.

#include "common.cuh"

#include <vector>
#include "sm100.cuh"
#include "tree_sum.cuh"

#include <dlfcn.h>
#include <nccl.h>

namespace sb {

constexpr int EP_MAX_WORLD = 8;
constexpr int EP_KE = 16;  // metadata entries per received row (top_k <= 16)
constexpr uint32_t EP_MAGIC = 0x53424550u;
constexpr int EP_THREADS = 256;

// Control block of a handle (device memory, zeroed at create).
struct EpCtrl {
  uint32_t epoch;
  uint32_t done_send;
  uint32_t done_ret;
  uint32_t error;  // bit 0: a dispatch wait ran out; bit 1: a return wait; bit 2: a bad expert id
  uint32_t send_cnt[8];  // rows claimed at each destination by this forward (zeroed after it)
};

// One rank's peer-visible buffer (byte offsets; the same on every rank).
struct EpLayout {
  int64_t dflag, rflag, rcount, meta_e, meta_w, rx, ret, total;
};

inline EpLayout ep_layout(int W, int64_t cap, int64_t H) {
  EpLayout L{};
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o = (int64_t)align_up((size_t)(o + bytes), 4096);
    return at;
  };
  L.dflag = take(4 * EP_MAX_WORLD);   // [W] raised by source s at [s]
  L.rflag = take(4 * EP_MAX_WORLD);   // [W] raised by destination g at [g]
  L.rcount = take(4 * EP_MAX_WORLD);  // [W] rows from source s
  L.meta_e = take((int64_t)W * cap * EP_KE);        // uint8 [W][cap][16]: local expert ids, 0xFF = none
  L.meta_w = take((int64_t)W * cap * EP_KE * 4);    // fp32 [W][cap][16]
  L.rx = take((int64_t)W * cap * H * 2);            // bf16 [W][cap][H]: rows from source s
  L.ret = take((int64_t)W * cap * H * 4);           // fp32 [W][cap][H]: partial sums from destination g
  L.total = o;
  return L;
}

struct EpArgs {
  uint8_t* peer[EP_MAX_WORLD];  // every rank's buffer as mapped here (peer[rank] = own)
  EpLayout L;
  int W, rank, E, El, k;
  int64_t cap, H;
  uint64_t limit_ns;
  EpCtrl* ctrl;
  const int32_t* perm;  // expert id -> position (null: the identity), sb_ep_set_placement
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

// Bounded wait for *flag == epoch.
__device__ bool ep_wait(const uint32_t* flag, uint32_t epoch, uint64_t limit_ns) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    __nanosleep(200);
    if (ld_acquire_sys(flag) == epoch) return true;
    if (globaltimer() - t0 > limit_ns) return false;
  }
}

// Position of the q-th (0-based) set bit of m (q < popc(m)).
__device__ __forceinline__ int nth_bit(unsigned m, int q) {
  for (int i = 0; i < q; ++i) m &= m - 1u;
  return __ffs(m) - 1;
}

__device__ __forceinline__ uint8_t* ep_at(const EpArgs& a, int g, int64_t off) { return a.peer[g] + off; }

// ---------------------------------------------------------------------------
// ep_send: rows and metadata into the destinations' receive buffers
// ---------------------------------------------------------------------------
// The last block to finish (counted in ctrl->*done) runs `last()`.  Each
// block orders its stores before its count with a GPU-scope fence; the last
// block, having seen every count, fences at system scope before `last()`
// raises flags that other GPUs acquire, so every block's stores (peer memory
// included) happen before the flag in the memory model's causality order.
template <typename F>
__device__ __forceinline__ void ep_last_block(uint32_t* done, F last) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      last();
      *done = 0u;
    }
  }
}

__global__ void __launch_bounds__(EP_THREADS) ep_send_kernel(const __nv_bfloat16* __restrict__ x,
                                                             const int32_t* __restrict__ ids,
                                                             const float* __restrict__ wts, int64_t B, EpArgs a,
                                                             int* __restrict__ send_pos) {
  const int lane = threadIdx.x & 31;
  const int n16 = (int)(a.H >> 3);  // 16-byte words per row
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < B;
       t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    // the token's slots: lane j < k holds slot j
    int e = -1;
    float w = 0.f;
    if (lane < a.k) {
      e = __ldg(ids + t * a.k + lane);
      w = wts ? __ldg(wts + t * a.k + lane) : 1.0f;
      if (e < 0 || e >= a.E) {
        atomicOr(&a.ctrl->error, 4u);
        e = -1;
      } else if (a.perm) {
        e = __ldg(a.perm + e);  // the expert's position: rank e / El, local id e % El
      }
    }
    const int dest = e >= 0 ? e / a.El : -1;
    unsigned mask = 0;  // destination ranks of the token
#pragma unroll
    for (int g = 0; g < EP_MAX_WORLD; ++g)
      if (__ballot_sync(0xffffffffu, dest == g)) mask |= 1u << g;
    if (lane < a.W) send_pos[t * a.W + lane] = -1;
    if (!mask) continue;
    // the row, loaded once for all its destinations (rows up to 4096 bf16 in registers)
    const uint4* src = reinterpret_cast<const uint4*>(x + t * a.H);
    const bool small = n16 <= 32 * 8;
    uint4 v[8];
    if (small) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (lane + 32 * u < n16) v[u] = __ldg(src + lane + 32 * u);
    }
    for (unsigned mm = mask; mm; mm &= mm - 1) {
      const int g = __ffs(mm) - 1;
      // this token's row at g: a slot of g's receive segment for this rank
      int pos = 0;
      if (lane == 0) pos = atomicAdd(reinterpret_cast<int*>(&a.ctrl->send_cnt[g]), 1);
      pos = __shfl_sync(0xffffffffu, pos, 0);
      if (lane == 0) send_pos[t * a.W + g] = pos;
      const int64_t row = (int64_t)a.rank * a.cap + pos;
      uint4* dst = reinterpret_cast<uint4*>(ep_at(a, g, a.L.rx) + row * a.H * 2);
      if (small) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (lane + 32 * u < n16) dst[lane + 32 * u] = v[u];
      } else {
        for (int c = lane; c < n16; c += 32) dst[c] = __ldg(src + c);
      }
      // metadata: the token's experts on g, ascending local id (then slot)
      const bool mine = dest == g;
      const int le = mine ? e - g * a.El : 0x7fffffff;
      int rank = 0;
      for (int j = 0; j < a.k; ++j) {
        const int q = __shfl_sync(0xffffffffu, le, j);
        rank += (q < le || (q == le && j < lane)) ? 1 : 0;
      }
      uint32_t byte = 0xFFu;
      float wq = 0.f;
#pragma unroll
      for (int q = 0; q < EP_KE; ++q) {
        const unsigned m = __ballot_sync(0xffffffffu, mine && rank == q);
        const int s = m ? __ffs(m) - 1 : 0;
        const int lq = __shfl_sync(0xffffffffu, le, s);
        const float wv = __shfl_sync(0xffffffffu, w, s);
        if (lane == q && m) {
          byte = (uint32_t)lq;
          wq = wv;
        }
      }
      // lanes 0..3 pack four bytes each; lanes 0..15 store one weight each
      const uint32_t b0 = __shfl_sync(0xffffffffu, byte, (4 * lane) & 31);
      const uint32_t b1 = __shfl_sync(0xffffffffu, byte, (4 * lane + 1) & 31);
      const uint32_t b2 = __shfl_sync(0xffffffffu, byte, (4 * lane + 2) & 31);
      const uint32_t b3 = __shfl_sync(0xffffffffu, byte, (4 * lane + 3) & 31);
      if (lane < 4)
        reinterpret_cast<uint32_t*>(ep_at(a, g, a.L.meta_e) + row * EP_KE)[lane] =
            b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
      if (lane < EP_KE) reinterpret_cast<float*>(ep_at(a, g, a.L.meta_w))[row * EP_KE + lane] = wq;
    }
  }
  ep_last_block(&a.ctrl->done_send, [&] {
    // a new forward: its epoch tags every flag this and the later kernels use
    const uint32_t epoch = a.ctrl->epoch + 1u;
    a.ctrl->epoch = epoch;
    for (int g = 0; g < a.W; ++g)
      reinterpret_cast<int*>(ep_at(a, g, a.L.rcount))[a.rank] = (int)atomicExch(&a.ctrl->send_cnt[g], 0u);
    __threadfence_system();
    for (int g = 0; g < a.W; ++g) st_release_sys(reinterpret_cast<uint32_t*>(ep_at(a, g, a.L.dflag)) + a.rank, epoch);
  });
}

// ---------------------------------------------------------------------------
// ep_wait: one block waits (bounded) until every rank raised its flag of this
// forward; the kernels after it in the stream read what the flags cover, and
// none of the heavy kernels ever spins
// ---------------------------------------------------------------------------
__global__ void ep_wait_kernel(EpArgs a, int64_t flag_off, unsigned err_bit) {
  const int tid = threadIdx.x;
  if (tid < a.W) {
    const uint32_t epoch = ld_volatile(&a.ctrl->epoch);
    if (!ep_wait(reinterpret_cast<const uint32_t*>(a.peer[a.rank] + flag_off) + tid, epoch, a.limit_ns)) {
      atomicOr(&a.ctrl->error, err_bit);
      set_status(ST_TIMEOUT_EP);
    }
  }
}

// ---------------------------------------------------------------------------
// ep_recv_plan: plan the local expert segments
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(PLAN_THREADS) ep_recv_plan_kernel(EpArgs a, int* __restrict__ rcnt,
                                                                    int* __restrict__ counts, int* __restrict__ offsets,
                                                                    int* __restrict__ cursor, MTile* __restrict__ mtiles,
                                                                    int* __restrict__ num_mtiles, int max_mtiles,
                                                                    int tile_rows) {
  extern __shared__ int sh_count[];  // [El]
  __shared__ int srcnt[EP_MAX_WORLD];
  const int tid = threadIdx.x;
  const uint8_t* own = a.peer[a.rank];
  for (int e = tid; e < a.El; e += PLAN_THREADS) sh_count[e] = 0;
  if (tid < a.W) {
    // the counts landed before the flags ep_wait_kernel saw (it ran just before)
    int c = reinterpret_cast<const volatile int*>(own + a.L.rcount)[tid];
    if (c < 0 || c > a.cap) {
      atomicOr(&a.ctrl->error, 4u);
      c = 0;
    }
    if (a.ctrl->error & 1u) c = 0;  // a dispatch wait ran out: nothing usable arrived
    srcnt[tid] = c;
    rcnt[tid] = c;
  }
  __syncthreads();
  const int64_t rows = (int64_t)a.W * a.cap;
  const uint4* me = reinterpret_cast<const uint4*>(own + a.L.meta_e);
  for (int64_t f = tid; f < rows; f += PLAN_THREADS) {
    const int s = (int)(f / a.cap);
    if (f - (int64_t)s * a.cap >= srcnt[s]) continue;
    const uint4 m = me[f];
    const uint32_t wd[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
    for (int q = 0; q < EP_KE; ++q) {
      const int le = (wd[q >> 2] >> (8 * (q & 3))) & 0xFF;
      if (le == 0xFF) break;
      if (le < a.El)
        atomicAdd(&sh_count[le], 1);
      else
        atomicOr(&a.ctrl->error, 4u);
    }
  }
  __syncthreads();
  plan_segments(a.El, [&](int e) { return sh_count[e]; }, true, counts, offsets, cursor, mtiles, num_mtiles,
                max_mtiles, tile_rows);
}

// ---------------------------------------------------------------------------
// ep_recv_scatter: received rows into their experts' segments
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(EP_THREADS) ep_recv_scatter_kernel(EpArgs a, const int* __restrict__ rcnt,
                                                                     const int* __restrict__ offsets,
                                                                     int* __restrict__ cursor,
                                                                     __nv_bfloat16* __restrict__ xp, int64_t ldx,
                                                                     float* __restrict__ row_w, int* __restrict__ inv) {
  const int lane = threadIdx.x & 31;
  const uint8_t* own = a.peer[a.rank];
  const int64_t rows = (int64_t)a.W * a.cap;
  const int n16 = (int)(a.H >> 3);
  for (int64_t f = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; f < rows;
       f += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int s = (int)(f / a.cap);
    if (f - (int64_t)s * a.cap >= __ldg(rcnt + s)) continue;
    const uint4 m = reinterpret_cast<const uint4*>(own + a.L.meta_e)[f];
    const float wl = lane < EP_KE ? reinterpret_cast<const float*>(own + a.L.meta_w)[f * EP_KE + lane] : 0.f;
    const uint32_t wd[4] = {m.x, m.y, m.z, m.w};
    const uint4* src = reinterpret_cast<const uint4*>(own + a.L.rx + f * a.H * 2);
    const bool small = n16 <= 32 * 8;
    uint4 v[8];
    if (small) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (lane + 32 * u < n16) v[u] = src[lane + 32 * u];
    }
#pragma unroll
    for (int q = 0; q < EP_KE; ++q) {
      const int le = (wd[q >> 2] >> (8 * (q & 3))) & 0xFF;
      if (le == 0xFF || le >= a.El) {
        if (lane == 0) inv[f * EP_KE + q] = -1;
        continue;
      }
      int pos = 0;
      if (lane == 0) pos = offsets[le] + atomicAdd(&cursor[le], 1);
      pos = __shfl_sync(0xffffffffu, pos, 0);
      const float w = __shfl_sync(0xffffffffu, wl, q);
      if (lane == 0) {
        inv[f * EP_KE + q] = pos;
        row_w[pos] = w;
      }
      uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)pos * ldx);
      if (small) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (lane + 32 * u < n16) dst[lane + 32 * u] = v[u];
      } else {
        for (int c = lane; c < n16; c += 32) dst[c] = src[c];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// ep_return: per received row, the tree sum of its entries -> source
// ---------------------------------------------------------------------------
template <int KC>
__global__ void __launch_bounds__(EP_THREADS) ep_return_kernel(EpArgs a, const int* __restrict__ rcnt,
                                                               const int* __restrict__ inv,
                                                               const float* __restrict__ yp) {
  const int lane = threadIdx.x & 31;
  const uint8_t* own = a.peer[a.rank];
  const int64_t rows = (int64_t)a.W * a.cap;
  const int n4 = (int)(a.H >> 2);
  for (int64_t f = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; f < rows;
       f += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int s = (int)(f / a.cap);
    const int64_t i = f - (int64_t)s * a.cap;
    if (i >= __ldg(rcnt + s)) continue;
    const uint4 m = reinterpret_cast<const uint4*>(own + a.L.meta_e)[f];
    const uint32_t wd[4] = {m.x, m.y, m.z, m.w};
    int n = 0;
    int lpos[KC];
    int64_t row[KC];
#pragma unroll
    for (int q = 0; q < KC; ++q) {
      const int le = (wd[q >> 2] >> (8 * (q & 3))) & 0xFF;
      const int pr = (le != 0xFF && le < a.El && n == q) ? __ldg(inv + f * EP_KE + q) : -1;
      lpos[q] = le;
      row[q] = pr;
      if (pr >= 0) n = q + 1;
    }
    // entries are stored in ascending local expert id: the positions of the tree
    const TreeSched sched = tree_schedule(n, [&](int q) {
      int v = 0;
#pragma unroll
      for (int j = 0; j < KC; ++j)
        if (j == q) v = lpos[j];
      return v;
    });
    float4* dst = reinterpret_cast<float4*>(ep_at(a, s, a.L.ret) + (((int64_t)a.rank * a.cap + i) * a.H) * 4);
    constexpr int CW = 2;
    for (int cb = 0; cb < n4; cb += 32 * CW) {  // warp-uniform bound
      const int c0 = cb + lane;
      float4 v[KC][CW];
#pragma unroll
      for (int q = 0; q < KC; ++q)
#pragma unroll
        for (int w = 0; w < CW; ++w) {
          const int c = c0 + 32 * w;
          v[q][w] = (q < n && c < n4) ? __ldg(reinterpret_cast<const float4*>(yp + row[q] * a.H) + c)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      tree_apply<KC, CW>(v, sched);
#pragma unroll
      for (int w = 0; w < CW; ++w)
        if (c0 + 32 * w < n4) dst[c0 + 32 * w] = v[0][w];
    }
  }
  ep_last_block(&a.ctrl->done_ret, [&] {
    const uint32_t epoch = ld_volatile(&a.ctrl->epoch);
    for (int g = 0; g < a.W; ++g) st_release_sys(reinterpret_cast<uint32_t*>(ep_at(a, g, a.L.rflag)) + a.rank, epoch);
  });
}

// ---------------------------------------------------------------------------
// ep_combine: per token, the tree sum of its destinations' partial sums
// ---------------------------------------------------------------------------
template <typename TO>
__global__ void __launch_bounds__(EP_THREADS) ep_combine_kernel(EpArgs a, int64_t B, const int* __restrict__ send_pos,
                                                                TO* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const uint8_t* own = a.peer[a.rank];
  const bool ok = (a.ctrl->error & 2u) == 0;  // set by ep_wait_kernel when a return wait ran out
  const int n4 = (int)(a.H >> 2);
  const float* ret = reinterpret_cast<const float*>(own + a.L.ret);
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < B;
       t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int pos = lane < a.W ? __ldg(send_pos + t * a.W + lane) : -1;
    const unsigned vm = __ballot_sync(0xffffffffu, pos >= 0);
    const int n = __popc(vm);
    int gpos[EP_MAX_WORLD];
    int64_t row[EP_MAX_WORLD];
#pragma unroll
    for (int q = 0; q < EP_MAX_WORLD; ++q) {
      const int g = q < n ? nth_bit(vm, q) : 0;
      const int pg = __shfl_sync(0xffffffffu, pos, g);
      gpos[q] = g;
      row[q] = ((int64_t)g * a.cap + (pg < 0 ? 0 : pg)) * a.H;
    }
    const TreeSched sched = tree_schedule(n, [&](int q) {
      int v = 0;
#pragma unroll
      for (int j = 0; j < EP_MAX_WORLD; ++j)
        if (j == q) v = gpos[j];
      return v;
    });
    constexpr int CW = 2;
    for (int cb = 0; cb < n4; cb += 32 * CW) {  // warp-uniform bound: every lane reaches the vote
      const int c0 = cb + lane;
      float4 v[EP_MAX_WORLD][CW];
#pragma unroll
      for (int q = 0; q < EP_MAX_WORLD; ++q)
#pragma unroll
        for (int w = 0; w < CW; ++w) {
          const int c = c0 + 32 * w;
          v[q][w] = (q < n && ok && c < n4) ? reinterpret_cast<const float4*>(ret + row[q])[c]
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      tree_apply<EP_MAX_WORLD, CW>(v, sched);
      bool bad = false;
#pragma unroll
      for (int w = 0; w < CW; ++w)
        bad |= !(isfinite(v[0][w].x) && isfinite(v[0][w].y) && isfinite(v[0][w].z) && isfinite(v[0][w].w));
      if (__any_sync(0xffffffffu, bad) && lane == 0) set_status(ST_RANGE);
#pragma unroll
      for (int w = 0; w < CW; ++w)
        if (c0 + 32 * w < n4) store4<TO>(out + t * a.H + 4 * (c0 + 32 * w), v[0][w]);
    }
  }
}

// Failure injection for tests: one bounded wait on this rank's own dispatch
// flag for a value no rank writes.
__global__ void ep_stale_wait_kernel(EpArgs a) {
  const uint32_t stale = ld_volatile(&a.ctrl->epoch) + 0x40000000u;
  if (!ep_wait(reinterpret_cast<const uint32_t*>(a.peer[a.rank] + a.L.dflag) + a.rank, stale, a.limit_ns)) {
    atomicOr(&a.ctrl->error, 1u);
    set_status(ST_TIMEOUT_EP);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct EpWorkspace {
  int64_t R, Rp, ldx, ldh, max_mt;
  size_t send_pos, rcnt, counts, offsets, cursor, nmt, mtiles, row_w, inv, xp, hp, yp, total;
};

}  // namespace sb

struct sb_ep {
  int device = 0;
  int W = 1, rank = 0, E = 0, El = 0, k = 0;
  int64_t cap = 0, H = 0, I = 0;
  int timeout_ms = 2000;
  sb::EpLayout L{};
  uint8_t* local = nullptr;
  uint8_t* peer[sb::EP_MAX_WORLD] = {};
  bool connected = false;
  sb::EpCtrl* ctrl = nullptr;
  int32_t* perm = nullptr;  // device [E], set by sb_ep_set_placement
};

namespace sb {
namespace {

struct EpHandleBytes {  // what sb_ep_export writes (SB_EP_HANDLE_BYTES)
  uint32_t magic, version;
  int32_t world, rank, n_experts, top_k;
  int64_t cap, hidden, total;
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(EpHandleBytes) <= SB_EP_HANDLE_BYTES, "handle bytes");

EpWorkspace ep_workspace(const sb_ep* h) {
  EpWorkspace w{};
  // every slot of every received row may name an expert of this rank (ids
  // may repeat), so the entries are bounded by k per row
  w.R = (int64_t)h->W * h->cap * h->k;
  w.Rp = w.R + 32 * (int64_t)h->El;
  w.ldx = (h->H + 63) / 64 * 64;
  w.ldh = (h->I + 63) / 64 * 64;
  w.max_mt = w.Rp / 128 + h->El + 1;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 1024);
    return at;
  };
  w.send_pos = take(sizeof(int) * (size_t)h->cap * h->W);
  w.rcnt = take(sizeof(int) * EP_MAX_WORLD);
  w.counts = take(sizeof(int) * h->El);
  w.offsets = take(sizeof(int) * h->El);
  w.cursor = take(sizeof(int) * h->El);
  w.nmt = take(sizeof(int));
  w.mtiles = take(sizeof(MTile) * (size_t)w.max_mt);
  w.row_w = take(sizeof(float) * (size_t)w.Rp);
  w.inv = take(sizeof(int) * (size_t)h->W * h->cap * EP_KE);
  w.xp = take((size_t)w.Rp * w.ldx * 2);
  w.hp = take((size_t)w.Rp * w.ldh * 2);
  w.yp = take((size_t)w.Rp * h->H * 4);
  w.total = o;
  return w;
}

EpArgs ep_args(const sb_ep* h) {
  EpArgs a{};
  for (int g = 0; g < EP_MAX_WORLD; ++g) a.peer[g] = h->peer[g];
  a.L = h->L;
  a.W = h->W;
  a.rank = h->rank;
  a.E = h->E;
  a.El = h->El;
  a.k = h->k;
  a.cap = h->cap;
  a.H = h->H;
  a.limit_ns = (uint64_t)h->timeout_ms * 1000000ull;
  a.ctrl = h->ctrl;
  a.perm = h->perm;
  return a;
}


}  // namespace
}  // namespace sb

extern "C" int sb_ep_create(const sb_ep_desc* d, sb_ep** out) {
  using namespace sb;
  SB_REQUIRE(d && out, "null argument");
  *out = nullptr;
  SB_REQUIRE(d->world >= 1 && d->world <= EP_MAX_WORLD, "world=%d must be 1..%d", d->world, EP_MAX_WORLD);
  SB_REQUIRE(d->rank >= 0 && d->rank < d->world, "rank=%d out of range", d->rank);
  SB_REQUIRE(d->n_experts >= d->world && d->n_experts % d->world == 0,
             "n_experts=%d must be a multiple of world=%d", d->n_experts, d->world);
  SB_REQUIRE(d->n_experts / d->world <= 255, "at most 255 experts per rank");
  SB_REQUIRE(d->top_k >= 1 && d->top_k <= EP_KE, "top_k=%d must be 1..%d", d->top_k, EP_KE);
  SB_REQUIRE(d->max_tokens >= 1 && d->max_tokens <= (1 << 22), "max_tokens=%lld out of range",
             (long long)d->max_tokens);
  SB_REQUIRE(d->hidden > 0 && d->hidden % 8 == 0 && d->hidden <= (1 << 16), "hidden=%lld must be a multiple of 8",
             (long long)d->hidden);
  SB_REQUIRE(d->intermediate > 0 && d->intermediate <= (1 << 20), "intermediate out of range");
  SB_REQUIRE(d->timeout_ms >= 0, "timeout_ms must not be negative");
  const int64_t cap = d->max_tokens;
  SB_REQUIRE((int64_t)d->world * cap * d->top_k < INT32_MAX / 2, "max_tokens too large for the receive planning");
  int device = 0;
  SB_CUDA_TRY(cudaGetDevice(&device));
  sb_ep* h = new sb_ep();
  h->device = device;
  h->W = d->world;
  h->rank = d->rank;
  h->E = d->n_experts;
  h->El = d->n_experts / d->world;
  h->k = d->top_k;
  h->cap = cap;
  h->H = d->hidden;
  h->I = d->intermediate;
  h->timeout_ms = d->timeout_ms ? d->timeout_ms : 2000;
  h->L = ep_layout(h->W, cap, h->H);
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&h->local), (size_t)h->L.total);
  if (e == cudaSuccess) e = cudaMemset(h->local, 0, (size_t)h->L.rx);  // flags, counts and metadata
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&h->ctrl), sizeof(EpCtrl));
  if (e == cudaSuccess) e = cudaMemset(h->ctrl, 0, sizeof(EpCtrl));
  if (e != cudaSuccess) {
    if (h->local) cudaFree(h->local);
    if (h->ctrl) cudaFree(h->ctrl);
    delete h;
    cudaGetLastError();
    return fail(e == cudaErrorMemoryAllocation ? SB_ERR_NOMEM : SB_ERR_CUDA, "sb_ep_create: %s",
                cudaGetErrorString(e));
  }
  h->peer[h->rank] = h->local;
  h->connected = h->W == 1;
  *out = h;
  return SB_OK;
}

extern "C" int sb_ep_export(const sb_ep* h, void* handle) {
  using namespace sb;
  SB_REQUIRE(h && handle, "null argument");
  DeviceGuard dg(h->device);
  EpHandleBytes b{};
  b.magic = EP_MAGIC;
  b.version = SB_ABI_VERSION;
  b.world = h->W;
  b.rank = h->rank;
  b.n_experts = h->E;
  b.top_k = h->k;
  b.cap = h->cap;
  b.hidden = h->H;
  b.total = h->L.total;
  SB_CUDA_TRY(cudaIpcGetMemHandle(&b.ipc, h->local));
  memset(handle, 0, SB_EP_HANDLE_BYTES);
  memcpy(handle, &b, sizeof(b));
  return SB_OK;
}

extern "C" int sb_ep_connect(sb_ep* h, const void* handles) {
  using namespace sb;
  SB_REQUIRE(h && handles, "null argument");
  SB_REQUIRE(!h->connected || h->W == 1, "handle is already connected");
  DeviceGuard dg(h->device);
  const uint8_t* all = static_cast<const uint8_t*>(handles);
  for (int s = 0; s < h->W; ++s) {
    EpHandleBytes b;
    memcpy(&b, all + (size_t)s * SB_EP_HANDLE_BYTES, sizeof(b));
    SB_REQUIRE(b.magic == EP_MAGIC && b.version == SB_ABI_VERSION, "handle %d is not an sb_ep handle", s);
    SB_REQUIRE(b.rank == s && b.world == h->W && b.n_experts == h->E && b.top_k == h->k && b.cap == h->cap &&
                   b.hidden == h->H && b.total == h->L.total,
               "handle %d describes another layer (rank %d, world %d, experts %d, top_k %d, max_tokens %lld, "
               "hidden %lld)",
               s, b.rank, b.world, b.n_experts, b.top_k, (long long)b.cap, (long long)b.hidden);
  }
  for (int s = 0; s < h->W; ++s) {
    if (s == h->rank) continue;
    EpHandleBytes b;
    memcpy(&b, all + (size_t)s * SB_EP_HANDLE_BYTES, sizeof(b));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, b.ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < s; ++j)
        if (j != h->rank && h->peer[j]) {
          cudaIpcCloseMemHandle(h->peer[j]);
          h->peer[j] = nullptr;
        }
      return fail(SB_ERR_CUDA, "cudaIpcOpenMemHandle of rank %d failed: %s", s, cudaGetErrorString(e));
    }
    h->peer[s] = static_cast<uint8_t*>(p);
  }
  h->connected = true;
  return SB_OK;
}

// NCCL is loaded at run time (the process that calls these has it already: a
// torch process maps libnccl.so.2), so the library itself has no link-time
// dependency on it.
namespace sb {
namespace {
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};
const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW);
    if (!lib) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(lib, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(lib, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(lib, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.error_string;
  });
  return api;
}
}  // namespace
}  // namespace sb

#define SB_NCCL_TRY(expr)                                                                                 \
  do {                                                                                                    \
    const ncclResult_t _r = (expr);                                                                       \
    if (_r != ncclSuccess) return ::sb::fail(SB_ERR_CUDA, "%s failed: %s", #expr, api.error_string(_r)); \
  } while (0)

extern "C" int sb_nccl_unique_id(void* id) {
  using namespace sb;
  SB_REQUIRE(id, "null argument");
  const NcclApi& api = nccl();
  if (!api.ok) return fail(SB_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  SB_NCCL_TRY(api.get_unique_id(&u));
  memcpy(id, &u, sizeof(u));
  return SB_OK;
}

extern "C" int sb_nccl_comm_init(int nranks, int rank, const void* id, void** comm) {
  using namespace sb;
  SB_REQUIRE(id && comm && nranks >= 1 && rank >= 0 && rank < nranks, "bad argument");
  const NcclApi& api = nccl();
  if (!api.ok) return fail(SB_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  SB_NCCL_TRY(api.comm_init_rank(&c, nranks, u, rank));
  *comm = c;
  return SB_OK;
}

extern "C" int sb_nccl_comm_destroy(void* comm) {
  using namespace sb;
  if (!comm) return SB_OK;
  const NcclApi& api = nccl();
  if (!api.ok) return fail(SB_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  SB_NCCL_TRY(api.comm_destroy(static_cast<ncclComm_t>(comm)));
  return SB_OK;
}

extern "C" int sb_ep_connect_nccl(sb_ep* h, void* comm, void* stream) {
  using namespace sb;
  SB_REQUIRE(h && comm, "null argument");
  const NcclApi& api = nccl();
  if (!api.ok) return fail(SB_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  DeviceGuard dg(h->device);
  std::vector<uint8_t> mine(SB_EP_HANDLE_BYTES), all((size_t)h->W * SB_EP_HANDLE_BYTES);
  int rc;
  if ((rc = sb_ep_export(h, mine.data()))) return rc;
  uint8_t* dbuf = nullptr;
  SB_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&dbuf), (size_t)(h->W + 1) * SB_EP_HANDLE_BYTES));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(dbuf, mine.data(), SB_EP_HANDLE_BYTES, cudaMemcpyHostToDevice, st);
  ncclResult_t r = ncclSuccess;
  if (e == cudaSuccess)
    r = api.all_gather(dbuf, dbuf + SB_EP_HANDLE_BYTES, SB_EP_HANDLE_BYTES, ncclUint8,
                       static_cast<ncclComm_t>(comm), st);
  if (e == cudaSuccess && r == ncclSuccess)
    e = cudaMemcpyAsync(all.data(), dbuf + SB_EP_HANDLE_BYTES, all.size(), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && r == ncclSuccess) e = cudaStreamSynchronize(st);
  cudaFree(dbuf);
  if (r != ncclSuccess) return fail(SB_ERR_CUDA, "ncclAllGather of the handles failed: %s", api.error_string(r));
  if (e != cudaSuccess) return fail(SB_ERR_CUDA, "handle exchange failed: %s", cudaGetErrorString(e));
  return sb_ep_connect(h, all.data());
}

extern "C" size_t sb_ep_workspace_bytes(const sb_ep* h) { return h ? sb::ep_workspace(h).total : 0; }

extern "C" int sb_ep_forward(sb_ep* h, const void* x, int x_dtype, int64_t batch, const int32_t* ids,
                             const float* weights, const uint32_t* gate, const uint32_t* up, const uint32_t* down,
                             const float* gate_scale, const float* up_scale, const float* down_scale, void* out,
                             int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sb;
  SB_REQUIRE(h, "null handle");
  SB_REQUIRE(h->connected, "sb_ep_connect has not run");
  SB_REQUIRE(x_dtype == SB_BF16, "the expert-parallel layer takes bf16 activations");
  SB_REQUIRE(out_dtype == SB_F32 || out_dtype == SB_BF16, "out dtype must be SB_F32 or SB_BF16");
  SB_REQUIRE(batch >= 0 && batch <= h->cap, "batch=%lld exceeds max_tokens=%lld", (long long)batch,
             (long long)h->cap);
  SB_REQUIRE(gate && up && down && gate_scale && up_scale && down_scale, "null expert weights");
  SB_REQUIRE(batch == 0 || (x && ids && out), "null pointer argument");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
             "x and out must be 16-byte aligned");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(gate) & 15u) == 0 && (reinterpret_cast<uintptr_t>(up) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(down) & 15u) == 0,
             "packed weights must be 16-byte aligned");
  SB_REQUIRE(h->H % 4 == 0, "hidden must be a multiple of 4");
  const EpWorkspace w = ep_workspace(h);
  if (!workspace || workspace_bytes < w.total)
    return fail(SB_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, w.total);
  SB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023u) == 0, "workspace must be 1024-byte aligned");
  DeviceGuard dg(h->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* send_pos = reinterpret_cast<int*>(ws + w.send_pos);
  int* rcnt = reinterpret_cast<int*>(ws + w.rcnt);
  int* counts = reinterpret_cast<int*>(ws + w.counts);
  int* offsets = reinterpret_cast<int*>(ws + w.offsets);
  int* cursor = reinterpret_cast<int*>(ws + w.cursor);
  int* nmt = reinterpret_cast<int*>(ws + w.nmt);
  MTile* mtiles = reinterpret_cast<MTile*>(ws + w.mtiles);
  float* row_w = reinterpret_cast<float*>(ws + w.row_w);
  int* inv = reinterpret_cast<int*>(ws + w.inv);
  __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(ws + w.xp);
  __half* hp = reinterpret_cast<__half*>(ws + w.hp);
  float* yp = reinterpret_cast<float*>(ws + w.yp);
  const EpArgs a = ep_args(h);
  const int sms = num_sms();
  int engine = ternary_engine();
  if (engine == ENGINE_PAIR && (h->H % 4) != 0) engine = ENGINE_TS;
  const int tile_rows = engine == ENGINE_PAIR ? TP_TILE_ROWS : 128;
  {
    ProfScope prof("ep_send", st);
    int64_t blocks = (batch * 32 + EP_THREADS - 1) / EP_THREADS;
    if (blocks > (int64_t)sms * 4) blocks = (int64_t)sms * 4;
    if (blocks < 1) blocks = 1;
    ep_send_kernel<<<(unsigned)blocks, EP_THREADS, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ids, weights,
                                                             batch, a, send_pos);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ep_wait_dispatch", st);
    ep_wait_kernel<<<1, 32, 0, st>>>(a, h->L.dflag, 1u);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ep_recv_plan", st);
    ep_recv_plan_kernel<<<1, PLAN_THREADS, sizeof(int) * h->El, st>>>(
        a, rcnt, counts, offsets, cursor, mtiles, nmt, (int)w.max_mt, tile_rows);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ep_recv_scatter", st);
    int64_t blocks = ((int64_t)h->W * h->cap * 32 + EP_THREADS - 1) / EP_THREADS;
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    ep_recv_scatter_kernel<<<(unsigned)blocks, EP_THREADS, 0, st>>>(a, rcnt, offsets, cursor, xp, w.ldx, row_w, inv);
    SB_CUDA_TRY(cudaGetLastError());
  }
  int rc;
  GroupedSwiGLU g{xp, hp, yp, w.Rp, w.ldx, w.ldh, h->H, h->I, h->El, mtiles, nmt, row_w,
                  gate, up, down, gate_scale, up_scale, down_scale, 1, engine};
  if ((rc = grouped_swiglu(g, st))) return rc;
  {
    ProfScope prof("ep_return", st);
    int64_t blocks = ((int64_t)h->W * h->cap * 32 + EP_THREADS - 1) / EP_THREADS;
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    if (h->k <= 8)
      ep_return_kernel<8><<<(unsigned)blocks, EP_THREADS, 0, st>>>(a, rcnt, inv, yp);
    else
      ep_return_kernel<16><<<(unsigned)blocks, EP_THREADS, 0, st>>>(a, rcnt, inv, yp);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ep_wait_return", st);
    ep_wait_kernel<<<1, 32, 0, st>>>(a, h->L.rflag, 2u);
    SB_CUDA_TRY(cudaGetLastError());
  }
  {
    ProfScope prof("ep_combine", st);
    int64_t blocks = (batch * 32 + EP_THREADS - 1) / EP_THREADS;
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    if (blocks < 1) blocks = 1;
    if (out_dtype == SB_F32)
      ep_combine_kernel<float><<<(unsigned)blocks, EP_THREADS, 0, st>>>(a, batch, send_pos, static_cast<float*>(out));
    else
      ep_combine_kernel<__nv_bfloat16><<<(unsigned)blocks, EP_THREADS, 0, st>>>(
          a, batch, send_pos, static_cast<__nv_bfloat16*>(out));
    SB_CUDA_TRY(cudaGetLastError());
  }
  return SB_OK;
}

extern "C" int sb_ep_status(sb_ep* h) {
  using namespace sb;
  SB_REQUIRE(h, "null handle");
  DeviceGuard dg(h->device);
  EpCtrl c{};
  SB_CUDA_TRY(cudaMemcpy(&c, h->ctrl, sizeof(c), cudaMemcpyDeviceToHost));
  if (c.error & 3u)
    return fail(SB_ERR_DEVICE_TIMEOUT,
                "expert-parallel exchange: a wait for a peer ran out (%s%s); the handle must be re-created",
                (c.error & 1u) ? "dispatch" : "", (c.error & 2u) ? " return" : "");
  if (c.error & 4u) return fail(SB_ERR_INVALID, "expert-parallel layer: an expert id or row count was out of range");
  return SB_OK;
}

extern "C" int sb_ep_inject_stale_wait(sb_ep* h, void* stream) {
  using namespace sb;
  SB_REQUIRE(h, "null handle");
  DeviceGuard dg(h->device);
  ep_stale_wait_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ep_args(h));
  SB_CUDA_TRY(cudaGetLastError());
  return SB_OK;
}

extern "C" int sb_ep_destroy(sb_ep* h) {
  using namespace sb;
  if (!h) return SB_OK;
  {
    DeviceGuard dg(h->device);
    for (int g = 0; g < EP_MAX_WORLD; ++g)
      if (g != h->rank && h->peer[g]) cudaIpcCloseMemHandle(h->peer[g]);
    if (h->local) cudaFree(h->local);
    if (h->ctrl) cudaFree(h->ctrl);
    if (h->perm) cudaFree(h->perm);
  }
  delete h;
  return SB_OK;
}

extern "C" int sb_ep_set_placement(sb_ep* h, const int32_t* perm) {
  using namespace sb;
  SB_REQUIRE(h, "null handle");
  DeviceGuard dg(h->device);
  if (!perm) {  // back to the identity
    if (h->perm) SB_CUDA_TRY(cudaFree(h->perm));
    h->perm = nullptr;
    return SB_OK;
  }
  std::vector<char> seen((size_t)h->E, 0);
  for (int e = 0; e < h->E; ++e) {
    SB_REQUIRE(perm[e] >= 0 && perm[e] < h->E && !seen[(size_t)perm[e]],
               "placement must be a permutation of [0, %d): entry %d is %d", h->E, e, perm[e]);
    seen[(size_t)perm[e]] = 1;
  }
  if (!h->perm) SB_CUDA_TRY(cudaMalloc(&h->perm, sizeof(int32_t) * (size_t)h->E));
  SB_CUDA_TRY(cudaMemcpy(h->perm, perm, sizeof(int32_t) * (size_t)h->E, cudaMemcpyHostToDevice));
  return SB_OK;
}
