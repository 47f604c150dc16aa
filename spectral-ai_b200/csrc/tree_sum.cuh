// tree_sum.cuh — the summation order of a token's expert outputs.
//
// A token's k weighted expert outputs are summed along a binary tree over the
// expert index space: two partial sums are added exactly where their experts'
// indices first differ, deepest bit first.  Because the tree is fixed by the
// expert indices alone, any aligned block of experts (the experts one GPU holds
// in the expert-parallel layer, E/W of them with E/W a power of two) is a
// subtree: summing each block on its own GPU and then the block sums at the
// token's GPU gives the same fp32 additions, in the same grouping, as summing
// everything on one GPU.  That is what makes the sharded layer equal the
// single-GPU layer bit for bit at every world size.  (The reference adds the
// slots in slot order, python/olmoe_extract.py:146-155; any order is the
// same sum up to fp32 rounding.)
//
// The tree is evaluated with a stack over the positions in ascending order:
// the boundary between neighbours p and q sits at level msb(p ^ q) (-1 for equal
// positions); a subtree whose left boundary is deeper than the next boundary
// joins its left neighbour first.  Each merge adds two values in place
// (fp32 addition is commutative, so only the grouping matters).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sb {

constexpr int TREE_MAX = 16;  // values per tree

// Merge schedule over n values held in ascending position order: up to n - 1
// merges "v[dst] += v[src]" (one byte each, dst << 4 | src), in s0 (merges 0..7)
// and s1 (8..14).
struct TreeSched {
  uint64_t s0 = 0, s1 = 0;
  int nm = 0;
};

__device__ __forceinline__ int tree_level(int p, int q) { return p == q ? -1 : 31 - __clz(p ^ q); }

// `pos(i)` returns the i-th position (ascending).  All lanes that call this
// with the same positions get the same schedule.
template <typename PosFn>
__device__ __forceinline__ TreeSched tree_schedule(int n, PosFn pos) {
  TreeSched s;
  int st[TREE_MAX], sd[TREE_MAX];
  int sp = 0, prev = 0;
  auto emit = [&](int dst, int src) {
    const uint64_t code = (uint64_t)((dst << 4) | src);
    if (s.nm < 8)
      s.s0 |= code << (8 * s.nm);
    else
      s.s1 |= code << (8 * (s.nm - 8));
    ++s.nm;
  };
  for (int i = 0; i < n; ++i) {
    const int p = pos(i);
    const int d = i == 0 ? 0x7fffffff : tree_level(prev, p);
    while (sp >= 2 && sd[sp - 1] < d) {
      emit(st[sp - 2], st[sp - 1]);
      --sp;
    }
    st[sp] = i;
    sd[sp] = d;
    ++sp;
    prev = p;
  }
  while (sp >= 2) {
    emit(st[sp - 2], st[sp - 1]);
    --sp;
  }
  return s;
}

__device__ __forceinline__ int tree_code(const TreeSched& s, int m) {
  return (int)(((m < 8 ? s.s0 >> (8 * m) : s.s1 >> (8 * (m - 8)))) & 0xFFu);
}

// One merge v[d] += v[s] of the code dst * NV + src, found by a binary search
// over the code range with compile-time indices at the leaves (the code is the
// same in every lane, so the branches never diverge and the values stay in
// registers).  CW column groups share the dispatch.
template <int NV, int CW, int LO, int HI>
__device__ __forceinline__ void tree_merge(float4 (&v)[NV][CW], int code) {
  if constexpr (HI - LO == 1) {
    constexpr int d = LO / NV, s = LO % NV;
    if constexpr (d < s) {
#pragma unroll
      for (int c = 0; c < CW; ++c) {
        v[d][c].x += v[s][c].x;
        v[d][c].y += v[s][c].y;
        v[d][c].z += v[s][c].z;
        v[d][c].w += v[s][c].w;
      }
    }
  } else {
    constexpr int MID = (LO + HI) / 2;
    if (code < MID)
      tree_merge<NV, CW, LO, MID>(v, code);
    else
      tree_merge<NV, CW, MID, HI>(v, code);
  }
}

// Applies the schedule to NV values of CW column groups (NV >= the tree's
// size; values past it are never read); the sums end in v[0][*].
template <int NV, int CW>
__device__ __forceinline__ void tree_apply(float4 (&v)[NV][CW], const TreeSched& s) {
#pragma unroll 1
  for (int m = 0; m < s.nm; ++m) {
    const int code = tree_code(s, m);
    tree_merge<NV, CW, 0, NV * NV>(v, (code >> 4) * NV + (code & 15));
  }
}

// A warp's k entries (lane j < n holds entry j with position `p` and a payload
// `idx`) in ascending (position, lane) order: every lane gets the sorted
// payloads (4 bits each, order[i] = lane of the i-th entry) and the tree
// schedule.  n <= 16.
struct WarpTree {
  uint64_t order = 0;
  TreeSched sched;
  int n = 0;
};

__device__ __forceinline__ WarpTree warp_tree(int p, int n) {
  const int lane = threadIdx.x & 31;
  WarpTree w;
  w.n = n;
  // rank of this lane's entry among the n entries
  int rank = 0;
  for (int j = 0; j < n; ++j) {
    const int q = __shfl_sync(0xffffffffu, p, j);
    rank += (q < p || (q == p && j < lane)) ? 1 : 0;
  }
  int sorted_pos[TREE_MAX];
#pragma unroll
  for (int r = 0; r < TREE_MAX; ++r) {
    if (r < n) {  // n is the same in every lane
      const unsigned m = __ballot_sync(0xffffffffu, lane < n && rank == r);
      const int src = __ffs(m) - 1;
      sorted_pos[r] = __shfl_sync(0xffffffffu, p, src);
      w.order |= (uint64_t)src << (4 * r);
    }
  }
  w.sched = tree_schedule(n, [&](int i) { return sorted_pos[i]; });
  return w;
}

__device__ __forceinline__ int tree_order(const WarpTree& w, int r) { return (int)((w.order >> (4 * r)) & 15u); }

}  // namespace sb
