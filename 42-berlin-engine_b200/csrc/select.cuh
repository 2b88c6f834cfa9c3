// select.cuh -- device pieces of the reference's top-K selection shared by
// the decode step's linear-mode selection and the isolated LSH attention:
// the BF16 dot in simd_dot_bf16_f32's order and the exact heap_push replay.
#pragma once
#include <cfloat>
#include <cstdint>

#include "ec_internal.cuh"

namespace ec {

__device__ __forceinline__ float dot_bf16_ref(const uint16_t* a, const float* b, int n) {
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; l++) acc[l] = 0.0f;
  int i = 0;
  for (; i + 7 < n; i += 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(a + i);
    float w[8];
    dec_bf16x2(u.x, w);
    dec_bf16x2(u.y, w + 2);
    dec_bf16x2(u.z, w + 4);
    dec_bf16x2(u.w, w + 6);
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = __fmaf_rn(w[l], b[i + l], acc[l]);
  }
  float s = __fadd_rn(0.0f, hsum8(acc));
  for (; i < n; i++) s = __fmaf_rn(bf16_to_f32(a[i]), b[i], s);
  return s;
}

// Exact replay of heap_push (ops_heap.h:40-100): a min-heap of at most `cap`
// entries; while not full a value is appended at position size+1 and sifted
// up past every ancestor strictly greater than it; once full, a value
// strictly greater than the root replaces it and is sifted down (the left
// child unless the right one is strictly smaller, while that child is
// strictly smaller than the value).  The result, in the reference's heap
// array order, is the index half of hp[1 .. size].
//
// Nodes are packed (score bits, index) pairs, 1-based, so a sibling pair is
// one 16-byte load; positions beyond `size` hold +inf, so a sift-down of
// fixed depth D (2^D > cap) needs no bound checks: an +inf child is never
// taken.  One warp: a ballot skips every candidate that cannot beat the
// current root (the root only grows), lane 0 runs the operations.
__device__ __forceinline__ void hnode_up(uint2* hp, int n, float v, int vi) {
  while (n > 1) {
    const int p = n >> 1;
    const uint2 pn = hp[p];
    if (__uint_as_float(pn.x) <= v) break;
    hp[n] = pn;
    n = p;
  }
  hp[n] = make_uint2(__float_as_uint(v), (unsigned)vi);
}

template <int D>
__device__ __forceinline__ void hnode_down(uint2* hp, float v, int vi) {
  int n = 1;
  bool go = true;
#pragma unroll
  for (int lv = 0; lv < D; lv++) {
    const int l = 2 * n;
    const uint4 pr = *reinterpret_cast<const uint4*>(hp + l);
    const bool right = __uint_as_float(pr.z) < __uint_as_float(pr.x);
    const uint2 cn = right ? make_uint2(pr.z, pr.w) : make_uint2(pr.x, pr.y);
    go = go && (__uint_as_float(cn.x) < v);
    if (go) {
      hp[n] = cn;
      n = l + right;
    }
  }
  hp[n] = make_uint2(__float_as_uint(v), (unsigned)vi);
}

// The same two operations run by a whole warp, for heaps of at most 511
// nodes (D <= 9): the path an operation walks is found in parallel, then
// every node on it moves in one store.
//   up: lane k loads the (k+1)-th ancestor of position n; the ancestors
//   before the first one that is not greater than v each move one level
//   down, and v lands above them.
//   down: lane i knows which child node i + 1 would send down (the left one
//   unless the right is strictly smaller); the path from the root follows
//   those choices; its nodes before the first one not smaller than v each
//   move one level up, and v lands below them.
// Both are heap_push's sift loops, step for step.  The caller __syncwarp()s
// between operations.
__device__ __forceinline__ void warp_heap_up(uint2* hp, int n, float v, int vi, int lane) {
  const int a = n >> (lane + 1);  // this lane's ancestor (0: none)
  const uint2 an = a >= 1 ? hp[a] : make_uint2(0u, 0u);
  const unsigned gt = __ballot_sync(0xffffffffu, a >= 1 && !(__uint_as_float(an.x) <= v));
  const int s = __ffs(~gt) - 1;  // ancestors that move down: up to the first that stays
  if (lane < s) hp[n >> lane] = an;
  if (lane == s) hp[n >> s] = make_uint2(__float_as_uint(v), (unsigned)vi);
}

// Returns the new root value.  Heaps of up to 2^D - 1 nodes, D <= 9: lanes
// 0..30 settle the child choices of levels 0..4 (nodes 1..31) and a shuffle
// chase walks them; below level 5 the path's subtree (levels 5..D-2, at most
// 7 internal nodes) is settled the same way and walked on.
template <int D>
__device__ __forceinline__ float warp_heap_down(uint2* hp, float v, int vi, int lane) {
  static_assert(D >= 6 && D <= 9, "warp_heap_down: 6 <= D <= 9");
  // node m's chosen child: the left one unless the right is strictly smaller
  auto choose = [&](int m, unsigned& cx, unsigned& cy, int& cpos) {
    const uint4 pr = *reinterpret_cast<const uint4*>(hp + 2 * m);
    const bool right = __uint_as_float(pr.z) < __uint_as_float(pr.x);
    cx = right ? pr.z : pr.x;
    cy = right ? pr.w : pr.y;
    cpos = 2 * m + (right ? 1 : 0);
  };
  unsigned ax, ay, bx = 0, by = 0;
  int apos, bpos = 0;
  choose(lane + 1, ax, ay, apos);  // levels 0..4 (lane 31: node 32, unused)
  // the path p_0 = 1, p_{k+1} = chosen child of p_k; lane k keeps p_k
  int p = 1, mine = 1;
#pragma unroll
  for (int k = 1; k <= 5; k++) {
    p = __shfl_sync(0xffffffffu, apos, p - 1);
    if (lane == k) mine = p;
  }
  constexpr int kDeep = D - 6;  // path steps below level 5
  int sub0 = 0;
  if constexpr (kDeep > 0) {
    // subtree of p_5: lane i < 2^kDeep - 1 takes its i-th internal node in
    // level order (p5; 2p5, 2p5+1; 4p5 .. 4p5+3)
    sub0 = p;
    const int lvl = 31 - __clz(lane + 1);  // 0, 1, 1, 2, 2, 2, 2
    const int node = (p << lvl) + (lane + 1 - (1 << lvl));
    if (lane < (1 << kDeep) - 1) choose(node, bx, by, bpos);
#pragma unroll
    for (int k = 6; k <= 5 + kDeep; k++) {
      const int l = k - 6;  // level of p_{k-1} inside the subtree
      p = __shfl_sync(0xffffffffu, bpos, (1 << l) - 1 + (p - (sub0 << l)));
      if (lane == k) mine = p;
    }
  }
  // lane k (k < D - 1): the node p_{k+1} (child of p_k), from the lane that
  // settled p_k
  constexpr int kSteps = D - 1;
  int src = 0;
  bool deep = false;
  if (lane < 5) {
    src = mine - 1;
  } else if (lane < kSteps) {
    const int l = lane - 5;
    src = (1 << l) - 1 + (mine - (sub0 << l));
    deep = true;
  }
  const unsigned kxa = __shfl_sync(0xffffffffu, ax, src);
  const unsigned kya = __shfl_sync(0xffffffffu, ay, src);
  const unsigned kxb = __shfl_sync(0xffffffffu, bx, src);
  const unsigned kyb = __shfl_sync(0xffffffffu, by, src);
  const unsigned kx = deep ? kxb : kxa, ky = deep ? kyb : kya;
  const unsigned lt = __ballot_sync(0xffffffffu, lane < kSteps && __uint_as_float(kx) < v);
  const int s = __ffs(~lt) - 1;  // path nodes that move up: up to the first that stays
  if (lane < s) hp[mine] = make_uint2(kx, ky);
  if (lane == s) hp[mine] = make_uint2(__float_as_uint(v), (unsigned)vi);
  const unsigned r0 = __shfl_sync(0xffffffffu, kx, 0);
  return s >= 1 ? __uint_as_float(r0) : v;
}

// hp holds 2^(D+1) nodes.  `ready(j)` (whole warp, j non-decreasing) returns
// once score[0..j] may be read, or false to give up.  idx == nullptr:
// candidate i carries index i + idx_base.  Candidates go by windows of 32: a
// ballot against the root at the window's start drops those that cannot be
// taken (the root only grows); the rest run in order -- by the whole warp
// for 6 <= D <= 9, by lane 0 otherwise.
template <int D, typename Ready>
__device__ int warp_heap_select(const float* score, const int* idx, int idx_base, int n, int cap,
                                uint2* hp, int lane, Ready ready) {
  for (int i = lane; i < (2 << D); i += 32) hp[i] = make_uint2(0x7F800000u, 0u);
  __syncwarp();
  if (cap <= 0) return 0;
  int size = 0;      // lane 0's copy is authoritative; broadcast per window
  float root = 0.0f;
  for (int base = 0; base < n; base += 32) {
    if (!ready(min(base + 31, n - 1))) return 0;
    const int i = base + lane;
    const bool full = size >= cap;
    const float sv = i < n ? score[i] : 0.0f;
    unsigned pend = __ballot_sync(0xffffffffu, i < n && (!full || sv > root));
    if constexpr (D >= 6 && D <= 9) {
      // every lane runs every operation (pend, size and root are uniform)
      while (pend) {
        const int k = base + __ffs(pend) - 1;
        pend &= pend - 1;
        const float v = __shfl_sync(0xffffffffu, sv, k - base);
        const int vi = idx ? idx[k] : k + idx_base;
        if (size < cap) {
          warp_heap_up(hp, ++size, v, vi, lane);
          __syncwarp();
          if (size == cap) root = __uint_as_float(hp[1].x);
        } else if (v > root) {
          root = warp_heap_down<D>(hp, v, vi, lane);
          __syncwarp();
        }
      }
    } else {
      if (lane == 0) {
        while (pend) {
          const int k = base + __ffs(pend) - 1;
          pend &= pend - 1;
          const float v = score[k];
          const int vi = idx ? idx[k] : k + idx_base;
          if (size < cap) {
            hnode_up(hp, ++size, v, vi);
            if (size == cap) root = __uint_as_float(hp[1].x);
          } else if (v > root) {
            hnode_down<D>(hp, v, vi);
            root = __uint_as_float(hp[1].x);
          }
        }
      }
      size = __shfl_sync(0xffffffffu, size, 0);
      root = __shfl_sync(0xffffffffu, root, 0);
    }
    __syncwarp();
  }
  return size;
}

}  // namespace ec
