// topk.cuh -- the reference's top-k selection (route.cu, router.cu): the std::partial_sort
// procedure of GNU libstdc++ restated for one token, and a warp's fast path for it.
#pragma once
#include <cstdint>

namespace uaii_b200 {
namespace {

// The reference ranks experts with std::partial_sort over (prob, index) pairs
// and the comparator a.prob > b.prob (transformer.cpp:564-570).  Equal
// probabilities are ordered by the procedure of the reference's standard
// library (GNU libstdc++): a binary heap over the first k pairs, each later
// pair replacing the root only when strictly greater, then a heap sort.  The
// same procedure is restated in the CPU oracle and pinned there against the
// reference build on tie-heavy inputs, so selection and order match the
// reference exactly, ties included.
struct Pair {
  float p;
  int e;
};
__device__ __forceinline__ bool before(const Pair& a, const Pair& b) { return a.p > b.p; }

__device__ void push_heap(Pair* h, int hole, int top, Pair v) {
  int parent = (hole - 1) / 2;
  while (hole > top && before(h[parent], v)) {
    h[hole] = h[parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  h[hole] = v;
}

__device__ void adjust_heap(Pair* h, int hole, int len, Pair v) {
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (before(h[child], h[child - 1])) child--;
    h[hole] = h[child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    h[hole] = h[child - 1];
    hole = child - 1;
  }
  push_heap(h, hole, top, v);
}

// The reference procedure for one token, serially: a heap over the first k
// pairs, each later pair replacing the root only when strictly greater, then a
// heap sort.  Writes the k ranked pairs to h.
__device__ void topk_heap(const float* __restrict__ row, int64_t E, int k, Pair* h) {
  for (int i = 0; i < k; ++i) h[i] = Pair{row[i], i};
  if (k >= 2)
    for (int parent = (k - 2) / 2;; --parent) {
      adjust_heap(h, parent, k, h[parent]);
      if (parent == 0) break;
    }
  for (int64_t i = k; i < E; ++i) {
    const Pair v{row[i], (int)i};
    if (before(v, h[0])) adjust_heap(h, 0, k, v);  // the displaced root leaves the selection
  }
  for (int last = k; last > 1;) {
    --last;
    const Pair v = h[last];
    h[last] = h[0];
    adjust_heap(h, 0, last, v);
  }
}

// One warp, one token: the k largest scores of `row` (E <= 1024, k <= 32) ranked into h
// (shared memory, k + 1 entries).  The warp extracts the k + 1 largest scores one at a time
// (warp arg-max rounds).  When those values are all distinct the reference's result is fixed
// -- the k largest in descending order -- and the rounds give it; any tie among them
// (selection or order then depend on the heap procedure) hands the token to lane 0, which runs
// the reference procedure itself.  Returns with h valid for every lane (after a __syncwarp).
__device__ __forceinline__ void warp_topk(const float* __restrict__ row, int64_t E, int k, Pair* h, int lane) {
  const int rounds = k < E ? k + 1 : k;
  uint32_t taken = 0;  // bit j: element lane + 32j already extracted
  bool tie = false;
  for (int r = 0; r < rounds; ++r) {
    float bv = 0.0f;
    int be = -1;
    for (int64_t e = lane, j = 0; e < E; e += 32, ++j) {
      const float v = row[e];
      if (!((taken >> j) & 1u) && (be < 0 || v > bv)) { bv = v; be = (int)e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // larger value wins; equal values: smaller index
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be))) { bv = ov; be = oe; }
    }
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    if (r > 0 && !(h[r - 1].p != bv)) tie = true;  // equal (or unordered) neighbours
    __syncwarp();
    if (lane == 0) h[r] = Pair{bv, be};
    __syncwarp();
  }
  if (tie) {
    if (lane == 0) topk_heap(row, E, k, h);
    __syncwarp();
  }
}

}  // namespace
}  // namespace uaii_b200
