// Exact top-k selection inside one CTA under the canonical tie rule.
//
// Items are (key32, idx32) pairs produced by a functor; key32 is an ordered score key
// (sva::ordered_key) and key32 == 0 marks an item that is not a candidate.  The selection
// order is the 64-bit composite  (key32 << 32) | ~idx32  taken in descending order, i.e.
// score descending, then key index ascending -- the rule the CPU oracle applies to every
// torch.topk of the reference (sva/llama.py:278, :295, :100, :113).
//
// The select is an MSB-first radix select with 8-bit digits.  Each level makes one pass over
// the items (a functor call per item, so the items may live in shared memory or be recomputed
// from global memory), builds a 256-bin histogram of the digit among items that still match
// the prefix, and fixes one digit.  It stops as soon as the boundary bin holds exactly the
// number of items still needed.  An item is selected iff key32 != 0 and
// (composite & mask) >= prefix.
#pragma once

#include "sva_common.cuh"

namespace sva {

struct SelectThreshold {
  unsigned long long prefix;
  unsigned long long mask;
};

__device__ __forceinline__ unsigned long long composite(uint32_t key, uint32_t idx) {
  return (static_cast<unsigned long long>(key) << 32) | static_cast<unsigned long long>(~idx);
}

__device__ __forceinline__ bool is_selected(const SelectThreshold& t, uint32_t key, uint32_t idx) {
  return key != 0u && (composite(key, idx) & t.mask) >= t.prefix;
}

// Shared scratch for cta_radix_select: 256-bin histogram plus a few broadcast slots.
struct SelectScratch {
  uint32_t hist[256];
  int warp_tot[9];
  int digit;
  int above;
  int count;
};

// Requires blockDim.x >= 256 and a multiple of 32.  `k` must not exceed the number of items
// with key32 != 0.  All threads of the block must call it.
template <class ItemFn>
__device__ SelectThreshold cta_radix_select(const ItemFn& item, int n, int k, SelectScratch* sc) {
  SelectThreshold thr;
  thr.prefix = 0ull;
  thr.mask = 0ull;
  if (k <= 0) {
    thr.prefix = ~0ull;  // selects nothing: (c & 0) >= ~0 is false
    thr.mask = 0ull;
    return thr;
  }
  int remaining = k;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  for (int level = 0; level < 8; ++level) {
    const int shift = 56 - 8 * level;
    for (int b = tid; b < 256; b += blockDim.x) sc->hist[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      uint32_t key, idx;
      item(i, key, idx);
      if (key == 0u) continue;
      unsigned long long c = composite(key, idx);
      if ((c & thr.mask) != thr.prefix) continue;
      atomicAdd(&sc->hist[(c >> shift) & 0xFFull], 1u);
    }
    __syncthreads();
    // Descending suffix scan over the 256 digits with warps 0..7 (thread t owns digit 255-t):
    // the owner of the first digit whose running count reaches `remaining` is the boundary.
    int v = 0, incl = 0;
    if (tid < 256) {
      v = static_cast<int>(sc->hist[255 - tid]);
      incl = warp_incl_scan(v);
      if (lane == 31) sc->warp_tot[tid >> 5] = incl;
    }
    __syncthreads();
    if (tid < 256) {
      int base = 0;
      for (int w = 0; w < (tid >> 5); ++w) base += sc->warp_tot[w];
      incl += base;
      if (incl >= remaining && incl - v < remaining) {
        sc->digit = 255 - tid;
        sc->above = incl - v;
        sc->count = v;
      }
    }
    __syncthreads();
    const int d = sc->digit;
    remaining -= sc->above;
    const int cnt = sc->count;
    thr.prefix |= static_cast<unsigned long long>(d) << shift;
    thr.mask |= 0xFFull << shift;
    __syncthreads();
    if (cnt == remaining) break;
  }
  return thr;
}

// Stable compaction of the selected items in item order: emit(pos, i, key, idx) is called once
// per selected item with consecutive positions starting at 0.  Returns the number emitted.
// Warps own contiguous item ranges, so output order equals item order.
template <class ItemFn, class EmitFn>
__device__ int cta_compact(const ItemFn& item, int n, const SelectThreshold& thr, const EmitFn& emit, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int per = (n + nwarps - 1) / nwarps;
  per = (per + 31) & ~31;
  const int lo = warp * per;
  const int hi = min(n, lo + per);
  int cnt = 0;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    bool sel = false;
    if (i < hi) {
      uint32_t key, idx;
      item(i, key, idx);
      sel = is_selected(thr, key, idx);
    }
    cnt += __popc(__ballot_sync(0xFFFFFFFFu, sel));
  }
  // exclusive scan over warps
  if (lane == 0) scratch[warp] = cnt;
  __syncthreads();
  if (warp == 0) {
    int v = (lane < nwarps) ? scratch[lane] : 0;
    int incl = warp_incl_scan(v);
    if (lane < nwarps) scratch[lane] = incl - v;
    if (lane == nwarps - 1) scratch[nwarps] = incl;
  }
  __syncthreads();
  int off = scratch[warp];
  const int total = scratch[nwarps];
  const unsigned lt = (1u << lane) - 1u;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    bool sel = false;
    uint32_t key = 0, idx = 0;
    if (i < hi) {
      item(i, key, idx);
      sel = is_selected(thr, key, idx);
    }
    const unsigned b = __ballot_sync(0xFFFFFFFFu, sel);
    if (sel) emit(off + __popc(b & lt), i, key, idx);
    off += __popc(b);
  }
  __syncthreads();
  return total;
}

// In-place ascending bitonic sort of n <= cap 64-bit keys in shared memory (cap a power of two;
// entries n..cap-1 are padded with ~0ull by the caller or here).
__device__ __forceinline__ void cta_bitonic_sort_u64(unsigned long long* v, int n, int cap) {
  for (int i = n + threadIdx.x; i < cap; i += blockDim.x) v[i] = ~0ull;
  __syncthreads();
  for (int size = 2; size <= cap; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < cap / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = ((lo & size) == 0);
        unsigned long long a = v[lo], b = v[hi];
        if ((a > b) == up) {
          v[lo] = b;
          v[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace sva
