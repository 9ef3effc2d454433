// Exact top-k selection inside one CTA under the canonical tie rule.
//
// Items are 64-bit composites produced by a functor, c = (key32 << 32) | ~idx32, where key32 is
// an ordered score key (sva::ordered_key); c == 0 marks an item that is not a candidate.  The
// selection order is c descending, i.e. score descending, then key index ascending -- the rule
// the CPU oracle applies to every torch.topk of the reference (sva/llama.py:278, :295, :100,
// :113).  A caller whose items share their top bits may pass a left-shifted composite that
// keeps only the varying bits, as long as the order is preserved and real items stay non-zero.
//
// The select is an MSB-first radix select with 8-bit digits starting at bit `top_bit`.  Each
// level makes one pass over the items (a functor call per item, so items may live in shared
// memory or be re-read from global memory), builds a 256-bin histogram of the digit among the
// items that still match the prefix, and fixes one digit.  It stops as soon as the boundary
// digit holds exactly the number of items still needed.  An item is selected iff c != 0 and
// (c & mask) >= prefix.
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

__device__ __forceinline__ bool is_selected(const SelectThreshold& t, unsigned long long c) {
  return c != 0ull && (c & t.mask) >= t.prefix;
}

// Shared scratch for cta_radix_select: 256-bin histogram plus a few broadcast slots.
struct SelectScratch {
  uint32_t hist[256];
  int warp_tot[9];
  int digit;
  int above;
  int count;
};

// Requires blockDim.x >= 256 and a multiple of 32.  `k` must not exceed the number of non-zero
// items.  All threads of the block must call it.  Digits are bits [top_bit-7, top_bit],
// [top_bit-15, top_bit-8], ... (top_bit in 7..63, the last digit may be narrower).
template <class ItemFn>
__device__ SelectThreshold cta_radix_select(const ItemFn& item, int n, int k, SelectScratch* sc, int top_bit = 63) {
  SelectThreshold thr;
  thr.prefix = 0ull;
  thr.mask = 0ull;
  if (k <= 0) {
    thr.prefix = ~0ull;  // (c & 0) >= ~0 is false for every item
    return thr;
  }
  int remaining = k;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  for (int hi = top_bit; hi >= 0; hi -= 8) {
    const int lo = hi >= 7 ? hi - 7 : 0;
    const int width = hi - lo + 1;
    const unsigned long long dmask = ((1ull << width) - 1ull) << lo;
    for (int b = tid; b < 256; b += blockDim.x) sc->hist[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const unsigned long long c = item(i);
      if (c == 0ull || (c & thr.mask) != thr.prefix) continue;
      atomicAdd(&sc->hist[(c >> lo) & ((1ull << width) - 1ull)], 1u);
    }
    __syncthreads();
    // Descending suffix scan over the digits with warps 0..7 (thread t owns digit 255-t): the
    // owner of the first digit whose running count reaches `remaining` is the boundary.
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
    const unsigned long long d = static_cast<unsigned long long>(sc->digit);
    remaining -= sc->above;
    const int cnt = sc->count;
    thr.prefix |= d << lo;
    thr.mask |= dmask;
    __syncthreads();
    if (cnt == remaining) break;
  }
  return thr;
}

// Stable compaction of the selected items in item order: emit(pos, i, c) is called once per
// selected item with consecutive positions from 0.  Returns the number emitted.  Warps own
// contiguous item ranges, so output order equals item order.
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
    const bool sel = (i < hi) && is_selected(thr, item(i));
    cnt += __popc(__ballot_sync(0xFFFFFFFFu, sel));
  }
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
    unsigned long long c = 0ull;
    bool sel = false;
    if (i < hi) {
      c = item(i);
      sel = is_selected(thr, c);
    }
    const unsigned b = __ballot_sync(0xFFFFFFFFu, sel);
    if (sel) emit(off + __popc(b & lt), i, c);
    off += __popc(b);
  }
  __syncthreads();
  return total;
}

// In-place ascending bitonic sort of n <= cap 64-bit keys in shared memory (cap a power of two;
// entries n..cap-1 are padded with ~0ull here).
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
