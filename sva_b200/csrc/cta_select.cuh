// Exact top-k selection inside one CTA under the canonical tie rule.
//
// Items are 64-bit composites produced by a functor, c = (key32 << 32) | ~idx32, where key32 is
// an ordered score key (sva::ordered_key); c == 0 marks an item that is not a candidate.  The
// selection order is c descending, i.e. score descending, then key index ascending -- the rule
// the CPU oracle applies to every torch.topk of the reference (sva/llama.py:278, :295, :100,
// :113).
//
// The select first finds the range [min, max] of the non-zero items, then runs an MSB-first
// radix select on (c - min) with 11-bit digits starting at the highest bit of (max - min): each
// level divides the current window into 2048 equal bins, counts the items of the window per bin
// (a functor call per item, so items may live in shared memory or be re-read from global
// memory) and keeps the bin holding the k-th item.  Starting at the range's own top bit keeps
// items that share their high bits (every candidate above a threshold does) from piling into
// one bin.  It stops as soon as the boundary bin holds exactly the number of items still
// needed.  The result is a plain threshold: an item is selected iff c != 0 and c >= prefix.
#pragma once

#include "sva_common.cuh"

namespace sva {

constexpr int kSelectBins = 2048;
constexpr int kSelectDigit = 11;

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

// Shared scratch for cta_radix_select: the bin counts plus a few broadcast slots.
struct SelectScratch {
  uint32_t hist[kSelectBins];
  unsigned long long lo_part[32];
  unsigned long long hi_part[32];
  int warp_tot[32];
  unsigned long long base;
  unsigned long long top;
  int digit;
  int above;
  int count;
};

// Requires blockDim.x in {256, 512, 1024}.  `k` should not exceed the number of non-zero items
// (if it does, every non-zero item is selected).  All threads of the block must call it.
template <class ItemFn>
__device__ SelectThreshold cta_radix_select(const ItemFn& item, int n, int k, SelectScratch* sc) {
  SelectThreshold thr;
  thr.mask = ~0ull;
  if (k <= 0) {
    thr.prefix = ~0ull;
    thr.mask = 0ull;  // (c & 0) >= ~0 is false for every item
    return thr;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  unsigned long long mn = ~0ull, mx = 0ull;
  for (int i = tid; i < n; i += blockDim.x) {
    const unsigned long long c = item(i);
    if (c != 0ull) {
      mn = c < mn ? c : mn;
      mx = c > mx ? c : mx;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long a = __shfl_xor_sync(0xFFFFFFFFu, mn, o);
    const unsigned long long b = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    mn = a < mn ? a : mn;
    mx = b > mx ? b : mx;
  }
  if (lane == 0) {
    sc->lo_part[warp] = mn;
    sc->hi_part[warp] = mx;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long a = ~0ull, b = 0ull;
    for (int w = 0; w < nwarps; ++w) {
      a = sc->lo_part[w] < a ? sc->lo_part[w] : a;
      b = sc->hi_part[w] > b ? sc->hi_part[w] : b;
    }
    sc->base = a;
    sc->top = b;
  }
  __syncthreads();
  unsigned long long base = sc->base;
  const unsigned long long top = sc->top;
  __syncthreads();
  if (top == 0ull || top == base) {  // no items, or all non-zero items equal
    thr.prefix = base;
    return thr;
  }
  int hi = 63 - __clzll(static_cast<long long>(top - base));
  int remaining = k;
  const int per = kSelectBins / blockDim.x;  // bins per thread in the scan
  for (;;) {
    const int lo = hi >= kSelectDigit - 1 ? hi - (kSelectDigit - 1) : 0;
    for (int b = tid; b < kSelectBins; b += blockDim.x) sc->hist[b] = 0u;
    if (tid == 0) sc->count = -1;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const unsigned long long c = item(i);
      if (c == 0ull || c < base) continue;
      const unsigned long long d = c - base;
      if (hi < 63 && (d >> (hi + 1)) != 0ull) continue;  // above the window [base, base + 2^(hi+1))
      atomicAdd(&sc->hist[d >> lo], 1u);
    }
    __syncthreads();
    // Descending scan: thread t owns bins kSelectBins-1-per*t ... kSelectBins-per*(t+1).
    int cnt = 0;
    for (int q = 0; q < per; ++q) cnt += static_cast<int>(sc->hist[kSelectBins - 1 - (per * tid + q)]);
    int incl = warp_incl_scan(cnt);
    if (lane == 31) sc->warp_tot[warp] = incl;
    __syncthreads();
    for (int w = 0; w < warp; ++w) incl += sc->warp_tot[w];
    const int excl = incl - cnt;
    if (excl < remaining && incl >= remaining) {
      int run = excl;
      for (int q = 0; q < per; ++q) {
        const int b = kSelectBins - 1 - (per * tid + q);
        const int v = static_cast<int>(sc->hist[b]);
        if (run + v >= remaining) {
          sc->digit = b;
          sc->above = run;
          sc->count = v;
          break;
        }
        run += v;
      }
    }
    __syncthreads();
    const int count = sc->count;
    if (count < 0) break;  // fewer items than k: keep the window's base, select all
    base += static_cast<unsigned long long>(sc->digit) << lo;
    remaining -= sc->above;
    __syncthreads();
    if (count == remaining || lo == 0) break;
    hi = lo - 1;
  }
  thr.prefix = base;
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
