// Exact top-k selection inside one CTA under the canonical tie rule.
//
// Items are 64-bit composites produced by a functor, c = (key32 << 32) | ~idx32, where key32 is
// an ordered score key (sva::ordered_key); c == 0 marks an item that is not a candidate.  The
// selection order is c descending, i.e. score descending, then key index ascending -- the rule
// the CPU oracle applies to every torch.topk of the reference (sva/llama.py:278, :295, :100,
// :113).
//
// Two selects, both exact and both returning a plain threshold (an item is selected iff c != 0
// and c >= prefix):
// * cta_radix_select finds the range [min, max] of the non-zero items, then runs an MSB-first
//   radix select on (c - min) with 10-bit digits starting at the highest bit of (max - min):
//   each level divides the current window into 1024 equal bins, counts the items of the window
//   per bin (a functor call per item, so items may live in shared memory or be re-read from
//   global memory) and keeps the bin holding the k-th item.  Starting at the range's own top
//   bit keeps items that share their high bits (every candidate above a threshold does) from
//   piling into one bin.  It stops as soon as the boundary bin holds exactly the number of
//   items still needed.
// * cta_select_linear takes a known score range, counts the items into 1024 equal-width score
//   bins in one pass and ranks the few items of the boundary bin directly.
#pragma once

#include "sva_common.cuh"

namespace sva {

constexpr int kSelectBins = 1024;
constexpr int kSelectDigit = 10;

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

// Shared scratch for cta_radix_select: two bin-count buffers (a level counts into one while the
// other is cleared for the next level) and per-buffer broadcast slots.
struct SelectScratch {
  uint32_t hist[2][kSelectBins];
  unsigned long long lo_part[32];
  unsigned long long hi_part[32];
  int warp_tot[2][32];
  int digit[2];
  int above[2];
  int count[2];
};

// `ts` (measurement only, may be NULL): thread 0 writes the global timer after the range pass
// and after each level into ts[0], ts[1], ... (at most ts_slots).
__device__ __forceinline__ void select_stamp(unsigned long long* ts, int slot) {
  if (ts && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    ts[slot] = t;
  }
}

// Requires blockDim.x in {256, 512, 1024}.  `k` should not exceed the number of non-zero items
// (if it does, every non-zero item is selected).  All threads of the block must call it.
// Barriers: one for the range, three per level.
template <class ItemFn>
__device__ SelectThreshold cta_radix_select(const ItemFn& item, int n, int k, SelectScratch* sc,
                                            unsigned long long* ts = nullptr, int ts_slots = 0) {
  SelectThreshold thr;
  thr.mask = ~0ull;
  if (k <= 0) {
    thr.prefix = ~0ull;
    thr.mask = 0ull;  // (c & 0) >= ~0 is false for every item
    return thr;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  // Item loops load kBatch items before using any of them, so their latencies overlap.
  constexpr int kBatch = 4;
  unsigned long long mn = ~0ull, mx = 0ull;
  for (int i0 = tid; i0 < n; i0 += kBatch * blockDim.x) {
    unsigned long long c[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * blockDim.x;
      c[u] = i < n ? item(i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (c[u] != 0ull) {
        mn = c[u] < mn ? c[u] : mn;
        mx = c[u] > mx ? c[u] : mx;
      }
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
  for (int b = tid; b < kSelectBins; b += blockDim.x) sc->hist[0][b] = 0u;
  __syncthreads();
  // every warp reduces the per-warp partials, one per lane
  unsigned long long base = lane < nwarps ? sc->lo_part[lane] : ~0ull;
  unsigned long long top = lane < nwarps ? sc->hi_part[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long a = __shfl_xor_sync(0xFFFFFFFFu, base, o);
    const unsigned long long b = __shfl_xor_sync(0xFFFFFFFFu, top, o);
    base = a < base ? a : base;
    top = b > top ? b : top;
  }
  if (ts_slots > 0) select_stamp(ts, 0);
  if (top == 0ull || top == base) {  // no items, or all non-zero items equal
    thr.prefix = base;
    return thr;
  }
  int hi = 63 - __clzll(static_cast<long long>(top - base));
  int remaining = k;
  int buf = 0;
  int lvl = 1;
  const int per = kSelectBins / blockDim.x;  // bins per thread in the scan
  for (;;) {
    const int lo = hi >= kSelectDigit - 1 ? hi - (kSelectDigit - 1) : 0;
    for (int i0 = tid; i0 < n; i0 += kBatch * blockDim.x) {
      unsigned long long c[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * blockDim.x;
        c[u] = i < n ? item(i) : 0ull;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const unsigned long long d = c[u] - base;
        // in the window [base, base + 2^(hi+1))
        if (c[u] != 0ull && c[u] >= base && (hi == 63 || (d >> (hi + 1)) == 0ull))
          atomicAdd(&sc->hist[buf][d >> lo], 1u);
      }
    }
    for (int b = tid; b < kSelectBins; b += blockDim.x) sc->hist[buf ^ 1][b] = 0u;  // next level's buffer
    __syncthreads();
    // descending scan: thread t owns bins kSelectBins-1-per*t ... kSelectBins-per*(t+1)
    int cnt = 0;
    for (int q = 0; q < per; ++q) cnt += static_cast<int>(sc->hist[buf][kSelectBins - 1 - (per * tid + q)]);
    const int incl_w = warp_incl_scan(cnt);
    if (lane == 31) sc->warp_tot[buf][warp] = incl_w;
    __syncthreads();
    // prefix of the warp totals, in every warp by shuffles
    const int wt = lane < nwarps ? sc->warp_tot[buf][lane] : 0;
    const int wincl = warp_incl_scan(wt);
    const int total = __shfl_sync(0xFFFFFFFFu, wincl, 31);
    const int wexcl = __shfl_sync(0xFFFFFFFFu, wincl - wt, warp);
    const int incl = incl_w + wexcl;
    const int excl = incl - cnt;
    if (excl < remaining && incl >= remaining) {
      int run = excl;
      for (int q = 0; q < per; ++q) {
        const int b = kSelectBins - 1 - (per * tid + q);
        const int v = static_cast<int>(sc->hist[buf][b]);
        if (run + v >= remaining) {
          sc->digit[buf] = b;
          sc->above[buf] = run;
          sc->count[buf] = v;
          break;
        }
        run += v;
      }
    }
    __syncthreads();
    if (total < remaining) break;  // fewer items than k: keep the window's base, select all
    const int count = sc->count[buf];
    base += static_cast<unsigned long long>(sc->digit[buf]) << lo;
    remaining -= sc->above[buf];
    if (lvl < ts_slots) select_stamp(ts, lvl++);
    if (count == remaining || lo == 0) break;
    hi = lo - 1;
    buf ^= 1;
  }
  thr.prefix = base;
  return thr;
}

// Locates the bin holding the k-th largest item of hist[0, kSelectBins) counted from the top:
// writes the bin to sc->digit[buf], the items in higher bins to sc->above[buf] and the bin's
// count to sc->count[buf]; returns the total count.  Two barriers; the results are visible to
// every thread on return.
__device__ __forceinline__ int select_find_bin(const uint32_t* hist, int remaining, SelectScratch* sc, int buf) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int per = kSelectBins / blockDim.x;
  int cnt = 0;
  for (int q = 0; q < per; ++q) cnt += static_cast<int>(hist[kSelectBins - 1 - (per * tid + q)]);
  const int incl_w = warp_incl_scan(cnt);
  if (lane == 31) sc->warp_tot[buf][warp] = incl_w;
  __syncthreads();
  const int wt = lane < nwarps ? sc->warp_tot[buf][lane] : 0;
  const int wincl = warp_incl_scan(wt);
  const int total = __shfl_sync(0xFFFFFFFFu, wincl, 31);
  const int wexcl = __shfl_sync(0xFFFFFFFFu, wincl - wt, warp);
  const int incl = incl_w + wexcl;
  const int excl = incl - cnt;
  if (excl < remaining && incl >= remaining) {
    int run = excl;
    for (int q = 0; q < per; ++q) {
      const int b = kSelectBins - 1 - (per * tid + q);
      const int v = static_cast<int>(hist[b]);
      if (run + v >= remaining) {
        sc->digit[buf] = b;
        sc->above[buf] = run;
        sc->count[buf] = v;
        break;
      }
      run += v;
    }
  }
  __syncthreads();
  return total;
}

constexpr int kLinearRankMax = kSelectBins / 2;  // boundary-bin items ranked directly (u64 in hist[1])

// Exact top-k like cta_radix_select, for items whose scores are known to lie in [lo, hi] (the
// score of item c is key_to_float(c >> 32)).  One counting pass puts every item into one of
// kSelectBins equal-width bins of [lo, hi]; the bin index is a monotone function of the score
// (scores outside the range land in the end bins), so every item of a higher bin ranks above
// every item of a lower one.  The items of the bin holding the k-th item are then ranked among
// themselves by composite.  Uses fallback() (another exact select) when the range is empty or
// not finite, or the boundary bin holds more than kLinearRankMax items.  Barriers: five.
template <class ItemFn, class Fallback>
__device__ SelectThreshold cta_select_linear(const ItemFn& item, int n, int k, float lo, float hi, SelectScratch* sc,
                                             const Fallback& fallback) {
  SelectThreshold thr;
  thr.mask = ~0ull;
  if (k <= 0) {
    thr.prefix = ~0ull;
    thr.mask = 0ull;
    return thr;
  }
  const float span = hi - lo;
  if (!(span > 0.f) || !isfinite(span)) return fallback();
  const float scale = (static_cast<float>(kSelectBins) - 0.5f) / span;
  if (!isfinite(scale) || !(scale > 0.f)) return fallback();
  const int tid = threadIdx.x;
  auto bin_of = [&](unsigned long long c) -> int {
    const uint32_t key = static_cast<uint32_t>(c >> 32);
    const float x = __fmul_rn(__fsub_rn(key_to_float(key), lo), scale);
    if (x != x) return key >= 0x80000000u ? kSelectBins - 1 : 0;  // NaN: where its key orders it
    return x > 0.f ? static_cast<int>(fminf(x, static_cast<float>(kSelectBins - 1))) : 0;
  };
  uint32_t* hist = sc->hist[0];
  for (int b = tid; b < kSelectBins; b += blockDim.x) hist[b] = 0u;
  if (tid == 0) sc->count[1] = 0;
  __syncthreads();
  constexpr int kBatch = 8;
  for (int i0 = tid; i0 < n; i0 += kBatch * blockDim.x) {
    unsigned long long c[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * blockDim.x;
      c[u] = i < n ? item(i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (c[u] != 0ull) atomicAdd(&hist[bin_of(c[u])], 1u);
  }
  __syncthreads();
  const int total = select_find_bin(hist, k, sc, 0);
  if (total < k) {  // fewer items than k: every non-zero item
    thr.prefix = 1ull;
    return thr;
  }
  const int bstar = sc->digit[0], need = k - sc->above[0], cnt = sc->count[0];
  if (cnt > kLinearRankMax) return fallback();
  unsigned long long* list = reinterpret_cast<unsigned long long*>(sc->hist[1]);
  for (int i0 = tid; i0 < n; i0 += kBatch * blockDim.x) {
    unsigned long long c[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * blockDim.x;
      c[u] = i < n ? item(i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (c[u] != 0ull && bin_of(c[u]) == bstar) list[atomicAdd(&sc->count[1], 1)] = c[u];
  }
  __syncthreads();
  // the need-th largest composite of the boundary bin (composites are distinct)
  for (int i = tid; i < cnt; i += blockDim.x) {
    const unsigned long long v = list[i];
    int above = 0;
    for (int j = 0; j < cnt; ++j) above += list[j] > v;
    if (above == need - 1) sc->lo_part[0] = v;
  }
  __syncthreads();
  thr.prefix = sc->lo_part[0];
  return thr;
}

// Items held in a shared-memory array.
struct U64Items {
  const unsigned long long* a;
  __device__ unsigned long long operator()(int i) const { return a[i]; }
};

// Selects over a shared-memory array of composites (one instantiation serves every caller in a
// kernel).
static __device__ __forceinline__ SelectThreshold radix_select_u64(const unsigned long long* a, int n, int k,
                                                                  SelectScratch* sc) {
  return cta_radix_select(U64Items{a}, n, k, sc);
}

// cta_select_linear over a[0, n) (fallback: radix_select_u64).  Not inlined: a kernel that selects
// twice (shortlist, then budget) runs one copy of the code, so the second select finds its
// instructions already fetched (a one-CTA-per-problem finish runs each phase once per problem,
// and instruction fetch is a large part of such a phase).
static __device__ __noinline__ SelectThreshold select_u64(const unsigned long long* a, int n, int k, float lo,
                                                            float hi, SelectScratch* sc) {
  return cta_select_linear(U64Items{a}, n, k, lo, hi, sc, [&]() { return radix_select_u64(a, n, k, sc); });
}

// Stable compaction of the selected items in item order: emit(pos, i, c) is called once per
// selected item with consecutive positions from 0.  Returns the number emitted.  Warps own
// contiguous item ranges, so output order equals item order.
template <class ItemFn, class EmitFn>
__device__ int cta_compact(const ItemFn& item, int n, const SelectThreshold& thr, const EmitFn& emit, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  constexpr int kBatch = 4;  // 32-item steps whose loads are issued together
  int per = (n + nwarps - 1) / nwarps;
  per = (per + 31) & ~31;
  const int lo = warp * per;
  const int hi = min(n, lo + per);
  int cnt = 0;
  for (int base = lo; base < hi; base += kBatch * 32) {
    bool sel[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * 32 + lane;
      sel[u] = (i < hi) && is_selected(thr, item(i));
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) cnt += __popc(__ballot_sync(0xFFFFFFFFu, sel[u]));
  }
  if (lane == 0) scratch[warp] = cnt;
  __syncthreads();
  // every warp: exclusive prefix of the warp counts, by shuffles
  const int v = lane < nwarps ? scratch[lane] : 0;
  const int incl = warp_incl_scan(v);
  const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  int off = __shfl_sync(0xFFFFFFFFu, incl - v, warp);
  const unsigned lt = (1u << lane) - 1u;
  for (int base = lo; base < hi; base += kBatch * 32) {
    unsigned long long c[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * 32 + lane;
      c[u] = i < hi ? item(i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * 32 + lane;
      const bool sel = (i < hi) && is_selected(thr, c[u]);
      const unsigned bm = __ballot_sync(0xFFFFFFFFu, sel);
      if (sel) emit(off + __popc(bm & lt), i, c[u]);
      off += __popc(bm);
    }
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

namespace sva {

// Stable compaction of the selected items of a[0, n): out[pos] = i for the pos-th selected item
// i in item order.  Returns the count; ends with a barrier.
static __device__ __noinline__ int compact_u64(const unsigned long long* a, int n, SelectThreshold thr, int32_t* out,
                                                  int* scratch) {
  return cta_compact(U64Items{a}, n, thr, [&](int pos, int i, unsigned long long) { out[pos] = i; }, scratch);
}

}  // namespace sva
