// Scan summon -> rank rescore -> exact verify (replaces sva/llama.py:171-328).
//
// Problems are (query head h, query token t) pairs.  Two schedules:
//
// * fused  (key_len <= kFusedMaxKeys): one CTA per problem does everything.  The ADC key of
//   every allowed key is computed once into shared memory; the shortlist is an exact CTA radix
//   select over it; the CTA then rescores the shortlist against k_low, selects the budget and
//   runs the verify.  One launch per call.
//
// * grid   (longer caches): the key range of each problem is cut into segments of kSegKeys.
//     qlut    : one CTA per problem builds q_low and the LUT into the workspace and clears the
//               problem's histogram / control block;
//     hist    : one CTA per segment builds a 4096-bin histogram of the top 12 bits of the
//               ordered ADC key and adds it to the problem's global histogram; the last CTA to
//               finish (ticket counter, no waiting) finds the boundary bin b* of the shortlist;
//     collect : one CTA per segment re-reads its codes (now in L2); keys above b* go straight
//               to the shortlist, keys in b* go to an edge buffer sized for the whole range;
//     problem : one CTA per problem selects the missing shortlist entries from the edge buffer
//               (exact, canonical; in shared memory when it fits, else streamed from L2), then
//               rescores / selects / verifies as in the fused schedule.
//
// Codes are read four keys per vector load (S bytes per key), four loads in flight per thread.
// Selection rule everywhere: score descending, key index ascending (see cta_select.cuh).
// ADC score: ((0 + lut[0][c0]) + lut[1][c1]) + ... in subspace order, then / sqrt(R)
// (reference sva/ops.py:64-71).  Rank score: tree_dot(k_low, q_low) / sqrt(R)
// (reference sva/llama.py:286-292).
#include "cta_select.cuh"
#include "qlut.cuh"
#include "sva_internal.h"
#include "verify.cuh"

namespace sva {

constexpr int kThreads = 512;
constexpr int kBins = 4096;
constexpr int kSegKeys = 16384;
constexpr int kFusedMaxKeys = 32768;
constexpr int kEdgeSmem = 12288;  // edge entries resolved in shared memory
constexpr int kScanThreads = 256;
constexpr int kGroupsInFlight = 4;

enum { CTRL_T_HIST = 0, CTRL_K, CTRL_BSTAR, CTRL_NABOVE, CTRL_NOUT, CTRL_NEDGE, CTRL_NVALID, CTRL_WORDS = 8 };

struct DecodeSmem {
  int qf, ql, lut, sc, scratch, sl, rk, fin, lg, acc, cache, total;
};

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

__host__ __device__ inline DecodeSmem decode_smem_layout(int head_dim, int sl_cap, int b_cap, int cache_bytes) {
  DecodeSmem s;
  int o = 0;
  s.qf = o;      o = align16(o + 4 * head_dim);
  s.ql = o;      o = align16(o + 4 * kMaxRank);
  s.lut = o;     o = align16(o + 4 * kMaxLut);
  s.sc = o;      o = align16(o + (int)sizeof(SelectScratch));
  s.scratch = o; o = align16(o + 4 * 64);
  s.sl = o;      o = align16(o + 4 * sl_cap);
  s.rk = o;      o = align16(o + 4 * sl_cap);
  s.fin = o;     o = align16(o + 4 * b_cap);
  s.lg = o;      o = align16(o + 4 * b_cap);
  s.acc = o;     o = align16(o + 8 * ((kThreads / 32) * 64 + kThreads / 32 + 1));
  s.cache = o;   o = align16(o + cache_bytes);
  s.total = o;
  return s;
}

struct DecodeParams {
  sva_decode_args a;
  int groups;
  int sub;
  int sqrt_r_pow2;
  float sqrt_r;
  float inv_sqrt_r;
  int sl_cap;
  int b_cap;
  int grid_mode;
  int nseg;
  int vec_codes;  // codes aligned for 4-key vector loads
  DecodeSmem lay;
  float* ws_qlow;
  float* ws_lut;
  uint32_t* ws_hist;
  uint32_t* ws_ctrl;
  int32_t* ws_part;
  uint2* ws_edge;
};

// ---------------------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ float finish_score(float sum, const DecodeParams& p) {
  return p.sqrt_r_pow2 ? __fmul_rn(sum, p.inv_sqrt_r) : __fdiv_rn(sum, p.sqrt_r);
}

__device__ __forceinline__ int64_t allowed_length(const DecodeParams& p, int t) {
  const int64_t L = p.a.key_len;
  int64_t n = p.a.allowed_len ? p.a.allowed_len[t] : (L - p.a.n_queries + t + 1);
  return n < 0 ? 0 : (n > L ? L : n);
}

__device__ __forceinline__ bool key_allowed(const DecodeParams& p, int t, int64_t i, int64_t len_t) {
  if (i >= len_t) return false;
  if (p.a.allowed_mask) return p.a.allowed_mask[t * p.a.mask_row_stride + i] != 0;
  return true;
}

// Ordered ADC key of key i (0 when not allowed), scalar code loads.
__device__ __forceinline__ uint32_t adc_key(const DecodeParams& p, const uint8_t* __restrict__ codes,
                                            const float* __restrict__ lut, int t, int64_t i, int64_t len_t) {
  if (!key_allowed(p, t, i, len_t)) return 0u;
  const int S = p.a.subspaces, C = p.a.codewords;
  const uint8_t* row = codes + i * S;
  float sum = 0.f;
  for (int s = 0; s < S; ++s) sum = __fadd_rn(sum, lut[s * C + __ldg(row + s)]);
  return ordered_key(finish_score(sum, p));
}

// Codes of four consecutive keys in one vector load (S = 1, 2, 4 or 8 bytes per key).
template <int S>
struct Codes4 {
  uint4 a, b;
};

template <int S>
__device__ __forceinline__ Codes4<S> load_codes4(const uint8_t* base, int64_t i) {
  Codes4<S> r;
  if (S == 1) {
    r.a.x = __ldg(reinterpret_cast<const uint32_t*>(base + i));
  } else if (S == 2) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(base + 2 * i));
    r.a.x = w.x;
    r.a.y = w.y;
  } else if (S == 4) {
    r.a = __ldg(reinterpret_cast<const uint4*>(base + 4 * i));
  } else {
    r.a = __ldg(reinterpret_cast<const uint4*>(base + 8 * i));
    r.b = __ldg(reinterpret_cast<const uint4*>(base + 8 * i + 16));
  }
  return r;
}

// Code of key j (0..3) in subspace s.
template <int S>
__device__ __forceinline__ uint32_t code_at(const Codes4<S>& c, int j, int s) {
  if (S == 1) return (c.a.x >> (8 * j)) & 0xFFu;
  if (S == 2) {
    const uint32_t w = (j < 2) ? c.a.x : c.a.y;
    return (w >> (16 * (j & 1) + 8 * s)) & 0xFFu;
  }
  if (S == 4) {
    const uint32_t w = (j == 0) ? c.a.x : (j == 1) ? c.a.y : (j == 2) ? c.a.z : c.a.w;
    return (w >> (8 * s)) & 0xFFu;
  }
  const uint4& v = (j < 2) ? c.a : c.b;
  const uint32_t w = ((j & 1) == 0) ? (s < 4 ? v.x : v.y) : (s < 4 ? v.z : v.w);
  return (w >> (8 * (s & 3))) & 0xFFu;
}

template <int S>
__device__ __forceinline__ uint32_t adc_key4(const DecodeParams& p, const Codes4<S>& c, int j,
                                             const float* __restrict__ lut) {
  const int C = p.a.codewords;
  float sum = 0.f;
#pragma unroll
  for (int s = 0; s < S; ++s) sum = __fadd_rn(sum, lut[s * C + code_at<S>(c, j, s)]);
  return ordered_key(finish_score(sum, p));
}

template <typename T>
__device__ void build_qlut(const DecodeParams& p, int h, int t, float* qf, float* ql, float* lut, float* stage) {
  const int D = p.a.head_dim, R = p.a.rank_dim, S = p.a.subspaces, C = p.a.codewords;
  const T* q = reinterpret_cast<const T*>(p.a.query) + h * p.a.q_head_stride + t * p.a.q_row_stride;
  const float* lo = p.a.lut_override ? p.a.lut_override + ((size_t)h * p.a.n_queries + t) * S * C : nullptr;
  build_query_lut<T>(q, D, R, S, C, p.a.q_proj + (size_t)h * D * R, __ldg(p.a.scale + h),
                     p.a.codebooks + (size_t)h * S * C * (R / S), lo, qf, ql, lut, stage);
}

// Block-wide sum of an int (all threads get the result).
__device__ __forceinline__ int block_sum_int(int v, int* scratch) {
  int total;
  (void)block_excl_scan(v, scratch, &total);
  return total;
}

// ---------------------------------------------------------------------------------------
// per-problem kernel: (fused) shortlist + rescore + budget select + verify
// ---------------------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kThreads) decode_problem_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qf = reinterpret_cast<float*>(smem + p.lay.qf);
  float* ql = reinterpret_cast<float*>(smem + p.lay.ql);
  float* lut = reinterpret_cast<float*>(smem + p.lay.lut);
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + p.lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + p.lay.scratch);
  int32_t* sl = reinterpret_cast<int32_t*>(smem + p.lay.sl);
  uint32_t* rk = reinterpret_cast<uint32_t*>(smem + p.lay.rk);
  int32_t* fin = reinterpret_cast<int32_t*>(smem + p.lay.fin);
  float* lg = reinterpret_cast<float*>(smem + p.lay.lg);
  double* acc = reinterpret_cast<double*>(smem + p.lay.acc);

  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries;
  const int t = prob - h * p.a.n_queries;
  const int kvh = h / p.groups;
  const int64_t L = p.a.key_len;
  const int64_t len_t = allowed_length(p, t);
  const uint8_t* codes = p.a.codes + h * p.a.codes_head_stride;
  const int R = p.a.rank_dim, D = p.a.head_dim;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;

  // ---- shortlist -------------------------------------------------------------------------
  int n_sl = 0;
  if (!p.grid_mode) {
    build_qlut<T>(p, h, t, qf, ql, lut, reinterpret_cast<float*>(smem + p.lay.cache));
    uint32_t* cache = reinterpret_cast<uint32_t*>(smem + p.lay.cache);
    int nv = 0;
    for (int64_t i = tid; i < L; i += blockDim.x) {
      const uint32_t key = adc_key(p, codes, lut, t, i, len_t);
      cache[i] = key;
      nv += (key != 0u);
    }
    const int n_valid = block_sum_int(nv, scratch);
    const int k = min(p.sl_cap, n_valid);
    auto item = [&](int i) -> unsigned long long {
      return cache[i] ? composite(cache[i], static_cast<uint32_t>(i)) : 0ull;
    };
    const SelectThreshold thr = cta_radix_select(item, static_cast<int>(L), k, sc);
    n_sl = cta_compact(item, static_cast<int>(L), thr, [&](int pos, int i, unsigned long long) { sl[pos] = i; },
                       scratch);
  } else {
    const T* q = reinterpret_cast<const T*>(p.a.query) + h * p.a.q_head_stride + t * p.a.q_row_stride;
    for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    for (int r = tid; r < R; r += blockDim.x) ql[r] = __ldcg(p.ws_qlow + (size_t)prob * kMaxRank + r);
    const uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
    const int k = static_cast<int>(__ldcg(ctrl + CTRL_K));
    const int n_part = min(static_cast<int>(__ldcg(ctrl + CTRL_NOUT)), k);
    const int64_t n_edge64 = __ldcg(ctrl + CTRL_NEDGE);
    const int n_edge = static_cast<int>(n_edge64 < L ? n_edge64 : L);
    const int32_t* part = p.ws_part + (size_t)prob * p.sl_cap;
    for (int i = tid; i < n_part; i += blockDim.x) sl[i] = __ldcg(part + i);
    const uint2* ge = p.ws_edge + (size_t)prob * L;
    // edge entries share the top 12 key bits: order them by the low 20 key bits, then index
    auto local = [](uint2 v) -> unsigned long long {
      return (static_cast<unsigned long long>(v.x & 0xFFFFFu) << 44) |
             (static_cast<unsigned long long>(~v.y) << 12) | 1ull;
    };
    const int need = k - n_part;
    if (n_edge <= kEdgeSmem) {
      uint2* edge = reinterpret_cast<uint2*>(smem + p.lay.cache);
      for (int i = tid; i < n_edge; i += blockDim.x) edge[i] = __ldcg(ge + i);
      __syncthreads();
      auto item = [&](int i) -> unsigned long long { return local(edge[i]); };
      const SelectThreshold thr = cta_radix_select(item, n_edge, need, sc);
      cta_compact(item, n_edge, thr, [&](int pos, int i, unsigned long long) { sl[n_part + pos] = edge[i].y; },
                  scratch);
    } else {
      auto item = [&](int i) -> unsigned long long { return local(__ldcg(ge + i)); };
      const SelectThreshold thr = cta_radix_select(item, n_edge, need, sc);
      cta_compact(item, n_edge, thr,
                  [&](int pos, int i, unsigned long long) { sl[n_part + pos] = __ldcg(ge + i).y; }, scratch);
    }
    n_sl = k;
  }
  __syncthreads();

  // ---- rank rescore: two rows per warp step (one per half-warp), 16 steps in flight -------
  {
    const int half = lane >> 4, l16 = lane & 15;
    const float4 q4 = (4 * l16 < R) ? make_float4(ql[4 * l16], ql[4 * l16 + 1], ql[4 * l16 + 2], ql[4 * l16 + 3])
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    const float* klb = p.a.k_low + h * p.a.k_low_head_stride;
    constexpr int U = 16;
    for (int base = warp * 2 * U; base < n_sl; base += nwarps * 2 * U) {
      float4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + 2 * u + half;
        r[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < n_sl && 4 * l16 < R) r[u] = load4<float>(klb + (int64_t)sl[j] * R, 4 * l16, R);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + 2 * u + half;
        const float s = tree16(lane4(r[u], q4));
        if (j < n_sl && l16 == 0) rk[j] = ordered_key(finish_score(s, p));
      }
    }
  }
  __syncthreads();

  // ---- budget select ----------------------------------------------------------------------
  const int b = min(p.b_cap, n_sl);
  int n_fin;
  {
    auto item = [&](int j) -> unsigned long long { return composite(rk[j], static_cast<uint32_t>(sl[j])); };
    const SelectThreshold thr = cta_radix_select(item, n_sl, b, sc);
    n_fin = cta_compact(item, n_sl, thr, [&](int pos, int j, unsigned long long) { fin[pos] = sl[j]; }, scratch);
  }

  // ---- verify ----------------------------------------------------------------------------
  verify_rows<T>(p.a.keys, p.a.k_head_stride, p.a.k_row_stride, p.a.values, p.a.v_head_stride, p.a.v_row_stride, kvh,
                 qf, D, fin, n_fin, p.a.softmax_scale, p.a.logits_mode, lg, acc, scratch,
                 reinterpret_cast<T*>(p.a.out) + h * p.a.out_head_stride + t * p.a.out_row_stride);

  // ---- debug outputs and counters -------------------------------------------------------
  if (p.a.shortlist_out || p.a.final_out) {
    unsigned long long* tmp = reinterpret_cast<unsigned long long*>(smem + p.lay.cache);
    if (p.a.shortlist_out) {
      int cap = 1;
      while (cap < n_sl) cap <<= 1;
      for (int i = tid; i < n_sl; i += blockDim.x) tmp[i] = static_cast<unsigned long long>(static_cast<uint32_t>(sl[i]));
      __syncthreads();
      cta_bitonic_sort_u64(tmp, n_sl, cap);
      int32_t* o = p.a.shortlist_out + (size_t)prob * p.a.shortlist;
      for (int i = tid; i < p.a.shortlist; i += blockDim.x) o[i] = (i < n_sl) ? static_cast<int32_t>(tmp[i]) : -1;
      __syncthreads();
    }
    if (p.a.final_out) {
      int cap = 1;
      while (cap < n_fin) cap <<= 1;
      for (int i = tid; i < n_fin; i += blockDim.x) tmp[i] = static_cast<unsigned long long>(static_cast<uint32_t>(fin[i]));
      __syncthreads();
      cta_bitonic_sort_u64(tmp, n_fin, cap);
      int32_t* o = p.a.final_out + (size_t)prob * p.a.budget;
      for (int i = tid; i < p.a.budget; i += blockDim.x) o[i] = (i < n_fin) ? static_cast<int32_t>(tmp[i]) : -1;
      __syncthreads();
    }
  }
  if (p.a.stats && tid == 0) {
    atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
    atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
  }
}

// ---------------------------------------------------------------------------------------
// grid schedule kernels
// ---------------------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(256) decode_qlut_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) float stage[];
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ float lut[kMaxLut];
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  build_qlut<T>(p, h, t, qf, ql, lut, stage);
  const int SC = p.a.subspaces * p.a.codewords;
  float* gl = p.ws_lut + (size_t)prob * kMaxLut;
  for (int e = threadIdx.x; e < SC; e += blockDim.x) gl[e] = lut[e];
  for (int r = threadIdx.x; r < p.a.rank_dim; r += blockDim.x) p.ws_qlow[(size_t)prob * kMaxRank + r] = ql[r];
  uint32_t* hist = p.ws_hist + (size_t)prob * kBins;
  for (int b = threadIdx.x; b < kBins; b += blockDim.x) hist[b] = 0u;
  if (threadIdx.x < CTRL_WORDS) p.ws_ctrl[(size_t)prob * CTRL_WORDS + threadIdx.x] = 0u;
}

// Calls f(i, key) for every key of [i0, i1) (key = 0 when not allowed).  With S > 0 each
// thread handles groups of four consecutive keys, kGroupsInFlight vector loads at a time.
// Iteration is warp-uniform: every lane calls f the same number of times (slots past the end
// come with i == i1 and key 0), so f may use warp collectives.
template <int S, class F>
__device__ __forceinline__ void scan_segment(const DecodeParams& p, const uint8_t* codes, const float* lut, int t,
                                             int64_t len_t, int64_t i0, int64_t i1, const F& f) {
  const int lane = threadIdx.x & 31;
  if constexpr (S > 0) {
    const int64_t ngroups = (i1 - i0 + 3) >> 2;
    const bool dense = (p.a.allowed_mask == nullptr) && (i1 <= len_t);
    for (int64_t gb = (threadIdx.x & ~31); gb < ngroups; gb += (int64_t)blockDim.x * kGroupsInFlight) {
      Codes4<S> c[kGroupsInFlight];
#pragma unroll
      for (int u = 0; u < kGroupsInFlight; ++u) {
        const int64_t g = gb + lane + (int64_t)u * blockDim.x;
        if (g < ngroups && i0 + 4 * g + 3 < i1) c[u] = load_codes4<S>(codes, i0 + 4 * g);
      }
#pragma unroll
      for (int u = 0; u < kGroupsInFlight; ++u) {
        const int64_t g = gb + lane + (int64_t)u * blockDim.x;
        const int64_t ib = i0 + 4 * g;
        const bool full = g < ngroups && ib + 3 < i1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t i = ib + j;
          const bool live = g < ngroups && i < i1;
          uint32_t key = 0u;
          if (full) {
            key = (dense || key_allowed(p, t, i, len_t)) ? adc_key4<S>(p, c[u], j, lut) : 0u;
          } else if (live) {
            key = adc_key(p, codes, lut, t, i, len_t);
          }
          f(live ? i : i1, key);
        }
      }
    }
  } else {
    for (int64_t wb = i0 + (threadIdx.x & ~31); wb < i1; wb += blockDim.x) {
      const int64_t i = wb + lane;
      const uint32_t key = (i < i1) ? adc_key(p, codes, lut, t, i, len_t) : 0u;
      f(i < i1 ? i : i1, key);
    }
  }
}

template <int S>
__global__ void __launch_bounds__(kScanThreads) decode_hist_kernel(const DecodeParams p) {
  __shared__ float lut[kMaxLut];
  __shared__ uint32_t hist[kBins];
  __shared__ int is_last;
  __shared__ int wsum[kScanThreads / 32];
  __shared__ int boundary[2];
  const int prob = blockIdx.y, seg = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  const int SC = p.a.subspaces * p.a.codewords;
  for (int e = threadIdx.x; e < SC; e += blockDim.x) lut[e] = __ldcg(p.ws_lut + (size_t)prob * kMaxLut + e);
  for (int b = threadIdx.x; b < kBins; b += blockDim.x) hist[b] = 0u;
  __syncthreads();
  const int64_t len_t = allowed_length(p, t);
  const uint8_t* codes = p.a.codes + h * p.a.codes_head_stride;
  const int64_t i0 = (int64_t)seg * kSegKeys;
  const int64_t i1 = min(p.a.key_len, i0 + kSegKeys);
  scan_segment<S>(p, codes, lut, t, len_t, i0, i1, [&](int64_t, uint32_t key) {
    if (key) atomicAdd(&hist[key >> 20], 1u);
  });
  __syncthreads();
  uint32_t* gh = p.ws_hist + (size_t)prob * kBins;
  for (int b = threadIdx.x; b < kBins; b += blockDim.x)
    if (hist[b]) atomicAdd(gh + b, hist[b]);
  __threadfence();
  __syncthreads();
  uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
  if (threadIdx.x == 0) is_last = (atomicAdd(ctrl + CTRL_T_HIST, 1u) == static_cast<uint32_t>(p.nseg - 1));
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Last CTA of this problem: find the boundary bin of the shortlist.  Thread j owns bins
  // 4095-16j .. 4080-16j (descending).
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t mine[16];
  int s = 0;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    mine[q] = __ldcg(gh + (kBins - 1 - (16 * tid + q)));
    s += static_cast<int>(mine[q]);
  }
  int incl = warp_incl_scan(s);
  if (lane == 31) wsum[tid >> 5] = incl;
  if (tid == 0) {
    boundary[0] = kBins;  // no key qualifies unless overwritten below
    boundary[1] = 0;
  }
  __syncthreads();
  int base = 0, total = 0;
  for (int w = 0; w < kScanThreads / 32; ++w) {
    if (w < (tid >> 5)) base += wsum[w];
    total += wsum[w];
  }
  const int k = min(p.sl_cap, total);
  incl += base;
  const int excl = incl - s;
  if (k > 0 && excl < k && incl >= k) {
    int run = excl;
    for (int q = 0; q < 16; ++q) {
      const int v = static_cast<int>(mine[q]);
      if (run + v >= k) {
        boundary[0] = kBins - 1 - (16 * tid + q);
        boundary[1] = run;
        break;
      }
      run += v;
    }
  }
  __syncthreads();
  if (tid == 0) {
    ctrl[CTRL_K] = static_cast<uint32_t>(k);
    ctrl[CTRL_BSTAR] = static_cast<uint32_t>(boundary[0]);
    ctrl[CTRL_NABOVE] = static_cast<uint32_t>(boundary[1]);
    ctrl[CTRL_NVALID] = static_cast<uint32_t>(total);
  }
}

template <int S>
__global__ void __launch_bounds__(kScanThreads) decode_collect_kernel(const DecodeParams p) {
  __shared__ float lut[kMaxLut];
  const int prob = blockIdx.y, seg = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
  const uint32_t bstar = __ldcg(ctrl + CTRL_BSTAR);
  if (bstar >= static_cast<uint32_t>(kBins)) return;
  const int SC = p.a.subspaces * p.a.codewords;
  for (int e = threadIdx.x; e < SC; e += blockDim.x) lut[e] = __ldcg(p.ws_lut + (size_t)prob * kMaxLut + e);
  __syncthreads();
  const int64_t len_t = allowed_length(p, t);
  const uint8_t* codes = p.a.codes + h * p.a.codes_head_stride;
  const int64_t i0 = (int64_t)seg * kSegKeys;
  const int64_t i1 = min(p.a.key_len, i0 + kSegKeys);
  int32_t* part = p.ws_part + (size_t)prob * p.sl_cap;
  uint2* edge = p.ws_edge + (size_t)prob * p.a.key_len;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  scan_segment<S>(p, codes, lut, t, len_t, i0, i1, [&](int64_t i, uint32_t key) {
    const uint32_t bin = key >> 20;
    const bool above = key != 0u && bin > bstar;
    const bool on = key != 0u && bin == bstar;
    const unsigned ba = __ballot_sync(0xFFFFFFFFu, above);
    const unsigned be = __ballot_sync(0xFFFFFFFFu, on);
    if ((ba | be) == 0u) return;
    uint32_t pa = 0, pe = 0;
    if (lane == 0) {
      if (ba) pa = atomicAdd(ctrl + CTRL_NOUT, static_cast<uint32_t>(__popc(ba)));
      if (be) pe = atomicAdd(ctrl + CTRL_NEDGE, static_cast<uint32_t>(__popc(be)));
    }
    pa = __shfl_sync(0xFFFFFFFFu, pa, 0);
    pe = __shfl_sync(0xFFFFFFFFu, pe, 0);
    if (above) {
      const uint32_t pos = pa + __popc(ba & lt);
      if (pos < static_cast<uint32_t>(p.sl_cap)) part[pos] = static_cast<int32_t>(i);
    }
    if (on) {
      const uint32_t pos = pe + __popc(be & lt);
      if (static_cast<int64_t>(pos) < p.a.key_len) edge[pos] = make_uint2(key, static_cast<uint32_t>(i));
    }
  });
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------

static bool pow2_float(double x) {
  int e;
  const double m = frexp(x, &e);
  return m == 0.5;
}

struct DecodePlan {
  DecodeParams p;
  size_t ws_bytes;
  size_t smem_bytes;
};

static int plan_decode(const sva_decode_args* a, DecodePlan* plan) {
  if (!a) return set_error(SVA_ERR_SHAPE, "null args");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads != 0)
    return set_error(SVA_ERR_SHAPE, "n_heads must be a positive multiple of n_kv_heads");
  if (a->n_queries <= 0) return set_error(SVA_ERR_SHAPE, "n_queries must be positive");
  if (a->head_dim <= 0 || a->head_dim > kMaxHeadDim) return set_error(SVA_ERR_SHAPE, "head_dim must be in 1..256");
  if (a->rank_dim <= 0 || a->rank_dim > kMaxRank || a->rank_dim % 4 != 0)
    return set_error(SVA_ERR_SHAPE, "rank_dim must be a multiple of 4 in 4..64");
  if (a->subspaces <= 0 || a->subspaces > kMaxSubspaces || a->rank_dim % a->subspaces != 0)
    return set_error(SVA_ERR_SHAPE, "subspaces must divide rank_dim and be <= 8");
  if (a->codewords <= 0 || a->codewords > kMaxCodewords) return set_error(SVA_ERR_SHAPE, "codewords must be in 1..256");
  if (a->subspaces * a->codewords > kMaxLut) return set_error(SVA_ERR_SHAPE, "subspaces*codewords must be <= 2048");
  if (a->key_len <= 0 || a->key_len > 0x7FFFFFFFll) return set_error(SVA_ERR_SHAPE, "key_len must be in 1..2^31-1");
  if (a->shortlist <= 0 || a->budget <= 0) return set_error(SVA_ERR_SHAPE, "shortlist and budget must be positive");
  if (a->shortlist > 16384 || a->budget > 8192) return set_error(SVA_ERR_SHAPE, "shortlist <= 16384 and budget <= 8192");
  if (a->qkv_dtype < 0 || a->qkv_dtype > 2) return set_error(SVA_ERR_DTYPE, "qkv_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
  if (!a->query || !a->q_proj || !a->scale || !a->codebooks || !a->codes || !a->k_low || !a->keys || !a->values || !a->out)
    return set_error(SVA_ERR_SHAPE, "a required pointer is null");
  DecodeParams& p = plan->p;
  memset(&p, 0, sizeof(p));
  p.a = *a;
  p.groups = a->n_heads / a->n_kv_heads;
  p.sub = a->rank_dim / a->subspaces;
  const double sr = sqrt(static_cast<double>(a->rank_dim));
  p.sqrt_r = static_cast<float>(sr);
  p.sqrt_r_pow2 = pow2_float(static_cast<double>(p.sqrt_r)) ? 1 : 0;
  p.inv_sqrt_r = 1.0f / p.sqrt_r;
  p.sl_cap = static_cast<int>(std::min<int64_t>(a->shortlist, a->key_len));
  p.b_cap = std::min(a->budget, p.sl_cap);
  const int S = a->subspaces;
  const bool vec_s = (S == 1 || S == 2 || S == 4 || S == 8);
  const uintptr_t align = static_cast<uintptr_t>(4 * S);
  p.vec_codes = (vec_s && (reinterpret_cast<uintptr_t>(a->codes) % align == 0) &&
                 (a->codes_head_stride % (4 * S)) == 0)
                    ? 1
                    : 0;
  const int64_t P = static_cast<int64_t>(a->n_heads) * a->n_queries;
  p.grid_mode = a->key_len > kFusedMaxKeys ? 1 : 0;
  p.nseg = static_cast<int>((a->key_len + kSegKeys - 1) / kSegKeys);
  const int stage_bytes = 4 * a->head_dim * a->rank_dim;
  int cache_bytes = p.grid_mode ? 8 * kEdgeSmem : std::max<int>(static_cast<int>(4 * a->key_len), stage_bytes);
  // debug outputs reuse the cache region for a 64-bit sort of up to pow2(shortlist) entries
  if (a->shortlist_out || a->final_out) {
    int cap = 1;
    while (cap < p.sl_cap) cap <<= 1;
    cache_bytes = std::max(cache_bytes, 8 * cap);
  }
  p.lay = decode_smem_layout(a->head_dim, p.sl_cap, p.b_cap, cache_bytes);
  plan->smem_bytes = static_cast<size_t>(p.lay.total);
  if (plan->smem_bytes > static_cast<size_t>(kMaxDynSmem)) return set_error(SVA_ERR_SHAPE, "shared memory plan exceeds 227 KB");
  size_t ws = 0;
  if (p.grid_mode) {
    auto take = [&](size_t bytes) {
      size_t o = ws;
      ws = (ws + bytes + 255) & ~static_cast<size_t>(255);
      return o;
    };
    const size_t o_ql = take(sizeof(float) * kMaxRank * P);
    const size_t o_lut = take(sizeof(float) * kMaxLut * P);
    const size_t o_hist = take(sizeof(uint32_t) * kBins * P);
    const size_t o_ctrl = take(sizeof(uint32_t) * CTRL_WORDS * P);
    const size_t o_part = take(sizeof(int32_t) * p.sl_cap * P);
    const size_t o_edge = take(sizeof(uint2) * static_cast<size_t>(a->key_len) * P);
    p.ws_qlow = reinterpret_cast<float*>(o_ql);
    p.ws_lut = reinterpret_cast<float*>(o_lut);
    p.ws_hist = reinterpret_cast<uint32_t*>(o_hist);
    p.ws_ctrl = reinterpret_cast<uint32_t*>(o_ctrl);
    p.ws_part = reinterpret_cast<int32_t*>(o_part);
    p.ws_edge = reinterpret_cast<uint2*>(o_edge);
  }
  plan->ws_bytes = ws;
  return SVA_OK;
}

template <int S>
static void launch_scan_kernels(const DecodeParams& p, int P, cudaStream_t stream) {
  dim3 grid(p.nseg, P);
  decode_hist_kernel<S><<<grid, kScanThreads, 0, stream>>>(p);
  profile_mark(1, stream);
  decode_collect_kernel<S><<<grid, kScanThreads, 0, stream>>>(p);
  profile_mark(2, stream);
}

template <typename T>
static int launch_decode(DecodePlan& plan, void* ws, cudaStream_t stream) {
  DecodeParams& p = plan.p;
  const int P = p.a.n_heads * p.a.n_queries;
  if (p.grid_mode) {
    char* base = static_cast<char*>(ws);
    p.ws_qlow = reinterpret_cast<float*>(base + reinterpret_cast<size_t>(p.ws_qlow));
    p.ws_lut = reinterpret_cast<float*>(base + reinterpret_cast<size_t>(p.ws_lut));
    p.ws_hist = reinterpret_cast<uint32_t*>(base + reinterpret_cast<size_t>(p.ws_hist));
    p.ws_ctrl = reinterpret_cast<uint32_t*>(base + reinterpret_cast<size_t>(p.ws_ctrl));
    p.ws_part = reinterpret_cast<int32_t*>(base + reinterpret_cast<size_t>(p.ws_part));
    p.ws_edge = reinterpret_cast<uint2*>(base + reinterpret_cast<size_t>(p.ws_edge));
    const int stage = 4 * p.a.head_dim * p.a.rank_dim;
    int rc = ensure_smem_attr(reinterpret_cast<const void*>(decode_qlut_kernel<T>), kMaxDynSmem - 16 * 1024);
    if (rc != SVA_OK) return rc;
    decode_qlut_kernel<T><<<P, 256, stage, stream>>>(p);
    profile_mark(0, stream);
    switch (p.vec_codes ? p.a.subspaces : 0) {
      case 1: launch_scan_kernels<1>(p, P, stream); break;
      case 2: launch_scan_kernels<2>(p, P, stream); break;
      case 4: launch_scan_kernels<4>(p, P, stream); break;
      case 8: launch_scan_kernels<8>(p, P, stream); break;
      default: launch_scan_kernels<0>(p, P, stream); break;
    }
  }
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(decode_problem_kernel<T>), kMaxDynSmem);
  if (rc != SVA_OK) return rc;
  decode_problem_kernel<T><<<P, kThreads, plan.smem_bytes, stream>>>(p);
  profile_mark(p.grid_mode ? 3 : 0, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

}  // namespace sva

extern "C" size_t sva_decode_workspace_size(const sva_decode_args* args) {
  sva::DecodePlan plan;
  if (sva::plan_decode(args, &plan) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_decode(const sva_decode_args* args, void* workspace, size_t workspace_bytes, void* stream) {
  sva::DecodePlan plan;
  int rc = sva::plan_decode(args, &plan);
  if (rc != SVA_OK) return rc;
  if (workspace_bytes < plan.ws_bytes || (plan.ws_bytes > 0 && workspace == nullptr))
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_decode_workspace_size()");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::launch_decode<float>(plan, workspace, s);
    case SVA_DTYPE_BF16: return sva::launch_decode<__nv_bfloat16>(plan, workspace, s);
    default: return sva::launch_decode<__half>(plan, workspace, s);
  }
}
