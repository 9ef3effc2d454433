// Scan summon -> rank rescore -> exact verify (replaces sva/llama.py:171-328).
//
// Problems are (query head h, query token t) pairs.  Two schedules:
//
// * fused  (key_len <= kFusedMaxKeys): one CTA per problem does everything.  The ADC key of
//   every allowed key is computed once into shared memory; the shortlist is an exact CTA radix
//   select over it; the CTA then rescores the shortlist against k_low, selects the budget and
//   runs the verify.  One launch per call.
//
// * grid   (longer caches), three launches:
//     prep    : one CTA per problem builds q_low and the LUT into the workspace, scores a
//               sample of 16384 keys (64 evenly spaced runs of 256) and takes the lower edge of
//               the key bin of the sample's r-th best key as a threshold T0 chosen so that about
//               2x the shortlist lies above it;
//     scan    : one CTA per segment of kScanKeys keys, the single full pass over the codes:
//               every allowed key with key >= T0 is appended to the problem's candidate list;
//     finish  : a cluster of kCluster CTAs per problem.  CTA 0 selects the exact shortlist from
//               the candidates (shared memory when they fit, else streamed from L2; if fewer
//               than `shortlist` keys reached T0 it re-selects exactly over every key and counts
//               a fallback), the rescore and the verify are split across the cluster through
//               distributed shared memory, and CTA 0 merges the fp64 partial outputs.
//   The threshold only decides how much work the finish does, never which keys are selected.
//
// Codes are read four keys per vector load (S bytes per key), four loads in flight per thread.
// Selection rule everywhere: score descending, key index ascending (see cta_select.cuh).
// ADC score: ((0 + lut[0][c0]) + lut[1][c1]) + ... in subspace order, then / sqrt(R)
// (reference sva/ops.py:64-71).  Rank score: tree_dot(k_low, q_low) / sqrt(R)
// (reference sva/llama.py:286-292).
#include <cooperative_groups.h>

#include <type_traits>

#include "cta_select.cuh"
#include "qlut.cuh"
#include "sva_internal.h"
#include "verify.cuh"

namespace sva {

namespace cg = cooperative_groups;

constexpr int kThreads = 512;
constexpr int kScanKeys = 32768;         // keys per scan CTA
constexpr int kFusedMaxKeys = 32768;
constexpr int kFusedSmallMaxKeys = 4096;  // longest cache of the fused schedule below kFusedMinProblems
constexpr int kFusedMinProblems = 148;
constexpr int kCandSmem = 12288;         // candidates selected in shared memory
constexpr int kScanThreads = 512;
constexpr int kGroupsInFlight = 4;
constexpr int kSampleRuns = 64;
constexpr int kSampleRunKeys = 256;
constexpr int kSample = kSampleRuns * kSampleRunKeys;
constexpr int kPrepCtas = 4;                // prep CTAs per problem, each samples kSample / kPrepCtas keys
constexpr int kPrepGroups = kSample / kPrepCtas / 4 / kThreads;  // 4-key sample groups per prep thread
constexpr int kPrepSmemLimit = 200 * 1024;  // dynamic shared memory of the prep kernel
constexpr int kCluster = 8;
constexpr int kScanLocalCands = 1024;
constexpr int kRepEntries = 256;  // largest S * C of the bank-replicated scan LUT
constexpr int kMinPageKeys = 64;  // smallest page of a paged catalog (a power of two)

// Control words per problem: the candidate count, the largest candidate key, and one threshold
// per prep CTA (the scan's threshold T0 is their minimum).
enum { CTRL_NCAND = 0, CTRL_MAXKEY, CTRL_T0, CTRL_WORDS = CTRL_T0 + kPrepCtas + 2 };

__device__ __forceinline__ uint32_t read_t0(const uint32_t* ctrl) {
  uint32_t t0 = __ldcg(ctrl + CTRL_T0);
#pragma unroll
  for (int c = 1; c < kPrepCtas; ++c) t0 = min(t0, __ldcg(ctrl + CTRL_T0 + c));
  return t0;
}

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
  s.acc = o;     o = align16(o + 8 * ((kThreads / 32) * 64 + kMaxHeadDim));
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
  int prep_rep;   // the prep kernel's sample lookups use a bank-replicated LUT
  int kv_stage;   // the finish kernel stages the shortlist's K and V rows in shared memory
  int q_host;     // the query is in page-locked host memory (not written by the kernels before)
  // batch layout (sva_decode_batched; sva_decode is one unpaged sequence).  Problem prob is
  // (sequence b, head h, token t) with prob = (b * H + h) * T + t.  Key l of sequence b lives on
  // "page" page_of(b, l), row l & page_mask of it: with a page table, page_table[b][l >> shift];
  // without one the page is the sequence itself (shift 62), so the page strides are then the
  // per-sequence strides.
  int batched;                // launched through sva_decode_batched (kernels instantiated with kB)
  int n_seqs;
  int n_probs;                // n_seqs * n_heads * n_queries
  const int64_t* seq_lens;    // [n_seqs] keys per sequence, or NULL (key_len each)
  int64_t q_seq_stride, out_seq_stride;
  const int32_t* page_table;  // [n_seqs][pt_stride] or NULL
  int64_t pt_stride;
  int page_shift;
  int64_t page_mask;
  int64_t codes_page_stride, k_low_page_stride, k_page_stride, v_page_stride;
  DecodeSmem lay;
  float* ws_qlow;
  float* ws_lut;
  uint32_t* ws_ctrl;
  uint2* ws_cand;  // [P][key_len] (key32, index)
  unsigned long long* dbg_ts;  // optional phase timestamps (measurement only)
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Records a phase timestamp for problem `prob` (slot < 16) when the timestamp hook is set.
__device__ __forceinline__ void stamp(const DecodeParams& p, int prob, int slot) {
  if (p.dbg_ts) p.dbg_ts[(size_t)prob * 16 + slot] = global_ns();
}

// ---------------------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------------------

__host__ __device__ __forceinline__ int64_t imin64(int64_t x, int64_t y) { return x < y ? x : y; }

// Out of line: the division's instruction sequence is not repeated at every unrolled call site.
__device__ __noinline__ float div_rn_outlined(float a, float b) { return __fdiv_rn(a, b); }

__device__ __forceinline__ float finish_score(float sum, const DecodeParams& p) {
  return p.sqrt_r_pow2 ? __fmul_rn(sum, p.inv_sqrt_r) : div_rn_outlined(sum, p.sqrt_r);
}

// (sequence, head, token) of problem `prob`.
struct ProbIdx {
  int b, h, t;
};

// Layout helpers.  kB (batch layout) is a compile-time flag of the kernels: the single-sequence
// instantiations (sva_decode, the shards) compile none of the batch / page arithmetic; the
// batched ones (sva_decode_batched) follow the layout described at DecodeParams.
template <bool kB>
__device__ __forceinline__ ProbIdx prob_index(const DecodeParams& p, int prob) {
  const int T = p.a.n_queries;
  ProbIdx r;
  if constexpr (kB) {
    const int HT = p.a.n_heads * T;
    r.b = prob / HT;
    const int rem = prob - r.b * HT;
    r.h = rem / T;
    r.t = rem - r.h * T;
  } else {
    r.b = 0;
    r.h = prob / T;
    r.t = prob - r.h * T;
  }
  return r;
}

// Keys of sequence b.
template <bool kB>
__device__ __forceinline__ int64_t seq_keys(const DecodeParams& p, int b) {
  if (!kB || !p.seq_lens) return p.a.key_len;
  const int64_t n = __ldg(p.seq_lens + b);
  return n < 0 ? 0 : (n > p.a.key_len ? p.a.key_len : n);
}

template <bool kB>
__device__ __forceinline__ int64_t allowed_length(const DecodeParams& p, int b, int t) {
  const int64_t L = seq_keys<kB>(p, b);
  const int64_t row = kB ? (int64_t)b * p.a.n_queries + t : t;
  int64_t n = p.a.allowed_len ? p.a.allowed_len[row] : (L - p.a.n_queries + t + 1);
  return n < 0 ? 0 : (n > L ? L : n);
}

template <bool kB>
__device__ __forceinline__ bool key_allowed(const DecodeParams& p, int b, int t, int64_t i, int64_t len_t) {
  if (i >= len_t) return false;
  const int64_t row = kB ? (int64_t)b * p.a.n_queries + t : t;
  if (p.a.allowed_mask) return p.a.allowed_mask[row * p.a.mask_row_stride + i] != 0;
  return true;
}

// Page of key l of sequence b (the sequence itself when there is no page table).
__device__ __forceinline__ int64_t page_of(const DecodeParams& p, int b, int64_t l) {
  return p.page_table ? static_cast<int64_t>(__ldg(p.page_table + b * p.pt_stride + (l >> p.page_shift))) : b;
}

// Base addresses of head h of sequence b: with a page table the pool's head base (pages are
// added per key); without one the sequence's own rows.
template <bool kB>
__device__ __forceinline__ const uint8_t* codes_base(const DecodeParams& p, int b, int h) {
  const uint8_t* base = p.a.codes + h * p.a.codes_head_stride;
  if constexpr (kB) base += p.page_table ? 0 : b * p.codes_page_stride;
  return base;
}
template <bool kB>
__device__ __forceinline__ const float* k_low_base(const DecodeParams& p, int b, int h) {
  const float* base = p.a.k_low + h * p.a.k_low_head_stride;
  if constexpr (kB) base += p.page_table ? 0 : b * p.k_low_page_stride;
  return base;
}
template <typename T, bool kB>
__device__ __forceinline__ const T* keys_base(const DecodeParams& p, int b, int kvh) {
  const T* base = reinterpret_cast<const T*>(p.a.keys) + kvh * p.a.k_head_stride;
  if constexpr (kB) base += p.page_table ? 0 : b * p.k_page_stride;
  return base;
}
template <typename T, bool kB>
__device__ __forceinline__ const T* values_base(const DecodeParams& p, int b, int kvh) {
  const T* base = reinterpret_cast<const T*>(p.a.values) + kvh * p.a.v_head_stride;
  if constexpr (kB) base += p.page_table ? 0 : b * p.v_page_stride;
  return base;
}

// Row addresses of key l from those bases.
template <bool kB>
__device__ __forceinline__ const uint8_t* key_codes(const DecodeParams& p, const uint8_t* base, int b, int64_t l) {
  if constexpr (kB) {
    if (p.page_table) return base + page_of(p, b, l) * p.codes_page_stride + (l & p.page_mask) * p.a.subspaces;
  }
  return base + l * p.a.subspaces;
}
template <bool kB>
__device__ __forceinline__ const float* key_k_low(const DecodeParams& p, const float* base, int b, int64_t l) {
  if constexpr (kB) {
    if (p.page_table) return base + page_of(p, b, l) * p.k_low_page_stride + (l & p.page_mask) * p.a.rank_dim;
  }
  return base + l * p.a.rank_dim;
}
template <typename T, bool kB>
__device__ __forceinline__ const T* key_row(const DecodeParams& p, const T* base, int b, int64_t l, int64_t page_stride,
                                            int64_t row_stride) {
  if constexpr (kB) {
    if (p.page_table) return base + page_of(p, b, l) * page_stride + (l & p.page_mask) * row_stride;
  }
  return base + l * row_stride;
}

// K (or V) row functors of the verify functions over key indices rows[j] of sequence b.
template <typename T, bool kB>
struct KeyRows {
  const DecodeParams* p;
  const T* base;
  const int32_t* rows;
  int b;
  int64_t page_stride, row_stride;
  __device__ __forceinline__ const T* operator()(int j) const {
    return key_row<T, kB>(*p, base, b, rows[j], page_stride, row_stride);
  }
};

template <typename T, bool kB>
__device__ __forceinline__ KeyRows<T, kB> k_rows(const DecodeParams& p, int b, int kvh, const int32_t* rows) {
  return KeyRows<T, kB>{&p, keys_base<T, kB>(p, b, kvh), rows, b, p.k_page_stride, p.a.k_row_stride};
}
template <typename T, bool kB>
__device__ __forceinline__ KeyRows<T, kB> v_rows(const DecodeParams& p, int b, int kvh, const int32_t* rows) {
  return KeyRows<T, kB>{&p, values_base<T, kB>(p, b, kvh), rows, b, p.v_page_stride, p.a.v_row_stride};
}

// Query and output rows of problem (b, h, t).
template <typename T, bool kB>
__device__ __forceinline__ const T* query_row(const DecodeParams& p, int b, int h, int t) {
  const T* q = reinterpret_cast<const T*>(p.a.query) + h * p.a.q_head_stride + t * p.a.q_row_stride;
  if constexpr (kB) q += b * p.q_seq_stride;
  return q;
}
template <typename T, bool kB>
__device__ __forceinline__ T* out_row(const DecodeParams& p, int b, int h, int t) {
  T* o = reinterpret_cast<T*>(p.a.out) + h * p.a.out_head_stride + t * p.a.out_row_stride;
  if constexpr (kB) o += b * p.out_seq_stride;
  return o;
}

// Ordered ADC key of key i (0 when not allowed), scalar code loads; `codes` from codes_base.
template <bool kB>
__device__ __forceinline__ uint32_t adc_key(const DecodeParams& p, const uint8_t* __restrict__ codes,
                                            const float* __restrict__ lut, int b, int t, int64_t i, int64_t len_t) {
  if (!key_allowed<kB>(p, b, t, i, len_t)) return 0u;
  const int S = p.a.subspaces, C = p.a.codewords;
  const uint8_t* row = key_codes<kB>(p, codes, b, i);
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
    r.a.x = __ldcs(reinterpret_cast<const uint32_t*>(base + i));
  } else if (S == 2) {
    const uint2 w = __ldcs(reinterpret_cast<const uint2*>(base + 2 * i));
    r.a.x = w.x;
    r.a.y = w.y;
  } else if (S == 4) {
    r.a = __ldcs(reinterpret_cast<const uint4*>(base + 4 * i));
  } else {
    r.a = __ldcs(reinterpret_cast<const uint4*>(base + 8 * i));
    r.b = __ldcs(reinterpret_cast<const uint4*>(base + 8 * i + 16));
  }
  return r;
}

// The same from shared memory (plain loads; the read-only path cannot address shared memory).
template <int S>
__device__ __forceinline__ Codes4<S> load_codes4_shared(const uint8_t* base, int i) {
  Codes4<S> r;
  if (S == 1) {
    r.a.x = *reinterpret_cast<const uint32_t*>(base + i);
  } else if (S == 2) {
    const uint2 w = *reinterpret_cast<const uint2*>(base + 2 * i);
    r.a.x = w.x;
    r.a.y = w.y;
  } else if (S == 4) {
    r.a = *reinterpret_cast<const uint4*>(base + 4 * i);
  } else {
    r.a = *reinterpret_cast<const uint4*>(base + 8 * i);
    r.b = *reinterpret_cast<const uint4*>(base + 8 * i + 16);
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

// Plain-layout ADC sum of key j (C == 0: the runtime codeword count Crt).
template <int S, int C>
__device__ __forceinline__ float adc_plain(const Codes4<S>& c, int j, const float* lut, int Crt) {
  const int cw = C > 0 ? C : Crt;
  float sum = lut[code_at<S>(c, j, 0)];
#pragma unroll
  for (int s2 = 1; s2 < S; ++s2) sum = __fadd_rn(sum, lut[s2 * cw + code_at<S>(c, j, s2)]);
  return sum;
}

template <typename T, bool kB>
__device__ void build_qlut(const DecodeParams& p, int prob, int b, int h, int t, float* qf, float* ql, float* lut,
                           float* stage) {
  const int D = p.a.head_dim, R = p.a.rank_dim, S = p.a.subspaces, C = p.a.codewords;
  const T* q = query_row<T, kB>(p, b, h, t);
  const float* lo = p.a.lut_override ? p.a.lut_override + (size_t)prob * S * C : nullptr;
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
// fused schedule: one CTA per problem (key_len <= kFusedMaxKeys)
// ---------------------------------------------------------------------------------------

// Rank keys of shortlist rows [0, n): two rows per warp step (one per half-warp), U steps in
// flight.  `rows` are key indices; rk[j] receives the ordered rank score of rows[j].  Each
// thread calls after_first_loads() once, after issuing its first round of row loads and before
// using them (so that other gathers can be issued while those are in flight).  Ends with a
// barrier.
struct NoHook {
  __device__ void operator()() const {}
};

template <int U, bool kB, class Hook = NoHook>
__device__ void rescore_rows(const DecodeParams& p, int b, int h, const float* ql, const int32_t* rows, int n,
                             uint32_t* rk, const Hook& after_first_loads = Hook()) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int half = lane >> 4, l16 = lane & 15;
  const int R = p.a.rank_dim;
  const float4 q4 = (4 * l16 < R) ? make_float4(ql[4 * l16], ql[4 * l16 + 1], ql[4 * l16 + 2], ql[4 * l16 + 3])
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
  const float* klb = k_low_base<kB>(p, b, h);
  float4 r[U];
  auto load = [&](int base) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + 2 * u + half;
      r[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < n && 4 * l16 < R) r[u] = load4<float>(key_k_low<kB>(p, klb, b, rows[j]), 4 * l16, R);
    }
  };
  int base = warp * 2 * U;
  load(base);
  after_first_loads();
  for (;;) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + 2 * u + half;
      const float s = tree16(lane4(r[u], q4));
      if (j < n && l16 == 0) rk[j] = ordered_key(finish_score(s, p));
    }
    base += nwarps * 2 * U;
    if (base >= n) break;
    load(base);
  }
  __syncthreads();
}

// Block copy of n candidates (coarse key, index) from global memory into shared memory as
// select composites (key << 32 | ~index), 16 loads in flight per thread; ends with a barrier.
__device__ inline void copy_batched(unsigned long long* dst, const uint2* src, int n) {
  constexpr int U = 16;
  for (int base = 0; base < n; base += blockDim.x * U) {
    uint2 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + threadIdx.x + u * blockDim.x;
      if (i < n) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + threadIdx.x + u * blockDim.x;
      if (i < n) dst[i] = composite(v[u].x, v[u].y);
    }
  }
  __syncthreads();
}

// Ascending copies of the shortlist / final index sets for the debug outputs.
__device__ void write_sorted(const int32_t* src, int n, int width, int32_t* dst, unsigned long long* tmp) {
  int cap = 1;
  while (cap < n) cap <<= 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) tmp[i] = static_cast<unsigned long long>(static_cast<uint32_t>(src[i]));
  __syncthreads();
  cta_bitonic_sort_u64(tmp, n, cap);
  for (int i = threadIdx.x; i < width; i += blockDim.x) dst[i] = (i < n) ? static_cast<int32_t>(tmp[i]) : -1;
  __syncthreads();
}

template <typename T, bool kB>
__global__ void __launch_bounds__(kThreads) decode_fused_kernel(const DecodeParams p) {
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
  uint32_t* cache = reinterpret_cast<uint32_t*>(smem + p.lay.cache);

  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int kvh = h / p.groups;
  const int64_t L = seq_keys<kB>(p, b);
  const int64_t len_t = allowed_length<kB>(p, b, t);
  const uint8_t* codes = codes_base<kB>(p, b, h);
  const int tid = threadIdx.x;

  build_qlut<T, kB>(p, prob, b, h, t, qf, ql, lut, reinterpret_cast<float*>(cache));
  int nv = 0;
  for (int64_t i = tid; i < L; i += blockDim.x) {
    const uint32_t key = adc_key<kB>(p, codes, lut, b, t, i, len_t);
    cache[i] = key;
    nv += (key != 0u);
  }
  const int n_valid = block_sum_int(nv, scratch);
  const int k = min(p.sl_cap, n_valid);
  int n_sl;
  {
    auto item = [&](int i) -> unsigned long long {
      return cache[i] ? composite(cache[i], static_cast<uint32_t>(i)) : 0ull;
    };
    const SelectThreshold thr = cta_radix_select(item, static_cast<int>(L), k, sc);
    n_sl = cta_compact(item, static_cast<int>(L), thr, [&](int pos, int i, unsigned long long) { sl[pos] = i; },
                       scratch);
  }
  rescore_rows<16, kB>(p, b, h, ql, sl, n_sl, rk);
  const int nb = min(p.b_cap, n_sl);
  int n_fin;
  {
    auto item = [&](int j) -> unsigned long long { return composite(rk[j], static_cast<uint32_t>(sl[j])); };
    const SelectThreshold thr = cta_radix_select(item, n_sl, nb, sc);
    n_fin = cta_compact(item, n_sl, thr, [&](int pos, int j, unsigned long long) { fin[pos] = sl[j]; }, scratch);
  }
  verify_rows_fn<T>(k_rows<T, kB>(p, b, kvh, fin), v_rows<T, kB>(p, b, kvh, fin), qf, p.a.head_dim, n_fin,
                    p.a.softmax_scale, p.a.logits_mode, lg, acc, scratch, out_row<T, kB>(p, b, h, t));
  unsigned long long* tmp = reinterpret_cast<unsigned long long*>(cache);
  if (p.a.shortlist_out) write_sorted(sl, n_sl, p.a.shortlist, p.a.shortlist_out + (size_t)prob * p.a.shortlist, tmp);
  if (p.a.final_out) write_sorted(fin, n_fin, p.a.budget, p.a.final_out + (size_t)prob * p.a.budget, tmp);
  if (p.a.stats && tid == 0) {
    atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
    atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
  }
}

// ---------------------------------------------------------------------------------------
// grid schedule
// ---------------------------------------------------------------------------------------

// Calls f(i, key) for every key of [i0, i1) (key = 0 when not allowed).  With S > 0 each
// thread handles groups of four consecutive keys, kGroupsInFlight vector loads at a time.
// Iteration is warp-uniform: every lane calls f the same number of times (slots past the end
// come with i == i1 and key 0), so f may use warp collectives.
// `codes` is codes_base(p, b, h); i0 is a multiple of four.
template <int S, bool kB, class F>
__device__ __forceinline__ void scan_segment(const DecodeParams& p, const uint8_t* codes, const float* lut, int b, int t,
                                             int64_t len_t, int64_t i0, int64_t i1, const F& f) {
  const int lane = threadIdx.x & 31;
  if constexpr (S > 0) {
    const int ngroups = static_cast<int>((i1 - i0 + 3) >> 2);
    const bool dense = (p.a.allowed_mask == nullptr) && (i1 <= len_t);
    for (int gb = (threadIdx.x & ~31); gb < ngroups; gb += blockDim.x * kGroupsInFlight) {
      Codes4<S> c[kGroupsInFlight];
#pragma unroll
      for (int u = 0; u < kGroupsInFlight; ++u) {
        const int g = gb + lane + u * blockDim.x;
        // a group of four keys never straddles a page (pages hold a multiple of four keys)
        if (g < ngroups && i0 + 4 * g + 3 < i1) c[u] = load_codes4<S>(key_codes<kB>(p, codes, b, i0 + 4 * g), 0);
      }
#pragma unroll
      for (int u = 0; u < kGroupsInFlight; ++u) {
        const int g = gb + lane + u * blockDim.x;
        const int64_t ib = i0 + 4 * g;
        const bool full = g < ngroups && ib + 3 < i1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t i = ib + j;
          const bool live = g < ngroups && i < i1;
          uint32_t key = 0u;
          if (full) {
            key = (dense || key_allowed<kB>(p, b, t, i, len_t)) ? adc_key4<S>(p, c[u], j, lut) : 0u;
          } else if (live) {
            key = adc_key<kB>(p, codes, lut, b, t, i, len_t);
          }
          f(live ? i : i1, key);
        }
      }
    }
  } else {
    for (int64_t wb = i0 + (threadIdx.x & ~31); wb < i1; wb += blockDim.x) {
      const int64_t i = wb + lane;
      const uint32_t key = (i < i1) ? adc_key<kB>(p, codes, lut, b, t, i, len_t) : 0u;
      f(i < i1 ? i : i1, key);
    }
  }
}

// Start key of sample group g (of kSample / 4): groups of four consecutive keys, group g lies in
// run g / (kSampleRunKeys / 4); the kSampleRuns runs are evenly spaced over the allowed range and
// start on multiples of four keys.
__device__ __forceinline__ int64_t sample_group_start(int64_t len_t, int g) {
  constexpr int kRunGroups = kSampleRunKeys / 4;
  const int run = g / kRunGroups, off = (g - run * kRunGroups) * 4;
  return ((len_t * run) / kSampleRuns & ~static_cast<int64_t>(3)) + off;
}

// Asynchronous global -> shared copy of one 4-key code group (4 * S bytes, aligned to that).
template <int S>
__device__ __forceinline__ void copy_group_async(uint8_t* dst, const uint8_t* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  if constexpr (S == 1) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(src) : "memory");
  } else if constexpr (S == 2) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(d), "l"(src) : "memory");
  } else if constexpr (S == 4) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
  } else {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d + 16), "l"(src + 16) : "memory");
  }
}

// Dynamic shared memory of a prep CTA: q_proj[h] (later the sampled keys), the codebooks of h,
// the sampled codes of the vector-code variants, and the bank-replicated LUT when S * C <=
// kRepEntries.
struct PrepSmem {
  int stage, cb, sample, rep, total;
};

__host__ __device__ inline PrepSmem prep_smem_layout(int head_dim, int rank_dim, int codewords, int S_vec, bool rep) {
  PrepSmem s;
  int o = 0;
  const int keys_bytes = 4 * 4 * kThreads * kPrepGroups;
  const int stage = 4 * head_dim * rank_dim > keys_bytes ? 4 * head_dim * rank_dim : keys_bytes;
  s.stage = o;  o = align16(o + stage);
  s.cb = o;     o = align16(o + 4 * codewords * rank_dim);
  s.sample = o; o = align16(o + 4 * kThreads * kPrepGroups * S_vec);
  s.rep = o;    o = align16(o + (rep ? 4 * 32 * kRepEntries : 0));
  s.total = o;
  return s;
}

// ADC sum of key j from a bank-replicated LUT with a runtime codeword count (codes clamped to
// the table, so a corrupt code cannot read outside it).
template <int S>
__device__ __forceinline__ float adc_rep_rt(const Codes4<S>& c, int j, const float* lut_lane, int C) {
  float sum = lut_lane[min(code_at<S>(c, j, 0), static_cast<uint32_t>(C - 1)) * 32];
#pragma unroll
  for (int s = 1; s < S; ++s)
    sum = __fadd_rn(sum, lut_lane[(s * C + min(code_at<S>(c, j, s), static_cast<uint32_t>(C - 1))) * 32]);
  return sum;
}

// 16-byte-vector copy of n floats (n % 4 == 0, both 16-byte aligned) or a scalar copy.
__device__ __forceinline__ void stage_floats(float* dst, const float* src, int n) {
  if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (n & 3) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int e = threadIdx.x; e < n / 4; e += blockDim.x) d4[e] = __ldg(s4 + e);
  } else {
    for (int e = threadIdx.x; e < n; e += blockDim.x) dst[e] = __ldg(src + e);
  }
}

// prep: q_low + LUT, and the sampled thresholds.  kPrepCtas CTAs per problem; CTA `part` scores
// the sample groups [part * kThreads * kPrepGroups, ...) (kSample / kPrepCtas keys) and writes
// T0_part, a lower bound of the r-th best of its sampled keys with r = ceil(2 * shortlist *
// n_part / len), n_part its number of allowed sampled keys.  The scan keeps keys >= T0 = min
// over parts: at least sum(r) >= 2 * shortlist * n / len keys of the whole sample are >= T0, so
// about twice the shortlist is expected among all keys, and fewer than the shortlist only if
// every part's estimate errs high together.  T0 only sizes the candidate set: if fewer keys
// than the shortlist reach it, the finish kernel selects over every key.  The bound is the lower
// edge of the bin below the one holding the r-th best key, in 1024 equal-width bins over the
// part's sampled score range (one counting pass, no exact select).  Every part computes q_low
// and the LUT (part 0 publishes them).  Inputs that are weights (q_proj, codebooks, the sampled
// codes) are staged before waiting for the predecessor; q and every workspace write come after.
template <typename T, int S, bool kB>
__global__ void __launch_bounds__(kThreads) decode_prep_kernel(const DecodeParams p, const PrepSmem lay) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ float lut[kMaxLut];
  __shared__ SelectScratch sel;
  float* stage = reinterpret_cast<float*>(dyn + lay.stage);
  float* cbs = reinterpret_cast<float*>(dyn + lay.cb);
  uint8_t* sample = dyn + lay.sample;
  float* lut_rep = reinterpret_cast<float*>(dyn + lay.rep);
  uint32_t* skeys = reinterpret_cast<uint32_t*>(dyn + lay.stage);  // after q_low: the sampled keys
  const int prob = blockIdx.x / kPrepCtas, part = blockIdx.x - prob * kPrepCtas;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = p.a.head_dim, R = p.a.rank_dim, S2 = p.a.subspaces, C = p.a.codewords;
  const int SC = S2 * C;
  pdl_launch_dependents();  // the scan may be scheduled now; it waits for this grid's results
  if (part == 0 && tid == 0) stamp(p, prob, 0);
  // lengths, page tables and codes are the caller's inputs (like the weights), staged before the
  // wait; the query and the workspace come after it
  const int64_t len_t = allowed_length<kB>(p, b, t);
  const uint8_t* codes = codes_base<kB>(p, b, h);
  const int g_first = part * kThreads * kPrepGroups;
  if constexpr (S > 0) {
#pragma unroll
    for (int u = 0; u < kPrepGroups; ++u) {
      const int gl = tid + u * kThreads;
      const int64_t g0 = sample_group_start(len_t, g_first + gl);
      if (g0 + 3 < len_t) copy_group_async<S>(sample + gl * 4 * S, key_codes<kB>(p, codes, b, g0));
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  const float* lo = p.a.lut_override ? p.a.lut_override + (size_t)prob * SC : nullptr;
  stage_floats(stage, p.a.q_proj + (size_t)h * D * R, D * R);
  if (!lo) stage_floats(cbs, p.a.codebooks + (size_t)h * C * R, C * R);
  {
    // a query in host memory is the caller's input, not a result of the kernels before, so its
    // PCIe round trip overlaps the wait; a device query may be the previous kernel's output
    const T* q = query_row<T, kB>(p, b, h, t);
    if (p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    pdl_wait();
    if (!p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  }
  __syncthreads();
  if (tid < R) {
    const float sc_h = __ldg(p.a.scale + h);
    float acc = 0.f;
#pragma unroll 16
    for (int d = 0; d < D; ++d) acc = mac(acc, qf[d], stage[d * R + tid]);
    ql[tid] = __fmul_rn(acc, sc_h);
  }
  __syncthreads();
  // the LUT's dot products with the subspace width known at compile time for the common widths
  const int sub = R / S2;
  const bool fixed = !lo && (reinterpret_cast<uintptr_t>(cbs) & 15u) == 0;
  if (fixed && sub == 16) query_lut_fixed<16>(S2, C, cbs, ql, lut);
  else if (fixed && sub == 32) query_lut_fixed<32>(S2, C, cbs, ql, lut);
  else if (fixed && sub == 64) query_lut_fixed<64>(S2, C, cbs, ql, lut);
  else if (fixed && sub == 8) query_lut_fixed<8>(S2, C, cbs, ql, lut);
  else query_lut<true>(R, S2, C, cbs, lo, ql, lut);
  if (part == 0 && tid == 0) stamp(p, prob, 9);
  if (part == 0) {
    float* gl = p.ws_lut + (size_t)prob * kMaxLut;
    for (int e = tid; e < SC; e += blockDim.x) gl[e] = lut[e];
    for (int r = tid; r < R; r += blockDim.x) p.ws_qlow[(size_t)prob * kMaxRank + r] = ql[r];
    if (tid == 0) {
      p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_NCAND] = 0u;
      p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_MAXKEY] = 0u;
    }
  }
  const bool rep = S > 0 && p.prep_rep;
  if (rep) {
    for (int e0 = warp * 32; e0 < SC; e0 += blockDim.x) {
      const float v = (e0 + lane < SC) ? lut[e0 + lane] : 0.f;
#pragma unroll 8
      for (int k = 0; k < 32; ++k) {
        const float x = __shfl_sync(0xFFFFFFFFu, v, k);
        if (e0 + k < SC) lut_rep[(e0 + k) * 32 + lane] = x;
      }
    }
  }
  if constexpr (S > 0) asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();
  int nv = 0;
  float smin = INFINITY, smax = -INFINITY;
  const float* rep_lane = lut_rep + lane;
#pragma unroll
  for (int u = 0; u < kPrepGroups; ++u) {
    const int gl = tid + u * kThreads;
    const int64_t g0 = sample_group_start(len_t, g_first + gl);
    uint32_t k4[4];
    if (S > 0 && g0 + 3 < len_t) {
      const Codes4<(S > 0 ? S : 1)> c = load_codes4_shared<(S > 0 ? S : 1)>(sample, gl * 4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float sum = rep ? adc_rep_rt<(S > 0 ? S : 1)>(c, j, rep_lane, C)
                              : adc_plain<(S > 0 ? S : 1), 0>(c, j, lut, C);
        k4[j] = key_allowed<kB>(p, b, t, g0 + j, len_t) ? ordered_key(finish_score(sum, p)) : 0u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) k4[j] = adc_key<kB>(p, codes, lut, b, t, g0 + j, len_t);
    }
    *reinterpret_cast<uint4*>(skeys + 4 * gl) = make_uint4(k4[0], k4[1], k4[2], k4[3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (k4[j] != 0u) {
        const float sc = key_to_float(k4[j]);
        smin = fminf(smin, sc);
        smax = fmaxf(smax, sc);
        ++nv;
      }
    }
  }
  if (part == 0 && tid == 0) stamp(p, prob, 10);
  // block totals of (count, min, max) in one barrier
  nv = __reduce_add_sync(0xFFFFFFFFu, nv);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    smin = fminf(smin, __shfl_xor_sync(0xFFFFFFFFu, smin, o));
    smax = fmaxf(smax, __shfl_xor_sync(0xFFFFFFFFu, smax, o));
  }
  if (lane == 0) {
    sel.warp_tot[1][warp] = nv;
    sel.lo_part[warp] = __float_as_uint(smin);
    sel.hi_part[warp] = __float_as_uint(smax);
  }
  for (int b = tid; b < kSelectBins; b += blockDim.x) sel.hist[0][b] = 0u;
  __syncthreads();
  {
    const int nw = blockDim.x >> 5;
    int c = lane < nw ? sel.warp_tot[1][lane] : 0;
    float a = lane < nw ? __uint_as_float(static_cast<uint32_t>(sel.lo_part[lane])) : INFINITY;
    float b = lane < nw ? __uint_as_float(static_cast<uint32_t>(sel.hi_part[lane])) : -INFINITY;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a = fminf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
      b = fmaxf(b, __shfl_xor_sync(0xFFFFFFFFu, b, o));
    }
    nv = c;
    smin = a;
    smax = b;
  }
  const int n_s = nv;
  const int64_t k_est = imin64(p.sl_cap, len_t);
  const int64_t r = len_t > 0 ? (2 * k_est * n_s + len_t - 1) / len_t : 0;
  uint32_t t0 = 1u;
  const float span = smax - smin;
  if (n_s > 0 && r >= 1 && r < n_s && isfinite(span)) {
    if (!(span > 0.f)) {
      t0 = ordered_key(smin);
    } else {
      const float scale = (static_cast<float>(kSelectBins) - 0.5f) / span;
      uint32_t* hist = sel.hist[0];
      for (int i = tid; i < 4 * kThreads * kPrepGroups; i += blockDim.x) {
        const uint32_t kk = skeys[i];
        if (kk != 0u) {
          const float x = __fmul_rn(__fsub_rn(key_to_float(kk), smin), scale);
          atomicAdd(&hist[x > 0.f ? static_cast<int>(fminf(x, static_cast<float>(kSelectBins - 1))) : 0], 1u);
        }
      }
      __syncthreads();
      (void)select_find_bin(hist, static_cast<int>(r), &sel, 0);
      const int bstar = sel.digit[0];
      t0 = ordered_key(bstar >= 1 ? __fadd_rn(smin, __fdiv_rn(static_cast<float>(bstar - 1), scale)) : smin);
    }
  }
  if (tid == 0) {
    p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_T0 + part] = t0 > 1u ? t0 : 1u;
    if (part == 0) stamp(p, prob, 1);
  }
}

// Wide prep: one CTA per problem, for launches with many problems.  The 4-CTA prep above stages
// its inputs in ~200 KB of shared memory per CTA to minimise the latency of a single decode; with
// hundreds of problems per launch that leaves one CTA per SM.  Here each problem's q_low and LUT
// come out of the same canonical arithmetic with the weights read from L2, and the threshold from
// a sample of kWideSample keys (kWideRuns evenly spaced runs), so a CTA needs ~50 KB and several
// problems share an SM.  The threshold rule is the 4-CTA prep's with one part and one extra rank
// of margin for the smaller sample; as there, it only sizes the candidate set.
constexpr int kWidePrepThreads = 256;
constexpr int kWideRuns = 64;
constexpr int kWideRunKeys = 128;
constexpr int kWideSample = kWideRuns * kWideRunKeys;

__host__ __device__ inline int wide_prep_smem_bytes() {
  return static_cast<int>(sizeof(SelectScratch)) + 4 * (kMaxHeadDim + kMaxRank + kMaxLut + kWideSample);
}

template <typename T, bool kB, int NT = kWidePrepThreads>
__global__ void __launch_bounds__(NT, NT >= 512 ? 1 : 2) decode_prep_wide_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) unsigned char wdyn[];
  SelectScratch& sel = *reinterpret_cast<SelectScratch*>(wdyn);
  float* qf = reinterpret_cast<float*>(wdyn + sizeof(SelectScratch));
  float* ql = qf + kMaxHeadDim;
  float* lut = ql + kMaxRank;
  uint32_t* skeys = reinterpret_cast<uint32_t*>(lut + kMaxLut);
  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = p.a.head_dim, R = p.a.rank_dim, S2 = p.a.subspaces, C = p.a.codewords;
  const int SC = S2 * C;
  pdl_launch_dependents();
  const int64_t len_t = allowed_length<kB>(p, b, t);
  const uint8_t* codes = codes_base<kB>(p, b, h);
  {
    const T* q = query_row<T, kB>(p, b, h, t);
    if (p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    pdl_wait();
    if (!p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  }
  __syncthreads();
  if (tid == 0) stamp(p, prob, 0);
  const float* qp = p.a.q_proj + (size_t)h * D * R;
  for (int r = tid; r < R; r += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = mac(acc, qf[d], __ldg(qp + d * R + r));
    ql[r] = __fmul_rn(acc, __ldg(p.a.scale + h));
  }
  __syncthreads();
  const float* lo = p.a.lut_override ? p.a.lut_override + (size_t)prob * SC : nullptr;
  query_lut<false>(R, S2, C, p.a.codebooks + (size_t)h * C * R, lo, ql, lut);
  {
    float* gl = p.ws_lut + (size_t)prob * kMaxLut;
    for (int e = tid; e < SC; e += blockDim.x) gl[e] = lut[e];
    for (int r = tid; r < R; r += blockDim.x) p.ws_qlow[(size_t)prob * kMaxRank + r] = ql[r];
    if (tid == 0) {
      p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_NCAND] = 0u;
      p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_MAXKEY] = 0u;
    }
  }
  if (tid == 0) stamp(p, prob, 9);
  // sample: kWideRuns runs of kWideRunKeys keys evenly spaced over the allowed range
  int nv = 0;
  float smin = INFINITY, smax = -INFINITY;
  auto sample_key = [&](int i) -> int64_t {
    const int run = i / kWideRunKeys, off = i - run * kWideRunKeys;
    return ((len_t * run) / kWideRuns) + off;
  };
  auto note = [&](int i, uint32_t k) {
    skeys[i] = k;
    if (k != 0u) {
      const float sc = key_to_float(k);
      smin = fminf(smin, sc);
      smax = fmaxf(smax, sc);
      ++nv;
    }
  };
  if (S2 == 4 && p.vec_codes && p.a.allowed_mask == nullptr) {
    // four subspaces, rows 4-byte aligned: a thread loads the code words of kBatch sample keys
    // before scoring any of them, so their latencies overlap (same sum as adc_key)
    constexpr int kPer = kWideSample / NT;
    constexpr int kBatch = kPer < 16 ? kPer : 16;
    for (int m0 = 0; m0 < kPer; m0 += kBatch) {
      uint32_t w[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t key = sample_key(tid + (m0 + u) * NT);
        w[u] = key < len_t ? __ldg(reinterpret_cast<const uint32_t*>(key_codes<kB>(p, codes, b, key))) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = tid + (m0 + u) * NT;
        uint32_t k = 0u;
        if (sample_key(i) < len_t) {
          float sum = 0.f;
#pragma unroll
          for (int s = 0; s < 4; ++s) sum = __fadd_rn(sum, lut[s * C + ((w[u] >> (8 * s)) & 0xFFu)]);
          k = ordered_key(finish_score(sum, p));
        }
        note(i, k);
      }
    }
  } else {
    for (int i = tid; i < kWideSample; i += blockDim.x) {
      const int64_t key = sample_key(i);
      note(i, (key < len_t) ? adc_key<kB>(p, codes, lut, b, t, key, len_t) : 0u);
    }
  }
  if (tid == 0) stamp(p, prob, 10);
  nv = __reduce_add_sync(0xFFFFFFFFu, nv);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    smin = fminf(smin, __shfl_xor_sync(0xFFFFFFFFu, smin, o));
    smax = fmaxf(smax, __shfl_xor_sync(0xFFFFFFFFu, smax, o));
  }
  if (lane == 0) {
    sel.warp_tot[1][warp] = nv;
    sel.lo_part[warp] = __float_as_uint(smin);
    sel.hi_part[warp] = __float_as_uint(smax);
  }
  for (int bn = tid; bn < kSelectBins; bn += blockDim.x) sel.hist[0][bn] = 0u;
  __syncthreads();
  {
    const int nw = blockDim.x >> 5;
    int c = lane < nw ? sel.warp_tot[1][lane] : 0;
    float a = lane < nw ? __uint_as_float(static_cast<uint32_t>(sel.lo_part[lane])) : INFINITY;
    float bb = lane < nw ? __uint_as_float(static_cast<uint32_t>(sel.hi_part[lane])) : -INFINITY;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a = fminf(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
      bb = fmaxf(bb, __shfl_xor_sync(0xFFFFFFFFu, bb, o));
    }
    nv = c;
    smin = a;
    smax = bb;
  }
  // samples can repeat keys when the range is shorter than the sample; they only size the set
  const int n_s = nv;
  const int64_t k_est = imin64(p.sl_cap, len_t);
  const int64_t r = len_t > 0 ? (2 * k_est * n_s + len_t - 1) / len_t + 1 : 0;
  uint32_t t0 = 1u;
  const float span = smax - smin;
  if (n_s > 0 && r >= 1 && r < n_s && len_t > kWideSample && isfinite(span)) {
    if (!(span > 0.f)) {
      t0 = ordered_key(smin);
    } else {
      const float scale = (static_cast<float>(kSelectBins) - 0.5f) / span;
      uint32_t* hist = sel.hist[0];
      for (int i = tid; i < kWideSample; i += blockDim.x) {
        const uint32_t kk = skeys[i];
        if (kk != 0u) {
          const float x = __fmul_rn(__fsub_rn(key_to_float(kk), smin), scale);
          atomicAdd(&hist[x > 0.f ? static_cast<int>(fminf(x, static_cast<float>(kSelectBins - 1))) : 0], 1u);
        }
      }
      __syncthreads();
      (void)select_find_bin(hist, static_cast<int>(r), &sel, 0);
      const int bstar = sel.digit[0];
      t0 = ordered_key(bstar >= 1 ? __fadd_rn(smin, __fdiv_rn(static_cast<float>(bstar - 1), scale)) : smin);
    }
  }
  if (tid < kPrepCtas) p.ws_ctrl[(size_t)prob * CTRL_WORDS + CTRL_T0 + tid] = t0 > 1u ? t0 : 1u;
  if (tid == 0) stamp(p, prob, 1);
}

// LUT lookup of key j in the bank-replicated table: entry e lives at lut[e * 32 + lane], so
// the 32 lanes of a warp read 32 different banks whatever their codes are.  C is a power of
// two; codes are masked to it (a valid catalog never holds a code >= C).  The byte offset of a
// lookup, code * 128 + lane * 4, is built from the code's byte in its 32-bit word with one
// shift and one and-or (the lane bits 2..6 and the code bits 7.. do not overlap); the
// subspace's table base is a constant offset.
template <int S>
__device__ __forceinline__ void code_pos(const Codes4<S>& c, int j, int s, uint32_t& word, int& byte) {
  if (S == 1) {
    word = c.a.x;
    byte = j;
  } else if (S == 2) {
    word = (j < 2) ? c.a.x : c.a.y;
    byte = 2 * (j & 1) + s;
  } else if (S == 4) {
    word = (j == 0) ? c.a.x : (j == 1) ? c.a.y : (j == 2) ? c.a.z : c.a.w;
    byte = s;
  } else {
    const uint4& v = (j < 2) ? c.a : c.b;
    word = ((j & 1) == 0) ? (s < 4 ? v.x : v.y) : (s < 4 ? v.z : v.w);
    byte = s & 3;
  }
}

// ld.shared.f32 at a 32-bit shared address plus a compile-time offset.
template <int OFF>
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(addr), "n"(OFF));
  return v;
}

// kOr: the table's shared address has no bit in common with the code field or 4 * lane, so the
// offset is one and-or of the shifted word (else an and, then an add).
template <int S, int C, int s, bool kOr>
__device__ __forceinline__ float adc_rep_from(const Codes4<S>& c, int j, uint32_t lane_base, float sum) {
  if constexpr (s == S) {
    return sum;
  } else {
    constexpr uint32_t kMask = static_cast<uint32_t>(C - 1) << 7;
    uint32_t w;
    int byte;
    code_pos<S>(c, j, s, w, byte);
    const int sh = 8 * byte - 7;  // compile-time after unrolling
    const uint32_t x = sh >= 0 ? (w >> sh) : (w << -sh);
    const uint32_t off = kOr ? ((x & kMask) | lane_base) : ((x & kMask) + lane_base);
    const float v = lds_f32<s * C * 128>(off);
    return adc_rep_from<S, C, s + 1, kOr>(c, j, lane_base, s == 0 ? v : __fadd_rn(sum, v));
  }
}

// lane_base = shared address of the replicated table + 4 * lane.
template <int S, int C, bool kOr = false>
__device__ __forceinline__ float adc_rep(const Codes4<S>& c, int j, uint32_t lane_base) {
  return adc_rep_from<S, C, 0, kOr>(c, j, lane_base, 0.f);
}

// scan: the single pass over the codes; keys >= T0 become candidates.  One CTA scans
// kScanKeys keys of one problem.  For the common codebook shapes (S * C <= 256, C a power of
// two) the LUT is replicated 32 times across the banks, so the random lookups are free of bank
// conflicts; the score of every key is the canonical sequential fp32 sum.  Candidates are rare
// (about 2x the shortlist among all keys), so each one takes a shared atomic of its own and the
// CTA publishes its list with one global atomic.
template <int S, int C, bool POW2, bool PAGED>
__global__ void __launch_bounds__(kScanThreads, 2) decode_scan_kernel(const DecodeParams p) {
  constexpr bool kRep = (S > 0) && (C > 0) && (S * C <= kRepEntries);
  // the LUT lives in dynamic shared memory (scan_lut_bytes), its start rounded up at run time to
  // a multiple of its row field so that lookups can or the lane into the offset
  extern __shared__ __align__(16) unsigned char scan_dyn[];
  __shared__ uint2 local[kScanLocalCands];  // this CTA's candidates, flushed with one atomic
  __shared__ uint32_t n_local;
  __shared__ uint32_t flush_base;
  __shared__ uint32_t max_key;
  __shared__ uint32_t seg_pages[PAGED ? kScanKeys / kMinPageKeys : 1];  // page table of this segment
  const int prob = blockIdx.y, seg = blockIdx.x;
  const ProbIdx pi = prob_index<true>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr uint32_t kLutAlign = kRep ? static_cast<uint32_t>(C > 0 ? C : 1) * 128u : 16u;
  const uint32_t dyn_base = static_cast<uint32_t>(__cvta_generic_to_shared(scan_dyn));
  float* lut = reinterpret_cast<float*>(scan_dyn + ((kLutAlign - (dyn_base & (kLutAlign - 1u))) & (kLutAlign - 1u)));
  pdl_launch_dependents();
  pdl_wait();  // prep's LUT, q_low and threshold
  uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
  const uint32_t t0 = read_t0(ctrl);
  const int SC = p.a.subspaces * p.a.codewords;
  const float* glut = p.ws_lut + (size_t)prob * kMaxLut;
  const int64_t len_t = allowed_length<true>(p, b, t);
  const int64_t i0 = (int64_t)seg * kScanKeys;
  const int64_t i1 = min(len_t, i0 + kScanKeys);
  if (i0 >= i1) return;  // uniform over the block
  if constexpr (PAGED) {
    // segments start on a page boundary (kScanKeys is a multiple of the page size)
    const int np = static_cast<int>(((i1 - i0) + p.page_mask) >> p.page_shift);
    const int32_t* pt = p.page_table + b * p.pt_stride + (i0 >> p.page_shift);
    for (int e = tid; e < np; e += blockDim.x) seg_pages[e] = static_cast<uint32_t>(__ldg(pt + e));
  }
  const bool fast = (S > 0) && p.a.allowed_mask == nullptr && ((i1 - i0) & 3) == 0;
  if (kRep && fast) {
    // warp w fills entries w*32 .. w*32+31 (+ multiples of blockDim.x); lane l writes copy l
    for (int e0 = warp * 32; e0 < SC; e0 += blockDim.x) {
      const float v = (e0 + lane < SC) ? __ldcg(glut + e0 + lane) : 0.f;
#pragma unroll 8
      for (int k = 0; k < 32; ++k) {
        const float x = __shfl_sync(0xFFFFFFFFu, v, k);
        if (e0 + k < SC) lut[(e0 + k) * 32 + lane] = x;
      }
    }
  } else {
    for (int e = tid; e < SC; e += blockDim.x) lut[e] = __ldcg(glut + e);
  }
  if (tid == 0) {
    n_local = 0u;
    max_key = 0u;
  }
  __syncthreads();
  const uint8_t* codes = codes_base<true>(p, b, h);
  uint2* cand = p.ws_cand + (size_t)prob * p.a.key_len;
  uint32_t my_max = 0u;  // largest key this thread took
  auto take = [&](uint32_t key, int64_t i) {
    my_max = max(my_max, key);
    const uint32_t pos = atomicAdd(&n_local, 1u);
    if (pos < static_cast<uint32_t>(kScanLocalCands)) {
      local[pos] = make_uint2(key, static_cast<uint32_t>(i));
    } else {
      const uint32_t g = atomicAdd(ctrl + CTRL_NCAND, 1u);
      if (static_cast<int64_t>(g) < p.a.key_len) cand[g] = make_uint2(key, static_cast<uint32_t>(i));
    }
  };
  if constexpr (S > 0) {
    if (fast) {
      const float t0f = (t0 <= 1u) ? -INFINITY : key_to_float(t0);
      const float scale = p.inv_sqrt_r;
      const int ngroups = static_cast<int>((i1 - i0) >> 2);
      const uint8_t* cbase = codes + i0 * S;
      // codes of the 4-key group g of the segment (groups never straddle a page)
      auto group_codes = [&](int g) -> Codes4<S> {
        if constexpr (PAGED) {
          const int k = 4 * g;
          return load_codes4<S>(codes + static_cast<int64_t>(seg_pages[k >> p.page_shift]) * p.codes_page_stride +
                                    static_cast<int64_t>(k & static_cast<int>(p.page_mask)) * S,
                                0);
        } else {
          return load_codes4<S>(cbase, 4 * g);
        }
      };
      const uint32_t lut_base = static_cast<uint32_t>(__cvta_generic_to_shared(lut));
      const uint32_t lane_base = lut_base + static_cast<uint32_t>(lane) * 4u;
      // the and-or offset needs a table address with no bit in the code field or below it
      const bool or_ok = kRep && (lut_base & ((static_cast<uint32_t>(C > 0 ? C : 1) << 7) - 1u)) == 0u;
      auto score = [&](const Codes4<S>& c, int j) -> float {
        float sum;
        if constexpr (kRep) sum = adc_rep<S, C>(c, j, lane_base);
        else sum = adc_plain<S, C>(c, j, lut, p.a.codewords);
        if constexpr (POW2) return __fmul_rn(sum, scale);
        else return __fdiv_rn(sum, p.sqrt_r);
      };
      // software pipeline: a thread scores kPipe groups while its next kPipe groups load
      constexpr int kPipe = S == 8 ? 1 : 2;
      const int tile = kScanThreads * kPipe;
      const int nfull = ngroups - ngroups % tile;
      auto main_loop = [&](auto or_tag) {
        constexpr bool kOr = decltype(or_tag)::value;
        auto score_fast = [&](const Codes4<S>& c, int j) -> float {
          float sum;
          if constexpr (kRep) sum = adc_rep<S, C, kOr>(c, j, lane_base);
          else sum = adc_plain<S, C>(c, j, lut, p.a.codewords);
          if constexpr (POW2) return __fmul_rn(sum, scale);
          else return __fdiv_rn(sum, p.sqrt_r);
        };
        Codes4<S> cur[kPipe];
        if (tid < nfull) {
#pragma unroll
          for (int u = 0; u < kPipe; ++u) cur[u] = group_codes(tid + u * kScanThreads);
        }
        for (int gb = tid; gb < nfull; gb += tile) {
          Codes4<S> nxt[kPipe];
          const int gn = gb + tile;
#pragma unroll
          for (int u = 0; u < kPipe; ++u) nxt[u] = gn < nfull ? group_codes(gn + u * kScanThreads) : cur[u];
#pragma unroll
          for (int u = 0; u < kPipe; ++u) {
            float sc[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[j] = score_fast(cur[u], j);
            // one compare per group of four keys; candidates are rare
            if (fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3])) >= t0f) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (sc[j] >= t0f) take(ordered_key(sc[j]), i0 + 4 * (gb + u * kScanThreads) + j);
            }
          }
#pragma unroll
          for (int u = 0; u < kPipe; ++u) cur[u] = nxt[u];
        }
      };
      if (or_ok) main_loop(std::true_type{});
      else main_loop(std::false_type{});
      for (int g = nfull + tid; g < ngroups; g += kScanThreads) {
        const Codes4<S> c = group_codes(g);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float sc = score(c, j);
          if (sc >= t0f) take(ordered_key(sc), i0 + 4 * g + j);
        }
      }
    }
  }
  if (!fast) {
    // masked or ragged segments: generic per-key path over the plain LUT layout
    scan_segment<S, true>(p, codes, lut, b, t, len_t, i0, i1, [&](int64_t i, uint32_t key) {
      if (key != 0u && key >= t0) take(key, i);
    });
  }
  my_max = __reduce_max_sync(0xFFFFFFFFu, my_max);
  if (lane == 0 && my_max != 0u) atomicMax(&max_key, my_max);
  __syncthreads();
  const uint32_t nl = min(n_local, static_cast<uint32_t>(kScanLocalCands));
  if (tid == 0 && nl > 0) flush_base = atomicAdd(ctrl + CTRL_NCAND, nl);
  if (tid == 0 && max_key != 0u) atomicMax(ctrl + CTRL_MAXKEY, max_key);
  __syncthreads();
  for (uint32_t e = tid; e < nl; e += blockDim.x) {
    const uint32_t g = flush_base + e;
    if (static_cast<int64_t>(g) < p.a.key_len) cand[g] = local[e];
  }
}

// Shortlist select over candidates streamed from L2 (more than fit in shared memory).  Writes
// out_idx[pos] = candidate position; returns the count.
static __device__ __forceinline__ int shortlist_from_l2(const uint2* gc, int n_cand, int k, float lo, float hi,
                                                       SelectScratch* sc, int* scratch, int32_t* out_idx) {
  auto item = [&](int i) -> unsigned long long {
    const uint2 v = __ldcg(gc + i);
    return composite(v.x, v.y);
  };
  const SelectThreshold thr =
      cta_select_linear(item, n_cand, k, lo, hi, sc, [&]() { return cta_radix_select(item, n_cand, k, sc); });
  return cta_compact(item, n_cand, thr, [&](int pos, int i, unsigned long long) { out_idx[pos] = i; }, scratch);
}

// Shortlist select over every allowed key (the sampled threshold was above the k-th best key).
// Writes out_idx[pos] = key index and, when out_c is set, out_c[pos] = its composite.
template <bool kB>
static __device__ __forceinline__ int shortlist_from_all(const DecodeParams& p, int prob, int b, int h, int t,
                                                        int64_t len_t, int k, float* lut, SelectScratch* sc,
                                                        int* scratch, int32_t* out_idx, unsigned long long* out_c) {
  for (int e = threadIdx.x; e < p.a.subspaces * p.a.codewords; e += blockDim.x)
    lut[e] = __ldcg(p.ws_lut + (size_t)prob * kMaxLut + e);
  __syncthreads();
  const uint8_t* codes = codes_base<kB>(p, b, h);
  auto item = [&](int i) -> unsigned long long {
    const uint32_t key = adc_key<kB>(p, codes, lut, b, t, i, len_t);
    return key ? composite(key, static_cast<uint32_t>(i)) : 0ull;
  };
  const SelectThreshold thr = cta_radix_select(item, static_cast<int>(len_t), k, sc);
  return cta_compact(item, static_cast<int>(len_t), thr,
                     [&](int pos, int i, unsigned long long c) {
                       out_idx[pos] = i;
                       if (out_c) out_c[pos] = c;
                     },
                     scratch);
}

// The exact shortlist of problem `prob` from the scan's candidates (CTA-cooperative):
// k = min(shortlist, allowed keys) keys by (coarse key desc, key index asc).  The candidates are
// selected in shared memory when they fit (`cand`, kCandSmem entries), else streamed from L2; if
// fewer than k keys reached the threshold the select runs exactly over every allowed key (using
// `lut`) and a fallback is counted when count_fallback is set.  Writes the selected keys'
// indices to out_idx[0, n) (and their composites to out_c when it is set) in a deterministic
// order; returns n.  Ends with a barrier.
template <bool kB>
static __device__ __forceinline__ int select_shortlist(const DecodeParams& p, int prob, int b, int h, int t,
                                                      int64_t len_t,
                                                      uint2* cand, float* lut, SelectScratch* sc, int* scratch,
                                                      int32_t* out_idx, unsigned long long* out_c,
                                                      bool count_fallback, int cand_cap = kCandSmem) {
  const int tid = threadIdx.x;
  const int64_t L = p.a.key_len;
  const uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
  const uint32_t t0 = read_t0(ctrl);
  const int64_t n_cand64 = __ldcg(ctrl + CTRL_NCAND);
  const int n_cand = static_cast<int>(n_cand64 < L ? n_cand64 : L);
  int64_t n_allowed = n_cand;
  if (t0 > 1u && n_cand < p.sl_cap) {
    if (!p.a.allowed_mask) {
      n_allowed = len_t;
    } else {
      int c = 0;
      const int64_t mr = kB ? (int64_t)b * p.a.n_queries + t : t;
      const uint8_t* mrow = p.a.allowed_mask + mr * p.a.mask_row_stride;
      for (int64_t i = tid; i < len_t; i += blockDim.x) c += mrow[i] != 0;
      n_allowed = block_sum_int(c, scratch);
    }
  }
  const int k = static_cast<int>(imin64(p.sl_cap, n_allowed));
  const uint2* gc = p.ws_cand + (size_t)prob * L;
  // every candidate key lies in [T0, the scan's largest candidate key]
  const uint32_t kmax = __ldcg(ctrl + CTRL_MAXKEY);
  const float lo = t0 > 1u ? key_to_float(t0) : -INFINITY;
  const float hi = kmax != 0u ? key_to_float(kmax) : INFINITY;
  int n_sl = 0;
  if (n_cand >= k) {
    if (n_cand <= cand_cap) {
      unsigned long long* c64 = reinterpret_cast<unsigned long long*>(cand);
      copy_batched(c64, gc, n_cand);
      if (tid == 0) stamp(p, prob, 12);
      const SelectThreshold thr = select_u64(c64, n_cand, k, lo, hi, sc);
      if (tid == 0) stamp(p, prob, 13);
      n_sl = compact_u64(c64, n_cand, thr, out_idx, scratch);
      if (tid == 0) stamp(p, prob, 14);
      for (int pos = tid; pos < n_sl; pos += blockDim.x) {
        const unsigned long long c = c64[out_idx[pos]];
        out_idx[pos] = static_cast<int32_t>(~static_cast<uint32_t>(c));
        if (out_c) out_c[pos] = c;
      }
    } else {
      n_sl = shortlist_from_l2(gc, n_cand, k, lo, hi, sc, scratch, out_idx);
      for (int pos = tid; pos < n_sl; pos += blockDim.x) {
        const uint2 v = __ldcg(gc + out_idx[pos]);
        out_idx[pos] = static_cast<int32_t>(v.y);
        if (out_c) out_c[pos] = composite(v.x, v.y);
      }
    }
  } else {
    n_sl = shortlist_from_all<kB>(p, prob, b, h, t, len_t, k, lut, sc, scratch, out_idx, out_c);
    if (count_fallback && p.a.stats && tid == 0) atomicAdd(p.a.stats + SVA_STAT_SELECT_FALLBACKS, 1ull);
  }
  __syncthreads();
  return n_sl;
}

struct FinishSmem {
  int qf, ql, lut, sc, scratch, misc, sl, rk, fin, lg, acc, parts, wt, orow, olg, fmark, kv, cand, total;
  int kv_rows;  // rows of each of the staged K and V slices (0: no staging)
};

// Entries of the finish kernel's candidate area: the shortlist select's candidates, later the
// budget select's composites followed by the shortlist logits (12 bytes per shortlist key).
__host__ __device__ inline int finish_cand_entries(int sl_cap, int dbg_cap) {
  const int need = (3 * sl_cap + 1) / 2;
  const int e = kCandSmem > dbg_cap ? kCandSmem : dbg_cap;
  return e > need ? e : need;
}

// stage_row_bytes: bytes of one staged K (and one V) row, 0 for no staging.
__host__ __device__ inline FinishSmem finish_smem_layout(int head_dim, int sl_cap, int b_cap, int cand_entries,
                                                        int stage_row_bytes) {
  FinishSmem s;
  const int chunk = (sl_cap + kCluster - 1) / kCluster;
  int o = 0;
  s.qf = o;      o = align16(o + 4 * head_dim);
  s.ql = o;      o = align16(o + 4 * kMaxRank);
  s.lut = o;     o = align16(o + 4 * kMaxLut);
  s.sc = o;      o = align16(o + (int)sizeof(SelectScratch));
  s.scratch = o; o = align16(o + 4 * 64);
  s.misc = o;    o = align16(o + 4 * 16);
  s.sl = o;      o = align16(o + 4 * sl_cap);
  s.rk = o;      o = align16(o + 4 * sl_cap);
  s.fin = o;     o = align16(o + 4 * b_cap);
  s.lg = o;      o = align16(o + 4 * b_cap);
  s.acc = o;     o = align16(o + 8 * ((kThreads / 32) * 64 + kMaxHeadDim));
  s.parts = o;   o = align16(o + 8 * kCluster * head_dim);
  s.wt = o;      o = align16(o + 4 * chunk);
  s.orow = o;    o = align16(o + 4 * chunk);
  s.olg = o;     o = align16(o + 4 * chunk);
  s.fmark = o;   o = align16(o + chunk);
  s.kv_rows = stage_row_bytes > 0 ? chunk : 0;
  s.kv = o;      o = align16(o + 2 * s.kv_rows * stage_row_bytes);
  s.cand = o;    o = align16(o + 8 * cand_entries);
  s.total = o;
  return s;
}

// One 16-byte global -> shared copy that does not wait (completion: cp.async.wait_all).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

// Split cluster barrier: arrive (release this CTA's shared-memory writes) without waiting, and
// the matching wait.  Every thread of every CTA of the cluster executes both, in this order.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }

// finish: one cluster of kCluster CTAs per problem.
//   1. every CTA selects the exact shortlist from the scan's candidates (the same deterministic
//      select in each, so no exchange is needed) and takes the slice [j0, j1) of it;
//   2. each CTA rescores its slice against k_low, stages the slice's K and V rows in its shared
//      memory (or prefetches them into L2), computes the slice's logits, and writes the rank keys,
//      the logits and the slice's rank-key range into CTA 0;
//   3. CTA 0 selects the budget, marks each final key in its owner CTA, and computes the softmax
//      max and fp64 denominator over the final logits;
//   4. each CTA forms the rounded weights of its own final keys and their fp64 weighted V sum;
//   5. CTA 0 adds the kCluster partial sums in CTA order and writes the output.
// Runs the shared (non-inlined) select and compaction code once on a synthetic set of
// kWarmItems composites in shared memory, so that their instructions are fetched while the
// kernel still waits for its inputs; the real calls overwrite every result.  c64 holds
// kWarmItems composites and out at least kWarmItems / 8 indices.  Block-cooperative.  Used by
// the one-CTA-per-problem finish, whose CTAs become resident while the scan's last waves run
// (select 7.8 -> 3.9 us per problem in a 144-problem call); the cluster finish of a single
// query starts only when the scan's one wave has left, so there it would add to the critical
// path instead.
constexpr int kWarmItems = 512;
__device__ __forceinline__ void warm_select_code(unsigned long long* c64, SelectScratch* sc, int* scratch,
                                                 int32_t* out) {
  for (int i = threadIdx.x; i < kWarmItems; i += blockDim.x)
    c64[i] = composite(ordered_key(1.0f + static_cast<float>(i) / kWarmItems), static_cast<uint32_t>(i));
  __syncthreads();
  const SelectThreshold thr = select_u64(c64, kWarmItems, kWarmItems / 8, 1.0f, 2.0f, sc);
  (void)compact_u64(c64, kWarmItems, thr, out, scratch);
}

template <typename T, bool kB>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    decode_finish_kernel(const DecodeParams p, const FinishSmem lay) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qf = reinterpret_cast<float*>(smem + lay.qf);
  float* ql = reinterpret_cast<float*>(smem + lay.ql);
  float* lut = reinterpret_cast<float*>(smem + lay.lut);
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + lay.scratch);
  int* misc = reinterpret_cast<int*>(smem + lay.misc);
  int32_t* sl = reinterpret_cast<int32_t*>(smem + lay.sl);
  uint32_t* rk = reinterpret_cast<uint32_t*>(smem + lay.rk);
  int32_t* fin = reinterpret_cast<int32_t*>(smem + lay.fin);
  float* lg = reinterpret_cast<float*>(smem + lay.lg);
  double* acc = reinterpret_cast<double*>(smem + lay.acc);
  double* parts = reinterpret_cast<double*>(smem + lay.parts);
  float* wt = reinterpret_cast<float*>(smem + lay.wt);
  int32_t* orow = reinterpret_cast<int32_t*>(smem + lay.orow);
  float* olg = reinterpret_cast<float*>(smem + lay.olg);
  uint8_t* fmark = smem + lay.fmark;
  uint2* cand = reinterpret_cast<uint2*>(smem + lay.cand);

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int prob = blockIdx.x / kCluster;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int kvh = h / p.groups;
  const int64_t len_t = allowed_length<kB>(p, b, t);
  const int D = p.a.head_dim;
  const int tid = threadIdx.x;

  {
    const T* q = query_row<T, kB>(p, b, h, t);
    pdl_launch_dependents();  // a following decode's prep may start prefetching its inputs
    // as in prep: a host-resident query is the caller's input and may be read before the wait;
    // a device query may be the output of the decode before this one
    if (p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    pdl_wait();  // the scan's candidates (and prep's q_low)
    if (!p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    for (int r = tid; r < p.a.rank_dim; r += blockDim.x) ql[r] = __ldcg(p.ws_qlow + (size_t)prob * kMaxRank + r);
    if (tid == 0) {
      misc[3] = 0;
      misc[6] = -1;  // smallest and largest rank key of the shortlist (CTA 0; atomics from all)
      misc[7] = 0;
    }
  }
  __syncthreads();

  // ---- phase 1 (every CTA): the exact shortlist ---------------------------------------------
  if (crank == 0 && tid == 0) stamp(p, prob, 2);
  const int n_sl = select_shortlist<kB>(p, prob, b, h, t, len_t, cand, lut, sc, scratch, sl, nullptr, crank == 0);
  if (crank == 0 && tid == 0) stamp(p, prob, 3);
  // CTA 0's candidate area and rank keys are written by the other CTAs below: arrive now, wait
  // before writing
  cluster_arrive();

  // ---- phase 2: rescore, logits, K/V staging of this CTA's slice ----------------------------
  const int chunk = (n_sl + kCluster - 1) / kCluster;
  const int j0 = min(n_sl, crank * chunk);
  const int j1 = min(n_sl, j0 + chunk);
  const int nj = j1 - j0;
  const int32_t* mine = sl + j0;  // key indices of the slice
  const bool staged = p.kv_stage != 0;
  T* kst = reinterpret_cast<T*>(smem + lay.kv);  // [kv_rows][D]
  T* vst = kst + (size_t)lay.kv_rows * D;
  const T* kb = keys_base<T, kB>(p, b, kvh);
  const T* vb = values_base<T, kB>(p, b, kvh);
  // the K/V gathers of the slice, issued while the k_low rows of the rescore are in flight
  auto gather_kv = [&]() {
    if (staged) {
      constexpr int kPer = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte copy
      const int cpr = D / kPer;
      if (blockDim.x % cpr == 0) {
        const int q = tid % cpr, step = blockDim.x / cpr;
        for (int jj = tid / cpr; jj < nj; jj += step) {
          const int64_t key = mine[jj];
          cp_async16(kst + jj * D + q * kPer, key_row<T, kB>(p, kb, b, key, p.k_page_stride, p.a.k_row_stride) + q * kPer);
          cp_async16(vst + jj * D + q * kPer, key_row<T, kB>(p, vb, b, key, p.v_page_stride, p.a.v_row_stride) + q * kPer);
        }
      } else {
        for (int e = tid; e < nj * cpr; e += blockDim.x) {
          const int jj = e / cpr, q = e - jj * cpr;
          const int64_t key = mine[jj];
          cp_async16(kst + jj * D + q * kPer, key_row<T, kB>(p, kb, b, key, p.k_page_stride, p.a.k_row_stride) + q * kPer);
          cp_async16(vst + jj * D + q * kPer, key_row<T, kB>(p, vb, b, key, p.v_page_stride, p.a.v_row_stride) + q * kPer);
        }
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
    } else {
      const int row_bytes = D * static_cast<int>(sizeof(T));
      const int lines = (row_bytes + 127) / 128;
      for (int e = tid; e < nj * lines; e += blockDim.x) {
        const int j = e / lines, o = (e - j * lines) * 128;
        const int64_t key = mine[j];
        const T* kr = key_row<T, kB>(p, kb, b, key, p.k_page_stride, p.a.k_row_stride);
        const T* vr = key_row<T, kB>(p, vb, b, key, p.v_page_stride, p.a.v_row_stride);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(kr) + o));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(vr) + o));
      }
    }
  };
  for (int jj = tid; jj < nj; jj += blockDim.x) fmark[jj] = 0;  // set by CTA 0 in phase 3
  rescore_rows<8, kB>(p, b, h, ql, mine, nj, rk, gather_kv);
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int jj = tid; jj < nj; jj += blockDim.x) {
    kmin = min(kmin, rk[jj]);
    kmax = max(kmax, rk[jj]);
  }
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  if (staged) {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    verify_logits<T, true>(kst, 0, D, 0, qf, D, nullptr, nj, p.a.softmax_scale, p.a.logits_mode, olg);
  } else {
    verify_logits_fn<T>(k_rows<T, kB>(p, b, kvh, mine), qf, D, nj, p.a.softmax_scale, p.a.logits_mode, olg);
  }
  cluster_wait();
  {
    uint32_t* rk0 = cluster.map_shared_rank(rk, 0);
    float* lgs0 = reinterpret_cast<float*>(cluster.map_shared_rank(cand, 0) + n_sl);  // after the composites
    for (int jj = tid; jj < nj; jj += blockDim.x) {
      rk0[j0 + jj] = rk[jj];
      lgs0[j0 + jj] = olg[jj];
    }
    if ((tid & 31) == 0 && kmax != 0u) {
      unsigned* m0 = reinterpret_cast<unsigned*>(cluster.map_shared_rank(misc, 0));
      atomicMin(m0 + 6, kmin);
      atomicMax(m0 + 7, kmax);
    }
  }
  cluster.sync();
  if (crank == 0 && tid == 0) stamp(p, prob, 4);

  // ---- phase 3 (CTA 0): budget select, final marks, softmax statistics ----------------------
  if (crank == 0) {
    const int nb = min(p.b_cap, n_sl);
    unsigned long long* c64 = reinterpret_cast<unsigned long long*>(cand);
    const float* lgs = reinterpret_cast<const float*>(c64 + n_sl);
    for (int j = tid; j < n_sl; j += blockDim.x) c64[j] = composite(rk[j], static_cast<uint32_t>(sl[j]));
    __syncthreads();
    const SelectThreshold thr = select_u64(c64, n_sl, nb, key_to_float(static_cast<uint32_t>(misc[6])),
                                           key_to_float(static_cast<uint32_t>(misc[7])), sc);
    const int n_fin = compact_u64(c64, n_sl, thr, fin, scratch);  // fin[pos] = shortlist position
    for (int pos = tid; pos < n_fin; pos += blockDim.x) {
      const int j = fin[pos];
      fin[pos] = sl[j];
      lg[pos] = lgs[j];
      const int owner = j / chunk;
      cluster.map_shared_rank(fmark, owner)[j - owner * chunk] = 1;
    }
    __syncthreads();
    float mx, denom;
    softmax_stats(lg, n_fin, scratch, acc, &mx, &denom);
    if (tid == 0) {
      misc[1] = n_fin;
      misc[4] = __float_as_int(mx);
      misc[5] = __float_as_int(denom);
    }
  }
  cluster.sync();
  if (crank == 0 && tid == 0) stamp(p, prob, 5);

  // ---- phase 4: weights and the fp64 weighted V sum of this CTA's final keys ----------------
  {
    const int* misc0 = cluster.map_shared_rank(misc, 0);
    const int n_fin = misc0[1];
    const float mx = __int_as_float(misc0[4]);
    const float denom = __int_as_float(misc0[5]);
    for (int jj = tid; jj < nj; jj += blockDim.x) {
      if (fmark[jj]) {
        const int slot = atomicAdd(misc + 3, 1);
        orow[slot] = staged ? jj : mine[jj];
        wt[slot] = round_to<T>(expf(olg[jj] - mx) / denom);
      }
    }
    __syncthreads();
    const int n_my = misc[3];
    double* sums = acc + (kThreads / 32) * 64;
    if (staged)
      accumulate_rows<T, true>(vst, 0, D, 0, D, orow, wt, n_my, acc, sums);
    else
      accumulate_rows_fn<T>(v_rows<T, kB>(p, b, kvh, orow), D, wt, n_my, acc, sums);
    double* parts0 = cluster.map_shared_rank(parts, 0);
    for (int d = tid; d < D; d += blockDim.x) parts0[crank * D + d] = sums[d];
    if (crank == 0 && tid == 0) stamp(p, prob, 6);
    cluster.sync();
    if (crank == 0 && tid == 0) stamp(p, prob, 7);

    // ---- phase 5 (CTA 0): merge, outputs, counters ------------------------------------------
    if (crank == 0) {
      T* out = out_row<T, kB>(p, b, h, t);
      for (int d = tid; d < D; d += blockDim.x) {
        double tot = 0.0;
        for (int c = 0; c < kCluster; ++c) tot += parts[c * D + d];
        out[d] = from_f32<T>(n_fin > 0 ? static_cast<float>(tot) : 0.f);
      }
      unsigned long long* tmp = reinterpret_cast<unsigned long long*>(cand);
      if (p.a.shortlist_out) write_sorted(sl, n_sl, p.a.shortlist, p.a.shortlist_out + (size_t)prob * p.a.shortlist, tmp);
      if (p.a.final_out) write_sorted(fin, n_fin, p.a.budget, p.a.final_out + (size_t)prob * p.a.budget, tmp);
      if (p.a.stats && tid == 0) {
        atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
        atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
        atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
        atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
      }
      if (tid == 0) stamp(p, prob, 8);
    }
  }
}

// ---------------------------------------------------------------------------------------
// wide finish: one CTA per problem, for launches with many problems
// ---------------------------------------------------------------------------------------
// The cluster finish above spreads one problem over kCluster CTAs of kThreads threads, which
// minimises the latency of a single decode; with hundreds of problems per launch (batches of
// sequences, throughput mode) it keeps a few problems resident at a time.  Here one CTA of
// kWideThreads threads does the whole finish of its problem with a small shared-memory
// footprint, so several problems share each SM and the gathers of many problems overlap:
// shortlist select, rank rescore, budget select, verify -- the same steps, selections and
// arithmetic as the cluster finish (and as the fused kernel).
constexpr int kWideThreads = 256;     // threads of a wide finish CTA when many problems share each SM
constexpr int kWideMaxThreads = 512;  // ... and when there is about one problem per SM
// candidates selected in shared memory (more are streamed from L2): 8192 (64 KB) with two CTAs
// per SM; ragged batches hold short sequences whose candidates are all of their keys, and a
// shared-memory select of those beats a third CTA per SM streaming them from L2
constexpr int kWideCands = 8192;
constexpr int kWideBigCands = 12288;  // ... when there is about one problem per SM
constexpr int kWideMinProblems = 64;  // problems per launch from which the wide finish is used
constexpr int kNumSmsHint = 148;      // B200 SMs: launches with at most this many problems give each 512 threads

struct WideSmem {
  int qf, ql, sc, scratch, sl, rk, fin, lg, acc, cand, total;
  int cand_cap;  // candidates selected in shared memory
};

__host__ __device__ inline WideSmem wide_smem_layout(int head_dim, int sl_cap, int b_cap, int dbg_cap,
                                                     int cand_cap = kWideCands) {
  WideSmem s;
  int o = 0;
  // the candidate area also holds the LUT of the exact fallback (kMaxLut floats), the budget
  // select's composites (8 bytes per shortlist key) and the debug outputs' sort buffer
  int cand = cand_cap;
  s.cand_cap = cand_cap;
  if (cand * 2 < kMaxLut) cand = kMaxLut / 2;
  if (cand < sl_cap) cand = sl_cap;
  if (cand < dbg_cap) cand = dbg_cap;
  s.qf = o;      o = align16(o + 4 * head_dim);
  s.ql = o;      o = align16(o + 4 * kMaxRank);
  s.sc = o;      o = align16(o + (int)sizeof(SelectScratch));
  s.scratch = o; o = align16(o + 4 * 64);
  s.sl = o;      o = align16(o + 4 * sl_cap);
  s.rk = o;      o = align16(o + 4 * sl_cap);
  s.fin = o;     o = align16(o + 4 * b_cap);
  s.lg = o;      o = align16(o + 4 * b_cap);
  s.acc = o;     o = align16(o + 8 * ((kWideMaxThreads / 32) * 64 + kMaxHeadDim));
  s.cand = o;    o = align16(o + 8 * cand);
  s.total = o;
  return s;
}

template <typename T, bool kB, int NT = kWideThreads>
__global__ void __launch_bounds__(NT, NT >= 512 ? 1 : 2) decode_finish_wide_kernel(const DecodeParams p,
                                                                                  const WideSmem lay) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qf = reinterpret_cast<float*>(smem + lay.qf);
  float* ql = reinterpret_cast<float*>(smem + lay.ql);
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + lay.scratch);
  int32_t* sl = reinterpret_cast<int32_t*>(smem + lay.sl);
  uint32_t* rk = reinterpret_cast<uint32_t*>(smem + lay.rk);
  int32_t* fin = reinterpret_cast<int32_t*>(smem + lay.fin);
  float* lg = reinterpret_cast<float*>(smem + lay.lg);
  double* acc = reinterpret_cast<double*>(smem + lay.acc);
  uint2* cand = reinterpret_cast<uint2*>(smem + lay.cand);
  float* lut = reinterpret_cast<float*>(smem + lay.cand);  // only for the exact fallback

  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int kvh = h / p.groups;
  const int64_t len_t = allowed_length<kB>(p, b, t);
  const int D = p.a.head_dim;
  const int tid = threadIdx.x;
  {
    const T* q = query_row<T, kB>(p, b, h, t);
    pdl_launch_dependents();
    if (p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    if (p.sl_cap >= kWarmItems / 8) warm_select_code(reinterpret_cast<unsigned long long*>(cand), sc, scratch, sl);
    pdl_wait();  // the scan's candidates (and prep's q_low)
    if (!p.q_host)
      for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    for (int r = tid; r < p.a.rank_dim; r += blockDim.x) ql[r] = __ldcg(p.ws_qlow + (size_t)prob * kMaxRank + r);
  }
  __syncthreads();
  if (tid == 0) stamp(p, prob, 2);
  const int n_sl =
      select_shortlist<kB>(p, prob, b, h, t, len_t, cand, lut, sc, scratch, sl, nullptr, true, lay.cand_cap);
  if (tid == 0) stamp(p, prob, 3);
  // four rows in flight per half-warp: one CTA runs this code once per problem, so a shorter
  // unrolled body (fewer instruction fetches) beats more loads in flight
  rescore_rows<4, kB>(p, b, h, ql, sl, n_sl, rk);
  if (tid == 0) stamp(p, prob, 4);
  // budget select over (rank key, key index) composites with the known rank-key range
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  unsigned long long* c64 = reinterpret_cast<unsigned long long*>(cand);
  for (int j = tid; j < n_sl; j += blockDim.x) {
    kmin = min(kmin, rk[j]);
    kmax = max(kmax, rk[j]);
    c64[j] = composite(rk[j], static_cast<uint32_t>(sl[j]));
  }
  kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
  kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
  if ((tid & 31) == 0) {
    sc->lo_part[tid >> 5] = kmin;
    sc->hi_part[tid >> 5] = kmax;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t a = 0xFFFFFFFFu, c = 0u;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      a = min(a, static_cast<uint32_t>(sc->lo_part[w]));
      c = max(c, static_cast<uint32_t>(sc->hi_part[w]));
    }
    scratch[0] = static_cast<int>(a);
    scratch[1] = static_cast<int>(c);
  }
  __syncthreads();
  const float lo = key_to_float(static_cast<uint32_t>(scratch[0])), hi = key_to_float(static_cast<uint32_t>(scratch[1]));
  __syncthreads();
  const int nb = min(p.b_cap, n_sl);
  const SelectThreshold thr = select_u64(c64, n_sl, nb, lo, hi, sc);
  const int n_fin = compact_u64(c64, n_sl, thr, fin, scratch);  // shortlist positions
  for (int pos = tid; pos < n_fin; pos += blockDim.x) fin[pos] = sl[fin[pos]];
  __syncthreads();
  if (tid == 0) stamp(p, prob, 5);
  // the candidate area is free from here on: when the final set's V rows fit there (and the
  // rows are 16-byte aligned), copy them to shared memory while the logits and the softmax are
  // computed, so that the weighted sum reads shared memory (the same arithmetic as verify_rows_fn)
  const bool v_stage =
      p.kv_stage != 0 && static_cast<size_t>(n_fin) * D * sizeof(T) <= static_cast<size_t>(lay.total - lay.cand);
  if (v_stage) {
    T* vst = reinterpret_cast<T*>(smem + lay.cand);
    const T* vb = values_base<T, kB>(p, b, kvh);
    constexpr int kPer = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte copy
    const int cpr = D / kPer;
    for (int e = tid; e < n_fin * cpr; e += blockDim.x) {
      const int jj = e / cpr, q = e - jj * cpr;
      cp_async16(vst + jj * D + q * kPer, key_row<T, kB>(p, vb, b, fin[jj], p.v_page_stride, p.a.v_row_stride) + q * kPer);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    verify_logits_fn<T, false, 4>(k_rows<T, kB>(p, b, kvh, fin), qf, D, n_fin, p.a.softmax_scale, p.a.logits_mode,
                                  lg);
    float mx, denom;
    softmax_stats(lg, n_fin, scratch, acc, &mx, &denom);
    softmax_weights<T>(lg, n_fin, mx, denom);
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    double* sums = acc + (blockDim.x >> 5) * 64;
    accumulate_rows_fn<T, true, 4>(StridedRows<T>{vst, D, nullptr}, D, lg, n_fin, acc, sums);
    T* o = out_row<T, kB>(p, b, h, t);
    for (int d = tid; d < D; d += blockDim.x) o[d] = from_f32<T>(n_fin > 0 ? static_cast<float>(sums[d]) : 0.f);
    __syncthreads();
  } else {
    verify_rows_fn<T, 4>(k_rows<T, kB>(p, b, kvh, fin), v_rows<T, kB>(p, b, kvh, fin), qf, D, n_fin,
                         p.a.softmax_scale, p.a.logits_mode, lg, acc, scratch, out_row<T, kB>(p, b, h, t));
  }
  if (tid == 0) stamp(p, prob, 6);
  unsigned long long* tmp = reinterpret_cast<unsigned long long*>(cand);
  if (p.a.shortlist_out) write_sorted(sl, n_sl, p.a.shortlist, p.a.shortlist_out + (size_t)prob * p.a.shortlist, tmp);
  if (p.a.final_out) write_sorted(fin, n_fin, p.a.budget, p.a.final_out + (size_t)prob * p.a.budget, tmp);
  if (p.a.stats && tid == 0) {
    atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
    atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------

// Launch as a programmatic dependent of the previous kernel in the stream (see pdl_wait).
template <typename... KArgs, typename... Args>
static cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static bool pow2_float(double x) {
  int e;
  const double m = frexp(x, &e);
  return m == 0.5;
}

struct DecodePlan {
  DecodeParams p;
  FinishSmem fin_lay;
  WideSmem wide_lay;
  bool wide;  // one-CTA-per-problem finish (many problems per launch)
  size_t ws_bytes;
  size_t smem_bytes;
};

static int plan_decode(const sva_decode_args* a, DecodePlan* plan, bool force_grid = false,
                       const sva_batch_layout* layout = nullptr) {
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
  // batch layout: one unpaged sequence unless a layout is given
  p.n_seqs = 1;
  p.page_shift = 62;
  p.page_mask = (int64_t{1} << 62) - 1;
  if (layout) {
    if (layout->n_seqs <= 0) return set_error(SVA_ERR_SHAPE, "n_seqs must be positive");
    p.batched = 1;
    p.n_seqs = layout->n_seqs;
    p.seq_lens = layout->seq_lens;
    p.q_seq_stride = layout->q_seq_stride;
    p.out_seq_stride = layout->out_seq_stride;
    p.codes_page_stride = layout->codes_page_stride;
    p.k_low_page_stride = layout->k_low_page_stride;
    p.k_page_stride = layout->k_page_stride;
    p.v_page_stride = layout->v_page_stride;
    if (layout->page_table) {
      const int pk = layout->page_keys;
      if (pk < kMinPageKeys || pk > kScanKeys || (pk & (pk - 1)) != 0)
        return set_error(SVA_ERR_SHAPE, "page_keys must be a power of two in 64..32768");
      if (layout->page_table_stride < (a->key_len + pk - 1) / pk)
        return set_error(SVA_ERR_SHAPE, "page_table_stride must cover key_len / page_keys pages");
      p.page_table = layout->page_table;
      p.pt_stride = layout->page_table_stride;
      p.page_shift = 0;
      while ((1 << p.page_shift) < pk) ++p.page_shift;
      p.page_mask = pk - 1;
    }
  }
  {
    const int64_t np = static_cast<int64_t>(p.n_seqs) * a->n_heads * a->n_queries;
    if (np > 0x7FFFFFF) return set_error(SVA_ERR_SHAPE, "n_seqs * n_heads * n_queries is too large");
    p.n_probs = static_cast<int>(np);
  }
  {
    // page-locked host buffers are read / written in place only where the device address of
    // the mapping is the host address itself (sva_host_buffer_device_accessible)
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, a->query) == cudaSuccess) {
      if (attr.type == cudaMemoryTypeHost && attr.devicePointer != a->query)
        return set_error(SVA_ERR_SHAPE, "query is host memory that the device cannot address at the same pointer");
      p.q_host = attr.type == cudaMemoryTypeHost ? 1 : 0;
    } else {
      cudaGetLastError();
    }
    if (cudaPointerGetAttributes(&attr, a->out) == cudaSuccess) {
      if (attr.type == cudaMemoryTypeHost && attr.devicePointer != a->out)
        return set_error(SVA_ERR_SHAPE, "out is host memory that the device cannot address at the same pointer");
    } else {
      cudaGetLastError();
    }
  }
  p.b_cap = std::min(a->budget, p.sl_cap);
  const int S = a->subspaces;
  const bool vec_s = (S == 1 || S == 2 || S == 4 || S == 8);
  const uintptr_t align = static_cast<uintptr_t>(4 * S);
  p.vec_codes = (vec_s && (reinterpret_cast<uintptr_t>(a->codes) % align == 0) &&
                 (a->codes_head_stride % (4 * S)) == 0 && (p.codes_page_stride % (4 * S)) == 0)
                    ? 1
                    : 0;
  const int64_t P = p.n_probs;
  // a few problems over a long-ish cache decode faster spread over the whole GPU (grid) than in
  // one CTA each (fused); many problems (prefill) keep the fused schedule
  p.grid_mode = (force_grid || a->key_len > kFusedMaxKeys ||
                 (P < kFusedMinProblems && a->key_len > kFusedSmallMaxKeys))
                    ? 1
                    : 0;
  int dbg_cap = 1;
  if (a->shortlist_out || a->final_out)
    while (dbg_cap < p.sl_cap) dbg_cap <<= 1;
  if (!p.grid_mode) {
    // one CTA per problem keeps every key's ADC key in shared memory; larger shortlists and
    // caches than fit go to the grid schedule
    const int stage_bytes = 4 * a->head_dim * a->rank_dim;
    int cache_bytes = std::max<int>(static_cast<int>(4 * a->key_len), stage_bytes);
    cache_bytes = std::max(cache_bytes, 8 * dbg_cap);
    p.lay = decode_smem_layout(a->head_dim, p.sl_cap, p.b_cap, cache_bytes);
    plan->smem_bytes = static_cast<size_t>(p.lay.total);
    if (p.lay.total > kMaxDynSmem) p.grid_mode = 1;
  }
  if (p.grid_mode && P > 65535)
    return set_error(SVA_ERR_SHAPE, "in the grid schedule, n_seqs * n_heads * n_queries must be <= 65535 per call");
  p.nseg = static_cast<int>((a->key_len + kScanKeys - 1) / kScanKeys);
  size_t ws = 0;
  if (!p.grid_mode) {
  } else {
    // the candidate area later holds the budget select's composites and the shortlist logits
    const int cand_entries = finish_cand_entries(p.sl_cap, dbg_cap);
    const int esz = a->qkv_dtype == SVA_DTYPE_F32 ? 4 : 2;
    const int row_bytes = a->head_dim * esz;
    const bool aligned = (row_bytes % 16 == 0) && ((a->k_row_stride * esz) % 16 == 0) &&
                         ((a->v_row_stride * esz) % 16 == 0) && ((a->k_head_stride * esz) % 16 == 0) &&
                         ((a->v_head_stride * esz) % 16 == 0) && ((p.k_page_stride * esz) % 16 == 0) &&
                         ((p.v_page_stride * esz) % 16 == 0) && (reinterpret_cast<uintptr_t>(a->keys) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(a->values) % 16 == 0);
    plan->fin_lay = finish_smem_layout(a->head_dim, p.sl_cap, p.b_cap, cand_entries, aligned ? row_bytes : 0);
    if (plan->fin_lay.total > kMaxDynSmem - 1024)
      plan->fin_lay = finish_smem_layout(a->head_dim, p.sl_cap, p.b_cap, cand_entries, 0);
    p.kv_stage = plan->fin_lay.kv_rows > 0 ? 1 : 0;
    plan->smem_bytes = static_cast<size_t>(plan->fin_lay.total);
    // with many problems per launch, one CTA per problem keeps more problems in flight than
    // one cluster per problem
    plan->wide_lay = wide_smem_layout(a->head_dim, p.sl_cap, p.b_cap, dbg_cap,
                                      P <= kNumSmsHint ? kWideBigCands : kWideCands);
    plan->wide = P >= kWideMinProblems && plan->wide_lay.total <= kMaxDynSmem;
    auto take = [&](size_t bytes) {
      size_t o = ws;
      ws = (ws + bytes + 255) & ~static_cast<size_t>(255);
      return o;
    };
    p.ws_qlow = reinterpret_cast<float*>(take(sizeof(float) * kMaxRank * P));
    p.ws_lut = reinterpret_cast<float*>(take(sizeof(float) * kMaxLut * P));
    p.ws_ctrl = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * CTRL_WORDS * P));
    p.ws_cand = reinterpret_cast<uint2*>(take(sizeof(uint2) * static_cast<size_t>(a->key_len) * P));
  }
  if (plan->smem_bytes > static_cast<size_t>(kMaxDynSmem)) return set_error(SVA_ERR_SHAPE, "shared memory plan exceeds 227 KB");
  plan->ws_bytes = ws;
  return SVA_OK;
}

// Dynamic shared memory of the scan kernel: its LUT plus the slack that aligns it.
template <int S, int C>
constexpr int scan_lut_bytes() {
  return (S > 0 && C > 0 && S * C <= kRepEntries) ? 4 * kRepEntries * 32 + C * 128 : 4 * kMaxLut;
}

template <int S, int C>
static int launch_scan(const DecodeParams& p, int P, cudaStream_t stream) {
  constexpr int smem = scan_lut_bytes<S, C>();
  auto k = p.page_table ? (p.sqrt_r_pow2 ? decode_scan_kernel<S, C, true, true> : decode_scan_kernel<S, C, false, true>)
                        : (p.sqrt_r_pow2 ? decode_scan_kernel<S, C, true, false> : decode_scan_kernel<S, C, false, false>);
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), smem);
  if (rc != SVA_OK) return rc;
  const cudaError_t e = launch_dependent(k, dim3(p.nseg, P), dim3(kScanThreads), smem, stream, p);
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

template <typename T, int S>
static int launch_prep(const DecodeParams& p, int P, const PrepSmem& lay, cudaStream_t stream) {
  auto k = p.batched ? decode_prep_kernel<T, S, true> : decode_prep_kernel<T, S, false>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), lay.total);
  if (rc != SVA_OK) return rc;
  const cudaError_t e = launch_dependent(k, dim3(P * kPrepCtas), dim3(kThreads), lay.total, stream, p, lay);
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

// The scan launch for the codes' layout (vector loads for 1, 2, 4 or 8 subspaces).
static int launch_scan_for(const DecodeParams& p, int P, cudaStream_t stream) {
  const int C = p.a.codewords;
  int rc;
  switch (p.vec_codes ? p.a.subspaces : 0) {
    case 1: rc = C == 256 ? launch_scan<1, 256>(p, P, stream) : launch_scan<1, 0>(p, P, stream); break;
    case 2: rc = C == 128 ? launch_scan<2, 128>(p, P, stream) : launch_scan<2, 0>(p, P, stream); break;
    case 4: rc = C == 64 ? launch_scan<4, 64>(p, P, stream) : launch_scan<4, 0>(p, P, stream); break;
    case 8: rc = C == 32 ? launch_scan<8, 32>(p, P, stream) : launch_scan<8, 0>(p, P, stream); break;
    default: rc = launch_scan<0, 0>(p, P, stream); break;
  }
  if (rc != SVA_OK) return rc;
  profile_mark(1, stream);
  return SVA_OK;
}

// Points the planned workspace offsets at `ws`.
static void bind_workspace(DecodeParams& p, void* ws) {
  char* base = static_cast<char*>(ws);
  p.ws_qlow = reinterpret_cast<float*>(base + reinterpret_cast<size_t>(p.ws_qlow));
  p.ws_lut = reinterpret_cast<float*>(base + reinterpret_cast<size_t>(p.ws_lut));
  p.ws_ctrl = reinterpret_cast<uint32_t*>(base + reinterpret_cast<size_t>(p.ws_ctrl));
  p.ws_cand = reinterpret_cast<uint2*>(base + reinterpret_cast<size_t>(p.ws_cand));
}

// The grid schedule's prep and scan launches (q_low, LUT, threshold, candidates).
template <typename T>
static int launch_prep_scan(DecodeParams& p, cudaStream_t stream) {
  const int P = p.n_probs;
  int rc;
  if (P >= kWideMinProblems) {
    // up to one problem per SM: 512 threads each (the latency of one problem bounds the launch);
    // more: 256 threads, two problems per SM
    const bool big = P <= kNumSmsHint;
    auto k = big ? (p.batched ? decode_prep_wide_kernel<T, true, 512> : decode_prep_wide_kernel<T, false, 512>)
                 : (p.batched ? decode_prep_wide_kernel<T, true> : decode_prep_wide_kernel<T, false>);
    const int smem = wide_prep_smem_bytes();
    rc = ensure_smem_attr(reinterpret_cast<const void*>(k), smem);
    if (rc != SVA_OK) return rc;
    const cudaError_t e = launch_dependent(k, dim3(P), dim3(big ? 512 : kWidePrepThreads), smem, stream, p);
    if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
    profile_mark(0, stream);
    return launch_scan_for(p, P, stream);
  }
  const int D = p.a.head_dim, R = p.a.rank_dim, C = p.a.codewords, S = p.a.subspaces;
  const bool prep_vec = p.vec_codes && prep_smem_layout(D, R, C, S, false).total <= kPrepSmemLimit;
  const bool want_rep = prep_vec && S * C <= kRepEntries;
  p.prep_rep = (want_rep && prep_smem_layout(D, R, C, S, true).total <= kPrepSmemLimit) ? 1 : 0;
  const PrepSmem lay = prep_smem_layout(D, R, C, prep_vec ? S : 0, p.prep_rep != 0);
  switch (prep_vec ? S : 0) {
    case 1: rc = launch_prep<T, 1>(p, P, lay, stream); break;
    case 2: rc = launch_prep<T, 2>(p, P, lay, stream); break;
    case 4: rc = launch_prep<T, 4>(p, P, lay, stream); break;
    case 8: rc = launch_prep<T, 8>(p, P, lay, stream); break;
    default: rc = launch_prep<T, 0>(p, P, lay, stream); break;
  }
  if (rc != SVA_OK) return rc;
  profile_mark(0, stream);
  return launch_scan_for(p, P, stream);
}

template <typename T>
static int launch_decode(DecodePlan& plan, void* ws, cudaStream_t stream) {
  DecodeParams& p = plan.p;
  const int P = p.n_probs;
  int rc;
  if (!p.grid_mode) {
    auto fk = p.batched ? decode_fused_kernel<T, true> : decode_fused_kernel<T, false>;
    rc = ensure_smem_attr(reinterpret_cast<const void*>(fk), kMaxDynSmem);
    if (rc != SVA_OK) return rc;
    fk<<<P, kThreads, plan.smem_bytes, stream>>>(p);
    profile_mark(0, stream);
  } else {
    bind_workspace(p, ws);
    p.dbg_ts = static_cast<unsigned long long*>(debug_timestamps());
    rc = launch_prep_scan<T>(p, stream);
    if (rc != SVA_OK) return rc;
    cudaError_t le;
    if (plan.wide) {
      const bool big = P <= kNumSmsHint;
      auto wk = big ? (p.batched ? decode_finish_wide_kernel<T, true, kWideMaxThreads>
                                 : decode_finish_wide_kernel<T, false, kWideMaxThreads>)
                    : (p.batched ? decode_finish_wide_kernel<T, true> : decode_finish_wide_kernel<T, false>);
      rc = ensure_smem_attr(reinterpret_cast<const void*>(wk), plan.wide_lay.total);
      if (rc != SVA_OK) return rc;
      le = launch_dependent(wk, dim3(P), dim3(big ? kWideMaxThreads : kWideThreads), plan.wide_lay.total, stream, p,
                            plan.wide_lay);
    } else {
      auto nk = p.batched ? decode_finish_kernel<T, true> : decode_finish_kernel<T, false>;
      rc = ensure_smem_attr(reinterpret_cast<const void*>(nk), static_cast<int>(plan.smem_bytes));
      if (rc != SVA_OK) return rc;
      le = launch_dependent(nk, dim3(P * kCluster), dim3(kThreads), plan.smem_bytes, stream, p, plan.fin_lay);
    }
    if (le != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(le));
    profile_mark(2, stream);
  }
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

extern "C" size_t sva_decode_batched_workspace_size(const sva_decode_args* args, const sva_batch_layout* layout) {
  sva::DecodePlan plan;
  if (!layout || sva::plan_decode(args, &plan, false, layout) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_decode_batched(const sva_decode_args* args, const sva_batch_layout* layout, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!layout) return sva::set_error(SVA_ERR_SHAPE, "layout is null");
  sva::DecodePlan plan;
  int rc = sva::plan_decode(args, &plan, false, layout);
  if (rc != SVA_OK) return rc;
  if (workspace_bytes < plan.ws_bytes || (plan.ws_bytes > 0 && workspace == nullptr))
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_decode_batched_workspace_size()");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::launch_decode<float>(plan, workspace, s);
    case SVA_DTYPE_BF16: return sva::launch_decode<__nv_bfloat16>(plan, workspace, s);
    default: return sva::launch_decode<__half>(plan, workspace, s);
  }
}

#include "decode_shard.cuh"
