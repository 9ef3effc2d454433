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
//     collect : one CTA per segment re-reads its codes; keys above b* go straight to the
//               shortlist, keys in b* go to a candidate buffer;
//     problem : one CTA per problem selects the missing shortlist entries from the candidate
//               buffer (exact, canonical), then rescores / selects / verifies as in the fused
//               schedule.  If the candidate buffer overflowed (huge score ties), it falls back
//               to an exact streaming select over all keys of the problem.
//
// Selection rule everywhere: score descending, key index ascending (see cta_select.cuh).
// ADC score: ((0 + lut[0][c0]) + lut[1][c1]) + ... in subspace order, then / sqrt(R)
// (reference sva/ops.py:64-71).  Rank score: tree_dot(k_low, q_low) / sqrt(R)
// (reference sva/llama.py:286-292).
#include "cta_select.cuh"
#include "sva_internal.h"

namespace sva {

constexpr int kThreads = 512;
constexpr int kBins = 4096;
constexpr int kSegKeys = 16384;
constexpr int kFusedMaxKeys = 32768;
constexpr int kCandCap = 16384;

enum { CTRL_T_HIST = 0, CTRL_T_COLLECT, CTRL_K, CTRL_BSTAR, CTRL_NABOVE, CTRL_NOUT, CTRL_NCAND, CTRL_NVALID, CTRL_WORDS };

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
  DecodeSmem lay;
  float* ws_qlow;
  float* ws_lut;
  uint32_t* ws_hist;
  uint32_t* ws_ctrl;
  int32_t* ws_part;
  uint2* ws_cand;
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

// Ordered ADC key of key i (0 when not allowed).
__device__ __forceinline__ uint32_t adc_key(const DecodeParams& p, const uint8_t* __restrict__ codes,
                                            const float* __restrict__ lut, int t, int64_t i, int64_t len_t) {
  if (!key_allowed(p, t, i, len_t)) return 0u;
  const int S = p.a.subspaces, C = p.a.codewords;
  const uint8_t* row = codes + i * S;
  float sum = 0.f;
  if (S == 4) {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(row));
    sum = __fadd_rn(sum, lut[(w & 0xFFu)]);
    sum = __fadd_rn(sum, lut[C + ((w >> 8) & 0xFFu)]);
    sum = __fadd_rn(sum, lut[2 * C + ((w >> 16) & 0xFFu)]);
    sum = __fadd_rn(sum, lut[3 * C + (w >> 24)]);
  } else {
    for (int s = 0; s < S; ++s) sum = __fadd_rn(sum, lut[s * C + __ldg(row + s)]);
  }
  return ordered_key(finish_score(sum, p));
}

template <typename T>
__device__ void build_qlut(const DecodeParams& p, int h, int t, float* qf, float* ql, float* lut) {
  const int D = p.a.head_dim, R = p.a.rank_dim, S = p.a.subspaces, C = p.a.codewords, sub = p.sub;
  const T* q = reinterpret_cast<const T*>(p.a.query) + h * p.a.q_head_stride + t * p.a.q_row_stride;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float* P = p.a.q_proj + (size_t)h * D * R + r;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = mac(acc, qf[d], __ldg(P + (size_t)d * R));
    ql[r] = __fmul_rn(acc, __ldg(p.a.scale + h));
  }
  __syncthreads();
  const int SC = S * C;
  if (p.a.lut_override) {
    const float* lo = p.a.lut_override + ((size_t)h * p.a.n_queries + t) * SC;
    for (int e = threadIdx.x; e < SC; e += blockDim.x) lut[e] = lo[e];
  } else {
    for (int e = threadIdx.x; e < SC; e += blockDim.x) {
      const int s = e / C;
      const float* cb = p.a.codebooks + (((size_t)h * S + s) * C + (e - s * C)) * sub;
      const float* qs = ql + s * sub;
      float acc = 0.f;
      for (int j = 0; j < sub; ++j) acc = mac(acc, qs[j], __ldg(cb + j));
      lut[e] = acc;
    }
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ const T* kv_row(const void* base, int64_t head_stride, int64_t row_stride, int kvh, int64_t i) {
  return reinterpret_cast<const T*>(base) + kvh * head_stride + i * row_stride;
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

  build_qlut<T>(p, h, t, qf, ql, lut);

  // ---- shortlist -------------------------------------------------------------------------
  int n_sl = 0;
  if (!p.grid_mode) {
    uint32_t* cache = reinterpret_cast<uint32_t*>(smem + p.lay.cache);
    int nv = 0;
    for (int64_t i = tid; i < L; i += blockDim.x) {
      const uint32_t key = adc_key(p, codes, lut, t, i, len_t);
      cache[i] = key;
      nv += (key != 0u);
    }
    const int n_valid = block_sum_int(nv, scratch);
    const int k = min(p.sl_cap, n_valid);
    auto item = [&](int i, uint32_t& key, uint32_t& idx) {
      key = cache[i];
      idx = static_cast<uint32_t>(i);
    };
    const SelectThreshold thr = cta_radix_select(item, static_cast<int>(L), k, sc);
    n_sl = cta_compact(item, static_cast<int>(L), thr,
                       [&](int pos, int i, uint32_t, uint32_t) { sl[pos] = i; }, scratch);
  } else {
    const uint32_t* ctrl = p.ws_ctrl + (size_t)prob * CTRL_WORDS;
    const int k = static_cast<int>(__ldcg(ctrl + CTRL_K));
    const int n_part = static_cast<int>(__ldcg(ctrl + CTRL_NOUT));
    const int n_cand = static_cast<int>(__ldcg(ctrl + CTRL_NCAND));
    const int32_t* part = p.ws_part + (size_t)prob * p.sl_cap;
    if (n_cand <= kCandCap && n_part <= k) {
      for (int i = tid; i < n_part; i += blockDim.x) sl[i] = __ldcg(part + i);
      uint2* cand = reinterpret_cast<uint2*>(smem + p.lay.cache);
      const uint2* gc = p.ws_cand + (size_t)prob * kCandCap;
      for (int i = tid; i < n_cand; i += blockDim.x) cand[i] = __ldcg(gc + i);
      __syncthreads();
      auto item = [&](int i, uint32_t& key, uint32_t& idx) {
        key = cand[i].x;
        idx = cand[i].y;
      };
      const SelectThreshold thr = cta_radix_select(item, n_cand, k - n_part, sc);
      const int got = cta_compact(item, n_cand, thr,
                                  [&](int pos, int, uint32_t, uint32_t idx) { sl[n_part + pos] = static_cast<int32_t>(idx); },
                                  scratch);
      n_sl = n_part + got;
    } else {
      // Exact streaming select over every key of the problem (candidate buffer overflow).
      auto item = [&](int i, uint32_t& key, uint32_t& idx) {
        key = adc_key(p, codes, lut, t, i, len_t);
        idx = static_cast<uint32_t>(i);
      };
      const SelectThreshold thr = cta_radix_select(item, static_cast<int>(L), k, sc);
      n_sl = cta_compact(item, static_cast<int>(L), thr,
                         [&](int pos, int i, uint32_t, uint32_t) { sl[pos] = i; }, scratch);
    }
  }
  __syncthreads();

  // ---- rank rescore: two rows per warp step (one per half-warp), 4 steps in flight ---------
  {
    const int half = lane >> 4, l16 = lane & 15;
    const float4 q4 = (4 * l16 < R) ? make_float4(ql[4 * l16], ql[4 * l16 + 1], ql[4 * l16 + 2], ql[4 * l16 + 3])
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    const float* klb = p.a.k_low + h * p.a.k_low_head_stride;
    constexpr int U = 4;
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
    auto item = [&](int j, uint32_t& key, uint32_t& idx) {
      key = rk[j];
      idx = static_cast<uint32_t>(sl[j]);
    };
    const SelectThreshold thr = cta_radix_select(item, n_sl, b, sc);
    n_fin = cta_compact(item, n_sl, thr,
                        [&](int pos, int, uint32_t, uint32_t idx) { fin[pos] = static_cast<int32_t>(idx); }, scratch);
  }

  // ---- verify: logits -------------------------------------------------------------------
  {
    const int half = lane >> 4, l16 = lane & 15;
    constexpr int U = 4;
    for (int base = warp * 2 * U; base < n_fin; base += nwarps * 2 * U) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + 2 * u + half;
        const bool ok = j < n_fin;
        const T* krow = ok ? kv_row<T>(p.a.keys, p.a.k_head_stride, p.a.k_row_stride, kvh, fin[j]) : nullptr;
        float part = 0.f;
        for (int c0 = 0; c0 < D; c0 += 64) {
          const int e = c0 + 4 * l16;
          if (!ok || e >= D) continue;
          const float4 k4 = load4<T>(krow, e, D);
          const float4 qv = make_float4(qf[e], (e + 1 < D) ? qf[e + 1] : 0.f, (e + 2 < D) ? qf[e + 2] : 0.f,
                                        (e + 3 < D) ? qf[e + 3] : 0.f);
          if (p.a.logits_mode == 1) {
            float s = round_to<T>(__fmul_rn(k4.x, qv.x));
            s = __fadd_rn(s, round_to<T>(__fmul_rn(k4.y, qv.y)));
            s = __fadd_rn(s, round_to<T>(__fmul_rn(k4.z, qv.z)));
            s = __fadd_rn(s, round_to<T>(__fmul_rn(k4.w, qv.w)));
            part = __fadd_rn(part, s);
          } else {
            part = __fadd_rn(part, lane4(k4, qv));
          }
        }
        float s = tree16(part);
        if (p.a.logits_mode == 1) {
          s = round_to<T>(s);
          s = round_to<T>(__fmul_rn(s, p.a.softmax_scale));
        } else {
          s = __fmul_rn(s, p.a.softmax_scale);
        }
        if (ok && l16 == 0) lg[j] = s;
      }
    }
  }
  __syncthreads();

  // ---- softmax (fp32 max, fp64 denominator) -------------------------------------------------
  float mx = -INFINITY;
  for (int j = tid; j < n_fin; j += blockDim.x) mx = fmaxf(mx, lg[j]);
  mx = warp_max(mx);
  float* redf = reinterpret_cast<float*>(scratch);
  if (lane == 0) redf[warp] = mx;
  __syncthreads();
  if (tid < 32) {
    float v = (tid < nwarps) ? redf[tid] : -INFINITY;
    v = warp_max(v);
    if (tid == 0) redf[32] = v;
  }
  __syncthreads();
  mx = redf[32];
  double se = 0.0;
  for (int j = tid; j < n_fin; j += blockDim.x) se += static_cast<double>(expf(lg[j] - mx));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xFFFFFFFFu, se, o);
  if (lane == 0) acc[warp] = se;
  __syncthreads();
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < nwarps; ++w) tot += acc[w];
    acc[nwarps] = tot;
  }
  __syncthreads();
  const float denom = static_cast<float>(acc[nwarps]);
  __syncthreads();
  for (int j = tid; j < n_fin; j += blockDim.x) lg[j] = round_to<T>(expf(lg[j] - mx) / denom);
  __syncthreads();

  // ---- aggregate: half-warp per row, lane owns 4 dims per 64-wide chunk; fp64 sums ----------
  {
    const int half = lane >> 4, l16 = lane & 15;
    const int nchunks = (D + 63) / 64;
    for (int c = 0; c < nchunks; ++c) {
      const int e = c * 64 + 4 * l16;
      double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
      constexpr int U = 4;
      for (int base = warp * 2 * U; base < n_fin; base += nwarps * 2 * U) {
        float4 v[U];
        float w[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int j = base + 2 * u + half;
          v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          w[u] = 0.f;
          if (j < n_fin && e < D) {
            v[u] = load4<T>(kv_row<T>(p.a.values, p.a.v_head_stride, p.a.v_row_stride, kvh, fin[j]), e, D);
            w[u] = lg[j];
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          a0 += static_cast<double>(round_to<T>(__fmul_rn(w[u], v[u].x)));
          a1 += static_cast<double>(round_to<T>(__fmul_rn(w[u], v[u].y)));
          a2 += static_cast<double>(round_to<T>(__fmul_rn(w[u], v[u].z)));
          a3 += static_cast<double>(round_to<T>(__fmul_rn(w[u], v[u].w)));
        }
      }
      // combine the two half-warps, then the warps
      a0 += __shfl_xor_sync(0xFFFFFFFFu, a0, 16);
      a1 += __shfl_xor_sync(0xFFFFFFFFu, a1, 16);
      a2 += __shfl_xor_sync(0xFFFFFFFFu, a2, 16);
      a3 += __shfl_xor_sync(0xFFFFFFFFu, a3, 16);
      double* wacc = acc;  // [nwarps][64]
      __syncthreads();
      if (half == 0) {
        wacc[warp * 64 + 4 * l16 + 0] = a0;
        wacc[warp * 64 + 4 * l16 + 1] = a1;
        wacc[warp * 64 + 4 * l16 + 2] = a2;
        wacc[warp * 64 + 4 * l16 + 3] = a3;
      }
      __syncthreads();
      if (tid < 64 && c * 64 + tid < D) {
        double tot = 0.0;
        for (int w2 = 0; w2 < nwarps; ++w2) tot += wacc[w2 * 64 + tid];
        T* out = reinterpret_cast<T*>(p.a.out) + h * p.a.out_head_stride + t * p.a.out_row_stride;
        out[c * 64 + tid] = from_f32<T>(n_fin > 0 ? static_cast<float>(tot) : 0.f);
      }
      __syncthreads();
    }
  }

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
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ float lut[kMaxLut];
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  build_qlut<T>(p, h, t, qf, ql, lut);
  const int SC = p.a.subspaces * p.a.codewords;
  float* gl = p.ws_lut + (size_t)prob * kMaxLut;
  for (int e = threadIdx.x; e < SC; e += blockDim.x) gl[e] = lut[e];
  for (int r = threadIdx.x; r < p.a.rank_dim; r += blockDim.x) p.ws_qlow[(size_t)prob * kMaxRank + r] = ql[r];
  uint32_t* hist = p.ws_hist + (size_t)prob * kBins;
  for (int b = threadIdx.x; b < kBins; b += blockDim.x) hist[b] = 0u;
  if (threadIdx.x < CTRL_WORDS) p.ws_ctrl[(size_t)prob * CTRL_WORDS + threadIdx.x] = 0u;
}

__global__ void __launch_bounds__(256) decode_hist_kernel(const DecodeParams p) {
  __shared__ float lut[kMaxLut];
  __shared__ uint32_t hist[kBins];
  __shared__ int is_last;
  __shared__ int wsum[9];
  __shared__ int boundary[3];
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
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const uint32_t key = adc_key(p, codes, lut, t, i, len_t);
    if (key) atomicAdd(&hist[key >> 20], 1u);
  }
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
  __syncthreads();
  int base = 0, total = 0;
  for (int w = 0; w < 8; ++w) {
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
  if (tid == 0 && k == 0) {
    boundary[0] = kBins;  // no key qualifies
    boundary[1] = 0;
  }
  __syncthreads();
  if (tid == 0) {
    ctrl[CTRL_K] = static_cast<uint32_t>(k);
    ctrl[CTRL_BSTAR] = static_cast<uint32_t>(boundary[0]);
    ctrl[CTRL_NABOVE] = static_cast<uint32_t>(boundary[1]);
    ctrl[CTRL_NVALID] = static_cast<uint32_t>(total);
  }
}

__global__ void __launch_bounds__(256) decode_collect_kernel(const DecodeParams p) {
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
  uint2* cand = p.ws_cand + (size_t)prob * kCandCap;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  // warp-uniform loop so the ballots below see all 32 lanes
  for (int64_t wb = i0 + (threadIdx.x & ~31); wb < i1; wb += blockDim.x) {
    const int64_t i = wb + lane;
    uint32_t key = 0u;
    if (i < i1) key = adc_key(p, codes, lut, t, i, len_t);
    const uint32_t bin = key >> 20;
    const bool above = key != 0u && bin > bstar;
    const bool edge = key != 0u && bin == bstar;
    const unsigned ba = __ballot_sync(0xFFFFFFFFu, above);
    const unsigned be = __ballot_sync(0xFFFFFFFFu, edge);
    uint32_t pa = 0, pe = 0;
    if (lane == 0) {
      if (ba) pa = atomicAdd(ctrl + CTRL_NOUT, static_cast<uint32_t>(__popc(ba)));
      if (be) pe = atomicAdd(ctrl + CTRL_NCAND, static_cast<uint32_t>(__popc(be)));
    }
    pa = __shfl_sync(0xFFFFFFFFu, pa, 0);
    pe = __shfl_sync(0xFFFFFFFFu, pe, 0);
    if (above) {
      const uint32_t pos = pa + __popc(ba & lt);
      if (pos < static_cast<uint32_t>(p.sl_cap)) part[pos] = static_cast<int32_t>(i);
    }
    if (edge) {
      const uint32_t pos = pe + __popc(be & lt);
      if (pos < static_cast<uint32_t>(kCandCap)) cand[pos] = make_uint2(key, static_cast<uint32_t>(i));
    }
  }
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
  if (a->subspaces == 4 && ((reinterpret_cast<uintptr_t>(a->codes) & 3u) || (a->codes_head_stride & 3)))
    return set_error(SVA_ERR_ALIGN, "codes must be 4-byte aligned when subspaces == 4");
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
  const int64_t P = static_cast<int64_t>(a->n_heads) * a->n_queries;
  p.grid_mode = a->key_len > kFusedMaxKeys ? 1 : 0;
  p.nseg = static_cast<int>((a->key_len + kSegKeys - 1) / kSegKeys);
  int cache_bytes;
  if (!p.grid_mode) {
    cache_bytes = static_cast<int>(4 * a->key_len);
  } else {
    cache_bytes = 8 * kCandCap;
  }
  // debug outputs reuse the cache region for a 64-bit sort of up to pow2(shortlist) entries
  if (a->shortlist_out || a->final_out) {
    int cap = 1;
    while (cap < p.sl_cap) cap <<= 1;
    cache_bytes = std::max(cache_bytes, 8 * cap);
  }
  p.lay = decode_smem_layout(a->head_dim, p.sl_cap, p.b_cap, cache_bytes);
  plan->smem_bytes = static_cast<size_t>(p.lay.total);
  if (plan->smem_bytes > 227 * 1024) return set_error(SVA_ERR_SHAPE, "shared memory plan exceeds 227 KB");
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
    const size_t o_cand = take(sizeof(uint2) * kCandCap * P);
    p.ws_qlow = reinterpret_cast<float*>(o_ql);
    p.ws_lut = reinterpret_cast<float*>(o_lut);
    p.ws_hist = reinterpret_cast<uint32_t*>(o_hist);
    p.ws_ctrl = reinterpret_cast<uint32_t*>(o_ctrl);
    p.ws_part = reinterpret_cast<int32_t*>(o_part);
    p.ws_cand = reinterpret_cast<uint2*>(o_cand);
  }
  plan->ws_bytes = ws;
  return SVA_OK;
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
    p.ws_cand = reinterpret_cast<uint2*>(base + reinterpret_cast<size_t>(p.ws_cand));
    decode_qlut_kernel<T><<<P, 256, 0, stream>>>(p);
    profile_mark(0, stream);
    dim3 grid(p.nseg, P);
    decode_hist_kernel<<<grid, 256, 0, stream>>>(p);
    profile_mark(1, stream);
    decode_collect_kernel<<<grid, 256, 0, stream>>>(p);
    profile_mark(2, stream);
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
