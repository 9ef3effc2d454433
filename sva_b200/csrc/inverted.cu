// Inverted-index summon -> rank rescore -> verify (static: sva/llama.py:427-576; dynamic:
// sva/llama.py:330-425) and the refill/dedupe select on explicit rows (sva/llama.py:83-116).
//
// The reference builds, per head, a padded candidate list (posting lists of the top cells of
// every subspace, then the tail keys or the current key), scores every entry with the exact
// rank-64 score, keeps a refill window of the best min(W, 2*budget) entries counting duplicates,
// and selects the best unique keys.  A key k of the posting lists occurs once per subspace whose
// top cells contain code(k, s), so its multiplicity is computable from its codes; the window is
// then a prefix of the unique keys in (score desc, key asc) order whose cumulative multiplicity
// before them is below the refill count.  This file computes exactly that:
//
//   prep    (1 CTA / head): q_low, LUT, top cells per subspace (code score desc, codeword asc),
//                           membership bitmaps, entry segments, tail, W and the refill count;
//   score   (grid / head) : enumerates the entries, keeps the first occurrence of each valid key
//                           with its multiplicity, rank-scores it (16-lane tree dot against
//                           k_low) into a candidate array and a 4096-bin histogram; the last CTA
//                           of a head finds the boundary bin of the top-`budget` unique keys;
//   collect (grid / head) : candidates above the boundary bin -> part list, in it -> edge list;
//   final   (1 CTA / head): exact canonical select of the edge, sort, refill window, adaptive
//                           budget, verify (fp32 logits), outputs and counters.
#include "cta_select.cuh"
#include "qlut.cuh"
#include "sva_internal.h"
#include "verify.cuh"

namespace sva {

constexpr int kInvThreads = 512;
constexpr int kInvBins = 4096;
constexpr int kInvEdgeCap = 16384;
constexpr int kInvMaxSeg = 2048;  // subspaces * cells
constexpr int kInvScoreThreads = 256;

enum {
  IC_T_SCORE = 0,
  IC_NCAND,
  IC_K,
  IC_BSTAR,
  IC_NABOVE,
  IC_NOUT,
  IC_NEDGE,
  IC_NVALID_ENTRIES,
  IC_WORDS = 16
};
enum { IM_EPOST = 0, IM_NTAIL, IM_TAIL_START, IM_CURRENT, IM_W, IM_RCNT, IM_WORDS = 8 };

struct InvParams {
  sva_inverted_args a;
  int groups;
  int sub;
  int cells;
  int nseg;  // subspaces * cells
  int sqrt_r_pow2;
  float sqrt_r;
  float inv_sqrt_r;
  int score_blocks;
  int collect_blocks;
  int64_t cand_cap;
  // key-range shards (sva_inverted_shard_*): every local key is in the posting lists, the
  // reference's single current-key entry belongs to the rank holding the global last key, and
  // the window width uses the global largest bucket (args.max_bucket)
  int shard;
  int holds_current;
  int64_t key_offset;
  float* ws_ql;         // [H][64]
  int32_t* ws_seg;      // [H][kInvMaxSeg + 1]
  int32_t* ws_topc;     // [H][kInvMaxSeg]
  uint32_t* ws_member;  // [H][8 subspaces][8 words]
  int64_t* ws_meta;     // [H][IM_WORDS]
  uint32_t* ws_hist;    // [H][kInvBins]
  uint32_t* ws_ctrl;    // [H][IC_WORDS]
  uint2* ws_cand;       // [H][cand_cap]  (key32, (idx << 4) | multiplicity)
  uint2* ws_part;       // [H][budget]
  uint2* ws_edge;       // [H][kInvEdgeCap]
};

__host__ __device__ __forceinline__ int64_t imin64(int64_t x, int64_t y) { return x < y ? x : y; }

__device__ __forceinline__ float inv_finish(float sum, const InvParams& p) {
  return p.sqrt_r_pow2 ? __fmul_rn(sum, p.inv_sqrt_r) : __fdiv_rn(sum, p.sqrt_r);
}

__device__ __forceinline__ bool member_of(const uint32_t* member, int s, int c) {
  return (member[s * 8 + (c >> 5)] >> (c & 31)) & 1u;
}

// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) inv_prep_kernel(const InvParams p) {
  extern __shared__ __align__(16) float stage[];
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ float lut[kMaxLut];
  __shared__ uint32_t ck[kMaxLut];
  __shared__ int32_t topc[kInvMaxSeg];
  __shared__ uint32_t member[kMaxSubspaces * 8];
  __shared__ int scratch[16];
  const int h = blockIdx.x;
  const sva_inverted_args& a = p.a;
  const int D = a.head_dim, R = a.rank_dim, S = a.subspaces, C = a.codewords;
  const int tid = threadIdx.x;
  const T* q = reinterpret_cast<const T*>(a.query) + h * a.q_head_stride;
  build_query_lut<T>(q, D, R, S, C, a.q_proj + (size_t)h * D * R, __ldg(a.scale + h),
                     a.codebooks + (size_t)h * S * C * p.sub, nullptr, qf, ql, lut, stage);
  for (int e = tid; e < S * C; e += blockDim.x) ck[e] = ordered_key(inv_finish(lut[e], p));
  for (int e = tid; e < S * 8; e += blockDim.x) member[e] = 0u;
  __syncthreads();
  for (int e = tid; e < S * C; e += blockDim.x) {
    const int s = e / C, c = e - s * C;
    const unsigned long long me = composite(ck[e], static_cast<uint32_t>(c));
    int rank = 0;
    for (int c2 = 0; c2 < C; ++c2) rank += composite(ck[s * C + c2], static_cast<uint32_t>(c2)) > me;
    if (rank < p.cells) {
      topc[s * p.cells + rank] = c;
      atomicOr(&member[s * 8 + (c >> 5)], 1u << (c & 31));
    }
  }
  __syncthreads();
  // entry segments: one per (subspace, rank) in the reference's candidate order
  const int per = (p.nseg + blockDim.x - 1) / blockDim.x;
  int local = 0;
  for (int k = 0; k < per; ++k) {
    const int j = tid * per + k;
    if (j < p.nseg) {
      const int s = j / p.cells;
      local += __ldg(a.post_counts + ((size_t)h * S + s) * C + topc[j]);
    }
  }
  int total;
  int run = block_excl_scan(local, scratch, &total);
  int32_t* seg = p.ws_seg + (size_t)h * (kInvMaxSeg + 1);
  for (int k = 0; k < per; ++k) {
    const int j = tid * per + k;
    if (j < p.nseg) {
      seg[j] = run;
      const int s = j / p.cells;
      run += __ldg(a.post_counts + ((size_t)h * S + s) * C + topc[j]);
    }
  }
  if (tid == 0) seg[p.nseg] = total;
  for (int j = tid; j < p.nseg; j += blockDim.x) p.ws_topc[(size_t)h * kInvMaxSeg + j] = topc[j];
  for (int e = tid; e < S * 8; e += blockDim.x) p.ws_member[(size_t)h * 64 + e] = member[e];
  for (int r = tid; r < R; r += blockDim.x) p.ws_ql[(size_t)h * kMaxRank + r] = ql[r];
  uint32_t* hist = p.ws_hist + (size_t)h * kInvBins;
  for (int b = tid; b < kInvBins; b += blockDim.x) hist[b] = 0u;
  if (tid < IC_WORDS) p.ws_ctrl[(size_t)h * IC_WORDS + tid] = 0u;
  if (tid == 0) {
    const int64_t L = a.key_len;
    int64_t tail_start = a.postings_len < 0 ? 0 : (a.postings_len > L ? L : a.postings_len);
    int64_t n_tail, current;
    if (p.shard) {
      n_tail = p.holds_current ? 1 : 0;
      current = p.holds_current;
    } else if (!a.dynamic && tail_start < L) {
      n_tail = L - tail_start;
      current = 0;
    } else {
      n_tail = 1;
      current = 1;
    }
    const int64_t maxb = a.max_bucket ? static_cast<int64_t>(__ldg(a.max_bucket)) : 0;
    // shards: the global candidate list has one current-key entry
    const int64_t W = static_cast<int64_t>(p.nseg) * (maxb > 1 ? maxb : 1) + (p.shard ? 1 : n_tail);
    const int64_t want = (int64_t)a.budget * (a.refill_factor > 1 ? a.refill_factor : 1);
    const int64_t rcnt = W < want ? W : want;
    int64_t* meta = p.ws_meta + (size_t)h * IM_WORDS;
    meta[IM_EPOST] = total;
    meta[IM_NTAIL] = n_tail;
    meta[IM_TAIL_START] = tail_start;
    meta[IM_CURRENT] = current;
    meta[IM_W] = W;
    meta[IM_RCNT] = rcnt;
  }
}

// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kInvScoreThreads) inv_score_kernel(const InvParams p) {
  __shared__ float ql[kMaxRank];
  __shared__ int32_t seg[kInvMaxSeg + 1];
  __shared__ int32_t topc[kInvMaxSeg];
  __shared__ uint32_t member[kMaxSubspaces * 8];
  __shared__ uint32_t hist[kInvBins];
  __shared__ int32_t qkey[kInvScoreThreads];
  __shared__ uint8_t qm[kInvScoreThreads];
  __shared__ int scratch[16];
  __shared__ uint32_t res_base;
  __shared__ int is_last;
  __shared__ int bound[3];
  const sva_inverted_args& a = p.a;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int S = a.subspaces, C = a.codewords, R = a.rank_dim;
  for (int r = tid; r < kMaxRank; r += blockDim.x) ql[r] = (r < R) ? p.ws_ql[(size_t)h * kMaxRank + r] : 0.f;
  for (int j = tid; j <= p.nseg; j += blockDim.x) seg[j] = p.ws_seg[(size_t)h * (kInvMaxSeg + 1) + j];
  for (int j = tid; j < p.nseg; j += blockDim.x) topc[j] = p.ws_topc[(size_t)h * kInvMaxSeg + j];
  for (int e = tid; e < S * 8; e += blockDim.x) member[e] = p.ws_member[(size_t)h * 64 + e];
  for (int b = tid; b < kInvBins; b += blockDim.x) hist[b] = 0u;
  const int64_t* meta = p.ws_meta + (size_t)h * IM_WORDS;
  const int64_t e_post = meta[IM_EPOST], n_tail = meta[IM_NTAIL], tail_start = meta[IM_TAIL_START];
  const bool current = meta[IM_CURRENT] != 0;
  const int64_t e_total = e_post + n_tail;
  const int64_t L = a.key_len;
  const uint8_t* codes = a.codes + h * a.codes_head_stride;
  uint32_t* ctrl = p.ws_ctrl + (size_t)h * IC_WORDS;
  uint2* cand = p.ws_cand + (size_t)h * p.cand_cap;
  const float* klb = a.k_low + h * a.k_low_head_stride;
  __syncthreads();
  int n_valid_entries = 0;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < e_total; base += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = base + tid;
    int64_t key = -1;
    bool valid = false, first = false;
    int m = 0;
    if (e < e_post) {
      int lo = 0, hi = p.nseg - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (seg[mid] <= e) lo = mid; else hi = mid - 1;
      }
      const int s = lo / p.cells;
      const int c = topc[lo];
      const int64_t slot = e - seg[lo];
      const size_t hs = (size_t)h * S + s;
      key = __ldg(a.post_ids + hs * a.post_ids_sub_stride + __ldg(a.post_offsets + hs * (C + 1) + c) + slot);
      valid = key < a.allowed_len && key < L && key < a.postings_len && (!a.allowed_mask || a.allowed_mask[key]);
      if (valid) {
        first = true;
        for (int s2 = 0; s2 < S; ++s2) {
          const bool in = member_of(member, s2, __ldg(codes + key * S + s2));
          m += in;
          if (in && s2 < s) first = false;
        }
        if (current && key == L - 1) m += 1;
      }
    } else if (e < e_total) {
      if (current) {
        key = L - 1;
        valid = key >= 0 && key < a.allowed_len && (!a.allowed_mask || a.allowed_mask[key]);
        if (valid) {
          int in = 0;
          if (key < a.postings_len)
            for (int s2 = 0; s2 < S; ++s2) in += member_of(member, s2, __ldg(codes + key * S + s2));
          first = (in == 0);
          m = in + 1;
        }
      } else {
        key = tail_start + (e - e_post);
        valid = key < a.allowed_len && (!a.allowed_mask || a.allowed_mask[key]);
        first = valid;
        m = 1;
      }
    }
    n_valid_entries += valid;
    const bool take = valid && first;
    int n_round;
    const int pos = block_excl_scan(take ? 1 : 0, scratch, &n_round);
    if (take) {
      qkey[pos] = static_cast<int32_t>(key);
      qm[pos] = static_cast<uint8_t>(m > 15 ? 15 : m);
    }
    if (tid == 0 && n_round > 0) res_base = atomicAdd(ctrl + IC_NCAND, static_cast<uint32_t>(n_round));
    __syncthreads();
    // rank-score the queued keys: one half-warp per key, kRows rows in flight per half-warp
    const int half = lane >> 4, l16 = lane & 15;
    const float4 q4 = make_float4(ql[4 * l16], ql[4 * l16 + 1], ql[4 * l16 + 2], ql[4 * l16 + 3]);
    constexpr int kRows = 4;
    for (int j0 = warp * 2 * kRows; j0 < n_round; j0 += nwarps * 2 * kRows) {
      float4 r4[kRows];
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        const int j = j0 + 2 * u + half;
        r4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < n_round && 4 * l16 < R) r4[u] = load4<float>(klb + (int64_t)qkey[j] * R, 4 * l16, R);
      }
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        const int j = j0 + 2 * u + half;
        const float s = tree16(lane4(r4[u], q4));
        if (j < n_round && l16 == 0) {
          const uint32_t k32 = ordered_key(inv_finish(s, p));
          const uint32_t slot = res_base + j;
          if (slot < p.cand_cap)
            cand[slot] = make_uint2(k32, (static_cast<uint32_t>(qkey[j]) << 4) | static_cast<uint32_t>(qm[j]));
          atomicAdd(&hist[k32 >> 20], 1u);
        }
      }
    }
    __syncthreads();
  }
  // counters and histogram flush
  int tot_valid;
  (void)block_excl_scan(n_valid_entries, scratch, &tot_valid);
  if (tid == 0 && tot_valid) atomicAdd(ctrl + IC_NVALID_ENTRIES, static_cast<uint32_t>(tot_valid));
  uint32_t* gh = p.ws_hist + (size_t)h * kInvBins;
  for (int b = tid; b < kInvBins; b += blockDim.x)
    if (hist[b]) atomicAdd(gh + b, hist[b]);
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(ctrl + IC_T_SCORE, 1u) == static_cast<uint32_t>(gridDim.x - 1));
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // last CTA of this head: boundary bin of the top-`budget` unique candidates
  uint32_t mine[16];
  int s16 = 0;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    mine[q] = __ldcg(gh + (kInvBins - 1 - (16 * tid + q)));
    s16 += static_cast<int>(mine[q]);
  }
  int incl = warp_incl_scan(s16);
  __shared__ int wsum[8];
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int basew = 0, total = 0;
  for (int w = 0; w < nwarps; ++w) {
    if (w < warp) basew += wsum[w];
    total += wsum[w];
  }
  const int n_unique = total;
  const int k = min(a.budget, n_unique);
  incl += basew;
  const int excl = incl - s16;
  if (k > 0 && excl < k && incl >= k) {
    int r = excl;
    for (int q = 0; q < 16; ++q) {
      const int v = static_cast<int>(mine[q]);
      if (r + v >= k) {
        bound[0] = kInvBins - 1 - (16 * tid + q);
        bound[1] = r;
        break;
      }
      r += v;
    }
  }
  if (tid == 0 && k == 0) {
    bound[0] = kInvBins;
    bound[1] = 0;
  }
  __syncthreads();
  if (tid == 0) {
    ctrl[IC_K] = static_cast<uint32_t>(k);
    ctrl[IC_BSTAR] = static_cast<uint32_t>(bound[0]);
    ctrl[IC_NABOVE] = static_cast<uint32_t>(bound[1]);
  }
}

// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) inv_collect_kernel(const InvParams p) {
  const int h = blockIdx.y;
  uint32_t* ctrl = p.ws_ctrl + (size_t)h * IC_WORDS;
  const uint32_t bstar = __ldcg(ctrl + IC_BSTAR);
  if (bstar >= static_cast<uint32_t>(kInvBins)) return;
  const int64_t n_cand = imin64(__ldcg(ctrl + IC_NCAND), p.cand_cap);
  const uint2* cand = p.ws_cand + (size_t)h * p.cand_cap;
  uint2* part = p.ws_part + (size_t)h * p.a.budget;
  uint2* edge = p.ws_edge + (size_t)h * kInvEdgeCap;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t wb = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); wb < n_cand;
       wb += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = wb + lane;
    uint2 v = make_uint2(0u, 0u);
    if (i < n_cand) v = __ldcg(cand + i);
    const uint32_t bin = v.x >> 20;
    const bool above = i < n_cand && v.x != 0u && bin > bstar;
    const bool on = i < n_cand && v.x != 0u && bin == bstar;
    const unsigned ba = __ballot_sync(0xFFFFFFFFu, above);
    const unsigned be = __ballot_sync(0xFFFFFFFFu, on);
    uint32_t pa = 0, pe = 0;
    if (lane == 0) {
      if (ba) pa = atomicAdd(ctrl + IC_NOUT, static_cast<uint32_t>(__popc(ba)));
      if (be) pe = atomicAdd(ctrl + IC_NEDGE, static_cast<uint32_t>(__popc(be)));
    }
    pa = __shfl_sync(0xFFFFFFFFu, pa, 0);
    pe = __shfl_sync(0xFFFFFFFFu, pe, 0);
    if (above) {
      const uint32_t pos = pa + __popc(ba & lt);
      if (pos < static_cast<uint32_t>(p.a.budget)) part[pos] = v;
    }
    if (on) {
      const uint32_t pos = pe + __popc(be & lt);
      if (pos < static_cast<uint32_t>(kInvEdgeCap)) edge[pos] = v;
    }
  }
}

// ---------------------------------------------------------------------------------------------
struct InvSmem {
  int qf, sc, scratch, comp, tmp, fin, lg, acc, total;
};

__host__ __device__ inline int inv_align(int x) { return (x + 15) & ~15; }

__host__ __device__ inline InvSmem inv_final_layout(int head_dim, int budget_pow2) {
  InvSmem s;
  int o = 0;
  s.qf = o;      o = inv_align(o + 4 * head_dim);
  s.sc = o;      o = inv_align(o + (int)sizeof(SelectScratch));
  s.scratch = o; o = inv_align(o + 4 * 64);
  s.comp = o;    o = inv_align(o + 8 * budget_pow2);
  s.tmp = o;     o = inv_align(o + 8 * kInvEdgeCap);
  s.fin = o;     o = inv_align(o + 4 * budget_pow2);
  s.lg = o;      o = inv_align(o + 4 * budget_pow2);
  s.acc = o;     o = inv_align(o + 8 * ((kInvThreads / 32) * 64 + kMaxHeadDim));
  s.total = o;
  return s;
}

// The k = min(budget, unique candidates) best unique candidates of head h as composites
// (rank key << 32 | ~(key << 4 | multiplicity)), from the collect stage's part / edge lists (or
// all candidates when the edge overflowed), sorted best first into comp[0, k); returns k.
// Block-cooperative; ends with a barrier.
__device__ int inv_topk_sorted(const InvParams& p, int h, unsigned long long* comp, uint2* tmp, SelectScratch* sc,
                               int* scratch, int budget_pow2) {
  const sva_inverted_args& a = p.a;
  const int tid = threadIdx.x;
  const uint32_t* ctrl = p.ws_ctrl + (size_t)h * IC_WORDS;
  const int k = static_cast<int>(__ldcg(ctrl + IC_K));
  const int n_part = min(static_cast<int>(__ldcg(ctrl + IC_NOUT)), a.budget);
  const int n_edge = static_cast<int>(__ldcg(ctrl + IC_NEDGE));
  const int64_t n_cand = imin64(__ldcg(ctrl + IC_NCAND), p.cand_cap);
  const uint2* gpart = p.ws_part + (size_t)h * a.budget;
  for (int i = tid; i < n_part; i += blockDim.x) {
    const uint2 v = __ldcg(gpart + i);
    comp[i] = composite(v.x, v.y);
  }
  if (k > 0 && n_part < k) {
    const int need = k - n_part;
    if (n_edge <= kInvEdgeCap) {
      const uint2* gedge = p.ws_edge + (size_t)h * kInvEdgeCap;
      for (int i = tid; i < n_edge; i += blockDim.x) tmp[i] = __ldcg(gedge + i);
      __syncthreads();
      auto item = [&](int i) -> unsigned long long { return composite(tmp[i].x, tmp[i].y); };
      const SelectThreshold thr = cta_radix_select(item, n_edge, need, sc);
      cta_compact(item, n_edge, thr, [&](int pos, int, unsigned long long c) { comp[n_part + pos] = c; }, scratch);
    } else {
      const uint2* gc = p.ws_cand + (size_t)h * p.cand_cap;
      auto item = [&](int i) -> unsigned long long {
        const uint2 v = __ldcg(gc + i);
        return composite(v.x, v.y);
      };
      const SelectThreshold thr = cta_radix_select(item, static_cast<int>(n_cand), k, sc);
      cta_compact(item, static_cast<int>(n_cand), thr, [&](int pos, int, unsigned long long c) { comp[pos] = c; },
                  scratch);
    }
  }
  __syncthreads();
  // best first: sort the complemented composites ascending
  for (int i = tid; i < k; i += blockDim.x) comp[i] = ~comp[i];
  __syncthreads();
  cta_bitonic_sort_u64(comp, k, budget_pow2);
  for (int i = tid; i < k; i += blockDim.x) comp[i] = ~comp[i];
  __syncthreads();
  return k;
}

template <typename T>
__global__ void __launch_bounds__(kInvThreads) inv_final_kernel(const InvParams p, const InvSmem lay, int budget_pow2) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qf = reinterpret_cast<float*>(smem + lay.qf);
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + lay.scratch);
  unsigned long long* comp = reinterpret_cast<unsigned long long*>(smem + lay.comp);
  uint2* tmp = reinterpret_cast<uint2*>(smem + lay.tmp);
  int32_t* fin = reinterpret_cast<int32_t*>(smem + lay.fin);
  float* lg = reinterpret_cast<float*>(smem + lay.lg);
  double* acc = reinterpret_cast<double*>(smem + lay.acc);
  __shared__ int n_fin_sh;
  __shared__ int budget_sh;
  const sva_inverted_args& a = p.a;
  const int h = blockIdx.x;
  const int tid = threadIdx.x;
  const int D = a.head_dim;
  const int kvh = h / p.groups;
  const uint32_t* ctrl = p.ws_ctrl + (size_t)h * IC_WORDS;
  const int64_t* meta = p.ws_meta + (size_t)h * IM_WORDS;
  const int k = static_cast<int>(__ldcg(ctrl + IC_K));
  const int n_part = min(static_cast<int>(__ldcg(ctrl + IC_NOUT)), a.budget);
  const int n_edge = static_cast<int>(__ldcg(ctrl + IC_NEDGE));
  const int64_t n_cand = imin64(__ldcg(ctrl + IC_NCAND), p.cand_cap);
  const int64_t rcnt = meta[IM_RCNT];
  const T* q = reinterpret_cast<const T*>(a.query) + h * a.q_head_stride;
  for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);

  // ---- the k best unique candidates ---------------------------------------------------------
  const uint2* gpart = p.ws_part + (size_t)h * a.budget;
  for (int i = tid; i < n_part; i += blockDim.x) {
    const uint2 v = __ldcg(gpart + i);
    comp[i] = composite(v.x, v.y);
  }
  if (k > 0 && n_part < k) {
    const int need = k - n_part;
    if (n_edge <= kInvEdgeCap) {
      const uint2* gedge = p.ws_edge + (size_t)h * kInvEdgeCap;
      for (int i = tid; i < n_edge; i += blockDim.x) tmp[i] = __ldcg(gedge + i);
      __syncthreads();
      auto item = [&](int i) -> unsigned long long { return composite(tmp[i].x, tmp[i].y); };
      const SelectThreshold thr = cta_radix_select(item, n_edge, need, sc);
      cta_compact(item, n_edge, thr, [&](int pos, int, unsigned long long c) { comp[n_part + pos] = c; }, scratch);
    } else {
      const uint2* gc = p.ws_cand + (size_t)h * p.cand_cap;
      auto item = [&](int i) -> unsigned long long {
        const uint2 v = __ldcg(gc + i);
        return composite(v.x, v.y);
      };
      const SelectThreshold thr = cta_radix_select(item, static_cast<int>(n_cand), k, sc);
      cta_compact(item, static_cast<int>(n_cand), thr, [&](int pos, int, unsigned long long c) { comp[pos] = c; },
                  scratch);
    }
  }
  __syncthreads();
  // best first: sort the complemented composites ascending
  for (int i = tid; i < k; i += blockDim.x) comp[i] = ~comp[i];
  __syncthreads();
  cta_bitonic_sort_u64(comp, k, budget_pow2);
  // comp[j] = ~composite of the j-th best; fin[] holds the refill validity prefix for now
  {
    // multiplicity prefix (static window): inclusive scan in blocks of blockDim
    int running = 0;
    for (int base = 0; base < k; base += blockDim.x) {
      const int j = base + tid;
      int m = 0;
      if (j < k) m = static_cast<int>((~static_cast<uint32_t>(~comp[j])) & 15u);
      int tot;
      const int ex = block_excl_scan(m, scratch, &tot);
      if (j < k) fin[j] = (a.dynamic || static_cast<int64_t>(running + ex) < rcnt) ? 1 : 0;
      running += tot;
    }
  }
  __syncthreads();
  // reference width of the selection and the adaptive budget
  const int width = a.dynamic ? k : static_cast<int>(imin64(a.budget, rcnt));
  if (tid == 0) {
    const float fmin = -3.4028234663852886e+38f;
    auto score_at = [&](int j) -> float {
      if (j < k && fin[j]) return key_to_float(static_cast<uint32_t>((~comp[j]) >> 32));
      return fmin;
    };
    int b;
    if (width > 1) {
      const int ref = min(a.min_budget, width) - 1;
      const float margin = __fsub_rn(score_at(0), score_at(ref));
      if (margin >= a.high_margin) b = a.min_budget;
      else if (margin >= a.low_margin) b = a.mid_budget;
      else b = a.budget;
      b = min(b, width);
    } else {
      b = a.dynamic ? min(a.min_budget, width) : 1;
    }
    budget_sh = b;
  }
  __syncthreads();
  const int bud = budget_sh;
  if (a.sel_idx_out || a.sel_valid_out || a.sel_score_out) {
    for (int j = tid; j < a.budget; j += blockDim.x) {
      const bool ok = j < k && j < width && fin[j];
      const unsigned long long c = ok ? ~comp[j] : 0ull;
      if (a.sel_idx_out) a.sel_idx_out[(size_t)h * a.budget + j] = ok ? static_cast<int32_t>((~static_cast<uint32_t>(c)) >> 4) : 0;
      if (a.sel_valid_out) a.sel_valid_out[(size_t)h * a.budget + j] = ok ? 1 : 0;
      if (a.sel_score_out)
        a.sel_score_out[(size_t)h * a.budget + j] = ok ? key_to_float(static_cast<uint32_t>(c >> 32)) : -3.4028234663852886e+38f;
    }
  }
  if (a.budget_out && tid == 0) a.budget_out[h] = bud;
  __syncthreads();
  // final key list: valid slots below the budget, in rank order
  if (tid == 0) {
    int n = 0;
    for (int j = 0; j < min(k, width); ++j)
      if (fin[j] && j < bud) fin[n++] = static_cast<int32_t>((~static_cast<uint32_t>(~comp[j])) >> 4);
    if (n == 0 && a.dynamic && k == 0 && a.allowed_len > 0) {
      // no candidate at all: the reference falls back to the last allowed key
      fin[n++] = static_cast<int32_t>(imin64(a.allowed_len, a.key_len) - 1);
    }
    n_fin_sh = n;
  }
  __syncthreads();
  const int n_fin = n_fin_sh;
  verify_rows<T>(a.keys, a.k_head_stride, a.k_row_stride, a.values, a.v_head_stride, a.v_row_stride, kvh, qf, D, fin,
                 n_fin, a.softmax_scale, 0, lg, acc, scratch, reinterpret_cast<T*>(a.out) + h * a.out_head_stride);
  if (a.stats && tid == 0) {
    atomicAdd(a.stats + SVA_STAT_QUERIES, 1ull);
    // static: valid candidate entries, duplicates included (sva/llama.py:561);
    // dynamic: unique candidates, or the single fallback key (sva/llama.py:409)
    const unsigned long long n_unique = __ldcg(ctrl + IC_NCAND);
    const unsigned long long summoned =
        a.dynamic ? (n_unique > 0 ? n_unique : static_cast<unsigned long long>(n_fin))
                  : static_cast<unsigned long long>(__ldcg(ctrl + IC_NVALID_ENTRIES));
    atomicAdd(a.stats + SVA_STAT_SUMMONED, summoned);
    if (!a.dynamic) atomicAdd(a.stats + SVA_STAT_REFILL_POOL, static_cast<unsigned long long>(rcnt));
    atomicAdd(a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
    atomicAdd(a.stats + SVA_STAT_CELL_VISITS, static_cast<unsigned long long>(p.nseg));
  }
}

// ---------------------------------------------------------------------------------------------
// key-range shards of the static inverted summon
// ---------------------------------------------------------------------------------------------
// Rank r holds keys [key_offset, key_offset + key_len) with posting lists over them.  The top cells
// come from the LUT, so they are the same on every rank; a key's multiplicity comes from its own
// codes; so the global candidate list is the union of the ranks' lists, and the global top-budget
// unique candidates are among the union of the ranks' top-budget lists.
//   summon : prep, score, collect as on one GPU, then the local top-budget unique candidates as
//            records (composite with the global key index, fp32 verify logit) -> all-gather
//   verify : every rank selects the same global top-budget from the gathered records, applies
//            the refill window and the adaptive budget, computes the softmax over the final keys'
//            logits and the fp64 partial output of its own final keys -> all-gather
//   combine: the output, summing the partials in rank order.

template <typename T>
__global__ void __launch_bounds__(kInvThreads) inv_shard_top_kernel(const InvParams p, const InvSmem lay,
                                                                    int budget_pow2, uint4* __restrict__ records) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* qf = reinterpret_cast<float*>(smem + lay.qf);
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + lay.scratch);
  unsigned long long* comp = reinterpret_cast<unsigned long long*>(smem + lay.comp);
  uint2* tmp = reinterpret_cast<uint2*>(smem + lay.tmp);
  int32_t* rows = reinterpret_cast<int32_t*>(smem + lay.fin);
  float* lg = reinterpret_cast<float*>(smem + lay.lg);
  const sva_inverted_args& a = p.a;
  const int h = blockIdx.x, tid = threadIdx.x, D = a.head_dim;
  const int kvh = h / p.groups;
  const T* q = reinterpret_cast<const T*>(a.query) + h * a.q_head_stride;
  for (int d = tid; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  const int k = inv_topk_sorted(p, h, comp, tmp, sc, scratch, budget_pow2);
  for (int j = tid; j < k; j += blockDim.x) rows[j] = static_cast<int32_t>((~static_cast<uint32_t>(comp[j])) >> 4);
  __syncthreads();
  verify_logits<T>(a.keys, a.k_head_stride, a.k_row_stride, kvh, qf, D, rows, k, a.softmax_scale, 0, lg);
  for (int j = tid; j < a.budget; j += blockDim.x) {
    uint4 rec = make_uint4(0u, 0u, 0u, 0u);
    if (j < k) {
      const uint32_t low = ~static_cast<uint32_t>(comp[j]);  // (local << 4) | multiplicity
      const uint32_t g = ((low >> 4) + static_cast<uint32_t>(p.key_offset)) << 4 | (low & 15u);
      const unsigned long long c = (comp[j] & 0xFFFFFFFF00000000ull) | static_cast<unsigned long long>(~g);
      rec = make_uint4(static_cast<uint32_t>(c), static_cast<uint32_t>(c >> 32), __float_as_uint(lg[j]), 0u);
    }
    records[(size_t)h * a.budget + j] = rec;
  }
}

template <typename T>
__global__ void __launch_bounds__(kInvThreads) inv_shard_verify_kernel(const InvParams p, const InvSmem lay,
                                                                       int budget_pow2, int world, int rank,
                                                                       const uint4* __restrict__ gathered,
                                                                       double* __restrict__ partial_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  SelectScratch* sc = reinterpret_cast<SelectScratch*>(smem + lay.sc);
  int* scratch = reinterpret_cast<int*>(smem + lay.scratch);
  unsigned long long* comp = reinterpret_cast<unsigned long long*>(smem + lay.comp);
  int32_t* fin = reinterpret_cast<int32_t*>(smem + lay.fin);
  float* lg = reinterpret_cast<float*>(smem + lay.lg);
  double* acc = reinterpret_cast<double*>(smem + lay.acc);
  float* wt = reinterpret_cast<float*>(smem + lay.tmp);                     // [budget]
  int32_t* rows = reinterpret_cast<int32_t*>(smem + lay.tmp) + budget_pow2;  // [budget]
  __shared__ int n_fin_sh, n_own_sh, budget_sh;
  const sva_inverted_args& a = p.a;
  const int h = blockIdx.x, tid = threadIdx.x, D = a.head_dim, B = a.budget;
  const int kvh = h / p.groups;
  const int H = a.n_heads;
  auto rec = [&](int i) -> uint4 {
    const int r = i / B, j = i - r * B;
    return __ldcg(gathered + ((size_t)r * H + h) * B + j);
  };
  auto item = [&](int i) -> unsigned long long {
    const uint4 v = rec(i);
    return (static_cast<unsigned long long>(v.y) << 32) | v.x;
  };
  const int N = world * B;
  int nz = 0;
  for (int i = tid; i < N; i += blockDim.x) nz += item(i) != 0ull;
  int tot;
  (void)block_excl_scan(nz, scratch, &tot);
  const int k = min(B, tot);
  const SelectThreshold thr = cta_radix_select(item, N, k, sc);
  // composites and logits of the selected records; the logit rides in a parallel array after sort
  cta_compact(item, N, thr, [&](int pos, int i, unsigned long long c) { comp[pos] = c; }, scratch);
  for (int i = tid; i < k; i += blockDim.x) comp[i] = ~comp[i];
  __syncthreads();
  cta_bitonic_sort_u64(comp, k, budget_pow2);
  for (int i = tid; i < k; i += blockDim.x) comp[i] = ~comp[i];
  __syncthreads();
  const int64_t rcnt = p.ws_meta[(size_t)h * IM_WORDS + IM_RCNT];
  {
    int running = 0;
    for (int base = 0; base < k; base += blockDim.x) {
      const int j = base + tid;
      int m = 0;
      if (j < k) m = static_cast<int>((~static_cast<uint32_t>(comp[j])) & 15u);
      int t2;
      const int ex = block_excl_scan(m, scratch, &t2);
      if (j < k) fin[j] = (static_cast<int64_t>(running + ex) < rcnt) ? 1 : 0;
      running += t2;
    }
  }
  __syncthreads();
  const int width = static_cast<int>(imin64(B, rcnt));
  if (tid == 0) {
    const float fmin = -3.4028234663852886e+38f;
    auto score_at = [&](int j) -> float {
      if (j < k && fin[j]) return key_to_float(static_cast<uint32_t>(comp[j] >> 32));
      return fmin;
    };
    int b;
    if (width > 1) {
      const int ref = min(a.min_budget, width) - 1;
      const float margin = __fsub_rn(score_at(0), score_at(ref));
      if (margin >= a.high_margin) b = a.min_budget;
      else if (margin >= a.low_margin) b = a.mid_budget;
      else b = a.budget;
      b = min(b, width);
    } else {
      b = 1;
    }
    budget_sh = b;
    int n = 0;
    for (int j = 0; j < min(k, width); ++j)
      if (fin[j] && j < b) fin[n++] = j;  // positions in comp
    n_fin_sh = n;
  }
  __syncthreads();
  const int n_fin = n_fin_sh;
  // logits of the final keys in rank order (the one-GPU path's order), from the records
  for (int j = tid; j < n_fin; j += blockDim.x) {
    const unsigned long long c = comp[fin[j]];
    float l = 0.f;
    for (int i = 0; i < N; ++i) {
      const uint4 v = rec(i);
      if (((static_cast<unsigned long long>(v.y) << 32) | v.x) == c) {
        l = __uint_as_float(v.z);
        break;
      }
    }
    lg[j] = l;
  }
  __syncthreads();
  float mx, denom;
  softmax_stats(lg, n_fin, scratch, acc, &mx, &denom);
  if (tid == 0) {
    int n = 0;
    for (int j = 0; j < n_fin; ++j) {
      const uint32_t g = (~static_cast<uint32_t>(comp[fin[j]])) >> 4;
      const int64_t l = static_cast<int64_t>(g) - p.key_offset;
      if (l >= 0 && l < a.key_len) {
        rows[n] = static_cast<int32_t>(l);
        wt[n] = round_to<T>(expf(lg[j] - mx) / denom);
        ++n;
      }
    }
    n_own_sh = n;
  }
  __syncthreads();
  double* sums = acc + (kInvThreads / 32) * 64;
  accumulate_rows<T>(a.values, a.v_head_stride, a.v_row_stride, kvh, D, rows, wt, n_own_sh, acc, sums);
  for (int d = tid; d < D; d += blockDim.x) partial_out[(size_t)h * D + d] = sums[d];
  if (a.stats && rank == 0 && tid == 0) {
    atomicAdd(a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
    atomicAdd(a.stats + SVA_STAT_CELL_VISITS, static_cast<unsigned long long>(p.nseg));
  }
}

template <typename T>
__global__ void inv_shard_combine_kernel(const sva_inverted_args a, int world, const double* __restrict__ gathered) {
  const int h = blockIdx.x;
  T* out = reinterpret_cast<T*>(a.out) + h * a.out_head_stride;
  for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
    double tot = 0.0;
    for (int r = 0; r < world; ++r) tot += __ldcg(gathered + ((size_t)r * a.n_heads + h) * a.head_dim + d);
    out[d] = from_f32<T>(static_cast<float>(tot));
  }
}

// ---------------------------------------------------------------------------------------------
// refill / dedupe select on explicit rows (sva/llama.py:83-116)
// ---------------------------------------------------------------------------------------------

constexpr int kTopUniqueMaxWidth = 8192;

__global__ void __launch_bounds__(kInvThreads) top_unique_kernel(const int64_t* __restrict__ idx,
                                                                 const float* __restrict__ scores,
                                                                 const uint8_t* __restrict__ valid, int width,
                                                                 int budget, int refill, int sel_count, int pow2w,
                                                                 int64_t* sel_idx, float* sel_scores,
                                                                 uint8_t* sel_valid) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* srt = reinterpret_cast<unsigned long long*>(smem);  // [pow2w]
  uint32_t* key = reinterpret_cast<uint32_t*>(smem + 8 * (size_t)pow2w);  // [width]
  uint32_t* kid = key + width;                                             // [width]
  uint8_t* rep = reinterpret_cast<uint8_t*>(kid + width);                  // [width]
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const float fmin = -3.4028234663852886e+38f;
  const int64_t* ri = idx + (size_t)row * width;
  const float* rs = scores + (size_t)row * width;
  const uint8_t* rv = valid + (size_t)row * width;
  for (int i = tid; i < width; i += blockDim.x) {
    const bool v = rv[i] != 0;
    key[i] = ordered_key(v ? rs[i] : fmin);
    kid[i] = static_cast<uint32_t>(ri[i]);
  }
  __syncthreads();
  // refill window: the `refill` best entries (duplicates of one key share a composite)
  auto item = [&](int i) -> unsigned long long { return key[i] ? composite(key[i], kid[i]) : 0ull; };
  const SelectThreshold win = cta_radix_select(item, width, refill, &sc);
  // one representative per key: sort (idx asc, key desc, validity first) and keep group heads
  for (int i = tid; i < pow2w; i += blockDim.x) {
    if (i < width) {
      const unsigned long long sk = (static_cast<unsigned long long>(kid[i]) << 32) |
                                    static_cast<unsigned long long>(~key[i]);
      srt[i] = (sk & ~0ull);
    }
  }
  __syncthreads();
  // pack position into the sort so that valid entries can be looked up afterwards
  // (entries with equal idx and key are interchangeable)
  cta_bitonic_sort_u64(srt, width, pow2w);
  for (int i = tid; i < width; i += blockDim.x) {
    const uint32_t id = static_cast<uint32_t>(srt[i] >> 32);
    const uint32_t k = ~static_cast<uint32_t>(srt[i]);
    const bool head = (i == 0) || (static_cast<uint32_t>(srt[i - 1] >> 32) != id);
    const float sv = key_to_float(k);
    // a valid entry has a real score; invalid ones were mapped to float min
    const bool in_window = is_selected(win, composite(k, id));
    rep[i] = (head && in_window && sv != fmin) ? 1 : 0;
  }
  __syncthreads();
  for (int i = tid; i < width; i += blockDim.x) {
    key[i] = rep[i] ? ~static_cast<uint32_t>(srt[i]) : 0u;
    kid[i] = static_cast<uint32_t>(srt[i] >> 32);
  }
  __syncthreads();
  int nrep_local = 0;
  for (int i = tid; i < width; i += blockDim.x) nrep_local += rep[i];
  int nrep;
  (void)block_excl_scan(nrep_local, scratch, &nrep);
  const int take = min(sel_count, nrep);
  const SelectThreshold thr = cta_radix_select(item, width, take, &sc);
  // collect the selected representatives and order them best first
  unsigned long long* best = srt;  // reuse
  int got = cta_compact(item, width, thr, [&](int pos, int, unsigned long long c) { best[pos] = ~c; }, scratch);
  int p2 = 1;
  while (p2 < got) p2 <<= 1;
  cta_bitonic_sort_u64(best, got, p2);
  for (int j = tid; j < sel_count; j += blockDim.x) {
    const bool ok = j < got;
    const unsigned long long c = ok ? ~best[j] : 0ull;
    sel_idx[(size_t)row * sel_count + j] = ok ? static_cast<int64_t>(~static_cast<uint32_t>(c)) : 0;
    sel_scores[(size_t)row * sel_count + j] = ok ? key_to_float(static_cast<uint32_t>(c >> 32)) : fmin;
    sel_valid[(size_t)row * sel_count + j] = ok ? 1 : 0;
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------

static bool inv_pow2(float x) {
  int e;
  return std::frexp(static_cast<double>(x), &e) == 0.5;
}

struct InvPlan {
  InvParams p;
  size_t ws_bytes;
  InvSmem lay;
  int budget_pow2;
};

static int plan_inverted(const sva_inverted_args* a, InvPlan* plan) {
  if (!a) return set_error(SVA_ERR_SHAPE, "null args");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return set_error(SVA_ERR_SHAPE, "n_heads must be a positive multiple of n_kv_heads");
  if (a->head_dim <= 0 || a->head_dim > kMaxHeadDim) return set_error(SVA_ERR_SHAPE, "head_dim must be in 1..256");
  if (a->rank_dim <= 0 || a->rank_dim > kMaxRank || a->rank_dim % 4)
    return set_error(SVA_ERR_SHAPE, "rank_dim must be a multiple of 4 in 4..64");
  if (a->subspaces <= 0 || a->subspaces > kMaxSubspaces || a->rank_dim % a->subspaces)
    return set_error(SVA_ERR_SHAPE, "subspaces must divide rank_dim and be <= 8");
  if (a->codewords <= 0 || a->codewords > kMaxCodewords) return set_error(SVA_ERR_SHAPE, "codewords must be in 1..256");
  if (a->key_len <= 0 || a->key_len >= (1ll << 28)) return set_error(SVA_ERR_SHAPE, "key_len must be in 1..2^28-1");
  if (a->budget <= 0 || a->budget > 8192) return set_error(SVA_ERR_SHAPE, "budget must be in 1..8192");
  if (a->cells <= 0) return set_error(SVA_ERR_SHAPE, "cells must be positive");
  if (a->min_budget <= 0 || a->mid_budget <= 0) return set_error(SVA_ERR_SHAPE, "adaptive budgets must be positive");
  if (a->qkv_dtype < 0 || a->qkv_dtype > 2) return set_error(SVA_ERR_DTYPE, "bad qkv dtype");
  if (!a->query || !a->q_proj || !a->scale || !a->codebooks || !a->codes || !a->post_counts || !a->post_offsets ||
      !a->post_ids || !a->max_bucket || !a->k_low || !a->keys || !a->values || !a->out)
    return set_error(SVA_ERR_SHAPE, "a required pointer is null");
  InvParams& p = plan->p;
  memset(&p, 0, sizeof(p));
  p.a = *a;
  p.groups = a->n_heads / a->n_kv_heads;
  p.sub = a->rank_dim / a->subspaces;
  p.cells = std::min(a->cells, a->codewords);
  p.nseg = a->subspaces * p.cells;
  p.sqrt_r = static_cast<float>(std::sqrt(static_cast<double>(a->rank_dim)));
  p.sqrt_r_pow2 = inv_pow2(p.sqrt_r) ? 1 : 0;
  p.inv_sqrt_r = 1.0f / p.sqrt_r;
  p.cand_cap = a->key_len;
  const int64_t entries_hint = std::min<int64_t>(a->key_len * a->subspaces, 1ll << 26);
  p.score_blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((entries_hint + 2047) / 2048, 592)));
  p.collect_blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((a->key_len + 4095) / 4096, 592)));
  plan->budget_pow2 = 1;
  while (plan->budget_pow2 < a->budget) plan->budget_pow2 <<= 1;
  plan->lay = inv_final_layout(a->head_dim, plan->budget_pow2);
  if (plan->lay.total > kMaxDynSmem) return set_error(SVA_ERR_SHAPE, "inverted final shared memory too large");
  const size_t H = a->n_heads;
  size_t ws = 0;
  auto take = [&](size_t bytes) {
    size_t o = ws;
    ws = (ws + bytes + 255) & ~static_cast<size_t>(255);
    return o;
  };
  const size_t o_ql = take(sizeof(float) * kMaxRank * H);
  const size_t o_seg = take(sizeof(int32_t) * (kInvMaxSeg + 1) * H);
  const size_t o_topc = take(sizeof(int32_t) * kInvMaxSeg * H);
  const size_t o_mem = take(sizeof(uint32_t) * 64 * H);
  const size_t o_meta = take(sizeof(int64_t) * IM_WORDS * H);
  const size_t o_hist = take(sizeof(uint32_t) * kInvBins * H);
  const size_t o_ctrl = take(sizeof(uint32_t) * IC_WORDS * H);
  const size_t o_cand = take(sizeof(uint2) * p.cand_cap * H);
  const size_t o_part = take(sizeof(uint2) * a->budget * H);
  const size_t o_edge = take(sizeof(uint2) * kInvEdgeCap * H);
  p.ws_ql = reinterpret_cast<float*>(o_ql);
  p.ws_seg = reinterpret_cast<int32_t*>(o_seg);
  p.ws_topc = reinterpret_cast<int32_t*>(o_topc);
  p.ws_member = reinterpret_cast<uint32_t*>(o_mem);
  p.ws_meta = reinterpret_cast<int64_t*>(o_meta);
  p.ws_hist = reinterpret_cast<uint32_t*>(o_hist);
  p.ws_ctrl = reinterpret_cast<uint32_t*>(o_ctrl);
  p.ws_cand = reinterpret_cast<uint2*>(o_cand);
  p.ws_part = reinterpret_cast<uint2*>(o_part);
  p.ws_edge = reinterpret_cast<uint2*>(o_edge);
  plan->ws_bytes = ws;
  return SVA_OK;
}

template <typename T>
static int launch_inverted(InvPlan& plan, void* ws, cudaStream_t st) {
  InvParams& p = plan.p;
  char* b = static_cast<char*>(ws);
  p.ws_ql = reinterpret_cast<float*>(b + reinterpret_cast<size_t>(p.ws_ql));
  p.ws_seg = reinterpret_cast<int32_t*>(b + reinterpret_cast<size_t>(p.ws_seg));
  p.ws_topc = reinterpret_cast<int32_t*>(b + reinterpret_cast<size_t>(p.ws_topc));
  p.ws_member = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_member));
  p.ws_meta = reinterpret_cast<int64_t*>(b + reinterpret_cast<size_t>(p.ws_meta));
  p.ws_hist = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_hist));
  p.ws_ctrl = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_ctrl));
  p.ws_cand = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_cand));
  p.ws_part = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_part));
  p.ws_edge = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_edge));
  const int H = p.a.n_heads;
  int rc0 = ensure_smem_attr(reinterpret_cast<const void*>(inv_prep_kernel<T>), 160 * 1024);
  if (rc0) return rc0;
  inv_prep_kernel<T><<<H, 256, 4 * p.a.head_dim * p.a.rank_dim, st>>>(p);
  profile_mark(0, st);
  inv_score_kernel<<<dim3(p.score_blocks, H), kInvScoreThreads, 0, st>>>(p);
  profile_mark(1, st);
  inv_collect_kernel<<<dim3(p.collect_blocks, H), 256, 0, st>>>(p);
  profile_mark(2, st);
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(inv_final_kernel<T>), kMaxDynSmem);
  if (rc) return rc;
  inv_final_kernel<T><<<H, kInvThreads, plan.lay.total, st>>>(p, plan.lay, plan.budget_pow2);
  profile_mark(3, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

}  // namespace sva

using namespace sva;

extern "C" size_t sva_inverted_workspace_size(const sva_inverted_args* args) {
  InvPlan plan;
  if (plan_inverted(args, &plan) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_decode_inverted(const sva_inverted_args* args, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  InvPlan plan;
  int rc = plan_inverted(args, &plan);
  if (rc != SVA_OK) return rc;
  if (workspace_bytes < plan.ws_bytes || !workspace) return set_error(SVA_ERR_WORKSPACE, "inverted workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return launch_inverted<float>(plan, workspace, st);
    case SVA_DTYPE_BF16: return launch_inverted<__nv_bfloat16>(plan, workspace, st);
    default: return launch_inverted<__half>(plan, workspace, st);
  }
}

static int plan_inverted_shard(const sva_inverted_args* a, int64_t key_offset, int32_t holds_current, InvPlan* plan) {
  int rc = plan_inverted(a, plan);
  if (rc != SVA_OK) return rc;
  if (a->dynamic) return set_error(SVA_ERR_SHAPE, "inverted shards take the static summon (dynamic == 0)");
  if (a->postings_len != a->key_len)
    return set_error(SVA_ERR_SHAPE, "inverted shards need posting lists over every local key (postings_len == key_len)");
  if (a->allowed_len != a->key_len || a->allowed_mask)
    return set_error(SVA_ERR_SHAPE, "inverted shards take no allowed_len limit or allowed_mask");
  if (a->sel_idx_out || a->sel_valid_out || a->sel_score_out || a->budget_out)
    return set_error(SVA_ERR_SHAPE, "inverted shards write no selection outputs");
  if (key_offset < 0 || key_offset + a->key_len >= (1ll << 28))
    return set_error(SVA_ERR_SHAPE, "key_offset + key_len must be below 2^28");
  plan->p.shard = 1;
  plan->p.holds_current = holds_current ? 1 : 0;
  plan->p.key_offset = key_offset;
  return SVA_OK;
}

static void bind_inverted_workspace(InvParams& p, void* ws) {
  char* b = static_cast<char*>(ws);
  p.ws_ql = reinterpret_cast<float*>(b + reinterpret_cast<size_t>(p.ws_ql));
  p.ws_seg = reinterpret_cast<int32_t*>(b + reinterpret_cast<size_t>(p.ws_seg));
  p.ws_topc = reinterpret_cast<int32_t*>(b + reinterpret_cast<size_t>(p.ws_topc));
  p.ws_member = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_member));
  p.ws_meta = reinterpret_cast<int64_t*>(b + reinterpret_cast<size_t>(p.ws_meta));
  p.ws_hist = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_hist));
  p.ws_ctrl = reinterpret_cast<uint32_t*>(b + reinterpret_cast<size_t>(p.ws_ctrl));
  p.ws_cand = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_cand));
  p.ws_part = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_part));
  p.ws_edge = reinterpret_cast<uint2*>(b + reinterpret_cast<size_t>(p.ws_edge));
}

template <typename T>
static int inverted_shard_summon(InvPlan& plan, void* ws, uint4* records, cudaStream_t st) {
  InvParams& p = plan.p;
  bind_inverted_workspace(p, ws);
  const int H = p.a.n_heads;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(inv_prep_kernel<T>), 160 * 1024);
  if (rc) return rc;
  inv_prep_kernel<T><<<H, 256, 4 * p.a.head_dim * p.a.rank_dim, st>>>(p);
  inv_score_kernel<<<dim3(p.score_blocks, H), kInvScoreThreads, 0, st>>>(p);
  inv_collect_kernel<<<dim3(p.collect_blocks, H), 256, 0, st>>>(p);
  rc = ensure_smem_attr(reinterpret_cast<const void*>(inv_shard_top_kernel<T>), kMaxDynSmem);
  if (rc) return rc;
  inv_shard_top_kernel<T><<<H, kInvThreads, plan.lay.total, st>>>(p, plan.lay, plan.budget_pow2, records);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

template <typename T>
static int inverted_shard_verify(InvPlan& plan, void* ws, int world, int rank, const uint4* gathered, double* partial,
                                 cudaStream_t st) {
  InvParams& p = plan.p;
  bind_inverted_workspace(p, ws);
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(inv_shard_verify_kernel<T>), kMaxDynSmem);
  if (rc) return rc;
  inv_shard_verify_kernel<T><<<p.a.n_heads, kInvThreads, plan.lay.total, st>>>(p, plan.lay, plan.budget_pow2, world,
                                                                               rank, gathered, partial);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" size_t sva_inverted_shard_workspace_size(const sva_inverted_args* args) {
  InvPlan plan;
  if (plan_inverted_shard(args, 0, 0, &plan) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_inverted_shard_summon(const sva_inverted_args* args, int64_t key_offset, int32_t holds_current,
                                         uint32_t* records_out, void* workspace, size_t workspace_bytes, void* stream) {
  InvPlan plan;
  int rc = plan_inverted_shard(args, key_offset, holds_current, &plan);
  if (rc != SVA_OK) return rc;
  if (!records_out) return set_error(SVA_ERR_SHAPE, "records_out is null");
  if (workspace_bytes < plan.ws_bytes || !workspace) return set_error(SVA_ERR_WORKSPACE, "inverted workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* r = reinterpret_cast<uint4*>(records_out);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return inverted_shard_summon<float>(plan, workspace, r, st);
    case SVA_DTYPE_BF16: return inverted_shard_summon<__nv_bfloat16>(plan, workspace, r, st);
    default: return inverted_shard_summon<__half>(plan, workspace, r, st);
  }
}

extern "C" int sva_inverted_shard_verify(const sva_inverted_args* args, int64_t key_offset, int32_t holds_current,
                                         int32_t world, int32_t rank, const uint32_t* gathered_records,
                                         double* partial_out, void* workspace, size_t workspace_bytes, void* stream) {
  InvPlan plan;
  int rc = plan_inverted_shard(args, key_offset, holds_current, &plan);
  if (rc != SVA_OK) return rc;
  if (world < 1 || rank < 0 || rank >= world) return set_error(SVA_ERR_SHAPE, "need 0 <= rank < world");
  if (!gathered_records || !partial_out) return set_error(SVA_ERR_SHAPE, "null pointer");
  if (workspace_bytes < plan.ws_bytes || !workspace) return set_error(SVA_ERR_WORKSPACE, "inverted workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* g = reinterpret_cast<const uint4*>(gathered_records);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return inverted_shard_verify<float>(plan, workspace, world, rank, g, partial_out, st);
    case SVA_DTYPE_BF16: return inverted_shard_verify<__nv_bfloat16>(plan, workspace, world, rank, g, partial_out, st);
    default: return inverted_shard_verify<__half>(plan, workspace, world, rank, g, partial_out, st);
  }
}

extern "C" int sva_inverted_shard_combine(const sva_inverted_args* args, int32_t world, const double* gathered_partials,
                                          void* stream) {
  if (!args || !args->out || !gathered_partials) return set_error(SVA_ERR_SHAPE, "null pointer");
  if (world < 1 || args->n_heads <= 0 || args->head_dim <= 0) return set_error(SVA_ERR_SHAPE, "bad sizes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: inv_shard_combine_kernel<float><<<args->n_heads, 128, 0, st>>>(*args, world, gathered_partials); break;
    case SVA_DTYPE_BF16:
      inv_shard_combine_kernel<__nv_bfloat16><<<args->n_heads, 128, 0, st>>>(*args, world, gathered_partials);
      break;
    default: inv_shard_combine_kernel<__half><<<args->n_heads, 128, 0, st>>>(*args, world, gathered_partials); break;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int sva_top_unique(const int64_t* idx, const float* scores, const uint8_t* valid, int32_t rows,
                              int32_t width, int32_t budget, int32_t refill_factor, int64_t* sel_idx,
                              float* sel_scores, uint8_t* sel_valid, int32_t* refill_out, void* stream) {
  if (rows < 0 || width < 0 || width > kTopUniqueMaxWidth) return set_error(SVA_ERR_SHAPE, "width must be <= 8192");
  if (width == 0 || budget <= 0 || rows == 0) {
    if (refill_out) *refill_out = 0;
    return SVA_OK;
  }
  const int refill = std::min(width, std::max(budget, budget * refill_factor));
  const int sel_count = std::min(budget, refill);
  if (refill_out) *refill_out = refill;
  int pow2w = 1;
  while (pow2w < width) pow2w <<= 1;
  const size_t smem = 8 * (size_t)pow2w + 9 * (size_t)width + 16;
  if (smem > (size_t)kMaxDynSmem) return set_error(SVA_ERR_SHAPE, "top_unique row too wide for shared memory");
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(top_unique_kernel), kMaxDynSmem);
  if (rc) return rc;
  top_unique_kernel<<<rows, kInvThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      idx, scores, valid, width, budget, refill, sel_count, pow2w, sel_idx, sel_scores, sel_valid);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}
