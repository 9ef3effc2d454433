// Key-range shards: the scan decode of one token per head when the catalog is split by key
// range across ranks (one process per GPU).  Compiled as part of decode.cu, whose prep and scan
// kernels, shortlist select, rescore and verify functions it reuses.
//
// Rank r holds keys [key_offset, key_offset + key_len) of every head in the arrays of its
// sva_decode_args.  The exact global result comes from four stages and three all-gathers that
// the host runs between them (sva_b200/sharded.py):
//
//   1 summon  : prep + scan over the local keys, then the exact local top-min(SL, key_len) by
//               (coarse key desc, global index asc) -> top [P][SL] composites (key << 32 |
//               ~global index), zero padded.                        all-gather -> [W][P][SL]
//   2 rescore : the global shortlist is the top-min(SL, candidates) of the gathered composites
//               (it is contained in the union of the local top lists); this rank rescores its own
//               members against k_low and computes their verify logits -> records [P][SL] of
//               (rank composite, logit), zero padded.               all-gather -> [W][P][SL]
//   3 verify  : the global budget set is the top-min(B, shortlist) of the gathered rank
//               composites; every rank computes the same softmax max and denominator over all
//               final logits, then the fp64 partial output of its own final keys with the
//               weights rounded to the value dtype -> partial [P][D].  all-gather -> [W][P][D]
//   4 combine : out = sum of the partials in rank order, rounded to the value dtype.
//
// Every key sees the same arithmetic as on one GPU (same LUT, ADC sum, rank score, logits,
// weights), so shortlist and final sets are identical to sva_decode over the whole key range,
// and the output differs at most by the order of exact fp64 sums.
#pragma once

namespace sva {

constexpr int kShardMaxShortlist = 8192;
constexpr int kShardMaxWorld = 64;

// Local key index <-> global key index of one rank.  Key-range shards: global = key_offset +
// local.  Page-dealt shards (page_world > 0): the pages of every sequence are dealt round-robin,
// global page g to rank g % page_world, so local page lp of this rank is global page
// lp * page_world + page_rank, and rows keep their offset inside the page.
struct ShardMap {
  int64_t key_offset;
  int page_world, page_rank, page_shift;
  __device__ __forceinline__ uint32_t to_global(int64_t l) const {
    if (page_world <= 0) return static_cast<uint32_t>(key_offset + l);
    const int64_t mask = (int64_t{1} << page_shift) - 1;
    return static_cast<uint32_t>((((l >> page_shift) * page_world + page_rank) << page_shift) | (l & mask));
  }
  __device__ __forceinline__ int64_t to_local(uint32_t g) const {
    if (page_world <= 0) return static_cast<int64_t>(g) - key_offset;
    const int64_t mask = (int64_t{1} << page_shift) - 1;
    return (((static_cast<int64_t>(g) >> page_shift) / page_world) << page_shift) | (static_cast<int64_t>(g) & mask);
  }
};

// Stage 1, after prep + scan: this rank's exact local top-k1 (k1 = p.sl_cap) of every problem as
// global composites, zero padded.
template <bool kB>
__global__ void __launch_bounds__(kThreads)
    shard_top_kernel(const DecodeParams p, const ShardMap map, int k1, unsigned long long* __restrict__ top_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint2* cand = reinterpret_cast<uint2*>(smem);  // kCandSmem entries
  __shared__ float lut[kMaxLut];
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int64_t len_t = allowed_length<kB>(p, pi.b, pi.t);
  unsigned long long* out = top_out + (size_t)prob * k1;
  int32_t* idx = reinterpret_cast<int32_t*>(smem + kCandSmem * sizeof(uint2));  // k1 entries
  pdl_wait();
  const int n = select_shortlist<kB>(p, prob, pi.b, pi.h, pi.t, len_t, cand, lut, &sc, scratch, idx, out, true);
  for (int j = threadIdx.x; j < k1; j += blockDim.x)
    out[j] = j < n ? composite(static_cast<uint32_t>(out[j] >> 32), map.to_global(idx[j])) : 0ull;
}

// Item functors of the shard kernels (plain structs: lambdas here trip the compiler's front end).
struct GatheredTop {
  const unsigned long long* g;
  int P, K, prob, base;
  __device__ unsigned long long operator()(int i) const {
    const int ii = base + i;
    const int r = ii / K, j = ii - r * K;
    return __ldcg(g + ((size_t)r * P + prob) * K + j);
  }
};

struct OwnShortlistEmit {
  int32_t* rows;
  uint32_t* gidx;
  ShardMap map;
  __device__ void operator()(int pos, int, unsigned long long c) const {
    const uint32_t g = ~static_cast<uint32_t>(c);
    gidx[pos] = g;
    rows[pos] = static_cast<int32_t>(map.to_local(g));
  }
};

// Stage 2: the global shortlist (top-min(SL, non-zero) of the W x k1 gathered composites); this
// rank rescores its own members and computes their verify logits -> records [P][k1] of (rank
// composite lo, hi, logit bits, 0).  A rank that sent k1 entries all inside the global shortlist
// may hold more members it did not send: the problem is then flagged in *saturated and the host
// repeats the exchange with k1 = SL.
// The gathered lists are staged in shared memory when they fit (`staged`, kShardStageItems): the
// select then runs the linear-bin select over the known key range (the same non-inlined code as
// the finish kernels) on shared memory instead of a radix select whose every level re-reads L2.
constexpr int kShardStageItems = 8192;

template <typename T, bool kB>
__global__ void __launch_bounds__(kThreads)
    shard_rescore_kernel(const DecodeParams p, const ShardMap map, int world, int rank, int k1,
                         const unsigned long long* __restrict__ gathered, uint4* __restrict__ records,
                         int* __restrict__ saturated, int staged) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* g64 = reinterpret_cast<unsigned long long*>(smem);  // world * k1 when staged
  int32_t* rows = reinterpret_cast<int32_t*>(smem + (staged ? 8 * (size_t)world * k1 : 0));
  uint32_t* gidx = reinterpret_cast<uint32_t*>(rows + k1);
  uint32_t* rk = gidx + k1;
  float* lg = reinterpret_cast<float*>(rk + k1);
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  __shared__ int per_rank[kShardMaxWorld];
  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h, t = pi.t;
  const int kvh = h / p.groups;
  const int P = p.n_probs;
  const int tid = threadIdx.x;
  {
    const T* q = query_row<T, kB>(p, b, h, t);
    for (int d = tid; d < p.a.head_dim; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    for (int r = tid; r < p.a.rank_dim; r += blockDim.x) ql[r] = __ldcg(p.ws_qlow + (size_t)prob * kMaxRank + r);
    for (int r = tid; r < world; r += blockDim.x) per_rank[r] = 0;
  }
  const GatheredTop item{gathered, P, k1, prob, 0};
  const int N = world * k1;
  int m;
  if (staged) {
    constexpr int kBatch = 8;
    for (int i0 = tid; i0 < N; i0 += kBatch * blockDim.x) {
      unsigned long long c[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) c[u] = i0 + u * blockDim.x < N ? item(i0 + u * blockDim.x) : 0ull;
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (i0 + u * blockDim.x < N) g64[i0 + u * blockDim.x] = c[u];
    }
    __syncthreads();
    // count and key range of the non-zero composites
    int nz = 0;
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int i = tid; i < N; i += blockDim.x) {
      const unsigned long long c = g64[i];
      if (c != 0ull) {
        ++nz;
        kmin = min(kmin, static_cast<uint32_t>(c >> 32));
        kmax = max(kmax, static_cast<uint32_t>(c >> 32));
      }
    }
    kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
    kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
    if ((tid & 31) == 0) {
      sc.lo_part[tid >> 5] = kmin;
      sc.hi_part[tid >> 5] = kmax;
    }
    nz = block_sum_int(nz, scratch);  // ends with a barrier: lo_part / hi_part are visible
    uint32_t lo = 0xFFFFFFFFu, hi = 0u;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      lo = min(lo, static_cast<uint32_t>(sc.lo_part[w]));
      hi = max(hi, static_cast<uint32_t>(sc.hi_part[w]));
    }
    __syncthreads();
    const int k = min(p.a.shortlist, nz);
    const SelectThreshold thr =
        nz > 0 ? select_u64(g64, N, k, key_to_float(lo), key_to_float(hi), &sc) : SelectThreshold{~0ull, 0ull};
    // members per rank; a rank whose k1 sent entries are all members may hold unsent members
    for (int i = tid; i < N; i += blockDim.x)
      if (is_selected(thr, g64[i])) atomicAdd(&per_rank[i / k1], 1);
    __syncthreads();
    if (tid < world && per_rank[tid] == k1 && k1 < p.a.shortlist && saturated) atomicOr(saturated, 1);
    m = cta_compact(U64Items{g64 + (size_t)rank * k1}, k1, thr, OwnShortlistEmit{rows, gidx, map}, scratch);
  } else {
    int nz = 0;
    for (int i = tid; i < N; i += blockDim.x) nz += item(i) != 0ull;
    nz = block_sum_int(nz, scratch);
    const int k = min(p.a.shortlist, nz);
    const SelectThreshold thr = cta_radix_select(item, N, k, &sc);
    // members per rank; a rank whose k1 sent entries are all members may hold unsent members
    for (int i = tid; i < N; i += blockDim.x)
      if (is_selected(thr, item(i))) atomicAdd(&per_rank[i / k1], 1);
    __syncthreads();
    if (tid < world && per_rank[tid] == k1 && k1 < p.a.shortlist && saturated) atomicOr(saturated, 1);
    const GatheredTop own{gathered, P, k1, prob, rank * k1};
    m = cta_compact(own, k1, thr, OwnShortlistEmit{rows, gidx, map}, scratch);
  }
  // four rows in flight per half-warp (a shorter body: this code runs once per problem)
  rescore_rows<4, kB>(p, b, h, ql, rows, m, rk);
  verify_logits_fn<T, false, 4>(k_rows<T, kB>(p, b, kvh, rows), qf, p.a.head_dim, m, p.a.softmax_scale,
                                p.a.logits_mode, lg);
  uint4* out = records + (size_t)prob * k1;
  for (int j = tid; j < k1; j += blockDim.x) {
    if (j < m) {
      const unsigned long long c = composite(rk[j], gidx[j]);
      out[j] = make_uint4(static_cast<uint32_t>(c), static_cast<uint32_t>(c >> 32), __float_as_uint(lg[j]), 0u);
    } else {
      out[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Stage 3: global budget set and softmax from the gathered records [W][P][k1]; fp64 partial
// output of this rank's final keys.
template <typename T, bool kB>
__global__ void __launch_bounds__(kThreads)
    shard_verify_kernel(const DecodeParams p, const ShardMap map, int world, int rank, int k1,
                        const uint4* __restrict__ gathered, double* __restrict__ partial_out, int staged) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int B = p.a.budget;
  double* acc = reinterpret_cast<double*>(smem);  // (kThreads / 32) * 64 + kMaxHeadDim doubles
  float* lgs = reinterpret_cast<float*>(acc + (kThreads / 32) * 64 + kMaxHeadDim);
  int32_t* rows = reinterpret_cast<int32_t*>(lgs + B);
  float* w = reinterpret_cast<float*>(rows + B);
  // staged: the gathered records' composites and logits (world * k1 of each) after w, 8-aligned
  unsigned long long* g64 = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(w + B) + 7u) & ~static_cast<uintptr_t>(7u));
  float* glg = reinterpret_cast<float*>(g64 + (staged ? (size_t)world * k1 : 0));
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int b = pi.b, h = pi.h;
  const int kvh = h / p.groups;
  const int P = p.n_probs;
  const int D = p.a.head_dim;
  const int tid = threadIdx.x;
  auto rec = [&](int i) -> uint4 {
    const int r = i / k1, j = i - r * k1;
    return __ldcg(gathered + ((size_t)r * P + prob) * k1 + j);
  };
  auto item = [&](int i) -> unsigned long long {
    const uint4 v = rec(i);
    return (static_cast<unsigned long long>(v.y) << 32) | v.x;
  };
  const int N = world * k1;
  int n_sl, n_fin, n_own;
  float mx, denom;
  if (staged) {
    constexpr int kBatch = 8;
    for (int i0 = tid; i0 < N; i0 += kBatch * blockDim.x) {
      uint4 v[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        v[u] = i0 + u * blockDim.x < N ? rec(i0 + u * blockDim.x) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < N) {
          g64[i] = (static_cast<unsigned long long>(v[u].y) << 32) | v[u].x;
          glg[i] = __uint_as_float(v[u].z);
        }
      }
    }
    __syncthreads();
    int nz = 0;
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int i = tid; i < N; i += blockDim.x) {
      const unsigned long long c = g64[i];
      if (c != 0ull) {
        ++nz;
        kmin = min(kmin, static_cast<uint32_t>(c >> 32));
        kmax = max(kmax, static_cast<uint32_t>(c >> 32));
      }
    }
    kmin = __reduce_min_sync(0xFFFFFFFFu, kmin);
    kmax = __reduce_max_sync(0xFFFFFFFFu, kmax);
    if ((tid & 31) == 0) {
      sc.lo_part[tid >> 5] = kmin;
      sc.hi_part[tid >> 5] = kmax;
    }
    n_sl = block_sum_int(nz, scratch);
    uint32_t lo = 0xFFFFFFFFu, hi = 0u;
    for (int wi = 0; wi < static_cast<int>(blockDim.x >> 5); ++wi) {
      lo = min(lo, static_cast<uint32_t>(sc.lo_part[wi]));
      hi = max(hi, static_cast<uint32_t>(sc.hi_part[wi]));
    }
    __syncthreads();
    const int nb = min(B, n_sl);
    const SelectThreshold thr =
        n_sl > 0 ? select_u64(g64, N, nb, key_to_float(lo), key_to_float(hi), &sc) : SelectThreshold{~0ull, 0ull};
    n_fin = cta_compact(U64Items{g64}, N, thr, [&](int pos, int i, unsigned long long) { lgs[pos] = glg[i]; },
                        scratch);
    softmax_stats(lgs, n_fin, scratch, acc, &mx, &denom);
    const float* own_lg = glg + (size_t)rank * k1;
    n_own = cta_compact(U64Items{g64 + (size_t)rank * k1}, k1, thr,
                        [&](int pos, int j, unsigned long long c) {
                          rows[pos] = static_cast<int32_t>(map.to_local(~static_cast<uint32_t>(c)));
                          w[pos] = round_to<T>(expf(own_lg[j] - mx) / denom);
                        },
                        scratch);
  } else {
    int nz = 0;
    for (int i = tid; i < N; i += blockDim.x) nz += item(i) != 0ull;
    n_sl = block_sum_int(nz, scratch);
    const int nb = min(B, n_sl);
    const SelectThreshold thr = cta_radix_select(item, N, nb, &sc);
    n_fin = cta_compact(item, N, thr,
                        [&](int pos, int i, unsigned long long) { lgs[pos] = __uint_as_float(rec(i).z); },
                        scratch);
    softmax_stats(lgs, n_fin, scratch, acc, &mx, &denom);
    auto own = [&](int j) -> unsigned long long { return item(rank * k1 + j); };
    n_own = cta_compact(own, k1, thr,
                        [&](int pos, int j, unsigned long long c) {
                          rows[pos] = static_cast<int32_t>(map.to_local(~static_cast<uint32_t>(c)));
                          const float lj = __uint_as_float(rec(rank * k1 + j).z);
                          w[pos] = round_to<T>(expf(lj - mx) / denom);
                        },
                        scratch);
  }
  double* sums = acc + (kThreads / 32) * 64;
  accumulate_rows_fn<T, false, 4>(v_rows<T, kB>(p, b, kvh, rows), D, w, n_own, acc, sums);
  for (int d = tid; d < D; d += blockDim.x) partial_out[(size_t)prob * D + d] = sums[d];
  if (p.a.stats && rank == 0 && tid == 0) {
    atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
    atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
  }
}

// Stage 4: the output, summing the ranks' partials in rank order.
template <typename T, bool kB>
__global__ void shard_combine_kernel(const DecodeParams p, int world, const double* __restrict__ gathered) {
  const int prob = blockIdx.x;
  const ProbIdx pi = prob_index<kB>(p, prob);
  const int P = p.n_probs;
  const int D = p.a.head_dim;
  T* out = out_row<T, kB>(p, pi.b, pi.h, pi.t);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double tot = 0.0;
    for (int r = 0; r < world; ++r) tot += __ldcg(gathered + ((size_t)r * P + prob) * D + d);
    out[d] = from_f32<T>(static_cast<float>(tot));
  }
}

// Plans one rank's stages.  k1 = entries each rank exchanges per problem (0: the shortlist).
static int plan_shard(const sva_decode_args* a, const sva_batch_layout* layout, const sva_shard_map* m, int k1,
                      DecodePlan* plan, ShardMap* map) {
  if (a && (a->shortlist > kShardMaxShortlist))
    return set_error(SVA_ERR_SHAPE, "shards take shortlist <= 8192");
  if (a && (k1 < 0 || k1 > a->shortlist)) return set_error(SVA_ERR_SHAPE, "exchange width must be in 0..shortlist");
  // the local decode keeps the local top-k1, not the global shortlist
  sva_decode_args local = a ? *a : sva_decode_args{};
  if (a && k1 > 0) local.shortlist = k1;
  int rc = plan_decode(a ? &local : nullptr, plan, /*force_grid=*/true, layout);
  if (rc != SVA_OK) return rc;
  plan->p.a.shortlist = a->shortlist;  // the global shortlist, for the rescore stage
  if (a->n_queries != 1) return set_error(SVA_ERR_SHAPE, "shards decode one query token per head (n_queries == 1)");
  if (a->allowed_len || a->allowed_mask) return set_error(SVA_ERR_SHAPE, "shards take no allowed_len / allowed_mask");
  if (a->shortlist_out || a->final_out) return set_error(SVA_ERR_SHAPE, "shards write no shortlist_out / final_out");
  map->key_offset = m ? m->key_offset : 0;
  map->page_world = m ? m->page_world : 0;
  map->page_rank = m ? m->page_rank : 0;
  map->page_shift = plan->p.page_table ? plan->p.page_shift : 0;
  if (map->page_world > 0) {
    if (!plan->p.page_table) return set_error(SVA_ERR_SHAPE, "page-dealt shards need a paged layout");
    if (map->page_rank < 0 || map->page_rank >= map->page_world)
      return set_error(SVA_ERR_SHAPE, "need 0 <= page_rank < page_world");
    if (((a->key_len + (int64_t{1} << map->page_shift) - 1) >> map->page_shift) * map->page_world
            << map->page_shift > 0x7FFFFFFFll)
      return set_error(SVA_ERR_SHAPE, "global key indices must stay below 2^31");
  } else if (map->key_offset < 0 || map->key_offset + a->key_len > 0x7FFFFFFFll) {
    return set_error(SVA_ERR_SHAPE, "key_offset + key_len must be in 0..2^31-1");
  }
  return SVA_OK;
}

static int shard_world_ok(int32_t world, int32_t rank) {
  if (world < 1 || world > kShardMaxWorld || rank < 0 || rank >= world)
    return set_error(SVA_ERR_SHAPE, "need 0 <= rank < world <= 64");
  return SVA_OK;
}

static int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

static int k1_of(const DecodePlan& plan, int k1) { return k1 > 0 ? k1 : plan.p.a.shortlist; }

template <typename T>
static int shard_summon(DecodePlan& plan, const ShardMap& map, int k1, unsigned long long* top_out, void* ws,
                        cudaStream_t st) {
  DecodeParams& p = plan.p;
  bind_workspace(p, ws);
  p.dbg_ts = nullptr;
  int rc = launch_prep_scan<T>(p, st);
  if (rc != SVA_OK) return rc;
  k1 = k1_of(plan, k1);
  const int smem = kCandSmem * static_cast<int>(sizeof(uint2)) + 4 * k1;
  auto k = p.batched ? shard_top_kernel<true> : shard_top_kernel<false>;
  rc = ensure_smem_attr(reinterpret_cast<const void*>(k), smem);
  if (rc != SVA_OK) return rc;
  const cudaError_t e = launch_dependent(k, dim3(p.n_probs), dim3(kThreads), smem, st, p, map, k1, top_out);
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  profile_mark(2, st);
  return launch_status();
}

template <typename T>
static int shard_rescore(DecodePlan& plan, const ShardMap& map, int world, int rank, int k1,
                         const unsigned long long* gathered, uint4* records, int* saturated, void* ws,
                         cudaStream_t st) {
  DecodeParams& p = plan.p;
  bind_workspace(p, ws);
  k1 = k1_of(plan, k1);
  const int staged = world * k1 <= kShardStageItems ? 1 : 0;
  const int smem = 16 * k1 + (staged ? 8 * world * k1 : 0);
  auto k = p.batched ? shard_rescore_kernel<T, true> : shard_rescore_kernel<T, false>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), smem);
  if (rc != SVA_OK) return rc;
  k<<<p.n_probs, kThreads, smem, st>>>(p, map, world, rank, k1, gathered, records, saturated, staged);
  return launch_status();
}

template <typename T>
static int shard_verify(DecodePlan& plan, const ShardMap& map, int world, int rank, int k1, const uint4* gathered,
                        double* partial, cudaStream_t st) {
  DecodeParams& p = plan.p;
  k1 = k1_of(plan, k1);
  const int staged = world * k1 <= kShardStageItems ? 1 : 0;
  const int smem = 8 * ((kThreads / 32) * 64 + kMaxHeadDim) + 12 * p.a.budget + 8 + (staged ? 12 * world * k1 : 0);
  auto k = p.batched ? shard_verify_kernel<T, true> : shard_verify_kernel<T, false>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(k), smem);
  if (rc != SVA_OK) return rc;
  k<<<p.n_probs, kThreads, smem, st>>>(p, map, world, rank, k1, gathered, partial, staged);
  return launch_status();
}

template <typename T>
static int shard_combine(DecodePlan& plan, int world, const double* gathered, cudaStream_t st) {
  auto k = plan.p.batched ? shard_combine_kernel<T, true> : shard_combine_kernel<T, false>;
  k<<<plan.p.n_probs, 128, 0, st>>>(plan.p, world, gathered);
  return launch_status();
}

}  // namespace sva

#define SVA_SHARD_DISPATCH(call) \
  switch (args->qkv_dtype) {     \
    case SVA_DTYPE_F32: return call(float);           \
    case SVA_DTYPE_BF16: return call(__nv_bfloat16);   \
    default: return call(__half);                      \
  }

extern "C" size_t sva_shard_batched_workspace_size(const sva_decode_args* args, const sva_batch_layout* layout,
                                                   const sva_shard_map* map, int32_t exchange_width) {
  sva::DecodePlan plan;
  sva::ShardMap m;
  if (!args || sva::plan_shard(args, layout, map, exchange_width, &plan, &m) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_shard_batched_summon(const sva_decode_args* args, const sva_batch_layout* layout,
                                        const sva_shard_map* map, int32_t exchange_width, uint64_t* top_out,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!args) return sva::set_error(SVA_ERR_SHAPE, "null args");
  sva::DecodePlan plan;
  sva::ShardMap m;
  int rc = sva::plan_shard(args, layout, map, exchange_width, &plan, &m);
  if (rc != SVA_OK) return rc;
  if (!top_out) return sva::set_error(SVA_ERR_SHAPE, "top_out is null");
  if (workspace_bytes < plan.ws_bytes || !workspace)
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_shard_batched_workspace_size()");
  auto* top = reinterpret_cast<unsigned long long*>(top_out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define CALL(T) sva::shard_summon<T>(plan, m, exchange_width, top, workspace, s)
  SVA_SHARD_DISPATCH(CALL)
#undef CALL
}

extern "C" int sva_shard_batched_rescore(const sva_decode_args* args, const sva_batch_layout* layout,
                                         const sva_shard_map* map, int32_t exchange_width, int32_t world,
                                         int32_t rank, const uint64_t* gathered_top, uint32_t* records_out,
                                         int32_t* saturated, void* workspace, size_t workspace_bytes, void* stream) {
  if (!args) return sva::set_error(SVA_ERR_SHAPE, "null args");
  sva::DecodePlan plan;
  sva::ShardMap m;
  int rc = sva::plan_shard(args, layout, map, exchange_width, &plan, &m);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, rank);
  if (rc != SVA_OK) return rc;
  if (!gathered_top || !records_out) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  if (workspace_bytes < plan.ws_bytes || !workspace)
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_shard_batched_workspace_size()");
  auto* g = reinterpret_cast<const unsigned long long*>(gathered_top);
  auto* r = reinterpret_cast<uint4*>(records_out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define CALL(T) sva::shard_rescore<T>(plan, m, world, rank, exchange_width, g, r, saturated, workspace, s)
  SVA_SHARD_DISPATCH(CALL)
#undef CALL
}

extern "C" int sva_shard_batched_verify(const sva_decode_args* args, const sva_batch_layout* layout,
                                        const sva_shard_map* map, int32_t exchange_width, int32_t world, int32_t rank,
                                        const uint32_t* gathered_records, double* partial_out, void* stream) {
  if (!args) return sva::set_error(SVA_ERR_SHAPE, "null args");
  sva::DecodePlan plan;
  sva::ShardMap m;
  int rc = sva::plan_shard(args, layout, map, exchange_width, &plan, &m);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, rank);
  if (rc != SVA_OK) return rc;
  if (!gathered_records || !partial_out) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  auto* g = reinterpret_cast<const uint4*>(gathered_records);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define CALL(T) sva::shard_verify<T>(plan, m, world, rank, exchange_width, g, partial_out, s)
  SVA_SHARD_DISPATCH(CALL)
#undef CALL
}

extern "C" int sva_shard_batched_combine(const sva_decode_args* args, const sva_batch_layout* layout, int32_t world,
                                         const double* gathered_partials, void* stream) {
  if (!args) return sva::set_error(SVA_ERR_SHAPE, "null args");
  sva::DecodePlan plan;
  sva::ShardMap m;
  int rc = sva::plan_shard(args, layout, nullptr, 0, &plan, &m);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, 0);
  if (rc != SVA_OK) return rc;
  if (!gathered_partials) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define CALL(T) sva::shard_combine<T>(plan, world, gathered_partials, s)
  SVA_SHARD_DISPATCH(CALL)
#undef CALL
}

// The single-sequence key-range entry points: the batched stages with one sequence, the exchange
// of the whole shortlist and the key offset as the map.
extern "C" size_t sva_shard_workspace_size(const sva_decode_args* args) {
  return sva_shard_batched_workspace_size(args, nullptr, nullptr, 0);
}

extern "C" int sva_shard_summon(const sva_decode_args* args, int64_t key_offset, uint64_t* top_out, void* workspace,
                                size_t workspace_bytes, void* stream) {
  const sva_shard_map m{key_offset, 0, 0};
  return sva_shard_batched_summon(args, nullptr, &m, 0, top_out, workspace, workspace_bytes, stream);
}

extern "C" int sva_shard_rescore(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                                 const uint64_t* gathered_top, uint32_t* records_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  const sva_shard_map m{key_offset, 0, 0};
  return sva_shard_batched_rescore(args, nullptr, &m, 0, world, rank, gathered_top, records_out, nullptr, workspace,
                                   workspace_bytes, stream);
}

extern "C" int sva_shard_verify(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                                const uint32_t* gathered_records, double* partial_out, void* stream) {
  const sva_shard_map m{key_offset, 0, 0};
  return sva_shard_batched_verify(args, nullptr, &m, 0, world, rank, gathered_records, partial_out, stream);
}

extern "C" int sva_shard_combine(const sva_decode_args* args, int32_t world, const double* gathered_partials,
                                 void* stream) {
  return sva_shard_batched_combine(args, nullptr, world, gathered_partials, stream);
}
