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

// Stage 1, after prep + scan: the exact local shortlist as global composites.
__global__ void __launch_bounds__(kThreads)
    shard_top_kernel(const DecodeParams p, int64_t key_offset, unsigned long long* __restrict__ top_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint2* cand = reinterpret_cast<uint2*>(smem);  // kCandSmem entries
  __shared__ float lut[kMaxLut];
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  const int64_t len_t = allowed_length<false>(p, 0, t);
  const int SL = p.a.shortlist;
  unsigned long long* out = top_out + (size_t)prob * SL;
  const uint32_t off = static_cast<uint32_t>(key_offset);
  int32_t* idx = reinterpret_cast<int32_t*>(smem + kCandSmem * sizeof(uint2));  // SL entries
  const int n = select_shortlist<false>(p, prob, 0, h, t, len_t, cand, lut, &sc, scratch, idx, out, true);
  for (int j = threadIdx.x; j < SL; j += blockDim.x)
    out[j] = j < n ? composite(static_cast<uint32_t>(out[j] >> 32), static_cast<uint32_t>(idx[j]) + off) : 0ull;
}

// Item functors of the shard kernels (plain structs: lambdas here trip the compiler's front end).
struct GatheredTop {
  const unsigned long long* g;
  int P, SL, prob, base;
  __device__ unsigned long long operator()(int i) const {
    const int ii = base + i;
    const int r = ii / SL, j = ii - r * SL;
    return __ldcg(g + ((size_t)r * P + prob) * SL + j);
  }
};

struct OwnShortlistEmit {
  int32_t* rows;
  uint32_t* gidx;
  uint32_t off;
  __device__ void operator()(int pos, int, unsigned long long c) const {
    const uint32_t g = ~static_cast<uint32_t>(c);
    gidx[pos] = g;
    rows[pos] = static_cast<int32_t>(g - off);
  }
};

// Stage 2: global shortlist from the gathered top lists; rescore + logits of this rank's members.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    shard_rescore_kernel(const DecodeParams p, int64_t key_offset, int world, int rank,
                         const unsigned long long* __restrict__ gathered, uint4* __restrict__ records) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int SL = p.a.shortlist;
  int32_t* rows = reinterpret_cast<int32_t*>(smem);
  uint32_t* gidx = reinterpret_cast<uint32_t*>(rows + SL);
  uint32_t* rk = gidx + SL;
  float* lg = reinterpret_cast<float*>(rk + SL);
  __shared__ float qf[kMaxHeadDim];
  __shared__ float ql[kMaxRank];
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  const int kvh = h / p.groups;
  const int P = p.n_probs;
  const int tid = threadIdx.x;
  {
    const T* q = reinterpret_cast<const T*>(p.a.query) + h * p.a.q_head_stride + t * p.a.q_row_stride;
    for (int d = tid; d < p.a.head_dim; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
    for (int r = tid; r < p.a.rank_dim; r += blockDim.x) ql[r] = __ldcg(p.ws_qlow + (size_t)prob * kMaxRank + r);
  }
  const GatheredTop item{gathered, P, SL, prob, 0};
  const int N = world * SL;
  int nz = 0;
  for (int i = tid; i < N; i += blockDim.x) nz += item(i) != 0ull;
  nz = block_sum_int(nz, scratch);
  const int k = min(SL, nz);
  const SelectThreshold thr = cta_radix_select(item, N, k, &sc);
  const GatheredTop own{gathered, P, SL, prob, rank * SL};
  const int m = cta_compact(own, SL, thr, OwnShortlistEmit{rows, gidx, static_cast<uint32_t>(key_offset)}, scratch);
  rescore_rows<8, false>(p, 0, h, ql, rows, m, rk);
  verify_logits<T>(p.a.keys, p.a.k_head_stride, p.a.k_row_stride, kvh, qf, p.a.head_dim, rows, m, p.a.softmax_scale,
                   p.a.logits_mode, lg);
  uint4* out = records + (size_t)prob * SL;
  for (int j = tid; j < SL; j += blockDim.x) {
    if (j < m) {
      const unsigned long long c = composite(rk[j], gidx[j]);
      out[j] = make_uint4(static_cast<uint32_t>(c), static_cast<uint32_t>(c >> 32), __float_as_uint(lg[j]), 0u);
    } else {
      out[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Stage 3: global budget set and softmax from the gathered records; fp64 partial output of this
// rank's final keys.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    shard_verify_kernel(const DecodeParams p, int64_t key_offset, int world, int rank,
                        const uint4* __restrict__ gathered, double* __restrict__ partial_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int B = p.a.budget;
  double* acc = reinterpret_cast<double*>(smem);  // (kThreads / 32) * 64 + kMaxHeadDim doubles
  float* lgs = reinterpret_cast<float*>(acc + (kThreads / 32) * 64 + kMaxHeadDim);
  int32_t* rows = reinterpret_cast<int32_t*>(lgs + B);
  float* w = reinterpret_cast<float*>(rows + B);
  __shared__ SelectScratch sc;
  __shared__ int scratch[64];
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  const int kvh = h / p.groups;
  const int P = p.n_probs;
  const int SL = p.a.shortlist;
  const int D = p.a.head_dim;
  const int tid = threadIdx.x;
  auto rec = [&](int i) -> uint4 {
    const int r = i / SL, j = i - r * SL;
    return __ldcg(gathered + ((size_t)r * P + prob) * SL + j);
  };
  auto item = [&](int i) -> unsigned long long {
    const uint4 v = rec(i);
    return (static_cast<unsigned long long>(v.y) << 32) | v.x;
  };
  const int N = world * SL;
  int nz = 0;
  for (int i = tid; i < N; i += blockDim.x) nz += item(i) != 0ull;
  const int n_sl = block_sum_int(nz, scratch);
  const int b = min(B, n_sl);
  const SelectThreshold thr = cta_radix_select(item, N, b, &sc);
  const int n_fin = cta_compact(item, N, thr,
                                [&](int pos, int i, unsigned long long) { lgs[pos] = __uint_as_float(rec(i).z); },
                                scratch);
  float mx, denom;
  softmax_stats(lgs, n_fin, scratch, acc, &mx, &denom);
  const uint32_t off = static_cast<uint32_t>(key_offset);
  auto own = [&](int j) -> unsigned long long { return item(rank * SL + j); };
  const int n_own = cta_compact(own, SL, thr,
                                [&](int pos, int j, unsigned long long c) {
                                  rows[pos] = static_cast<int32_t>(~static_cast<uint32_t>(c) - off);
                                  const float lj = __uint_as_float(rec(rank * SL + j).z);
                                  w[pos] = round_to<T>(expf(lj - mx) / denom);
                                },
                                scratch);
  double* sums = acc + (kThreads / 32) * 64;
  accumulate_rows<T>(p.a.values, p.a.v_head_stride, p.a.v_row_stride, kvh, D, rows, w, n_own, acc, sums);
  for (int d = tid; d < D; d += blockDim.x) partial_out[(size_t)prob * D + d] = sums[d];
  if (p.a.stats && rank == 0 && tid == 0) {
    atomicAdd(p.a.stats + SVA_STAT_QUERIES, 1ull);
    atomicAdd(p.a.stats + SVA_STAT_SUMMONED, static_cast<unsigned long long>(n_sl));
    atomicAdd(p.a.stats + SVA_STAT_EXACT_SCORED, static_cast<unsigned long long>(n_fin));
    atomicAdd(p.a.stats + SVA_STAT_VERIFIED, static_cast<unsigned long long>(n_fin));
  }
}

// Stage 4: the output, summing the ranks' partials in rank order.
template <typename T>
__global__ void shard_combine_kernel(const DecodeParams p, int world, const double* __restrict__ gathered) {
  const int prob = blockIdx.x;
  const int h = prob / p.a.n_queries, t = prob - h * p.a.n_queries;
  const int P = p.n_probs;
  const int D = p.a.head_dim;
  T* out = reinterpret_cast<T*>(p.a.out) + h * p.a.out_head_stride + t * p.a.out_row_stride;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double tot = 0.0;
    for (int r = 0; r < world; ++r) tot += __ldcg(gathered + ((size_t)r * P + prob) * D + d);
    out[d] = from_f32<T>(static_cast<float>(tot));
  }
}

static int plan_shard(const sva_decode_args* a, int64_t key_offset, DecodePlan* plan) {
  int rc = plan_decode(a, plan, /*force_grid=*/true);
  if (rc != SVA_OK) return rc;
  if (a->n_queries != 1) return set_error(SVA_ERR_SHAPE, "shards decode one query token per head (n_queries == 1)");
  if (a->allowed_len || a->allowed_mask) return set_error(SVA_ERR_SHAPE, "shards take no allowed_len / allowed_mask");
  if (a->shortlist_out || a->final_out) return set_error(SVA_ERR_SHAPE, "shards write no shortlist_out / final_out");
  if (a->shortlist > kShardMaxShortlist) return set_error(SVA_ERR_SHAPE, "shards take shortlist <= 8192");
  if (key_offset < 0 || key_offset + a->key_len > 0x7FFFFFFFll)
    return set_error(SVA_ERR_SHAPE, "key_offset + key_len must be in 0..2^31-1");
  return SVA_OK;
}

static int shard_world_ok(int32_t world, int32_t rank) {
  if (world < 1 || rank < 0 || rank >= world) return set_error(SVA_ERR_SHAPE, "need 0 <= rank < world");
  return SVA_OK;
}

static int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

template <typename T>
static int shard_summon(DecodePlan& plan, int64_t key_offset, unsigned long long* top_out, void* ws, cudaStream_t st) {
  DecodeParams& p = plan.p;
  bind_workspace(p, ws);
  p.dbg_ts = nullptr;
  int rc = launch_prep_scan<T>(p, st);
  if (rc != SVA_OK) return rc;
  const int smem = kCandSmem * static_cast<int>(sizeof(uint2)) + 4 * p.a.shortlist;
  rc = ensure_smem_attr(reinterpret_cast<const void*>(shard_top_kernel), smem);
  if (rc != SVA_OK) return rc;
  shard_top_kernel<<<p.a.n_heads, kThreads, smem, st>>>(p, key_offset, top_out);
  profile_mark(2, st);
  return launch_status();
}

template <typename T>
static int shard_rescore(DecodePlan& plan, int64_t key_offset, int world, int rank, const unsigned long long* gathered,
                         uint4* records, void* ws, cudaStream_t st) {
  DecodeParams& p = plan.p;
  bind_workspace(p, ws);
  const int smem = 16 * p.a.shortlist;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(shard_rescore_kernel<T>), smem);
  if (rc != SVA_OK) return rc;
  shard_rescore_kernel<T><<<p.a.n_heads, kThreads, smem, st>>>(p, key_offset, world, rank, gathered, records);
  return launch_status();
}

template <typename T>
static int shard_verify(DecodePlan& plan, int64_t key_offset, int world, int rank, const uint4* gathered,
                        double* partial, cudaStream_t st) {
  DecodeParams& p = plan.p;
  const int smem = 8 * ((kThreads / 32) * 64 + kMaxHeadDim) + 12 * p.a.budget;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(shard_verify_kernel<T>), smem);
  if (rc != SVA_OK) return rc;
  shard_verify_kernel<T><<<p.a.n_heads, kThreads, smem, st>>>(p, key_offset, world, rank, gathered, partial);
  return launch_status();
}

template <typename T>
static int shard_combine(DecodePlan& plan, int world, const double* gathered, cudaStream_t st) {
  shard_combine_kernel<T><<<plan.p.a.n_heads, 128, 0, st>>>(plan.p, world, gathered);
  return launch_status();
}

}  // namespace sva

extern "C" size_t sva_shard_workspace_size(const sva_decode_args* args) {
  sva::DecodePlan plan;
  if (sva::plan_shard(args, 0, &plan) != SVA_OK) return 0;
  return plan.ws_bytes;
}

extern "C" int sva_shard_summon(const sva_decode_args* args, int64_t key_offset, uint64_t* top_out, void* workspace,
                                size_t workspace_bytes, void* stream) {
  sva::DecodePlan plan;
  int rc = sva::plan_shard(args, key_offset, &plan);
  if (rc != SVA_OK) return rc;
  if (!top_out) return sva::set_error(SVA_ERR_SHAPE, "top_out is null");
  if (workspace_bytes < plan.ws_bytes || !workspace)
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_shard_workspace_size()");
  auto* top = reinterpret_cast<unsigned long long*>(top_out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::shard_summon<float>(plan, key_offset, top, workspace, s);
    case SVA_DTYPE_BF16: return sva::shard_summon<__nv_bfloat16>(plan, key_offset, top, workspace, s);
    default: return sva::shard_summon<__half>(plan, key_offset, top, workspace, s);
  }
}

extern "C" int sva_shard_rescore(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                                 const uint64_t* gathered_top, uint32_t* records_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  sva::DecodePlan plan;
  int rc = sva::plan_shard(args, key_offset, &plan);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, rank);
  if (rc != SVA_OK) return rc;
  if (!gathered_top || !records_out) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  if (workspace_bytes < plan.ws_bytes || !workspace)
    return sva::set_error(SVA_ERR_WORKSPACE, "workspace smaller than sva_shard_workspace_size()");
  auto* g = reinterpret_cast<const unsigned long long*>(gathered_top);
  auto* r = reinterpret_cast<uint4*>(records_out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::shard_rescore<float>(plan, key_offset, world, rank, g, r, workspace, s);
    case SVA_DTYPE_BF16: return sva::shard_rescore<__nv_bfloat16>(plan, key_offset, world, rank, g, r, workspace, s);
    default: return sva::shard_rescore<__half>(plan, key_offset, world, rank, g, r, workspace, s);
  }
}

extern "C" int sva_shard_verify(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                                const uint32_t* gathered_records, double* partial_out, void* stream) {
  sva::DecodePlan plan;
  int rc = sva::plan_shard(args, key_offset, &plan);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, rank);
  if (rc != SVA_OK) return rc;
  if (!gathered_records || !partial_out) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  auto* g = reinterpret_cast<const uint4*>(gathered_records);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::shard_verify<float>(plan, key_offset, world, rank, g, partial_out, s);
    case SVA_DTYPE_BF16: return sva::shard_verify<__nv_bfloat16>(plan, key_offset, world, rank, g, partial_out, s);
    default: return sva::shard_verify<__half>(plan, key_offset, world, rank, g, partial_out, s);
  }
}

extern "C" int sva_shard_combine(const sva_decode_args* args, int32_t world, const double* gathered_partials,
                                 void* stream) {
  sva::DecodePlan plan;
  int rc = sva::plan_shard(args, 0, &plan);
  if (rc == SVA_OK) rc = sva::shard_world_ok(world, 0);
  if (rc != SVA_OK) return rc;
  if (!gathered_partials) return sva::set_error(SVA_ERR_SHAPE, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->qkv_dtype) {
    case SVA_DTYPE_F32: return sva::shard_combine<float>(plan, world, gathered_partials, s);
    case SVA_DTYPE_BF16: return sva::shard_combine<__nv_bfloat16>(plan, world, gathered_partials, s);
    default: return sva::shard_combine<__half>(plan, world, gathered_partials, s);
  }
}
