/*
 * sva_b200.h -- C ABI of the B200 (sm_100a) summon -> verify decode path.
 *
 * Every entry point takes device pointers, sizes in elements, and a cudaStream_t passed as
 * void*.  Nothing here allocates device memory: callers pass outputs and a workspace sized by
 * the matching *_workspace_size() call.  No entry point synchronises the stream.  Each returns
 * SVA_OK or an sva_status error code; sva_last_error() gives a one-line message for the last
 * failure on the calling thread.
 *
 * Reference interfaces replaced (asystemoffields/sva):
 *   sva_catalog_encode      sva/llama.py:578-624 (_key_catalog: k_low einsum + encode_product_keys)
 *                           sva/ops.py:24-47 (encode_product_keys), sva/ops.py:10-21 (assign_to_centroids)
 *   sva_assign_centroids    sva/ops.py:10-21 (assign_to_centroids)
 *   sva_pq_scores           sva/ops.py:50-71 (product_quantized_scores)
 *   sva_decode              sva/llama.py:171-328 (SVALlamaAttention.sva_attention, scan summon path)
 *   sva_decode_batched      sva/llama.py:171-328 over the sequences of a batch (the reference takes batch 1)
 *   sva_postings_build      sva/llama.py:626-657 (_rebuild_postings)
 *   sva_decode_inverted     sva/llama.py:427-576 (_inverted_static_decode_attention) and
 *                           sva/llama.py:330-425 (_inverted_decode_attention)
 *   sva_top_unique          sva/llama.py:83-116 (_top_unique_candidates)
 *   sva_adapter_forward     experiments/sva_late4_logit_distill.py:37-51 (SVAResidualOutputAdapter) + o_proj
 */
#ifndef SVA_B200_H_
#define SVA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum sva_status {
  SVA_OK = 0,
  SVA_ERR_SHAPE = 1,     /* unsupported or inconsistent sizes */
  SVA_ERR_WORKSPACE = 2, /* workspace smaller than *_workspace_size() */
  SVA_ERR_TIMEOUT = 3,   /* a bounded wait gave up */
  SVA_ERR_CUDA = 4,      /* a CUDA launch or runtime call failed */
  SVA_ERR_ALIGN = 5,     /* pointer or stride alignment not supported */
  SVA_ERR_DTYPE = 6      /* unsupported dtype code */
} sva_status;

typedef enum sva_dtype { SVA_DTYPE_F32 = 0, SVA_DTYPE_BF16 = 1, SVA_DTYPE_F16 = 2 } sva_dtype;

/* Device counters accumulated by the decode entry points (unsigned 64-bit). */
enum {
  SVA_STAT_QUERIES = 0,
  SVA_STAT_SUMMONED = 1,
  SVA_STAT_REFILL_POOL = 2,
  SVA_STAT_EXACT_SCORED = 3,
  SVA_STAT_VERIFIED = 4,
  SVA_STAT_CELL_VISITS = 5,
  SVA_STAT_SELECT_FALLBACKS = 6, /* million-key schedule: sampled threshold too high, exact rescan */
  SVA_STAT_COUNT = 8
};

/* Library version string and last error message (thread-local). */
const char* sva_version(void);
const char* sva_last_error(void);

/* Timing hook (no reference counterpart; measurement only).  When set on the calling thread,
 * every multi-kernel entry point records events[i] (a cudaEvent_t created with timing enabled)
 * on its stream right after its i-th internal kernel launch, for i < n.  Events are recorded as
 * external events, so the hook also works inside CUDA-graph capture.  Pass n = 0 to clear. */
int sva_profile_events(void* const* events, int32_t n);

/* 1 if p is page-locked host memory that device code can read and write at the same address
 * (cudaHostAlloc / cudaMallocHost memory, mapped in the unified address space), else 0.  No
 * reference counterpart: sva_decode accepts such buffers for `query` and `out`, so that a host
 * caller's per-token input and output cross PCIe inside the kernels instead of in separate copy
 * operations; this is the check a caller makes before passing them. */
int sva_host_buffer_device_accessible(const void* p);

/* Phase-timestamp hook (no reference counterpart; measurement only).  When set on the calling
 * thread, the million-key schedule of sva_decode writes %globaltimer nanoseconds at its phase
 * boundaries into device_buffer[problem * 16 + slot] (slots 0..15).  Pass NULL to clear. */
int sva_debug_timestamps(void* device_buffer);

/* ---------------------------------------------------------------------------------------
 * Write path: key catalog.
 * k_low[h][l][:] = K[h / (H/Hkv)][l][:] . k_proj[h]        (fp32, sequential order over D)
 * codes[h][l][s] = argmin_c (|x|^2 - 2 x.c) + |c|^2,  x = k_low[h][l][s*R/S:(s+1)*R/S]
 * for l in [start, start + count).  Layouts: keys [Hkv][*][D] with the given strides;
 * k_proj [H][D][R]; codebooks [H][S][C][R/S]; k_low [H][*][R] (row stride R);
 * codes [H][*][S] uint8 (row stride S).  Either k_low or codes may be NULL to skip it
 * (codes still need k_low values, which are then kept in registers only).
 * Replaces sva/llama.py:578-624 and sva/ops.py:10-47.
 * ------------------------------------------------------------------------------------- */
int sva_catalog_encode(const void* keys, int32_t key_dtype, int64_t key_head_stride, int64_t key_row_stride,
                       int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t rank_dim,
                       const float* k_proj, const float* codebooks, int32_t subspaces, int32_t codewords,
                       int64_t start, int64_t count, float* k_low, int64_t k_low_head_stride, uint8_t* codes,
                       int64_t codes_head_stride, void* stream);

/* The same for rows [*start, *start + count) with the start row read from device memory, so that
 * the call can sit in a captured CUDA graph whose replays append at a moving position; rows at or
 * beyond `limit` (the capacity of keys, k_low and codes) are skipped.  No reference counterpart:
 * the reference appends with torch.cat (sva/llama.py:599-613). */
int sva_catalog_encode_at(const void* keys, int32_t key_dtype, int64_t key_head_stride, int64_t key_row_stride,
                          int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t rank_dim,
                          const float* k_proj, const float* codebooks, int32_t subspaces, int32_t codewords,
                          const int64_t* start, int64_t count, int64_t limit, float* k_low,
                          int64_t k_low_head_stride, uint8_t* codes, int64_t codes_head_stride, void* stream);

/* The same on the tensor cores: k_low = K . Kproj by tcgen05 MMA (bf16 operands, fp32
 * accumulator in tensor memory), then the same nearest-codeword assignment on the fp32 rows.
 * K must be bf16 with 16-byte aligned rows; Kproj is rounded to bf16, which is exact for bf16
 * artifacts; head_dim a multiple of 16 up to 128, rank_dim a multiple of 16 up to 64.  k_low
 * differs from sva_catalog_encode's only in the fp32 summation order (a few ulp), so codes can
 * differ only where two codewords are that close.  *status (device int, may be NULL) is set to
 * SVA_ERR_TIMEOUT if a tile's tensor-core wait ran out.  Replaces sva/llama.py:578-624. */
int sva_catalog_encode_tc(const void* keys, int32_t key_dtype, int64_t key_head_stride, int64_t key_row_stride,
                          int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t rank_dim,
                          const float* k_proj, const float* codebooks, int32_t subspaces, int32_t codewords,
                          int64_t start, int64_t count, float* k_low, int64_t k_low_head_stride, uint8_t* codes,
                          int64_t codes_head_stride, int32_t* status, void* stream);

/* Nearest centroid of each row of x [n][dim] (row stride x_row_stride) among centroids
 * [C][dim]; labels as int64.  Replaces sva/ops.py:10-21. */
int sva_assign_centroids(const float* x, int64_t n, int32_t dim, int64_t x_row_stride, const float* centroids,
                         int32_t codewords, int64_t* labels, void* stream);

/* ADC scores: scores[h][t][l] = (sum_s lut[h][t][s][codes[h][l][s]]) / sqrt(R) with
 * lut[h][t][s][c] = q_low[h][t][s-part] . codebooks[h][s][c].  q_low [H][T][R];
 * codes [H][L][S] uint8; scores [H][T][L] fp32.  Replaces sva/ops.py:50-71. */
int sva_pq_scores(const float* q_low, int32_t n_heads, int32_t n_queries, int32_t rank_dim, const float* codebooks,
                  int32_t subspaces, int32_t codewords, const uint8_t* codes, int64_t key_len, float* scores,
                  void* stream);

/* ---------------------------------------------------------------------------------------
 * Scan summon -> rank rescore -> exact verify for H heads x T query tokens.
 * Replaces sva/llama.py:171-328.  Per (head h, token t):
 *   q_low = (q . q_proj[h]) * scale[h]; lut = q_low parts . codebooks;
 *   shortlist = top-min(shortlist, allowed) allowed keys by ADC score (score desc, index asc);
 *   final = top-min(budget, |shortlist|) of the shortlist by q_low . k_low / sqrt(R);
 *   out = softmax(q . K[final] * softmax_scale) @ V[final].
 * ------------------------------------------------------------------------------------- */
typedef struct sva_decode_args {
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t n_queries;
  int32_t head_dim;
  int32_t rank_dim;
  int32_t subspaces;
  int32_t codewords;
  int32_t shortlist;
  int32_t budget;
  int32_t qkv_dtype;   /* sva_dtype of query, keys, values and out */
  int32_t logits_mode; /* 0: fp32 logits; 1: logits rounded like the value dtype (scan path) */
  float softmax_scale;
  int64_t key_len;
  /* query side */
  const void* query; /* [H][T][D]; device memory or page-locked host memory (see
                       sva_host_buffer_device_accessible) */
  int64_t q_head_stride, q_row_stride;
  const float* q_proj;       /* [H][D][R] */
  const float* scale;        /* [H], clamp(exp(logit_scale), 0.01, 100) */
  const float* codebooks;    /* [H][S][C][R/S] */
  const float* lut_override; /* [H][T][S][C] or NULL */
  /* catalog and cache */
  const uint8_t* codes; /* [H][L][S] */
  int64_t codes_head_stride;
  const float* k_low; /* [H][L][R] */
  int64_t k_low_head_stride;
  const void* keys; /* [Hkv][L][D] */
  int64_t k_head_stride, k_row_stride;
  const void* values; /* [Hkv][L][D] */
  int64_t v_head_stride, v_row_stride;
  /* masking: key l is allowed for token t iff l < allowed_len[t] (NULL: L - T + t + 1) and
   * (allowed_mask == NULL or allowed_mask[t * mask_row_stride + l] != 0) */
  const int64_t* allowed_len;
  const uint8_t* allowed_mask;
  int64_t mask_row_stride;
  /* outputs */
  void* out; /* [H][T][D]; device memory or page-locked host memory */
  int64_t out_head_stride, out_row_stride;
  int32_t* shortlist_out;    /* [H][T][shortlist] ascending key index, -1 padded, or NULL */
  int32_t* final_out;        /* [H][T][budget] ascending key index, -1 padded, or NULL */
  unsigned long long* stats; /* [SVA_STAT_COUNT] accumulated, or NULL */
} sva_decode_args;

size_t sva_decode_workspace_size(const sva_decode_args* args);
int sva_decode(const sva_decode_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Batched, ragged and paged scan decode: the decode of sva_decode for n_seqs sequences in one
 * call, each with its own cache length and (optionally) a paged catalog.  The reference decodes
 * one sequence per call (sva/llama.py:182-183 rejects batch != 1); this replaces a loop of its
 * sva/llama.py:171-328 over the sequences of a batch.
 *
 * Problems are (sequence b, head h, token t).  args describes one sequence as for sva_decode;
 * args->key_len is the largest sequence length (the workspace is sized for it).  Sequence b:
 *   keys           seq_lens[b] (NULL: args->key_len for every sequence);
 *   query / out    args->query + b * q_seq_stride (out_seq_stride), then the head / token strides;
 *   allowed_len    [n_seqs][T] (NULL: seq_lens[b] - T + t + 1); allowed_mask rows b * T + t;
 *   shortlist_out / final_out  [n_seqs][H][T][...].
 * Key l of sequence b, head h (kvh = h / (H / Hkv) for K and V):
 *   unpaged (page_table == NULL): codes + h * codes_head_stride + b * codes_page_stride + l * S,
 *     and the same with k_low_page_stride, k_page_stride, v_page_stride (per-sequence strides);
 *   paged: page = page_table[b * page_table_stride + l / page_keys], row = l % page_keys:
 *     codes + h * codes_head_stride + page * codes_page_stride + row * S, and the same for k_low
 *     (row * R), K (row * k_row_stride) and V (row * v_row_stride).
 * page_keys is a power of two in 64..32768.  Over 32768 keys, n_seqs * H * T <= 65535 per call.
 * Every problem's shortlist, final set and output equal sva_decode's for that sequence alone.
 * ------------------------------------------------------------------------------------- */
typedef struct sva_batch_layout {
  int32_t n_seqs;
  int32_t page_keys;
  const int64_t* seq_lens;    /* [n_seqs] device, or NULL */
  const int32_t* page_table;  /* [n_seqs][page_table_stride] device, or NULL */
  int64_t page_table_stride;
  int64_t q_seq_stride, out_seq_stride;          /* elements */
  int64_t codes_page_stride, k_low_page_stride;  /* elements per page (paged) or sequence */
  int64_t k_page_stride, v_page_stride;
} sva_batch_layout;

size_t sva_decode_batched_workspace_size(const sva_decode_args* args, const sva_batch_layout* layout);
int sva_decode_batched(const sva_decode_args* args, const sva_batch_layout* layout, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Key-range shards: the scan decode of one token per head with the catalog split by key range
 * across ranks, one process per GPU.  Replaces the single-device sva/llama.py:171-328 when the
 * cache does not live on one GPU (the reference itself is single-device).
 *
 * Rank r's args describe its own keys, global indices [key_offset, key_offset + key_len), with
 * n_queries == 1, no allowed_len / allowed_mask and no shortlist_out / final_out; shortlist
 * <= 8192.  The same args go to every stage of one decode.  The host all-gathers each stage's
 * output over the W ranks, in rank order, before the next stage ([W][...] below):
 *   sva_shard_summon : top_out [H][shortlist] u64 composites (coarse key << 32 | ~global index)
 *                      of the exact local shortlist, zero padded.  Uses the workspace.
 *   sva_shard_rescore: from gathered_top [W][H][shortlist], the global shortlist; this rank's
 *                      members rescored and their verify logits computed -> records_out
 *                      [H][shortlist][4] u32 (rank composite lo, hi, logit bits, 0), zero
 *                      padded.  Takes the workspace sva_shard_summon filled, unchanged.
 *   sva_shard_verify : from gathered_records [W][H][shortlist][4], the global budget set and
 *                      softmax; partial_out [H][head_dim] f64 = this rank's share of the output.
 *   sva_shard_combine: from gathered_partials [W][H][head_dim], writes args->out.
 * Shortlist and final sets equal sva_decode's over the concatenated keys; the output equals it
 * up to the order of exact fp64 sums.  Stats (queries, summoned, verified) are counted on rank 0.
 * ------------------------------------------------------------------------------------- */
size_t sva_shard_workspace_size(const sva_decode_args* args);
int sva_shard_summon(const sva_decode_args* args, int64_t key_offset, uint64_t* top_out, void* workspace,
                     size_t workspace_bytes, void* stream);
int sva_shard_rescore(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                      const uint64_t* gathered_top, uint32_t* records_out, void* workspace, size_t workspace_bytes,
                      void* stream);
int sva_shard_verify(const sva_decode_args* args, int64_t key_offset, int32_t world, int32_t rank,
                     const uint32_t* gathered_records, double* partial_out, void* stream);
int sva_shard_combine(const sva_decode_args* args, int32_t world, const double* gathered_partials, void* stream);

/* ---------------------------------------------------------------------------------------
 * Batched shards: the same four stages for a batch of sequences (sva_batch_layout) and with a
 * narrower first exchange.  Replaces the single-device sva/llama.py:171-328 for batches whose
 * caches are split across ranks (the reference is single-device).
 *
 * sva_shard_map gives each rank's local -> global key numbering (the tie rule uses global
 * indices): key-range shards (page_world == 0) hold global keys [key_offset, key_offset + L_r)
 * of every sequence; page-dealt shards (page_world > 0, paged layout required) hold global page
 * g of every sequence on rank g % page_world as local page g / page_world, rows unchanged.
 *
 * exchange_width k1 (0 < k1 <= shortlist, 0 meaning the shortlist): each rank sends its local
 * top-k1 per problem (top_out [P][k1] u64) and the records of its shortlist members
 * (records_out [P][k1][4] u32); the host all-gathers them to [W][P][k1] as before.  The global
 * shortlist is exact whenever no rank has more than k1 members; the rescore stage sets
 * *saturated (device int32, may be NULL) when a rank sent k1 entries that are all members, in
 * which case the host must repeat the decode with exchange_width = shortlist.  With k1 near
 * shortlist / W the first two exchanges shrink about W-fold.  P = n_seqs * n_heads problems
 * (n_queries == 1); partial_out and gathered partials are [P][head_dim] as before.
 * ------------------------------------------------------------------------------------- */
typedef struct sva_shard_map {
  int64_t key_offset;
  int32_t page_world;
  int32_t page_rank;
} sva_shard_map;

size_t sva_shard_batched_workspace_size(const sva_decode_args* args, const sva_batch_layout* layout,
                                        const sva_shard_map* map, int32_t exchange_width);
int sva_shard_batched_summon(const sva_decode_args* args, const sva_batch_layout* layout, const sva_shard_map* map,
                             int32_t exchange_width, uint64_t* top_out, void* workspace, size_t workspace_bytes,
                             void* stream);
int sva_shard_batched_rescore(const sva_decode_args* args, const sva_batch_layout* layout, const sva_shard_map* map,
                              int32_t exchange_width, int32_t world, int32_t rank, const uint64_t* gathered_top,
                              uint32_t* records_out, int32_t* saturated, void* workspace, size_t workspace_bytes,
                              void* stream);
int sva_shard_batched_verify(const sva_decode_args* args, const sva_batch_layout* layout, const sva_shard_map* map,
                             int32_t exchange_width, int32_t world, int32_t rank, const uint32_t* gathered_records,
                             double* partial_out, void* stream);
int sva_shard_batched_combine(const sva_decode_args* args, const sva_batch_layout* layout, int32_t world,
                              const double* gathered_partials, void* stream);

/* ---------------------------------------------------------------------------------------
 * Posting lists of the static inverted index.  Replaces sva/llama.py:626-657.
 * For every (head, subspace): counts [H][S][C], offsets [H][S][C+1] (CSR) and ids
 * [H][S][ids_sub_stride] holding the keys [0, key_len) grouped by code, ascending inside a cell.
 * *max_bucket (device int32) receives the largest cell size over all heads and subspaces.
 * ------------------------------------------------------------------------------------- */
size_t sva_postings_workspace_size(int32_t n_heads, int32_t subspaces, int32_t codewords, int64_t key_len);
int sva_postings_build(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads, int32_t subspaces,
                       int32_t codewords, int64_t key_len, int32_t* counts, int32_t* offsets, int32_t* ids,
                       int64_t ids_sub_stride, int32_t* max_bucket, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---------------------------------------------------------------------------------------
 * Incremental posting lists (replaces sva/llama.py:659-693, _append_postings): keys
 * [start, start + count) are appended, in key order, to the lists of their codes, so every list
 * stays ascending and equals what sva_postings_build would give for keys [0, start + count).
 * The layout is padded: cell c of (head, subspace) owns id slots [offsets[c], offsets[c + 1]),
 * counts[c] of them used; a key that would pass its cell's end is skipped and *overflow (device
 * int32) is set, so callers size the cells from a bound on the counts (and rebuild when the bound
 * reaches the cell size).  *max_bucket is raised to the largest count written.
 * ------------------------------------------------------------------------------------- */
int sva_postings_append(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads, int32_t subspaces,
                        int32_t codewords, int64_t start, int64_t count, int32_t* counts, const int32_t* offsets,
                        int32_t* ids, int64_t ids_sub_stride, int32_t* max_bucket, int32_t* overflow, void* stream);

/* ---------------------------------------------------------------------------------------
 * No-alloc variant of sva_postings_build.  No reference counterpart: the reference builds its
 * posting lists with torch ops that allocate as they go (sva/llama.py:626-657).
 *
 * For callers that cannot allocate device memory on the call path: a host runtime bound to
 * this library through a C foreign-function interface, which has no device allocator of its
 * own, or a server that fixes its device memory when it starts.  The chunk histograms live in
 * a buffer inside the library, SVA_POSTINGS_NOALLOC_SCRATCH_BYTES per device, so the call takes
 * no workspace; the outputs are the caller's, exactly as for sva_postings_build.
 * Limit: sva_postings_workspace_size(n_heads, subspaces, codewords, key_len), that is
 * 4 * H * S * C * ceil(L / 4096) bytes, must not exceed the buffer, else SVA_ERR_WORKSPACE
 * (9 heads of 4x64 codes: up to 3.7M keys; 1 head of 1x256 codes: up to 33M keys).
 * Calls on one device share the buffer: two calls that may overlap in time (on different
 * streams, or from host threads without ordering between them) race and corrupt each other's
 * lists, so issue them on one stream.  The first call on each device looks up the buffer's
 * address, which may load the library's device module: make it before any stream capture.
 * The address is kept per device together with the id of the context it belongs to, and looked
 * up again when a call comes from another context (after cudaDeviceReset, or under a context
 * the caller created with the driver API); such a first call is also a set-up call.
 * Nothing is claimed about CUDA graph capture of this entry point.
 * ------------------------------------------------------------------------------------- */
#define SVA_POSTINGS_NOALLOC_SCRATCH_BYTES (8u << 20)
int sva_postings_build_noalloc(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads, int32_t subspaces,
                               int32_t codewords, int64_t key_len, int32_t* counts, int32_t* offsets, int32_t* ids,
                               int64_t ids_sub_stride, int32_t* max_bucket, void* stream);

/* ---------------------------------------------------------------------------------------
 * Inverted-index summon -> rank rescore -> verify for one query token per head.
 * static  (dynamic == 0), replaces sva/llama.py:427-576: candidates are the posting lists of the
 *         top `cells` codewords per subspace (code score desc, codeword asc) plus the tail keys
 *         [postings_len, key_len) (or the current key key_len-1 when there is no tail); the
 *         refill window is the first min(W, max(budget, budget * refill_factor)) entries in
 *         (rank score desc, key asc) order counting duplicates, W the reference's padded width;
 *         the window's unique keys, best first, are the selection (sva/llama.py:83-116).
 * dynamic (dynamic == 1), replaces sva/llama.py:330-425: all unique candidates plus the current
 *         key are ranked; no tail, no window.
 * Both then apply the adaptive budget rule (margin between the best and the min_budget-th
 * rank score) and verify with fp32 logits.  `budget` is the already clamped max budget,
 * min_budget / mid_budget are clamped as the reference clamps them.
 * ------------------------------------------------------------------------------------- */
typedef struct sva_inverted_args {
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t rank_dim;
  int32_t subspaces;
  int32_t codewords;
  int32_t budget;
  int32_t cells;
  int32_t refill_factor;
  int32_t dynamic;
  int32_t min_budget;
  int32_t mid_budget;
  int32_t qkv_dtype;
  float low_margin;
  float high_margin;
  float softmax_scale;
  int64_t key_len;      /* keys in k_low / K / V */
  int64_t postings_len; /* keys covered by the posting lists */
  int64_t allowed_len;  /* keys [0, allowed_len) are allowed ... */
  const uint8_t* allowed_mask; /* ... and, if not NULL, only keys with allowed_mask[key] != 0 */
  const void* query;    /* [H][D], one token per head */
  int64_t q_head_stride;
  const float* q_proj;
  const float* scale;
  const float* codebooks;
  const uint8_t* codes; /* [H][>= postings_len][S] */
  int64_t codes_head_stride;
  const int32_t* post_counts;  /* [H][S][C] */
  const int32_t* post_offsets; /* [H][S][C+1] */
  const int32_t* post_ids;     /* [H][S][post_ids_sub_stride] */
  int64_t post_ids_sub_stride;
  const int32_t* max_bucket; /* device int32 from sva_postings_build */
  const float* k_low;        /* [H][key_len][R] */
  int64_t k_low_head_stride;
  const void* keys; /* [Hkv][key_len][D] */
  int64_t k_head_stride, k_row_stride;
  const void* values;
  int64_t v_head_stride, v_row_stride;
  void* out; /* [H][D] */
  int64_t out_head_stride;
  int32_t* sel_idx_out;      /* [H][budget] selection, best first (0 in invalid slots), or NULL */
  uint8_t* sel_valid_out;    /* [H][budget] refill validity before the budget cut, or NULL */
  float* sel_score_out;      /* [H][budget] rank scores (float min in invalid slots), or NULL */
  int32_t* budget_out;       /* [H] adaptive budget per head, or NULL */
  unsigned long long* stats; /* [SVA_STAT_COUNT] accumulated, or NULL */
} sva_inverted_args;

size_t sva_inverted_workspace_size(const sva_inverted_args* args);
int sva_decode_inverted(const sva_inverted_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Key-range shards of the static inverted-index summon.  Replaces sva/llama.py:427-576 when the
 * static catalog is split by key range across ranks (the reference is single-device).
 * Rank r's args describe its own keys, global indices [key_offset, key_offset + key_len), with
 * posting lists over all of them (postings_len == key_len), dynamic == 0, allowed_len ==
 * key_len, no allowed_mask and no selection outputs; max_bucket points to the largest posting
 * list of the whole (global) catalog, and holds_current is 1 on the rank holding the global last
 * key (the reference's current-key candidate), 0 elsewhere.  key_offset + key_len < 2^28.
 *   sva_inverted_shard_summon : records_out [H][budget][4] u32: the rank's top-budget unique
 *                               candidates (rank composite with the global key index and the
 *                               multiplicity, fp32 verify logit), zero padded.  all-gather.
 *   sva_inverted_shard_verify : from gathered [W][H][budget][4], the global selection, refill
 *                               window, adaptive budget and softmax; partial_out [H][head_dim] f64
 *                               = this rank's share of the output.  Takes the workspace the
 *                               summon filled.  all-gather.
 *   sva_inverted_shard_combine: from gathered partials [W][H][head_dim], writes args->out.
 * The final sets equal sva_decode_inverted's over the concatenated keys; outputs equal it up to
 * the order of exact fp64 sums.
 * ------------------------------------------------------------------------------------- */
size_t sva_inverted_shard_workspace_size(const sva_inverted_args* args);
int sva_inverted_shard_summon(const sva_inverted_args* args, int64_t key_offset, int32_t holds_current,
                              uint32_t* records_out, void* workspace, size_t workspace_bytes, void* stream);
int sva_inverted_shard_verify(const sva_inverted_args* args, int64_t key_offset, int32_t holds_current, int32_t world,
                              int32_t rank, const uint32_t* gathered_records, double* partial_out, void* workspace,
                              size_t workspace_bytes, void* stream);
int sva_inverted_shard_combine(const sva_inverted_args* args, int32_t world, const double* gathered_partials,
                               void* stream);

/* ---------------------------------------------------------------------------------------
 * Refill-and-dedupe selection on explicit candidate rows.  Replaces sva/llama.py:83-116
 * (_top_unique_candidates).  idx [rows][width] int64, scores [rows][width] fp32, valid
 * [rows][width] uint8; outputs [rows][min(budget, refill)] best first: sel_idx int64 (0 in
 * invalid slots), sel_scores (float min in invalid slots), sel_valid uint8; *refill_out (host
 * int32) receives the refill count.  width <= 8192.
 * ------------------------------------------------------------------------------------- */
int sva_top_unique(const int64_t* idx, const float* scores, const uint8_t* valid, int32_t rows, int32_t width,
                   int32_t budget, int32_t refill_factor, int64_t* sel_idx, float* sel_scores, uint8_t* sel_valid,
                   int32_t* refill_out, void* stream);

/* ---------------------------------------------------------------------------------------
 * Residual output adapter fused with o_proj, for decode-sized row counts.  Replaces the late-layer
 * socket's SVAResidualOutputAdapter.forward (experiments/sva_late4_logit_distill.py:37-51) plus
 * the wrapped attention's o_proj (sva/llama.py:169):
 *   o   = attn . o_weight^T (+ o_bias), rounded to dtype     attn [N][in_dim], o_weight [hidden][in_dim]
 *   c   = up . gelu(down . [float(hidden), float(o)]) * scale  (fp32; down [rank][2 hidden], up [hidden][rank])
 *   out = round(o + round(c))                               [N][hidden]
 * hidden / attn / o_weight / o_bias / out share `dtype` (sva_dtype); down and up are fp32.
 * hidden_dim <= 4096 with 16 * (2 hidden_dim + rank) + small slices fitting shared memory.
 * ------------------------------------------------------------------------------------- */
int sva_adapter_forward(const void* hidden, int64_t hidden_row_stride, const void* attn, int64_t attn_row_stride,
                        int32_t dtype, const void* o_weight, const void* o_bias, const float* down, const float* up,
                        float scale, int32_t n_rows, int32_t hidden_dim, int32_t in_dim, int32_t rank, void* out,
                        int64_t out_row_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SVA_B200_H_ */
