// Posting lists of the static inverted index (replaces sva/llama.py:626-657, _rebuild_postings).
//
// For every (head h, subspace s) the keys [0, L) are grouped by their code into CSR posting
// lists: counts[h][s][c], offsets[h][s][c] (offsets[..][C] = L) and ids[h][s][offsets..] with key
// ids ascending inside each cell (a stable counting sort, so the layout is deterministic).  The
// reference stores the same lists padded to the largest bucket; it also needs that largest
// bucket size, which is written to *max_bucket (a device int).
//
// Three passes over the codes, no atomics on the ids:
//   1. per chunk of kChunk keys: histogram of codes -> chunk_hist[hs][chunk][c]
//   2. per (h, s): counts, offsets, and the base of every (chunk, c) run (in place)
//   3. per chunk: stable scatter; within a round of 256 keys the rank of a key among same-code
//      keys comes from a warp match plus per-warp counters, so ids keep key order.
#include <mutex>

#include "sva_common.cuh"
#include "sva_internal.h"

namespace sva {

constexpr int kPostChunk = 4096;
constexpr int kPostThreads = 256;

struct PostParams {
  const uint8_t* codes;
  int64_t codes_head_stride;
  int H, S, C;
  int64_t L;
  int nchunks;
  int32_t* counts;   // [H][S][C]
  int32_t* offsets;  // [H][S][C+1]
  int32_t* ids;      // [H][S][ids_sub_stride]
  int64_t ids_sub_stride;
  int32_t* max_bucket;
  int32_t* chunk_hist;  // [H*S][nchunks][C]
};

__global__ void __launch_bounds__(kPostThreads) post_hist_kernel(const PostParams p) {
  __shared__ int hist[kMaxCodewords];
  const int hs = blockIdx.y, chunk = blockIdx.x;
  const int h = hs / p.S, s = hs - h * p.S;
  for (int c = threadIdx.x; c < p.C; c += blockDim.x) hist[c] = 0;
  __syncthreads();
  const uint8_t* cb = p.codes + h * p.codes_head_stride + s;
  const int64_t i0 = (int64_t)chunk * kPostChunk;
  const int64_t i1 = min(p.L, i0 + kPostChunk);
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int c = __ldg(cb + i * p.S);
    if (c < p.C) atomicAdd(&hist[c], 1);
  }
  __syncthreads();
  int32_t* out = p.chunk_hist + ((size_t)hs * p.nchunks + chunk) * p.C;
  for (int c = threadIdx.x; c < p.C; c += blockDim.x) out[c] = hist[c];
}

__global__ void __launch_bounds__(kPostThreads) post_scan_kernel(const PostParams p) {
  __shared__ int tot[kMaxCodewords];
  __shared__ int scratch[kPostThreads / 32 + 1];
  const int hs = blockIdx.x;
  const int c = threadIdx.x;
  int32_t* ch = p.chunk_hist + (size_t)hs * p.nchunks * p.C;
  int total = 0;
  if (c < p.C)
    for (int k = 0; k < p.nchunks; ++k) total += ch[(size_t)k * p.C + c];
  int all;
  const int excl = block_excl_scan(c < p.C ? total : 0, scratch, &all);
  if (c < p.C) {
    tot[c] = total;
    p.counts[(size_t)hs * p.C + c] = total;
    p.offsets[(size_t)hs * (p.C + 1) + c] = excl;
    if (c == p.C - 1) p.offsets[(size_t)hs * (p.C + 1) + p.C] = excl + total;
    int run = excl;
    for (int k = 0; k < p.nchunks; ++k) {
      const int v = ch[(size_t)k * p.C + c];
      ch[(size_t)k * p.C + c] = run;  // becomes the base of (chunk k, code c)
      run += v;
    }
    if (total > 0) atomicMax(p.max_bucket, total);
  }
}

__global__ void __launch_bounds__(kPostThreads) post_scatter_kernel(const PostParams p) {
  __shared__ int base[kMaxCodewords];     // running position per code inside this chunk
  __shared__ int wcnt[kPostThreads / 32][kMaxCodewords];
  const int hs = blockIdx.y, chunk = blockIdx.x;
  const int h = hs / p.S, s = hs - h * p.S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int32_t* cbase = p.chunk_hist + ((size_t)hs * p.nchunks + chunk) * p.C;
  for (int c = tid; c < p.C; c += blockDim.x) base[c] = cbase[c];
  const uint8_t* cb = p.codes + h * p.codes_head_stride + s;
  int32_t* ids = p.ids + (size_t)hs * p.ids_sub_stride;
  const int64_t i0 = (int64_t)chunk * kPostChunk;
  const int64_t i1 = min(p.L, i0 + kPostChunk);
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t r0 = i0; r0 < i1; r0 += blockDim.x) {
    for (int e = tid; e < nwarps * p.C; e += blockDim.x) wcnt[e / p.C][e % p.C] = 0;
    __syncthreads();
    const int64_t i = r0 + tid;
    const bool ok = i < i1;
    int c = ok ? static_cast<int>(__ldg(cb + i * p.S)) : -1;
    if (c >= p.C) c = -1;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, c);
    const int rank_in_warp = __popc(same & lt);
    if (c >= 0 && rank_in_warp == 0) wcnt[warp][c] = __popc(same);
    __syncthreads();
    if (c >= 0) {
      int pos = base[c] + rank_in_warp;
      for (int w = 0; w < warp; ++w) pos += wcnt[w][c];
      ids[pos] = static_cast<int32_t>(i);
    }
    __syncthreads();
    for (int cc = tid; cc < p.C; cc += blockDim.x) {
      int add = 0;
      for (int w = 0; w < nwarps; ++w) add += wcnt[w][cc];
      base[cc] += add;
    }
    __syncthreads();
  }
}

}  // namespace sva

using namespace sva;

extern "C" size_t sva_postings_workspace_size(int32_t n_heads, int32_t subspaces, int32_t codewords, int64_t key_len) {
  if (n_heads <= 0 || subspaces <= 0 || codewords <= 0 || key_len <= 0) return 0;
  const int64_t nchunks = (key_len + kPostChunk - 1) / kPostChunk;
  return sizeof(int32_t) * (size_t)n_heads * subspaces * nchunks * codewords;
}

extern "C" int sva_postings_build(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads, int32_t subspaces,
                                  int32_t codewords, int64_t key_len, int32_t* counts, int32_t* offsets, int32_t* ids,
                                  int64_t ids_sub_stride, int32_t* max_bucket, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (n_heads <= 0 || subspaces <= 0 || subspaces > kMaxSubspaces || codewords <= 0 || codewords > kMaxCodewords)
    return set_error(SVA_ERR_SHAPE, "bad postings shape");
  if (key_len < 0 || key_len > 0x7FFFFFFFll) return set_error(SVA_ERR_SHAPE, "key_len out of range");
  if (ids_sub_stride < key_len) return set_error(SVA_ERR_SHAPE, "ids_sub_stride must be >= key_len");
  if (!counts || !offsets || !ids || !max_bucket || (key_len > 0 && !codes))
    return set_error(SVA_ERR_SHAPE, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(max_bucket, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  const size_t need = sva_postings_workspace_size(n_heads, subspaces, codewords, key_len);
  if (key_len == 0) {
    e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * n_heads * subspaces * codewords, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(offsets, 0, sizeof(int32_t) * n_heads * subspaces * (codewords + 1), st);
    return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  }
  if (workspace_bytes < need || !workspace) return set_error(SVA_ERR_WORKSPACE, "postings workspace too small");
  PostParams p;
  p.codes = codes;
  p.codes_head_stride = codes_head_stride;
  p.H = n_heads;
  p.S = subspaces;
  p.C = codewords;
  p.L = key_len;
  p.nchunks = static_cast<int>((key_len + kPostChunk - 1) / kPostChunk);
  p.counts = counts;
  p.offsets = offsets;
  p.ids = ids;
  p.ids_sub_stride = ids_sub_stride;
  p.max_bucket = max_bucket;
  p.chunk_hist = static_cast<int32_t*>(workspace);
  dim3 grid(p.nchunks, n_heads * subspaces);
  post_hist_kernel<<<grid, kPostThreads, 0, st>>>(p);
  profile_mark(0, st);
  post_scan_kernel<<<n_heads * subspaces, kPostThreads, 0, st>>>(p);
  profile_mark(1, st);
  post_scatter_kernel<<<grid, kPostThreads, 0, st>>>(p);
  profile_mark(2, st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

// ---- incremental append ------------------------------------------------------------------
// Keys [start, start + count) are appended to the lists of their codes, in key order, so every
// list stays ascending: one thread per (head, subspace) walks the new keys.  Each cell c owns the
// id slots [offsets[c], offsets[c + 1]) (a padded layout); a key that would pass its cell's end is
// not written and *overflow is set, so a caller sizes the cells from a bound on the counts.
__global__ void post_append_kernel(const uint8_t* __restrict__ codes, int64_t codes_head_stride, int H, int S, int C,
                                   int64_t start, int64_t count, int32_t* __restrict__ counts,
                                   const int32_t* __restrict__ offsets, int32_t* __restrict__ ids,
                                   int64_t ids_sub_stride, int32_t* __restrict__ max_bucket,
                                   int32_t* __restrict__ overflow) {
  const int hs = blockIdx.x * blockDim.x + threadIdx.x;
  if (hs >= H * S) return;
  const int h = hs / S, s = hs - h * S;
  const uint8_t* cb = codes + h * codes_head_stride + s;
  int32_t* cnt = counts + (size_t)hs * C;
  const int32_t* off = offsets + (size_t)hs * (C + 1);
  int32_t* id = ids + (size_t)hs * ids_sub_stride;
  int biggest = 0;
  for (int64_t l = start; l < start + count; ++l) {
    const int c = __ldg(cb + l * S);
    if (c >= C) continue;
    const int pos = cnt[c];
    if (off[c] + pos >= off[c + 1]) {
      atomicExch(overflow, 1);
      continue;
    }
    id[off[c] + pos] = static_cast<int32_t>(l);
    cnt[c] = pos + 1;
    biggest = max(biggest, pos + 1);
  }
  if (biggest > 0) atomicMax(max_bucket, biggest);
}

// ---- no-alloc variant ---------------------------------------------------------------------
// The chunk histograms come from a fixed buffer inside the library (one per device, created
// with the module) instead of a caller-provided workspace.  Nothing in it has to start at zero:
// the histogram pass writes every entry the later passes read, and the call zeroes *max_bucket.

static __device__ __align__(256) unsigned char g_postings_scratch[SVA_POSTINGS_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kTrackedDevices = 64;
std::mutex g_postings_scratch_mu;
// Per device ordinal: the buffer's device address and the id of the context it was looked up
// in.  A device address is only valid in its own context, so the address is looked up again
// when the calling thread's current context is another one (after cudaDeviceReset, or under a
// context the caller created with the driver API).
struct ScratchAddr {
  unsigned long long ctx_id;
  void* addr;
};
ScratchAddr g_postings_scratch_addr[kTrackedDevices] = {};

using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

// Unique id of the calling thread's current CUDA context (0 if it cannot be read).  The driver
// entry points come through the runtime, so the library needs no link to the driver library.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
    cudaGetLastError();
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
  return 0;
}
}  // namespace

extern "C" int sva_postings_build_noalloc(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads,
                                          int32_t subspaces, int32_t codewords, int64_t key_len, int32_t* counts,
                                          int32_t* offsets, int32_t* ids, int64_t ids_sub_stride, int32_t* max_bucket,
                                          void* stream) {
  const size_t need = sva_postings_workspace_size(n_heads, subspaces, codewords, key_len);
  if (need > static_cast<size_t>(SVA_POSTINGS_NOALLOC_SCRATCH_BYTES))
    return set_error(SVA_ERR_WORKSPACE, "postings need more than the static scratch of sva_postings_build_noalloc");
  void* scratch = nullptr;
  if (need > 0) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kTrackedDevices) return set_error(SVA_ERR_CUDA, "device ordinal out of range");
    // 0 before the runtime has made a context current: the address is then looked up on every
    // call until one is (the lookup itself initialises the context and loads the module)
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_postings_scratch_mu);
    ScratchAddr& slot = g_postings_scratch_addr[dev];
    if (!slot.addr || ctx == 0 || slot.ctx_id != ctx) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_postings_scratch);  // resolved in the current context
      if (e != cudaSuccess || addr == nullptr)
        return set_error(SVA_ERR_CUDA, e != cudaSuccess ? cudaGetErrorString(e) : "null scratch address");
      slot.addr = addr;
      slot.ctx_id = ctx;
    }
    scratch = slot.addr;
  }
  return sva_postings_build(codes, codes_head_stride, n_heads, subspaces, codewords, key_len, counts, offsets, ids,
                            ids_sub_stride, max_bucket, scratch, need, stream);
}

extern "C" int sva_postings_append(const uint8_t* codes, int64_t codes_head_stride, int32_t n_heads, int32_t subspaces,
                                   int32_t codewords, int64_t start, int64_t count, int32_t* counts,
                                   const int32_t* offsets, int32_t* ids, int64_t ids_sub_stride, int32_t* max_bucket,
                                   int32_t* overflow, void* stream) {
  if (n_heads <= 0 || subspaces <= 0 || subspaces > kMaxSubspaces || codewords <= 0 || codewords > kMaxCodewords)
    return set_error(SVA_ERR_SHAPE, "bad postings shape");
  if (start < 0 || count < 0 || start + count > 0x7FFFFFFFll) return set_error(SVA_ERR_SHAPE, "key range out of range");
  if (!codes || !counts || !offsets || !ids || !max_bucket || !overflow) return set_error(SVA_ERR_SHAPE, "null pointer");
  if (count == 0) return SVA_OK;
  const int hs = n_heads * subspaces;
  post_append_kernel<<<(hs + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      codes, codes_head_stride, n_heads, subspaces, codewords, start, count, counts, offsets, ids, ids_sub_stride,
      max_bucket, overflow);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}
