// Key catalog write path and the ops-level PQ kernels.
//
//   sva_catalog_encode   : k_low = K . Kproj[h] (fp32), codes = nearest codeword per subspace
//                          (replaces sva/llama.py:598,615 and sva/ops.py:10-47)
//   sva_assign_centroids : nearest centroid of arbitrary rows (sva/ops.py:10-21)
//   sva_pq_scores        : ADC scores for every key (sva/ops.py:50-71)
//
// This is the exact CUDA-core path: every dot product is the canonical sequential fp32 order
// (see sva_common.cuh), so codes and k_low are bit-identical to the CPU oracle.  Distances use
// the reference's expansion and evaluation order: (|x|^2 - 2 x.c) + |c|^2, lowest index on
// ties (torch.argmin).
#include "sva_common.cuh"
#include "sva_internal.h"

namespace sva {

constexpr int kCatKeys = 128;  // keys per CTA, one per thread

struct CatalogParams {
  const void* keys;
  int64_t key_head_stride, key_row_stride;
  int n_heads, groups, D, R, S, C, sub;
  const float* k_proj;
  const float* codebooks;
  int64_t start, count;
  const int64_t* start_dev;  // when set, rows start at *start_dev + start (read on the device) ...
  int64_t limit;             // ... and rows >= limit are skipped
  float* k_low;
  int64_t k_low_head_stride;
  uint8_t* codes;
  int64_t codes_head_stride;
  // shared-memory offsets (floats)
  int o_p, o_cbt, o_cn, o_x, o_kl, total_floats;
};

static void catalog_layout(CatalogParams& p) {
  int o = 0;
  p.o_p = o;   o += p.D * p.R;
  p.o_cbt = o; o += p.C * p.R;
  p.o_cn = o;  o += p.S * p.C;
  p.o_x = o;   o += kCatKeys * (p.D + 1);
  p.o_kl = o;  o += kCatKeys * (p.R + 1);
  p.total_floats = o;
}

// Codebook of head h into shared memory transposed to [S][sub][C]; block-cooperative.
__device__ void stage_codebooks(const CatalogParams& p, int h, float* cbt) {
  const int S = p.S, C = p.C, sub = p.sub;
  const float* cb = p.codebooks + (size_t)h * S * C * sub;  // [S][C][sub]
  // consecutive threads take consecutive codewords, so the transposed shared-memory writes
  // fall in consecutive banks
  for (int e = threadIdx.x; e < S * C * sub; e += blockDim.x) {
    const int c = e % C;
    const int sj = e / C;  // s * sub + j
    const int s = sj / sub, j = sj - s * sub;
    cbt[sj * C + c] = __ldg(cb + ((size_t)s * C + c) * sub + j);
  }
}

// |c|^2 of every codeword (sequential order); block-cooperative, reads the staged codebook.
__device__ void codeword_norms(const CatalogParams& p, const float* cbt, float* cn) {
  const int C = p.C, sub = p.sub;
  for (int e = threadIdx.x; e < p.S * C; e += blockDim.x) {
    const int s = e / C, c = e - s * C;
    float a = 0.f;
    for (int j = 0; j < sub; ++j) {
      const float v = cbt[(s * sub + j) * C + c];
      a = mac(a, v, v);
    }
    cn[e] = a;
  }
}

// Codes of one low-rank key y [R]: per subspace the codeword minimising (|x|^2 - 2 x.c) + |c|^2,
// lowest index on ties (torch.argmin), dot products in sequential order.
__device__ void assign_row(const CatalogParams& p, const float* cbt, const float* cn, const float* y, uint8_t* crow) {
  const int S = p.S, C = p.C, sub = p.sub;
  for (int s = 0; s < S; ++s) {
    const float* xsb = y + s * sub;
    float xn = 0.f;
    for (int j = 0; j < sub; ++j) xn = mac(xn, xsb[j], xsb[j]);
    int best = 0;
    float bestd = 0.f;
    int c = 0;
    for (; c + 4 <= C; c += 4) {
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
      for (int j = 0; j < sub; ++j) {
        const float xv = xsb[j];
        const float* row = cbt + (s * sub + j) * C + c;
        d0 = mac(d0, xv, row[0]);
        d1 = mac(d1, xv, row[1]);
        d2 = mac(d2, xv, row[2]);
        d3 = mac(d3, xv, row[3]);
      }
      const float dd[4] = {d0, d1, d2, d3};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float dist = __fadd_rn(__fsub_rn(xn, __fmul_rn(2.f, dd[q])), cn[s * C + c + q]);
        if ((c + q) == 0 || dist < bestd) {
          bestd = dist;
          best = c + q;
        }
      }
    }
    for (; c < C; ++c) {
      float dv = 0.f;
      for (int j = 0; j < sub; ++j) dv = mac(dv, xsb[j], cbt[(s * sub + j) * C + c]);
      const float dist = __fadd_rn(__fsub_rn(xn, __fmul_rn(2.f, dv)), cn[s * C + c]);
      if (c == 0 || dist < bestd) {
        bestd = dist;
        best = c;
      }
    }
    crow[s] = static_cast<uint8_t>(best);
  }
}

// Rows [0, nrows) of kl ([128][R+1] floats) -> k_low rows l0.. of head h; block-cooperative.
__device__ void store_k_low(const CatalogParams& p, int h, int64_t l0, int nrows, const float* kl) {
  const int R = p.R;
  float* ob = p.k_low + h * p.k_low_head_stride + l0 * R;
  for (int e = threadIdx.x; e < nrows * R; e += blockDim.x) {
    const int r = e / R, c = e - r * R;
    ob[e] = kl[r * (R + 1) + c];
  }
}

template <typename T>
__global__ void __launch_bounds__(kCatKeys) catalog_encode_kernel(const CatalogParams p) {
  extern __shared__ __align__(16) float sm[];
  float* P = sm + p.o_p;      // [D][R]
  float* cbt = sm + p.o_cbt;  // [S][sub][C]  (transposed codebook)
  float* cn = sm + p.o_cn;    // [S][C]
  float* xs = sm + p.o_x;     // [128][D+1]
  float* kl = sm + p.o_kl;    // [128][R+1]
  const int h = blockIdx.y;
  const int kvh = h / p.groups;
  const int tid = threadIdx.x;
  const int D = p.D, R = p.R;
  const int64_t start = p.start_dev ? __ldg(p.start_dev) + p.start : p.start;
  const int64_t l0 = start + (int64_t)blockIdx.x * kCatKeys;
  const int64_t l_end = min(start + p.count, p.limit);
  if (l0 < 0 || l0 >= l_end) return;  // uniform over the block
  const int nrows = (l_end - l0 < kCatKeys) ? (int)(l_end - l0) : kCatKeys;

  const float* Pg = p.k_proj + (size_t)h * D * R;
  for (int e = tid; e < D * R; e += blockDim.x) P[e] = __ldg(Pg + e);
  if (p.codes) stage_codebooks(p, h, cbt);
  const T* kb = reinterpret_cast<const T*>(p.keys) + kvh * p.key_head_stride;
  for (int e = tid; e < nrows * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    xs[r * (D + 1) + d] = to_f32<T>(kb[(l0 + r) * p.key_row_stride + d]);
  }
  __syncthreads();
  if (p.codes) codeword_norms(p, cbt, cn);
  __syncthreads();

  if (tid < nrows) {
    const float* x = xs + tid * (D + 1);
    float* y = kl + tid * (R + 1);
    for (int r = 0; r < R; r += 4) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int d = 0; d < D; ++d) {
        const float xv = x[d];
        const float4 pv = *reinterpret_cast<const float4*>(P + d * R + r);
        a0 = mac(a0, xv, pv.x);
        a1 = mac(a1, xv, pv.y);
        a2 = mac(a2, xv, pv.z);
        a3 = mac(a3, xv, pv.w);
      }
      y[r] = a0;
      y[r + 1] = a1;
      y[r + 2] = a2;
      y[r + 3] = a3;
    }
    if (p.codes) assign_row(p, cbt, cn, y, p.codes + h * p.codes_head_stride + (l0 + tid) * p.S);
  }
  __syncthreads();
  if (p.k_low) store_k_low(p, h, l0, nrows, kl);
}

// Bulk path for head_dim = rank_dim = 64 and subspaces of SUB = 8, 16 or 32 values: the same
// canonical arithmetic as catalog_encode_kernel (every projection output and every distance is
// one thread's sequential fp32 dot product, the nearest codeword the first minimum in codeword
// order), organised for occupancy: a thread holds its key row in registers and produces one
// subspace at a time (SUB projection outputs, then that subspace's code), so shared memory holds
// only the projection and the codebook (~33 KB) and several CTAs share each SM.  A CTA stages the
// head's tables once and walks key tiles of kRegKeys keys.
constexpr int kRegKeys = 128;
constexpr int kRegCtasPerSm = 4;

template <typename T, int SUB>
__global__ void __launch_bounds__(kRegKeys, kRegCtasPerSm) catalog_encode_reg_kernel(const CatalogParams p,
                                                                                   int vec_keys, int vec_out) {
  constexpr int D = 64, R = 64, S = R / SUB;
  extern __shared__ __align__(16) float sm[];
  float* P = sm;                  // [D][R]
  float* cbt = sm + D * R;        // [S][SUB][C]  (transposed codebook)
  float* cn = cbt + R * p.C;      // [S][C]
  const int h = blockIdx.y;
  const int kvh = h / p.groups;
  const int tid = threadIdx.x;
  const int C = p.C;
  const int64_t start = p.start_dev ? __ldg(p.start_dev) + p.start : p.start;
  const int64_t l_end = min(start + p.count, p.limit);
  if (start < 0 || start >= l_end) return;  // uniform over the grid
  const int64_t n_tiles = (l_end - start + kRegKeys - 1) / kRegKeys;
  if (blockIdx.x >= n_tiles) return;
  const float* Pg = p.k_proj + (size_t)h * D * R;
  for (int e = tid; e < D * R / 4; e += blockDim.x)
    reinterpret_cast<float4*>(P)[e] = __ldg(reinterpret_cast<const float4*>(Pg) + e);
  if (p.codes) stage_codebooks(p, h, cbt);
  __syncthreads();
  if (p.codes) codeword_norms(p, cbt, cn);
  __syncthreads();
  const T* kb = reinterpret_cast<const T*>(p.keys) + kvh * p.key_head_stride;
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int64_t l = start + tile * kRegKeys + tid;
    if (l >= l_end) continue;
    const T* kr = kb + l * p.key_row_stride;
    float x[D];
    if (vec_keys) {
      constexpr int kPer = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte load
#pragma unroll
      for (int v = 0; v < D / kPer; ++v) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(kr) + v);
        const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int k = 0; k < kPer; ++k) x[v * kPer + k] = to_f32<T>(e[k]);
      }
    } else {
#pragma unroll
      for (int d = 0; d < D; ++d) x[d] = to_f32<T>(kr[d]);
    }
    float* kout = p.k_low ? p.k_low + h * p.k_low_head_stride + l * R : nullptr;
    uint8_t* crow = p.codes ? p.codes + h * p.codes_head_stride + l * S : nullptr;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      float y[SUB];
#pragma unroll
      for (int j = 0; j < SUB; ++j) y[j] = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const float xv = x[d];
        const float4* prow = reinterpret_cast<const float4*>(P + d * R + s * SUB);
#pragma unroll
        for (int j = 0; j < SUB / 4; ++j) {
          const float4 pv = prow[j];
          y[4 * j] = mac(y[4 * j], xv, pv.x);
          y[4 * j + 1] = mac(y[4 * j + 1], xv, pv.y);
          y[4 * j + 2] = mac(y[4 * j + 2], xv, pv.z);
          y[4 * j + 3] = mac(y[4 * j + 3], xv, pv.w);
        }
      }
      if (kout) {
        if (vec_out) {
#pragma unroll
          for (int j = 0; j < SUB / 4; ++j)
            reinterpret_cast<float4*>(kout + s * SUB)[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < SUB; ++j) kout[s * SUB + j] = y[j];
        }
      }
      if (crow) {
        float xn = 0.f;
#pragma unroll
        for (int j = 0; j < SUB; ++j) xn = mac(xn, y[j], y[j]);
        int best = 0;
        float bestd = 0.f;
        for (int c = 0; c < C; c += 4) {  // C is a multiple of 4
          float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
          for (int j = 0; j < SUB; ++j) {
            const float4 cw = *reinterpret_cast<const float4*>(cbt + (s * SUB + j) * C + c);
            d0 = mac(d0, y[j], cw.x);
            d1 = mac(d1, y[j], cw.y);
            d2 = mac(d2, y[j], cw.z);
            d3 = mac(d3, y[j], cw.w);
          }
          const float dd[4] = {d0, d1, d2, d3};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float dist = __fadd_rn(__fsub_rn(xn, __fmul_rn(2.f, dd[q])), cn[s * C + c + q]);
            if ((c + q) == 0 || dist < bestd) {
              bestd = dist;
              best = c + q;
            }
          }
        }
        crow[s] = static_cast<uint8_t>(best);
      }
    }
  }
}

// Append path for a few keys (decode steps): one CTA per (key, head), so a one-key append is
// spread over the threads of many CTAs instead of one thread of a 128-key tile.  Same canonical
// arithmetic as catalog_encode_kernel: every projection output and every distance is one thread's
// sequential fp32 dot product; the nearest codeword is the first minimum in codeword order.
constexpr int kAppendThreads = 128;
constexpr int kAppendMaxKeys = 8;  // appends of at most this many keys take this kernel

template <typename T>
__global__ void __launch_bounds__(kAppendThreads) catalog_append_kernel(const CatalogParams p) {
  __shared__ float x[kMaxHeadDim];
  __shared__ float y[kMaxRank];
  __shared__ float bd[kAppendThreads / 32][kMaxSubspaces];
  __shared__ int bc[kAppendThreads / 32][kMaxSubspaces];
  const int h = blockIdx.y;
  const int kvh = h / p.groups;
  const int tid = threadIdx.x;
  const int D = p.D, R = p.R, S = p.S, C = p.C, sub = p.sub;
  const int64_t start = p.start_dev ? __ldg(p.start_dev) + p.start : p.start;
  const int64_t l = start + blockIdx.x;
  if (l < 0 || l >= min(start + p.count, p.limit)) return;  // uniform over the block
  const T* kr = reinterpret_cast<const T*>(p.keys) + kvh * p.key_head_stride + l * p.key_row_stride;
  for (int d = tid; d < D; d += blockDim.x) x[d] = to_f32<T>(kr[d]);
  __syncthreads();
  const float* Pg = p.k_proj + (size_t)h * D * R;
  for (int r = tid; r < R; r += blockDim.x) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = mac(a, x[d], __ldg(Pg + d * R + r));
    y[r] = a;
  }
  __syncthreads();
  if (p.k_low)
    for (int r = tid; r < R; r += blockDim.x) p.k_low[h * p.k_low_head_stride + l * R + r] = y[r];
  if (!p.codes) return;
  const int lane = tid & 31, warp = tid >> 5;
  for (int sp = 0; sp < S; ++sp) {
    const float* xs = y + sp * sub;
    float xn = 0.f;
    for (int j = 0; j < sub; ++j) xn = mac(xn, xs[j], xs[j]);
    // this thread's best codeword of the subspace: first minimum, NaN distances never win
    float best = INFINITY;
    int bi = C;
    bool nan0 = false;
    for (int c = tid; c < C; c += blockDim.x) {
      const float* cw = p.codebooks + (((size_t)h * S + sp) * C + c) * sub;
      float dv = 0.f, cn = 0.f;
      for (int j = 0; j < sub; ++j) {
        const float v = __ldg(cw + j);
        dv = mac(dv, xs[j], v);
        cn = mac(cn, v, v);
      }
      const float dist = __fadd_rn(__fsub_rn(xn, __fmul_rn(2.f, dv)), cn);
      if (c == 0 && isnan(dist)) nan0 = true;
      if (dist < best) {
        best = dist;
        bi = c;
      }
    }
    // the sequential rule keeps codeword 0 when its distance is NaN
    nan0 = __any_sync(0xFFFFFFFFu, nan0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ob < best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      bd[warp][sp] = best;
      bc[warp][sp] = nan0 ? -1 : bi;
    }
  }
  __syncthreads();
  if (tid < S) {
    float best = INFINITY;
    int bi = C;
    bool nan0 = false;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      if (bc[w][tid] < 0) nan0 = true;
      if (bd[w][tid] < best || (bd[w][tid] == best && bc[w][tid] < bi)) {
        best = bd[w][tid];
        bi = bc[w][tid];
      }
    }
    // every distance NaN or infinite: the sequential scan keeps codeword 0
    if (nan0 || bi >= C || bi < 0) bi = 0;
    p.codes[h * p.codes_head_stride + l * S + tid] = static_cast<uint8_t>(bi);
  }
}

__global__ void __launch_bounds__(256) assign_centroids_kernel(const float* __restrict__ x, int64_t n, int dim,
                                                               int64_t stride, const float* __restrict__ cent, int C,
                                                               int64_t* __restrict__ labels) {
  extern __shared__ float sm[];
  float* cs = sm;             // [C][dim]
  float* cn = sm + C * dim;   // [C]
  for (int e = threadIdx.x; e < C * dim; e += blockDim.x) cs[e] = cent[e];
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float a = 0.f;
    for (int j = 0; j < dim; ++j) a = mac(a, cs[c * dim + j], cs[c * dim + j]);
    cn[c] = a;
  }
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* xr = x + i * stride;
  float xv[kMaxRank];
  float xn = 0.f;
  for (int j = 0; j < dim; ++j) {
    xv[j] = xr[j];
    xn = mac(xn, xv[j], xv[j]);
  }
  int best = 0;
  float bestd = 0.f;
  for (int c = 0; c < C; ++c) {
    float dv = 0.f;
    for (int j = 0; j < dim; ++j) dv = mac(dv, xv[j], cs[c * dim + j]);
    const float dist = __fadd_rn(__fsub_rn(xn, __fmul_rn(2.f, dv)), cn[c]);
    if (c == 0 || dist < bestd) {
      bestd = dist;
      best = c;
    }
  }
  labels[i] = best;
}

__global__ void __launch_bounds__(256) pq_scores_kernel(const float* __restrict__ q_low, int T, int R,
                                                        const float* __restrict__ codebooks, int S, int C,
                                                        const uint8_t* __restrict__ codes, int64_t L,
                                                        float* __restrict__ scores, float sqrt_r, int sqrt_r_pow2) {
  __shared__ float lut[kMaxLut];
  const int prob = blockIdx.y;
  const int h = prob / T;
  const int sub = R / S;
  const float* ql = q_low + (size_t)prob * R;
  for (int e = threadIdx.x; e < S * C; e += blockDim.x) {
    const int s = e / C, c = e - s * C;
    const float* cb = codebooks + (((size_t)h * S + s) * C + c) * sub;
    float a = 0.f;
    for (int j = 0; j < sub; ++j) a = mac(a, ql[s * sub + j], cb[j]);
    lut[e] = a;
  }
  __syncthreads();
  const uint8_t* cr = codes + (size_t)h * L * S;
  const float inv = 1.0f / sqrt_r;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < L; i += (int64_t)gridDim.x * blockDim.x) {
    float sum = 0.f;
    for (int s = 0; s < S; ++s) sum = __fadd_rn(sum, lut[s * C + cr[i * S + s]]);
    scores[(size_t)prob * L + i] = sqrt_r_pow2 ? __fmul_rn(sum, inv) : __fdiv_rn(sum, sqrt_r);
  }
}

// ---- tensor-core write path ------------------------------------------------------------
// k_low = K . Kproj[h] on the 5th-generation tensor cores: one CTA per 128 keys of a head is
// one UMMA tile (M = 128 keys, N = R, K = D) with bf16 operands and an fp32 accumulator in
// tensor memory.  K is bf16 and Kproj is rounded to bf16 (exact for bf16 artifacts), so every
// product is exact and only the fp32 accumulation order differs from the exact path.  Each
// thread then reads its key's row from tensor memory and runs the same nearest-codeword
// assignment as the exact path.
//
// Shared-memory operand layout (K-major, no swizzle): 8-row x 16-byte core matrices; a K chunk
// of 8 elements holds all rows contiguously (row r at byte 16 r), chunks are LBO = 16 * rows
// bytes apart, 8-row groups SBO = 128 bytes apart.  One MMA consumes two chunks (K = 16).
constexpr int kTcKeys = 128;         // UMMA M
constexpr int kTcTmemCols = 64;      // fp32 accumulator columns (R <= 64)
constexpr int kTcWaitSpins = 1 << 20;

struct TcLayout {
  int a, b, cbt, cn, kl, total;
};

static TcLayout tc_layout(const CatalogParams& p) {
  auto up = [](int x, int a) { return (x + a - 1) / a * a; };
  TcLayout L;
  int o = 0;
  L.a = o;   o = up(o + 16 * kTcKeys * (p.D / 8), 1024);
  L.b = o;   o = up(o + 16 * p.R * (p.D / 8), 1024);
  L.cbt = o; o = up(o + 4 * p.C * p.R, 16);
  L.cn = o;  o = up(o + 4 * p.S * p.C, 16);
  L.kl = o;  o = up(o + 4 * kTcKeys * (p.R + 1), 16);
  // at least 1/8 of an SM's shared memory, so that at most 8 CTAs (8 x 64 of the 512
  // tensor-memory columns) share an SM and an allocation never waits
  L.total = o > 29 * 1024 ? o : 29 * 1024;
  return L;
}

__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// Shared-memory matrix descriptor: start, leading and stride byte offsets (>> 4), version 1,
// no swizzle.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((start >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Bounded wait for phase `parity` of an mbarrier; returns false when the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t mbar, uint32_t parity) {
  for (int it = 0; it < kTcWaitSpins; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__global__ void __launch_bounds__(kTcKeys) catalog_encode_tc_kernel(const CatalogParams p, const TcLayout L,
                                                                    int* status) {
  extern __shared__ __align__(1024) unsigned char smc[];
  __shared__ __align__(8) unsigned long long mbar;
  __shared__ uint32_t tmem_base;
  unsigned char* a_tile = smc + L.a;
  unsigned char* b_tile = smc + L.b;
  float* cbt = reinterpret_cast<float*>(smc + L.cbt);
  float* cn = reinterpret_cast<float*>(smc + L.cn);
  float* kl = reinterpret_cast<float*>(smc + L.kl);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y;
  const int kvh = h / p.groups;
  const int D = p.D, R = p.R;
  const int64_t l0 = p.start + (int64_t)blockIdx.x * kTcKeys;
  const int64_t l_end = p.start + p.count;
  const int nrows = (l_end - l0 < kTcKeys) ? (int)(l_end - l0) : kTcKeys;
  const uint32_t mb = smem_addr(&mbar);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mb), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // A: key row r = tid, one 16-byte chunk of 8 elements at a time
  {
    const __nv_bfloat16* row =
        reinterpret_cast<const __nv_bfloat16*>(p.keys) + kvh * p.key_head_stride + (l0 + tid) * p.key_row_stride;
    for (int c = 0; c < D / 8; ++c) {
      const uint4 v = tid < nrows ? __ldg(reinterpret_cast<const uint4*>(row + 8 * c)) : make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(a_tile + c * (16 * kTcKeys) + tid * 16) = v;
    }
  }
  // B: row n = output column, K chunk c holds Kproj[8c .. 8c+7][n] rounded to bf16
  {
    const float* P = p.k_proj + (size_t)h * D * R;
    for (int q = tid; q < R * (D / 8); q += blockDim.x) {
      const int n = q % R, c = q / R;
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat16 lo = __float2bfloat16_rn(__ldg(P + (8 * c + 2 * j) * R + n));
        const __nv_bfloat16 hi = __float2bfloat16_rn(__ldg(P + (8 * c + 2 * j + 1) * R + n));
        w[j] = static_cast<uint32_t>(__bfloat16_as_ushort(lo)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
      }
      *reinterpret_cast<uint4*>(b_tile + c * (16 * R) + n * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (p.codes) stage_codebooks(p, h, cbt);
  // operands written by the generic proxy, read by the tensor cores (async proxy)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  if (tid == 0) {
    // kind::f16, D fp32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both K-major,
    // N >> 3 at bit 17, M >> 4 at bit 24
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(R >> 3) << 17) |
                           (static_cast<uint32_t>(kTcKeys >> 4) << 24);
    const uint32_t a0 = smem_addr(a_tile), b0 = smem_addr(b_tile);
    for (int kb = 0; kb < D / 16; ++kb) {
      const uint64_t ad = umma_smem_desc(a0 + kb * 2 * (16 * kTcKeys), 16 * kTcKeys, 128);
      const uint64_t bd = umma_smem_desc(b0 + kb * 2 * (16 * R), 16 * R, 128);
      const uint32_t accumulate = kb > 0 ? 1u : 0u;
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "setp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
          "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate)
          : "memory");
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mb)
                 : "memory");
  }
  if (p.codes) codeword_norms(p, cbt, cn);
  bool ok = mbar_wait_bounded(mb, 0);
  if (!ok) {
    if (status) atomicExch(status, SVA_ERR_TIMEOUT);
    ok = mbar_wait_bounded(mb, 0);  // the MMA must finish before its tensor memory is released
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok) {
    // warp w reads tensor-memory lanes 32w .. 32w+31 = its threads' keys, 16 columns at a time
    float* y = kl + tid * (R + 1);
    for (int c0 = 0; c0 < R; c0 += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(c0))
          : "memory");
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 16; ++j) y[c0 + j] = __uint_as_float(v[j]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (ok) {
    if (p.codes && tid < nrows)
      assign_row(p, cbt, cn, kl + tid * (R + 1), p.codes + h * p.codes_head_stride + (l0 + tid) * p.S);
    if (p.k_low) store_k_low(p, h, l0, nrows, kl);
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
  }
}

}  // namespace sva

using namespace sva;

static int catalog_encode_impl(const void* keys, int32_t key_dtype, int64_t key_head_stride, int64_t key_row_stride,
                               int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t rank_dim,
                               const float* k_proj, const float* codebooks, int32_t subspaces, int32_t codewords,
                               int64_t start, const int64_t* start_dev, int64_t count, int64_t limit, float* k_low,
                               int64_t k_low_head_stride, uint8_t* codes, int64_t codes_head_stride, void* stream) {
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return set_error(SVA_ERR_SHAPE, "bad head counts");
  if (head_dim <= 0 || head_dim > kMaxHeadDim) return set_error(SVA_ERR_SHAPE, "head_dim must be in 1..256");
  if (rank_dim <= 0 || rank_dim > kMaxRank || rank_dim % 4) return set_error(SVA_ERR_SHAPE, "rank_dim must be a multiple of 4 <= 64");
  if (subspaces <= 0 || rank_dim % subspaces || subspaces > kMaxSubspaces) return set_error(SVA_ERR_SHAPE, "bad subspaces");
  if (codewords <= 0 || codewords > kMaxCodewords) return set_error(SVA_ERR_SHAPE, "codewords must be in 1..256");
  if (start < 0 || count < 0) return set_error(SVA_ERR_SHAPE, "negative key range");
  if (key_dtype < 0 || key_dtype > 2) return set_error(SVA_ERR_DTYPE, "bad key dtype");
  if (!keys || !k_proj || (codes && !codebooks)) return set_error(SVA_ERR_SHAPE, "null pointer");
  if (count == 0) return SVA_OK;
  CatalogParams p;
  p.keys = keys;
  p.key_head_stride = key_head_stride;
  p.key_row_stride = key_row_stride;
  p.n_heads = n_heads;
  p.groups = n_heads / n_kv_heads;
  p.D = head_dim;
  p.R = rank_dim;
  p.S = subspaces;
  p.C = codewords;
  p.sub = rank_dim / subspaces;
  p.k_proj = k_proj;
  p.codebooks = codebooks;
  p.start = start;
  p.count = count;
  p.start_dev = start_dev;
  p.limit = limit;
  p.k_low = k_low;
  p.k_low_head_stride = k_low_head_stride;
  p.codes = codes;
  p.codes_head_stride = codes_head_stride;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (count <= kAppendMaxKeys) {
    dim3 agrid((unsigned)count, (unsigned)n_heads);
    switch (key_dtype) {
      case SVA_DTYPE_F32: catalog_append_kernel<float><<<agrid, kAppendThreads, 0, s>>>(p); break;
      case SVA_DTYPE_BF16: catalog_append_kernel<__nv_bfloat16><<<agrid, kAppendThreads, 0, s>>>(p); break;
      default: catalog_append_kernel<__half><<<agrid, kAppendThreads, 0, s>>>(p); break;
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  }
  if (head_dim == 64 && rank_dim == 64 && codewords % 4 == 0 &&
      (p.sub == 8 || p.sub == 16 || p.sub == 32) && reinterpret_cast<uintptr_t>(k_proj) % 16 == 0 &&
      (!codes || reinterpret_cast<uintptr_t>(codebooks) % 16 == 0)) {
    const int esz = key_dtype == SVA_DTYPE_F32 ? 4 : 2;
    const int vec_keys = (reinterpret_cast<uintptr_t>(keys) % 16 == 0 && (key_head_stride * esz) % 16 == 0 &&
                          (key_row_stride * esz) % 16 == 0)
                             ? 1
                             : 0;
    const int vec_out = (!k_low || (reinterpret_cast<uintptr_t>(k_low) % 16 == 0 && k_low_head_stride % 4 == 0)) ? 1 : 0;
    const size_t rsmem = sizeof(float) * (64 * 64 + (size_t)64 * codewords + (size_t)subspaces * codewords);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    // tiles of the whole range (a device start may shift it by at most the rows past `start`)
    const int64_t span = start_dev ? std::min<int64_t>(count, std::max<int64_t>(limit, 0)) : count;
    const int64_t n_tiles = (span + kRegKeys - 1) / kRegKeys;
    const int64_t want = std::max<int64_t>(1, (int64_t)sms * kRegCtasPerSm * 2 / n_heads);
    dim3 rgrid((unsigned)std::max<int64_t>(1, std::min<int64_t>(n_tiles, want)), (unsigned)n_heads);
    auto launch = [&](auto kernel) -> int {
      const int rc2 = ensure_smem_attr(reinterpret_cast<const void*>(kernel), static_cast<int>(rsmem));
      if (rc2) return rc2;
      kernel<<<rgrid, kRegKeys, rsmem, s>>>(p, vec_keys, vec_out);
      const cudaError_t e2 = cudaGetLastError();
      return e2 == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e2));
    };
    switch (key_dtype * 3 + (p.sub == 8 ? 0 : p.sub == 16 ? 1 : 2)) {
      case 0: return launch(catalog_encode_reg_kernel<float, 8>);
      case 1: return launch(catalog_encode_reg_kernel<float, 16>);
      case 2: return launch(catalog_encode_reg_kernel<float, 32>);
      case 3: return launch(catalog_encode_reg_kernel<__nv_bfloat16, 8>);
      case 4: return launch(catalog_encode_reg_kernel<__nv_bfloat16, 16>);
      case 5: return launch(catalog_encode_reg_kernel<__nv_bfloat16, 32>);
      case 6: return launch(catalog_encode_reg_kernel<__half, 8>);
      case 7: return launch(catalog_encode_reg_kernel<__half, 16>);
      default: return launch(catalog_encode_reg_kernel<__half, 32>);
    }
  }
  catalog_layout(p);
  const size_t smem = sizeof(float) * p.total_floats;
  if (smem > (size_t)kMaxDynSmem) return set_error(SVA_ERR_SHAPE, "catalog tile exceeds shared memory");
  dim3 grid((unsigned)((count + kCatKeys - 1) / kCatKeys), (unsigned)n_heads);
  int rc;
  switch (key_dtype) {
    case SVA_DTYPE_F32:
      rc = ensure_smem_attr(reinterpret_cast<const void*>(catalog_encode_kernel<float>), kMaxDynSmem);
      if (rc) return rc;
      catalog_encode_kernel<float><<<grid, kCatKeys, smem, s>>>(p);
      break;
    case SVA_DTYPE_BF16:
      rc = ensure_smem_attr(reinterpret_cast<const void*>(catalog_encode_kernel<__nv_bfloat16>), kMaxDynSmem);
      if (rc) return rc;
      catalog_encode_kernel<__nv_bfloat16><<<grid, kCatKeys, smem, s>>>(p);
      break;
    default:
      rc = ensure_smem_attr(reinterpret_cast<const void*>(catalog_encode_kernel<__half>), kMaxDynSmem);
      if (rc) return rc;
      catalog_encode_kernel<__half><<<grid, kCatKeys, smem, s>>>(p);
      break;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

extern "C" int sva_catalog_encode(const void* keys, int32_t key_dtype, int64_t key_head_stride,
                                  int64_t key_row_stride, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                  int32_t rank_dim, const float* k_proj, const float* codebooks, int32_t subspaces,
                                  int32_t codewords, int64_t start, int64_t count, float* k_low,
                                  int64_t k_low_head_stride, uint8_t* codes, int64_t codes_head_stride, void* stream) {
  return catalog_encode_impl(keys, key_dtype, key_head_stride, key_row_stride, n_heads, n_kv_heads, head_dim, rank_dim,
                             k_proj, codebooks, subspaces, codewords, start, nullptr, count, start + count, k_low,
                             k_low_head_stride, codes, codes_head_stride, stream);
}

extern "C" int sva_catalog_encode_at(const void* keys, int32_t key_dtype, int64_t key_head_stride,
                                     int64_t key_row_stride, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                     int32_t rank_dim, const float* k_proj, const float* codebooks, int32_t subspaces,
                                     int32_t codewords, const int64_t* start, int64_t count, int64_t limit,
                                     float* k_low, int64_t k_low_head_stride, uint8_t* codes, int64_t codes_head_stride,
                                     void* stream) {
  if (!start) return set_error(SVA_ERR_SHAPE, "start is null");
  if (limit < 0) return set_error(SVA_ERR_SHAPE, "negative limit");
  return catalog_encode_impl(keys, key_dtype, key_head_stride, key_row_stride, n_heads, n_kv_heads, head_dim, rank_dim,
                             k_proj, codebooks, subspaces, codewords, 0, start, count, limit, k_low, k_low_head_stride,
                             codes, codes_head_stride, stream);
}

extern "C" int sva_assign_centroids(const float* x, int64_t n, int32_t dim, int64_t x_row_stride,
                                    const float* centroids, int32_t codewords, int64_t* labels, void* stream) {
  if (dim <= 0 || dim > kMaxRank || codewords <= 0 || codewords > 4096) return set_error(SVA_ERR_SHAPE, "bad dims");
  if (n < 0) return set_error(SVA_ERR_SHAPE, "negative row count");
  if (n == 0) return SVA_OK;
  const size_t smem = sizeof(float) * ((size_t)codewords * dim + codewords);
  if (smem > (size_t)kMaxDynSmem) return set_error(SVA_ERR_SHAPE, "centroids exceed shared memory");
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(assign_centroids_kernel), kMaxDynSmem);
  if (rc) return rc;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  assign_centroids_kernel<<<blocks, 256, smem, static_cast<cudaStream_t>(stream)>>>(x, n, dim, x_row_stride, centroids,
                                                                                     codewords, labels);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

extern "C" int sva_pq_scores(const float* q_low, int32_t n_heads, int32_t n_queries, int32_t rank_dim,
                             const float* codebooks, int32_t subspaces, int32_t codewords, const uint8_t* codes,
                             int64_t key_len, float* scores, void* stream) {
  if (n_heads <= 0 || n_queries <= 0 || rank_dim <= 0 || rank_dim > kMaxRank || subspaces <= 0 ||
      rank_dim % subspaces || codewords <= 0 || codewords > kMaxCodewords || subspaces * codewords > kMaxLut)
    return set_error(SVA_ERR_SHAPE, "bad pq shape");
  if (key_len <= 0) return SVA_OK;
  const double sr = std::sqrt((double)rank_dim);
  int e2;
  const bool pow2 = std::frexp((double)(float)sr, &e2) == 0.5;
  const unsigned bx = (unsigned)std::min<int64_t>((key_len + 255) / 256, 1024);
  dim3 grid(bx, (unsigned)(n_heads * n_queries));
  pq_scores_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(q_low, n_queries, rank_dim, codebooks,
                                                                        subspaces, codewords, codes, key_len, scores,
                                                                        (float)sr, pow2 ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}

extern "C" int sva_catalog_encode_tc(const void* keys, int32_t key_dtype, int64_t key_head_stride, int64_t key_row_stride,
                                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t rank_dim,
                                     const float* k_proj, const float* codebooks, int32_t subspaces,
                                     int32_t codewords, int64_t start, int64_t count, float* k_low,
                                     int64_t k_low_head_stride, uint8_t* codes, int64_t codes_head_stride,
                                     int32_t* status, void* stream) {
  if (key_dtype != SVA_DTYPE_BF16) return set_error(SVA_ERR_DTYPE, "tensor-core write path: keys must be bf16");
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return set_error(SVA_ERR_SHAPE, "bad head counts");
  if (head_dim <= 0 || head_dim > 128 || head_dim % 16)
    return set_error(SVA_ERR_SHAPE, "tensor-core write path: head_dim must be a multiple of 16 <= 128");
  if (rank_dim <= 0 || rank_dim > kTcTmemCols || rank_dim % 16)
    return set_error(SVA_ERR_SHAPE, "tensor-core write path: rank_dim must be a multiple of 16 <= 64");
  if (subspaces <= 0 || rank_dim % subspaces || subspaces > kMaxSubspaces) return set_error(SVA_ERR_SHAPE, "bad subspaces");
  if (codewords <= 0 || codewords > kMaxCodewords) return set_error(SVA_ERR_SHAPE, "codewords must be in 1..256");
  if (start < 0 || count < 0) return set_error(SVA_ERR_SHAPE, "negative key range");
  if (!keys || !k_proj || (codes && !codebooks)) return set_error(SVA_ERR_SHAPE, "null pointer");
  if ((reinterpret_cast<uintptr_t>(keys) & 15) || ((key_row_stride * 2) & 15) || ((key_head_stride * 2) & 15))
    return set_error(SVA_ERR_ALIGN, "tensor-core write path: key rows must be 16-byte aligned");
  if (count == 0) return SVA_OK;
  CatalogParams p;
  memset(&p, 0, sizeof(p));
  p.keys = keys;
  p.key_head_stride = key_head_stride;
  p.key_row_stride = key_row_stride;
  p.n_heads = n_heads;
  p.groups = n_heads / n_kv_heads;
  p.D = head_dim;
  p.R = rank_dim;
  p.S = subspaces;
  p.C = codewords;
  p.sub = rank_dim / subspaces;
  p.k_proj = k_proj;
  p.codebooks = codebooks;
  p.start_dev = nullptr;
  p.limit = start + count;
  p.start = start;
  p.count = count;
  p.k_low = k_low;
  p.k_low_head_stride = k_low_head_stride;
  p.codes = codes;
  p.codes_head_stride = codes_head_stride;
  const TcLayout L = tc_layout(p);
  if (L.total > kMaxDynSmem - 64) return set_error(SVA_ERR_SHAPE, "catalog tile exceeds shared memory");
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(catalog_encode_tc_kernel), L.total);
  if (rc != SVA_OK) return rc;
  dim3 grid((unsigned)((count + kTcKeys - 1) / kTcKeys), (unsigned)n_heads);
  catalog_encode_tc_kernel<<<grid, kTcKeys, L.total, static_cast<cudaStream_t>(stream)>>>(p, L, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
  return SVA_OK;
}
