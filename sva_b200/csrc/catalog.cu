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
  const int D = p.D, R = p.R, S = p.S, C = p.C, sub = p.sub;
  const int64_t l0 = p.start + (int64_t)blockIdx.x * kCatKeys;
  const int64_t l_end = p.start + p.count;
  const int nrows = (l_end - l0 < kCatKeys) ? (int)(l_end - l0) : kCatKeys;

  const float* Pg = p.k_proj + (size_t)h * D * R;
  for (int e = tid; e < D * R; e += blockDim.x) P[e] = __ldg(Pg + e);
  if (p.codes) {
    const float* cb = p.codebooks + (size_t)h * S * C * sub;  // [S][C][sub]
    for (int e = tid; e < S * C * sub; e += blockDim.x) {
      const int s = e / (C * sub);
      const int rem = e - s * C * sub;
      const int c = rem / sub, j = rem - c * sub;
      cbt[(s * sub + j) * C + c] = __ldg(cb + e);
    }
  }
  const T* kb = reinterpret_cast<const T*>(p.keys) + kvh * p.key_head_stride;
  for (int e = tid; e < nrows * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    xs[r * (D + 1) + d] = to_f32<T>(kb[(l0 + r) * p.key_row_stride + d]);
  }
  __syncthreads();
  if (p.codes) {
    for (int e = tid; e < S * C; e += blockDim.x) {
      const int s = e / C, c = e - s * C;
      float a = 0.f;
      for (int j = 0; j < sub; ++j) {
        const float v = cbt[(s * sub + j) * C + c];
        a = mac(a, v, v);
      }
      cn[e] = a;
    }
  }
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
    if (p.codes) {
      uint8_t* crow = p.codes + h * p.codes_head_stride + (l0 + tid) * S;
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
  }
  __syncthreads();
  if (p.k_low) {
    float* ob = p.k_low + h * p.k_low_head_stride + l0 * R;
    for (int e = tid; e < nrows * R; e += blockDim.x) {
      const int r = e / R, c = e - r * R;
      ob[e] = kl[r * (R + 1) + c];
    }
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

}  // namespace sva

using namespace sva;

extern "C" int sva_catalog_encode(const void* keys, int32_t key_dtype, int64_t key_head_stride,
                                  int64_t key_row_stride, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                  int32_t rank_dim, const float* k_proj, const float* codebooks, int32_t subspaces,
                                  int32_t codewords, int64_t start, int64_t count, float* k_low,
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
  p.k_low = k_low;
  p.k_low_head_stride = k_low_head_stride;
  p.codes = codes;
  p.codes_head_stride = codes_head_stride;
  catalog_layout(p);
  const size_t smem = sizeof(float) * p.total_floats;
  if (smem > (size_t)kMaxDynSmem) return set_error(SVA_ERR_SHAPE, "catalog tile exceeds shared memory");
  dim3 grid((unsigned)((count + kCatKeys - 1) / kCatKeys), (unsigned)n_heads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
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
