// Residual output adapter fused with the attention output projection (o_proj) for decode steps.
//
// The late-layer socket of the reference wraps a patched attention layer in a residual adapter
// (experiments/sva_late4_logit_distill.py:37-51):
//     o          = o_proj(attn)                                   (model dtype, torch linear)
//     correction = up(gelu(down(cat[float(hidden), float(o)]))) * scale    (fp32)
//     out        = o + correction.to(dtype)
// Eager, that is an o_proj GEMM and seven small elementwise / GEMV kernels per layer and step.
// Here it is one launch: a thread-block cluster of kAdCluster CTAs per block of up to kAdRows
// token rows.  Each CTA owns a slice of the output features and of the adapter rank, and the
// slices meet through distributed shared memory:
//   1. CTA c computes o for its features (every row of the block) and rounds it to the dtype;
//   2. every CTA gathers the full o rows from its peers, next to float(hidden);
//   3. CTA c computes its rank slice of down(.) and the exact-erf gelu;
//   4. every CTA gathers the full gelu vector; CTA c computes up(.) * scale for its features and
//      writes out = round(o + round(correction)).
// Weights are read once per cluster (o_proj as the model dtype, down / up as fp32); every dot
// product accumulates in fp32.
#include <cooperative_groups.h>

#include "sva_common.cuh"
#include "sva_internal.h"

namespace sva {

namespace cg = cooperative_groups;

constexpr int kAdCluster = 8;
constexpr int kAdRows = 16;
constexpr int kAdThreads = 256;
constexpr int kAdMaxHidden = 4096;
constexpr int kAdMaxRank = 512;

struct AdapterParams {
  const void* hidden;  // [N][hidden_dim]
  int64_t hidden_row_stride;
  const void* attn;  // [N][in_dim], the attention output before o_proj
  int64_t attn_row_stride;
  const void* o_weight;  // [hidden_dim][in_dim]
  const void* o_bias;    // [hidden_dim] or NULL
  const float* down;     // [rank][2 * hidden_dim]
  const float* up;       // [hidden_dim][rank]
  float scale;
  int n_rows, hidden_dim, in_dim, rank;
  void* out;  // [N][hidden_dim]
  int64_t out_row_stride;
};

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// Warp-cooperative fp32 dot product of n elements (lane-strided), result in every lane.
template <typename A, typename B>
__device__ __forceinline__ float warp_dot(const A* a, const B* b, int n) {
  float acc = 0.f;
  for (int k = threadIdx.x & 31; k < n; k += 32) acc = fmaf(to_f32<A>(a[k]), to_f32<B>(b[k]), acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  return acc;
}

template <typename T>
__global__ void __cluster_dims__(kAdCluster, 1, 1) __launch_bounds__(kAdThreads)
    adapter_fused_kernel(const AdapterParams p) {
  extern __shared__ __align__(16) float ad_smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int row0 = (blockIdx.x / kAdCluster) * kAdRows;
  const int nrows = min(kAdRows, p.n_rows - row0);
  const int Hd = p.hidden_dim, In = p.in_dim, Rk = p.rank;
  const int X = 2 * Hd;
  const int fslice = (Hd + kAdCluster - 1) / kAdCluster;  // output features per CTA
  const int rslice = (Rk + kAdCluster - 1) / kAdCluster;  // adapter rank per CTA
  const int f0 = min(Hd, crank * fslice), f1 = min(Hd, f0 + fslice);
  const int r0 = min(Rk, crank * rslice), r1 = min(Rk, r0 + rslice);
  // shared: o slice [kAdRows][fslice] (read by peers), gelu slice [kAdRows][rslice] (read by
  // peers), x [kAdRows][2 Hd] (hidden, o), g [kAdRows][Rk]
  float* o_loc = ad_smem;
  float* g_loc = o_loc + kAdRows * fslice;
  float* x = g_loc + kAdRows * rslice;
  float* g = x + kAdRows * X;
  const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const T* ow = reinterpret_cast<const T*>(p.o_weight);
  const T* ob = reinterpret_cast<const T*>(p.o_bias);

  // 1. o for this CTA's features
  for (int e = warp; e < nrows * (f1 - f0); e += nwarps) {
    const int n = e / (f1 - f0), j = f0 + e % (f1 - f0);
    const T* a = reinterpret_cast<const T*>(p.attn) + (int64_t)(row0 + n) * p.attn_row_stride;
    float v = warp_dot<T, T>(a, ow + (int64_t)j * In, In);
    if (ob) v += to_f32<T>(ob[j]);
    if (lane == 0) o_loc[n * fslice + (j - f0)] = round_to<T>(v);
  }
  // hidden rows as fp32
  for (int e = threadIdx.x; e < nrows * Hd; e += blockDim.x) {
    const int n = e / Hd, d = e - n * Hd;
    x[n * X + d] = to_f32<T>(reinterpret_cast<const T*>(p.hidden)[(int64_t)(row0 + n) * p.hidden_row_stride + d]);
  }
  cluster.sync();
  // 2. the full o rows from every CTA
  for (int c = 0; c < kAdCluster; ++c) {
    const float* src = cluster.map_shared_rank(o_loc, c);
    const int c0 = min(Hd, c * fslice), c1 = min(Hd, c0 + fslice);
    for (int e = threadIdx.x; e < nrows * (c1 - c0); e += blockDim.x) {
      const int n = e / (c1 - c0), j = e - n * (c1 - c0);
      x[n * X + Hd + c0 + j] = src[n * fslice + j];
    }
  }
  __syncthreads();
  // 3. this CTA's slice of down(.) and gelu
  for (int e = warp; e < nrows * (r1 - r0); e += nwarps) {
    const int n = e / (r1 - r0), r = r0 + e % (r1 - r0);
    const float d = warp_dot<float, float>(x + n * X, p.down + (int64_t)r * X, X);
    if (lane == 0) g_loc[n * rslice + (r - r0)] = gelu_erf(d);
  }
  cluster.sync();
  for (int c = 0; c < kAdCluster; ++c) {
    const float* src = cluster.map_shared_rank(g_loc, c);
    const int c0 = min(Rk, c * rslice), c1 = min(Rk, c0 + rslice);
    for (int e = threadIdx.x; e < nrows * (c1 - c0); e += blockDim.x) {
      const int n = e / (c1 - c0), r = e - n * (c1 - c0);
      g[n * Rk + c0 + r] = src[n * rslice + r];
    }
  }
  // peers read this CTA's slices only before this barrier
  cluster.sync();
  // 4. up(.) * scale for this CTA's features and the residual sum
  T* out = reinterpret_cast<T*>(p.out);
  for (int e = warp; e < nrows * (f1 - f0); e += nwarps) {
    const int n = e / (f1 - f0), j = f0 + e % (f1 - f0);
    const float c = warp_dot<float, float>(g + n * Rk, p.up + (int64_t)j * Rk, Rk) * p.scale;
    if (lane == 0) {
      const float o = x[n * X + Hd + j];
      out[(int64_t)(row0 + n) * p.out_row_stride + j] = from_f32<T>(o + round_to<T>(c));
    }
  }
}

template <typename T>
static int launch_adapter(const AdapterParams& p, cudaStream_t st) {
  const int fslice = (p.hidden_dim + kAdCluster - 1) / kAdCluster;
  const int rslice = (p.rank + kAdCluster - 1) / kAdCluster;
  const size_t smem = sizeof(float) * (kAdRows * fslice + kAdRows * rslice + kAdRows * 2 * p.hidden_dim +
                                       kAdRows * p.rank);
  if (smem > static_cast<size_t>(kMaxDynSmem)) return set_error(SVA_ERR_SHAPE, "adapter shapes exceed shared memory");
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(adapter_fused_kernel<T>), static_cast<int>(smem));
  if (rc != SVA_OK) return rc;
  const int blocks = (p.n_rows + kAdRows - 1) / kAdRows;
  adapter_fused_kernel<T><<<blocks * kAdCluster, kAdThreads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SVA_OK : set_error(SVA_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace sva

extern "C" int sva_adapter_forward(const void* hidden, int64_t hidden_row_stride, const void* attn,
                                   int64_t attn_row_stride, int32_t dtype, const void* o_weight, const void* o_bias,
                                   const float* down, const float* up, float scale, int32_t n_rows,
                                   int32_t hidden_dim, int32_t in_dim, int32_t rank, void* out,
                                   int64_t out_row_stride, void* stream) {
  using namespace sva;
  if (n_rows < 0 || hidden_dim <= 0 || hidden_dim > kAdMaxHidden || in_dim <= 0 || in_dim > 4 * kAdMaxHidden ||
      rank <= 0 || rank > kAdMaxRank)
    return set_error(SVA_ERR_SHAPE, "adapter sizes out of range");
  if (!hidden || !attn || !o_weight || !down || !up || !out) return set_error(SVA_ERR_SHAPE, "a required pointer is null");
  if (n_rows == 0) return SVA_OK;
  AdapterParams p{hidden, hidden_row_stride, attn, attn_row_stride, o_weight, o_bias, down, up, scale,
                  n_rows,  hidden_dim,        in_dim, rank,          out,    out_row_stride};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SVA_DTYPE_F32: return launch_adapter<float>(p, st);
    case SVA_DTYPE_BF16: return launch_adapter<__nv_bfloat16>(p, st);
    case SVA_DTYPE_F16: return launch_adapter<__half>(p, st);
    default: return set_error(SVA_ERR_DTYPE, "dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
  }
}
