// Exact verify over selected keys, shared by the scan and inverted decode kernels
// (replaces sva/llama.py:304-317 and :532-553).
//
// logits : q . K[key] * softmax_scale, one half-warp per key row (16 lanes x 4 elements per
//          64-wide chunk, tree order).  logits_mode 1 reproduces the reference scan path for
//          bf16 / fp16 models: every product rounded to the value dtype, the sum rounded, the
//          scaled logit rounded.  logits_mode 0 keeps fp32 logits (static path, benchmark).
// softmax: fp32 max, fp64 denominator; weights rounded to the value dtype (the reference casts
//          the fp32 softmax to the query dtype).
// output : sum_j round(w_j * V[j]) accumulated in fp64 (exact for bf16 products, so the result
//          does not depend on the order of the selected keys or on how rows are split between
//          CTAs), rounded to the value dtype.
// Every function is block-cooperative and ends with a barrier.
#pragma once

#include "sva_common.cuh"

namespace sva {

constexpr int kVerifyUnroll = 8;

// Row addressing of the verify functions: row(j) is the address of the j-th selected key's K
// (or V) row.  StridedRows covers one head of a [heads][keys][D] cache with arbitrary strides;
// the decode kernels pass their own functors for paged and batched caches.
template <typename T>
struct StridedRows {
  const T* base;        // the head's row 0
  int64_t row_stride;   // elements
  const int32_t* rows;  // key indices, or NULL for rows 0..n-1
  __device__ __forceinline__ const T* operator()(int j) const { return base + (int64_t)(rows ? rows[j] : j) * row_stride; }
};

template <typename T>
__device__ __forceinline__ StridedRows<T> strided_rows(const void* base, int64_t head_stride, int64_t row_stride,
                                                        int kvh, const int32_t* rows) {
  return StridedRows<T>{reinterpret_cast<const T*>(base) + kvh * head_stride, row_stride, rows};
}

struct NoPrefetch {
  __device__ __forceinline__ const void* operator()(int) const { return nullptr; }
};

// logits of n selected keys: lg[j] = q . K[row(j)] * softmax_scale (see the file comment).
// `vrow` (optional): the V rows of the same keys are prefetched into L2 while the K rows load,
// so that the weighted sum that follows reads them from L2.
// kShared: the rows live in shared memory (staged copies), read with plain loads.  U: rows in
// flight per half-warp.
template <typename T, bool kShared = false, int U = kVerifyUnroll, class KRow, class VRow = NoPrefetch>
__device__ void verify_logits_fn(const KRow& krow, const float* qf, int D, int n, float softmax_scale,
                                 int logits_mode, float* lg, const VRow& vrow = VRow(), bool prefetch_v = false) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int half = lane >> 4, l16 = lane & 15;
  for (int base = warp * 2 * U; base < n; base += nwarps * 2 * U) {
    float part[U];
#pragma unroll
    for (int u = 0; u < U; ++u) part[u] = 0.f;
    for (int c0 = 0; c0 < D; c0 += 64) {
      const int e = c0 + 4 * l16;
      float4 k4[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + 2 * u + half;
        if (j < n && e < D) {
          const T* kr = krow(j);
          k4[u] = kShared ? load4s<T>(kr, e, D) : load4<T>(kr, e, D);
        } else {
          k4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      if (prefetch_v) {
        // one prefetch per 128-byte line of each row's chunk: lanes l16 = 0, 8 of every half-warp
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int j = base + 2 * u + half;
          if (j < n && e < D && ((e * static_cast<int>(sizeof(T))) & 127) == 0)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const T*>(vrow(j)) + e));
        }
      }
      const float4 qv = (e < D) ? make_float4(qf[e], (e + 1 < D) ? qf[e + 1] : 0.f, (e + 2 < D) ? qf[e + 2] : 0.f,
                                              (e + 3 < D) ? qf[e + 3] : 0.f)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (logits_mode == 1) {
          float s = round_to<T>(__fmul_rn(k4[u].x, qv.x));
          s = __fadd_rn(s, round_to<T>(__fmul_rn(k4[u].y, qv.y)));
          s = __fadd_rn(s, round_to<T>(__fmul_rn(k4[u].z, qv.z)));
          s = __fadd_rn(s, round_to<T>(__fmul_rn(k4[u].w, qv.w)));
          part[u] = __fadd_rn(part[u], s);
        } else {
          part[u] = __fadd_rn(part[u], lane4(k4[u], qv));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + 2 * u + half;
      float s = tree16(part[u]);
      if (logits_mode == 1) {
        s = round_to<T>(s);
        s = round_to<T>(__fmul_rn(s, softmax_scale));
      } else {
        s = __fmul_rn(s, softmax_scale);
      }
      if (j < n && l16 == 0) lg[j] = s;
    }
  }
  __syncthreads();
}

// The same over one head of a strided cache; `rows` are key indices, NULL means rows 0..n-1.
// `values` (optional): prefetch the V rows of the same keys into L2.
template <typename T, bool kShared = false>
__device__ void verify_logits(const void* keys, int64_t k_head_stride, int64_t k_row_stride, int kvh, const float* qf,
                              int D, const int32_t* rows, int n, float softmax_scale, int logits_mode, float* lg,
                              const void* values = nullptr, int64_t v_head_stride = 0, int64_t v_row_stride = 0) {
  const StridedRows<T> kr = strided_rows<T>(keys, k_head_stride, k_row_stride, kvh, rows);
  if (values) {
    const StridedRows<T> vr = strided_rows<T>(values, v_head_stride, v_row_stride, kvh, rows);
    verify_logits_fn<T, kShared>(kr, qf, D, n, softmax_scale, logits_mode, lg, vr, true);
  } else {
    verify_logits_fn<T, kShared>(kr, qf, D, n, softmax_scale, logits_mode, lg);
  }
}

// Max (fp32) and fp64 denominator of softmax over lg[0, n); every thread gets both.
// `red` needs (blockDim.x / 32 + 1) doubles, `scratch` 33 ints.
__device__ inline void softmax_stats(const float* lg, int n, int* scratch, double* red, float* mx_out,
                                     float* denom_out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  float mx = -INFINITY;
  for (int j = tid; j < n; j += blockDim.x) mx = fmaxf(mx, lg[j]);
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
  for (int j = tid; j < n; j += blockDim.x) se += static_cast<double>(expf(lg[j] - mx));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xFFFFFFFFu, se, o);
  if (lane == 0) red[warp] = se;
  __syncthreads();
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < nwarps; ++w) tot += red[w];
    red[nwarps] = tot;
  }
  __syncthreads();
  *mx_out = mx;
  *denom_out = static_cast<float>(red[nwarps]);
  __syncthreads();
}

// w[j] = round_T(exp(lg[j] - mx) / denom) for j in [0, n), in place.
template <typename T>
__device__ void softmax_weights(float* lg, int n, float mx, float denom) {
  for (int j = threadIdx.x; j < n; j += blockDim.x) lg[j] = round_to<T>(expf(lg[j] - mx) / denom);
  __syncthreads();
}

// out[d] = sum_j round_T(w[j] * V[row(j)][d]) in fp64 for d < D (written by threads 0..63 per
// 64-wide chunk).  `acc` needs (blockDim.x / 32) * 64 doubles.  U: rows in flight per half-warp.
template <typename T, bool kShared = false, int U = kVerifyUnroll, class VRow>
__device__ void accumulate_rows_fn(const VRow& vrow, int D, const float* w, int n, double* acc, double* out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int half = lane >> 4, l16 = lane & 15;
  const int nchunks = (D + 63) / 64;
  for (int c = 0; c < nchunks; ++c) {
    const int e = c * 64 + 4 * l16;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    for (int base = warp * 2 * U; base < n; base += nwarps * 2 * U) {
      float4 v[U];
      float wu[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + 2 * u + half;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        wu[u] = 0.f;
        if (j < n && e < D) {
          const T* vr = vrow(j);
          v[u] = kShared ? load4s<T>(vr, e, D) : load4<T>(vr, e, D);
          wu[u] = w[j];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        a0 += static_cast<double>(round_to<T>(__fmul_rn(wu[u], v[u].x)));
        a1 += static_cast<double>(round_to<T>(__fmul_rn(wu[u], v[u].y)));
        a2 += static_cast<double>(round_to<T>(__fmul_rn(wu[u], v[u].z)));
        a3 += static_cast<double>(round_to<T>(__fmul_rn(wu[u], v[u].w)));
      }
    }
    a0 += __shfl_xor_sync(0xFFFFFFFFu, a0, 16);
    a1 += __shfl_xor_sync(0xFFFFFFFFu, a1, 16);
    a2 += __shfl_xor_sync(0xFFFFFFFFu, a2, 16);
    a3 += __shfl_xor_sync(0xFFFFFFFFu, a3, 16);
    __syncthreads();
    if (half == 0) {
      acc[warp * 64 + 4 * l16 + 0] = a0;
      acc[warp * 64 + 4 * l16 + 1] = a1;
      acc[warp * 64 + 4 * l16 + 2] = a2;
      acc[warp * 64 + 4 * l16 + 3] = a3;
    }
    __syncthreads();
    if (tid < 64 && c * 64 + tid < D) {
      double tot = 0.0;
      for (int w2 = 0; w2 < nwarps; ++w2) tot += acc[w2 * 64 + tid];
      out[c * 64 + tid] = tot;
    }
    __syncthreads();
  }
}

// The same over one head of a strided cache; `rows` are key indices.
template <typename T, bool kShared = false>
__device__ void accumulate_rows(const void* values, int64_t v_head_stride, int64_t v_row_stride, int kvh, int D,
                                const int32_t* rows, const float* w, int n, double* acc, double* out) {
  accumulate_rows_fn<T, kShared>(strided_rows<T>(values, v_head_stride, v_row_stride, kvh, rows), D, w, n, acc, out);
}

// The whole verify inside one CTA.  Shared memory: lg[n_fin] floats; acc[(nwarps * 64) +
// nwarps + 1] doubles; red[kMaxHeadDim] doubles for the output sums; scratch[64] ints.  U: rows
// in flight per half-warp.
template <typename T, int U = kVerifyUnroll, class KRow, class VRow>
__device__ void verify_rows_fn(const KRow& krow, const VRow& vrow, const float* qf, int D, int n_fin,
                               float softmax_scale, int logits_mode, float* lg, double* acc, int* scratch, T* out) {
  verify_logits_fn<T, false, U>(krow, qf, D, n_fin, softmax_scale, logits_mode, lg);
  float mx, denom;
  const int nwarps = blockDim.x >> 5;
  softmax_stats(lg, n_fin, scratch, acc, &mx, &denom);
  softmax_weights<T>(lg, n_fin, mx, denom);
  double* sums = acc + nwarps * 64;  // D doubles after the per-warp partials
  accumulate_rows_fn<T, false, U>(vrow, D, lg, n_fin, acc, sums);
  for (int d = threadIdx.x; d < D; d += blockDim.x) out[d] = from_f32<T>(n_fin > 0 ? static_cast<float>(sums[d]) : 0.f);
  __syncthreads();
}

template <typename T>
__device__ void verify_rows(const void* keys, int64_t k_head_stride, int64_t k_row_stride, const void* values,
                            int64_t v_head_stride, int64_t v_row_stride, int kvh, const float* qf, int D,
                            const int32_t* fin, int n_fin, float softmax_scale, int logits_mode, float* lg,
                            double* acc, int* scratch, T* out) {
  verify_rows_fn<T>(strided_rows<T>(keys, k_head_stride, k_row_stride, kvh, fin),
                    strided_rows<T>(values, v_head_stride, v_row_stride, kvh, fin), qf, D, n_fin, softmax_scale,
                    logits_mode, lg, acc, scratch, out);
}

}  // namespace sva
