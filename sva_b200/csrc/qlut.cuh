// Query side of a summon: q_low = (q . q_proj[h]) * scale[h] and the per-subspace LUT
// lut[s][c] = q_low[s-part] . codebook[s][c], both in the canonical sequential fp32 order
// (reference sva/llama.py:211 and sva/ops.py:63-68).  Block-cooperative; ends with a barrier.
// `stage` (>= D*R floats of shared memory) receives q_proj[h] so that the 64 dependent
// multiply-adds of every q_low element read shared memory; each thread loads its codebook row
// with one batch of vector loads before its multiply-add chain.
#pragma once

#include "sva_common.cuh"

namespace sva {

// q_low = (q . q_proj[h]) * scale[h] into ql (and q as fp32 into qf).  Ends with a barrier.
// kWaitForQ: q_proj is staged first, then the kernel waits for its predecessor (pdl_wait)
// before reading q.
template <typename T, bool kWaitForQ = false>
__device__ void query_low_smem(const T* q, int D, int R, const float* q_proj_h, float scale_h, float* qf, float* ql,
                               float* stage) {
  if (!kWaitForQ)
    for (int d = threadIdx.x; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  const int DR = D * R;
  if ((reinterpret_cast<uintptr_t>(q_proj_h) & 15u) == 0 && (DR & 3) == 0) {
    const float4* src = reinterpret_cast<const float4*>(q_proj_h);
    float4* dst = reinterpret_cast<float4*>(stage);
    for (int e = threadIdx.x; e < DR / 4; e += blockDim.x) dst[e] = __ldg(src + e);
  } else {
    for (int e = threadIdx.x; e < DR; e += blockDim.x) stage[e] = __ldg(q_proj_h + e);
  }
  if (kWaitForQ) {
    pdl_wait();
    for (int d = threadIdx.x; d < D; d += blockDim.x) qf[d] = to_f32<T>(q[d]);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = mac(acc, qf[d], stage[d * R + r]);
    ql[r] = __fmul_rn(acc, scale_h);
  }
  __syncthreads();
}

// lut[s][c] = q_low[s-part] . codebook[s][c] (sequential order).  kCbShared: the codebook is
// already in shared memory (plain loads).  Ends with a barrier.
template <bool kCbShared = false>
__device__ void query_lut(int R, int S, int C, const float* codebooks_h, const float* lut_override, const float* ql,
                          float* lut) {
  const int sub = R / S;
  const int SC = S * C;
  if (lut_override) {
    for (int e = threadIdx.x; e < SC; e += blockDim.x) lut[e] = lut_override[e];
  } else {
    for (int e = threadIdx.x; e < SC; e += blockDim.x) {
      const int s = e / C;
      const float* cb = codebooks_h + (size_t)e * sub;
      const float* qs = ql + s * sub;
      float acc = 0.f;
      if ((sub & 3) == 0 && (reinterpret_cast<uintptr_t>(cb) & 15u) == 0 && sub <= kMaxRank) {
        float4 row[kMaxRank / 4];
#pragma unroll
        for (int j = 0; j < kMaxRank / 4; ++j)
          if (4 * j < sub)
            row[j] = kCbShared ? reinterpret_cast<const float4*>(cb)[j] : __ldg(reinterpret_cast<const float4*>(cb) + j);
#pragma unroll
        for (int j = 0; j < kMaxRank / 4; ++j) {
          if (4 * j < sub) {
            acc = mac(acc, qs[4 * j + 0], row[j].x);
            acc = mac(acc, qs[4 * j + 1], row[j].y);
            acc = mac(acc, qs[4 * j + 2], row[j].z);
            acc = mac(acc, qs[4 * j + 3], row[j].w);
          }
        }
      } else {
        for (int j = 0; j < sub; ++j) acc = mac(acc, qs[j], kCbShared ? cb[j] : __ldg(cb + j));
      }
      lut[e] = acc;
    }
  }
  __syncthreads();
}

// query_lut for a compile-time subspace width SUB (a multiple of 4) with the codebook in shared
// memory: the row is SUB / 4 vector loads and the chain is fully unrolled.  Same order and
// result as query_lut.  Ends with a barrier.
template <int SUB>
__device__ void query_lut_fixed(int S, int C, const float* codebooks_h, const float* ql, float* lut) {
  const int SC = S * C;
  for (int e = threadIdx.x; e < SC; e += blockDim.x) {
    const int s = e / C;
    const float4* cb = reinterpret_cast<const float4*>(codebooks_h + (size_t)e * SUB);
    const float* qs = ql + s * SUB;
    float4 row[SUB / 4];
#pragma unroll
    for (int j = 0; j < SUB / 4; ++j) row[j] = cb[j];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < SUB / 4; ++j) {
      acc = mac(acc, qs[4 * j + 0], row[j].x);
      acc = mac(acc, qs[4 * j + 1], row[j].y);
      acc = mac(acc, qs[4 * j + 2], row[j].z);
      acc = mac(acc, qs[4 * j + 3], row[j].w);
    }
    lut[e] = acc;
  }
  __syncthreads();
}

template <typename T>
__device__ void build_query_lut(const T* q, int D, int R, int S, int C, const float* q_proj_h, float scale_h,
                                const float* codebooks_h, const float* lut_override, float* qf, float* ql, float* lut,
                                float* stage) {
  query_low_smem<T>(q, D, R, q_proj_h, scale_h, qf, ql, stage);
  query_lut<false>(R, S, C, codebooks_h, lut_override, ql, lut);
}

}  // namespace sva
