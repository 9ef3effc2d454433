// Shared device helpers for the SVA summon -> verify kernels (sm_100a).
//
// Canonical arithmetic.  Every fp32 dot product that feeds a selection is evaluated in one of
// two fixed orders with separately rounded multiplies and adds (__fmul_rn / __fadd_rn, which
// the compiler never contracts into an FMA):
//   seq_dot : acc = 0; for i: acc = acc + a[i]*b[i]
//   tree_dot: 16 lanes; lane j sums elements 4j..4j+3 in order; lanes combined by a butterfly
//             xor 8, 4, 2, 1 (the shuffle order of a 16-lane reduction).
// The CPU oracle (oracle/sva_oracle.py) evaluates the same orders, so codes, shortlists and
// final indices are bit-identical between the two.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sva_b200.h"

namespace sva {

constexpr int kMaxRank = 64;        // rank_dim <= 64, multiple of 4
constexpr int kMaxSubspaces = 8;
constexpr int kMaxCodewords = 256;  // uint8 codes
constexpr int kMaxLut = 2048;       // subspaces * codewords
constexpr int kMaxHeadDim = 256;

// ---------------------------------------------------------------------------------------
// ordered keys
// ---------------------------------------------------------------------------------------

// Map an fp32 score to a uint32 whose unsigned order is the float order; -0 folds onto +0.
// Valid scores never map to 0 (that would be a negative NaN), so 0 marks "not a candidate".
__device__ __forceinline__ uint32_t ordered_key(float s) {
  uint32_t u = __float_as_uint(s);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// ---------------------------------------------------------------------------------------
// element loads
// ---------------------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// Round an fp32 value to the storage precision of T (identity for float).
template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<float>(float v) { return v; }
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
template <>
__device__ __forceinline__ float round_to<__half>(float v) { return __half2float(__float2half_rn(v)); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// The same from memory the read-only path cannot address (shared memory): plain loads.
template <typename T>
__device__ __forceinline__ float4 load4s(const T* row, int e, int n) {
  float4 r;
  r.x = (e + 0 < n) ? to_f32<T>(row[e + 0]) : 0.f;
  r.y = (e + 1 < n) ? to_f32<T>(row[e + 1]) : 0.f;
  r.z = (e + 2 < n) ? to_f32<T>(row[e + 2]) : 0.f;
  r.w = (e + 3 < n) ? to_f32<T>(row[e + 3]) : 0.f;
  return r;
}

// Vector forms of load4s when row + e is aligned to the four elements and in range.
template <>
__device__ __forceinline__ float4 load4s<float>(const float* row, int e, int n) {
  if (e + 4 <= n && ((reinterpret_cast<uintptr_t>(row + e) & 15u) == 0)) return *reinterpret_cast<const float4*>(row + e);
  float4 r;
  r.x = (e + 0 < n) ? row[e + 0] : 0.f;
  r.y = (e + 1 < n) ? row[e + 1] : 0.f;
  r.z = (e + 2 < n) ? row[e + 2] : 0.f;
  r.w = (e + 3 < n) ? row[e + 3] : 0.f;
  return r;
}
template <>
__device__ __forceinline__ float4 load4s<__nv_bfloat16>(const __nv_bfloat16* row, int e, int n) {
  if (e + 4 <= n && ((reinterpret_cast<uintptr_t>(row + e) & 7u) == 0)) {
    const uint2 raw = *reinterpret_cast<const uint2*>(row + e);
    return make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u), __uint_as_float(raw.y << 16),
                       __uint_as_float(raw.y & 0xFFFF0000u));
  }
  float4 r;
  r.x = (e + 0 < n) ? __bfloat162float(row[e + 0]) : 0.f;
  r.y = (e + 1 < n) ? __bfloat162float(row[e + 1]) : 0.f;
  r.z = (e + 2 < n) ? __bfloat162float(row[e + 2]) : 0.f;
  r.w = (e + 3 < n) ? __bfloat162float(row[e + 3]) : 0.f;
  return r;
}
template <>
__device__ __forceinline__ float4 load4s<__half>(const __half* row, int e, int n) {
  if (e + 4 <= n && ((reinterpret_cast<uintptr_t>(row + e) & 7u) == 0)) {
    const uint2 raw = *reinterpret_cast<const uint2*>(row + e);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  float4 r;
  r.x = (e + 0 < n) ? __half2float(row[e + 0]) : 0.f;
  r.y = (e + 1 < n) ? __half2float(row[e + 1]) : 0.f;
  r.z = (e + 2 < n) ? __half2float(row[e + 2]) : 0.f;
  r.w = (e + 3 < n) ? __half2float(row[e + 3]) : 0.f;
  return r;
}

// Four consecutive elements starting at e (elements at or beyond n read as 0).
template <typename T>
__device__ __forceinline__ float4 load4(const T* __restrict__ row, int e, int n) {
  float4 r;
  r.x = (e + 0 < n) ? to_f32<T>(row[e + 0]) : 0.f;
  r.y = (e + 1 < n) ? to_f32<T>(row[e + 1]) : 0.f;
  r.z = (e + 2 < n) ? to_f32<T>(row[e + 2]) : 0.f;
  r.w = (e + 3 < n) ? to_f32<T>(row[e + 3]) : 0.f;
  return r;
}

// Vectorised variants when the row pointer + element offset is suitably aligned and in range.
template <>
__device__ __forceinline__ float4 load4<float>(const float* __restrict__ row, int e, int n) {
  if (e + 4 <= n && ((reinterpret_cast<uintptr_t>(row + e) & 15u) == 0)) return __ldg(reinterpret_cast<const float4*>(row + e));
  float4 r;
  r.x = (e + 0 < n) ? row[e + 0] : 0.f;
  r.y = (e + 1 < n) ? row[e + 1] : 0.f;
  r.z = (e + 2 < n) ? row[e + 2] : 0.f;
  r.w = (e + 3 < n) ? row[e + 3] : 0.f;
  return r;
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* __restrict__ row, int e, int n) {
  if (e + 4 <= n && ((reinterpret_cast<uintptr_t>(row + e) & 7u) == 0)) {
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(row + e));
    float4 r;
    r.x = __uint_as_float(raw.x << 16);
    r.y = __uint_as_float(raw.x & 0xFFFF0000u);
    r.z = __uint_as_float(raw.y << 16);
    r.w = __uint_as_float(raw.y & 0xFFFF0000u);
    return r;
  }
  float4 r;
  r.x = (e + 0 < n) ? __bfloat162float(row[e + 0]) : 0.f;
  r.y = (e + 1 < n) ? __bfloat162float(row[e + 1]) : 0.f;
  r.z = (e + 2 < n) ? __bfloat162float(row[e + 2]) : 0.f;
  r.w = (e + 3 < n) ? __bfloat162float(row[e + 3]) : 0.f;
  return r;
}

// ---------------------------------------------------------------------------------------
// canonical dot products
// ---------------------------------------------------------------------------------------

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may
// start while its predecessor in the stream still runs; it waits here before touching anything
// the predecessor writes (a no-op for an ordinary launch).  The predecessor lets it start once
// every one of its CTAs has run launch_dependents.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float mac(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }

// Partial of one tree_dot lane: elements 4j..4j+3 summed in order from 0.
__device__ __forceinline__ float lane4(float4 a, float4 b) {
  float p = __fmul_rn(a.x, b.x);
  p = mac(p, a.y, b.y);
  p = mac(p, a.z, b.z);
  p = mac(p, a.w, b.w);
  return p;
}

// Butterfly over 16 lanes of a warp (lanes 0-15 and 16-31 reduce independently).
__device__ __forceinline__ float tree16(float p) {
  p = __fadd_rn(p, __shfl_xor_sync(0xFFFFFFFFu, p, 8));
  p = __fadd_rn(p, __shfl_xor_sync(0xFFFFFFFFu, p, 4));
  p = __fadd_rn(p, __shfl_xor_sync(0xFFFFFFFFu, p, 2));
  p = __fadd_rn(p, __shfl_xor_sync(0xFFFFFFFFu, p, 1));
  return p;
}

// ---------------------------------------------------------------------------------------
// block helpers
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Exclusive scan of one int per thread across the block; returns the exclusive prefix and
// writes the block total to *total.  `scratch` needs (blockDim.x / 32 + 1) ints.
__device__ __forceinline__ int block_excl_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int incl = warp_incl_scan(v);
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < nwarps) ? scratch[lane] : 0;
    int wi = warp_incl_scan(w);
    if (lane < nwarps) scratch[lane] = wi - w;
    if (lane == nwarps - 1) scratch[nwarps] = wi;
  }
  __syncthreads();
  int res = scratch[warp] + incl - v;
  *total = scratch[nwarps];
  __syncthreads();
  return res;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

}  // namespace sva
