// Router gate with fp32 logits: logits[b,s] = sum_d x[b,s,d] * w[d] + bias.
// This is TopKRouter's gate (hspmn_v2_1.py:84,96, an nn.Linear(dim, 1)) without
// the rounding of the GEMV result to the module dtype, so the selection ranks
// fp32 values and ties between neighbouring bf16 logits mostly disappear.
//
// Summation order (fixed, so a row's logit depends only on its x row, w, bias
// and D, never on the launch): the row is cut into 16-byte vectors of E
// elements (E = 8 for 16-bit types, 4 for f32); lane l of the row's warp owns
// vectors l, l+32, l+64, ... and keeps one fp32 accumulator per slot e < E,
// acc[e] = fma(x, w, acc[e]) over its vectors in ascending order. The lane
// total is a pairwise tree over the slots, the warp total a xor butterfly
// (offsets 16, 8, 4, 2, 1), and the bias is added last. For bf16/f16 inputs
// every product is exact in fp32, so the result is reproducible bit for bit
// on the host.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace hspmn {

constexpr int kGateThreads = 256;
constexpr int kGateWarps = kGateThreads / 32;
constexpr int kGateUnroll = 8;  // 16-byte loads of x in flight per lane

template <typename T>
struct GateVec;

template <>
struct GateVec<float> {
  static constexpr int E = 4;
  __device__ __forceinline__ static void fma(float (&acc)[E], const uint4& x, const uint4& w) {
    acc[0] = fmaf(__uint_as_float(x.x), __uint_as_float(w.x), acc[0]);
    acc[1] = fmaf(__uint_as_float(x.y), __uint_as_float(w.y), acc[1]);
    acc[2] = fmaf(__uint_as_float(x.z), __uint_as_float(w.z), acc[2]);
    acc[3] = fmaf(__uint_as_float(x.w), __uint_as_float(w.w), acc[3]);
  }
  __device__ __forceinline__ static float load(const void* p) { return *static_cast<const float*>(p); }
};

template <typename H2>
__device__ __forceinline__ float2 to_float2(uint32_t v);
template <>
__device__ __forceinline__ float2 to_float2<__nv_bfloat162>(uint32_t v) {
  // bf16 -> f32 is exact: the 16 bits move to the top of the word
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ float2 to_float2<__half2>(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, sizeof(h));
  return __half22float2(h);
}

template <typename H2>
struct GateVec16 {
  static constexpr int E = 8;
  __device__ __forceinline__ static void fma2(float (&acc)[E], int e, uint32_t x, uint32_t w) {
    const float2 xf = to_float2<H2>(x), wf = to_float2<H2>(w);
    acc[e] = fmaf(xf.x, wf.x, acc[e]);
    acc[e + 1] = fmaf(xf.y, wf.y, acc[e + 1]);
  }
  __device__ __forceinline__ static void fma(float (&acc)[E], const uint4& x, const uint4& w) {
    fma2(acc, 0, x.x, w.x);
    fma2(acc, 2, x.y, w.y);
    fma2(acc, 4, x.z, w.z);
    fma2(acc, 6, x.w, w.w);
  }
};

template <>
struct GateVec<__nv_bfloat16> : GateVec16<__nv_bfloat162> {
  __device__ __forceinline__ static float load(const void* p) {
    return __bfloat162float(*static_cast<const __nv_bfloat16*>(p));
  }
};
template <>
struct GateVec<__half> : GateVec16<__half2> {
  __device__ __forceinline__ static float load(const void* p) {
    return __half2float(*static_cast<const __half*>(p));
  }
};

template <int E>
__device__ __forceinline__ float slot_tree(const float (&a)[E]) {
  if constexpr (E == 4) {
    return (a[0] + a[1]) + (a[2] + a[3]);
  } else {
    return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
  }
}

// One warp per (b, s) row, rows strided over the grid. x rows and w are read
// as 16-byte vectors (the host checks the alignment); x streams through once
// (evict-first loads), w stays in L1.
template <typename T>
__global__ void __launch_bounds__(kGateThreads) gate_logits_kernel(
    const char* __restrict__ x, int64_t x_sb, int64_t x_ss, const uint4* __restrict__ w,
    const void* __restrict__ bias, int64_t B, int64_t S, int nvec, float* __restrict__ logits, int64_t logits_rs) {
  using G = GateVec<T>;
  constexpr int E = G::E;
  const int lane = threadIdx.x & 31;
  const float b0 = bias ? G::load(bias) : 0.0f;
  const int64_t rows = B * S;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kGateWarps + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * kGateWarps) {
    const int64_t b = r / S, s = r - b * S;
    const uint4* xr = reinterpret_cast<const uint4*>(x + b * x_sb + s * x_ss);
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.0f;
    int v = lane;
    for (; v + 32 * (kGateUnroll - 1) < nvec; v += 32 * kGateUnroll) {
      uint4 xa[kGateUnroll];
#pragma unroll
      for (int u = 0; u < kGateUnroll; ++u) xa[u] = __ldcs(xr + v + 32 * u);
#pragma unroll
      for (int u = 0; u < kGateUnroll; ++u) G::fma(acc, xa[u], __ldg(w + v + 32 * u));
    }
    for (; v < nvec; v += 32) G::fma(acc, __ldcs(xr + v), __ldg(w + v));
    float t = slot_tree<E>(acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
    if (lane == 0) logits[b * logits_rs + s] = t + b0;
  }
}

}  // namespace hspmn
