// Row gather / scatter between the [B,S,D] stream and the [B,K,D] selected
// rows (hspmn_v2_1.py:185-186 and :195-196). Rows are opaque byte strings
// moved with the widest vector the pointers, strides and row length allow
// (16 bytes for every shape on the path); one warp moves one row with all its
// loads in flight before the stores.
#pragma once

#include "common.cuh"

namespace hspmn {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kScatterRowsPerCta = 32;

template <typename V>
__device__ __forceinline__ void copy_row(V* __restrict__ dst, const V* __restrict__ src, int64_t nvec, int lane) {
  constexpr int U = 8;
  int64_t v = lane;
  for (; v + 32 * (U - 1) < nvec; v += 32 * U) {
    V tmp[U];
#pragma unroll
    for (int u = 0; u < U; ++u) tmp[u] = __ldcs(src + v + 32 * u);
#pragma unroll
    for (int u = 0; u < U; ++u) __stcs(dst + v + 32 * u, tmp[u]);
  }
  for (; v < nvec; v += 32) __stcs(dst + v, __ldcs(src + v));
}

template <typename V>
__device__ __forceinline__ void zero_row(V* __restrict__ dst, int64_t nvec, int lane) {
  V z;
  memset(&z, 0, sizeof(V));
  for (int64_t v = lane; v < nvec; v += 32) __stcs(dst + v, z);
}

// dst[b,i,:] = src[b, idx[b,i], :]; positions outside [0,S) write a zero row
// and raise HSPMN_DEVERR_POSITION.
template <typename V>
__global__ void __launch_bounds__(kRowThreads) gather_rows_kernel(
    const char* __restrict__ src, int64_t src_sb, int64_t src_ss, const int64_t* __restrict__ idx,
    int64_t idx_sb, char* __restrict__ dst, int64_t dst_sb, int64_t dst_sk, int64_t B, int64_t S, int64_t K,
    int64_t nvec) {
  const int lane = threadIdx.x & 31;
  const int64_t nrows = B * K;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < nrows;
       r += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int64_t b = r / K, i = r - b * K;
    const int64_t s = __ldg(idx + b * idx_sb + i);
    V* d = reinterpret_cast<V*>(dst + b * dst_sb + i * dst_sk);
    if (s < 0 || s >= S) {
      if (lane == 0) raise_device_error(HSPMN_DEVERR_POSITION);
      zero_row(d, nvec, lane);
      continue;
    }
    copy_row(d, reinterpret_cast<const V*>(src + b * src_sb + s * src_ss), nvec, lane);
  }
}

__device__ __forceinline__ int64_t lower_bound_i64(const int64_t* a, int64_t n, int64_t x) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(a + mid) < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// One CTA per (window of kScatterRowsPerCta positions, sequence): binary
// searches find the selected entries inside the window, then every position
// of the window is written once, either its attention row or zeros.
template <typename V>
__global__ void __launch_bounds__(kRowThreads) scatter_rows_kernel(
    const char* __restrict__ src, int64_t src_sb, int64_t src_sk, const int64_t* __restrict__ idx,
    int64_t idx_sb, char* __restrict__ dst, int64_t dst_sb, int64_t dst_ss, int64_t S, int64_t K, int64_t nvec) {
  __shared__ int64_t win_lo, win_hi;
  __shared__ int slot[kScatterRowsPerCta];
  const int64_t b = blockIdx.y;
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kScatterRowsPerCta;
  const int64_t s1 = min(S, s0 + kScatterRowsPerCta);
  const int64_t* irow = idx + b * idx_sb;
  if (threadIdx.x == 0) win_lo = lower_bound_i64(irow, K, s0);
  if (threadIdx.x == 32) win_hi = lower_bound_i64(irow, K, s1);
  if (threadIdx.x < kScatterRowsPerCta) slot[threadIdx.x] = -1;
  __syncthreads();
  const int64_t lo = win_lo, hi = win_hi;
  for (int64_t j = lo + threadIdx.x; j < hi; j += kRowThreads) {
    const int64_t s = __ldg(irow + j);
    if (j > 0 && __ldg(irow + j - 1) >= s) raise_device_error(HSPMN_DEVERR_UNSORTED);
    if (s >= s0 && s < s1) slot[s - s0] = static_cast<int>(j);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t s = s0 + (threadIdx.x >> 5); s < s1; s += kRowWarps) {
    V* d = reinterpret_cast<V*>(dst + b * dst_sb + s * dst_ss);
    const int j = slot[s - s0];
    if (j >= 0) copy_row(d, reinterpret_cast<const V*>(src + b * src_sb + j * src_sk), nvec, lane);
    else zero_row(d, nvec, lane);
  }
}

}  // namespace hspmn
