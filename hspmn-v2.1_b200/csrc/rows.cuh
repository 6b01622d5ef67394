// Row gather / scatter between the [B,S,D] stream and the [B,K,D] selected
// rows (hspmn_v2_1.py:185-186 and :195-196). Rows are opaque byte strings
// moved with the widest vector the pointers, strides and row length allow
// (16 bytes for every shape on the path); one warp moves one row with all its
// loads in flight before the stores.
#pragma once

#include <type_traits>

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

namespace hspmn {

// ---------------------------------------------------------------------------
// Rotary embedding fused into the gather of the selected rows.
//
// out[b,i,h,:] = rope(src row r, position idx[b,i]) with r = idx[b,i] when the
// source holds all S positions, or r = i when it already holds the selected
// rows. rope is apply_rotary_pos_emb (hspmn_v2_1.py:34-38,66-68) evaluated
// with the reference's per-operation rounding in the element type T:
//   t1 = T(x[d] * cos[p,d]);  t2 = T(rot[d] * sin[p,d]);  out = T(t1 + t2)
// with rot = cat(-x[hd/2:], x[:hd/2]); products and the sum are single fp32
// operations (products of two 16-bit values are exact in fp32), so the result
// is bit-identical to running the three PyTorch ops on the full tensor.
// ---------------------------------------------------------------------------

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  __device__ static float f(float v) { return v; }
  __device__ static float r(float v) { return v; }
};
template <>
struct Elem<__nv_bfloat16> {
  __device__ static float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __nv_bfloat16 r(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct Elem<__half> {
  __device__ static float f(__half v) { return __half2float(v); }
  __device__ static __half r(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ T rope_elem(T x, T partner, bool low_half, T c, T s) {
  const float xf = Elem<T>::f(x);
  const float rot = low_half ? -Elem<T>::f(partner) : Elem<T>::f(partner);
  const T t1 = Elem<T>::r(__fmul_rn(xf, Elem<T>::f(c)));
  const T t2 = Elem<T>::r(__fmul_rn(rot, Elem<T>::f(s)));
  return Elem<T>::r(__fadd_rn(Elem<T>::f(t1), Elem<T>::f(t2)));
}

// 16-bit element types: the same three roundings with packed 16-bit
// arithmetic, two elements per instruction. The product of two 16-bit values
// is exact in fp32, so T(x*c) is the correctly rounded 16-bit product that
// mul.rn.{bf16,f16}x2 returns; fp32 adds two 16-bit values exactly unless
// their exponents differ so much that the smaller is far below half a
// 16-bit ulp, so T(t1 + t2) is the correctly rounded 16-bit sum that
// add.rn.*x2 returns; and rounding to nearest commutes with negation, so
// T(-p * s) is the sign-flipped T(p * s). Bit-identical to rope_elem.
template <bool kBF16>
__device__ __forceinline__ uint32_t rope_pair16(uint32_t x, uint32_t p, uint32_t c, uint32_t s, uint32_t neg) {
  uint32_t t1, t2, o;
  if constexpr (kBF16) {
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t1) : "r"(x), "r"(c));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(t2) : "r"(p), "r"(s));
    t2 ^= neg;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(o) : "r"(t1), "r"(t2));
  } else {
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(t1) : "r"(x), "r"(c));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(t2) : "r"(p), "r"(s));
    t2 ^= neg;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(o) : "r"(t1), "r"(t2));
  }
  return o;
}

template <typename T>
__device__ __forceinline__ uint4 rope_vec(uint4 xv, uint4 pv, bool low, uint4 cv, uint4 sv) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value) {
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    const uint32_t neg = low ? 0x80008000u : 0u;  // rot = -partner in the low half of a head
    uint4 o;
    o.x = rope_pair16<kBF16>(xv.x, pv.x, cv.x, sv.x, neg);
    o.y = rope_pair16<kBF16>(xv.y, pv.y, cv.y, sv.y, neg);
    o.z = rope_pair16<kBF16>(xv.z, pv.z, cv.z, sv.z, neg);
    o.w = rope_pair16<kBF16>(xv.w, pv.w, cv.w, sv.w, neg);
    return o;
  } else {
    constexpr int V = 16 / sizeof(T);
    const T* xa = reinterpret_cast<const T*>(&xv);
    const T* pa = reinterpret_cast<const T*>(&pv);
    const T* ca = reinterpret_cast<const T*>(&cv);
    const T* sa = reinterpret_cast<const T*>(&sv);
    uint4 ov;
    T* oa = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int u = 0; u < V; ++u) oa[u] = rope_elem<T>(xa[u], pa[u], low, ca[u], sa[u]);
    return ov;
  }
}

// One warp per selected row. Each lane takes units of one 16-byte group (V
// elements of T) of a head's low half and its partner group in the high half,
// so every source and table byte is read once per row and both outputs come
// from the same registers (rope(x)[d] pairs x[d] with x[d +- hd/2]); reading
// each group and its partner separately ran at 4.8 TB/s against 5.6. hd is a
// multiple of 2*V so a group never straddles the two halves of a head.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) rope_gather_rows_kernel(
    const T* __restrict__ src, int64_t src_sb, int64_t src_ss, int src_by_position, const int64_t* __restrict__ idx,
    int64_t idx_sb, const T* __restrict__ cos_t, const T* __restrict__ sin_t, int64_t tab_ss, T* __restrict__ dst,
    int64_t dst_sb, int64_t dst_sk, int64_t B, int64_t S, int64_t K, int H, int hd) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int row_elems = H * hd;
  const int nvec = row_elems / V;
  const int half = hd / 2;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < B * K;
       r += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int64_t b = r / K, i = r - b * K;
    const int64_t pos = __ldg(idx + b * idx_sb + i);
    T* d = dst + b * dst_sb + i * dst_sk;
    if (pos < 0 || pos >= S) {
      if (lane == 0) raise_device_error(HSPMN_DEVERR_POSITION);
      for (int v = lane; v < nvec; v += 32) reinterpret_cast<uint4*>(d)[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const T* s = src + b * src_sb + (src_by_position ? pos : i) * src_ss;
    const T* cr = cos_t + pos * tab_ss;
    const T* sr = sin_t + pos * tab_ss;
    // one unit = a low-half group and its partner: each source byte read once
    const int gph = half / V, units = H * gph;
    for (int u = lane; u < units; u += 32) {
      const int h = u / gph;
      const int dd = (u - h * gph) * V;
      const int e = h * hd + dd;
      const uint4 xl = __ldg(reinterpret_cast<const uint4*>(s + e));
      const uint4 xh = __ldg(reinterpret_cast<const uint4*>(s + e + half));
      const uint4 cl = __ldg(reinterpret_cast<const uint4*>(cr + dd));
      const uint4 ch = __ldg(reinterpret_cast<const uint4*>(cr + dd + half));
      const uint4 sl = __ldg(reinterpret_cast<const uint4*>(sr + dd));
      const uint4 sh = __ldg(reinterpret_cast<const uint4*>(sr + dd + half));
      reinterpret_cast<uint4*>(d + e)[0] = rope_vec<T>(xl, xh, true, cl, sl);
      reinterpret_cast<uint4*>(d + e + half)[0] = rope_vec<T>(xh, xl, false, ch, sh);
    }
  }
}

// Rotary embedding of every row of a [B,S,H,hd] tensor whose position is its
// row number (plus pos0): the K RoPE of hspmn_v2_1.py:226-227 in one pass,
// with no index array. Each unit is one 16-byte group of a head's low half and
// its partner group in the high half, so a thread loads x_lo, x_hi and the
// four table groups once and writes both outputs (rope(x)[d] pairs x[d] with
// x[d +- hd/2]). A warp covers one row per iteration, two rows in flight.
// Every unit reads its inputs before writing, so dst may be src itself.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) rope_rows_kernel(
    const T* src, int64_t src_sb, int64_t src_ss, const T* __restrict__ cos_t,
    const T* __restrict__ sin_t, int64_t tab_ss, int64_t pos0, T* dst, int64_t dst_sb, int64_t dst_ss,
    int64_t B, int64_t S, int H, int hd) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int half = hd / 2;
  const int gph = half / V;  // 16-byte groups per half head
  const int units = H * gph;
  const int64_t rows = B * S;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kRowWarps;
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5)) * 2; r0 < rows;
       r0 += 2 * nwarps) {
    for (int u = lane; u < units; u += 32) {
      const int h = u / gph;
      const int d = (u - h * gph) * V;  // column in the low half
      const int e = h * hd + d;
      uint4 xl[2], xh[2], cl[2], ch[2], sl[2], sh[2];
      int64_t bb[2], ss[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t r = min(r0 + k, rows - 1);  // a lone last row is simply done twice
        bb[k] = r / S;
        ss[k] = r - bb[k] * S;
        const T* x = src + bb[k] * src_sb + ss[k] * src_ss + e;
        const int64_t p = (pos0 + ss[k]) * tab_ss + d;
        xl[k] = *reinterpret_cast<const uint4*>(x);
        xh[k] = *reinterpret_cast<const uint4*>(x + half);
        cl[k] = __ldg(reinterpret_cast<const uint4*>(cos_t + p));
        ch[k] = __ldg(reinterpret_cast<const uint4*>(cos_t + p + half));
        sl[k] = __ldg(reinterpret_cast<const uint4*>(sin_t + p));
        sh[k] = __ldg(reinterpret_cast<const uint4*>(sin_t + p + half));
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (r0 + k >= rows) break;
        T* o = dst + bb[k] * dst_sb + ss[k] * dst_ss + e;
        const uint4 lo = rope_vec<T>(xl[k], xh[k], true, cl[k], sl[k]);
        const uint4 hi = rope_vec<T>(xh[k], xl[k], false, ch[k], sh[k]);
        __stcs(reinterpret_cast<uint4*>(o), lo);
        __stcs(reinterpret_cast<uint4*>(o + half), hi);
      }
    }
  }
}

// dst[b, idx[b,i], :] = T(dst[b, idx[b,i], :] + src[b,i,:]) — the residual
// add of hspmn_v2_1.py:238 restricted to the rows the attention wrote (every
// other row of o_proj(scatter(...)) is zero). One warp per selected row.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) scatter_add_rows_kernel(
    const T* __restrict__ src, int64_t src_sb, int64_t src_sk, const int64_t* __restrict__ idx, int64_t idx_sb,
    T* __restrict__ dst, int64_t dst_sb, int64_t dst_ss, int64_t B, int64_t S, int64_t K, int64_t row_elems) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t nvec = row_elems / V;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < B * K;
       r += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int64_t b = r / K, i = r - b * K;
    const int64_t pos = __ldg(idx + b * idx_sb + i);
    if (pos < 0 || pos >= S) {
      if (lane == 0) raise_device_error(HSPMN_DEVERR_POSITION);
      continue;
    }
    const uint4* sv = reinterpret_cast<const uint4*>(src + b * src_sb + i * src_sk);
    uint4* dv = reinterpret_cast<uint4*>(dst + b * dst_sb + pos * dst_ss);
    for (int64_t v = lane; v < nvec; v += 32) {
      const uint4 a = __ldcs(sv + v);
      const uint4 o = dv[v];
      const T* aa = reinterpret_cast<const T*>(&a);
      const T* oa = reinterpret_cast<const T*>(&o);
      uint4 w;
      T* wa = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int u = 0; u < V; ++u) wa[u] = Elem<T>::r(__fadd_rn(Elem<T>::f(oa[u]), Elem<T>::f(aa[u])));
      dv[v] = w;
    }
  }
}

}  // namespace hspmn
