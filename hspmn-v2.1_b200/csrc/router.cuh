// Router top-K selection (TopKRouter.forward, hspmn_v2_1.py:98,104-105,112-120).
//
// One CTA per sequence, or, for a few long sequences, one cluster of
// kRouterClusterCtas CTAs per sequence, each owning a slice of the row and
// combining histograms and counts through distributed shared memory.
// Each logit becomes an order-preserving unsigned key
// of the rounded `noisy` value (16 bits for bf16/f16, 32 bits for f32); an
// MSB-first radix select with 256-bin shared-memory histograms finds the K-th
// largest key T; one pass in position order then keeps every key > T and the
// first (K - #{key > T}) keys == T, writing positions ascending and the mask.
// Keys live in shared memory when the row fits, otherwise they are recomputed
// from the (L2-resident) logits on every pass.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace hspmn {

constexpr int kRouterThreads = 512;
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kRouterItems = 8;  // consecutive positions per thread per chunk
constexpr int kRouterChunk = kRouterThreads * kRouterItems;
constexpr int kRouterSmemKeyBytes = 96 * 1024;
// rows of at least this many positions, few enough to fill no more than about
// one wave, are split over a cluster of kRouterClusterCtas CTAs
constexpr int kRouterClusterMinS = 32768;
constexpr int kRouterClusterCtas = 8;

__device__ __forceinline__ uint32_t router_key(float logit, float temp, bool divide, int noisy_dtype) {
  const float q = divide ? __fdiv_rn(logit, temp) : logit;
  if (noisy_dtype == HSPMN_F32) {
    if (q != q) return 0xFFFFFFFFu;
    const uint32_t u = __float_as_uint(q);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  uint32_t u;
  bool nan;
  if (noisy_dtype == HSPMN_BF16) {
    const __nv_bfloat16 h = __float2bfloat16_rn(q);
    u = static_cast<uint32_t>(__bfloat16_as_ushort(h));
    nan = __hisnan(h);
  } else {
    const __half h = __float2half_rn(q);
    u = static_cast<uint32_t>(__half_as_ushort(h));
    nan = __hisnan(h);
  }
  if (nan) return 0xFFFFu;
  return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
}

// Block-wide exclusive prefix sum of one value per thread; returns the prefix
// and writes the block total to *total. `scratch` holds kRouterWarps + 1 ints.
__device__ __forceinline__ int router_block_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kRouterWarps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kRouterWarps) scratch[lane] = w;  // inclusive warp totals
    if (lane == kRouterWarps - 1) scratch[kRouterWarps] = w;
  }
  __syncthreads();
  const int before = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[kRouterWarps];
  const int excl = before + x - v;
  __syncthreads();  // scratch is reused by the next call
  return excl;
}

// One row per cluster of `nct` CTAs (an ordinary launch is a cluster of one):
// CTA `rank` owns positions [rank * slice, (rank + 1) * slice). Every pass
// combines the CTAs through distributed shared memory between hardware
// cluster barriers, so nothing waits on a flag and no global scratch is used.
template <bool kKeysInSmem>
__global__ void __launch_bounds__(kRouterThreads) router_topk_kernel(
    const void* __restrict__ logits, int logits_dtype, int64_t logits_rs, const void* __restrict__ temp,
    int temp_dtype, int noisy_dtype, int S, int K, int64_t* __restrict__ indices, int64_t indices_rs,
    uint8_t* __restrict__ mask, int64_t mask_rs, int slice) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) unsigned char router_smem[];
  __shared__ int hist[256];
  __shared__ int scan_scratch[kRouterWarps + 1];
  __shared__ uint32_t sel_digit_hi;
  __shared__ int sel_remaining;
  __shared__ int slice_gt, slice_eq;  // keys > T and == T in this CTA's slice

  const int nct = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  // a cluster of one (the ordinary launch) needs only block barriers
  auto sync_all = [&]() {
    if (nct > 1) cluster.sync(); else __syncthreads();
  };
  const int b = static_cast<int>(blockIdx.x) / nct;
  const int tid = threadIdx.x;
  const int lo = min(S, rank * slice), hi = min(S, lo + slice);
  const bool divide = temp != nullptr;
  const float t = divide ? load_as_float(temp, temp_dtype, 0) : 1.0f;
  const int64_t row = static_cast<int64_t>(b) * logits_rs;
  const bool wide = noisy_dtype == HSPMN_F32;
  uint32_t* kcache32 = reinterpret_cast<uint32_t*>(router_smem);
  uint16_t* kcache16 = reinterpret_cast<uint16_t*>(router_smem);

  auto compute_key = [&](int s) -> uint32_t {
    return router_key(load_as_float(logits, logits_dtype, row + s), t, divide, noisy_dtype);
  };
  auto key_at = [&](int s) -> uint32_t {  // s in [lo, hi)
    if constexpr (kKeysInSmem) {
      return wide ? kcache32[s - lo] : static_cast<uint32_t>(kcache16[s - lo]);
    } else {
      return compute_key(s);
    }
  };

  if constexpr (kKeysInSmem) {
    for (int s = lo + tid; s < hi; s += kRouterThreads) {
      const uint32_t k = compute_key(s);
      if (wide) kcache32[s - lo] = k; else kcache16[s - lo] = static_cast<uint16_t>(k);
    }
  }

  // ---- radix select: the K-th largest key --------------------------------
  uint32_t prefix = 0, prefix_mask = 0;
  int remaining = K;
  const int nbits = wide ? 32 : 16;
  for (int shift = nbits - 8; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kRouterThreads) hist[i] = 0;
    __syncthreads();
    // kRouterItems consecutive positions per thread per chunk, all loaded
    // before any is counted, so each thread keeps several loads in flight
    for (int c0 = lo; c0 < hi; c0 += kRouterChunk) {
      const int s0 = c0 + tid * kRouterItems;
      uint32_t keys[kRouterItems];
#pragma unroll
      for (int j = 0; j < kRouterItems; ++j) keys[j] = s0 + j < hi ? key_at(s0 + j) : 0u;
#pragma unroll
      for (int j = 0; j < kRouterItems; ++j)
        if (s0 + j < hi && (keys[j] & prefix_mask) == prefix) atomicAdd(&hist[(keys[j] >> shift) & 0xFFu], 1);
    }
    sync_all();  // every slice histogram is complete
    if (rank == 0 && tid < 32) {
      // lane l owns digits [8*(31-l), 8*(31-l)+8): lane 0 the highest ones;
      // counts summed over the cluster's slices
      const int lane = tid;
      const int base = 8 * (31 - lane);
      int c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) c[j] = 0;
      for (int r = 0; r < nct; ++r) {
        const int* h = cluster.map_shared_rank(hist, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] += h[base + j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += c[j];
      int incl = sum;  // inclusive scan over lanes = counts of digits >= base
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      const int above = incl - sum;  // count of digits above this lane's range
      // the digit holding the remaining-th largest key is in the lane where
      // above < remaining <= incl
      if (above < remaining && remaining <= incl) {
        int acc = above;
        for (int j = 7; j >= 0; --j) {
          if (acc + c[j] >= remaining) {
            sel_digit_hi = static_cast<uint32_t>(base + j);
            sel_remaining = remaining - acc;
            break;
          }
          acc += c[j];
        }
      }
    }
    sync_all();  // the selection is published in CTA 0
    const uint32_t digit = *cluster.map_shared_rank(&sel_digit_hi, 0);
    remaining = *cluster.map_shared_rank(&sel_remaining, 0);
    prefix |= digit << shift;
    prefix_mask |= 0xFFu << shift;
    sync_all();  // everyone has read it before CTA 0 writes the next one
  }
  const uint32_t T = prefix;      // K-th largest key
  const int need_eq = remaining;  // how many keys == T are kept (lowest positions first)

  // ---- where this slice's output starts ------------------------------------
  int out_base = 0, eq_base = 0;
  if (nct > 1) {
    int n_gt = 0, n_eq = 0;
    for (int s = lo + tid; s < hi; s += kRouterThreads) {
      const uint32_t k = key_at(s);
      n_gt += k > T ? 1 : 0;
      n_eq += k == T ? 1 : 0;
    }
    int tot;
    router_block_scan(n_gt, scan_scratch, &tot);
    if (tid == 0) slice_gt = tot;
    router_block_scan(n_eq, scan_scratch, &tot);
    if (tid == 0) slice_eq = tot;
    cluster.sync();
    for (int r = 0; r < rank; ++r) {  // lower positions live in lower ranks
      const int g = *cluster.map_shared_rank(&slice_gt, r);
      const int e = *cluster.map_shared_rank(&slice_eq, r);
      const int kept = min(e, max(0, need_eq - eq_base));
      out_base += g + kept;
      eq_base += e;
    }
  }

  // ---- compaction in position order --------------------------------------
  int64_t* out_row = indices + static_cast<int64_t>(b) * indices_rs;
  uint8_t* mask_row = mask ? mask + static_cast<int64_t>(b) * mask_rs : nullptr;
  for (int c0 = lo; c0 < hi; c0 += kRouterChunk) {
    const int s0 = c0 + tid * kRouterItems;
    uint32_t keys[kRouterItems];
    int n_eq_c = 0;
#pragma unroll
    for (int j = 0; j < kRouterItems; ++j) {
      const int s = s0 + j;
      keys[j] = s < hi ? key_at(s) : 0u;
      n_eq_c += (s < hi && keys[j] == T) ? 1 : 0;
    }
    int eq_total;
    const int eq_before = eq_base + router_block_scan(n_eq_c, scan_scratch, &eq_total);
    bool sel[kRouterItems];
    int n_sel = 0, e = eq_before;
#pragma unroll
    for (int j = 0; j < kRouterItems; ++j) {
      const int s = s0 + j;
      bool keep = false;
      if (s < hi) {
        if (keys[j] > T) keep = true;
        else if (keys[j] == T) { keep = e < need_eq; ++e; }
      }
      sel[j] = keep;
      n_sel += keep ? 1 : 0;
    }
    int sel_total;
    int pos = out_base + router_block_scan(n_sel, scan_scratch, &sel_total);
#pragma unroll
    for (int j = 0; j < kRouterItems; ++j) {
      const int s = s0 + j;
      if (s < hi) {
        if (sel[j]) out_row[pos++] = s;
        if (mask_row) mask_row[s] = sel[j] ? 1 : 0;
      }
    }
    out_base += sel_total;
    eq_base += eq_total;
  }
  if (nct > 1) cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace hspmn
