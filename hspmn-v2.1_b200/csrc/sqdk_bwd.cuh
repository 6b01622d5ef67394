// Backward of the sparse-query dense-key causal attention on tcgen05 / TMEM /
// TMA (sm_100a): gradients of sqdk_fwd_kernel's output with respect to the
// selected queries, the keys and the values. The reference trains this path
// through FlexAttention's backward (hspmn_v2_1.py:200-216, mask
// (q_idx >= kv_idx) & mask[b, q_idx], GQA as enable_gqa).
//
// Work unit: one sequence b, one K/V head g and a block of 128 keys
// [n0, n0 + 128). The CTA walks the query blocks that can see these keys:
// 64 rows (query, head) r = q * G + h of head group g (the order a TMA box
// over [B,K,H,hd] lands in shared memory), for the queries whose positions
// reach n0 (indices are sorted: a suffix of the query list). Per block j:
//   S^T  = K Q^T       tcgen05.mma SS, M=128 keys, N=64 rows, K=hd
//   dP^T = V dO^T      tcgen05.mma SS, same shape
//   P^T  = 2^(S^T c - lse2),  dS^T / scale = P^T (dP^T - Delta)
//                      one thread per key (TMEM lane); P^T and dS^T go back to
//                      TMEM as 16-bit operands, dS^T also to shared memory
//   dV  += P^T dO      tcgen05.mma TS (A = P^T in TMEM, B = dO MN-major)
//   dK  += dS^T Q      tcgen05.mma TS (A = dS^T in TMEM, B = Q MN-major)
//                      (dS^T / scale: dK and dQ take the scale in fp32, at the
//                      dK store and in the dQ cast)
//   dQ^T = K^T dS      tcgen05.mma SS (A = K MN-major, B = dS MN-major), into
//                      the columns dP^T used; staged in shared memory one
//                      64-column chunk at a time and added into an fp32 dQ in
//                      global memory with one bulk tensor reduce per chunk
//                      (other key blocks add to the same rows)
// dK and dV accumulate in TMEM over all query blocks and are stored once.
//
// TMEM (512 columns, one CTA per SM): two sets of [S^T | dP^T] (64 + 64
// columns; block j uses set j % 2, so the next block's S^T and dP^T overlap
// this block's softmax), dV (128), dK (128).
//
// Warp roles (448 threads):
//   warp 0      setup: K / V loads, then the search for the first query
//               block; TMA producer: Q_j and dO_j through a 3-stage
//               ring (a stage is refilled only after the dK / dV products of
//               the block before last have read it, so two stages would leave
//               the load latency exposed); writes each block's per-row data
//               (position, lse, Delta) a block ahead into a 4-slot ring
//   warp 1      TMEM allocation + MMA issue (the converged warp runs the
//               issue loop; one elected lane issues each product)
//   warps 2..5  P^T / dS^T of rows 0..31 (thread = key), then the dV store
//   warps 6..9  dQ: TMEM -> registers -> shared staging (thread = column d),
//               then one thread issues the bulk reduces into global dQ
//   warps 10..13 P^T / dS^T of rows 32..63, then the dK store
// Each softmax group writes its 16-bit P^T and dS^T only into the S^T
// columns it read itself ([P^T 16 | dS^T 16] per 32 rows), so the two groups
// need no ordering between them; the dV / dK products address each 16-row
// step of their TMEM operand where its group put it.
// Every mbarrier wait is bounded; a wait that gives up flags
// HSPMN_DEVERR_TIMEOUT, the other roles stop, and the CTA drains its copies
// and MMAs and frees its tensor memory before returning. TMEM loads and
// stores are warp-collective: every lane of a warp issues them, and only the
// global stores that follow depend on the lane.
#pragma once

#include "common.cuh"
#include "sqdk.cuh"

namespace hspmn {

constexpr int kBwdKeys = 128;   // keys per CTA (M of the key-major products)
constexpr int kBwdRows = 64;    // rows (query, head) per query block
constexpr int kBwdThreads = 448;
constexpr int kBwdSoftmaxArrivals = 8;  // softmax warps arriving on pfull per block
constexpr int kBwdHD = 128;     // head_dim tile (hd <= 128; columns past hd are zero)
constexpr int kBwdDQBar = 1;    // named barrier of the four dQ warps
constexpr int kBwdEpiBar = 2;   // named barriers 2 and 3: the dV / dK store of each softmax group
constexpr int kBwdStages = 3;   // Q / dO ring depth
constexpr int kBwdInfo = 4;     // per-row block data ring depth (written one block ahead of the stage wait)
static_assert(kBwdRows == 64, "the producer writes two rows of block data per lane");

struct SqdkBwdLayout {
  static constexpr int kChunks = kBwdHD / 64;
  static constexpr int kKVChunkBytes = kBwdKeys * 128;   // 16 KB: 128 rows x 128 B
  static constexpr int kKVBytes = kChunks * kKVChunkBytes;
  static constexpr int kRowChunkBytes = kBwdRows * 128;  // 8 KB
  static constexpr int kRowBytes = kChunks * kRowChunkBytes;
  static constexpr int kDSBytes = kBwdKeys * 128;        // 128 keys x 64 rows x 2 B
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kKVBytes;
  static constexpr int kQOff = kVOff + kKVBytes;
  static constexpr int kDOOff = kQOff + kBwdStages * kRowBytes;
  static constexpr int kDSOff = kDOOff + kBwdStages * kRowBytes;
  static constexpr int kDQChunkBytes = kBwdRows * 64 * 4;  // 64 rows x 64 fp32 columns, row-major
  static constexpr int kDQOff = kDSOff + 2 * kDSBytes;
  static constexpr int kBytes = kDQOff + kDQChunkBytes;  // one 64-column chunk of dQ staged at a time
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kSetCols = 128;  // S^T at +0, dP^T / dQ^T at +64
  static constexpr int kDVCol = 256;
  static constexpr int kDKCol = 384;
};

struct SqdkBwdParams {
  const int64_t* idx;
  int64_t idx_sb, idx_sk;
  const float* lse;    // [B,K,H] natural-log log-sum-exp from the forward
  const float* delta;  // [B,K,H] rowsum(dO * O)
  int64_t row_sb, row_sk;  // strides of lse / delta (elements; head stride 1)
  float* dq;           // fp32 [B,K,H,hd] accumulator (zeroed by the host; written through tmDQ)
  void* dk;
  void* dv;
  int64_t dk_sb, dk_ss, dk_sh, dv_sb, dv_ss, dv_sh;
  int B, K, S, H, Hkv, G, QTb, hd, nkb;
  int chunk;  // (sequence, head) pairs per CTA-order chunk, >= 1
  float scale, scale_log2;
};

// Block index -> (key block kb, sequence b, kv head g). The (sequence, head)
// pairs are taken in chunks of p.chunk pairs, and inside a chunk the low key
// blocks (the ones most queries see, the longest CTAs) come first. CTAs that
// run at the same time then share a few pairs' Q, dO and dQ rows, which stay
// in L2 across their key blocks; in key-block-major order every resident CTA
// would stream a different pair's rows from HBM.
__device__ __forceinline__ void sqdk_bwd_coords(const SqdkBwdParams& p, int item, int& kb, int& b, int& g) {
  const int BG = p.B * p.Hkv;
  const int per_chunk = p.chunk * p.nkb;
  const int c = item / per_chunk;
  const int r = item - c * per_chunk;
  const int pairs = min(p.chunk, BG - c * p.chunk);
  kb = r / pairs;
  const int bg = c * p.chunk + (r - kb * pairs);
  b = bg / p.Hkv;
  g = bg - b * p.Hkv;
}

template <bool kBF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    sqdk_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmDV,
                    const __grid_constant__ CUtensorMap tmDK, const SqdkBwdParams p) {
  using L = SqdkBwdLayout;
  extern __shared__ uint8_t sqdk_bwd_smem_raw[];
  __shared__ __align__(8) uint64_t bar_kv, bar_qfull[kBwdStages], bar_qempty[kBwdStages], bar_sfull[2], bar_pfull[2];
  __shared__ __align__(8) uint64_t bar_dqfull[2], bar_setfree[2], bar_final, bar_drain;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int first_block_sh, nblk_sh;
  // per-row block data: position (-1 = no query), -lse in log2 units, -Delta
  // (negated so the softmax adds them with packed f32x2 instructions), and
  // whether every row of the block sees all 128 keys (no causal mask)
  __shared__ __align__(16) int info_pos[kBwdInfo][kBwdRows];
  __shared__ __align__(16) float info_nlse2[kBwdInfo][kBwdRows];
  __shared__ __align__(16) float info_ndelta[kBwdInfo][kBwdRows];
  __shared__ int info_full[kBwdInfo];
  __shared__ volatile uint32_t abort_flag;

  const uint32_t sbase = (smem_u32(sqdk_bwd_smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kb, b, g;
  sqdk_bwd_coords(p, static_cast<int>(blockIdx.x), kb, b, g);
  const int n0 = kb * kBwdKeys;
  const int nqb = (p.K + p.QTb - 1) / p.QTb;  // query blocks of the whole sequence

  if (threadIdx.x == 0) {
    mbar_init(&bar_kv, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&bar_qfull[s], 1);
      mbar_init(&bar_qempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_sfull[s], 1);
      mbar_init(&bar_pfull[s], kBwdSoftmaxArrivals);
      mbar_init(&bar_dqfull[s], 1);
      mbar_init(&bar_setfree[s], 4);
    }
    mbar_init(&bar_final, 1);
    mbar_init(&bar_drain, 1);
    abort_flag = 0u;
    fence_mbar_init();
    // K and V of the key block do not depend on the query range: their loads
    // start before the search below (drained before exit even if no query
    // block turns out to see these keys)
    mbar_arrive_expect_tx(&bar_kv, 2 * L::kKVBytes);
    for (int c = 0; c < L::kChunks; ++c) {
      tma_load_4d(sbase + L::kKOff + c * L::kKVChunkBytes, &tmK, &bar_kv, c * 64, g, n0, b);
      tma_load_4d(sbase + L::kVOff + c * L::kKVChunkBytes, &tmV, &bar_kv, c * 64, g, n0, b);
    }
  }
  if (warp == 0) {
    // First query whose position reaches n0 (positions ascend along the row):
    // a 32-way search, each round one load per lane over an interval 32 times
    // shorter than the last (two rounds for a thousand queries instead of ten
    // dependent loads). The answer stays in [lo, hi].
    const int64_t* ib = p.idx + static_cast<int64_t>(b) * p.idx_sb;
    int lo = 0, hi = p.K;
    while (lo < hi) {
      const int step = (hi - lo + 31) / 32;
      const int at = lo + lane * step;
      const bool below = at < hi && __ldg(ib + static_cast<int64_t>(at) * p.idx_sk) < n0;
      const int c = __popc(__ballot_sync(0xFFFFFFFFu, below));
      if (c == 0) break;  // idx[lo] >= n0
      const int nlo = lo + (c - 1) * step + 1;
      hi = min(hi, lo + c * step);
      lo = nlo;
    }
    if (lane == 0) {
      first_block_sh = lo / p.QTb;
      nblk_sh = lo < p.K ? nqb - lo / p.QTb : 0;
      // the first query block's Q / dO are requested now (bytes expected, no
      // arrival): the producer arrives once the block's row data is written,
      // so the stage cannot complete before the softmax may read that data
      if (lo < p.K) {
        mbar_expect_tx(&bar_qfull[0], static_cast<uint32_t>(2 * L::kChunks * p.G * p.QTb * 128));
        for (int c = 0; c < L::kChunks; ++c) {
          tma_load_4d(sbase + L::kQOff + c * L::kRowChunkBytes, &tmQ, &bar_qfull[0], c * 64, g * p.G,
                      (lo / p.QTb) * p.QTb, b);
          tma_load_4d(sbase + L::kDOOff + c * L::kRowChunkBytes, &tmDO, &bar_qfull[0], c * 64, g * p.G,
                      (lo / p.QTb) * p.QTb, b);
        }
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, L::kTmemCols);
    tmem_relinquish();
  }
  // rows of the query tiles past G * QTb are never written by TMA: zero them
  // once, so the row sums of dV / dK see exact zeros there
  {
    const int used = p.G * p.QTb;
    if (used < kBwdRows) {
      for (int i = threadIdx.x; i < 2 * kBwdStages * L::kChunks * (kBwdRows - used) * 8; i += kBwdThreads) {
        const int unit = i & 7;
        int rest = i >> 3;
        const int row = used + rest % (kBwdRows - used);
        rest /= (kBwdRows - used);
        const int c = rest % L::kChunks;
        rest /= L::kChunks;
        const int s = rest % kBwdStages;
        const int which = rest / kBwdStages;  // 0 = Q, 1 = dO
        const uint32_t a =
            sbase + (which ? L::kDOOff : L::kQOff) + s * L::kRowBytes + c * L::kRowChunkBytes + row * 128 + unit * 16;
        st_shared_v4(a, make_uint4(0u, 0u, 0u, 0u));
      }
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int jb0 = first_block_sh, nblk = nblk_sh;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int nq = 0;
    bool live = true;
    // Row data of query block qb (two rows per lane): the raw position, the
    // position before it, lse and Delta. Nothing here uses the loaded values:
    // they are consumed (checked, converted, written to the ring) one
    // iteration later, so the load latency never stalls the producer.
    struct Rows {
      int64_t ps[2], prev[2];
      float lse[2], dl[2];
      bool valid[2], first[2];
    };
    auto load_rows = [&](int qb, Rows& r) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = lane + 32 * u;
        const int qloc = c / p.G;
        const int qi = qb * p.QTb + qloc;
        r.valid[u] = qloc < p.QTb && qi < p.K;
        // the key block's first query came from a binary search over the
        // row, which needs ascending positions; the key block at 0 visits
        // every query block, so every row is checked by some CTA
        r.first[u] = r.valid[u] && qi > 0 && c - qloc * p.G == 0;
        r.ps[u] = -1;
        r.prev[u] = -1;
        r.lse[u] = 0.0f;
        r.dl[u] = 0.0f;
        if (r.valid[u]) {
          const int64_t* ib = p.idx + static_cast<int64_t>(b) * p.idx_sb + static_cast<int64_t>(qi) * p.idx_sk;
          r.ps[u] = __ldg(ib);
          if (r.first[u]) r.prev[u] = __ldg(ib - p.idx_sk);
          const int64_t ro =
              static_cast<int64_t>(b) * p.row_sb + static_cast<int64_t>(qi) * p.row_sk + g * p.G + (c - qloc * p.G);
          r.lse[u] = __ldg(p.lse + ro);
          r.dl[u] = __ldg(p.delta + ro);
        }
      }
    };
    // The row data of block j + 1 is loaded while block j waits for its
    // stage, and written to the ring before block j + 1's wait: slot j % 4 was
    // last read by the softmax of block j - 4, which finished before the dK /
    // dV products of that block, whose completion freed the stage the
    // producer waited for in iteration j - 1.
    Rows rows;
    if (nblk > 0) load_rows(jb0, rows);
    for (int j = 0; j < nblk; ++j) {
      const int s = j % kBwdStages;
      const int slot = j & (kBwdInfo - 1);
      const int qb = jb0 + j;
      bool sees_all = true;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = lane + 32 * u;
        const int64_t ps = rows.ps[u];
        if (rows.first[u] && ps < rows.prev[u]) raise_device_error(HSPMN_DEVERR_UNSORTED);
        const int pos = (!rows.valid[u] || ps < 0 || ps >= p.S) ? -1 : static_cast<int>(ps);
        sees_all = sees_all && pos >= n0 + kBwdKeys - 1;
        info_pos[slot][c] = pos;
        info_nlse2[slot][c] = -(rows.lse[u] * 1.4426950408889634f);
        info_ndelta[slot][c] = -rows.dl[u];
      }
      sees_all = __all_sync(0xFFFFFFFFu, sees_all);
      if (lane == 0) info_full[slot] = sees_all ? 1 : 0;
      if (j + 1 < nblk) load_rows(qb + 1, rows);
      if (j >= kBwdStages) {
        bool okw = true;
        if (lane == 0) okw = mbar_wait(&bar_qempty[s], ((j - kBwdStages) / kBwdStages) & 1, &abort_flag);
        live = __shfl_sync(0xFFFFFFFFu, okw ? 1 : 0, 0) != 0;
        if (!live) break;
      }
      __syncwarp();
      if (lane == 0 && j == 0) {
        mbar_arrive(&bar_qfull[0]);  // its loads were issued at setup
      } else if (lane == 0) {
        mbar_arrive_expect_tx(&bar_qfull[s], static_cast<uint32_t>(2 * L::kChunks * p.G * p.QTb * 128));
        for (int c = 0; c < L::kChunks; ++c) {
          tma_load_4d(sbase + L::kQOff + s * L::kRowBytes + c * L::kRowChunkBytes, &tmQ, &bar_qfull[s], c * 64,
                      g * p.G, qb * p.QTb, b);
          tma_load_4d(sbase + L::kDOOff + s * L::kRowBytes + c * L::kRowChunkBytes, &tmDO, &bar_qfull[s], c * 64,
                      g * p.G, qb * p.QTb, b);
        }
      }
      ++nq;
    }
    if (lane == 0) {
      mbar_wait_drain(&bar_kv, 0);
      // the last load issued into each stage
      for (int s = 0; s < kBwdStages; ++s) {
        if (nq <= s) continue;
        const int last = s + ((nq - 1 - s) / kBwdStages) * kBwdStages;
        mbar_wait_drain(&bar_qfull[s], (last / kBwdStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // The warp runs the issue loop converged (operands stay warp-uniform,
    // which makes each tcgen05.mma much cheaper to issue than from a lone
    // lane); one elected lane issues every product and commit.
    if (nblk > 0) {
      constexpr int kAB = kBF16 ? 1 : 0;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBwdKeys, kBwdRows, kAB, false, false);
      constexpr uint32_t idesc_kv = umma_idesc_f16(kBwdKeys, kBwdHD, kAB, false, true);
      constexpr uint32_t idesc_q = umma_idesc_f16(kBwdHD, kBwdRows, kAB, true, true);
      const uint64_t kdesc = sw128_desc(sbase + L::kKOff, 16, 1024);
      const uint64_t vdesc = sw128_desc(sbase + L::kVOff, 16, 1024);
      const uint64_t qdesc = sw128_desc(sbase + L::kQOff, 16, 1024);
      const uint64_t dodesc = sw128_desc(sbase + L::kDOOff, 16, 1024);
      // the same Q / dO tiles read MN-major (N = hd in 64-column chunks, K = rows)
      const uint64_t qdesc_mn = sw128_desc(sbase + L::kQOff, L::kRowChunkBytes, 1024);
      const uint64_t dodesc_mn = sw128_desc(sbase + L::kDOOff, L::kRowChunkBytes, 1024);
      // K read MN-major as the A of dQ^T (M = hd in 64-column chunks, K = keys)
      const uint64_t kdesc_mn = sw128_desc(sbase + L::kKOff, L::kKVChunkBytes, 1024);
      const uint64_t dsdesc = sw128_desc(sbase + L::kDSOff, L::kDSBytes, 1024);
      bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_kv, 0, &abort_flag));
      tc_fence_after();
      auto issue_rest = [&](int jj) -> bool {
        const int set = jj & 1, st = jj % kBwdStages;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar_pfull[set], (jj >> 1) & 1, &abort_flag))) return false;
        tc_fence_after();
        const uint32_t tS = tmem + set * L::kSetCols;
        const uint64_t rowoff = static_cast<uint64_t>((st * L::kRowBytes) >> 4);
        // dQ^T first, with its own commit: the dQ warps read it out of the
        // dP^T columns while dV and dK run, so the next block but one can
        // take those columns as soon as the pipe reaches it
        const uint64_t dsoff = static_cast<uint64_t>((set * L::kDSBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBwdKeys / 16; ++kk) {
          const uint64_t step = static_cast<uint64_t>((kk * 16 * 128) >> 4);
          umma_ss_warp(tS + 64, kdesc_mn + step, dsdesc + dsoff + step, idesc_q, kk > 0 ? 1u : 0u);
        }
        umma_commit_warp(&bar_dqfull[set]);
#pragma unroll
        for (int kk = 0; kk < kBwdRows / 16; ++kk) {
          const uint64_t step = static_cast<uint64_t>((kk * 16 * 128) >> 4);
          // rows 16 kk .. 16 kk + 15 of P^T: group kk / 2's columns [0, 16)
          umma_ts_warp(tmem + L::kDVCol, tS + (kk >> 1) * 32 + (kk & 1) * 8, dodesc_mn + rowoff + step, idesc_kv,
                       (jj > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < kBwdRows / 16; ++kk) {
          const uint64_t step = static_cast<uint64_t>((kk * 16 * 128) >> 4);
          // and of dS^T: group kk / 2's columns [16, 32)
          umma_ts_warp(tmem + L::kDKCol, tS + (kk >> 1) * 32 + 16 + (kk & 1) * 8, qdesc_mn + rowoff + step, idesc_kv,
                       (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_warp(&bar_qempty[st]);
        return true;
      };
      for (int j = 0; ok && j < nblk; ++j) {
        const int set = j & 1, st = j % kBwdStages;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar_qfull[st], (j / kBwdStages) & 1, &abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tS = tmem + set * L::kSetCols;
        const uint64_t rowoff = static_cast<uint64_t>((st * L::kRowBytes) >> 4);
        // S^T into this set's first 64 columns, whose P^T / dS^T of block j-2
        // the dV / dK products issued before it have read
#pragma unroll
        for (int kk = 0; kk < kBwdHD / 16; ++kk) {
          const int c = kk >> 2, w = kk & 3;
          const uint64_t ka = static_cast<uint64_t>((c * L::kKVChunkBytes + w * 32) >> 4);
          const uint64_t qa = rowoff + static_cast<uint64_t>((c * L::kRowChunkBytes + w * 32) >> 4);
          umma_ss_warp(tS, kdesc + ka, qdesc + qa, idesc_s, kk > 0 ? 1u : 0u);
        }
        // dP^T goes where the dQ^T of block j-2 is: wait until it has been read
        if (j >= 2 && !__all_sync(0xFFFFFFFFu, mbar_wait(&bar_setfree[set], ((j - 2) >> 1) & 1, &abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBwdHD / 16; ++kk) {
          const int c = kk >> 2, w = kk & 3;
          const uint64_t va = static_cast<uint64_t>((c * L::kKVChunkBytes + w * 32) >> 4);
          const uint64_t da = rowoff + static_cast<uint64_t>((c * L::kRowChunkBytes + w * 32) >> 4);
          umma_ss_warp(tS + 64, vdesc + va, dodesc + da, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit_warp(&bar_sfull[set]);
        if (j >= 1 && !issue_rest(j - 1)) ok = false;
      }
      if (ok) ok = issue_rest(nblk - 1);
      if (ok) umma_commit_warp(&bar_final);
      umma_commit_warp(&bar_drain);
      if (lane == 0) mbar_wait_drain(&bar_drain, 0);
      __syncwarp();
    }
  } else if (warp < 6 || warp >= 10) {
    // ------------------------------------------------------------ P^T, dS^T
    const int grp = warp >= 10 ? 1 : 0;    // rows 32 grp .. 32 grp + 31
    const int kr = 32 * (warp & 3) + lane;  // key row = TMEM lane
    const int n = n0 + kr;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
    bool ok = nblk > 0;
    // P^T and dS^T / scale of four rows c .. c + 3 from S^T and dP^T, two rows
    // per packed f32x2 instruction; kMask applies the causal mask and drops
    // rows without a query (blocks whose rows all see every key skip it). The
    // softmax scale of dS is applied to dK and dQ in fp32 after the products.
    // Each lane holds the row data of row 32 grp + lane and the rows reach
    // the other lanes by shuffles, which return sooner than the broadcast
    // 16-byte shared loads they replace (fewer long-scoreboard stalls on the
    // softmax's critical path; the load/store pipe sees as many wavefronts).
    float my_nl = 0.0f, my_nd = 0.0f;
    auto rows4 = [&](auto kMaskTag, const uint32_t (&sv)[32], const uint32_t (&dv)[32], int o, int c, int slot,
                     uint32_t& p01, uint32_t& p23, uint32_t& d01, uint32_t& d23) {
      constexpr bool kMask = decltype(kMaskTag)::value;
      const float4 nl = make_float4(__shfl_sync(0xFFFFFFFFu, my_nl, o), __shfl_sync(0xFFFFFFFFu, my_nl, o + 1),
                                    __shfl_sync(0xFFFFFFFFu, my_nl, o + 2), __shfl_sync(0xFFFFFFFFu, my_nl, o + 3));
      const float4 nd = make_float4(__shfl_sync(0xFFFFFFFFu, my_nd, o), __shfl_sync(0xFFFFFFFFu, my_nd, o + 1),
                                    __shfl_sync(0xFFFFFFFFu, my_nd, o + 2), __shfl_sync(0xFFFFFFFFu, my_nd, o + 3));
      float x0, x1, x2, x3;
      f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[o]), __uint_as_float(sv[o + 1])), c2, f2_pack(nl.x, nl.y)), x0, x1);
      f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[o + 2]), __uint_as_float(sv[o + 3])), c2, f2_pack(nl.z, nl.w)), x2,
                x3);
      float e0 = fast_exp2(x0), e1 = fast_exp2(x1), e2 = fast_exp2(x2), e3 = fast_exp2(x3);
      if constexpr (kMask) {
        const int my_ps = info_pos[slot][c - o + lane];
        const int4 ps = make_int4(__shfl_sync(0xFFFFFFFFu, my_ps, o), __shfl_sync(0xFFFFFFFFu, my_ps, o + 1),
                                  __shfl_sync(0xFFFFFFFFu, my_ps, o + 2), __shfl_sync(0xFFFFFFFFu, my_ps, o + 3));
        e0 = n <= ps.x ? e0 : 0.0f;
        e1 = n <= ps.y ? e1 : 0.0f;
        e2 = n <= ps.z ? e2 : 0.0f;
        e3 = n <= ps.w ? e3 : 0.0f;
      }
      float g0, g1, g2, g3;
      f2_unpack(f2_mul(f2_pack(e0, e1),
                       f2_add(f2_pack(__uint_as_float(dv[o]), __uint_as_float(dv[o + 1])), f2_pack(nd.x, nd.y))),
                g0, g1);
      f2_unpack(f2_mul(f2_pack(e2, e3),
                       f2_add(f2_pack(__uint_as_float(dv[o + 2]), __uint_as_float(dv[o + 3])), f2_pack(nd.z, nd.w))),
                g2, g3);
      p01 = pack2<kBF16>(e0, e1);
      p23 = pack2<kBF16>(e2, e3);
      d01 = pack2<kBF16>(g0, g1);
      d23 = pack2<kBF16>(g2, g3);
    };
    for (int j = 0; ok && j < nblk; ++j) {
      const int set = j & 1, slot = j & (kBwdInfo - 1);
      // the row data of this block (written by the producer before its
      // arrival) and the S^T / dP^T of this block
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_qfull[j % kBwdStages], (j / kBwdStages) & 1, &abort_flag) &&
                                       mbar_wait(&bar_sfull[set], (j >> 1) & 1, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + set * L::kSetCols;
      uint32_t pp[16], dd[16];
      {
        uint32_t sr[32], dr[32];
        tmem_ld32(tS + 32 * grp, sr);
        tmem_ld32(tS + 64 + 32 * grp, dr);
        tmem_wait_ld();
        my_nl = info_nlse2[slot][32 * grp + lane];
        my_nd = info_ndelta[slot][32 * grp + lane];
        if (info_full[slot]) {
#pragma unroll
          for (int o = 0; o < 32; o += 4)
            rows4(std::false_type{}, sr, dr, o, 32 * grp + o, slot, pp[o >> 1], pp[(o >> 1) + 1], dd[o >> 1],
                  dd[(o >> 1) + 1]);
        } else {
#pragma unroll
          for (int o = 0; o < 32; o += 4)
            rows4(std::true_type{}, sr, dr, o, 32 * grp + o, slot, pp[o >> 1], pp[(o >> 1) + 1], dd[o >> 1],
                  dd[(o >> 1) + 1]);
        }
      }
      // [P^T | dS^T] of the group's 32 rows into the S^T columns it read
      tmem_st16(tS + 32 * grp, pp);
      tmem_st16(tS + 32 * grp + 16, dd);
      // the group's half of this key's dS^T row in the MN-major B tile of
      // dQ^T: 128 bytes per key, 16-byte units XOR-swizzled by key % 8
      const uint32_t rowb = sbase + L::kDSOff + set * L::kDSBytes + kr * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        st_shared_v4(rowb + (((4 * grp + u) ^ (kr & 7)) << 4),
                     make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]));
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_pfull[set]);
    }
    // ------------------------------------------------------------ dV (group 0) / dK (group 1)
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_final, 0, &abort_flag));
    // The group's 128 x 128 accumulator goes through shared memory (the Q
    // ring, idle once every product has completed) in the 128-byte-swizzled
    // layout of the K / V tiles, one 16 KB tile per 64 columns, and out with
    // one TMA store per tile (keys past S and columns past hd are clipped by
    // the tensor map). Storing each key's row straight from registers would
    // write 16-byte pieces of 128 rows 1 KB apart. The TMEM loads are
    // warp-collective: every lane runs them.
    if (ok || nblk == 0) {
      tc_fence_after();
      const uint32_t tcol = tmem + lane_base + (grp ? L::kDKCol : L::kDVCol);
      const float f = grp ? p.scale : 1.0f;
      const uint32_t stg = sbase + L::kQOff + grp * L::kKVBytes;
#pragma unroll 1
      for (int c = 0; c < kBwdHD; c += 32) {
        uint32_t rr[32];
        if (nblk > 0) {
          tmem_ld32(tcol + c, rr);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = 0u;
        }
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int col = c + 8 * v;
          uint4 w;
          w.x = pack2<kBF16>(__uint_as_float(rr[8 * v + 0]) * f, __uint_as_float(rr[8 * v + 1]) * f);
          w.y = pack2<kBF16>(__uint_as_float(rr[8 * v + 2]) * f, __uint_as_float(rr[8 * v + 3]) * f);
          w.z = pack2<kBF16>(__uint_as_float(rr[8 * v + 4]) * f, __uint_as_float(rr[8 * v + 5]) * f);
          w.w = pack2<kBF16>(__uint_as_float(rr[8 * v + 6]) * f, __uint_as_float(rr[8 * v + 7]) * f);
          const int unit = (col & 63) >> 3;
          st_shared_v4(stg + (col >> 6) * L::kKVChunkBytes + kr * 128 + ((unit ^ (kr & 7)) << 4), w);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(kBwdEpiBar + grp, 128);
      if ((warp & 3) == 2 && lane == 0) {
        for (int ch = 0; ch < L::kChunks && ch * 64 < p.hd; ++ch)
          tma_store_4d(grp ? &tmDK : &tmDV, stg + ch * L::kKVChunkBytes, ch * 64, g, n0, b);
        tma_store_commit();
        tma_store_wait_read();
      }
    }
  } else {
    // ------------------------------------------------------------ dQ
    const int d = 32 * (warp & 3) + lane;  // head-dim column = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    bool ok = nblk > 0;
    for (int j = 0; ok && j < nblk; ++j) {
      const int set = j & 1;
      // the four dQ warps agree on the wait's outcome, so all of them take the
      // named barriers below the same number of times
      ok = named_bar_and(kBwdDQBar, 128, mbar_wait(&bar_dqfull[set], (j >> 1) & 1, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t tQ = tmem + lane_base + set * L::kSetCols + 64;
      tmem_ld32(tQ, r0);
      tmem_ld32(tQ + 32, r1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_setfree[set]);
      // one 64-column chunk at a time through the staging tile: the two warps
      // holding the chunk's columns write it (a warp writes 32 consecutive
      // floats of a row at a time), one thread issues its bulk reduce
      const uint32_t col = sbase + L::kDQOff + (d & 63) * 4;
      for (int ch = 0; ch < L::kChunks && ch * 64 < p.hd; ++ch) {
        // the previous reduce has read the staging tile
        if (warp == 6 && lane == 0) tma_store_wait_read();
        named_bar_sync(kBwdDQBar, 128);
        if ((d >> 6) == ch) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(col + c * 256), "r"(r0[c]) : "memory");
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(col + (c + 32) * 256), "r"(r1[c]) : "memory");
          }
          fence_proxy_async_smem();
        }
        named_bar_sync(kBwdDQBar, 128);
        if (warp == 6 && lane == 0) {
          // rows past the K selected queries are clipped by the tensor map
          tma_reduce_add_4d(&tmDQ, sbase + L::kDQOff, ch * 64, g * p.G, (jb0 + j) * p.QTb, b);
          tma_store_commit();
        }
      }
    }
    if (warp == 6 && lane == 0) tma_store_wait_read();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// Delta[b,i,h] = sum_d dO[b,i,h,d] * O[b,i,h,d] in fp32 (one warp per row).
template <typename T>
__global__ void __launch_bounds__(256) sqdk_bwd_delta_kernel(const T* __restrict__ o, int64_t o_sb, int64_t o_sk,
                                                            int64_t o_sh, const T* __restrict__ d_o, int64_t do_sb,
                                                            int64_t do_sk, int64_t do_sh, float* __restrict__ delta,
                                                            int B, int K, int H, int hd) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(B) * K * H;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t b = r / (static_cast<int64_t>(K) * H);
    const int64_t rem = r - b * K * H;
    const int64_t i = rem / H, h = rem - i * H;
    const T* orow = o + b * o_sb + i * o_sk + h * o_sh;
    const T* drow = d_o + b * do_sb + i * do_sk + h * do_sh;
    float acc = 0.0f;
    for (int c = lane; c < hd; c += 32) acc = fmaf(static_cast<float>(orow[c]), static_cast<float>(drow[c]), acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0) delta[r] = acc;
  }
}

// scale x dq (fp32 accumulator of K^T (dS / scale), dense [B,K,H,hd]) -> the
// caller's dtype and strides.
template <typename T>
__global__ void __launch_bounds__(256) sqdk_bwd_dq_cast_kernel(const float* __restrict__ acc, T* __restrict__ dq,
                                                              int64_t sb, int64_t sk, int64_t sh, int B, int K, int H,
                                                              int hd, float scale) {
  const int64_t n = static_cast<int64_t>(B) * K * H * hd;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * 256) {
    int64_t rest = e;
    const int64_t d = rest % hd;
    rest /= hd;
    const int64_t h = rest % H;
    rest /= H;
    const int64_t i = rest % K;
    const int64_t b = rest / K;
    dq[b * sb + i * sk + h * sh + d] = static_cast<T>(acc[e] * scale);
  }
}

}  // namespace hspmn
