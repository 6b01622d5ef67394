// Sparse-query dense-key causal attention on tcgen05 / TMEM / TMA (sm_100a).
//
// Replaces _sqdk_fwd_kernel (kernels_v2_1.py:11-139) with the grouped-head
// semantics of the reference's Flex path (hspmn_v2_1.py:212).
//
// Head dims up to 128 (multiples of 8) run on a 64- or 128-wide tile: the TMA
// boxes are always 64 columns wide and zero-fill the columns past head_dim,
// which add nothing to Q K^T and produce zero O columns that are not stored.
//
// Work unit ("tile"): one sequence b, one K/V head g and QT = 128 / G
// consecutive selected queries together with the G query heads that read
// head g, i.e. 128 rows (query, head) that all share the same K/V blocks.
// Rows are ordered r = q * G + h, exactly the order a TMA box over the
// [B,K,H,hd] query tensor lands in shared memory.
//
// Per tile the key loop runs over 64-key blocks up to the largest position in
// the tile (indices are sorted, so tiles near the end of the sequence are the
// long ones and are launched first). Each block:
//   S  = Q K^T        tcgen05.mma SS, M=128 N=64 K=hd, S in TMEM (2 buffers)
//   P  = exp2(S*c - m) softmax warps: one thread per row, TMEM -> registers,
//                     causal mask on the diagonal blocks, P written back to
//                     TMEM as bf16/f16 over the S buffer it came from
//   O += P V          tcgen05.mma TS, A = P from TMEM, B = V (MN-major smem)
// O stays in TMEM for the whole tile. A block is first exponentiated against
// the row's running maximum m without computing the block's own maximum:
// softmax is exact for any m as long as nothing overflows, and the block's
// row sum (needed anyway) bounds every term. Only a row's first block, or a
// block whose sum exceeds the bound (the maximum grew a lot), takes the exact
// path: block maximum, O and l rescaled, P recomputed.
//
// Warp roles (192 threads, two CTAs per SM):
//   warp 0      TMA producer: Q once, then K and V through 2-stage rings,
//               K_{j+1} requested ahead of V_j
//   warp 1      TMEM allocation + MMA issue: per block, Q K^T of block j,
//               one commit, P V of block j-1. The warp runs the issue loop
//               converged and one elected lane issues (operands stay
//               warp-uniform, so each product costs its issuer far fewer
//               cycles); it waits and commits as little as the ordering
//               allows, since its steps per block bound the pipeline
//   warps 2..5  softmax, lazy O correction, epilogue (row = TMEM lane): O / l
//               staged in the freed Q tile, stored by one thread with TMA
// Every mbarrier wait is bounded (common.cuh); a wait that gives up flags
// HSPMN_DEVERR_TIMEOUT, tells the other roles to stop, drains what this CTA
// has in flight and frees its tensor memory before returning.
#pragma once

#include "common.cuh"

namespace hspmn {

constexpr int kSqdkBM = 128;       // rows per tile
constexpr int kSqdkBN = 64;        // keys per block
constexpr int kSqdkStages = 2;     // depth of the K ring and of the V ring
constexpr int kSqdkThreads = 192;  // 6 warps
// Largest row sum of one block accepted without an exact row maximum: every
// p of the row is below it, so P stays finite in bf16 (and below 65504 in
// f16) and O = sum(P V) in fp32 cannot overflow.
template <bool kBF16>
constexpr float kSqdkSumBound = kBF16 ? 1048576.0f : 32768.0f;
constexpr int kSqdkPairGroup = 16;  // (sequence, kv-head) pairs scheduled together (16 beat 4, 8 and 32)
constexpr int kSqdkEpilogueBar = 1;  // named barrier of the four softmax warps
constexpr int kSqdkLongRange = 32;   // key blocks from which P V goes without its own commit

template <int HD>
struct SqdkLayout {
  static constexpr int kChunks = HD / 64;                    // 128-byte column chunks per row
  static constexpr int kQChunkBytes = kSqdkBM * 128;         // 16 KB
  static constexpr int kKVChunkBytes = kSqdkBN * 128;        // 8 KB
  static constexpr int kKVBytes = kChunks * kKVChunkBytes;   // one K or V block
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kChunks * kQChunkBytes;
  static constexpr int kVOff = kKOff + kSqdkStages * kKVBytes;
  static constexpr int kBytes = kVOff + kSqdkStages * kKVBytes;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
  static constexpr uint32_t kTmemCols = 256;    // S0 | S1 | O
  static constexpr int kOCol = 2 * kSqdkBN;
  static_assert(kOCol + HD <= static_cast<int>(kTmemCols), "TMEM budget");
};

struct SqdkParams {
  const int64_t* idx;
  int hd;      // real head_dim (<= the padded tile width HD)
  int nsplit;  // CTAs per tile, each over a contiguous share of the tile's key blocks
  float* part_o;   // nsplit > 1: [tile*nsplit + split][128][HD] unnormalised fp32 O
  float* part_ml;  // nsplit > 1: [tile*nsplit + split][128][2] running max (log2 units), row sum
  int64_t idx_sb, idx_sk;
  void* o;
  int64_t o_sb, o_sk, o_sh;  // elements
  int B, K, S, H, Hkv, G, QT, T;
  float scale_log2;
  float* lse;  // optional [B,K,H] (strides lse_sb, lse_sk, 1): natural-log log-sum-exp of each row's scores
  int64_t lse_sb, lse_sk;
};

constexpr float kLn2 = 0.69314718055994531f;

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Wait used only while tearing down: ignores the abort flag, keeps the limit.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < kWaitLimitIters; ++it) {
    if (mbar_try_wait(bar, parity)) return;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  raise_device_error(HSPMN_DEVERR_TIMEOUT);
}

// Tile index -> (query tile t, sequence b, kv head g): (sequence, kv-head)
// pairs in groups of kSqdkPairGroup so the K/V blocks a group streams stay in
// L2; inside a group the longest query tiles (highest t) come first.
__device__ __forceinline__ void sqdk_tile_coords(const SqdkParams& p, int tile, int& t, int& b, int& g) {
  const int BG = p.B * p.Hkv;
  const int grp = tile / (kSqdkPairGroup * p.T);
  const int in_grp = tile - grp * kSqdkPairGroup * p.T;
  const int npairs = min(kSqdkPairGroup, BG - grp * kSqdkPairGroup);
  t = p.T - 1 - in_grp / npairs;
  const int bg = grp * kSqdkPairGroup + in_grp % npairs;
  b = bg / p.Hkv;
  g = bg % p.Hkv;
}

template <int HD, bool kBF16>
__global__ void __launch_bounds__(kSqdkThreads, 2)
    sqdk_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const SqdkParams p) {
  using L = SqdkLayout<HD>;
  extern __shared__ uint8_t sqdk_smem_raw[];
  __shared__ __align__(8) uint64_t bar_q;
  // One thread issues every MMA, and they complete in issue order, so
  // bar_sfull[j & 1] completing (Q K^T of block j done) also means P V of
  // block j-2 is done: K stage j % 2 (read by that Q K^T) is free again, and
  // on long key ranges V stage j % 2 (read by that P V) too. There P V needs
  // no commit of its own except the second-to-last (bar_vempty[0], which no
  // later Q K^T follows); short ranges, where requesting V after Q K^T rather
  // than after P V costs more than the commit, keep one per P V.
  static_assert(kSqdkStages == 2, "the K and V rings reuse the S-buffer barriers");
  __shared__ __align__(8) uint64_t bar_kfull[kSqdkStages];
  __shared__ __align__(8) uint64_t bar_vfull[kSqdkStages], bar_vempty[kSqdkStages];
  __shared__ __align__(8) uint64_t bar_sfull[2], bar_pfull[2];
  __shared__ __align__(8) uint64_t bar_ofinal, bar_drain;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int warp_maxpos[4];  // largest query position seen by each softmax warp
  __shared__ volatile uint32_t abort_flag;

  const uint32_t sbase = (smem_u32(sqdk_smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int item = static_cast<int>(blockIdx.x);
  const int split = item % p.nsplit;
  int t, b, g;
  sqdk_tile_coords(p, item / p.nsplit, t, b, g);

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < kSqdkStages; ++s) {
      mbar_init(&bar_kfull[s], 1);
      mbar_init(&bar_vfull[s], 1);
      mbar_init(&bar_vempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_sfull[s], 1);
      mbar_init(&bar_pfull[s], 4);  // one arrival per softmax warp
    }
    mbar_init(&bar_ofinal, 1);
    mbar_init(&bar_drain, 1);
    abort_flag = 0u;
    fence_mbar_init();
    if (p.nsplit == 1) {
      // an unsplit tile starts at key block 0 whatever its positions: this
      // thread (the producer) requests Q and K_0 now, so their latency
      // overlaps the index loads and the barrier below
      mbar_arrive_expect_tx(&bar_q, static_cast<uint32_t>(L::kChunks * p.G * p.QT * 128));
      for (int c = 0; c < L::kChunks; ++c)
        tma_load_4d(sbase + L::kQOff + c * L::kQChunkBytes, &tmQ, &bar_q, c * 64, g * p.G, t * p.QT, b);
      mbar_arrive_expect_tx(&bar_kfull[0], L::kKVBytes);
      for (int c = 0; c < L::kChunks; ++c)
        tma_load_4d(sbase + L::kKOff + c * L::kKVChunkBytes, &tmK, &bar_kfull[0], c * 64, g, 0, b);
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, L::kTmemCols);
    tmem_relinquish();
  }

  // softmax rows: which (query, head) this thread owns and its position
  int pos = -1, qi = 0, hh = 0;
  bool row_valid = false;
  if (warp >= 2) {
    const int r = 32 * (warp & 3) + lane;
    const int qloc = r / p.G;
    qi = t * p.QT + qloc;
    hh = g * p.G + (r - qloc * p.G);
    if (qloc < p.QT && qi < p.K) {
      int64_t ps = __ldg(p.idx + static_cast<int64_t>(b) * p.idx_sb + static_cast<int64_t>(qi) * p.idx_sk);
      row_valid = true;
      if (ps < 0 || ps >= p.S) {
        raise_device_error(HSPMN_DEVERR_POSITION);
        ps = ps < 0 ? -1 : p.S - 1;
      }
      pos = static_cast<int>(ps);
    }
    const int wmax = __reduce_max_sync(0xFFFFFFFFu, pos);
    if (lane == 0) warp_maxpos[warp & 3] = wmax;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  // this CTA's share of the tile's key blocks: [j0, j0 + nblk). Every CTA of
  // a tile derives the same tile_blocks from the same positions.
  const int tile_maxpos = max(max(warp_maxpos[0], warp_maxpos[1]), max(warp_maxpos[2], warp_maxpos[3]));
  const int tile_blocks = tile_maxpos < 0 ? 0 : tile_maxpos / kSqdkBN + 1;
  const int per_split = (tile_blocks + p.nsplit - 1) / p.nsplit;
  const int j0 = split * per_split;
  const int nblk = max(0, min(tile_blocks, j0 + per_split) - j0);
  const bool long_range = nblk >= kSqdkLongRange;  // same for every role of the CTA

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const bool early = p.nsplit == 1;  // Q and K_0 already requested in the prologue
    if (lane == 0 && nblk > 0) {
      if (!early) {
        mbar_arrive_expect_tx(&bar_q, static_cast<uint32_t>(L::kChunks * p.G * p.QT * 128));
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sbase + L::kQOff + c * L::kQChunkBytes, &tmQ, &bar_q, c * 64, g * p.G, t * p.QT, b);
      }
      // K runs one block ahead of V: K_{j+1} is requested (once Q K^T of
      // block j-1 has freed its stage) before V_j, so a K block never waits
      // behind a V stage that P V of an older block still holds.
      int nk = early ? 1 : 0, nv = 0;
      auto load_k = [&](int j) -> bool {
        const int s = j % kSqdkStages, r = j / kSqdkStages;
        if (r > 0 && !mbar_wait(&bar_sfull[s], (r - 1) & 1, &abort_flag)) return false;
        mbar_arrive_expect_tx(&bar_kfull[s], L::kKVBytes);
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sbase + L::kKOff + s * L::kKVBytes + c * L::kKVChunkBytes, &tmK, &bar_kfull[s], c * 64, g,
                      (j0 + j) * kSqdkBN, b);
        ++nk;
        return true;
      };
      bool live = early || load_k(0);
      for (int j = 0; live && j < nblk; ++j) {
        if (j + 1 < nblk && !load_k(j + 1)) break;
        const int s = j % kSqdkStages, r = j / kSqdkStages;
        // stage s held V_{j-2}: free once its P V is done (or Q K^T of block j, issued after it)
        if (r > 0 && !(long_range ? mbar_wait(&bar_sfull[s], r & 1, &abort_flag)
                                  : mbar_wait(&bar_vempty[s], (r - 1) & 1, &abort_flag)))
          break;
        mbar_arrive_expect_tx(&bar_vfull[s], L::kKVBytes);
        for (int c = 0; c < L::kChunks; ++c)
          tma_load_4d(sbase + L::kVOff + s * L::kKVBytes + c * L::kKVChunkBytes, &tmV, &bar_vfull[s], c * 64, g,
                      (j0 + j) * kSqdkBN, b);
        ++nv;
      }
      // every copy this thread issued has landed before the CTA may exit
      mbar_wait_drain(&bar_q, 0);
      for (int s = 0; s < kSqdkStages; ++s) {
        if (nk > s) mbar_wait_drain(&bar_kfull[s], ((nk - 1 - s) / kSqdkStages) & 1);
        if (nv > s) mbar_wait_drain(&bar_vfull[s], ((nv - 1 - s) / kSqdkStages) & 1);
      }
    } else if (lane == 0 && early) {
      // a tile without visible keys: drain the prologue's two loads
      mbar_wait_drain(&bar_q, 0);
      mbar_wait_drain(&bar_kfull[0], 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // The warp runs the issue loop converged (operands stay warp-uniform,
    // which makes each tcgen05.mma much cheaper to issue than from a lone
    // lane); one elected lane issues every product and commit.
    if (nblk > 0) {
      constexpr int kAB = kBF16 ? 1 : 0;
      constexpr uint32_t idesc_s = umma_idesc_f16(kSqdkBM, kSqdkBN, kAB, false, false);
      constexpr uint32_t idesc_o = umma_idesc_f16(kSqdkBM, HD, kAB, false, true);
      const uint32_t tO = tmem + L::kOCol;
      // shared-memory descriptors built once; a step inside a tile is a
      // constant added to the 14-bit start-address field (addresses < 256 KB,
      // so the field never carries)
      const uint64_t qdesc = sw128_desc(sbase + L::kQOff, 16, 1024);
      const uint64_t kdesc = sw128_desc(sbase + L::kKOff, 16, 1024);
      // V block, MN-major: 16 keys = 2 groups of 8 rows (SBO 1024 B), hd in
      // 64-column chunks L::kKVChunkBytes apart (LBO)
      const uint64_t vdesc = sw128_desc(sbase + L::kVOff, L::kKVChunkBytes, 1024);
      bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_q, 0, &abort_flag));
      tc_fence_after();
      // P V of block jj once P_jj is written and V_jj has landed (one
      // overlapped probe of both barriers)
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj % kSqdkStages, r = jj / kSqdkStages, sb = jj & 1;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait2(&bar_pfull[sb], (jj >> 1) & 1, &bar_vfull[s], r & 1, &abort_flag)))
          return false;
        tc_fence_after();
        const uint64_t vd = vdesc + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
        const uint32_t ta = tmem + sb * kSqdkBN;
        umma_ts_warp(tO, ta, vd, idesc_o, jj > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < kSqdkBN / 16; ++kk)
          umma_ts_warp(tO, ta + kk * 8, vd + static_cast<uint64_t>((kk * 16 * 128) >> 4), idesc_o, 1u);
        if (!long_range) umma_commit_warp(&bar_vempty[s]);
        else if (jj == nblk - 2) umma_commit_warp(&bar_vempty[0]);  // no Q K^T follows to signal it
        return true;
      };
      // unrolled by the ring depth: stage, buffer and descriptor offsets
      // become constants
#pragma unroll 2
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % kSqdkStages, r = j / kSqdkStages, sb = j & 1;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bar_kfull[s], r & 1, &abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t kd = kdesc + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int c = kk >> 2, w = kk & 3;  // 64-column chunk, 32-byte step inside the swizzle row
          umma_ss_warp(tmem + sb * kSqdkBN, qdesc + static_cast<uint64_t>((c * L::kQChunkBytes + w * 32) >> 4),
                       kd + static_cast<uint64_t>((c * L::kKVChunkBytes + w * 32) >> 4), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit_warp(&bar_sfull[sb]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) ok = issue_pv(nblk - 1);
      if (ok) umma_commit_warp(&bar_ofinal);
      umma_commit_warp(&bar_drain);
      if (lane == 0) mbar_wait_drain(&bar_drain, 0);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ softmax
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t tS = tmem + lane_base;
    const uint32_t tO = tmem + lane_base + L::kOCol;
    const float c2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = nblk > 0;
    for (int j = 0; ok && j < nblk; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_sfull[sb], (j >> 1) & 1, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      float sv[kSqdkBN];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(tS + sb * kSqdkBN, r0);
        tmem_ld32(tS + sb * kSqdkBN + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = __uint_as_float(r0[i]);
          sv[32 + i] = __uint_as_float(r1[i]);
        }
      }
      const int lim = pos - (j0 + j) * kSqdkBN;  // columns <= lim are visible to this row
      // warp-uniform: does any row of this warp need the causal mask here?
      const bool diag = __any_sync(0xFFFFFFFFu, lim < kSqdkBN - 1);
      if (diag) {
#pragma unroll
        for (int c = 0; c < kSqdkBN; ++c) sv[c] = (c <= lim) ? sv[c] : -INFINITY;
      }
      // p = 2^(s*c2 - m) with packed FMAs and MUFU exp2, packed to bf16/f16
      // pairs; the block's row sum is returned
      uint32_t pk[kSqdkBN / 2];
      auto exponentiate = [&](float m) -> float {
        const float neg_m = (m == -INFINITY) ? 0.0f : -m;
        const uint64_t cc = f2_pack(c2, c2), nm = f2_pack(neg_m, neg_m);
        uint64_t acc0 = f2_pack(0.0f, 0.0f), acc1 = acc0;
#pragma unroll
        for (int c = 0; c < kSqdkBN; c += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(sv[c], sv[c + 1]), cc, nm), x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          if ((c >> 1) & 1) acc1 = f2_add(acc1, f2_pack(p0, p1));
          else acc0 = f2_add(acc0, f2_pack(p0, p1));
          pk[c >> 1] = pack2<kBF16>(p0, p1);
        }
        float a0, a1, b0, b1;
        f2_unpack(acc0, a0, a1);
        f2_unpack(acc1, b0, b1);
        return (a0 + a1) + (b0 + b1);
      };
      // Optimistic pass: exponentiate against the running maximum without
      // reducing this block's maximum. Any m works for softmax as long as
      // nothing overflows; the block's row sum bounds every p of the row, so
      // a sum below kSqdkSumBound proves the block is representable.
      bool done = false;
      if (__all_sync(0xFFFFFFFFu, m_run != -INFINITY)) {
        const float lb = exponentiate(m_run);
        if (__all_sync(0xFFFFFFFFu, lb < kSqdkSumBound<kBF16>)) {
          l_run += lb;
          done = true;
        }
      }
      if (!done) {
        // exact pass: this block's row maximum, O rescaled when it grew
        float mq[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int c = 4; c < kSqdkBN; c += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) mq[u] = fmaxf(mq[u], sv[c + u]);
        }
        const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        const float m_new = fmaxf(m_run, mx * c2);
        const bool need_o = j > 0 && (m_run != -INFINITY) && (m_new > m_run);
        if (__any_sync(0xFFFFFFFFu, need_o)) {
          // O holds P_0..P_{j-1} V; the PV of block j-1 must have landed first:
          // Q K^T of block j+1, issued after it, completes later (and is
          // the next S this warp waits for anyway)
          bool landed;
          if (!long_range)
            landed = mbar_wait(&bar_vempty[(j - 1) % kSqdkStages], ((j - 1) / kSqdkStages) & 1, &abort_flag);
          else if (j + 1 < nblk)
            landed = mbar_wait(&bar_sfull[(j + 1) & 1], ((j + 1) >> 1) & 1, &abort_flag);
          else
            landed = mbar_wait(&bar_vempty[0], 0, &abort_flag);
          ok = __all_sync(0xFFFFFFFFu, landed);
          if (!ok) break;
          tc_fence_after();
          const float alpha = need_o ? fast_exp2(m_run - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t r[32];
            tmem_ld32(tO + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + c, r);
          }
          tmem_wait_st();
        }
        if (m_new != m_run) {
          l_run = (m_run == -INFINITY) ? 0.0f : l_run * fast_exp2(m_run - m_new);
          m_run = m_new;
        }
        l_run += exponentiate(m_run);
      }
      tmem_st32(tS + sb * kSqdkBN, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_pfull[sb]);
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nblk > 0) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bar_ofinal, 0, &abort_flag));
    using Elt = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    const int r = 32 * (warp & 3) + lane;
    if (p.nsplit > 1) {
      // partial result of this share of the key blocks: unnormalised O, the
      // running maximum it is relative to, and the row sum
      const int64_t prow = static_cast<int64_t>(item) * kSqdkBM + r;
      if (ok && nblk > 0) {
        tc_fence_after();
        float* dst = p.part_o + prow * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t rr[32];
          tmem_ld32(tO + c, rr);
          tmem_wait_ld();
          if (row_valid) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              reinterpret_cast<float4*>(dst + c)[v] =
                  make_float4(__uint_as_float(rr[4 * v]), __uint_as_float(rr[4 * v + 1]),
                              __uint_as_float(rr[4 * v + 2]), __uint_as_float(rr[4 * v + 3]));
          }
        }
        if (row_valid) reinterpret_cast<float2*>(p.part_ml)[prow] = make_float2(m_run, l_run);
      } else if (row_valid) {
        reinterpret_cast<float2*>(p.part_ml)[prow] = make_float2(-INFINITY, 0.0f);  // nothing in this share
      }
    } else {
      Elt* orow = static_cast<Elt*>(p.o) + static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(qi) * p.o_sk +
                  static_cast<int64_t>(hh) * p.o_sh;
      // the four softmax warps agree first (a warp whose wait gave up writes nothing)
      if (named_bar_and(kSqdkEpilogueBar, 128, ok && nblk > 0)) {
        // O / l in the Q tile's place (free once the last P V is done), laid out
        // as the Q load left it: 64-column chunks of 128-byte rows, 16-byte units
        // XOR-swizzled by row % 8; one thread then stores the tile with TMA
        tc_fence_after();
        const float inv_l = 1.0f / l_run;
        if (p.lse && row_valid)
          p.lse[static_cast<int64_t>(b) * p.lse_sb + static_cast<int64_t>(qi) * p.lse_sk + hh] =
              (m_run + log2f(l_run)) * kLn2;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t rr[32];
          tmem_ld32(tO + c, rr);
          tmem_wait_ld();
          const uint32_t rowb = sbase + L::kQOff + (c >> 6) * L::kQChunkBytes + r * 128;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack2<kBF16>(__uint_as_float(rr[8 * v + 0]) * inv_l, __uint_as_float(rr[8 * v + 1]) * inv_l);
            w.y = pack2<kBF16>(__uint_as_float(rr[8 * v + 2]) * inv_l, __uint_as_float(rr[8 * v + 3]) * inv_l);
            w.z = pack2<kBF16>(__uint_as_float(rr[8 * v + 4]) * inv_l, __uint_as_float(rr[8 * v + 5]) * inv_l);
            w.w = pack2<kBF16>(__uint_as_float(rr[8 * v + 6]) * inv_l, __uint_as_float(rr[8 * v + 7]) * inv_l);
            const int unit = ((c & 63) >> 3) + v;  // 16-byte unit in the 128-byte row
            st_shared_v4(rowb + ((unit ^ (r & 7)) << 4), w);
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(kSqdkEpilogueBar, 128);
        if (warp == 2 && lane == 0) {
          for (int ch = 0; ch < L::kChunks; ++ch)
            tma_store_4d(&tmO, sbase + L::kQOff + ch * L::kQChunkBytes, ch * 64, g * p.G, t * p.QT, b);
          tma_store_commit();
          tma_store_wait_read();
        }
      } else if (tile_blocks == 0 && row_valid) {
        // every position in the tile was negative: softmax over nothing
        const uint32_t nanw = pack2<kBF16>(__int_as_float(0x7FC00000), __int_as_float(0x7FC00000));
        uint4* dst = reinterpret_cast<uint4*>(orow);
        for (int v = 0; v < p.hd / 8; ++v) dst[v] = make_uint4(nanw, nanw, nanw, nanw);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// Merge of the nsplit partial results of each row (split key ranges):
//   M = max_s m_s,  w_s = 2^(m_s - M),  o = sum_s w_s O_s / sum_s w_s l_s
// One warp per (tile, row); lane l owns columns [4l, 4l+4) of each partial.
template <int HD, bool kBF16>
__global__ void __launch_bounds__(256) sqdk_combine_kernel(const SqdkParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t ntiles = static_cast<int64_t>(p.T) * p.B * p.Hkv;
  if (wid >= ntiles * kSqdkBM) return;
  const int tile = static_cast<int>(wid / kSqdkBM);
  const int r = static_cast<int>(wid - static_cast<int64_t>(tile) * kSqdkBM);
  int t, b, g;
  sqdk_tile_coords(p, tile, t, b, g);
  const int qloc = r / p.G;
  const int qi = t * p.QT + qloc;
  const int hh = g * p.G + (r - qloc * p.G);
  if (!(qloc < p.QT && qi < p.K)) return;
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml);
  float M = -INFINITY;
  for (int sidx = 0; sidx < p.nsplit; ++sidx)
    M = fmaxf(M, ml[(static_cast<int64_t>(tile) * p.nsplit + sidx) * kSqdkBM + r].x);
  float acc[HD / 32];
#pragma unroll
  for (int u = 0; u < HD / 32; ++u) acc[u] = 0.0f;
  float L = 0.0f;
  for (int sidx = 0; sidx < p.nsplit; ++sidx) {
    const int64_t prow = (static_cast<int64_t>(tile) * p.nsplit + sidx) * kSqdkBM + r;
    const float2 v = ml[prow];
    if (v.x == -INFINITY) continue;  // this share saw no visible key (its O was not written)
    const float w = fast_exp2(v.x - M);
    L += w * v.y;
    const float* po = p.part_o + prow * HD;
#pragma unroll
    for (int u = 0; u < HD / 32; ++u) acc[u] += w * po[32 * u + lane];
  }
  const float inv_l = 1.0f / L;
  if (p.lse && lane == 0)
    p.lse[static_cast<int64_t>(b) * p.lse_sb + static_cast<int64_t>(qi) * p.lse_sk + hh] = (M + log2f(L)) * kLn2;
  using Elt = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  Elt* orow = static_cast<Elt*>(p.o) + static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(qi) * p.o_sk +
              static_cast<int64_t>(hh) * p.o_sh;
#pragma unroll
  for (int u = 0; u < HD / 32; ++u) {
    const int c = 32 * u + lane;
    if (c < p.hd) {
      if constexpr (kBF16) orow[c] = __float2bfloat16_rn(acc[u] * inv_l);
      else orow[c] = __float2half_rn(acc[u] * inv_l);
    }
  }
}

}  // namespace hspmn
