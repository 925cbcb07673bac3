// Shared-sequence indexer kernel (prefill): one CTA serves four consecutive
// query rows that read the same pages (the causal rows of one sequence share
// its block-table row), so every K tile is loaded once and feeds one
// tcgen05.mma with N = 4 queries x 64 heads = 256.
//
// One CTA per SM (18 warps, 512 TMEM columns):
//   warp 0      TMA producer: the four query boxes once, then per tile two
//               8 KB page boxes and two 256 B scale rows into a 4-stage ring;
//   warp 1      TMEM owner and MMA issuer: D[128 keys x 256] (fp32 in TMEM,
//               2 buffers) = K_tile[128 x 128 e4m3] . Q[256 x 128 e4m3]^T as
//               four tcgen05.mma kind::f8f6f4 (K = 32 each);
//   warps 2..17 four epilogue groups of four warps, group j = query row j:
//               thread = TMEM lane = key; tcgen05.ld of its 64 head columns
//               of query j, relu / head weight / scale in registers, then the
//               row's own threshold filter and candidate buffer (cut to the
//               best 2048 when nearly full), synchronised per group only.
// After the stream two 256-thread pairs of groups take two rows each: exact
// radix select down to 2048 when more remain, then the bucket ordering and
// the translation to physical slots (the same primitives as the per-row
// kernel). Scores never go to HBM.
//
// A CTA first checks that its rows really share their pages: every row's
// block-table entries over its visible keys must equal those of the longest
// row. If not, it marks its rows as not handled and exits; the per-row
// kernel launched after it serves them. The reference has no counterpart:
// its scoring kernel runs one (row, page) pair per CTA with heads on M
// (solution/cuda/kernel.cu:209-452).
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"
#include "select.cuh"
#include "indexer_kernel.cuh"
#include "dsa_topk_indexer.h"

namespace dsa {

constexpr int kPQ = kGroupRows;                    // query rows per CTA (4)
constexpr int kPStages = 4;                        // K ring stages
constexpr int kPWarps = 2 + 4 * kPQ;               // producer, MMA, 4 epilogue warps per row
constexpr int kPThreads = 32 * kPWarps;            // 576
constexpr int kPCap = 3584;                        // candidate keys per row
constexpr int kPBufCols = kPQ * kHeads;            // TMEM columns of one tile (N = 256)
constexpr int kPTmemCols = 2 * kPBufCols;          // two buffers: all 512 columns

// Shared memory map (byte offsets from a 1024-aligned base).
constexpr int kPOffK = 0;                                  // kPStages x 16384, swizzled K tiles
constexpr int kPOffQ = kPOffK + kPStages * 16384;          // kPQ x 8192, swizzled Q (N = 256 rows)
constexpr int kPOffScale = kPOffQ + kPQ * 8192;            // kPStages x 512
constexpr int kPOffCand = kPOffScale + kPStages * 512;     // kPQ x kPCap x 8
constexpr int kPOffHist = kPOffCand + kPQ * kPCap * 8;     // kPQ x 256 x 4
constexpr int kPOffW = kPOffHist + kPQ * 256 * 4;          // kPQ x 64 x 4
constexpr int kPOffBar = kPOffW + kPQ * kHeads * 4;        // 256
constexpr int kPOffMisc = kPOffBar + 256;                  // kPQ x 128 per row + 128 shared
constexpr int kPSmemUsed = kPOffMisc + kPQ * 128 + 128;
constexpr int kPSmemBytes = kPSmemUsed + 1024;             // alignment slack
static_assert(kPSmemBytes <= 232448, "one CTA per SM");
static_assert((2 * kPStages + 2 * 2 + 1) * 8 <= 256, "barrier area");
// After the stream the K ring and Q area hold the ordering scratch of the two
// pairs: tmp 2048 x 8, bucket ids 2048 x 2, three 2048-word count arrays.
constexpr int kPRankBytes = kTopK * 8 + kTopK * 2 + 3 * 2048 * 4;
static_assert(2 * kPRankBytes <= kPOffScale, "ordering scratch of both pairs fits in the K ring and Q area");
static_assert(kPRankBytes % 16 == 0, "16-byte aligned scratch");

// Per-row misc words (uint32 at kPOffMisc + 128 * j).
enum PRowWord : int {
  kPRot = 0,     // 3 rotating append counters
  kPCount = 3,   // candidates after a compaction
  kPSel = 4,     // 3 words: digit scan result
  kPFinal = 7,   // candidates at the end of the stream
  kPWsum = 8,    // 8 words: warp offset scans
  kPMM = 24,     // 2 x u64: min / max (word 24 = byte 96, 8-byte aligned)
};
// Shared misc words (uint32 at kPOffMisc + 128 * kPQ).
enum PSharedWord : int { kPTmem = 0, kPAbort = 1, kPBad = 2 };

// Named barriers: 1..4 the row groups (128 threads), 5..6 the tail pairs (256).
constexpr int kPBarRow0 = 1;
constexpr int kPBarPair0 = 5;

struct PrefillParams {
  const int32_t* group_order;  // [ceil(B/4)] group served by CTA c (longest first), or null
  int32_t* handled;            // [B] out: 1 = row served here, 0 = left to the per-row kernel
};

template <int kMode>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_s,
                   const __grid_constant__ CUtensorMap tm_q, const IndexerParams p, const PrefillParams pp) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);
  uint32_t* shared_misc = reinterpret_cast<uint32_t*>(smem + kPOffMisc + 128 * kPQ);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(shared_misc + kPAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = pp.group_order ? pp.group_order[blockIdx.x] : static_cast<int>(blockIdx.x);
  const int r0 = g * kPQ;
  const int nq = (p.batch - r0) < kPQ ? (p.batch - r0) : kPQ;

  // ---- rows: clamped lengths, key ranges, the longest row ----
  const int64_t cap_keys = static_cast<int64_t>(p.max_pages) * kPage;
  int64_t lo = kMode == kModePartial ? (p.key_begin < 0 ? 0 : p.key_begin) : 0;
  lo = lo < cap_keys ? lo : cap_keys;
  // End of row j's key range: its length clamped to the block table, and to
  // key_end in partial mode (0 for rows past the batch).
  auto row_hi = [&](int j) -> int64_t {
    int64_t len = j < nq ? static_cast<int64_t>(p.seq_lens[r0 + j]) : 0;
    len = len < 0 ? 0 : (len > cap_keys ? cap_keys : len);
    if (kMode == kModePartial) len = p.key_end < len ? p.key_end : len;
    return len;
  };
  int ref = 0;
  int64_t hi_max = 0;
#pragma unroll
  for (int j = 0; j < kPQ; ++j) {
    const int64_t h = row_hi(j);
    if (h > hi_max) {
      hi_max = h;
      ref = j;
    }
  }
  if (threadIdx.x == 0) {
    for (int j = 0; j < nq; ++j)
      if (p.seq_lens[r0 + j] > cap_keys) atomicOr(&g_dsa_status, DSA_STATUS_SEQ_CLAMPED);
  }
  const int page_lo = static_cast<int>(lo / kPage);
  const int32_t* bt_ref = p.block_table + static_cast<int64_t>(r0 + ref) * p.max_pages;

  // ---- do the rows share their pages? ----
  {
    bool bad = false;
#pragma unroll 1
    for (int j = 0; j < nq; ++j) {
      if (j == ref) continue;
      const int32_t* bt_j = p.block_table + static_cast<int64_t>(r0 + j) * p.max_pages;
      const int npg = static_cast<int>((row_hi(j) + kPage - 1) / kPage);  // the row's visible pages
      for (int pg = page_lo + static_cast<int>(threadIdx.x); pg < npg; pg += kPThreads)
        bad |= bt_j[pg] != bt_ref[pg];
    }
    if (__syncthreads_or(bad ? 1 : 0)) {
      if (threadIdx.x < static_cast<unsigned>(nq)) pp.handled[r0 + threadIdx.x] = 0;
      return;  // before any barrier, TMEM or TMA use
    }
    if (threadIdx.x < static_cast<unsigned>(nq)) pp.handled[r0 + threadIdx.x] = 1;
  }
  const int page_hi = static_cast<int>((hi_max + kPage - 1) / kPage);
  const int n_tiles = page_hi > page_lo ? (page_hi - page_lo + 1) / 2 : 0;

  const uint32_t bar_full = base_addr + kPOffBar;       // [kPStages]
  const uint32_t bar_empty = bar_full + 8 * kPStages;   // [kPStages]
  const uint32_t bar_tfull = bar_empty + 8 * kPStages;  // [2]
  const uint32_t bar_tempty = bar_tfull + 16;           // [2]
  const uint32_t bar_q = bar_tempty + 16;               // [1]

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1 + 4 * kPQ);  // MMA commit + every epilogue warp
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_tfull + 8 * i, 1);
      ptx::mbar_init(bar_tempty + 8 * i, 4 * kPQ);
    }
    ptx::mbar_init(bar_q, 1);
    ptx::fence_mbar_init();
    shared_misc[kPAbort] = 0u;
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_s);
    ptx::prefetch_tmap(&tm_q);
  }
  if (threadIdx.x < kPQ * 32) {  // misc words of the four rows
    reinterpret_cast<uint32_t*>(smem + kPOffMisc)[threadIdx.x] = 0u;
  }
  if (warp == 1) {
    ptx::tmem_alloc(base_addr + kPOffMisc + 128 * kPQ + 4 * kPTmem, kPTmemCols);
    ptx::tmem_relinquish();
  }
  {
    float* s_w = reinterpret_cast<float*>(smem + kPOffW);
    for (int i = threadIdx.x; i < kPQ * kHeads; i += kPThreads) {
      const int j = i / kHeads;
      s_w[i] = j < nq ? p.weights[static_cast<int64_t>(r0 + j) * kHeads + (i % kHeads)] : 0.f;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = shared_misc[kPTmem];

  int issued = 0, skipped = -1, mma_issued = 0;
  bool aborted = false;

  if (warp == 0) {
    // ===================== TMA producer =====================
    const uint64_t pol_stream = ptx::policy_evict_last();  // the pages are re-read by the next groups
    if (n_tiles > 0 && lane == 0) {
      ptx::mbar_arrive_expect_tx(bar_q, static_cast<uint32_t>(nq) * kHeads * kDim);
      for (int j = 0; j < nq; ++j)
        ptx::tma_load_2d(base_addr + kPOffQ + j * 8192, &tm_q, bar_q, 0, (r0 + j) * kHeads,
                         ptx::policy_evict_first());
    }
    const int pg_end = page_hi;
    int32_t pg_batch = 0;
#pragma unroll 1
    for (int i = 0; i < n_tiles; ++i) {
      if ((i & 15) == 0) {
        const int pidx = page_lo + 2 * i + lane;
        pg_batch = (pidx < pg_end) ? bt_ref[pidx] : 0;
      }
      const int32_t pa = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * i) & 31);
      const int32_t pb = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * i + 1) & 31);
      const bool has_b = (page_lo + 2 * i + 1) < pg_end;
      const int s = i % kPStages;
      const uint32_t ph = static_cast<uint32_t>(i / kPStages) & 1u;
      const bool ok = ptx::mbar_wait(bar_empty + 8 * s, ph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT,
                                     p.wait_ns);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      if (i == p.skip_tile) {  // test hook: this tile's loads are never issued
        skipped = i;
        issued = i + 1;
        continue;
      }
      if (lane == 0) {
        if (static_cast<uint64_t>(static_cast<uint32_t>(pa)) >= static_cast<uint64_t>(p.num_pages) ||
            (has_b && static_cast<uint64_t>(static_cast<uint32_t>(pb)) >= static_cast<uint64_t>(p.num_pages)))
          atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);  // TMA zero-fills out-of-range boxes
        const uint32_t bytes = has_b ? 2u * (kPageData + 256u) : (kPageData + 256u);
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t kdst = base_addr + kPOffK + s * 16384;
        const uint32_t sdst = base_addr + kPOffScale + s * 512;
        ptx::mbar_arrive_expect_tx(fb, bytes);
        ptx::tma_load_3d(kdst, &tm_k, fb, 0, 0, pa, pol_stream);
        ptx::tma_load_2d(sdst, &tm_s, fb, 0, pa, pol_stream);
        if (has_b) {
          ptx::tma_load_3d(kdst + kPageData, &tm_k, fb, 0, 0, pb, pol_stream);
          ptx::tma_load_2d(sdst + 256, &tm_s, fb, 0, pb, pol_stream);
        }
      }
      __syncwarp();
      issued = i + 1;
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    constexpr uint32_t idesc = ptx::idesc_e4m3_f32(kTileKeys, kPBufCols);
    bool ok = true;
    if (n_tiles > 0)
      ok = ptx::mbar_wait(bar_q, 0u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
    const uint64_t qdesc = ptx::sw128_kmajor_desc(base_addr + kPOffQ);
#pragma unroll 1
    for (int i = 0; i < n_tiles && !aborted; ++i) {
      const int s = i % kPStages;
      const uint32_t ph = static_cast<uint32_t>(i / kPStages) & 1u;
      const int buf = i & 1;
      const uint32_t bph = static_cast<uint32_t>(i >> 1) & 1u;
      ok = ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns) &&
           ptx::mbar_wait(bar_tempty + 8 * buf, bph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT,
                          p.wait_ns);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      __syncwarp();
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint64_t adesc = ptx::sw128_kmajor_desc(base_addr + kPOffK + s * 16384);
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kPBufCols);
#pragma unroll
        for (int kk = 0; kk < kDim / 32; ++kk)
          ptx::mma_f8f6f4(d, adesc + 2ull * kk, qdesc + 2ull * kk, idesc, kk > 0 ? 1u : 0u);
        ptx::mma_commit(bar_empty + 8 * s);
        ptx::mma_commit(bar_tfull + 8 * buf);
      }
      __syncwarp();
      mma_issued = i + 1;
    }
  } else {
    // ===================== epilogue: group j = query row j =====================
    const int j = (warp - 2) >> 2;
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;
    const int gt = threadIdx.x - 64 - 128 * j;  // 0..127 within the group
    const uint32_t bar_row = kPBarRow0 + j;
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    const float* s_w = reinterpret_cast<const float*>(smem + kPOffW) + j * kHeads;
    uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kPOffCand) + j * kPCap;
    uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kPOffHist) + j * 256;
    uint32_t* rmisc = reinterpret_cast<uint32_t*>(smem + kPOffMisc + 128 * j);
    volatile uint32_t* rmisc_v = rmisc;
    unsigned long long* mm = reinterpret_cast<unsigned long long*>(rmisc + kPMM);
    const int64_t key_hi = row_hi(j);
    uint64_t thr = 0;  // keys below thr can no longer reach the row's top 2048
    int since = 0;
    int check_every = kPCap / kTileKeys;
    // Same append protocol as the per-row kernel: keys of the current check
    // interval take slots n_base + (rotating counter `slot`), each warp
    // storing a tile's keys one tile late once its slot atomic has returned.
    uint32_t n_base = 0, slot = 0, pm = 0, pbase = 0;
    int pleader = 0;
    bool pkeep = false;
    uint64_t pkey = 0;
    auto flush = [&]() {
      if (pm) {
        const uint32_t pbv = __shfl_sync(0xFFFFFFFFu, pbase, pleader);
        if (pkeep) cand[n_base + pbv + __popc(pm & lanemask_lt())] = pkey;
      }
      pm = 0u;
    };
    // A warp whose wait gave up (`aborted`, warp-uniform) stops touching the
    // pipeline but keeps walking the same tile schedule with no keys, so it
    // still meets its group at every check barrier.
#pragma unroll 1
    for (int i = 0; i < n_tiles; ++i) {
      const int s = i % kPStages;
      const uint32_t ph = static_cast<uint32_t>(i / kPStages) & 1u;
      const int buf = i & 1;
      const int64_t tile_key0 = static_cast<int64_t>(page_lo + 2 * i) * kPage;
      const bool live = tile_key0 < key_hi && tile_key0 + kTileKeys > lo;  // tile holds keys of this row
      float score = 0.f;
      if (!aborted) {
        const bool ok =
            ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
        if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
      }
      if (!aborted) {
        // Generic-proxy read of the scale, then the proxy fence before the
        // stage is released to the next TMA write (see indexer_kernel).
        const float scale = ptx::lds_f32_ordered(base_addr + kPOffScale + 4u * (s * kTileKeys + row));
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
        const uint32_t bph = static_cast<uint32_t>(i >> 1) & 1u;
        const bool ok =
            ptx::mbar_wait(bar_tfull + 8 * buf, bph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
        if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
        if (!aborted) {
          __syncwarp();
          ptx::tc_fence_after();
          if (live) {
            float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            uint32_t acc[32];
            const uint32_t ta = tmem + t_lane + static_cast<uint32_t>(buf * kPBufCols + j * kHeads);
            ptx::tmem_ld_32x32b_x32_sync(ta, acc);
            if (scale >= 0.f)
              head_reduce_half<false>(acc, s_w, 0, sums);
            else
              head_reduce_half<true>(acc, s_w, 0, sums);
            ptx::tmem_ld_32x32b_x32_sync(ta + 32u, acc);
            if (scale >= 0.f)
              head_reduce_half<false>(acc, s_w, 32, sums);
            else
              head_reduce_half<true>(acc, s_w, 32, sums);
            score = (((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]))) *
                    fabsf(scale);
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * buf);
        }
      }
      const int64_t pos = tile_key0 + row;
      const bool valid = !aborted && pos >= lo && pos < key_hi;
      const uint64_t key = pack_key(score, static_cast<uint32_t>(pos));
      const bool keep = valid && key >= thr;
      flush();
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      pm = m;
      pkeep = keep;
      pkey = key;
      if (m) {
        pleader = __ffs(m) - 1;
        pbase = 0u;
        if (lane == pleader) pbase = atomicAdd(rmisc + kPRot + slot, static_cast<uint32_t>(__popc(m)));
      }
      // Every check_every tiles the row's buffer may be nearly full: the
      // group meets, reads the interval's count, moves to the next counter
      // and clears the one used two intervals ago; when fewer than two tiles
      // of room are left it cuts the buffer to exactly the best 2048. The
      // schedule depends only on tile counts, so the group's four warps take
      // the same barriers.
      if (++since == check_every && i + 1 < n_tiles) {
        since = 0;
        flush();
        ptx::named_bar(bar_row, 128);
        const uint32_t n = n_base + rmisc_v[kPRot + slot];
        if (gt == 0) rmisc[kPRot + (slot + 2u) % 3u] = 0u;
        n_base = n;
        slot = (slot + 1u) % 3u;
        if (n > static_cast<uint32_t>(kPCap - 2 * kTileKeys)) {
          if (gt == 0) {
            mm[0] = ~0ull;
            mm[1] = 0ull;
          }
          ptx::named_bar(bar_row, 128);
          group_minmax<128>(cand, n, mm, gt, bar_row);
          const uint64_t T = group_select<128>(cand, n, kTopK, mm, hist, rmisc + kPSel, gt, bar_row);
          group_compact_chunked<128, 8>(cand, n, T, rmisc + kPCount, rmisc + kPWsum, gt, bar_row);
          thr = T;
          n_base = rmisc_v[kPCount];
        }
        check_every = static_cast<int>((kPCap - n_base) / kTileKeys);
      }
    }
    flush();
    if (gt == 0) {  // read after the barrier below
      rmisc[kPFinal] = n_base;
      rmisc[kPSel] = slot;  // the counter in use at the end (sel words are free now)
    }
  }
  // ---- end of the stream: drain, release TMEM ----
  if (aborted) *abort_flag = 1u;
  ptx::tc_fence_before();
  __syncthreads();
  if (shared_misc[kPAbort] != 0u) {
    volatile uint32_t no_abort = 0u;
    if (warp == 0 && lane == 0) {
      for (int i = (issued > kPStages ? issued - kPStages : 0); i < issued; ++i)
        if (i != skipped)
          ptx::mbar_wait(bar_full + 8 * (i % kPStages), static_cast<uint32_t>(i / kPStages) & 1u, &no_abort,
                         &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    }
    if (warp == 1 && lane == 0 && mma_issued > 0) {
      const int last = mma_issued - 1;
      ptx::mbar_wait(bar_tfull + 8 * (last & 1), static_cast<uint32_t>(last >> 1) & 1u, &no_abort, &g_dsa_status,
                     DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    }
    __syncthreads();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kPTmemCols);
  }
  if (warp < 2) return;

  // ---- tail: pair q2 (warps 2+8*q2 .. 9+8*q2) selects and orders rows 2*q2, 2*q2+1 ----
  const int pair = (warp - 2) >> 3;
  const int pt = threadIdx.x - 64 - 256 * pair;  // 0..255
  const uint32_t bar_pair = kPBarPair0 + pair;
  uint32_t* pmisc = reinterpret_cast<uint32_t*>(smem + kPOffMisc + 128 * (2 * pair));
  RankScratch sc;
  sc.tmp = reinterpret_cast<uint64_t*>(smem + kPOffK + pair * kPRankBytes);
  sc.tmpd = reinterpret_cast<uint16_t*>(smem + kPOffK + pair * kPRankBytes + kTopK * 8);
  sc.cnt = reinterpret_cast<uint32_t*>(smem + kPOffK + pair * kPRankBytes + kTopK * 10);
  sc.start = sc.cnt + 2048;
  sc.fill = sc.start + 2048;
  sc.wsum = pmisc + kPWsum;
#pragma unroll 1
  for (int jj = 0; jj < 2; ++jj) {
    const int j = 2 * pair + jj;
    if (j >= nq) break;  // uniform over the pair
    uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kPOffCand) + j * kPCap;
    uint32_t* rmisc = reinterpret_cast<uint32_t*>(smem + kPOffMisc + 128 * j);
    unsigned long long* mm = reinterpret_cast<unsigned long long*>(rmisc + kPMM);
    uint32_t n = rmisc[kPFinal] + rmisc[kPRot + rmisc[kPSel]];
    ptx::named_bar(bar_pair, 256);  // every thread has read n before mm / sel are reused
    if (pt == 0) {
      mm[0] = ~0ull;
      mm[1] = 0ull;
    }
    ptx::named_bar(bar_pair, 256);
    group_minmax<256>(cand, n, mm, pt, bar_pair);
    uint64_t kmin = mm[0];
    const uint64_t kmax = mm[1];
    if (n > static_cast<uint32_t>(kTopK)) {
      const uint64_t T = group_select<256>(cand, n, kTopK, mm, reinterpret_cast<uint32_t*>(smem + kPOffHist) + j * 256,
                                           rmisc + kPSel, pt, bar_pair);
      group_compact_chunked<256, 8>(cand, n, T, rmisc + kPCount, pmisc + kPWsum, pt, bar_pair);
      n = kTopK;
      kmin = T;
    }
    const int64_t o = static_cast<int64_t>(r0 + j) * kTopK;
    const int32_t* bt_row = p.block_table + static_cast<int64_t>(r0 + j) * p.max_pages;
    if (kMode == kModeTopK) {
      EmitSlots e{p.out + o, bt_row};
      block_rank_emit<8>(cand, n, kmin, kmax, sc, e, pt, bar_pair);
    } else {
      EmitCandidates e{p.cand_scores + o, p.cand_pos + o};
      block_rank_emit<8>(cand, n, kmin, kmax, sc, e, pt, bar_pair);
    }
    ptx::named_bar(bar_pair, 256);  // the scratch is reused by the next row
  }
}

}  // namespace dsa
