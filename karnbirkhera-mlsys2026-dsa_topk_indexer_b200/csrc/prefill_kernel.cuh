// Shared-sequence indexer kernel (prefill): one CTA serves four consecutive
// query rows that read the same pages (the causal rows of one sequence share
// its block-table row), so every K tile is loaded once and feeds the MMAs of
// all four rows.
//
// One CTA per SM (19 warps, 512 TMEM columns):
//   warp 0      TMA producer: the four query boxes once, then per tile two
//               8 KB page boxes into a 4-stage ring (freed when both MMA
//               issuers have committed);
//   warps 1, 18 MMA issuers, one per row pair (warp 1 also owns TMEM):
//               D[128 keys x 128] (fp32 in TMEM, one buffer per tile parity
//               and pair) = K_tile[128 x 128 e4m3] . Q_pair[128 x 128 e4m3]^T
//               as four tcgen05.mma kind::f8f6f4 (K = 32). A pair whose
//               epilogue is busy (a candidate-buffer cut) holds up only its
//               own issuer;
//   warps 2..17 sixteen epilogue warps: warp (parity, pair, quarter) takes the
//               tiles of one parity, the two rows of one pair, and the 32 keys
//               of one TMEM lane quarter (thread = key). Per tile it waits
//               for the accumulators once (key scales come from the page
//               pool with global loads issued two tiles ahead), then scores
//               both rows from their 64 head columns (relu / head weight /
//               scale in registers) and appends the keys above each row's
//               threshold to that row's candidate buffer, cut to the best
//               2048 when nearly full. The eight warps of a pair (both
//               parities) meet only at those checks.
// Scoring two rows per warp shares every per-tile wait and TMEM hand-off
// between them; the math itself (64 max + 32 packed FMA per key
// and row) is what bounds the kernel.
// After the stream each pair's 256 threads take its two rows in turn: exact
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
constexpr int kPWarps = 3 + 16;                    // producer, two MMA issuers, 16 epilogue warps
constexpr int kPThreads = 32 * kPWarps;            // 608
constexpr int kPMmaWarp1 = 18;                     // MMA issuer of row pair 1 (warp 1: pair 0)
constexpr int kPCap = 3968;                        // candidate keys per row (the rest of the 227 KB)
constexpr int kPBufCols = 2 * kHeads;              // TMEM columns of one row pair's tile (N = 128)
constexpr int kPTmemCols = 4 * kPBufCols;          // (parity, pair) buffers: all 512 columns

// Shared memory map (byte offsets from a 1024-aligned base).
constexpr int kPOffK = 0;                                  // kPStages x 16384, swizzled K tiles
constexpr int kPOffQ = kPOffK + kPStages * 16384;          // kPQ x 8192, swizzled Q (4 x 64 head rows)
constexpr int kPOffCand = kPOffQ + kPQ * 8192;             // kPQ x kPCap x 8
constexpr int kPOffHist = kPOffCand + kPQ * kPCap * 8;     // kPQ x 256 x 4
constexpr int kPOffW = kPOffHist + kPQ * 256 * 4;          // kPQ x 64 x 4
constexpr int kPOffBar = kPOffW + kPQ * kHeads * 4;        // 256
constexpr int kPOffMisc = kPOffBar + 256;                  // kPQ x 128 per row + 128 shared
constexpr int kPSmemUsed = kPOffMisc + kPQ * 128 + 128;
constexpr int kPSmemBytes = kPSmemUsed + 1024;             // alignment slack
static_assert(kPSmemBytes <= 232448, "one CTA per SM");
static_assert((2 * kPStages + 2 * 4 + 1) * 8 <= 256, "barrier area");
// After the stream the K ring and Q area hold the ordering scratch of the two
// pairs: tmp 2048 x 8, bucket ids 2048 x 2, three 2048-word count arrays.
constexpr int kPRankBytes = kTopK * 8 + kTopK * 2 + 3 * 2048 * 4;
static_assert(2 * kPRankBytes <= kPOffCand, "ordering scratch of both pairs fits in the K ring and Q area");
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

// Named barriers 1..2: the 256 epilogue threads of row pair 0 / 1 (both
// tile parities), at the buffer checks and in the tail.
constexpr int kPBarPair0 = 1;
static_assert(kPQ == 4, "two row pairs of two rows");

struct PrefillParams {
  const int32_t* group_order;  // [ceil(B/4)] group served by CTA c (longest first), or null
  int32_t* handled;            // [B] out: 1 = row served here, 0 = left to the per-row kernel
};

// 19 warps: five of them share one SM sub-partition's 16384 registers, so
// 96 registers per thread is the ceiling.
template <int kMode>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                   const IndexerParams p, const PrefillParams pp) {
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
    int npg[kPQ];  // pages whose entries must match: the row's visible pages
    int npg_max = 0;
#pragma unroll
    for (int j = 0; j < kPQ; ++j) {
      npg[j] = j == ref ? 0 : static_cast<int>((row_hi(j) + kPage - 1) / kPage);
      npg_max = npg[j] > npg_max ? npg[j] : npg_max;
    }
    bool bad = false;
    for (int pg = page_lo + static_cast<int>(threadIdx.x); pg < npg_max; pg += kPThreads) {
      const int32_t r = bt_ref[pg];
#pragma unroll
      for (int j = 0; j < kPQ; ++j)
        if (pg < npg[j]) bad |= p.block_table[static_cast<int64_t>(r0 + j) * p.max_pages + pg] != r;
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
  const uint32_t bar_tfull = bar_empty + 8 * kPStages;  // [parity][pair]
  const uint32_t bar_tempty = bar_tfull + 32;           // [parity][pair]
  const uint32_t bar_q = bar_tempty + 32;               // [1]

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 2);  // both issuers' MMA commits: the epilogue never reads the ring
    }
    for (int i = 0; i < 4; ++i) {
      ptx::mbar_init(bar_tfull + 8 * i, 1);
      ptx::mbar_init(bar_tempty + 8 * i, 4);  // the pair's four warps of the tile's parity
    }
    ptx::mbar_init(bar_q, 1);
    ptx::fence_mbar_init();
    shared_misc[kPAbort] = 0u;
    ptx::prefetch_tmap(&tm_k);
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
        const uint32_t bytes = has_b ? 2u * kPageData : kPageData;
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t kdst = base_addr + kPOffK + s * 16384;
        ptx::mbar_arrive_expect_tx(fb, bytes);
        ptx::tma_load_3d(kdst, &tm_k, fb, 0, 0, pa, pol_stream);
        if (has_b) ptx::tma_load_3d(kdst + kPageData, &tm_k, fb, 0, 0, pb, pol_stream);
      }
      __syncwarp();
      issued = i + 1;
    }
  } else if (warp == 1 || warp == kPMmaWarp1) {
    // ===================== MMA issuers, one per row pair =====================
    // Each pair has its own TMEM buffers and barriers, so a pair that is
    // cutting a candidate buffer holds up only its own MMAs; the other pair
    // runs on until the ring (freed by both issuers' commits) is full.
    const int q = warp == 1 ? 0 : 1;
    constexpr uint32_t idesc = ptx::idesc_e4m3_f32(kTileKeys, kPBufCols);
    bool ok = true;
    if (n_tiles > 0)
      ok = ptx::mbar_wait(bar_q, 0u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
    const uint64_t qdesc = ptx::sw128_kmajor_desc(base_addr + kPOffQ + q * 2 * 8192);  // rows 128q..128q+127
#pragma unroll 1
    for (int i = 0; i < n_tiles && !aborted; ++i) {
      const int s = i % kPStages;
      const uint32_t ph = static_cast<uint32_t>(i / kPStages) & 1u;
      const int buf = 2 * (i & 1) + q;
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
    // ===================== epilogue =====================
    const int ew = warp - 2;
    const int par = ew >> 3;                    // tiles of this parity
    const int qp = (ew >> 2) & 1;               // rows 2*qp and 2*qp + 1
    const int q4 = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;             // key of the tile
    const int gt = ((ew & 3) + 4 * par) * 32 + lane;  // 0..255 within the pair's eight warps
    const uint32_t bar_qp = kPBarPair0 + qp;
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    const int jA = 2 * qp, jB = 2 * qp + 1;
    const float* w_A = reinterpret_cast<const float*>(smem + kPOffW) + jA * kHeads;
    const float* w_B = w_A + kHeads;
    uint64_t* cand_A = reinterpret_cast<uint64_t*>(smem + kPOffCand) + jA * kPCap;
    uint64_t* cand_B = cand_A + kPCap;
    uint32_t* misc_A = reinterpret_cast<uint32_t*>(smem + kPOffMisc + 128 * jA);
    uint32_t* misc_B = misc_A + 32;
    // Key positions fit in 32 bits: max_pages * 64 <= INT32_MAX (host check).
    const uint32_t hi_A = static_cast<uint32_t>(row_hi(jA)), hi_B = static_cast<uint32_t>(row_hi(jB));
    const uint32_t lo32 = static_cast<uint32_t>(lo);
    const int n_pairs_full = n_tiles >> 1;
    // Key scales straight from the page pool, two tiles of the parity ahead
    // (page ids one tile ahead of that), as in the per-row kernel: the
    // epilogue never waits for or releases a K ring stage.
    const uint8_t* scale_base = p.kcache + kPageData + 4 * (row & (kPage - 1));
    auto page_of = [&](int t) -> int32_t {  // warp-uniform; -1: no page
      const int pi = page_lo + 2 * t + (q4 >> 1);
      return (t < n_tiles && pi < page_hi) ? __ldg(bt_ref + pi) : -1;
    };
    auto scale_of = [&](int32_t pid) -> float {
      return static_cast<uint64_t>(static_cast<uint32_t>(pid)) < static_cast<uint64_t>(p.num_pages)
                 ? __ldg(reinterpret_cast<const float*>(scale_base + static_cast<int64_t>(pid) * kPageBytes))
                 : 0.f;
    };
    float sc_next = scale_of(page_of(par)), sc_after = scale_of(page_of(par + 2));
    int32_t pid_ahead = page_of(par + 4);
    uint64_t thr_A = 0, thr_B = 0;  // keys below thr can no longer reach the row's top 2048
    uint32_t nb_A = 0, nb_B = 0;    // candidates counted at the last check
    uint32_t slot = 0;              // rotating append counter of the current interval (both rows)
    int since = 0;
    int check_every = kPCap / (2 * kTileKeys);  // tile pairs between checks
    // Same append protocol as the per-row kernel, per row: keys of the
    // current interval take slots nb + (rotating counter `slot`), each warp
    // storing a tile's keys one tile later, once its slot atomic has returned.
    struct Pending {
      uint32_t m = 0, base = 0;
      int leader = 0;
      bool keep = false;
      uint64_t key = 0;
    };
    Pending pa, pb;
    auto flush = [&](Pending& q, uint64_t* cand, uint32_t nb) {
      if (q.m) {
        const uint32_t b0 = __shfl_sync(0xFFFFFFFFu, q.base, q.leader);
        if (q.keep) cand[nb + b0 + __popc(q.m & lanemask_lt())] = q.key;
      }
      q.m = 0u;
    };
    auto append = [&](Pending& q, uint32_t* misc, uint64_t key, bool keep) {
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      q.m = m;
      q.keep = keep;
      q.key = key;
      if (m) {
        q.leader = __ffs(m) - 1;
        q.base = 0u;
        if (lane == q.leader) q.base = atomicAdd(misc + kPRot + slot, static_cast<uint32_t>(__popc(m)));
      }
    };
    // Cut of one row's buffer to exactly its best 2048 (all 256 threads).
    auto cut = [&](uint64_t* cand, uint32_t* misc, uint32_t n, int j) -> uint64_t {
      unsigned long long* mm = reinterpret_cast<unsigned long long*>(misc + kPMM);
      if (gt == 0) {
        mm[0] = ~0ull;
        mm[1] = 0ull;
      }
      ptx::named_bar(bar_qp, 256);
      group_minmax<256>(cand, n, mm, gt, bar_qp);
      uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kPOffHist) + j * 256;
      const uint64_t T = group_select<256>(cand, n, kTopK, mm, hist, misc + kPSel, gt, bar_qp);
      group_compact_chunked<256, 8>(cand, n, T, misc + kPCount, misc + kPWsum, gt, bar_qp);
      return T;
    };
    // A warp whose wait gave up (`aborted`, warp-uniform) stops touching the
    // pipeline but keeps walking the same tile schedule with no keys, so it
    // still meets its pair at every check barrier.
#pragma unroll 1
    for (int i = par; i < n_tiles; i += 2) {
      const float scale = sc_next;
      sc_next = sc_after;
      sc_after = scale_of(pid_ahead);  // tile i + 4
      pid_ahead = page_of(i + 6);
      const uint32_t tile_key0 = static_cast<uint32_t>(page_lo + 2 * i) * kPage;
      const bool live_A = tile_key0 < hi_A && tile_key0 + kTileKeys > lo32;  // the tile holds keys of row A
      const bool live_B = tile_key0 < hi_B && tile_key0 + kTileKeys > lo32;
      float sc_A = 0.f, sc_B = 0.f;
      if (!aborted) {
        const uint32_t bph = static_cast<uint32_t>(i >> 1) & 1u;
        const bool ok = ptx::mbar_wait(bar_tfull + 8 * (2 * par + qp), bph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT,
                                       p.wait_ns);
        if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
        if (!aborted) {
          __syncwarp();
          ptx::tc_fence_after();
          const uint32_t ta = tmem + t_lane + static_cast<uint32_t>((2 * par + qp) * kPBufCols);
          if (live_A) sc_A = key_score(ta, w_A, scale);
          if (live_B) sc_B = key_score(ta + static_cast<uint32_t>(kHeads), w_B, scale);
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * (2 * par + qp));
        }
      }
      const uint32_t pos = tile_key0 + static_cast<uint32_t>(row);
      const bool in_range = !aborted && pos >= lo32;
      const uint64_t key_A = pack_key(sc_A, pos);
      const uint64_t key_B = pack_key(sc_B, pos);
      flush(pa, cand_A, nb_A);
      append(pa, misc_A, key_A, in_range && pos < hi_A && key_A >= thr_A);
      flush(pb, cand_B, nb_B);
      append(pb, misc_B, key_B, in_range && pos < hi_B && key_B >= thr_B);
      // Every check_every tile pairs the buffers may be nearly full: the
      // pair's eight warps meet, read each row's interval count, move to the
      // next counter and clear the one used two intervals ago; a row with
      // fewer than two tile pairs of room left is cut to exactly its best
      // 2048. The schedule depends only on tile counts, so both parities take
      // the same checks.
      if (++since == check_every) {
        since = 0;
        if ((i >> 1) < n_pairs_full) {
          flush(pa, cand_A, nb_A);
          flush(pb, cand_B, nb_B);
          ptx::named_bar(bar_qp, 256);
          const uint32_t n_A = nb_A + reinterpret_cast<volatile uint32_t*>(misc_A)[kPRot + slot];
          const uint32_t n_B = nb_B + reinterpret_cast<volatile uint32_t*>(misc_B)[kPRot + slot];
          if (gt == 0) {
            misc_A[kPRot + (slot + 2u) % 3u] = 0u;
            misc_B[kPRot + (slot + 2u) % 3u] = 0u;
          }
          nb_A = n_A;
          nb_B = n_B;
          slot = (slot + 1u) % 3u;
          if (n_A > static_cast<uint32_t>(kPCap - 4 * kTileKeys)) {
            thr_A = cut(cand_A, misc_A, n_A, jA);
            nb_A = reinterpret_cast<volatile uint32_t*>(misc_A)[kPCount];
          }
          if (n_B > static_cast<uint32_t>(kPCap - 4 * kTileKeys)) {
            thr_B = cut(cand_B, misc_B, n_B, jB);
            nb_B = reinterpret_cast<volatile uint32_t*>(misc_B)[kPCount];
          }
          const uint32_t room = kPCap - (nb_A > nb_B ? nb_A : nb_B);
          check_every = static_cast<int>(room / (2 * kTileKeys));
        }
      }
    }
    flush(pa, cand_A, nb_A);
    flush(pb, cand_B, nb_B);
    if (gt == 0) {  // read after the barrier below
      misc_A[kPFinal] = nb_A;
      misc_A[kPSel] = slot;  // the counter in use at the end (sel words are free now)
      misc_B[kPFinal] = nb_B;
      misc_B[kPSel] = slot;
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
    if ((warp == 1 || warp == kPMmaWarp1) && lane == 0 && mma_issued > 0) {
      const int last = mma_issued - 1;
      const int q = warp == 1 ? 0 : 1;
      ptx::mbar_wait(bar_tfull + 8 * (2 * (last & 1) + q), static_cast<uint32_t>(last >> 1) & 1u, &no_abort,
                     &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    }
    __syncthreads();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kPTmemCols);
  }
  if (warp < 2 || warp >= kPMmaWarp1) return;

  // ---- tail: the eight warps of row pair `pair` select and order its two rows ----
  const int pair = ((warp - 2) >> 2) & 1;
  const int pt = ((((warp - 2) & 3) + 4 * ((warp - 2) >> 3)) * 32) + lane;  // 0..255 within the pair
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
