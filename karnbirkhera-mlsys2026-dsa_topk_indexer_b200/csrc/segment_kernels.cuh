// Segment-scheduled indexer: three kernels launched back to back.
//
//   segment_plan_kernel    (1 CTA)   orders the rows longest first, cuts every
//                                    row into segments of `seg_tiles` tiles and
//                                    writes the segment list, the per-row slot
//                                    ranges and a zeroed work counter;
//   segment_stream_kernel  (2 CTAs per SM, persistent, no clusters) pulls
//                                    segments from the work counter and
//                                    streams them through the same pipeline as
//                                    indexer_kernel (TMA ring -> tcgen05 MMA ->
//                                    two epilogue groups) without draining
//                                    between segments; at a segment's end its
//                                    candidate keys (<= kSegCap) go to the
//                                    segment's workspace slot;
//   segment_merge_kernel   (one cluster of G CTAs per row) reads the row's
//                                    segment lists, filters them against a
//                                    running cut, then runs the cluster-wide
//                                    select / DSM exchange / ordering / emit of
//                                    cluster_select_emit.
//
// Every SM streams until the work runs out, whatever the row lengths, so HBM
// stays busy and no row waits for a later wave; the merges of all rows run in
// one short kernel afterwards. Candidate lists (8 bytes per surviving key, at
// most 3072 per segment) round-trip through L2/HBM; scores never do.
#pragma once
#include "indexer_kernel.cuh"

namespace dsa {

// Candidate keys per segment (the stream kernel's buffer and the length of a
// workspace list); sized so the stream kernel keeps two CTAs per SM.
constexpr int kSegCap = 3072;

// ------------------------------------------------------------------ plan
struct SegPlan {
  uint32_t* ctrl;        // [0] next segment to hand out, [1] number of segments
  int32_t* order;        // [B] rows, longest first
  int32_t* seg_first;    // [B] first slot of row b
  int32_t* seg_cnt;      // [B] segments of row b
  int4* segs;            // [slots] (row, first tile, end tile, slot)
};

constexpr int kSegPlanThreads = 1024;

__device__ __forceinline__ int row_tiles(const int32_t* seq_lens, int b, int max_pages) {
  int64_t len = seq_lens[b];
  const int64_t cap = static_cast<int64_t>(max_pages) * kPage;
  len = len < 0 ? 0 : (len > cap ? cap : len);
  return static_cast<int>((len + 2 * kPage - 1) / (2 * kPage));
}

// Block-wide exclusive scan of one value per thread (1024 threads).
__device__ __forceinline__ uint32_t plan_exclusive_scan(uint32_t v, uint32_t* wsum, uint32_t* total) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t x = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += x;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  uint32_t base = incl - v;
  for (int k = 0; k < w; ++k) base += wsum[k];
  if (t == kSegPlanThreads - 1) *total = base + v;
  __syncthreads();
  return base;
}

__global__ void __launch_bounds__(kSegPlanThreads, 1)
    segment_plan_kernel(const int32_t* __restrict__ seq_lens, int batch, int max_pages, int seg_tiles, SegPlan pl) {
  __shared__ uint32_t cnt[kPlanBuckets];
  __shared__ uint32_t start[kPlanBuckets];
  __shared__ uint32_t wsum[kSegPlanThreads / 32];
  __shared__ uint32_t total;
  const int t = threadIdx.x;
  ptx::grid_dep_launch();  // the stream kernel may start its prologue now
  const int max_tiles = (max_pages + 1) / 2;
  int shift = 0;
  while ((max_tiles >> shift) >= kPlanBuckets) ++shift;
  // 1. longest-first order (counting sort of the tile counts, descending)
  for (int i = t; i < kPlanBuckets; i += kSegPlanThreads) cnt[i] = 0u;
  __syncthreads();
  for (int b = t; b < batch; b += kSegPlanThreads) {
    atomicAdd(&cnt[(kPlanBuckets - 1) - (row_tiles(seq_lens, b, max_pages) >> shift)], 1u);
    if (static_cast<int64_t>(seq_lens[b]) > static_cast<int64_t>(max_pages) * kPage)
      atomicOr(&g_dsa_status, DSA_STATUS_SEQ_CLAMPED);
  }
  __syncthreads();
  {
    uint32_t c[4], s = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c[j] = cnt[4 * t + j];
      s += c[j];
    }
    uint32_t base = plan_exclusive_scan(s, wsum, &total);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      start[4 * t + j] = base;
      base += c[j];
    }
  }
  __syncthreads();
  for (int b = t; b < batch; b += kSegPlanThreads)
    pl.order[atomicAdd(&start[(kPlanBuckets - 1) - (row_tiles(seq_lens, b, max_pages) >> shift)], 1u)] = b;
  __syncthreads();
  // 2. segments per row, slots in longest-first row order (each thread owns
  //    a contiguous range of order positions)
  const int per = (batch + kSegPlanThreads - 1) / kSegPlanThreads;
  const int k0 = t * per < batch ? t * per : batch;
  const int k1 = k0 + per < batch ? k0 + per : batch;
  uint32_t mine = 0;
  for (int k = k0; k < k1; ++k) {
    const int tiles = row_tiles(seq_lens, pl.order[k], max_pages);
    mine += tiles > 0 ? static_cast<uint32_t>((tiles + seg_tiles - 1) / seg_tiles) : 1u;
  }
  uint32_t slot = plan_exclusive_scan(mine, wsum, &total);
  for (int k = k0; k < k1; ++k) {
    const int b = pl.order[k];
    const int tiles = row_tiles(seq_lens, b, max_pages);
    const int ns = tiles > 0 ? (tiles + seg_tiles - 1) / seg_tiles : 1;
    pl.seg_first[b] = static_cast<int32_t>(slot);
    pl.seg_cnt[b] = ns;
    for (int s = 0; s < ns; ++s) {
      const int lo = s * seg_tiles;
      const int hi = (lo + seg_tiles < tiles) ? lo + seg_tiles : tiles;
      pl.segs[slot] = make_int4(b, lo, hi, static_cast<int>(slot));
      ++slot;
    }
  }
  if (t == 0) {
    pl.ctrl[0] = 0u;
    pl.ctrl[1] = total;
  }
}

// ------------------------------------------------------------------ stream kernel layout
// Per-stage tile descriptor written by the producer, read by the MMA warp and
// the epilogue after the stage's full barrier.
struct TileDesc {
  int32_t b;       // row
  int32_t slot;    // segment slot (workspace index)
  int32_t pos0;    // logical position of the tile's first key
  int32_t key_hi;  // keys at positions >= key_hi are not visible
  int32_t t;       // tile index inside the segment
  int32_t flags;
  int32_t qb;      // query / weights buffer of the segment
  int32_t pad;
};
constexpr int kTileFirstPair = 1;  // t < 2
constexpr int kTileLastPair = 2;   // one of the segment's last two tiles
constexpr int kTileLast = 4;       // the segment's last tile
constexpr int kTileDummy = 8;      // padding tile (odd tile count): no keys
constexpr int kTileEnd = 16;       // no more work

constexpr int kS_OffK = 0;                                   // kStages x 16384
constexpr int kS_OffQ = kS_OffK + kStages * 16384;           // 2 x 8192 (swizzled)
constexpr int kS_OffScale = kS_OffQ + 2 * 8192;              // kStages x 512
constexpr int kS_OffW = kS_OffScale + kStages * 512;         // 2 x 256
constexpr int kS_OffDesc = kS_OffW + 2 * 256;                // kStages x 32
constexpr int kS_OffCand = kS_OffDesc + kStages * 32;        // kSegCap x 8
constexpr int kS_OffHist = kS_OffCand + kSegCap * 8;            // 256 x 4
constexpr int kS_OffBar = kS_OffHist + 256 * 4;              // 20 x 8
constexpr int kS_OffMisc = kS_OffBar + 256;                  // misc words
constexpr int kS_SmemUsed = kS_OffMisc + 128;
constexpr int kS_SmemBytes = kS_SmemUsed + 1024;
static_assert(kS_OffQ % 1024 == 0, "Q buffers must be 1024-aligned for the 128-byte swizzle");

struct StreamParams {
  const int32_t* seq_lens;
  const int32_t* block_table;
  const int4* segs;
  uint32_t* ctrl;
  uint64_t* ws_cand;  // [slots][kSegCap]
  uint32_t* ws_n;     // [slots]
  int64_t num_pages;
  int32_t max_pages;
  int32_t batch;
};

__global__ void __launch_bounds__(kThreads, 2)
    segment_stream_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_s,
                          const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_w,
                          const StreamParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);

  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kS_OffCand);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kS_OffHist);
  TileDesc* desc = reinterpret_cast<TileDesc*>(smem + kS_OffDesc);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + kS_OffMisc);
  uint32_t* misc_nv = reinterpret_cast<uint32_t*>(smem + kS_OffMisc);
  volatile uint32_t* abort_flag = misc + kMiscAbort;
  unsigned long long* mm = reinterpret_cast<unsigned long long*>(smem + kS_OffMisc + 4 * kMiscMM);

  const uint32_t bar_full = base_addr + kS_OffBar;         // [kStages]
  const uint32_t bar_empty = bar_full + 8 * kStages;       // [kStages]
  const uint32_t bar_tfull = bar_empty + 8 * kStages;      // [kTmemBufs]
  const uint32_t bar_tempty = bar_tfull + 8 * kTmemBufs;   // [kTmemBufs]
  const uint32_t bar_qfull = bar_tempty + 8 * kTmemBufs;   // [2]
  const uint32_t bar_qempty = bar_qfull + 16;              // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1 + 4);
    }
    for (int i = 0; i < kTmemBufs; ++i) {
      ptx::mbar_init(bar_tfull + 8 * i, 1);
      ptx::mbar_init(bar_tempty + 8 * i, 4);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_qfull + 8 * i, 1);
      ptx::mbar_init(bar_qempty + 8 * i, 2);  // last MMA commit of the segment + epilogue after its dump
    }
    ptx::fence_mbar_init();
    misc_nv[kMiscCount] = 0u;
    misc_nv[kMiscAbort] = 0u;
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_s);
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_w);
  }
  if (warp == 1) {
    ptx::tmem_alloc(base_addr + kS_OffMisc + 4 * kMiscTmem, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc_nv[kMiscTmem];
  // Barriers and TMEM are set up; from here on the plan's output is read.
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();  // the merge kernel may start its prologue once all CTAs got here

  int issued = 0, mma_issued = 0;
  bool aborted = false;

  if (warp == 0) {
    // ===================== producer: segments -> tiles =====================
    const uint64_t pol_stream = ptx::policy_evict_first();
    const uint64_t pol_keep = ptx::policy_evict_last();
    const uint32_t nseg = p.ctrl[1];
    int i = 0, lseg = 0;
    bool done = false;
#pragma unroll 1
    while (!done && !aborted) {
      uint32_t idx = 0;
      if (lane == 0) idx = atomicAdd(&p.ctrl[0], 1u);
      idx = __shfl_sync(0xFFFFFFFFu, idx, 0);
      int b = 0, tlo = 0, ntile = 0, slot = 0, npages = 0;
      int64_t len = 0;
      if (idx < nseg) {
        const int4 d = p.segs[idx];
        b = d.x;
        tlo = d.y;
        ntile = d.z - d.y;
        slot = d.w;
        len = p.seq_lens[b];
        const int64_t cap = static_cast<int64_t>(p.max_pages) * kPage;
        len = len < 0 ? 0 : (len > cap ? cap : len);
        npages = static_cast<int>((len + kPage - 1) / kPage);
        if (ntile <= 0) {
          if (lane == 0) p.ws_n[slot] = 0u;
          continue;
        }
      } else {
        done = true;
      }
      const int n_pad = done ? 2 : ntile + (ntile & 1);
      const int qb = lseg & 1;
      if (!done) {
        const bool ok = ptx::mbar_wait(bar_qempty + 8 * qb, (static_cast<uint32_t>(lseg >> 1) & 1u) ^ 1u, abort_flag,
                                       &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
        if (__any_sync(0xFFFFFFFFu, !ok)) {
          aborted = true;
          break;
        }
        if (lane == 0) {
          const uint32_t qf = bar_qfull + 8 * qb;
          ptx::mbar_arrive_expect_tx(qf, kHeads * kDim + kHeads * 4);
          ptx::tma_load_2d(base_addr + kS_OffQ + qb * 8192, &tm_q, qf, 0, b * kHeads, pol_keep);
          ptx::tma_load_2d(base_addr + kS_OffW + qb * 256, &tm_w, qf, 0, b, pol_keep);
        }
      }
      const int32_t* bt_row = p.block_table + static_cast<int64_t>(b) * p.max_pages;
      int32_t pg_batch = 0;
#pragma unroll 1
      for (int t = 0; t < n_pad; ++t, ++i) {
        if (!done && (t & 15) == 0) {
          const int pidx = 2 * (tlo + t) + lane;
          pg_batch = (pidx < npages) ? bt_row[pidx] : 0;
        }
        const int32_t pa = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * t) & 31);
        const int32_t pb = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * t + 1) & 31);
        const int s = i % kStages;
        const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
        const bool ok = ptx::mbar_wait(bar_empty + 8 * s, ph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
        if (__any_sync(0xFFFFFFFFu, !ok)) {
          aborted = true;
          break;
        }
        if (lane == 0) {
          const bool dummy = done || t >= ntile;
          const bool has_a = !dummy && 2 * (tlo + t) < npages;
          const bool has_b = !dummy && 2 * (tlo + t) + 1 < npages;
          TileDesc& d = desc[s];
          d.b = b;
          d.slot = slot;
          d.pos0 = 2 * (tlo + t) * kPage;
          d.key_hi = static_cast<int32_t>(len);
          d.t = t;
          d.flags = (t < 2 ? kTileFirstPair : 0) | (t >= n_pad - 2 ? kTileLastPair : 0) |
                    (t == n_pad - 1 ? kTileLast : 0) | (dummy ? kTileDummy : 0) | (done ? kTileEnd : 0);
          d.qb = qb;
          if ((has_a && static_cast<uint64_t>(static_cast<uint32_t>(pa)) >= static_cast<uint64_t>(p.num_pages)) ||
              (has_b && static_cast<uint64_t>(static_cast<uint32_t>(pb)) >= static_cast<uint64_t>(p.num_pages)))
            atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);
          const uint32_t bytes = (has_a ? kPageData + 256u : 0u) + (has_b ? kPageData + 256u : 0u);
          const uint32_t fb = bar_full + 8 * s;
          const uint32_t kdst = base_addr + kS_OffK + s * 16384;
          const uint32_t sdst = base_addr + kS_OffScale + s * 512;
          ptx::mbar_arrive_expect_tx(fb, bytes);
          if (has_a) {
            ptx::tma_load_3d(kdst, &tm_k, fb, 0, 0, pa, pol_stream);
            ptx::tma_load_2d(sdst, &tm_s, fb, 0, pa, pol_stream);
          }
          if (has_b) {
            ptx::tma_load_3d(kdst + kPageData, &tm_k, fb, 0, 0, pb, pol_stream);
            ptx::tma_load_2d(sdst + 256, &tm_s, fb, 0, pb, pol_stream);
          }
        }
        __syncwarp();
        issued = i + 1;
      }
      ++lseg;
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    constexpr uint32_t idesc = ptx::idesc_e4m3_f32(kTileKeys, kHeads);
    int lseg = 0;
#pragma unroll 1
    for (int i = 0;; ++i) {
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      bool ok = ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      const int flags = desc[s].flags;
      const int qb = desc[s].qb;
      if (flags & kTileEnd) break;
      if (desc[s].t == 0) {
        ok = ptx::mbar_wait(bar_qfull + 8 * qb, static_cast<uint32_t>(lseg >> 1) & 1u, abort_flag, &g_dsa_status,
                            DSA_STATUS_WAIT_TIMEOUT);
        ++lseg;
      }
      const int buf = i % kTmemBufs;
      const uint32_t bph = static_cast<uint32_t>(i / kTmemBufs) & 1u;
      ok = ok && ptx::mbar_wait(bar_tempty + 8 * buf, bph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      __syncwarp();
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint64_t adesc = ptx::sw128_kmajor_desc(base_addr + kS_OffK + s * 16384);
        const uint64_t qdesc = ptx::sw128_kmajor_desc(base_addr + kS_OffQ + qb * 8192);
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kHeads);
#pragma unroll
        for (int kk = 0; kk < kDim / 32; ++kk)
          ptx::mma_f8f6f4(d, adesc + 2ull * kk, qdesc + 2ull * kk, idesc, kk > 0 ? 1u : 0u);
        ptx::mma_commit(bar_empty + 8 * s);
        ptx::mma_commit(bar_tfull + 8 * buf);
        if (flags & kTileLast) ptx::mma_commit(bar_qempty + 8 * qb);
      }
      __syncwarp();
      mma_issued = i + 1;
    }
  } else {
    // ===================== epilogue: two groups of four warps =====================
    const int grp = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int et = threadIdx.x - 64;
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    uint64_t thr = 0;
    int since = 0;
    int check_every = kSegCap / (2 * kTileKeys);
    int lseg = 0;
#pragma unroll 1
    for (int i = grp;; i += 2) {
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      bool ok = ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      const TileDesc d = desc[s];
      if (d.flags & kTileEnd) break;
      if (d.flags & kTileFirstPair) {
        ok = ptx::mbar_wait(bar_qfull + 8 * d.qb, static_cast<uint32_t>(lseg >> 1) & 1u, abort_flag, &g_dsa_status,
                            DSA_STATUS_WAIT_TIMEOUT);
        if (__any_sync(0xFFFFFFFFu, !ok)) {
          aborted = true;
          break;
        }
      }
      // Read this stage's scale (and descriptor, above) before releasing the
      // stage; the proxy fence orders these generic reads before the
      // producer's next TMA write into the stage.
      const float scale = ptx::lds_f32_ordered(base_addr + kS_OffScale + 4u * (s * kTileKeys + row));
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
      const int buf = i % kTmemBufs;
      const uint32_t bph = static_cast<uint32_t>(i / kTmemBufs) & 1u;
      ok = ptx::mbar_wait(bar_tfull + 8 * buf, bph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      __syncwarp();
      ptx::tc_fence_after();
      const float* s_w = reinterpret_cast<const float*>(smem + kS_OffW + d.qb * 256);
      float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      {
        uint32_t acc[32];
        const uint32_t ta = tmem + t_lane + static_cast<uint32_t>(buf * kHeads);
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
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * buf);

      const float score =
          (((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]))) *
          fabsf(scale);
      const int32_t pos = d.pos0 + row;
      const bool valid = !(d.flags & kTileDummy) && pos < d.key_hi;
      const uint64_t key = pack_key(score, static_cast<uint32_t>(pos));
      const bool keep = valid && key >= thr;
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      if (m) {
        const int leader = __ffs(m) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(misc_nv + kMiscCount, static_cast<uint32_t>(__popc(m)));
        base = __shfl_sync(0xFFFFFFFFu, base, leader);
        if (keep) cand[base + __popc(m & lanemask_lt())] = key;
      }
      if (d.flags & kTileLastPair) {
        // End of the segment: both groups meet, the candidates go to the
        // segment's workspace slot and the buffer starts empty again.
        ptx::named_bar(kBarEpi, kEpiThreads);
        const uint32_t n = misc[kMiscCount];
        uint64_t* dst = p.ws_cand + static_cast<size_t>(d.slot) * kSegCap;
        for (uint32_t j = et; j < n; j += kEpiThreads) dst[j] = cand[j];
        if (et == 0) {
          p.ws_n[d.slot] = n;
          misc_nv[kMiscCount] = 0u;
        }
        ptx::named_bar(kBarEpi, kEpiThreads);
        if (et == 0) ptx::mbar_arrive(bar_qempty + 8 * d.qb);  // weights of this segment no longer read
        thr = 0;
        since = 0;
        check_every = kSegCap / (2 * kTileKeys);
        ++lseg;
      } else if (++since == check_every) {
        // Same cut schedule as indexer_kernel, within the segment.
        since = 0;
        ptx::named_bar(kBarEpi, kEpiThreads);
        uint32_t n = misc[kMiscCount];
        if (et == 0) {
          mm[0] = ~0ull;
          mm[1] = 0ull;
        }
        ptx::named_bar(kBarEpi, kEpiThreads);
        if (n > static_cast<uint32_t>(kSegCap - 4 * kTileKeys)) {  // fewer than two tile pairs of room
          group_minmax<kEpiThreads, kBarEpi>(cand, n, mm, et);
          uint32_t kept = 0;
          uint64_t T = group_cut<kEpiThreads, kBarEpi>(cand, n, kTopK, mm, hist, misc_nv + kMiscSel, et, &kept);
          if (kept > static_cast<uint32_t>(kSegCap - 4 * kTileKeys))
            T = group_select<kEpiThreads, kBarEpi>(cand, n, kTopK, mm, hist, misc_nv + kMiscSel, et);
          group_compact<kEpiThreads, kBarEpi, kSegCap / kEpiThreads>(cand, n, T, misc_nv + kMiscCount, misc_nv + kMiscWsum, et);
          thr = T;
          n = misc[kMiscCount];
        }
        check_every = static_cast<int>((kSegCap - n) / (2 * kTileKeys));
      }
    }
  }

  // ---- teardown ----
  if (aborted) *abort_flag = 1u;
  ptx::tc_fence_before();
  __syncthreads();
  if (misc[kMiscAbort] != 0u) {
    volatile uint32_t no_abort = 0u;
    if (warp == 0 && lane == 0) {
      for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
        ptx::mbar_wait(bar_full + 8 * (i % kStages), static_cast<uint32_t>(i / kStages) & 1u, &no_abort,
                       &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
    }
    if (warp == 1 && lane == 0 && mma_issued > 0) {
      const int last = mma_issued - 1;
      ptx::mbar_wait(bar_tfull + 8 * (last % kTmemBufs), static_cast<uint32_t>(last / kTmemBufs) & 1u,
                     &no_abort, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
    }
    __syncthreads();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ merge kernel
// One cluster of G CTAs per row (rows in the plan's longest-first order). CTA
// r copies segment lists r, r+G, ... of its row from the workspace into one
// large shared-memory buffer with asynchronous 8-byte copies (no register
// round trip, no barrier per list); only when the next lists would not fit is
// the buffer cut back to its exact best 2048. Then the cluster selects,
// exchanges, orders and emits exactly as the streaming cluster kernel does.
struct MergeParams {
  const int32_t* order;
  const int32_t* seg_first;
  const int32_t* seg_cnt;
  const uint64_t* ws_cand;
  const uint32_t* ws_n;
};

constexpr int kMergeKeys = 11264;                             // candidate keys per merge CTA
constexpr int kM_OffFinal = 0;                                // 2048 x 8 (remote survivors)
constexpr int kM_OffCand = kM_OffFinal + kTopK * 8;           // kMergeKeys x 8
constexpr int kM_OffHist = kM_OffCand + kMergeKeys * 8;       // 2 x 256 x 4
constexpr int kM_OffTot = kM_OffHist + 2 * 256 * 4;           // 256 x 4
constexpr int kM_OffSegN = kM_OffTot + 256 * 4;               // kThreads x 4: list lengths
constexpr int kM_OffSegOff = kM_OffSegN + kThreads * 4;       // kThreads x 4: list offsets
constexpr int kM_OffWsum = kM_OffSegOff + kThreads * 4;       // 16 x 4
constexpr int kM_OffMisc = kM_OffWsum + 64;                   // misc words
constexpr int kM_SmemBytes = kM_OffMisc + 128 + 1024;
static_assert(kMergeKeys >= 2 * kSegCap + kTopK, "a cut buffer must take two more lists");
static_assert(kTopK * 8 + 3 * 2048 * 4 + kTopK * 2 <= kMergeKeys * 8, "ordering scratch must fit in the candidate buffer");
static_assert(2 * (kM_SmemBytes + 1024) <= 233472, "two merge CTAs per SM");

struct MergeSelectLayout {
  static constexpr bool kSolo = false;
  static constexpr int kSoloTmp = 0, kSoloD = 0, kSoloCnt = 0;
  static constexpr int kCand = kM_OffCand, kHist = kM_OffHist, kTot = kM_OffTot, kMisc = kM_OffMisc;
  static constexpr int kFinal = kM_OffFinal, kRankTmp = kM_OffCand, kRankCnt = kM_OffCand + kTopK * 8;
  static constexpr int kRankD = kRankCnt + 3 * 2048 * 4;
};

// Inclusive scan of one value per thread over the CTA's kThreads threads;
// *total receives the sum. Contains two __syncthreads.
__device__ __forceinline__ uint32_t cta_inclusive_scan(uint32_t v, uint32_t* wsum, uint32_t* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t x = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += x;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  uint32_t base = 0, tot = 0;
#pragma unroll
  for (int k = 0; k < kThreads / 32; ++k) {
    const uint32_t x = wsum[k];
    base += (k < w) ? x : 0u;
    tot += x;
  }
  *total = tot;
  __syncthreads();
  return base + incl;
}

__global__ void __launch_bounds__(kThreads, 2)
    segment_merge_kernel(const MergeParams mp, const IndexerParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kM_OffCand);
  uint64_t* fin = reinterpret_cast<uint64_t*>(smem + kM_OffFinal);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kM_OffHist);
  uint32_t* seg_n = reinterpret_cast<uint32_t*>(smem + kM_OffSegN);
  uint32_t* seg_off = reinterpret_cast<uint32_t*>(smem + kM_OffSegOff);
  uint32_t* wsum = reinterpret_cast<uint32_t*>(smem + kM_OffWsum);
  uint32_t* misc_nv = reinterpret_cast<uint32_t*>(smem + kM_OffMisc);
  volatile uint32_t* misc = misc_nv;
  unsigned long long* mm = reinterpret_cast<unsigned long long*>(smem + kM_OffMisc + 4 * kMiscMM);
  const int tid = threadIdx.x;
  const uint32_t G = ptx::cluster_nctarank();
  const uint32_t rank = ptx::cluster_ctarank();
  ptx::grid_dep_wait();  // the stream kernel's lists are complete and visible
  const int b = mp.order[blockIdx.x / G];
  const int first = mp.seg_first[b], nseg = mp.seg_cnt[b];
  const int mine = nseg > static_cast<int>(rank) ? (nseg - static_cast<int>(rank) + static_cast<int>(G) - 1) / static_cast<int>(G) : 0;
  const uint32_t cand_addr = base_addr + kM_OffCand;
  uint32_t n = 0;
#pragma unroll 1
  for (int c0 = 0; c0 < mine;) {
    // Lengths of the next (up to kThreads) lists, their offsets in the
    // buffer, and how many of them fit behind the n keys already held.
    const int j = c0 + tid;
    const uint32_t m = j < mine ? mp.ws_n[first + static_cast<int>(rank) + j * static_cast<int>(G)] : 0u;
    uint32_t chunk = 0;
    const uint32_t incl = cta_inclusive_scan(m, wsum, &chunk);
    const bool fits = j < mine && n + incl <= static_cast<uint32_t>(kMergeKeys);
    seg_n[tid] = m;
    seg_off[tid] = n + incl - m;
    const int nfit = __syncthreads_count(fits);
    uint32_t added = 0;
#pragma unroll 1
    for (int k = 0; k < nfit; ++k) {
      const uint32_t mk = seg_n[k];
      const uint32_t dst = cand_addr + 8u * seg_off[k];
      const uint64_t* src = mp.ws_cand + static_cast<size_t>(first + static_cast<int>(rank) + (c0 + k) * static_cast<int>(G)) * kSegCap;
      for (uint32_t i = tid; i < mk; i += kThreads) ptx::cp_async8(dst + 8u * i, src + i);
      added += mk;
    }
    ptx::cp_async_wait_all();
    __syncthreads();
    n += added;
    c0 += nfit;
    if (c0 < mine && n > static_cast<uint32_t>(kMergeKeys - kSegCap)) {
      // The next list may not fit: keep the exact best 2048 (staged through
      // the survivor area, which no other CTA writes before the cluster
      // select below).
      if (tid == 0) {
        mm[0] = ~0ull;
        mm[1] = 0ull;
      }
      __syncthreads();
      group_minmax<kThreads, 0>(cand, n, mm, tid);
      const uint64_t T = group_select<kThreads, 0>(cand, n, kTopK, mm, hist, misc_nv + kMiscSel, tid);
      uint32_t wlo, whi, kept = 0;
      warp_range(n, tid >> 5, kThreads / 32, &wlo, &whi);
      const uint32_t wbase = group_warp_offset<kThreads, 0>(warp_count_ge(cand, wlo, whi, T), wsum, &kept, tid);
      warp_write_ge(cand, wlo, whi, T, base_addr + kM_OffFinal + 8u * wbase);
      if (tid == 0) misc_nv[kMiscCount] = kept;
      __syncthreads();
      n = misc[kMiscCount];
      for (uint32_t i = tid; i < n; i += kThreads) cand[i] = fin[i];
      __syncthreads();
    }
  }
  __syncthreads();
  cluster_select_emit<kModeTopK, MergeSelectLayout>(smem, base_addr, n, G, rank, b,
                                                    p.block_table + static_cast<int64_t>(b) * p.max_pages, p);
}

}  // namespace dsa
