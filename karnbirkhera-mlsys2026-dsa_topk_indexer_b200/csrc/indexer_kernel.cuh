// Fused paged-gather + tcgen05 scoring + cluster top-K kernel.
//
// One thread-block cluster of G CTAs serves one request (one query row).
// The request's pages are cut into tiles of two pages (128 keys, the MMA M
// dimension) and the tiles are split evenly over the G CTAs. Each CTA is
// warp-specialised:
//   warp 0      TMA producer: per tile, two 8 KB page-data boxes (128-byte
//               swizzle) and two 256 B scale rows into a 4-stage ring;
//   warp 1      TMEM owner and MMA issuer: D[128 keys x 64 heads] (fp32, TMEM,
//               double-buffered) = K_tile[128 x 128 e4m3] . Q[64 x 128 e4m3]^T
//               as four tcgen05.mma kind::f8f6f4 (K = 32 each);
//   warps 2..5  epilogue: thread = TMEM lane = key; tcgen05.ld of its 64
//               head columns, relu / head-weight / scale reduction in
//               registers, then a threshold filter into a shared-memory
//               candidate buffer with periodic exact compaction to the best
//               2048;
//   all warps   after the stream: cluster-wide radix select of the best 2048
//               over every CTA's candidates (histograms summed through
//               distributed shared memory), survivors written into CTA 0's
//               shared memory, sorted there and translated to physical slots.
// Scores never go to HBM in the top-K modes.
//
// Reference counterparts: fp8_mma_final_scores_kernel
// (solution/cuda/kernel.cu:209-452) for the scoring, and
// block_topk_translate{,_small,_tiny,_cluster}_kernel (:472-813) for the
// selection and translation.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"
#include "select.cuh"
#include "dsa_topk_indexer.h"

namespace dsa {

constexpr int kHeads = 64;
constexpr int kDim = 128;
constexpr int kPage = 64;
constexpr int kPageBytes = 8448;
constexpr int kPageData = 8192;
constexpr int kTileKeys = 128;
constexpr int kStages = 4;
constexpr int kThreads = 256;
constexpr int kCap = 3072;  // candidate keys per CTA (>= 2048 + 128 * 8)
constexpr int kTmemCols = 128;

enum Mode : int { kModeTopK = 0, kModeScores = 1, kModePartial = 2 };

// Shared memory map (byte offsets from a 1024-aligned base).
constexpr int kOffK = 0;                                  // kStages x 16384, swizzled K tiles
constexpr int kOffQ = kOffK + kStages * 16384;            // 8192, swizzled Q
constexpr int kOffScale = kOffQ + 8192;                   // kStages x 512 (128 fp32)
constexpr int kOffCand = kOffScale + kStages * 512;       // kCap x 8
constexpr int kOffHist = kOffCand + kCap * 8;             // 2 x 256 x 4
constexpr int kOffTot = kOffHist + 2 * 256 * 4;           // 256 x 4
constexpr int kOffW = kOffTot + 256 * 4;                  // 64 x 4
constexpr int kOffBar = kOffW + 256;                      // (2*kStages + 5) x 8
constexpr int kOffMisc = kOffBar + 128;                   // small words
constexpr int kSmemUsed = kOffMisc + 128;
constexpr int kSmemBytes = kSmemUsed + 1024;              // alignment slack
constexpr int kOffFinal = kOffK;                          // 2048 x 8, reuses the K ring after the stream
static_assert(kOffFinal + kTopK * 8 <= kOffQ, "final buffer must fit in the K ring");
static_assert(kStages * 16384 % 1024 == 0, "K tiles must stay 1024-aligned");

// Misc word indices (uint32 at kOffMisc).
enum MiscWord : int {
  kMiscTmem = 0,   // TMEM base address
  kMiscCount = 1,  // candidates in the buffer
  kMiscAbort = 2,  // pipeline abort flag
  kMiscSel = 4,    // 3 words: digit scan result
  kMiscPub = 8,    // 2 words read by other CTAs of the cluster
  kMiscTotal = 10,
  kMiscOffset = 11,
  kMiscWrite = 12,
};

struct IndexerParams {
  const int32_t* seq_lens;     // [B]
  const int32_t* block_table;  // [B, max_pages]
  const float* weights;        // [B, 64]
  int32_t* out;                // kModeTopK: [B, 2048]
  float* scores;               // kModeScores: [B, score_stride]
  float* cand_scores;          // kModePartial: [B, 2048]
  int32_t* cand_pos;           // kModePartial: [B, 2048]
  int64_t score_stride;
  int64_t key_begin, key_end;  // kModePartial key range
  int64_t num_pages;
  int32_t max_pages;
  int32_t batch;
};

__device__ unsigned int g_dsa_status;

// score = sum_h w_h * relu(scale * acc_h), evaluated as
// |scale| * sum_h w_h * relu(sign(scale) * acc_h): the scale is applied once
// per key instead of once per head (exact up to fp32 rounding, any sign).
__device__ __forceinline__ float head_reduce(const uint32_t (&acc)[64], const float* s_w,
                                             float scale) {
  const float4* w4 = reinterpret_cast<const float4*>(s_w);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (scale >= 0.f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = w4[j];
      s0 = fmaf(w.x, fmaxf(__uint_as_float(acc[4 * j + 0]), 0.f), s0);
      s1 = fmaf(w.y, fmaxf(__uint_as_float(acc[4 * j + 1]), 0.f), s1);
      s2 = fmaf(w.z, fmaxf(__uint_as_float(acc[4 * j + 2]), 0.f), s2);
      s3 = fmaf(w.w, fmaxf(__uint_as_float(acc[4 * j + 3]), 0.f), s3);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = w4[8 + j];
      s0 = fmaf(w.x, fmaxf(__uint_as_float(acc[32 + 4 * j + 0]), 0.f), s0);
      s1 = fmaf(w.y, fmaxf(__uint_as_float(acc[32 + 4 * j + 1]), 0.f), s1);
      s2 = fmaf(w.z, fmaxf(__uint_as_float(acc[32 + 4 * j + 2]), 0.f), s2);
      s3 = fmaf(w.w, fmaxf(__uint_as_float(acc[32 + 4 * j + 3]), 0.f), s3);
    }
    return ((s0 + s1) + (s2 + s3)) * scale;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 w = w4[j];
    s0 = fmaf(w.x, fmaxf(-__uint_as_float(acc[4 * j + 0]), 0.f), s0);
    s1 = fmaf(w.y, fmaxf(-__uint_as_float(acc[4 * j + 1]), 0.f), s1);
    s2 = fmaf(w.z, fmaxf(-__uint_as_float(acc[4 * j + 2]), 0.f), s2);
    s3 = fmaf(w.w, fmaxf(-__uint_as_float(acc[4 * j + 3]), 0.f), s3);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 w = w4[8 + j];
    s0 = fmaf(w.x, fmaxf(-__uint_as_float(acc[32 + 4 * j + 0]), 0.f), s0);
    s1 = fmaf(w.y, fmaxf(-__uint_as_float(acc[32 + 4 * j + 1]), 0.f), s1);
    s2 = fmaf(w.z, fmaxf(-__uint_as_float(acc[32 + 4 * j + 2]), 0.f), s2);
    s3 = fmaf(w.w, fmaxf(-__uint_as_float(acc[32 + 4 * j + 3]), 0.f), s3);
  }
  return ((s0 + s1) + (s2 + s3)) * (-scale);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 2)
    indexer_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_s,
                   const __grid_constant__ CUtensorMap tm_q, const IndexerParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);

  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kOffCand);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kOffHist);
  uint32_t* tot = reinterpret_cast<uint32_t*>(smem + kOffTot);
  float* s_w = reinterpret_cast<float*>(smem + kOffW);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc);
  uint32_t* misc_nv = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile uint32_t* abort_flag = misc + kMiscAbort;

  const uint32_t bar_full = base_addr + kOffBar;              // [kStages]
  const uint32_t bar_empty = bar_full + 8 * kStages;          // [kStages]
  const uint32_t bar_tfull = bar_empty + 8 * kStages;         // [2]
  const uint32_t bar_tempty = bar_tfull + 16;                 // [2]
  const uint32_t bar_q = bar_tempty + 16;                     // [1]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t G = ptx::cluster_nctarank();
  const uint32_t rank = ptx::cluster_ctarank();
  const int b = static_cast<int>(blockIdx.x / G);

  // ---- request geometry (identical in every thread) ----
  int64_t len = p.seq_lens[b];
  const int64_t cap_keys = static_cast<int64_t>(p.max_pages) * kPage;
  if (len < 0) len = 0;
  if (len > cap_keys) {
    len = cap_keys;
    if (threadIdx.x == 0 && rank == 0) atomicOr(&g_dsa_status, DSA_STATUS_SEQ_CLAMPED);
  }
  int64_t key_lo = 0, key_hi = len;
  if (kMode == kModePartial) {
    key_lo = p.key_begin < 0 ? 0 : p.key_begin;
    key_hi = p.key_end < len ? p.key_end : len;
    if (key_hi < key_lo) key_hi = key_lo;
  }
  const int page_lo = static_cast<int>(key_lo / kPage);
  const int page_hi = static_cast<int>((key_hi + kPage - 1) / kPage);
  const int n_tiles = (page_hi - page_lo + 1) / 2;
  const int t0 = static_cast<int>((static_cast<int64_t>(n_tiles) * rank) / G);
  const int t1 = static_cast<int>((static_cast<int64_t>(n_tiles) * (rank + 1)) / G);
  const int my_tiles = t1 - t0;
  const int pg_first = page_lo + 2 * t0;
  const int pg_end = (page_lo + 2 * t1 < page_hi) ? page_lo + 2 * t1 : page_hi;
  const int32_t* bt_row = p.block_table + static_cast<int64_t>(b) * p.max_pages;

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1 + 4);  // MMA commit + 4 epilogue warps (scales read)
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_tfull + 8 * i, 1);
      ptx::mbar_init(bar_tempty + 8 * i, 4);
    }
    ptx::mbar_init(bar_q, 1);
    ptx::fence_mbar_init();
    misc_nv[kMiscCount] = 0u;
    misc_nv[kMiscAbort] = 0u;
    misc_nv[kMiscPub + 1] = 0u;
    misc_nv[kMiscWrite] = 0u;
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_s);
    ptx::prefetch_tmap(&tm_q);
  }
  if (warp == 1) {
    ptx::tmem_alloc(base_addr + kOffMisc + 4 * kMiscTmem, kTmemCols);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x < kHeads) s_w[threadIdx.x] = p.weights[static_cast<int64_t>(b) * kHeads + threadIdx.x];
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc_nv[kMiscTmem];

  int issued = 0;       // producer: tiles whose loads were issued
  int mma_issued = 0;   // MMA warp: tiles whose MMAs were issued
  bool aborted = false;

  if (warp == 0) {
    // ===================== TMA producer =====================
    const uint64_t pol_stream = ptx::policy_evict_first();
    if (my_tiles > 0 && lane == 0) {
      ptx::mbar_arrive_expect_tx(bar_q, kHeads * kDim);
      ptx::tma_load_2d(base_addr + kOffQ, &tm_q, bar_q, 0, b * kHeads, ptx::policy_evict_last());
    }
    int32_t pg_batch = 0;
#pragma unroll 1
    for (int i = 0; i < my_tiles; ++i) {
      if ((i & 15) == 0) {
        const int pidx = pg_first + 2 * i + lane;
        pg_batch = (pidx < pg_end) ? bt_row[pidx] : 0;
      }
      const int32_t pa = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * i) & 31);
      const int32_t pb = __shfl_sync(0xFFFFFFFFu, pg_batch, (2 * i + 1) & 31);
      const bool has_b = (pg_first + 2 * i + 1) < pg_end;
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      const bool ok = ptx::mbar_wait(bar_empty + 8 * s, ph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      if (lane == 0) {
        if (static_cast<uint64_t>(static_cast<uint32_t>(pa)) >= static_cast<uint64_t>(p.num_pages) ||
            (has_b && static_cast<uint64_t>(static_cast<uint32_t>(pb)) >= static_cast<uint64_t>(p.num_pages)))
          atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);  // TMA zero-fills out-of-range boxes
        const uint32_t bytes = has_b ? 2u * (kPageData + 256u) : (kPageData + 256u);
        const uint32_t fb = bar_full + 8 * s;
        const uint32_t kdst = base_addr + kOffK + s * 16384;
        const uint32_t sdst = base_addr + kOffScale + s * 512;
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
    constexpr uint32_t idesc = ptx::idesc_e4m3_f32(kTileKeys, kHeads);
    bool ok = true;
    if (my_tiles > 0) ok = ptx::mbar_wait(bar_q, 0u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
    if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
    const uint64_t qdesc = ptx::sw128_kmajor_desc(base_addr + kOffQ);
#pragma unroll 1
    for (int i = 0; i < my_tiles && !aborted; ++i) {
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      const int buf = i & 1;
      const uint32_t bph = static_cast<uint32_t>(i >> 1) & 1u;
      ok = ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT) &&
           ptx::mbar_wait(bar_tempty + 8 * buf, bph ^ 1u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      __syncwarp();
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint64_t adesc = ptx::sw128_kmajor_desc(base_addr + kOffK + s * 16384);
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kHeads);
#pragma unroll
        for (int kk = 0; kk < kDim / 32; ++kk)
          ptx::mma_f8f6f4(d, adesc + 2ull * kk, qdesc + 2ull * kk, idesc, kk > 0 ? 1u : 0u);
        ptx::mma_commit(bar_empty + 8 * s);
        ptx::mma_commit(bar_tfull + 8 * buf);
      }
      __syncwarp();
      mma_issued = i + 1;
    }
  } else if (warp < 6) {
    // ===================== epilogue =====================
    const int q4 = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;     // key row inside the 128-key tile
    const int et = threadIdx.x - 64;    // 0..127 inside the epilogue group
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    uint64_t thr = 0;                   // keys below thr can no longer reach the top 2048
    int since = 0;
    int check_every = kCap / kTileKeys;
#pragma unroll 1
    for (int i = 0; i < my_tiles; ++i) {
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      bool ok = ptx::mbar_wait(bar_full + 8 * s, ph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      // The scale is read with a generic-proxy load, and the producer's next
      // TMA into this stage writes through the async proxy as soon as the MMA
      // commit and all four epilogue warps have arrived. Without the proxy
      // fence that write-after-read is unordered: on L2-resident pages the
      // refill landed first and the key was scaled by the scale of the tile
      // four steps ahead.
      const float scale = ptx::lds_f32_ordered(base_addr + kOffScale + 4u * (s * kTileKeys + row));
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_empty + 8 * s);
      const int buf = i & 1;
      const uint32_t bph = static_cast<uint32_t>(i >> 1) & 1u;
      ok = ptx::mbar_wait(bar_tfull + 8 * buf, bph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        aborted = true;
        break;
      }
      __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
      ptx::tc_fence_after();
      uint32_t acc[64];
      ptx::tmem_ld_32x32b_x64_sync(tmem + t_lane + static_cast<uint32_t>(buf * kHeads), acc);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * buf);

      const float score = head_reduce(acc, s_w, scale);
      const int64_t pos = static_cast<int64_t>(pg_first + 2 * i) * kPage + row;
      const bool valid = pos >= key_lo && pos < key_hi;
      if (kMode == kModeScores) {
        if (valid) p.scores[static_cast<int64_t>(b) * p.score_stride + pos] = score;
      } else {
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
        // Every check_every tiles the buffer may be full: compact it to the
        // exact best 2048 and raise the threshold. The schedule depends only
        // on tile counts, so all four warps take the same barriers.
        if (++since == check_every) {
          ptx::named_bar(1, 128);
          uint32_t n = misc[kMiscCount];
          ptx::named_bar(1, 128);
          if (n > static_cast<uint32_t>(kTopK)) {
            thr = group_select<128, 1>(cand, n, kTopK, hist, misc_nv + kMiscSel, et);
            group_compact<128, 1, kCap / 128>(cand, n, thr, misc_nv + kMiscCount, et);
            n = kTopK;
          }
          since = 0;
          check_every = static_cast<int>((kCap - n) / kTileKeys);
        }
      }
    }
  }
  // ---- end of the stream: drain, release TMEM ----
  if (aborted) *abort_flag = 1u;
  ptx::tc_fence_before();
  __syncthreads();
  if (misc[kMiscAbort] != 0u) {
    // A wait gave up. Before TMEM is freed and the CTA can exit, wait (again
    // bounded) for the loads and MMAs this CTA has in flight.
    volatile uint32_t no_abort = 0u;
    if (warp == 0 && lane == 0) {
      for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
        ptx::mbar_wait(bar_full + 8 * (i % kStages), static_cast<uint32_t>(i / kStages) & 1u, &no_abort,
                       &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
    }
    if (warp == 1 && lane == 0 && mma_issued > 0) {
      const int last = mma_issued - 1;
      ptx::mbar_wait(bar_tfull + 8 * (last & 1), static_cast<uint32_t>(last >> 1) & 1u, &no_abort,
                     &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
    }
    __syncthreads();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
  if (kMode == kModeScores) return;

  // ---- cluster-wide exact selection of the best 2048 keys ----
  const int tid = threadIdx.x;
  const uint32_t n = misc_nv[kMiscCount];
  const uint32_t pub_addr = base_addr + kOffMisc + 4 * kMiscPub;
  if (tid == 0) misc_nv[kMiscPub] = n;
  ptx::cluster_sync();
  if (warp == 0) {
    uint32_t v = (static_cast<uint32_t>(lane) < G) ? ptx::ld_dsmem_u32(ptx::mapa(pub_addr, lane)) : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (lane == 0) misc_nv[kMiscTotal] = v;
  }
  __syncthreads();
  const uint32_t total = misc_nv[kMiscTotal];
  uint64_t T = 0;
  if (total > static_cast<uint32_t>(kTopK)) {
    uint64_t prefix = 0;
    uint32_t krem = kTopK;
    int pass = 0;
#pragma unroll 1
    for (int shift = 56; shift >= 0; shift -= 8, ++pass) {
      uint32_t* hb = hist + (pass & 1) * 256;
      hb[tid] = 0u;
      __syncthreads();
      const uint64_t hi_mask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
      for (uint32_t i0 = 0; i0 < n; i0 += kThreads) {
        const uint32_t i = i0 + tid;
        const uint64_t key = i < n ? cand[i] : 0ull;
        warp_hist_add(hb, i < n && (key & hi_mask) == prefix, static_cast<uint32_t>(key >> shift) & 255u);
      }
      ptx::cluster_sync();  // every CTA's histogram of this pass is complete
      const uint32_t hb_addr = ptx::smem_addr(hb + tid);
      uint32_t sum = 0;
      for (uint32_t r = 0; r < G; ++r) sum += ptx::ld_dsmem_u32(ptx::mapa(hb_addr, r));
      tot[tid] = sum;
      __syncthreads();
      if (warp == 0) find_digit_warp(tot, krem, misc_nv + kMiscSel);
      __syncthreads();
      const uint32_t d = misc_nv[kMiscSel], cgt = misc_nv[kMiscSel + 1], cd = misc_nv[kMiscSel + 2];
      prefix |= static_cast<uint64_t>(d) << shift;
      krem -= cgt;
      if (cd == krem) break;
    }
    T = prefix;
  }
  // Count this CTA's survivors, publish, and get this CTA's output offset.
  {
    uint32_t c = 0;
    for (uint32_t i = tid; i < n; i += kThreads) c += (cand[i] >= T) ? 1u : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, off);
    if (lane == 0 && c) atomicAdd(misc_nv + kMiscPub + 1, c);
  }
  ptx::cluster_sync();
  if (warp == 0) {
    uint32_t v = (static_cast<uint32_t>(lane) < rank) ? ptx::ld_dsmem_u32(ptx::mapa(pub_addr + 4, lane)) : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (lane == 0) misc_nv[kMiscOffset] = v;
  }
  __syncthreads();
  const uint32_t nsel = total < static_cast<uint32_t>(kTopK) ? total : static_cast<uint32_t>(kTopK);
  {
    const uint32_t my_off = misc_nv[kMiscOffset];
    const uint32_t fin_remote = ptx::mapa(base_addr + kOffFinal, 0);
#pragma unroll 1
    for (uint32_t i0 = 0; i0 < n; i0 += kThreads) {
      const uint32_t i = i0 + tid;
      const uint64_t key = (i < n) ? cand[i] : 0ull;
      const bool keep = (i < n) && key >= T;
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      if (m) {
        const int leader = __ffs(m) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(misc_nv + kMiscWrite, static_cast<uint32_t>(__popc(m)));
        base = __shfl_sync(0xFFFFFFFFu, base, leader);
        if (keep) ptx::st_dsmem_u64(fin_remote + 8u * (my_off + base + __popc(m & lanemask_lt())), key);
      }
    }
    if (rank == 0) {
      uint64_t* fin = reinterpret_cast<uint64_t*>(smem + kOffFinal);
      for (uint32_t i = nsel + tid; i < static_cast<uint32_t>(kTopK); i += kThreads) fin[i] = 0ull;
    }
  }
  ptx::cluster_sync();
  if (rank != 0) return;

  // ---- CTA 0: sort the survivors and emit ----
  uint64_t v[8];
  block_sort_desc_2048(reinterpret_cast<uint64_t*>(smem + kOffFinal), v);
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const uint32_t i = static_cast<uint32_t>(tid * 8 + r);
    const bool live = i < nsel;
    const uint32_t pos = key_pos(v[r]);
    const int64_t o = static_cast<int64_t>(b) * kTopK + i;
    if (kMode == kModeTopK) {
      p.out[o] = live ? bt_row[pos >> 6] * kPage + static_cast<int32_t>(pos & 63u) : -1;
    } else {
      p.cand_scores[o] = live ? ordered_to_float(static_cast<uint32_t>(v[r] >> 32)) : -__int_as_float(0x7f800000);
      p.cand_pos[o] = live ? static_cast<int32_t>(pos) : -1;
    }
  }
}

}  // namespace dsa
