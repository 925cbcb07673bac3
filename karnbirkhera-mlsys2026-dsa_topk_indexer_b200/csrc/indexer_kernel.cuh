// Fused paged-gather + tcgen05 scoring + cluster top-K kernel.
//
// One thread-block cluster of G CTAs serves one request (one query row).
// The request's pages are cut into tiles of two pages (128 keys, the MMA M
// dimension) and the tiles are split evenly over the G CTAs. Each CTA is
// warp-specialised (10 warps):
//   warp 0      TMA producer: per tile, two 8 KB page-data boxes (128-byte
//               swizzle) into a 4-stage ring, a stage freed by the MMA commit;
//   warp 1      TMEM owner and MMA issuer: D[128 keys x 64 heads] (fp32 in
//               TMEM, 4 buffers) = K_tile[128 x 128 e4m3] . Q[64 x 128 e4m3]^T
//               as four tcgen05.mma kind::f8f6f4 (K = 32 each);
//   warps 2..9  two epilogue groups of four warps (even / odd tiles): thread =
//               TMEM lane = key; tcgen05.ld of its 64 head columns, relu /
//               head-weight / scale reduction in registers (packed fp32x2
//               FMA; the key's scale from its own global load, issued two
//               tiles ahead), then a threshold filter into a shared-memory
//               candidate buffer that is cut back to the best 2048 when it
//               fills;
//   all warps   after the stream: cluster-wide exact radix select of the best
//               2048 over every CTA's candidates (histograms summed through
//               distributed shared memory), survivors written into CTA 0's
//               shared memory, ordered there and translated to physical slots.
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
constexpr int kThreads = 320;     // 10 warps
constexpr int kEpiThreads = 256;  // warps 2..9
constexpr int kCap = 4608;        // candidate keys per CTA (the rest of half an SM)
constexpr int kSoloCap = 3072;    // candidates a one-CTA row ranks at once (12 per thread)
constexpr int kTmemBufs = 4;
constexpr int kTmemCols = kTmemBufs * kHeads;

enum Mode : int { kModeTopK = 0, kModeScores = 1, kModePartial = 2 };

// Named barriers (0 is __syncthreads).
constexpr int kBarEpi = 1;   // the 256 epilogue threads
constexpr int kBarLow = 2;   // threads 0..255 (final ordering in CTA 0)

// Shared memory map (byte offsets from a 1024-aligned base).
constexpr int kOffK = 0;                                  // kStages x 16384, swizzled K tiles
constexpr int kOffQ = kOffK + kStages * 16384;            // 8192, swizzled Q
constexpr int kOffCand = kOffQ + 8192;                    // kCap x 8
constexpr int kOffHist = kOffCand + kCap * 8;             // 2 x 256 x 4
constexpr int kOffTot = kOffHist + 2 * 256 * 4;           // 256 x 4
constexpr int kOffW = kOffTot + 256 * 4;                  // 64 x 4
constexpr int kOffBar = kOffW + 256;                      // (2*kStages + 2*kTmemBufs + 1) x 8
constexpr int kOffMisc = kOffBar + 256;                   // small words
constexpr int kSmemUsed = kOffMisc + 128;
constexpr int kSmemBytes = kSmemUsed + 1024;              // alignment slack
// After the stream the K ring is free: CTA 0 orders the survivors there.
constexpr int kOffFinal = kOffK;                          // 2048 x 8
constexpr int kOffRankTmp = kOffFinal + kTopK * 8;        // 2048 x 8
constexpr int kOffRankCnt = kOffRankTmp + kTopK * 8;      // 3 x 2048 x 4 (cnt, start, fill)
constexpr int kOffRankD = kOffRankCnt + 3 * 2048 * 4;     // 2048 x 2 (bucket of each tmp slot)
static_assert(kOffRankD + kTopK * 2 <= kOffQ, "ordering scratch must fit in the K ring");
// One-CTA rows with up to kSoloCap candidates rank them all in place of the
// cluster select; the K ring then holds that ordering's scratch instead.
constexpr int kOffSoloTmp = kOffK;                        // kSoloCap x 8
constexpr int kOffSoloD = kOffSoloTmp + kSoloCap * 8;     // kSoloCap x 2
constexpr int kOffSoloCnt = kOffSoloD + kSoloCap * 2;     // 3 x 2048 x 4
static_assert(kOffSoloCnt % 16 == 0 && kOffSoloCnt + 3 * 2048 * 4 <= kOffQ, "solo ordering scratch");
static_assert(2 * (kSmemBytes + 1024) <= 233472, "two CTAs per SM");
static_assert(kStages * 16384 % 1024 == 0, "K tiles must stay 1024-aligned");
static_assert((2 * kStages + 2 * kTmemBufs + 1) * 8 <= 256, "barrier area");

// Misc word indices (uint32 at kOffMisc).
enum MiscWord : int {
  kMiscTmem = 0,   // TMEM base address
  kMiscCount = 1,  // candidates in the buffer (after a compaction)
  kMiscAbort = 2,  // pipeline abort flag
  kMiscSlot = 3,   // epilogue: append counter in use at the end of the stream
  kMiscSel = 4,    // 3 words: digit scan result
  kMiscPub = 8,    // 2 words read by other CTAs of the cluster
  kMiscTotal = 10,
  kMiscOffset = 11,
  kMiscRot = 12,    // 3 rotating append counters of the epilogue
  kMiscNBase = 15,  // epilogue: candidates below the current append interval
  kMiscMM = 16,     // 2 x u64: min / max of the local candidates
  kMiscPubMM = 20,  // 2 x u64 read by other CTAs of the cluster
  kMiscWsum = 24,   // 8 words: scan scratch of the final ordering
};

struct IndexerParams {
  const uint8_t* kcache;       // page pool (the epilogue reads the key scales from it)
  const int32_t* order;        // [B] request served by cluster c (longest first), or null
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
  // >= 0: no order array; the cluster serves the row whose longest-first
  // rank is order_base + cluster index, computed in the kernel (small
  // batches: saves the plan launch).
  int32_t order_base = -1;
  // Test hook (off: -1): every CTA's producer skips the loads of its local
  // tile `skip_tile`, so the waits for that tile run out after wait_ns and
  // the kernel takes its abort path.
  int32_t skip_tile = -1;
  uint64_t wait_ns = ptx::kWaitTimeoutNs;  // bound of every pipeline wait
  // [B] or null: rows whose entry is nonzero were served by the
  // shared-sequence kernel launched before this one and are skipped.
  const int32_t* handled = nullptr;
  // Two-class launch with in-kernel ranking: role 0 is the launch at
  // cluster size split_ghi over every rank, role 1 the launch at split_glo
  // over ranks >= split_r. From the real lengths the kernel decides whether
  // the split pays (split_beats_waves); if it does, role 0 serves ranks <
  // split_r and role 1 the rest, else role 0 serves every rank (in waves,
  // longest first) and role 1 exits. -1: no two-class launch.
  int32_t split_role = -1;
  int32_t split_r = 0, split_ghi = 0, split_glo = 0, split_slots = 0;
};

constexpr int kInKernelOrderMax = 256;  // rows ranked in-kernel at most
static_assert(kCap * 8 >= kInKernelOrderMax * 12, "in-kernel row ranking scratch (candidate buffer)");

// Longest-first rank -> row, computed by every CTA from the clamped lengths
// (ties: smaller row first, as the plan kernel's counting sort would give
// within a bucket). All kThreads threads; `scratch` holds 3 x
// kInKernelOrderMax words; *total is 64-bit scratch. kTwoClass: it also
// decides the two-class launch (*split = 1 if the split pays,
// split_beats_waves).
__device__ __forceinline__ bool split_beats_waves(const IndexerParams& p, const int32_t* sorted_tiles, int64_t total);

template <bool kTwoClass>
__device__ __forceinline__ int row_of_rank(const IndexerParams& p, int target, int32_t* scratch, uint32_t* result,
                                           uint32_t* split, unsigned long long* total) {
  // Row j's key (tiles << 32 | ~j) is unique and orders the rows longest
  // first, ties by row: the rank of row i is the number of larger keys,
  // counted by thread i over all keys two at a time (broadcast loads).
  const int64_t cap = static_cast<int64_t>(p.max_pages) * kPage;
  const int B = p.batch;
  const int Bp = (B + 1) & ~1;  // padded with key 0, below every row's key
  uint64_t* key = reinterpret_cast<uint64_t*>(scratch);
  int32_t* sorted_tiles = scratch + 2 * kInKernelOrderMax;
  for (int j = threadIdx.x; j < Bp; j += kThreads) {
    uint64_t k = 0ull;
    if (j < B) {
      int64_t l = p.seq_lens[j];
      l = l < 0 ? 0 : (l > cap ? cap : l);
      const uint64_t t = static_cast<uint64_t>((l + 2 * kPage - 1) / (2 * kPage));  // tiles
      k = (t << 32) | static_cast<uint64_t>(0xFFFFFFFFu - static_cast<uint32_t>(j));
    }
    key[j] = k;
  }
  if (threadIdx.x == 0) {
    *result = 0u;
    if constexpr (kTwoClass) *total = 0ull;
  }
  __syncthreads();
  const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(key);
  for (int i = threadIdx.x; i < B; i += kThreads) {
    const uint64_t ki = key[i];
    int r = 0;
#pragma unroll 8
    for (int q = 0; q < Bp / 2; ++q) {
      const ulonglong2 v = k2[q];
      r += (v.x > ki ? 1 : 0) + (v.y > ki ? 1 : 0);
    }
    if (r == target) *result = static_cast<uint32_t>(i);
    if constexpr (kTwoClass) sorted_tiles[r] = static_cast<int32_t>(ki >> 32);
  }
  if constexpr (kTwoClass) {  // total tiles: warp sums, one shared atomic per warp
    unsigned long long sum = 0ull;
    for (int j = threadIdx.x; j < B; j += kThreads) sum += key[j] >> 32;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, off);
    if ((threadIdx.x & 31) == 0 && sum) atomicAdd(total, sum);
  }
  __syncthreads();
  if constexpr (kTwoClass) {
    if (threadIdx.x == 0) *split = split_beats_waves(p, sorted_tiles, static_cast<int64_t>(*total)) ? 1u : 0u;
    __syncthreads();
  }
  return static_cast<int>(*result);
}

// Two-class launch or waves? Estimated makespans in tiles per CTA, from the
// tile counts sorted longest first:
//   split: one wave, max(t[0] / ghi, t[r] / glo) (the longest row of each class);
//   waves: every row at ghi, longest first, slots / ghi clusters at a time:
//          max(t[0] / ghi, (t[c-1] + t[c]) / ghi, total / slots) plus one more
//          row tail (select and ordering, about kWaveTailTiles tiles of time).
// Measured on B200: log-uniform 512..32k-key rows (64) run 45 us split vs
// 51 us in waves; uniform 16k..131k-key rows (64) 0.20 ms split vs 0.16 ms
// in waves.
constexpr int64_t kWaveTailTiles = 25;

__device__ __forceinline__ bool split_beats_waves(const IndexerParams& p, const int32_t* t, int64_t total) {
  const int64_t ghi = p.split_ghi, glo = p.split_glo, slots = p.split_slots, B = p.batch, r = p.split_r;
  auto ceil_div = [](int64_t a, int64_t b) { return (a + b - 1) / b; };
  const int64_t split = ceil_div(t[0], ghi) > ceil_div(t[r], glo) ? ceil_div(t[0], ghi) : ceil_div(t[r], glo);
  const int64_t c = slots / ghi;
  int64_t waves = ceil_div(t[0], ghi);
  if (c >= 1 && c < B) {
    const int64_t two = ceil_div(static_cast<int64_t>(t[c - 1]) + t[c], ghi);
    waves = two > waves ? two : waves;
  }
  const int64_t fill = ceil_div(total, slots);
  waves = (fill > waves ? fill : waves) + kWaveTailTiles;
  return split < waves;
}

__device__ unsigned int g_dsa_status;

// acc[h] for 32 heads [h0, h0+32): s[] += w_h * relu(sgn * acc_h) with
// packed fp32x2 FMAs into four independent accumulator pairs. The per-key
// scale is applied by the caller once to the sum: relu(scale * x) =
// |scale| * relu(sign(scale) * x). relu is fmaxf(x, 0) (NaN -> 0), as in the
// reference epilogue (solution/cuda/kernel.cu:423-430).
//
// kFast: the heads accumulated into s[1] and s[3] take x + |x| = 2 relu(x)
// instead (an add on the FMA pipe rather than a max on the half-rate ALU
// pipe); the caller halves those two accumulators, which gives exactly the
// same value, because scaling by 2 and 1/2 is exact in fp32. Only a NaN
// accumulator (possible only from NaN input bytes) behaves differently: it
// turns the sum into NaN, and the caller then recomputes with kFast = false.
template <bool kNeg, bool kFast>
__device__ __forceinline__ void head_reduce_half(const uint32_t (&acc)[32], const float* s_w, int h0,
                                                 float2 (&s)[4]) {
  const float4* w4 = reinterpret_cast<const float4*>(s_w + h0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 w = w4[j];
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = __uint_as_float(acc[4 * j + e]);
      const float x = kNeg ? -v : v;
      r[e] = (kFast && e >= 2) ? x + fabsf(x) : fmaxf(x, 0.f);
    }
    const int a = (j & 1) * 2;
    s[a] = __ffma2_rn(make_float2(w.x, w.y), make_float2(r[0], r[1]), s[a]);
    s[a + 1] = __ffma2_rn(make_float2(w.z, w.w), make_float2(r[2], r[3]), s[a + 1]);
  }
}

template <bool kFast>
__device__ __forceinline__ float key_score_pass(uint32_t ta, const float* s_w, float scale) {
  uint32_t a[32];
  float2 s[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  ptx::tmem_ld_32x32b_x32_sync(ta, a);
  if (scale >= 0.f)
    head_reduce_half<false, kFast>(a, s_w, 0, s);
  else
    head_reduce_half<true, kFast>(a, s_w, 0, s);
  ptx::tmem_ld_32x32b_x32_sync(ta + 32u, a);
  if (scale >= 0.f)
    head_reduce_half<false, kFast>(a, s_w, 32, s);
  else
    head_reduce_half<true, kFast>(a, s_w, 32, s);
  const float h = kFast ? 0.5f : 1.f;
  return (((s[0].x + s[0].y) + h * (s[1].x + s[1].y)) + ((s[2].x + s[2].y) + h * (s[3].x + s[3].y))) *
         fabsf(scale);
}

// Score of this thread's key from its 64 TMEM accumulator columns at `ta`
// (one query's heads): sum_h w_h * relu(scale * acc_h). The summation order
// is fixed (four packed accumulator pairs, then a pairwise tree), so every
// kernel that calls this produces bit-identical scores. Called by the whole
// warp (tcgen05.ld is warp-collective).
__device__ __forceinline__ float key_score(uint32_t ta, const float* s_w, float scale) {
  const float f = key_score_pass<true>(ta, s_w, scale);
  if (__any_sync(0xFFFFFFFFu, f != f)) return key_score_pass<false>(ta, s_w, scale);  // NaN inputs: exact relu
  return f;
}

// Cluster-wide exact selection of the best 2048 of all candidates held by the
// G CTAs of this cluster (n in this CTA's cand buffer), survivors gathered in
// CTA 0's shared memory, ordered and emitted for row b. Called by all
// kThreads threads of every CTA of the cluster, with the K ring free.
// Shared-memory offsets cluster_select_emit works with. `Final` receives the
// survivors of every CTA (written remotely) and must not overlap `Cand`;
// the ordering scratch (`RankTmp`, `RankCnt`) is only touched after the last
// cluster barrier, when `Cand` is dead.
struct StreamSelectLayout {
  static constexpr bool kSolo = true;  // scratch for ranking all candidates of a one-CTA row
  static constexpr int kSoloTmp = kOffSoloTmp, kSoloD = kOffSoloD, kSoloCnt = kOffSoloCnt;
  static constexpr int kCand = kOffCand, kHist = kOffHist, kTot = kOffTot, kMisc = kOffMisc;
  static constexpr int kFinal = kOffFinal, kRankTmp = kOffRankTmp, kRankCnt = kOffRankCnt, kRankD = kOffRankD;
};

template <int kMode, class L>
__device__ __forceinline__ void cluster_select_emit(uint8_t* smem, uint32_t base_addr, uint32_t n, uint32_t G,
                                                    uint32_t rank, int b, const int32_t* bt_row,
                                                    const IndexerParams& p) {
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + L::kCand);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + L::kHist);
  uint32_t* tot = reinterpret_cast<uint32_t*>(smem + L::kTot);
  uint32_t* misc_nv = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  unsigned long long* mm = reinterpret_cast<unsigned long long*>(smem + L::kMisc + 4 * kMiscMM);
  unsigned long long* pub_mm = reinterpret_cast<unsigned long long*>(smem + L::kMisc + 4 * kMiscPubMM);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  if constexpr (L::kSolo) {
    if (G == 1 && n <= static_cast<uint32_t>(kSoloCap)) {
      // One CTA holds every candidate of the row: rank them all and emit the
      // best 2048 (no threshold search, exchange or second pass).
      if (tid == 0) {
        mm[0] = ~0ull;
        mm[1] = 0ull;
      }
      __syncthreads();
      group_minmax<kThreads>(cand, n, mm, tid, 0);
      if (tid >= 256) return;
      RankScratch sc;
      sc.tmp = reinterpret_cast<uint64_t*>(smem + L::kSoloTmp);
      sc.tmpd = reinterpret_cast<uint16_t*>(smem + L::kSoloD);
      sc.cnt = reinterpret_cast<uint32_t*>(smem + L::kSoloCnt);
      sc.start = sc.cnt + 2048;
      sc.fill = sc.start + 2048;
      sc.wsum = misc_nv + kMiscWsum;
      const int64_t o = static_cast<int64_t>(b) * kTopK;
      if (kMode == kModeTopK) {
        EmitSlots e{p.out + o, bt_row};
        block_rank_emit<kSoloCap / 256>(cand, n, mm[0], mm[1], sc, e, tid, kBarLow);
      } else {
        EmitCandidates e{p.cand_scores + o, p.cand_pos + o};
        block_rank_emit<kSoloCap / 256>(cand, n, mm[0], mm[1], sc, e, tid, kBarLow);
      }
      return;
    }
  }
  // ---- cluster-wide exact selection of the best 2048 keys ----
  const uint32_t pub_addr = base_addr + L::kMisc + 4 * kMiscPub;
  const uint32_t pub_mm_addr = base_addr + L::kMisc + 4 * kMiscPubMM;
  if (tid == 0) {
    mm[0] = ~0ull;
    mm[1] = 0ull;
  }
  __syncthreads();
  group_minmax<kThreads>(cand, n, mm, tid, 0);
  if (tid == 0) {
    misc_nv[kMiscPub] = n;
    pub_mm[0] = mm[0];
    pub_mm[1] = mm[1];
  }
  ptx::cluster_sync();
  if (warp == 0) {
    // Cluster totals: candidate count, smallest and largest key.
    uint32_t v = 0;
    unsigned long long lo = ~0ull, hi = 0ull;
    if (static_cast<uint32_t>(lane) < G) {
      v = ptx::ld_dsmem_u32(ptx::mapa(pub_addr, lane));
      const uint32_t a = ptx::mapa(pub_mm_addr, lane);
      lo = (static_cast<unsigned long long>(ptx::ld_dsmem_u32(a + 4)) << 32) | ptx::ld_dsmem_u32(a);
      hi = (static_cast<unsigned long long>(ptx::ld_dsmem_u32(a + 12)) << 32) | ptx::ld_dsmem_u32(a + 8);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
      const unsigned long long x = __shfl_xor_sync(0xFFFFFFFFu, lo, off);
      const unsigned long long y = __shfl_xor_sync(0xFFFFFFFFu, hi, off);
      lo = x < lo ? x : lo;
      hi = y > hi ? y : hi;
    }
    if (lane == 0) {
      misc_nv[kMiscTotal] = v;
      mm[0] = lo;
      mm[1] = hi;
    }
  }
  __syncthreads();
  const uint32_t total = misc_nv[kMiscTotal];
  uint64_t T = 0;
  if (total > static_cast<uint32_t>(kTopK)) {
    RadixState st = radix_start(mm[0], mm[1], kTopK);
    int pass = 0;
#pragma unroll 1
    while (true) {
      uint32_t* hb = hist + (pass & 1) * 256;
      if (tid < 256) hb[tid] = 0u;
      __syncthreads();
      radix_hist<kThreads>(cand, n, st, hb, tid);
      ptx::cluster_sync();  // every CTA's histogram of this pass is complete
      if (tid < 256) {
        const uint32_t hb_addr = ptx::smem_addr(hb + tid);
        uint32_t sum = 0;
        for (uint32_t r = 0; r < G; ++r) sum += ptx::ld_dsmem_u32(ptx::mapa(hb_addr, r));
        tot[tid] = sum;
      }
      __syncthreads();
      if (warp == 0) find_digit_warp(tot, st.krem, misc_nv + kMiscSel);
      __syncthreads();
      if (radix_advance(st, misc_nv + kMiscSel)) break;
      ++pass;
    }
    T = st.prefix;
  }
  // Count this CTA's survivors per warp (each warp owns a contiguous range of
  // the buffer), publish the CTA total, and get this CTA's output offset.
  const uint32_t nsel = total < static_cast<uint32_t>(kTopK) ? total : static_cast<uint32_t>(kTopK);
  uint32_t wlo, whi;
  warp_range(n, warp, kThreads / 32, &wlo, &whi);
  const uint32_t wc = warp_count_ge(cand, wlo, whi, T);
  if (lane == 0) tot[warp] = wc;  // the digit totals are no longer needed
  __syncthreads();
  if (tid == 0) {
    uint32_t c = 0;
    for (int k = 0; k < kThreads / 32; ++k) c += tot[k];
    misc_nv[kMiscPub + 1] = c;
  }
  ptx::cluster_sync();
  if (warp == 0) {
    uint32_t v = (static_cast<uint32_t>(lane) < rank) ? ptx::ld_dsmem_u32(ptx::mapa(pub_addr + 4, lane)) : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (lane == 0) misc_nv[kMiscOffset] = v;
  }
  __syncthreads();
  {
    uint32_t off = misc_nv[kMiscOffset];
    for (int k = 0; k < warp; ++k) off += tot[k];
    warp_write_ge(cand, wlo, whi, T, ptx::mapa(base_addr + L::kFinal, 0) + 8u * off);
  }
  ptx::cluster_sync();
  if (rank != 0 || tid >= 256) return;

  // ---- CTA 0, threads 0..255: order the survivors and emit ----
  // Every survivor lies in [T, cluster max] (T = 0 when all were taken).
  const uint64_t kmin = T > mm[0] ? T : static_cast<uint64_t>(mm[0]);
  const uint64_t kmax = mm[1];
  RankScratch sc;
  sc.tmp = reinterpret_cast<uint64_t*>(smem + L::kRankTmp);
  sc.tmpd = reinterpret_cast<uint16_t*>(smem + L::kRankD);
  sc.cnt = reinterpret_cast<uint32_t*>(smem + L::kRankCnt);
  sc.start = sc.cnt + 2048;
  sc.fill = sc.start + 2048;
  sc.wsum = misc_nv + kMiscWsum;
  const uint64_t* fin = reinterpret_cast<const uint64_t*>(smem + L::kFinal);
  const int64_t o = static_cast<int64_t>(b) * kTopK;
  if (kMode == kModeTopK) {
    EmitSlots e{p.out + o, bt_row};
    block_rank_emit<8>(fin, nsel, kmin, kmax, sc, e, tid, kBarLow);
  } else {
    EmitCandidates e{p.cand_scores + o, p.cand_pos + o};
    block_rank_emit<8>(fin, nsel, kmin, kmax, sc, e, tid, kBarLow);
  }
}

// kTwoClass: one of the two launches of the two-class schedule with
// in-kernel ranking (IndexerParams::split_role); a separate instantiation
// so that the single-launch kernel carries none of it.
template <int kMode, bool kTwoClass = false>
__global__ void __launch_bounds__(kThreads, 2)
    indexer_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                   const IndexerParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_addr(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_addr - raw_addr);

  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kOffCand);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + kOffHist);
  float* s_w = reinterpret_cast<float*>(smem + kOffW);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc);
  uint32_t* misc_nv = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile uint32_t* abort_flag = misc + kMiscAbort;
  unsigned long long* mm = reinterpret_cast<unsigned long long*>(smem + kOffMisc + 4 * kMiscMM);

  const uint32_t bar_full = base_addr + kOffBar;                // [kStages]
  const uint32_t bar_empty = bar_full + 8 * kStages;            // [kStages]
  const uint32_t bar_tfull = bar_empty + 8 * kStages;           // [kTmemBufs]
  const uint32_t bar_tempty = bar_tfull + 8 * kTmemBufs;        // [kTmemBufs]
  const uint32_t bar_q = bar_tempty + 8 * kTmemBufs;            // [1]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t G = ptx::cluster_nctarank();
  const uint32_t rank = ptx::cluster_ctarank();
  const int b = p.order_base >= 0
                    ? row_of_rank<kTwoClass>(p, p.order_base + static_cast<int>(blockIdx.x / G),
                                             reinterpret_cast<int32_t*>(smem + kOffCand), misc_nv + kMiscSel,
                                             misc_nv + kMiscSel + 1, mm)
                    : (p.order ? p.order[blockIdx.x / G] : static_cast<int>(blockIdx.x / G));
  if (p.handled && p.handled[b]) return;  // uniform over the cluster, before any barrier or TMEM use
  if constexpr (kTwoClass) {  // does this launch serve this rank? (uniform over the cluster)
    const bool split = misc_nv[kMiscSel + 1] != 0u;
    const int k = p.order_base + static_cast<int>(blockIdx.x / G);
    if (p.split_role == 0 ? (split && k >= p.split_r) : !split) return;
  }

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

  // ---- key scales (epilogue) ----
  // Key scales come straight from the page pool with global loads issued
  // two tiles of the epilogue group ahead (their page ids one tile ahead of
  // that), so the epilogue never waits for or releases a K ring stage: the
  // MMA commit alone frees a stage. The first loads are issued before the
  // setup below, which hides their latency. Epilogue warp (group g, lane
  // quarter q) scores key row 32q + lane of the group's tiles; its 32 keys
  // lie in one page of the tile (quarters 0-1: the first page, 2-3: the
  // second).
  const int epi_q4 = warp & 3;
  const int epi_row = epi_q4 * 32 + lane;
  const int epi_grp = (warp - 2) >> 2;
  const uint8_t* scale_base = p.kcache + kPageData + 4 * (epi_row & (kPage - 1));
  auto page_of = [&](int t) -> int32_t {  // warp-uniform; -1: no page
    const int pi = pg_first + 2 * t + (epi_q4 >> 1);
    return (t < my_tiles && pi < pg_end) ? __ldg(bt_row + pi) : -1;
  };
  auto scale_of = [&](int32_t pid) -> float {  // out-of-range ids read nothing (TMA zero-fills their keys)
    return static_cast<uint64_t>(static_cast<uint32_t>(pid)) < static_cast<uint64_t>(p.num_pages)
               ? __ldg(reinterpret_cast<const float*>(scale_base + static_cast<int64_t>(pid) * kPageBytes))
               : 0.f;
  };
  float sc_next = 0.f, sc_after = 0.f;  // scales of the group's tiles i and i + 2
  int32_t pid_ahead = -1;               // page id for tile i + 4
  if (warp >= 2) {
    sc_next = scale_of(page_of(epi_grp));
    sc_after = scale_of(page_of(epi_grp + 2));
    pid_ahead = page_of(epi_grp + 4);
  }

  // ---- setup ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar_full + 8 * s, 1);
      ptx::mbar_init(bar_empty + 8 * s, 1);  // the MMA commit: the epilogue never reads the K ring
    }
    for (int i = 0; i < kTmemBufs; ++i) {
      ptx::mbar_init(bar_tfull + 8 * i, 1);
      ptx::mbar_init(bar_tempty + 8 * i, 4);
    }
    ptx::mbar_init(bar_q, 1);
    ptx::fence_mbar_init();
    misc_nv[kMiscCount] = 0u;
    misc_nv[kMiscAbort] = 0u;
    misc_nv[kMiscRot] = misc_nv[kMiscRot + 1] = misc_nv[kMiscRot + 2] = 0u;
    misc_nv[kMiscNBase] = misc_nv[kMiscSlot] = 0u;
    ptx::prefetch_tmap(&tm_k);
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

  int issued = 0;      // producer: tiles whose loads were issued
  int skipped = -1;    // producer: the tile the test hook left unloaded
  int mma_issued = 0;  // MMA warp: tiles whose MMAs were issued
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
        const uint32_t kdst = base_addr + kOffK + s * 16384;
        ptx::mbar_arrive_expect_tx(fb, bytes);
        ptx::tma_load_3d(kdst, &tm_k, fb, 0, 0, pa, pol_stream);
        if (has_b) ptx::tma_load_3d(kdst + kPageData, &tm_k, fb, 0, 0, pb, pol_stream);
      }
      __syncwarp();
      issued = i + 1;
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    constexpr uint32_t idesc = ptx::idesc_e4m3_f32(kTileKeys, kHeads);
    bool ok = true;
    if (my_tiles > 0) ok = ptx::mbar_wait(bar_q, 0u, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
    const uint64_t qdesc = ptx::sw128_kmajor_desc(base_addr + kOffQ);
#pragma unroll 1
    for (int i = 0; i < my_tiles && !aborted; ++i) {
      const int s = i % kStages;
      const uint32_t ph = static_cast<uint32_t>(i / kStages) & 1u;
      const int buf = i % kTmemBufs;
      const uint32_t bph = static_cast<uint32_t>(i / kTmemBufs) & 1u;
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
  } else {
    // ===================== epilogue: two groups of four warps =====================
    // Group 0 (warps 2-5) takes the even tiles, group 1 (warps 6-9) the odd
    // ones, so two tiles are reduced at once. Within a group, warp w reads
    // TMEM lane quarter w % 4, i.e. thread = key row of the tile.
    const int grp = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int et = threadIdx.x - 64;  // 0..255 over both groups
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    const int n_pairs_full = my_tiles >> 1;
    uint64_t thr = 0;  // keys below thr can no longer reach the top 2048
    int since = 0;
    int check_every = kCap / (2 * kTileKeys);
    // Candidates [0, n_base) were counted at the last check; the keys of the
    // current interval take slots n_base + (rotating counter `slot`). Each
    // warp stores a tile's keys one tile late, once its slot atomic has
    // returned (pm/pkeep/pkey/pbase/pleader: the pending append).
    uint32_t n_base = 0, slot = 0, pm = 0, pbase = 0;
    int pleader = 0;
    bool pkeep = false;
    uint64_t pkey = 0;
    auto flush = [&]() {
      if (pm) {
        const uint32_t pb = __shfl_sync(0xFFFFFFFFu, pbase, pleader);
        if (pkeep) cand[n_base + pb + __popc(pm & lanemask_lt())] = pkey;
      }
      pm = 0u;
    };
    // A warp whose wait gave up (`aborted`, warp-uniform) stops touching the
    // pipeline but keeps walking the same tile schedule with no keys, so it
    // still meets the other group at every check barrier below: leaving the
    // loop early would strand the other group at a named barrier.
#pragma unroll 1
    for (int i = grp; i < my_tiles; i += 2) {
      float score = 0.f;
      const float scale = sc_next;
      sc_next = sc_after;
      sc_after = scale_of(pid_ahead);  // tile i + 4
      pid_ahead = page_of(i + 6);
      const int buf = i % kTmemBufs;
      if (!aborted) {
        const uint32_t bph = static_cast<uint32_t>(i / kTmemBufs) & 1u;
        const bool ok = ptx::mbar_wait(bar_tfull + 8 * buf, bph, abort_flag, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT,
                                       p.wait_ns);
        if (__any_sync(0xFFFFFFFFu, !ok)) aborted = true;
        if (!aborted) {
          __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
          ptx::tc_fence_after();
          score = key_score(tmem + t_lane + static_cast<uint32_t>(buf * kHeads), s_w, scale);
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_tempty + 8 * buf);
        }
      }
      const int64_t pos = static_cast<int64_t>(pg_first + 2 * i) * kPage + row;
      const bool valid = !aborted && pos >= key_lo && pos < key_hi;
      if (kMode == kModeScores) {
        if (valid) p.scores[static_cast<int64_t>(b) * p.score_stride + pos] = score;
      } else {
        const uint64_t key = pack_key(score, static_cast<uint32_t>(pos));
        const bool keep = valid && key >= thr;
        flush();  // the previous tile's keys (their slot atomic has returned)
        const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
        pm = m;
        pkeep = keep;
        pkey = key;
        if (m) {
          pleader = __ffs(m) - 1;
          pbase = 0u;
          if (lane == pleader) pbase = atomicAdd(misc_nv + kMiscRot + slot, static_cast<uint32_t>(__popc(m)));
        }
        // After every check_every tile pairs the buffer may be nearly full:
        // both groups meet (one barrier), read the interval's count and move
        // to the next counter; the one used two intervals ago, read by every
        // warp before this barrier, is cleared for reuse. The schedule
        // depends only on tile counts, so all eight warps take the same
        // barriers.
        if (++since == check_every) {
          since = 0;
          if ((i >> 1) < n_pairs_full) {
            flush();
            ptx::named_bar(kBarEpi, kEpiThreads);
            const uint32_t n = n_base + misc[kMiscRot + slot];
            if (et == 0) misc_nv[kMiscRot + (slot + 2u) % 3u] = 0u;
            n_base = n;
            slot = (slot + 1u) % 3u;
            // Cut only when fewer than two tile pairs of room are left, and
            // then exactly to the best 2048: between checks the threshold
            // rejects most keys, so cuts (and the checks, scheduled by the
            // free room) stay rare.
            if (n > static_cast<uint32_t>(kCap - 4 * kTileKeys)) {
              if (et == 0) {
                mm[0] = ~0ull;
                mm[1] = 0ull;
              }
              ptx::named_bar(kBarEpi, kEpiThreads);
              group_minmax<kEpiThreads>(cand, n, mm, et, kBarEpi);
              const uint64_t T = group_select<kEpiThreads>(cand, n, kTopK, mm, hist, misc_nv + kMiscSel, et, kBarEpi);
              group_compact<kEpiThreads, kCap / kEpiThreads>(cand, n, T, misc_nv + kMiscCount, misc_nv + kMiscWsum,
                                                            et, kBarEpi);
              thr = T;
              n_base = misc[kMiscCount];
            }
            check_every = static_cast<int>((kCap - n_base) / (2 * kTileKeys));
          }
        }
      }
    }
    if (kMode != kModeScores) {
      flush();
      if (et == 0) {  // uniform over the epilogue; read after the barrier below
        misc_nv[kMiscNBase] = n_base;
        misc_nv[kMiscSlot] = slot;
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
        if (i != skipped)
          ptx::mbar_wait(bar_full + 8 * (i % kStages), static_cast<uint32_t>(i / kStages) & 1u, &no_abort,
                         &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    }
    if (warp == 1 && lane == 0 && mma_issued > 0) {
      const int last = mma_issued - 1;
      ptx::mbar_wait(bar_tfull + 8 * (last % kTmemBufs), static_cast<uint32_t>(last / kTmemBufs) & 1u,
                     &no_abort, &g_dsa_status, DSA_STATUS_WAIT_TIMEOUT, p.wait_ns);
    }
    __syncthreads();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
  if (kMode == kModeScores) return;

  // Every epilogue warp stored its last keys before the barrier above.
  const uint32_t n_final = misc_nv[kMiscNBase] + misc_nv[kMiscRot + misc_nv[kMiscSlot]];
  cluster_select_emit<kMode, StreamSelectLayout>(smem, base_addr, n_final, G, rank, b, bt_row, p);
}

// Longest-first request order for the indexer's clusters (one CTA of 1024
// threads): counting sort of the rows' tile counts, descending. Rows whose
// counts fall in the same bucket keep no particular order. With group_order
// non-null it also orders the groups of kGroupRows consecutive rows (the
// shared-sequence kernel's work items) by their longest row, the same way.
constexpr int kPlanThreads = 1024;
constexpr int kPlanBuckets = 4096;
constexpr int kGroupRows = 4;

// Descending counting sort of n items by tile count tiles(i) in [0, max_tiles]
// into out[0..n). All kPlanThreads threads; cnt/start hold kPlanBuckets words.
template <class Tiles>
__device__ void plan_sort_desc(int n, int max_tiles, Tiles tiles, int32_t* __restrict__ out, uint32_t* cnt,
                               uint32_t* start, uint32_t* wsum) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int shift = 0;
  while ((max_tiles >> shift) >= kPlanBuckets) ++shift;
  for (int i = t; i < kPlanBuckets; i += kPlanThreads) cnt[i] = 0u;
  __syncthreads();
  auto bucket = [&](int i) { return (kPlanBuckets - 1) - (tiles(i) >> shift); };  // longest in bucket 0
  for (int i = t; i < n; i += kPlanThreads) atomicAdd(&cnt[bucket(i)], 1u);
  __syncthreads();
  // exclusive scan over the 4096 buckets: thread t owns buckets 4t..4t+3
  uint32_t c[4], tot = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    c[j] = cnt[4 * t + j];
    tot += c[j];
  }
  uint32_t incl = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  uint32_t base = incl - tot;
  for (int k = 0; k < w; ++k) base += wsum[k];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    start[4 * t + j] = base;
    base += c[j];
  }
  __syncthreads();
  for (int i = t; i < n; i += kPlanThreads) out[atomicAdd(&start[bucket(i)], 1u)] = i;
  __syncthreads();
}

__global__ void __launch_bounds__(kPlanThreads, 1)
    lpt_order_kernel(const int32_t* __restrict__ seq_lens, int batch, int max_pages, int32_t* __restrict__ order,
                     int32_t* __restrict__ group_order) {
  __shared__ uint32_t cnt[kPlanBuckets];
  __shared__ uint32_t start[kPlanBuckets];
  __shared__ uint32_t wsum[kPlanThreads / 32];
  const int max_tiles = (max_pages + 1) / 2;
  auto row_tiles = [&](int b) {
    int64_t len = seq_lens[b];
    len = len < 0 ? 0 : (len > static_cast<int64_t>(max_pages) * kPage ? static_cast<int64_t>(max_pages) * kPage : len);
    return static_cast<int>((len + 2 * kPage - 1) / (2 * kPage));
  };
  plan_sort_desc(batch, max_tiles, row_tiles, order, cnt, start, wsum);
  if (group_order) {
    auto group_tiles = [&](int g) {
      int m = 0;
      for (int r = g * kGroupRows; r < (g + 1) * kGroupRows && r < batch; ++r) {
        const int x = row_tiles(r);
        m = x > m ? x : m;
      }
      return m;
    };
    plan_sort_desc((batch + kGroupRows - 1) / kGroupRows, max_tiles, group_tiles, group_order, cnt, start, wsum);
  }
}

}  // namespace dsa
