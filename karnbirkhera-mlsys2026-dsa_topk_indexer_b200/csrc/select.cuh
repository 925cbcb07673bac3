// Exact top-K selection primitives shared by the indexer kernels.
//
// A candidate is one 64-bit key: the high word is the score mapped to an
// order-preserving uint32, the low word is (0xFFFFFFFF - logical position).
// Larger key = better candidate; equal scores rank the smaller position
// first, which is the order a stable descending radix sort of (score,
// position) gives (the reference's cub::BlockRadixSort::SortDescending,
// solution/cuda/kernel.cu:511). Keys are unique, so "the K largest keys" is
// a well-defined set and no tie handling is left to do.
#pragma once
#include <cstdint>
#include "ptx.cuh"

namespace dsa {

constexpr int kTopK = 2048;

__device__ __forceinline__ uint32_t ordered_u32(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
__device__ __forceinline__ uint64_t pack_key(float score, uint32_t pos) {
  return (static_cast<uint64_t>(ordered_u32(score)) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - pos);
}
__device__ __forceinline__ uint32_t key_pos(uint64_t k) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(k);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Group barrier: bar == 0 is __syncthreads(), otherwise named barrier `bar`
// over the NT threads of the group (a warp-aligned set of warps).
template <int NT>
__device__ __forceinline__ void group_sync(uint32_t bar) {
  if (bar == 0)
    __syncthreads();
  else
    ptx::named_bar(bar, NT);
}

// Radix-select state: the top `top` bits of the sought key are known and
// equal `prefix` (lower bits zero); krem keys are still to be taken from the
// keys that share that prefix.
struct RadixState {
  uint64_t prefix;
  int top;
  uint32_t krem;
};

__device__ __forceinline__ uint64_t high_mask(int top) { return top <= 0 ? 0ull : (~0ull << (64 - top)); }

// Next digit window below the known prefix: [shift, shift + width).
__device__ __forceinline__ int window_width(int top) { return (64 - top) < 8 ? (64 - top) : 8; }

// Start state for selecting among keys in [lo, hi]: their common leading bits
// are already known, so the first pass looks at the first bits that differ.
__device__ __forceinline__ RadixState radix_start(uint64_t lo, uint64_t hi, uint32_t k) {
  RadixState st;
  const uint64_t x = lo ^ hi;
  st.top = x ? __clzll(static_cast<long long>(x)) : 64;
  st.prefix = lo & high_mask(st.top);
  st.krem = k;
  return st;
}

// One warp scans a 256-bin histogram from the top digit down and finds the
// digit d with count(digits > d) < krem <= count(digits >= d).
// Writes sel = {d, count(digits > d), count(d)}.
__device__ __forceinline__ void find_digit_warp(const uint32_t* hist, uint32_t krem, uint32_t* sel) {
  const int lane = threadIdx.x & 31;
  uint32_t h[8];
  uint32_t sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    h[j] = hist[lane * 8 + j];
    sum += h[j];
  }
  uint32_t incl = sum;  // inclusive suffix sum over lanes (higher lanes = larger digits)
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_down_sync(0xFFFFFFFFu, incl, off);
    if (lane + off < 32) incl += t;
  }
  const uint32_t above = incl - sum;
  if (above < krem && krem <= incl) {
    uint32_t c = above;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (c + h[j] >= krem) {
        sel[0] = static_cast<uint32_t>(lane * 8 + j);
        sel[1] = c;
        sel[2] = h[j];
        break;
      }
      c += h[j];
    }
  }
}

// Min and max of cand[0..n) over a group (results in mm[0], mm[1]; mm must be
// preset to {~0, 0} before the group barrier that precedes the call).
template <int NT>
__device__ void group_minmax(const uint64_t* cand, uint32_t n, unsigned long long* mm, int gt, uint32_t bar) {
  unsigned long long lo = ~0ull, hi = 0ull;
  for (uint32_t i = gt; i < n; i += NT) {
    const unsigned long long k = cand[i];
    lo = k < lo ? k : lo;
    hi = k > hi ? k : hi;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long a = __shfl_xor_sync(0xFFFFFFFFu, lo, off);
    const unsigned long long b = __shfl_xor_sync(0xFFFFFFFFu, hi, off);
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&mm[0], lo);
    atomicMax(&mm[1], hi);
  }
  group_sync<NT>(bar);
}

// One histogram pass of the radix select over cand[0..n) (plain per-lane
// atomics: below the common prefix the digits are spread out).
template <int NT>
__device__ __forceinline__ void radix_hist(const uint64_t* cand, uint32_t n, const RadixState& st, uint32_t* hist,
                                           int gt) {
  const int width = window_width(st.top);
  const int shift = 64 - st.top - width;
  const uint64_t hm = high_mask(st.top);
  const uint32_t dmask = (1u << width) - 1u;
  uint32_t i = gt;
  // Four keys per step, loaded before any of their (non-returning) atomics.
  for (; i + 3 * NT < n; i += 4 * NT) {
    uint64_t k[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) k[u] = cand[i + u * NT];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if ((k[u] & hm) == st.prefix) atomicAdd(&hist[static_cast<uint32_t>(k[u] >> shift) & dmask], 1u);
  }
  for (; i < n; i += NT) {
    const uint64_t key = cand[i];
    if ((key & hm) == st.prefix) atomicAdd(&hist[static_cast<uint32_t>(key >> shift) & dmask], 1u);
  }
}

// Applies the digit scan result of one pass. Returns true when done.
__device__ __forceinline__ bool radix_advance(RadixState& st, const uint32_t* sel) {
  const int width = window_width(st.top);
  const int shift = 64 - st.top - width;
  st.prefix |= static_cast<uint64_t>(sel[0]) << shift;
  st.top += width;
  st.krem -= sel[1];
  return sel[2] == st.krem || st.top >= 64;
}

// Exact radix select over keys cand[0..n) held in shared memory by a group of
// NT threads (gt = thread index in the group; warp 0 of the group scans).
// Precondition: n > k, group synchronised, mm = {min, max} of the keys.
// Returns T such that exactly k keys are >= T.
template <int NT>
__device__ uint64_t group_select(const uint64_t* cand, uint32_t n, uint32_t k, const unsigned long long* mm,
                                 uint32_t* hist, uint32_t* sel, int gt, uint32_t bar) {
  RadixState st = radix_start(mm[0], mm[1], k);
#pragma unroll 1
  while (true) {
    for (int i = gt; i < 256; i += NT) hist[i] = 0u;
    group_sync<NT>(bar);
    radix_hist<NT>(cand, n, st, hist, gt);
    group_sync<NT>(bar);
    if (gt < 32) find_digit_warp(hist, st.krem, sel);
    group_sync<NT>(bar);
    if (radix_advance(st, sel)) break;
  }
  return st.prefix;
}

// Exclusive offset of this warp's count among the NT/32 warps of a group,
// and the group total. wsum: NT/32 words; one group barrier inside, and the
// caller must pass another barrier before wsum is written again.
template <int NT>
__device__ __forceinline__ uint32_t group_warp_offset(uint32_t wcount, uint32_t* wsum, uint32_t* total, int gt,
                                                      uint32_t bar) {
  const int gw = gt >> 5;
  if ((gt & 31) == 0) wsum[gw] = wcount;
  group_sync<NT>(bar);
  uint32_t base = 0, tot = 0;
#pragma unroll
  for (int k = 0; k < NT / 32; ++k) {
    const uint32_t x = wsum[k];
    base += (k < gw) ? x : 0u;
    tot += x;
  }
  *total = tot;
  return base;
}

// Keeps the keys >= T of cand[0..n) and packs them to the front; `counter`
// ends holding the number kept. MAXPER >= ceil(n / NT). The keys are held in
// registers, so the packing is in place; output slots come from per-warp
// ballot counts and one offset scan (no returning atomics in the loop).
template <int NT, int MAXPER>
__device__ void group_compact(uint64_t* cand, uint32_t n, uint64_t T, uint32_t* counter, uint32_t* wsum, int gt,
                              uint32_t bar) {
  const int lane = threadIdx.x & 31;
  uint64_t v[MAXPER];
  uint32_t m[MAXPER];
  uint32_t cnt = 0;
#pragma unroll
  for (int j = 0; j < MAXPER; ++j) {
    const uint32_t i = gt + j * NT;
    v[j] = (i < n) ? cand[i] : 0ull;
  }
#pragma unroll
  for (int j = 0; j < MAXPER; ++j) {
    const uint32_t i = gt + j * NT;
    m[j] = __ballot_sync(0xFFFFFFFFu, (i < n) && (v[j] >= T));
    cnt += static_cast<uint32_t>(__popc(m[j]));
  }
  uint32_t total = 0;
  uint32_t base = group_warp_offset<NT>(cnt, wsum, &total, gt, bar);  // every load is done past this barrier
#pragma unroll
  for (int j = 0; j < MAXPER; ++j) {
    if ((m[j] >> lane) & 1u) cand[base + __popc(m[j] & lanemask_lt())] = v[j];
    base += static_cast<uint32_t>(__popc(m[j]));
  }
  if (gt == 0) *counter = total;
  group_sync<NT>(bar);
}

// The same in chunks of NT * PER keys, for buffers longer than the registers
// can hold at once: a key only moves to a lower index, and a chunk is loaded
// into registers before any of its keys is written, so packing in place
// chunk by chunk is safe.
template <int NT, int PER>
__device__ void group_compact_chunked(uint64_t* cand, uint32_t n, uint64_t T, uint32_t* counter, uint32_t* wsum,
                                      int gt, uint32_t bar) {
  const int lane = threadIdx.x & 31;
  uint32_t base_all = 0;
#pragma unroll 1
  for (uint32_t c0 = 0; c0 < n; c0 += NT * PER) {
    uint64_t v[PER];
    uint32_t m[PER];
    uint32_t cnt = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const uint32_t i = c0 + gt + j * NT;
      v[j] = (i < n) ? cand[i] : 0ull;
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const uint32_t i = c0 + gt + j * NT;
      m[j] = __ballot_sync(0xFFFFFFFFu, (i < n) && (v[j] >= T));
      cnt += static_cast<uint32_t>(__popc(m[j]));
    }
    uint32_t total = 0;
    uint32_t base = base_all + group_warp_offset<NT>(cnt, wsum, &total, gt, bar);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if ((m[j] >> lane) & 1u) cand[base + __popc(m[j] & lanemask_lt())] = v[j];
      base += static_cast<uint32_t>(__popc(m[j]));
    }
    base_all += total;
    group_sync<NT>(bar);  // wsum is rewritten by the next chunk
  }
  if (gt == 0) *counter = base_all;
  group_sync<NT>(bar);
}

// Survivor count (keys >= T) of src[lo, hi), by one warp over consecutive
// 32-key rows (loads are independent, so the loop pipelines).
__device__ __forceinline__ uint32_t warp_count_ge(const uint64_t* src, uint32_t lo, uint32_t hi, uint64_t T) {
  const int lane = threadIdx.x & 31;
  uint32_t c = 0;
#pragma unroll 4
  for (uint32_t i0 = lo; i0 < hi; i0 += 32) {
    const uint32_t i = i0 + lane;
    const uint64_t k = i < hi ? src[i] : 0ull;
    c += static_cast<uint32_t>(__popc(__ballot_sync(0xFFFFFFFFu, i < hi && k >= T)));
  }
  return c;
}

// Writes the keys >= T of src[lo, hi) (same warp and rows as warp_count_ge)
// to consecutive 8-byte slots from shared::cluster address dst (this CTA's
// or another CTA's shared memory).
__device__ __forceinline__ void warp_write_ge(const uint64_t* src, uint32_t lo, uint32_t hi, uint64_t T,
                                              uint32_t dst) {
  const int lane = threadIdx.x & 31;
  for (uint32_t i0 = lo; i0 < hi; i0 += 32) {
    const uint32_t i = i0 + lane;
    const uint64_t k = i < hi ? src[i] : 0ull;
    const bool keep = i < hi && k >= T;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
    if (keep) ptx::st_dsmem_u64(dst + 8u * static_cast<uint32_t>(__popc(m & lanemask_lt())), k);
    dst += 8u * static_cast<uint32_t>(__popc(m));
  }
}

// The warp-contiguous row range of warp gw (of NW) over n keys.
__device__ __forceinline__ void warp_range(uint32_t n, int gw, int NW, uint32_t* lo, uint32_t* hi) {
  const uint32_t chunk = ((n + NW * 32 - 1) / (NW * 32)) * 32;
  const uint32_t a = static_cast<uint32_t>(gw) * chunk;
  *lo = a < n ? a : n;
  *hi = a + chunk < n ? a + chunk : n;
}

// Shared-memory scratch of block_rank_emit: tmp (2048 keys), the bucket of
// each tmp slot (2048 x 16 bits) and three arrays of 4096 16-bit bucket
// fields packed two per word (2048 words each).
struct RankScratch {
  uint64_t* tmp;
  uint16_t* tmpd;
  uint32_t* cnt;
  uint32_t* start;
  uint32_t* fill;
  uint32_t* wsum;  // 8 words
};

constexpr int kRankBuckets = 4096;

__device__ __forceinline__ uint32_t half16(const uint32_t* a, uint32_t d) {
  return (a[d >> 1] >> ((d & 1u) * 16u)) & 0xFFFFu;
}

// Ranks the n <= 256 * KPT unique keys of keys[] in descending order and
// hands each of the best 2048 to the emitter with its rank: emit.load(key)
// fetches what is written for the key (issued for all of a thread's keys
// before any store), emit.store(rank, value) writes it, emit.pad(i) fills
// ranks n..2047 when n < 2048. tmp and tmpd hold 256 * KPT entries.
// 256 threads (t = 0..255, their index in the group; the group is
// warp-aligned) synchronised by barrier `bar`; kmin <= every key <= kmax. Instead of a sorting network (which on 256 threads is bound by
// shared-memory traffic or shuffle latency at tens of thousands of cycles for
// 2048 64-bit keys), keys are counted into 4096 buckets, scattered bucket by
// bucket, and each key's rank is the number of keys in higher buckets plus
// the number of larger keys in its own bucket. Exact for any input as long
// as the bucket of a key is a non-decreasing function of the key. The cost
// is dominated by the in-bucket comparisons, so buckets are many (16-bit
// counters, two per word) and evenly used:
//
// they split the score range [score(kmin), score(kmax)] linearly, so a bucket
// holds a few keys however the range sits relative to powers of two (a window
// of key bits would put the whole set into one or two buckets whenever the
// range crosses one, since the first differing bits are then exponent bits).
// When the score range is empty or not finite the 12 key bits below the
// common prefix of kmin and kmax are used instead (equal scores then spread
// by position).
template <int KPT, class Emit>
__device__ __forceinline__ void block_rank_emit(const uint64_t* keys, uint32_t n, uint64_t kmin, uint64_t kmax,
                                                const RankScratch sc, Emit& emit, int t, uint32_t bar) {
  const int lane = t & 31, w = t >> 5;
  {  // clear cnt and fill (2048 words each) with 16-byte stores
    uint4* c4 = reinterpret_cast<uint4*>(sc.cnt);
    uint4* f4 = reinterpret_cast<uint4*>(sc.fill);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      c4[t + 256 * j] = z;
      f4[t + 256 * j] = z;
    }
  }
  const float smin = ordered_to_float(static_cast<uint32_t>(kmin >> 32));
  const float smax = ordered_to_float(static_cast<uint32_t>(kmax >> 32));
  const float range = smax - smin;
  const float scale = static_cast<float>(kRankBuckets) / range;
  const bool lin = isfinite(smin) && isfinite(smax) && range > 0.f && isfinite(range) && isfinite(scale);
  const uint64_t x = kmin ^ kmax;
  const int top = x ? __clzll(static_cast<long long>(x)) : 64;
  const int shift = (64 - top - 12) > 0 ? (64 - top - 12) : 0;
  auto bucket = [&](uint64_t k) -> uint32_t {
    if (lin) {
      const float f = (ordered_to_float(static_cast<uint32_t>(k >> 32)) - smin) * scale;
      return f >= static_cast<float>(kRankBuckets - 1) ? static_cast<uint32_t>(kRankBuckets - 1)
                                                        : static_cast<uint32_t>(f);
    }
    return static_cast<uint32_t>(k >> shift) & static_cast<uint32_t>(kRankBuckets - 1);
  };
  static_assert(256 * KPT >= kTopK, "at least 2048 keys");
  uint64_t k[KPT];
  uint32_t d[KPT];
#pragma unroll
  for (int j = 0; j < KPT; ++j) {
    const uint32_t i = t + 256 * j;
    k[j] = i < n ? keys[i] : 0ull;
    d[j] = bucket(k[j]);
  }
  group_sync<256>(bar);
#pragma unroll
  for (int j = 0; j < KPT; ++j)
    if (t + 256 * j < n) atomicAdd(&sc.cnt[d[j] >> 1], 1u << ((d[j] & 1u) * 16u));
  group_sync<256>(bar);
  // Exclusive scan in descending bucket order; thread t owns words
  // 2047-8t down to 2040-8t, i.e. buckets 4095-16t down to 4080-16t (in a
  // word the odd bucket, high half, comes first).
  {
    uint32_t c[8], tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = sc.cnt[2047 - 8 * t - j];
      tot += (c[j] >> 16) + (c[j] & 0xFFFFu);
    }
    uint32_t incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) sc.wsum[w] = incl;
    group_sync<256>(bar);
    uint32_t base = incl - tot;
    for (int q = 0; q < w; ++q) base += sc.wsum[q];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t hi = base;
      const uint32_t lo = base + (c[j] >> 16);
      sc.start[2047 - 8 * t - j] = (hi << 16) | lo;
      base = lo + (c[j] & 0xFFFFu);
    }
  }
  group_sync<256>(bar);
  {  // scatter: all slot atomics first, then the stores that need them
    uint32_t slot[KPT];
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
      const uint32_t sh = (d[j] & 1u) * 16u;
      slot[j] = (t + 256 * j < n)
                    ? half16(sc.start, d[j]) + ((atomicAdd(&sc.fill[d[j] >> 1], 1u << sh) >> sh) & 0xFFFFu)
                    : 0u;
    }
#pragma unroll
    for (int j = 0; j < KPT; ++j)
      if (t + 256 * j < n) {
        sc.tmp[slot[j]] = k[j];
        sc.tmpd[slot[j]] = static_cast<uint16_t>(d[j]);
      }
  }
  group_sync<256>(bar);
  // In-bucket ranks. First pass: the first four keys of every bucket, as
  // straight-line code over all of a thread's keys (their load chains
  // overlap); second pass: the rest of the rare buckets holding more.
  constexpr uint32_t kLast = 256u * KPT - 1u;
  uint32_t r[KPT], b0[KPT], c[KPT];
#pragma unroll
  for (int j = 0; j < KPT; ++j) {
    const uint32_t i = t + 256 * j;
    const bool live = i < n;
    const uint32_t ii = live ? i : 0u;
    k[j] = sc.tmp[ii];
    // Slots >= n were never written (all of tmpd when n == 0): dead lanes
    // use bucket 0, and a stored id is masked to the bucket range.
    const uint32_t dd = live ? (static_cast<uint32_t>(sc.tmpd[ii]) & static_cast<uint32_t>(kRankBuckets - 1)) : 0u;
    b0[j] = half16(sc.start, dd);
    c[j] = live ? half16(sc.cnt, dd) : 0u;
    uint32_t rr = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t q = b0[j] + m;
      rr += (static_cast<uint32_t>(m) < c[j] && sc.tmp[q < kLast ? q : kLast] > k[j]) ? 1u : 0u;
    }
    r[j] = b0[j] + rr;
  }
#pragma unroll
  for (int j = 0; j < KPT; ++j)
    for (uint32_t q = b0[j] + 4; q < b0[j] + c[j]; ++q) r[j] += (sc.tmp[q] > k[j]) ? 1u : 0u;
  // Only the best 2048 are written (n may exceed 2048 when KPT > 8).
  typename Emit::Value v[KPT];
#pragma unroll
  for (int j = 0; j < KPT; ++j)
    if (t + 256 * j < n && r[j] < static_cast<uint32_t>(kTopK)) v[j] = emit.load(k[j]);
#pragma unroll
  for (int j = 0; j < KPT; ++j)
    if (t + 256 * j < n && r[j] < static_cast<uint32_t>(kTopK)) emit.store(r[j], v[j]);
  for (uint32_t i = n + t; i < static_cast<uint32_t>(kTopK); i += 256) emit.pad(i);
}

// Emitters: the top-K physical slots of one row, or its (score, logical
// position) candidate list.
struct EmitSlots {
  using Value = int32_t;
  int32_t* out;           // row of 2048
  const int32_t* bt_row;  // block-table row
  __device__ __forceinline__ int32_t load(uint64_t key) const {
    const uint32_t pos = key_pos(key);
    return bt_row[pos >> 6] * 64 + static_cast<int32_t>(pos & 63u);
  }
  __device__ __forceinline__ void store(uint32_t r, int32_t v) const { out[r] = v; }
  __device__ __forceinline__ void pad(uint32_t i) const { out[i] = -1; }
};

struct EmitCandidates {
  using Value = uint64_t;
  float* scores;  // row of 2048
  int32_t* pos;   // row of 2048
  __device__ __forceinline__ uint64_t load(uint64_t key) const { return key; }
  __device__ __forceinline__ void store(uint32_t r, uint64_t key) const {
    scores[r] = ordered_to_float(static_cast<uint32_t>(key >> 32));
    pos[r] = static_cast<int32_t>(key_pos(key));
  }
  __device__ __forceinline__ void pad(uint32_t i) const {
    scores[i] = -__int_as_float(0x7f800000);
    pos[i] = -1;
  }
};

}  // namespace dsa
