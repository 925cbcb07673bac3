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

// Group barrier: BAR == 0 is __syncthreads(), otherwise a named barrier over
// the NT threads of the group.
template <int NT, int BAR>
__device__ __forceinline__ void group_sync() {
  if (BAR == 0)
    __syncthreads();
  else
    ptx::named_bar(BAR, NT);
}

// Adds this lane's digit to hist (256 bins), one atomic per distinct digit in
// the warp. Scores of one row share their high bits, so plain per-lane
// atomics would serialise on one or two bins. All 32 lanes must call it.
__device__ __forceinline__ void warp_hist_add(uint32_t* hist, bool active, uint32_t digit) {
  const uint32_t d = active ? digit : 256u;
  const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
  const int lane = threadIdx.x & 31;
  if (active && (__ffs(peers) - 1) == lane) atomicAdd(&hist[d], static_cast<uint32_t>(__popc(peers)));
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

// Radix select over keys cand[0..n) held in shared memory by a group of NT
// threads (gt = thread index in the group, warp 0 of the group does the
// digit scan). Precondition: n > k, group synchronised. Returns T such that
// exactly k keys are >= T. Eight passes of 8 bits at most; stops as soon as
// the boundary bucket is taken whole.
template <int NT, int BAR>
__device__ uint64_t group_select(const uint64_t* cand, uint32_t n, uint32_t k, uint32_t* hist, uint32_t* sel,
                                 int gt) {
  uint64_t prefix = 0;
  uint32_t krem = k;
#pragma unroll 1
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = gt; i < 256; i += NT) hist[i] = 0u;
    group_sync<NT, BAR>();
    const uint64_t hi_mask = (shift == 56) ? 0ull : (~0ull << (shift + 8));
    for (uint32_t i0 = 0; i0 < n; i0 += NT) {
      const uint32_t i = i0 + gt;
      const uint64_t key = i < n ? cand[i] : 0ull;
      warp_hist_add(hist, i < n && (key & hi_mask) == prefix, static_cast<uint32_t>(key >> shift) & 255u);
    }
    group_sync<NT, BAR>();
    if (gt < 32) find_digit_warp(hist, krem, sel);
    group_sync<NT, BAR>();
    const uint32_t d = sel[0], cgt = sel[1], cd = sel[2];
    prefix |= static_cast<uint64_t>(d) << shift;
    krem -= cgt;
    if (cd == krem) break;
  }
  return prefix;
}

// Keeps the keys >= T of cand[0..n) and packs them to the front; `counter`
// ends holding the number kept. MAXPER >= ceil(n / NT).
template <int NT, int BAR, int MAXPER>
__device__ void group_compact(uint64_t* cand, uint32_t n, uint64_t T, uint32_t* counter, int gt) {
  uint64_t v[MAXPER];
#pragma unroll
  for (int j = 0; j < MAXPER; ++j) {
    const uint32_t i = gt + j * NT;
    v[j] = (i < n) ? cand[i] : 0ull;
  }
  if (gt == 0) *counter = 0u;
  group_sync<NT, BAR>();
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < MAXPER; ++j) {
    const uint32_t i = gt + j * NT;
    const bool keep = (i < n) && (v[j] >= T);
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
    if (m) {
      const int leader = __ffs(m) - 1;
      uint32_t base = 0;
      if (lane == leader) base = atomicAdd(counter, static_cast<uint32_t>(__popc(m)));
      base = __shfl_sync(0xFFFFFFFFu, base, leader);
      if (keep) cand[base + __popc(m & lanemask_lt())] = v[j];
    }
  }
  group_sync<NT, BAR>();
}

// Sorts buf[0..2048) descending. 256 threads; thread t owns elements
// [8t, 8t+8). Bitonic network: partner distances 1..4 inside a thread,
// 8..128 across lanes of a warp (shuffles), 256..1024 through shared memory.
__device__ __forceinline__ void cmpx(uint64_t& a, uint64_t& b, bool desc) {
  const bool sw = desc ? (a < b) : (a > b);
  const uint64_t x = sw ? b : a, y = sw ? a : b;
  a = x;
  b = y;
}

__device__ void block_sort_desc_2048(uint64_t* buf, uint64_t (&v)[8]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int r = 0; r < 8; ++r) v[r] = buf[t * 8 + r];
#pragma unroll
  for (int k = 2; k <= 2048; k <<= 1) {
    if (k >= 512) {
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 8; ++r) buf[t * 8 + r] = v[r];
      __syncthreads();
#pragma unroll
      for (int j = k >> 1; j >= 256; j >>= 1) {
        const int lj = __ffs(j) - 1;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int p = t + 256 * m;
          const int i = ((p >> lj) << (lj + 1)) | (p & (j - 1));
          const int l = i | j;
          uint64_t a = buf[i], c = buf[l];
          cmpx(a, c, (i & k) == 0);
          buf[i] = a;
          buf[l] = c;
        }
        __syncthreads();
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) v[r] = buf[t * 8 + r];
    }
#pragma unroll
    for (int j = ((k >> 1) < 128 ? (k >> 1) : 128); j >= 1; j >>= 1) {
      if (j >= 8) {
        const int lx = j >> 3;
        const bool lower = ((t & lx) == 0);
        const bool desc = ((t * 8) & k) == 0;
        const bool keep_max = (lower == desc);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint64_t p = __shfl_xor_sync(0xFFFFFFFFu, v[r], lx);
          v[r] = keep_max ? (v[r] > p ? v[r] : p) : (v[r] < p ? v[r] : p);
        }
      } else {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if ((r & j) == 0) cmpx(v[r], v[r | j], ((t * 8 + r) & k) == 0);
        }
      }
    }
  }
}

}  // namespace dsa
