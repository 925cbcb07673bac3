// Key-axis sharding without a collective library: the exchange of candidate
// lists, their merge and the distribution of the merged rows as one protocol
// over NVLink peer memory.
//
// Every rank owns one region, opened by every other rank through a CUDA IPC
// handle (plain peer loads and stores, no multicast):
//   [0, L)           cand_scores [B, 2048] fp32   (this rank's key range)
//   [L, 2L)          cand_pos    [B, 2048] int32  (logical positions)
//   [2L, 3L)         out         [B, 2048] int32  (merged rows, written by
//                                                  the rank that merges them)
//   [3L, 3L + 256)   ready flags [64] uint32      (flag s = step counter of
//   [3L+256, 3L+512) done flags  [64] uint32       rank s)
// with L = B * 2048 * 4 bytes. One step, rank r of N, step counter e:
//   signal ready  every rank's ready[r] = e (after r's partial lists are written);
//   merge         rows [B r / N, B (r+1) / N): wait for ready[0..N) = e in
//                 r's own region, merge the N lists read from the peers'
//                 regions (the same merge-path fold as the one-GPU merge),
//                 translate through the block table and store each row into
//                 every rank's out;
//   signal done   every rank's done[r] = e;
//   wait done     until done[0..N) = e in r's own region: every row of out
//                 has landed and no peer still reads r's lists.
// Every wait is bounded (%globaltimer); a wait that runs out raises
// DSA_STATUS_WAIT_TIMEOUT and its CTA writes nothing. Writes before a flag
// are published with a system-scope fence and a release store; flags are
// read with acquire loads. The reference has no multi-GPU path; this is the
// exchange its north star names (all-gather of candidate lists over NVLink,
// then a GPU merge), fused into the merge kernel.
#pragma once
#include <cstdint>
#include "dsa_topk_indexer.h"
#include "indexer_kernel.cuh"

namespace dsa {

constexpr int kPeerMaxRanks = 64;
constexpr int kPeerFlagBytes = 2 * kPeerMaxRanks * 4;

struct PeerLayout {
  int64_t list_bytes;  // B * 2048 * 4
  __host__ __device__ int64_t scores() const { return 0; }
  __host__ __device__ int64_t pos() const { return list_bytes; }
  __host__ __device__ int64_t out() const { return 2 * list_bytes; }
  __host__ __device__ int64_t flags(int which) const { return 3 * list_bytes + which * kPeerMaxRanks * 4; }
  __host__ __device__ int64_t total() const { return 3 * list_bytes + kPeerFlagBytes; }
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Whole CTA: true once flags[0..n) all reached `epoch` (wrap-safe), false
// after limit_ns (status bit raised). Thread t < n watches flag t.
__device__ __forceinline__ bool peer_wait_flags(const uint32_t* flags, int n, uint32_t epoch, uint64_t limit_ns) {
  bool ok = true;
  if (static_cast<int>(threadIdx.x) < n) {
    const uint64_t t0 = ptx::globaltimer();
    while (static_cast<int32_t>(ld_acquire_sys(flags + threadIdx.x) - epoch) < 0) {
      if (ptx::globaltimer() - t0 > limit_ns) {
        ok = false;
        atomicOr(&g_dsa_status, DSA_STATUS_WAIT_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

struct PeerParams {
  const uint64_t* bases;  // [nranks] region base of every rank, as this rank addresses it
  int32_t nranks, rank;
  uint32_t epoch;
  PeerLayout lay;
  int32_t batch, max_pages;
  int32_t row_begin;      // first row this rank merges
  const int32_t* block_table;
  uint64_t wait_ns;
};

// One CTA, nranks threads: flag `which` (0 ready, 1 done) of this rank in
// every rank's region.
__global__ void peer_signal_kernel(const PeerParams p, int which) {
  __threadfence_system();  // everything this rank wrote before is visible first
  if (static_cast<int>(threadIdx.x) < p.nranks) {
    uint8_t* base = reinterpret_cast<uint8_t*>(p.bases[threadIdx.x]);
    st_release_sys(reinterpret_cast<uint32_t*>(base + p.lay.flags(which)) + p.rank, p.epoch);
  }
}

// One CTA: waits for flag `which` of every rank in this rank's own region.
__global__ void peer_wait_kernel(const PeerParams p, int which) {
  const uint8_t* base = reinterpret_cast<const uint8_t*>(p.bases[p.rank]);
  peer_wait_flags(reinterpret_cast<const uint32_t*>(base + p.lay.flags(which)), p.nranks, p.epoch, p.wait_ns);
}

// One list's eight entries of this thread ([8t, 8t+8) of the row), fetched
// with four 16-byte loads that are all in flight at once: a list in a peer's
// memory costs one NVLink round trip, not eight.
struct PeerListRegs {
  float4 s0, s1;
  int4 p0, p1;
};

__device__ __forceinline__ PeerListRegs peer_fetch(const PeerParams& p, int r, int64_t row) {
  const uint8_t* base = reinterpret_cast<const uint8_t*>(p.bases[r]);
  const float4* s = reinterpret_cast<const float4*>(base + p.lay.scores()) + (row + threadIdx.x * 8) / 4;
  const int4* q = reinterpret_cast<const int4*>(base + p.lay.pos()) + (row + threadIdx.x * 8) / 4;
  return PeerListRegs{s[0], s[1], q[0], q[1]};
}

// The keys of load_list (same packing, same treatment of out-of-range
// positions) from fetched registers.
__device__ __forceinline__ void peer_store_keys(const PeerListRegs& v, uint64_t* dst, int64_t key_cap) {
  const float sc[8] = {v.s0.x, v.s0.y, v.s0.z, v.s0.w, v.s1.x, v.s1.y, v.s1.z, v.s1.w};
  const int32_t ps[8] = {v.p0.x, v.p0.y, v.p0.z, v.p0.w, v.p1.x, v.p1.y, v.p1.z, v.p1.w};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool ok = ps[k] >= 0 && static_cast<int64_t>(ps[k]) < key_cap;
    if (ps[k] >= 0 && !ok) atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);
    dst[threadIdx.x * 8 + k] = ok ? pack_key(sc[k], static_cast<uint32_t>(ps[k])) : 0ull;
  }
}

// One CTA (kMergeThreads) per merged row: row p.row_begin + blockIdx.x.
__global__ void __launch_bounds__(kMergeThreads) peer_merge_kernel(const PeerParams p) {
  static_assert(kMergeThreads * 8 == kTopK, "eight entries of a list per thread");
  extern __shared__ __align__(16) uint8_t msmem[];
  uint64_t* cur = reinterpret_cast<uint64_t*>(msmem);
  uint64_t* nxt = cur + kTopK;
  uint64_t* res = nxt + kTopK;
  const uint8_t* own = reinterpret_cast<const uint8_t*>(p.bases[p.rank]);
  if (!peer_wait_flags(reinterpret_cast<const uint32_t*>(own + p.lay.flags(0)), p.nranks, p.epoch, p.wait_ns))
    return;  // uniform over the CTA
  const int b = p.row_begin + static_cast<int>(blockIdx.x);
  const int64_t row = static_cast<int64_t>(b) * kTopK;
  const int64_t key_cap = static_cast<int64_t>(p.max_pages) * kPage;
  // Lists 0 and 1 are fetched together; list j + 1 is in flight while list
  // j is merged.
  const PeerListRegs first = peer_fetch(p, 0, row);
  PeerListRegs next = first;
  if (p.nranks > 1) next = peer_fetch(p, 1, row);
  peer_store_keys(first, cur, key_cap);
#pragma unroll 1
  for (int j = 1; j < p.nranks; ++j) {
    peer_store_keys(next, nxt, key_cap);
    if (j + 1 < p.nranks) next = peer_fetch(p, j + 1, row);
    __syncthreads();
    merge_top(cur, nxt, res);
    __syncthreads();
    uint64_t* t = cur;
    cur = res;
    res = t;
  }
  __syncthreads();
  const int32_t* bt_row = p.block_table + static_cast<int64_t>(b) * p.max_pages;
  int4 v[2];
  int32_t* vv = reinterpret_cast<int32_t*>(v);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint64_t key = cur[threadIdx.x * 8 + k];
    const uint32_t pos = key_pos(key);
    vv[k] = key ? bt_row[pos >> 6] * kPage + static_cast<int32_t>(pos & 63u) : -1;
  }
  // The row goes to every rank's out (two 16-byte stores per thread and rank).
#pragma unroll 1
  for (int r = 0; r < p.nranks; ++r) {
    int4* dst = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(p.bases[r]) + p.lay.out()) +
                (row + threadIdx.x * 8) / 4;
    dst[0] = v[0];
    dst[1] = v[1];
  }
  __threadfence_system();
}

}  // namespace dsa
