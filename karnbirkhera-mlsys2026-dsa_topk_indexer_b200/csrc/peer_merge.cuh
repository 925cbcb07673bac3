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

// One CTA (kMergeThreads) per merged row: row p.row_begin + blockIdx.x.
__global__ void __launch_bounds__(kMergeThreads) peer_merge_kernel(const PeerParams p) {
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
  auto list = [&](int r, uint64_t* dst) {
    const uint8_t* base = reinterpret_cast<const uint8_t*>(p.bases[r]);
    load_list(reinterpret_cast<const float*>(base + p.lay.scores()) + row,
              reinterpret_cast<const int32_t*>(base + p.lay.pos()) + row, dst, key_cap);
  };
  list(0, cur);
#pragma unroll 1
  for (int j = 1; j < p.nranks; ++j) {
    list(j, nxt);
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
