// Device work queue across decode steps.
//
// A serving loop calls the indexer once per decode step against the same
// requests: each request's length grows by one token per step and its block
// table grows by one page every 64 tokens, while requests are admitted and
// retired between steps. Here the request table (length and block-table row
// of every request slot) stays in device memory from step to step, and a
// step ships one small record of what changed plus the step's batch as a
// list of slots. Two kernels turn that record into the indexer's inputs:
//   decode_queue_apply_kernel   one CTA: the record's events, in order
//                               (admit with a page list, append one page,
//                               set a length, retire);
//   decode_queue_gather_kernel  one CTA per batch row: advance the listed
//                               request's length and copy its visible
//                               block-table entries into the batch buffers
//                               (rows past the batch get length 0).
// Every index is checked; a malformed record raises DSA_STATUS_BAD_RECORD and
// the offending event or row is skipped (an empty row), never a fault.
// The reference has no counterpart: its entry point takes a host-built batch
// on every call (solution/cuda/kernel.cu:818-887).
#pragma once
#include <cstdint>
#include "dsa_topk_indexer.h"
#include "indexer_kernel.cuh"  // g_dsa_status

namespace dsa {

constexpr int kQueueThreads = 256;

// Header words of a record; events start at DSA_QUEUE_HEADER_WORDS.
struct QueueHeader {
  int64_t words, events_end, batch, batch_off;
  int32_t advance, n_events;
  bool ok;
};

__device__ __forceinline__ QueueHeader read_queue_header(const int32_t* rec, int64_t rec_words, int64_t capacity) {
  QueueHeader h;
  h.words = rec[0];
  h.n_events = rec[1];
  h.batch = rec[2];
  h.advance = rec[3];
  h.batch_off = rec[4];
  h.events_end = h.batch_off;
  h.ok = h.words >= DSA_QUEUE_HEADER_WORDS && h.words <= rec_words && h.n_events >= 0 && h.batch >= 0 &&
         h.batch <= capacity && h.advance >= 0 && h.batch_off >= DSA_QUEUE_HEADER_WORDS &&
         h.batch_off + h.batch <= h.words;
  return h;
}

__global__ void __launch_bounds__(kQueueThreads)
    decode_queue_apply_kernel(const int32_t* __restrict__ rec, int64_t rec_words, int32_t* __restrict__ req_len,
                              int32_t* __restrict__ req_bt, int64_t num_slots, int32_t max_pages,
                              int64_t capacity) {
  const QueueHeader h = read_queue_header(rec, rec_words, capacity);
  if (!h.ok) {
    if (threadIdx.x == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
    return;
  }
  // Every thread reads the same words, so every branch below is uniform.
  int64_t off = DSA_QUEUE_HEADER_WORDS;
  for (int e = 0; e < h.n_events; ++e) {
    if (off + 4 > h.events_end) {
      if (threadIdx.x == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
      return;
    }
    const int32_t type = rec[off], slot = rec[off + 1], a = rec[off + 2], b = rec[off + 3];
    off += 4;
    const bool slot_ok = slot >= 0 && static_cast<int64_t>(slot) < num_slots;
    int32_t* row = req_bt + static_cast<int64_t>(slot_ok ? slot : 0) * max_pages;
    bool bad = !slot_ok;
    if (type == DSA_QUEUE_ADMIT) {
      // a = length, b = pages listed next (padded to a multiple of 4 words)
      const int64_t pw = (static_cast<int64_t>(b) + 3) & ~static_cast<int64_t>(3);
      if (b < 0 || b > max_pages || off + pw > h.events_end) {
        if (threadIdx.x == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
        return;  // the rest of the record cannot be located
      }
      bad |= a < 0;
      if (!bad) {
        for (int i = threadIdx.x; i < b; i += kQueueThreads) row[i] = rec[off + i];
        if (threadIdx.x == 0) req_len[slot] = a;
      }
      off += pw;
    } else if (type == DSA_QUEUE_APPEND_PAGE) {  // a = page index in the row, b = page id
      bad |= a < 0 || a >= max_pages;
      if (!bad && threadIdx.x == 0) row[a] = b;
    } else if (type == DSA_QUEUE_SET_LEN) {  // a = length
      bad |= a < 0;
      if (!bad && threadIdx.x == 0) req_len[slot] = a;
    } else if (type == DSA_QUEUE_RETIRE) {
      if (!bad && threadIdx.x == 0) req_len[slot] = -1;
    } else {
      if (threadIdx.x == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
      return;  // unknown event: the record is not trusted past this point
    }
    if (bad && threadIdx.x == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
    __syncthreads();  // a later event may touch the same row
  }
}

__global__ void __launch_bounds__(kQueueThreads)
    decode_queue_gather_kernel(const int32_t* __restrict__ rec, int64_t rec_words, int32_t* __restrict__ req_len,
                               const int32_t* __restrict__ req_bt, int64_t num_slots, int32_t max_pages,
                               int32_t* __restrict__ seq_lens, int32_t* __restrict__ block_table,
                               int64_t capacity) {
  const int64_t b = blockIdx.x;
  const QueueHeader h = read_queue_header(rec, rec_words, capacity);
  if (!h.ok || b >= h.batch) {
    if (threadIdx.x == 0) seq_lens[b] = 0;  // the apply kernel reported a bad header
    return;
  }
  const int32_t slot = rec[h.batch_off + b];
  const bool slot_ok = slot >= 0 && static_cast<int64_t>(slot) < num_slots;
  const int32_t len0 = slot_ok ? req_len[slot] : -1;
  if (len0 < 0) {  // out of range or not admitted: an empty row
    if (threadIdx.x == 0) {
      seq_lens[b] = 0;
      atomicOr(&g_dsa_status, DSA_STATUS_BAD_RECORD);
    }
    return;
  }
  const int64_t len64 = static_cast<int64_t>(len0) + h.advance;
  const int32_t len = len64 > INT32_MAX ? INT32_MAX : static_cast<int32_t>(len64);
  __syncthreads();  // every thread has read req_len[slot] before it changes
  if (threadIdx.x == 0) {
    req_len[slot] = len;
    seq_lens[b] = len;
  }
  int64_t npg = (static_cast<int64_t>(len) + 63) / 64;
  npg = npg < max_pages ? npg : max_pages;
  const int32_t* src = req_bt + static_cast<int64_t>(slot) * max_pages;
  int32_t* dst = block_table + b * max_pages;
  for (int64_t i = threadIdx.x; i < npg; i += kQueueThreads) dst[i] = src[i];
}

}  // namespace dsa
