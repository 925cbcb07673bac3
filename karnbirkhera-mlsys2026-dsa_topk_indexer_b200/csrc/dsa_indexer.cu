// C-ABI implementation of the B200 DSA lightning-indexer top-K.
// Kernels: indexer_kernel<mode> (indexer_kernel.cuh) and merge_kernel below.
// Host responsibilities: argument checks, TMA tensor maps, cluster sizing,
// launches. No device allocation, no stream synchronisation.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "dsa_topk_indexer.h"
#include "indexer_kernel.cuh"
#include "prefill_kernel.cuh"
#include "cache_writer.cuh"
#include "sparse_attention.cuh"
#include "decode_queue.cuh"

namespace dsa {

// --------------------------------------------------------------- merge kernel
// Merges nparts best-first candidate lists (score, logical position) of one
// request into its final top-2048 physical slots (key-axis sharding: each
// list is one key range's best 2048, already in descending key order). One
// 256-thread CTA per request folds the lists in one at a time with a
// merge-path merge that keeps the top 2048: thread t finds by binary search
// how many of its 8 output ranks [8t, 8t+8) come from each list, then merges
// those 8 sequentially. The result is sorted, so it is translated and written
// directly. Missing entries (position < 0) become key 0, below every real key.
constexpr int kMergeThreads = 256;
constexpr int kMergeSmem = 3 * kTopK * 8;  // current result, next list, output

// Positions outside [0, key_cap) (key_cap = max_pages * 64) are treated as
// missing: they could not be translated through the block-table row, so a
// list that holds one (e.g. lists paired with the wrong block-table rows)
// flags DSA_STATUS_BAD_PAGE instead of reading past the row.
__device__ __forceinline__ void load_list(const float* __restrict__ sc, const int32_t* __restrict__ ps,
                                          uint64_t* dst, int64_t key_cap) {
  for (int i = threadIdx.x; i < kTopK; i += kMergeThreads) {
    const int32_t pos = ps[i];
    const bool ok = pos >= 0 && static_cast<int64_t>(pos) < key_cap;
    if (pos >= 0 && !ok) atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);
    dst[i] = ok ? pack_key(sc[i], static_cast<uint32_t>(pos)) : 0ull;
  }
}

// C[0..2048) = the 2048 largest of A[0..2048) and B[0..2048), descending
// (both inputs descending; ties, only between padding zeros, go to B).
__device__ __forceinline__ void merge_top(const uint64_t* A, const uint64_t* B, uint64_t* C) {
  const int d = threadIdx.x * 8;
  int lo = 0, hi = d;  // number of A elements among the first d outputs
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (A[mid] > B[d - 1 - mid]) lo = mid + 1; else hi = mid;
  }
  int i = lo, j = d - lo;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool take_a = i < kTopK && (j >= kTopK || A[i] > B[j]);
    C[d + k] = take_a ? A[i] : B[j];
    i += take_a ? 1 : 0;
    j += take_a ? 0 : 1;
  }
}

__global__ void __launch_bounds__(kMergeThreads)
    merge_kernel(const float* __restrict__ cand_scores, const int32_t* __restrict__ cand_pos, int nparts,
                 const int32_t* __restrict__ block_table, int32_t* __restrict__ out, int batch, int max_pages) {
  extern __shared__ __align__(16) uint8_t msmem[];
  uint64_t* cur = reinterpret_cast<uint64_t*>(msmem);
  uint64_t* nxt = cur + kTopK;
  uint64_t* res = nxt + kTopK;
  const int b = blockIdx.x;
  const int64_t row = static_cast<int64_t>(b) * kTopK;
  const int64_t part = static_cast<int64_t>(batch) * kTopK;
  const int64_t key_cap = static_cast<int64_t>(max_pages) * kPage;
  load_list(cand_scores + row, cand_pos + row, cur, key_cap);
#pragma unroll 1
  for (int j = 1; j < nparts; ++j) {
    load_list(cand_scores + j * part + row, cand_pos + j * part + row, nxt, key_cap);
    __syncthreads();
    merge_top(cur, nxt, res);
    __syncthreads();
    uint64_t* t = cur;
    cur = res;
    res = t;
  }
  __syncthreads();
  const int32_t* bt_row = block_table + static_cast<int64_t>(b) * max_pages;
  int32_t v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint64_t key = cur[threadIdx.x * 8 + k];
    const uint32_t pos = key_pos(key);
    v[k] = key ? bt_row[pos >> 6] * kPage + static_cast<int32_t>(pos & 63u) : -1;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) out[row + threadIdx.x * 8 + k] = v[k];
}

// Fills a float buffer (used for the -inf background of the score rows).
__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

thread_local int t_last_launches = 0;
thread_local const char* t_last_path = "";

// Optional per-kernel timing (dsa_topk_indexer_set_timing).
std::atomic<int> g_timing{0};
thread_local cudaEvent_t t_ev_begin = nullptr, t_ev_end = nullptr;
thread_local bool t_timed = false;

// Brackets the dominant kernel of a call with timing events when timing is
// on and the stream is not being captured.
struct KernelTimer {
  cudaStream_t stream;
  bool on = false;
  explicit KernelTimer(cudaStream_t s) : stream(s) {
    t_timed = false;
    if (!g_timing.load()) return;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return;
    if (!t_ev_begin && (cudaEventCreate(&t_ev_begin) != cudaSuccess || cudaEventCreate(&t_ev_end) != cudaSuccess))
      return;
    on = cudaEventRecord(t_ev_begin, s) == cudaSuccess;
  }
  void stop() {
    if (on && cudaEventRecord(t_ev_end, stream) == cudaSuccess) t_timed = true;
    on = false;
  }
};

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  bool ready = false;
  int num_sms = 148;
  int64_t l2_bytes = 0;
};
DeviceInfo g_devices[kMaxDevices];
std::mutex g_dev_mutex;

// Per-device one-time set-up: architecture check and kernel attributes.
int prepare_device(int* num_sms, int64_t* l2_bytes = nullptr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_devices[dev];
  if (!d.ready) {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return DSA_ERR_CUDA;
    if (prop.major != 10 || prop.minor != 0) return DSA_ERR_NO_DEVICE;
    d.num_sms = prop.multiProcessorCount;
    d.l2_bytes = prop.l2CacheSize;
    const void* fns[5] = {reinterpret_cast<const void*>(&indexer_kernel<kModeTopK>),
                          reinterpret_cast<const void*>(&indexer_kernel<kModeScores>),
                          reinterpret_cast<const void*>(&indexer_kernel<kModePartial>),
                          reinterpret_cast<const void*>(&indexer_kernel<kModeTopK, true>),
                          reinterpret_cast<const void*>(&indexer_kernel<kModePartial, true>)};
    for (const void* f : fns) {
      if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess ||
          cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return DSA_ERR_CUDA;
    }
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(&prefill_kernel<kModeTopK>),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(&prefill_kernel<kModePartial>),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes) != cudaSuccess)
      return DSA_ERR_CUDA;
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(&merge_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kMergeSmem) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(&cache_write_kernel<true>),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, WriterGeom<true>::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(&cache_write_kernel<false>),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, WriterGeom<false>::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(&sparse_attention_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SaLayout::kBytes) != cudaSuccess)
      return DSA_ERR_CUDA;
    d.ready = true;
  }
  *num_sms = d.num_sms;
  if (l2_bytes) *l2_bytes = d.l2_bytes;
  return DSA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Library-owned device workspace, one per (device, stream): calls on one
// stream are ordered, so its contents are never shared by work in flight on
// two streams. Allocated outside stream capture the first time a launch
// needs it and grown (never shrunk) on demand; replaced buffers are kept
// until exit because work queued earlier may still read them.
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  // Second stream for a concurrent launch, with the events that fork it
  // from and join it back to the caller's stream (created outside capture).
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::map<std::pair<int, cudaStream_t>, Workspace> g_workspaces;
std::vector<void*> g_retired;
std::mutex g_ws_mutex;

// Returns the workspace of (current device, stream) with at least `bytes`, or
// null if it would have to be allocated while the stream is being captured.
void* workspace(cudaStream_t stream, size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  Workspace& ws = g_workspaces[{dev, stream}];
  if (ws.bytes >= bytes) return ws.ptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return nullptr;
  size_t want = bytes < (1u << 16) ? (1u << 16) : bytes;
  if (want < 2 * ws.bytes) want = 2 * ws.bytes;
  void* fresh = nullptr;
  if (cudaMalloc(&fresh, want) != cudaSuccess) return nullptr;
  if (ws.ptr) g_retired.push_back(ws.ptr);
  ws.ptr = fresh;
  ws.bytes = want;
  return ws.ptr;
}

// The side stream and fork/join events of (current device, stream); false if
// they would have to be created while the stream is being captured.
bool side_stream(cudaStream_t stream, cudaStream_t* side, cudaEvent_t* fork, cudaEvent_t* join) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  Workspace& ws = g_workspaces[{dev, stream}];
  if (!ws.side) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return false;
    cudaStream_t s = nullptr;
    cudaEvent_t f = nullptr, j = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return false;
    if (cudaEventCreateWithFlags(&f, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&j, cudaEventDisableTiming) != cudaSuccess) {
      if (f) cudaEventDestroy(f);
      cudaStreamDestroy(s);
      return false;
    }
    ws.side = s;
    ws.fork = f;
    ws.join = j;
  }
  *side = ws.side;
  *fork = ws.fork;
  *join = ws.join;
  return true;
}

// Tensor maps over the caller's buffers (encoded per call: they hold the
// base address).
int make_maps(const void* q, const void* kcache, int64_t batch, int64_t num_pages, CUtensorMap* tk,
              CUtensorMap* tq) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return DSA_ERR_CUDA;
  std::memset(tk, 0, sizeof(*tk));
  std::memset(tq, 0, sizeof(*tq));
  const cuuint32_t estr[3] = {1, 1, 1};
  {  // page data: {128 bytes, 64 tokens, num_pages}, box = one page, 128-byte swizzle
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(kPage),
                                static_cast<cuuint64_t>(num_pages)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(kPageBytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kDim), static_cast<cuuint32_t>(kPage), 1};
    if (enc(tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(kcache), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DSA_ERR_CUDA;
  }
  {  // q: {128 bytes, B*64 head rows}, box = one query (64 heads), 128-byte swizzle
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(batch * kHeads)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kDim)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kDim), static_cast<cuuint32_t>(kHeads)};
    if (enc(tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

// CTAs per request (the cluster size). About four CTAs per SM in total, so
// short batches split their rows widely (latency) while large batches keep
// whole rows on few CTAs (less merging per byte); rounded down above 2 (one
// fewer cluster wave beats one more CTA per row); never fewer than about 4
// tiles per CTA. Measured on B200 (config 2 rows): B=64 -> 8 (best of
// 4/6/7/8/16), B=128 -> 4 (best of 3/4/5/6), B=256 -> 2 (2 and 3 equal),
// B=512 -> 2 (best of 1/2/4/8). 16-CTA clusters lost everywhere.
int choose_cluster(int64_t batch, int64_t span_pages, int num_sms) {
  // DSA_TOPK_CLUSTER=<1..16> overrides the choice (tuning and tests; sizes
  // above 8 are a non-portable cluster size B200 supports).
  if (const char* env = std::getenv("DSA_TOPK_CLUSTER")) {
    const int g = std::atoi(env);
    if (g >= 1 && g <= 16) return g;
  }
  const int64_t tiles = (span_pages + 1) / 2;
  int64_t g = (4 * static_cast<int64_t>(num_sms) + batch - 1) / batch;
  if (g > 2) g = (4 * static_cast<int64_t>(num_sms)) / batch;
  const int64_t g_floor = (tiles + 3) / 4;
  if (g > g_floor) g = g_floor;
  if (g < 1) g = 1;
  if (g > 8) g = 8;
  return static_cast<int>(g);
}

int check_common(const void* q, const void* kcache, const float* w, const int32_t* sl, const int32_t* bt,
                 int64_t batch, int64_t max_pages, int64_t num_pages) {
  if (batch < 0 || max_pages < 1 || num_pages < 1) return DSA_ERR_INVALID_ARG;
  if (batch == 0) return DSA_OK;
  if (!q || !kcache || !w || !sl || !bt) return DSA_ERR_INVALID_ARG;
  if (num_pages > INT32_MAX || max_pages > INT32_MAX / kPage || batch > INT32_MAX / kHeads)
    return DSA_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(kcache)) return DSA_ERR_MISALIGNED;
  return DSA_OK;
}

// Batches of at least kPrefillMinRows rows whose block table must share
// pages (more entries than kPrefillShareFactor times the pool holds pages:
// causal prefill rows of one sequence) first go through the shared-sequence
// kernel (prefill_kernel), which serves every group of four consecutive rows
// that really read the same pages and leaves the others to the per-row
// kernel. Measured on B200: 8192-row causal prefill 0.913 vs 0.951 ms,
// 2048-row long context 4.00 vs 4.07 ms. Decode batches (distinct pages per
// row) never take it: its launches would add ~10 us for nothing.
// DSA_TOPK_PREFILL=0 turns it off, =1 tries it on any batch of 256+ rows.
constexpr int64_t kPrefillMinRows = 256;
// Cluster sizes up to which the last partial wave runs as its own launch.
constexpr int kTailMaxG = 4;
constexpr int64_t kPrefillShareFactor = 4;

template <int kMode>
int launch_indexer(const void* q, const void* kcache, const IndexerParams& prm, int64_t span_pages,
                   cudaStream_t stream) {
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  CUtensorMap tk, tq;
  rc = make_maps(q, kcache, prm.batch, prm.num_pages, &tk, &tq);
  if (rc != DSA_OK) return rc;
  const int G = choose_cluster(prm.batch, span_pages, num_sms);
  IndexerParams params = prm;
  int launches = 1;
  auto launch = [&](const IndexerParams& pp, int64_t rows, int g, cudaStream_t st) -> int {
    // Two-class launches with in-kernel ranking use the instantiation that
    // decides the split on the device.
    void (*kern)(CUtensorMap, CUtensorMap, IndexerParams) = indexer_kernel<kMode>;
    if constexpr (kMode != kModeScores) {
      if (pp.split_role >= 0) kern = indexer_kernel<kMode, true>;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(g * rows), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(g);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tk, tq, pp) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
  };

  // Shared-sequence stage: plan (row order + group order), then the prefill
  // kernel over the groups, longest first; the per-row kernel below skips
  // the rows it served.
  if constexpr (kMode != kModeScores) {
    const char* env = std::getenv("DSA_TOPK_PREFILL");
    const int64_t B = prm.batch;
    const int64_t ngroups = (B + kGroupRows - 1) / kGroupRows;
    bool shared = B >= kPrefillMinRows && B * static_cast<int64_t>(prm.max_pages) > kPrefillShareFactor * prm.num_pages;
    if (env && env[0] == '0') shared = false;
    if (env && env[0] == '1') shared = B >= kPrefillMinRows;
    uint8_t* ws = shared ? static_cast<uint8_t*>(workspace(stream, static_cast<size_t>(8 * B + 4 * ngroups)))
                         : nullptr;
    if (ws) {
      int32_t* order = reinterpret_cast<int32_t*>(ws);
      int32_t* handled = order + B;
      int32_t* group_order = handled + B;
      lpt_order_kernel<<<1, kPlanThreads, 0, stream>>>(prm.seq_lens, prm.batch, prm.max_pages, order, group_order);
      if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
      PrefillParams pp{group_order, handled};
      KernelTimer timer(stream);
      prefill_kernel<kMode><<<static_cast<unsigned>(ngroups), kPThreads, kPSmemBytes, stream>>>(tk, tq, prm, pp);
      if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
      params.order = order;
      params.order_base = -1;
      params.handled = handled;
      if ((rc = launch(params, prm.batch, G, stream)) != DSA_OK) return rc;
      timer.stop();
      t_last_launches = 3;
      t_last_path = "prefill+cluster";
      return DSA_OK;
    }
  }

  // More clusters than fit at once: serve the longest rows first so that no
  // long row starts in the last wave. Small batches rank their rows inside
  // the kernel (no plan launch); larger ones get a one-CTA plan kernel.
  if (prm.batch > 1 && static_cast<int64_t>(G) * prm.batch > 2 * num_sms) {
    int32_t* order = nullptr;
    if (prm.batch <= kInKernelOrderMax) {
      params.order = nullptr;
      params.order_base = 0;
    } else {
      order = static_cast<int32_t*>(workspace(stream, static_cast<size_t>(prm.batch) * sizeof(int32_t)));
      if (order) {
        lpt_order_kernel<<<1, kPlanThreads, 0, stream>>>(prm.seq_lens, prm.batch, prm.max_pages, order, nullptr);
        if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
        params.order = order;
        launches = 2;
      }
    }
    // Several waves of G-CTA clusters end in a partial wave that holds the
    // shortest rows and fills the GPU poorly. Those rows run as a second
    // launch with more CTAs per row, issued after the first on a second
    // stream, so that their clusters take the slots of the first launch's
    // last wave as they free (DSA_TOPK_TAIL=0 turns this off). Measured on
    // B200 for config 2 (512 rows: three waves of 148 two-CTA clusters, then
    // 68 rows that filled 136 of 296 slots; now at 4 CTAs each): 0.800 ->
    // 0.776 ms; 128-row batches at 4 CTAs (54 rows at 5): 0.260 -> 0.253 ms.
    // It takes precedence over the two-class launch below.
    if ((order || params.order_base >= 0) && G <= kTailMaxG) {
      const int64_t per_wave = (2 * static_cast<int64_t>(num_sms)) / G;
      const int64_t rem = prm.batch % per_wave;
      int64_t g_tail = rem > 0 ? (2 * static_cast<int64_t>(num_sms)) / rem : 0;
      if (g_tail > 8) g_tail = 8;
      const char* tail_env = std::getenv("DSA_TOPK_TAIL");
      cudaStream_t side = nullptr;
      cudaEvent_t fork = nullptr, join = nullptr;
      if (prm.batch > per_wave && g_tail > G && !(tail_env && tail_env[0] == '0') &&
          side_stream(stream, &side, &fork, &join)) {
        KernelTimer timer(stream);
        if (cudaEventRecord(fork, stream) != cudaSuccess || cudaStreamWaitEvent(side, fork, 0) != cudaSuccess)
          return DSA_ERR_CUDA;
        IndexerParams tail = params;
        if (order)
          tail.order = order + (prm.batch - rem);
        else
          tail.order_base = static_cast<int32_t>(prm.batch - rem);
        if ((rc = launch(params, prm.batch - rem, G, stream)) != DSA_OK) return rc;
        if ((rc = launch(tail, rem, static_cast<int>(g_tail), side)) != DSA_OK) return rc;
        if (cudaEventRecord(join, side) != cudaSuccess || cudaStreamWaitEvent(stream, join, 0) != cudaSuccess)
          return DSA_ERR_CUDA;
        timer.stop();
        t_last_launches = launches + 1;
        t_last_path = "cluster-tail";
        return DSA_OK;
      }
    }
    if (order || params.order_base >= 0) {
      // When the short rows fit at two CTAs each, run everything in one
      // wave: the R longest rows at G CTAs and the rest at 2, as two
      // launches on two streams (DSA_TOPK_SPLIT=0 turns this off).
      constexpr int kGLow = 2;
      const int64_t R = (2 * static_cast<int64_t>(num_sms) - kGLow * prm.batch) / (G - kGLow > 0 ? G - kGLow : 1);
      const char* split_env = std::getenv("DSA_TOPK_SPLIT");
      cudaStream_t side = nullptr;
      cudaEvent_t fork = nullptr, join = nullptr;
      if (G > kGLow && R >= 1 && R < prm.batch && !(split_env && split_env[0] == '0') &&
          side_stream(stream, &side, &fork, &join)) {
        KernelTimer timer(stream);
        if (cudaEventRecord(fork, stream) != cudaSuccess || cudaStreamWaitEvent(side, fork, 0) != cudaSuccess)
          return DSA_ERR_CUDA;
        IndexerParams hi = params, lo = params;
        int64_t hi_rows = R;
        if (order) {
          lo.order = order + R;
        } else if (kMode == kModeScores) {
          lo.order_base = static_cast<int32_t>(R);
        } else {
          // In-kernel ranking: the kernel itself decides, from the lengths,
          // between this split and all rows at G in waves; the G launch then
          // covers every rank and the other one may find nothing to do.
          lo.order_base = static_cast<int32_t>(R);
          hi.split_role = 0;
          lo.split_role = 1;
          for (IndexerParams* q : {&hi, &lo}) {
            q->split_r = static_cast<int32_t>(R);
            q->split_ghi = G;
            q->split_glo = kGLow;
            q->split_slots = 2 * num_sms;
          }
          hi_rows = prm.batch;
        }
        // The small-cluster launch goes first: when the split is taken its
        // clusters get their slots before the G launch's surplus clusters
        // (ranks >= R, which exit at once) are dispatched.
        if ((rc = launch(lo, prm.batch - R, kGLow, side)) != DSA_OK) return rc;
        if ((rc = launch(hi, hi_rows, G, stream)) != DSA_OK) return rc;
        if (cudaEventRecord(join, side) != cudaSuccess || cudaStreamWaitEvent(stream, join, 0) != cudaSuccess)
          return DSA_ERR_CUDA;
        timer.stop();
        t_last_launches = launches + 1;
        t_last_path = "cluster-split";
        return DSA_OK;
      }
    }
  }
  KernelTimer timer(stream);
  if ((rc = launch(params, prm.batch, G, stream)) != DSA_OK) return rc;
  timer.stop();
  t_last_launches = launches;
  t_last_path = "cluster";
  return DSA_OK;
}

// Test hook of dsa_topk_indexer_set_test_fault (off by default).
std::atomic<int> g_test_skip_tile{-1};
std::atomic<uint64_t> g_test_wait_ns{ptx::kWaitTimeoutNs};

IndexerParams base_params(const void* kcache, const float* w, const int32_t* sl, const int32_t* bt, int64_t batch,
                          int64_t max_pages, int64_t num_pages) {
  IndexerParams p{};
  p.kcache = static_cast<const uint8_t*>(kcache);
  p.skip_tile = g_test_skip_tile.load();
  p.wait_ns = g_test_wait_ns.load();
  p.seq_lens = sl;
  p.block_table = bt;
  p.weights = w;
  p.num_pages = num_pages;
  p.max_pages = static_cast<int32_t>(max_pages);
  p.batch = static_cast<int32_t>(batch);
  return p;
}

}  // namespace
}  // namespace dsa

#include "peer_merge.cuh"  // uses load_list / merge_top above

using namespace dsa;

extern "C" int dsa_topk_indexer_launch(const void* q, const void* k_cache, const float* weights,
                                       const int32_t* seq_lens, const int32_t* block_table, int32_t* topk_indices,
                                       int64_t batch, int64_t max_pages, int64_t num_pages, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  int rc = check_common(q, k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  if (rc != DSA_OK || batch == 0) return rc;
  if (!topk_indices) return DSA_ERR_INVALID_ARG;
  IndexerParams p = base_params(k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  p.out = topk_indices;
  return launch_indexer<kModeTopK>(q, k_cache, p, max_pages, static_cast<cudaStream_t>(stream));
}

extern "C" int dsa_topk_indexer_scores(const void* q, const void* k_cache, const float* weights,
                                       const int32_t* seq_lens, const int32_t* block_table, float* scores,
                                       int64_t score_stride, int64_t batch, int64_t max_pages, int64_t num_pages,
                                       void* stream) {
  t_last_launches = 0;
  t_timed = false;
  int rc = check_common(q, k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  if (rc != DSA_OK || batch == 0) return rc;
  if (!scores || score_stride < max_pages * kPage) return DSA_ERR_INVALID_ARG;
  // Columns past each row's length read -inf, as in the reference's
  // final_scores (kernel.cu:433-434).
  const int64_t n = score_stride * batch;
  const int64_t blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  fill_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      scores, n, -__builtin_huge_valf());
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  IndexerParams p = base_params(k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  p.scores = scores;
  p.score_stride = score_stride;
  rc = launch_indexer<kModeScores>(q, k_cache, p, max_pages, static_cast<cudaStream_t>(stream));
  if (rc == DSA_OK) t_last_launches += 1;  // the -inf fill
  return rc;
}

extern "C" int dsa_topk_indexer_partial(const void* q, const void* k_cache, const float* weights,
                                        const int32_t* seq_lens, const int32_t* block_table, int64_t key_begin,
                                        int64_t key_end, float* cand_scores, int32_t* cand_pos, int64_t batch,
                                        int64_t max_pages, int64_t num_pages, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  int rc = check_common(q, k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  if (rc != DSA_OK || batch == 0) return rc;
  if (!cand_scores || !cand_pos || key_begin < 0 || key_end < key_begin) return DSA_ERR_INVALID_ARG;
  IndexerParams p = base_params(k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  p.cand_scores = cand_scores;
  p.cand_pos = cand_pos;
  p.key_begin = key_begin;
  p.key_end = key_end;
  int64_t span = (key_end - key_begin + 2 * kPage - 1) / kPage;
  if (span > max_pages) span = max_pages;
  return launch_indexer<kModePartial>(q, k_cache, p, span, static_cast<cudaStream_t>(stream));
}

extern "C" int dsa_topk_indexer_merge(const float* cand_scores, const int32_t* cand_pos, int64_t nparts,
                                      const int32_t* seq_lens, const int32_t* block_table, int32_t* topk_indices,
                                      int64_t batch, int64_t max_pages, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  if (batch < 0 || nparts < 1 || max_pages < 1 || max_pages > INT32_MAX / kPage || batch > INT32_MAX)
    return DSA_ERR_INVALID_ARG;
  if (batch == 0) return DSA_OK;
  if (!cand_scores || !cand_pos || !seq_lens || !block_table || !topk_indices) return DSA_ERR_INVALID_ARG;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  merge_kernel<<<static_cast<unsigned>(batch), kMergeThreads, kMergeSmem, static_cast<cudaStream_t>(stream)>>>(
      cand_scores, cand_pos, static_cast<int>(nparts), block_table, topk_indices, static_cast<int>(batch),
      static_cast<int>(max_pages));
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  t_last_launches = 1;
  return DSA_OK;
}

// ---------------------------------------------------------------------------
// No-allocation variant of the indexer launch. Its only scratch, the
// longest-first row order, is this fixed array (4 bytes x
// DSA_NOALLOC_MAX_BATCH rows) instead of the per-stream workspace. Host code
// must not pass the array's name to a kernel (in host code it is a host-side
// stand-in, not a device address): the device address is looked up once per
// device with cudaGetSymbolAddress, with that device current.
static __device__ __align__(256) int32_t g_noalloc_order[DSA_NOALLOC_MAX_BATCH];

namespace {
int32_t* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mutex;

int noalloc_scratch(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_order) != cudaSuccess || !ptr) return DSA_ERR_CUDA;
    g_noalloc_addr[dev] = static_cast<int32_t*>(ptr);
  }
  *out = g_noalloc_addr[dev];
  return DSA_OK;
}
}  // namespace

extern "C" int dsa_topk_indexer_launch_noalloc(const void* q, const void* k_cache, const float* weights,
                                               const int32_t* seq_lens, const int32_t* block_table,
                                               int32_t* topk_indices, int64_t batch, int64_t max_pages,
                                               int64_t num_pages, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  int rc = check_common(q, k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  if (rc != DSA_OK || batch == 0) return rc;
  if (!topk_indices) return DSA_ERR_INVALID_ARG;
  if (batch > DSA_NOALLOC_MAX_BATCH) return DSA_ERR_TOO_LARGE;
  int num_sms = 0;
  rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  int32_t* order = nullptr;
  rc = noalloc_scratch(&order);
  if (rc != DSA_OK) return rc;
  CUtensorMap tk, tq;
  rc = make_maps(q, k_cache, batch, num_pages, &tk, &tq);
  if (rc != DSA_OK) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  IndexerParams p = base_params(k_cache, weights, seq_lens, block_table, batch, max_pages, num_pages);
  p.out = topk_indices;
  const int G = choose_cluster(batch, max_pages, num_sms);
  int launches = 1;
  if (batch > 1 && static_cast<int64_t>(G) * batch > 2 * num_sms) {
    if (batch <= kInKernelOrderMax) {
      p.order_base = 0;  // rows ranked inside the kernel: no scratch at all
    } else {
      // The plan kernel writes all `batch` entries the indexer reads.
      lpt_order_kernel<<<1, kPlanThreads, 0, st>>>(seq_lens, static_cast<int>(batch), static_cast<int>(max_pages),
                                                   order, nullptr);
      if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
      p.order = order;
      launches = 2;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(G * batch), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(G);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KernelTimer timer(st);
  if (cudaLaunchKernelEx(&cfg, indexer_kernel<kModeTopK>, tk, tq, p) != cudaSuccess) return DSA_ERR_CUDA;
  timer.stop();
  t_last_launches = launches;
  t_last_path = "noalloc";
  return DSA_OK;
}

extern "C" int dsa_topk_indexer_set_test_fault(int skip_tile, int64_t wait_ns) {
  if (skip_tile < -1 || wait_ns < 0 || wait_ns > static_cast<int64_t>(ptx::kWaitTimeoutNs) ||
      (wait_ns > 0 && wait_ns < 100000))
    return DSA_ERR_INVALID_ARG;
  g_test_skip_tile.store(skip_tile);
  g_test_wait_ns.store(wait_ns == 0 ? ptx::kWaitTimeoutNs : static_cast<uint64_t>(wait_ns));
  return DSA_OK;
}

extern "C" int dsa_topk_indexer_set_device(int device) {
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur == device) return DSA_OK;
  return cudaSetDevice(device) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

extern "C" int dsa_topk_indexer_status(int device, uint32_t* status, int clear) {
  if (!status) return DSA_ERR_INVALID_ARG;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return DSA_ERR_CUDA;
  if (device != prev && cudaSetDevice(device) != cudaSuccess) return DSA_ERR_CUDA;
  unsigned int v = 0;
  int rc = DSA_OK;
  if (cudaMemcpyFromSymbol(&v, g_dsa_status, sizeof(v)) != cudaSuccess) rc = DSA_ERR_CUDA;
  if (rc == DSA_OK && clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_dsa_status, &zero, sizeof(zero)) != cudaSuccess) rc = DSA_ERR_CUDA;
  }
  *status = v;
  if (device != prev) cudaSetDevice(prev);
  return rc;
}

extern "C" const char* dsa_topk_indexer_error_string(int code) {
  switch (code) {
    case DSA_OK:
      return "ok";
    case DSA_ERR_INVALID_ARG:
      return "invalid argument (null pointer, negative or oversized dimension)";
    case DSA_ERR_MISALIGNED:
      return "q and k_cache must be 16-byte aligned";
    case DSA_ERR_CUDA:
      return "CUDA runtime or driver call failed";
    case DSA_ERR_NO_DEVICE:
      return "current device is not an sm_100 (B200) GPU";
    case DSA_ERR_TOO_LARGE:
      return "batch exceeds the no-allocation entry point's fixed scratch (DSA_NOALLOC_MAX_BATCH = 65536 rows)";
    default:
      return "unknown error";
  }
}

extern "C" int dsa_topk_indexer_last_launch_count(void) { return t_last_launches; }

extern "C" const char* dsa_topk_indexer_last_path(void) { return t_last_path; }

extern "C" int dsa_topk_indexer_set_timing(int on) {
  g_timing.store(on ? 1 : 0);
  return DSA_OK;
}

extern "C" int dsa_topk_indexer_kernel_ms(float* ms) {
  if (!ms || !t_timed) return DSA_ERR_INVALID_ARG;
  if (cudaEventSynchronize(t_ev_end) != cudaSuccess) return DSA_ERR_CUDA;
  return cudaEventElapsedTime(ms, t_ev_begin, t_ev_end) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

extern "C" int dsa_index_cache_write(const void* k, int k_dtype, const int64_t* slots, void* k_cache,
                                     int64_t num_tokens, int64_t num_pages, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  if (num_tokens < 0 || num_pages < 1) return DSA_ERR_INVALID_ARG;
  if (num_tokens == 0) return DSA_OK;
  if (!k || !slots || !k_cache || (k_dtype != DSA_DTYPE_BF16 && k_dtype != DSA_DTYPE_F32))
    return DSA_ERR_INVALID_ARG;
  if (!aligned16(k) || !aligned16(k_cache) || !aligned16(slots)) return DSA_ERR_MISALIGNED;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  const bool bf16 = k_dtype == DSA_DTYPE_BF16;
  const int64_t per_chunk = bf16 ? WriterGeom<true>::kTokens : WriterGeom<false>::kTokens;
  int64_t blocks = (num_tokens + per_chunk - 1) / per_chunk;
  const int64_t cap = static_cast<int64_t>(num_sms) * 4;  // four 50 KB rings per SM
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf16)
    cache_write_kernel<true><<<static_cast<unsigned>(blocks), 32 * kWriterWarps, WriterGeom<true>::kSmem, st>>>(
        k, slots, static_cast<uint8_t*>(k_cache), num_tokens, num_pages);
  else
    cache_write_kernel<false><<<static_cast<unsigned>(blocks), 32 * kWriterWarps, WriterGeom<false>::kSmem, st>>>(
        k, slots, static_cast<uint8_t*>(k_cache), num_tokens, num_pages);
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  t_last_launches = 1;
  return DSA_OK;
}

// ------------------------------------------------- key-axis peer exchange
extern "C" int dsa_peer_region_bytes(int64_t batch, int64_t* bytes) {
  if (batch < 1 || batch > INT32_MAX || !bytes) return DSA_ERR_INVALID_ARG;
  *bytes = PeerLayout{batch * kTopK * 4}.total();
  return DSA_OK;
}

extern "C" int dsa_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes < 1 || !ptr || !ipc_handle) return DSA_ERR_INVALID_ARG;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) return DSA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return DSA_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return DSA_OK;
}

extern "C" int dsa_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return DSA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

extern "C" int dsa_peer_close(void* ptr) {
  if (!ptr) return DSA_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

extern "C" int dsa_peer_free(void* ptr) {
  if (!ptr) return DSA_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

extern "C" int dsa_peer_merge(const uint64_t* bases, int32_t nranks, int32_t rank, uint32_t epoch, int64_t batch,
                              const int32_t* block_table, int64_t max_pages, int32_t phases, int64_t wait_ns,
                              void* stream) {
  t_last_launches = 0;
  t_timed = false;
  if (!bases || !block_table || nranks < 1 || nranks > kPeerMaxRanks || rank < 0 || rank >= nranks ||
      batch < 1 || batch > INT32_MAX || max_pages < 1 || max_pages > INT32_MAX / kPage || (phases & ~15) != 0 ||
      wait_ns < 0)
    return DSA_ERR_INVALID_ARG;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  PeerParams p{};
  p.bases = bases;
  p.nranks = nranks;
  p.rank = rank;
  p.epoch = epoch;
  p.lay = PeerLayout{batch * kTopK * 4};
  p.batch = static_cast<int32_t>(batch);
  p.max_pages = static_cast<int32_t>(max_pages);
  const int64_t r0 = batch * rank / nranks, r1 = batch * (rank + 1) / nranks;
  p.row_begin = static_cast<int32_t>(r0);
  p.block_table = block_table;
  p.wait_ns = wait_ns > 0 ? static_cast<uint64_t>(wait_ns) : ptx::kWaitTimeoutNs;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int launches = 0;
  if (phases & 1) {
    peer_signal_kernel<<<1, 64, 0, st>>>(p, 0);
    ++launches;
  }
  if ((phases & 2) && r1 > r0) {
    peer_merge_kernel<<<static_cast<unsigned>(r1 - r0), kMergeThreads, kMergeSmem, st>>>(p);
    ++launches;
  }
  if (phases & 4) {
    peer_signal_kernel<<<1, 64, 0, st>>>(p, 1);
    ++launches;
  }
  if (phases & 8) {
    peer_wait_kernel<<<1, 64, 0, st>>>(p, 1);
    ++launches;
  }
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  t_last_launches = launches;
  return DSA_OK;
}

extern "C" int dsa_decode_queue_apply(const int32_t* record, int64_t record_words, int32_t* req_len,
                                      int32_t* req_block_table, int64_t num_slots, int64_t max_pages,
                                      int32_t* seq_lens, int32_t* block_table, int64_t capacity, void* stream) {
  t_last_launches = 0;
  t_timed = false;
  if (!record || !req_len || !req_block_table || !seq_lens || !block_table) return DSA_ERR_INVALID_ARG;
  if (record_words < DSA_QUEUE_HEADER_WORDS || num_slots < 1 || num_slots > INT32_MAX || max_pages < 1 ||
      max_pages > INT32_MAX / 64 || capacity < 1 || capacity > INT32_MAX)
    return DSA_ERR_INVALID_ARG;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int32_t mp = static_cast<int32_t>(max_pages);
  decode_queue_apply_kernel<<<1, kQueueThreads, 0, st>>>(record, record_words, req_len, req_block_table, num_slots,
                                                        mp, capacity);
  decode_queue_gather_kernel<<<static_cast<unsigned>(capacity), kQueueThreads, 0, st>>>(
      record, record_words, req_len, req_block_table, num_slots, mp, seq_lens, block_table, capacity);
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  t_last_launches = 2;
  return DSA_OK;
}

// ------------------------------------------------------- sparse attention
namespace dsa {
namespace {

// Split-combine buffers of the sparse attention, one set per (device,
// stream): partial outputs and (max, sum) per split, and one counter per
// token that must be zero between launches (zeroed here when allocated, reset
// by the kernel after each use). Grown outside stream capture only; replaced
// buffers are kept because work queued earlier may still use them.
struct AttnWorkspace {
  void* parts = nullptr;
  size_t part_bytes = 0;
  uint32_t* counters = nullptr;
  int64_t ncounters = 0;
};
std::map<std::pair<int, cudaStream_t>, AttnWorkspace> g_attn_ws;

int attn_workspace(cudaStream_t stream, size_t part_bytes, int64_t ncounters, void** parts, uint32_t** counters) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  AttnWorkspace& ws = g_attn_ws[{dev, stream}];
  if (ws.part_bytes < part_bytes || ws.ncounters < ncounters) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
      return DSA_ERR_CUDA;  // first use of this size must happen outside capture
  }
  if (ws.part_bytes < part_bytes) {
    size_t want = part_bytes < 2 * ws.part_bytes ? 2 * ws.part_bytes : part_bytes;
    void* fresh = nullptr;
    if (cudaMalloc(&fresh, want) != cudaSuccess) return DSA_ERR_CUDA;
    if (ws.parts) g_retired.push_back(ws.parts);
    ws.parts = fresh;
    ws.part_bytes = want;
  }
  if (ws.ncounters < ncounters) {
    int64_t want = ncounters < 2 * ws.ncounters ? 2 * ws.ncounters : ncounters;
    if (want < 1024) want = 1024;
    void* fresh = nullptr;
    if (cudaMalloc(&fresh, static_cast<size_t>(want) * 4) != cudaSuccess) return DSA_ERR_CUDA;
    if (cudaMemsetAsync(fresh, 0, static_cast<size_t>(want) * 4, stream) != cudaSuccess) return DSA_ERR_CUDA;
    if (ws.counters) g_retired.push_back(ws.counters);
    ws.counters = static_cast<uint32_t*>(fresh);
    ws.ncounters = want;
  }
  *parts = ws.parts;
  *counters = ws.counters;
  return DSA_OK;
}

// Splits of each token's index list: the count that minimises
// waves x (tiles per CTA + one tile's worth for the partial's round trip)
// + the combine (one CTA pulls all S partials of 32 KB, about a quarter of a
// tile's time each), one CTA per SM; ties go to fewer splits. Each split
// holds at most kSaMaxChunk entries.
int choose_splits(int64_t tokens, int64_t ntiles, int num_sms) {
  if (ntiles <= 1) return 1;  // an empty or one-tile list is never split
  // DSA_SA_SPLITS=<n> forces n splits when that is a valid split of the list
  // (tuning and tests).
  if (const char* env = std::getenv("DSA_SA_SPLITS")) {
    const int64_t s = std::atoi(env);
    const int64_t min_s = (ntiles * kSaTile + kSaMaxChunk - 1) / kSaMaxChunk;
    if (s >= min_s && s >= 1 && s <= kSaMaxSplits && s <= ntiles) {
      const int64_t per = (ntiles + s - 1) / s;
      if ((ntiles + per - 1) / per == s) return static_cast<int>(s);
    }
  }
  const int64_t min_s = (ntiles * kSaTile + kSaMaxChunk - 1) / kSaMaxChunk;
  int best = static_cast<int>(min_s < 1 ? 1 : min_s);
  double best_cost = -1.0;
  for (int64_t s = best; s <= kSaMaxSplits && s <= (ntiles < 1 ? 1 : ntiles); ++s) {
    const int64_t per = (ntiles + s - 1) / s;
    const int64_t used = (ntiles + per - 1) / per;  // splits that hold a tile
    if (used != s) continue;
    const int64_t waves = (tokens * s + num_sms - 1) / num_sms;
    const double cost = static_cast<double>(waves) * static_cast<double>(per + (s > 1 ? 1 : 0)) +
                        (s > 1 ? static_cast<double>(s) / 4.0 : 0.0);
    if (best_cost < 0.0 || cost < best_cost) {
      best_cost = cost;
      best = static_cast<int>(s);
    }
  }
  return best;
}

}  // namespace
}  // namespace dsa

extern "C" int dsa_sparse_attention_launch(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                           const void* kpe_cache, const int32_t* sparse_indices, float sm_scale,
                                           void* output, float* lse, int64_t num_tokens, int64_t num_indices,
                                           int64_t num_pages, void* stream) {
  using namespace dsa;
  t_last_launches = 0;
  t_timed = false;
  if (num_tokens < 0 || num_indices < 0 || num_pages < 1) return DSA_ERR_INVALID_ARG;
  if (num_tokens == 0) return DSA_OK;
  if (!q_nope || !q_pe || !ckv_cache || !kpe_cache || !output || !lse || (num_indices > 0 && !sparse_indices))
    return DSA_ERR_INVALID_ARG;
  if (num_indices > static_cast<int64_t>(kSaMaxChunk) * kSaMaxSplits) return DSA_ERR_TOO_LARGE;
  if (!aligned16(q_nope) || !aligned16(q_pe) || !aligned16(ckv_cache) || !aligned16(kpe_cache) ||
      (reinterpret_cast<uintptr_t>(output) & 3u) || (reinterpret_cast<uintptr_t>(lse) & 3u) ||
      (reinterpret_cast<uintptr_t>(sparse_indices) & 3u))
    return DSA_ERR_MISALIGNED;
  if (num_tokens * kSaMaxSplits > 0x7FFFFFFFll) return DSA_ERR_TOO_LARGE;
  int num_sms = 0;
  int rc = prepare_device(&num_sms);
  if (rc != DSA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ntiles = (num_indices + kSaTile - 1) / kSaTile;
  const int splits = choose_splits(num_tokens, ntiles, num_sms);
  const int64_t per = splits > 1 ? (ntiles + splits - 1) / splits : ntiles;
  SparseAttnParams prm{};
  prm.q_nope = static_cast<const __nv_bfloat16*>(q_nope);
  prm.q_pe = static_cast<const __nv_bfloat16*>(q_pe);
  prm.ckv = static_cast<const __nv_bfloat16*>(ckv_cache);
  prm.kpe = static_cast<const __nv_bfloat16*>(kpe_cache);
  prm.indices = sparse_indices;
  prm.out = static_cast<__nv_bfloat16*>(output);
  prm.lse = lse;
  prm.num_slots = num_pages * 64;
  prm.num_indices = static_cast<int32_t>(num_indices);
  prm.splits = splits;
  prm.chunk = static_cast<int32_t>((per < 1 ? 1 : per) * kSaTile);
  prm.scale_log2 = static_cast<float>(static_cast<double>(sm_scale) * 1.4426950408889634);
  if (splits > 1) {
    void* parts = nullptr;
    uint32_t* counters = nullptr;
    const size_t part_bytes = static_cast<size_t>(num_tokens) * splits * kSaHeads * (kSaCkv + 2) * sizeof(float);
    rc = attn_workspace(st, part_bytes, num_tokens, &parts, &counters);
    if (rc != DSA_OK) return rc;
    prm.part_o = static_cast<float*>(parts);
    prm.part_ml = prm.part_o + static_cast<size_t>(num_tokens) * splits * kSaHeads * kSaCkv;
    prm.counters = counters;
  }
  KernelTimer timer(st);
  sparse_attention_kernel<<<static_cast<unsigned>(num_tokens * splits), kSaThreads, SaLayout::kBytes, st>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return DSA_ERR_CUDA;
  timer.stop();
  t_last_launches = 1;
  return DSA_OK;
}
