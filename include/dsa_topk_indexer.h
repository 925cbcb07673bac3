/*
 * C ABI of the B200 (sm_100a) DSA lightning-indexer top-K.
 *
 * All pointers are caller-owned, contiguous DEVICE buffers on the current
 * CUDA device; every call is asynchronous on `stream` (a cudaStream_t, NULL
 * for the legacy default stream) and never synchronises it. Return value:
 * DSA_OK or a DSA_ERR_* code.
 *
 * Device memory the library allocates itself (never per call):
 *   - dsa_topk_indexer_launch: a small per-(device, stream) workspace (the
 *     longest-first row order and per-row flags, a few bytes per row) with
 *     cudaMalloc, and a side stream with two events for its two-kernel
 *     launch, on the first call on a stream whose batch needs them; grown
 *     (never shrunk) when a later call needs more. Make the first call on a
 *     stream outside stream capture.
 *   - dsa_sparse_attention_launch: per-(device, stream) split buffers and
 *     counters, allocated the first time a shape needs them (outside capture).
 *   - dsa_topk_indexer_launch_noalloc allocates nothing (see below).
 *   - dsa_peer_alloc allocates the peer-exchange region it is asked for.
 *   The other entry points allocate no device memory.
 *
 * Layouts (the reference operator dsa_topk_indexer_fp8_h64_d128_topk2048_ps64):
 *   q            [B, 64, 128]  FP8 e4m3 bytes
 *   k_cache      [num_pages, 8448] bytes: per page 64 tokens x 128 e4m3
 *                bytes (token-major), then 64 fp32 scales
 *   weights      [B, 64]       fp32
 *   seq_lens     [B]           int32
 *   block_table  [B, max_pages] int32 physical page ids
 *   topk_indices [B, 2048]     int32 physical slots page*64+offset, best
 *                first (ties: smaller logical position first), -1 padded
 */
#ifndef DSA_TOPK_INDEXER_H
#define DSA_TOPK_INDEXER_H

#include <stdint.h>

#if defined(__GNUC__)
#define DSA_API __attribute__((visibility("default")))
#else
#define DSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DSA_OK 0
#define DSA_ERR_INVALID_ARG 1 /* null pointer, negative size, bad stride  */
#define DSA_ERR_MISALIGNED 2  /* q / k_cache not 16-byte aligned          */
#define DSA_ERR_CUDA 3        /* a CUDA runtime/driver call failed        */
#define DSA_ERR_NO_DEVICE 4   /* current device is not sm_100             */
#define DSA_ERR_TOO_LARGE 5   /* batch above DSA_NOALLOC_MAX_BATCH (no-allocation entry point) */

/* Largest batch dsa_topk_indexer_launch_noalloc accepts. */
#define DSA_NOALLOC_MAX_BATCH 65536

/* Bits of the per-device status word the kernels raise (sticky until read
 * with clear != 0). */
#define DSA_STATUS_WAIT_TIMEOUT 0x1u /* a pipeline wait gave up (kernel ended early) */
#define DSA_STATUS_BAD_PAGE 0x2u     /* block_table held an id outside [0, num_pages) */
#define DSA_STATUS_SEQ_CLAMPED 0x4u  /* seq_len > max_pages*64; clamped              */
#define DSA_STATUS_BAD_RECORD 0x8u   /* a decode-queue record held an invalid event or row; skipped */

/*
 * The indexer: scores every visible key of every request and writes the
 * top-2048 physical slots. Replaces the reference host entry
 * `launch_topk_c(q_index_fp8, k_index_cache_fp8, weights, seq_lens,
 * block_table, topk_indices)` (solution/cuda/kernel.cu:818-887), without its
 * N_max <= 8192 limit (kernel.cu:858-859).
 */
DSA_API int dsa_topk_indexer_launch(const void* q, const void* k_cache, const float* weights,
                            const int32_t* seq_lens, const int32_t* block_table,
                            int32_t* topk_indices, int64_t batch, int64_t max_pages,
                            int64_t num_pages, void* stream);

/*
 * Scores only: scores[b, t] = sum_h w[b,h]*relu(scale[t]*q[b,h].k[t]) for
 * t < seq_len[b], -inf for seq_len[b] <= t < score_stride. Same scoring path
 * as the indexer; replaces the reference's fp32 `final_scores` intermediate
 * written by fp8_mma_final_scores_kernel (solution/cuda/kernel.cu:209-452,
 * buffer allocated at :847). Used for tolerance checks.
 */
DSA_API int dsa_topk_indexer_scores(const void* q, const void* k_cache, const float* weights,
                            const int32_t* seq_lens, const int32_t* block_table, float* scores,
                            int64_t score_stride, int64_t batch, int64_t max_pages,
                            int64_t num_pages, void* stream);

/*
 * Key-range partial top-K for key-axis sharding of long sequences: request
 * b only considers logical keys [key_begin, min(key_end, seq_len[b])).
 * Writes its best 2048 candidates as (score, logical position) pairs,
 * best first, padded with (-inf, -1). No counterpart in the reference (it has
 * no multi-GPU path); it is the per-GPU half of the sharded indexer.
 */
DSA_API int dsa_topk_indexer_partial(const void* q, const void* k_cache, const float* weights,
                             const int32_t* seq_lens, const int32_t* block_table,
                             int64_t key_begin, int64_t key_end, float* cand_scores,
                             int32_t* cand_pos, int64_t batch, int64_t max_pages,
                             int64_t num_pages, void* stream);

/*
 * Merges `nparts` candidate lists per request ([nparts, B, 2048] each, as
 * written by dsa_topk_indexer_partial) into the final top-2048 physical
 * slots, with the indexer's order and padding rules. The second half of the
 * sharded indexer; no counterpart in the reference.
 */
DSA_API int dsa_topk_indexer_merge(const float* cand_scores, const int32_t* cand_pos, int64_t nparts,
                           const int32_t* seq_lens, const int32_t* block_table,
                           int32_t* topk_indices, int64_t batch, int64_t max_pages, void* stream);

/*
 * Same operation and arguments as dsa_topk_indexer_launch, for callers that
 * must not allocate device memory: code that runs where cudaMalloc is
 * forbidden or unsafe (inside a custom allocator, a memory-pool callback, a
 * tightly budgeted inference server that pre-reserves all of HBM) or that
 * cannot tolerate the first-call allocation of the launch entry point's
 * per-stream workspace. It has no counterpart in the reference.
 *
 * The scratch it needs (the longest-first row order, 4 bytes per row) lives
 * in a fixed array inside this library, DSA_NOALLOC_MAX_BATCH rows (256 KiB)
 * on every GPU that loads the library, held until the process exits. Larger
 * batches are rejected with DSA_ERR_TOO_LARGE. The first call on a device
 * looks up that array's device address (with the device current), so make
 * that first call before any stream capture. All calls on a device share the
 * array: calls that can overlap on the GPU (different streams, no ordering
 * between them) race on it and must be serialised by the caller. Nothing in
 * the array needs clearing between calls; every call rewrites the entries it
 * reads.
 */
DSA_API int dsa_topk_indexer_launch_noalloc(const void* q, const void* k_cache, const float* weights,
                                            const int32_t* seq_lens, const int32_t* block_table,
                                            int32_t* topk_indices, int64_t batch, int64_t max_pages,
                                            int64_t num_pages, void* stream);

/* Index-K cache writer (the producer of the page format above; the
 * reference only consumes it, solution/cuda/kernel.cu:22-25). Quantises
 * `num_tokens` vectors of 128 values (`k`: bf16 or fp32, [num_tokens, 128],
 * contiguous, 16-byte aligned, finite) to FP8 e4m3 with one fp32 scale per
 * token: scale = max|x| / 448, inv = 448 / max|x| (both 1 when scale is not
 * positive or inv not finite, e.g. an all-zero vector), values x * inv
 * rounded to nearest even and saturated, and
 * writes token t into slot `slots[t]` (int64 array, 16-byte aligned;
 * page * 64 + offset) of `k_cache` ([num_pages, 8448] bytes): bytes
 * [offset*128, +128) of the page and its fp32 scale at byte 8192 + offset*4.
 * Negative slots are skipped; slots past num_pages*64 are skipped and flag
 * DSA_STATUS_BAD_PAGE. Tokens sharing a slot: one of them wins.
 * Asynchronous on `stream`. */
#define DSA_DTYPE_BF16 0
#define DSA_DTYPE_F32 1
DSA_API int dsa_index_cache_write(const void* k, int k_dtype, const int64_t* slots, void* k_cache,
                                  int64_t num_tokens, int64_t num_pages, void* stream);

/* Sparse MLA attention over the selected slots: the consumer of
 * topk_indices, operator dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64
 * (named by the reference at FAQ.md:83 and EVALUATION.md:54-57,87; it
 * carries no implementation). Per token t and head h (16 heads), over the
 * entries s of sparse_indices[t] that are >= 0:
 *   logit_s  = (q_nope[t,h] . ckv[s] + q_pe[t,h] . kpe[s]) * sm_scale
 *   output[t,h] = sum_s softmax(logit)_s * ckv[s]       bf16 [T, 16, 512]
 *   lse[t,h]    = log2(sum_s exp(logit_s))               fp32 [T, 16]
 * Inputs (bf16, contiguous, 16-byte aligned): q_nope [T, 16, 512], q_pe
 * [T, 16, 64], ckv_cache [num_pages, 64, 512], kpe_cache [num_pages, 64, 64];
 * sparse_indices [T, num_indices] int32 slots page*64+offset (-1 = none;
 * entries past num_pages*64 are ignored and flag DSA_STATUS_BAD_PAGE). A
 * token with no valid entry gets output 0 and lse -inf. num_indices is at
 * most 65536 (the operator uses 2048). Long lists are split across CTAs and
 * combined on the device; the split buffers are library-owned and allocated
 * (outside stream capture) the first time a shape needs them. Asynchronous
 * on `stream`. */
DSA_API int dsa_sparse_attention_launch(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                        const void* kpe_cache, const int32_t* sparse_indices, float sm_scale,
                                        void* output, float* lse, int64_t num_tokens, int64_t num_indices,
                                        int64_t num_pages, void* stream);

/* Key-axis sharding over NVLink peer memory, without a collective library
 * (the exchange and merge that dsa_topk_indexer_partial / _merge and NCCL
 * otherwise do). Each rank allocates one region of dsa_peer_region_bytes(B)
 * bytes with dsa_peer_alloc (cudaMalloc, zeroed; `ipc_handle` receives its
 * 64-byte CUDA IPC handle), hands the handle to every other rank, and opens
 * theirs with dsa_peer_open. Region layout, L = B*2048*4 bytes:
 *   [0, L) cand_scores [B,2048] fp32 | [L, 2L) cand_pos [B,2048] int32 |
 *   [2L, 3L) out [B,2048] int32 | then ready flags [64] and done flags [64]
 *   (uint32 step counters, one per rank).
 * Per step each rank writes its key range's best-first lists into its own
 * cand_scores / cand_pos (dsa_topk_indexer_partial with those pointers), then
 * calls dsa_peer_merge with `bases` = a DEVICE array [nranks] of every rank's
 * region address as this rank maps it (its own allocation, the peers' opened
 * addresses) and the same `epoch` on every rank, increasing by one per step
 * (first step 1). Phases (bit mask, 15 = all, in this order on `stream`):
 *   1 signal ready: ready[rank] = epoch in every region;
 *   2 merge: CTA per row of rows [B*rank/nranks, B*(rank+1)/nranks): wait
 *     until ready[0..nranks) = epoch in this rank's region, merge the lists of
 *     every rank (peer loads), translate through block_table [B, max_pages]
 *     and store the row into every rank's out (peer stores);
 *   4 signal done: done[rank] = epoch in every region;
 *   8 wait done: until done[0..nranks) = epoch in this rank's region; then
 *     out holds all B rows, and no peer reads this rank's lists any more.
 * Waits give up after wait_ns (0: 2 s) and raise DSA_STATUS_WAIT_TIMEOUT
 * (the CTA that gave up writes nothing). At most 64 ranks. Plain peer loads
 * and stores, no multicast. Results equal dsa_topk_indexer_merge over the
 * same lists bit for bit. The reference has no multi-GPU path; this is the
 * exchange its north star names (candidate lists gathered over NVLink, then
 * a GPU merge), fused into one kernel. dsa_peer_alloc allocates (its purpose);
 * call it outside stream capture. */
DSA_API int dsa_peer_region_bytes(int64_t batch, int64_t* bytes);
DSA_API int dsa_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
DSA_API int dsa_peer_open(const void* ipc_handle, void** ptr);
DSA_API int dsa_peer_close(void* ptr);
DSA_API int dsa_peer_free(void* ptr);
DSA_API int dsa_peer_merge(const uint64_t* bases, int32_t nranks, int32_t rank, uint32_t epoch, int64_t batch,
                           const int32_t* block_table, int64_t max_pages, int32_t phases, int64_t wait_ns,
                           void* stream);

/* Device work queue across decode steps. The request table stays in device
 * memory between steps: req_len [num_slots] int32 (-1 = slot not in use)
 * and req_block_table [num_slots, max_pages] int32 page ids. A step ships
 * one record (int32 words, device memory, `record_words` capacity):
 *   [0] words used   [1] events   [2] batch B   [3] advance (>= 0)
 *   [4] offset of the batch list  [5..7] 0
 *   events from word DSA_QUEUE_HEADER_WORDS, 4 words each, in order:
 *     {DSA_QUEUE_ADMIT, slot, length, n}  followed by n page ids, padded
 *                                          with zeros to a multiple of 4 words
 *     {DSA_QUEUE_APPEND_PAGE, slot, page_index, page_id}
 *     {DSA_QUEUE_SET_LEN, slot, length, 0}
 *     {DSA_QUEUE_RETIRE, slot, 0, 0}
 *   the batch list: B distinct slots, at the offset in word [4].
 * The call applies the events, then for every batch row b adds `advance` to
 * req_len[slot_b] and writes seq_lens[b] (the new length) and the row's
 * visible entries block_table[b, 0 .. ceil(len/64)) (width max_pages);
 * rows B .. capacity-1 get seq_lens 0, so the indexer over `capacity` rows
 * returns -1 for them. Events or rows naming a slot outside [0, num_slots),
 * a slot not in use, or a page index outside [0, max_pages) are skipped and
 * raise DSA_STATUS_BAD_RECORD; a record whose header or event list cannot
 * be read is dropped whole. A slot listed twice in one batch is advanced an
 * unspecified number of times. Two launches (one CTA, then `capacity` CTAs),
 * asynchronous on `stream`, no allocation, capturable into a CUDA graph
 * together with the indexer call that consumes seq_lens / block_table. No
 * counterpart in the reference, whose entry point takes a host-built batch
 * per call (solution/cuda/kernel.cu:818-887). */
#define DSA_QUEUE_HEADER_WORDS 8
#define DSA_QUEUE_ADMIT 1
#define DSA_QUEUE_APPEND_PAGE 2
#define DSA_QUEUE_SET_LEN 3
#define DSA_QUEUE_RETIRE 4
DSA_API int dsa_decode_queue_apply(const int32_t* record, int64_t record_words, int32_t* req_len,
                                   int32_t* req_block_table, int64_t num_slots, int64_t max_pages,
                                   int32_t* seq_lens, int32_t* block_table, int64_t capacity, void* stream);

/* Test hook for the bounded-wait abort path (off by default). Every
 * pipeline wait of the indexer kernels gives up after a time limit (2 s),
 * raises DSA_STATUS_WAIT_TIMEOUT and ends the kernel early without a fault;
 * this hook lets a test make that happen. While skip_tile >= 0, every CTA of
 * later indexer calls (all entry points, all threads) never issues the loads
 * of its local tile `skip_tile`, so the waits for it run out; wait_ns sets
 * the limit of every wait (100 us .. 2 s; 0 restores the 2 s default).
 * Outputs of such calls are meaningless. Call with (-1, 0) to turn it off.
 * No counterpart in the reference, whose waits spin without a bound
 * (solution/cuda/kernel.cu:107-120). */
DSA_API int dsa_topk_indexer_set_test_fault(int skip_tile, int64_t wait_ns);

/* Makes `device` the current CUDA device of the calling host thread for this
 * library (the entry points above run on the current device). Callers that
 * link their own CUDA runtime (PyTorch, TVM-FFI hosts) call it with the
 * tensors' device before each launch. No counterpart in the reference, whose
 * host code does the same with at::cuda::CUDAGuard (kernel.cu:826). */
DSA_API int dsa_topk_indexer_set_device(int device);

/* Reads (and optionally clears) the status word of device `device`.
 * Synchronous with respect to the device. */
DSA_API int dsa_topk_indexer_status(int device, uint32_t* status, int clear);

/* Human-readable text for a DSA_* return code. */
DSA_API const char* dsa_topk_indexer_error_string(int code);

/* Number of kernel launches the last successful call on this host thread made. */
DSA_API int dsa_topk_indexer_last_launch_count(void);

/* Schedule the last successful top-K call on this host thread took:
 * "cluster" (one cluster kernel, optionally after the longest-first plan),
 * "cluster-split" (two concurrent cluster kernels, the longest rows with more
 * CTAs), "cluster-tail" (two cluster kernels, the rows of the last partial
 * wave with more CTAs), "prefill+cluster" (the
 * shared-sequence kernel, then the cluster kernel for the rows it left) or
 * "noalloc" (the no-allocation entry point's cluster kernel). */
DSA_API const char* dsa_topk_indexer_last_path(void);

/* Per-kernel timing for profiling, off by default. While on, every call
 * records CUDA events on its stream around its dominant kernel or kernels
 * and dsa_topk_indexer_kernel_ms waits for the last call on this host thread
 * and returns that kernel's device time in milliseconds. The events keep the
 * bracketed launch from overlapping its neighbours, so timed calls are not
 * the fastest; calls made while their stream is being captured are not
 * timed (kernel_ms then returns DSA_ERR_INVALID_ARG). */
DSA_API int dsa_topk_indexer_set_timing(int on);
DSA_API int dsa_topk_indexer_kernel_ms(float* ms);

#ifdef __cplusplus
}
#endif
#endif /* DSA_TOPK_INDEXER_H */
