// Sparse MLA attention over the slots the indexer selected: the consumer of
// `topk_indices` (operator dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64,
// named by the reference's FAQ.md:83 and EVALUATION.md:54-57,87; the
// reference repository carries no code for it).
//
// Per token t and head h (16 heads), over the valid entries j of the token's
// index list (slot = page * 64 + offset; -1 = none):
//   logit_j = (q_nope[t,h] . ckv[slot_j] + q_pe[t,h] . kpe[slot_j]) * sm_scale
//   out[t,h] = sum_j softmax(logit)_j * ckv[slot_j]          (bf16, 512 values)
//   lse[t,h] = log2(sum_j exp(logit_j))                        (base 2)
// A token without valid entries gets out = 0 and lse = -inf.
//
// Data: q_nope [T,16,512], q_pe [T,16,64], ckv [slots,512], kpe [slots,64]
// (bf16, the caches are the page pools [pages,64,512] / [pages,64,64]).
// Per key 1152 bytes are gathered and 34,816 FLOPs spent (16 heads x
// 2 x (576 + 512)): about 30 FLOP/byte, far below the tensor ridge, so the
// kernel is bound by the gather's HBM bandwidth.
//
// Schedule: one CTA (8 warps) per (token, split of the index list), one CTA
// per SM (the three-stage ring takes most of shared memory). Rows of 64
// selected keys are gathered with cp.async into a 3-stage ring (16-byte
// chunks XOR-swizzled by row so ldmatrix is conflict-free), two tiles in
// flight while the third is computed. The 16 heads are exactly the M of the
// m16n8k16 bf16 MMA, so both products run on register fragments:
//   S = Q K^T: warp w takes keys 8w..8w+7 of the tile, Q's fragments stay in
//              registers for the whole kernel;
//   O += P V:  warp w owns value columns 64w..64w+63; P (bf16) goes through a
//              2 KB shared block laid out as ready A fragments.
// Softmax is online in base 2 (running max and sum per head, identical in
// every warp). Splits of one token are combined by the last CTA of the
// token to finish (a counter per token, no waiting), which also resets the
// counter for the next launch.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "indexer_kernel.cuh"

namespace dsa {

constexpr int kSaHeads = 16;
constexpr int kSaCkv = 512;
constexpr int kSaKpe = 64;
constexpr int kSaRowBytes = (kSaCkv + kSaKpe) * 2;  // 1152 gathered bytes per key
constexpr int kSaRowChunks = kSaRowBytes / 16;      // 72
constexpr int kSaTile = 64;                         // keys per tile
constexpr int kSaStages = 3;
constexpr int kSaWarps = 8;
constexpr int kSaThreads = 32 * kSaWarps;
constexpr int kSaMaxChunk = 2048;  // index entries one CTA handles at most
constexpr int kSaMaxSplits = 32;
constexpr int kSaCombineParts = 4;  // partials per round of the split combine (128 KB)
constexpr float kSaSlack = 8.f;    // base-2 headroom of the lazy softmax maximum

struct SaLayout {
  static constexpr int kStage = kSaTile * kSaRowBytes;  // 73,728
  static constexpr int kOffQ = 2 * kStage;              // Q staged in stage 2 before its first tile
  static constexpr int kOffP = kSaStages * kStage;      // 4 k-blocks x 32 lanes x 16 B
  static constexpr int kOffRed = kOffP + 4 * 32 * 16;   // 8 warps x 16 heads fp32
  static constexpr int kOffIdx = kOffRed + kSaWarps * kSaHeads * 4;
  static constexpr int kOffMisc = kOffIdx + kSaMaxChunk * 4;
  static constexpr int kBytes = kOffMisc + 64;
};
static_assert(SaLayout::kBytes <= 232448, "sparse attention shared memory above the per-CTA limit");
static_assert(kSaHeads * kSaRowBytes <= SaLayout::kStage, "Q must fit in one stage");
static_assert(kSaThreads / 8 * 2 == kSaTile, "the gather runs eight threads per key in two passes over a tile");
static_assert(kSaRowChunks == 9 * 8, "a key's row is 8 x 128 bytes of ckv and 128 bytes of kpe");
static_assert(kSaMaxSplits * kSaHeads * 12 <= SaLayout::kStage, "combine weights and partial (max, sum) live in stage 0");
static_assert(kSaCombineParts * kSaHeads * kSaCkv * 4 <= 2 * SaLayout::kStage, "a combine round fits in stages 1-2");

struct SparseAttnParams {
  const __nv_bfloat16* q_nope;  // [T, 16, 512]
  const __nv_bfloat16* q_pe;    // [T, 16, 64]
  const __nv_bfloat16* ckv;     // [num_slots, 512]
  const __nv_bfloat16* kpe;     // [num_slots, 64]
  const int32_t* indices;       // [T, num_indices]
  __nv_bfloat16* out;           // [T, 16, 512]
  float* lse;                   // [T, 16]
  float* part_o;                // [T * splits, 16, 512]   (splits > 1)
  float* part_ml;               // [T * splits, 16, 2]     (splits > 1)
  uint32_t* counters;           // [T], zero between launches (splits > 1)
  int64_t num_slots;
  int32_t num_indices;
  int32_t splits;
  int32_t chunk;                // index entries per split, a multiple of kSaTile
  float scale_log2;             // sm_scale * log2(e)
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(kSaThreads, 1) sparse_attention_kernel(const SparseAttnParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sbase = ptx::smem_addr(sm);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int64_t t = blockIdx.x / p.splits;
  const int split = static_cast<int>(blockIdx.x - t * p.splits);
  const int kbeg = split * p.chunk;
  const int nkeys = max(min(p.chunk, p.num_indices - kbeg), 0);
  int32_t* sidx = reinterpret_cast<int32_t*>(sm + SaLayout::kOffIdx);
  float* red = reinterpret_cast<float*>(sm + SaLayout::kOffRed);
  int* misc = reinterpret_cast<int*>(sm + SaLayout::kOffMisc);

  // Stage this split's index entries (invalid or out-of-range ones become
  // -1; the tail of the last tile is padded with -1) and find the last
  // valid one, which ends the tile loop.
  if (tid == 0) misc[0] = -1;
  __syncthreads();
  {
    const int32_t* irow = p.indices + t * p.num_indices + kbeg;
    const int padded = (nkeys + kSaTile - 1) / kSaTile * kSaTile;
    int last = -1;
    for (int i = tid; i < padded; i += kSaThreads) {
      int32_t v = -1;
      if (i < nkeys) {
        v = irow[i];
        if (v >= p.num_slots) {
          atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);
          v = -1;
        }
        if (v < 0) v = -1;
      }
      sidx[i] = v;
      if (v >= 0) last = i;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) last = max(last, __shfl_xor_sync(0xFFFFFFFFu, last, off));
    if (lane == 0 && last >= 0) atomicMax(&misc[0], last);
  }
  __syncthreads();
  const int ntiles = (misc[0] + kSaTile) / kSaTile;

  const uint8_t* ckv_b = reinterpret_cast<const uint8_t*>(p.ckv);
  const uint8_t* kpe_b = reinterpret_cast<const uint8_t*>(p.kpe);
  // Gathers tile j (keys 64j..64j+63 of this split) into `stage`: eight
  // threads per key, 32 keys per pass, two passes. Thread l8 of a key copies
  // the 16-byte chunks c = 8m + l8 (m < 8) of its 1 KB ckv row and chunk
  // 64 + l8 of its kpe row; chunk c of row r lands at position c ^ (r & 7),
  // i.e. at byte 128 (c / 8) + 16 (l8 ^ (r & 7)) of the row. Invalid keys
  // (-1) read nothing and zero-fill their row.
  auto issue_tile = [&](int j, int stage) {
    const int l8 = tid & 7;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const int r = pass * 32 + (tid >> 3);
      const int32_t idx = sidx[j * kSaTile + r];
      const uint32_t nb = idx >= 0 ? 16u : 0u;
      const int64_t row = idx >= 0 ? idx : 0;
      const uint32_t dst = sbase + stage * SaLayout::kStage + r * kSaRowBytes + ((l8 ^ (r & 7)) << 4);
      const uint8_t* src = ckv_b + row * (kSaCkv * 2) + l8 * 16;
#pragma unroll
      for (int m = 0; m < 8; ++m) ptx::cp_async16(dst + m * 128, src + m * 128, nb);
      ptx::cp_async16(dst + 8 * 128, kpe_b + row * (kSaKpe * 2) + l8 * 16, nb);
    }
  };

  // Group 0: Q (into stage 2's space) and tile 0; group 1: tile 1.
  {
    const uint8_t* qn = reinterpret_cast<const uint8_t*>(p.q_nope) + t * kSaHeads * (kSaCkv * 2);
    const uint8_t* qp = reinterpret_cast<const uint8_t*>(p.q_pe) + t * kSaHeads * (kSaKpe * 2);
    for (int q = tid; q < kSaHeads * kSaRowChunks; q += kSaThreads) {
      const int h = q / kSaRowChunks, c = q - h * kSaRowChunks;
      const uint8_t* src = c < 64 ? qn + h * (kSaCkv * 2) + c * 16 : qp + h * (kSaKpe * 2) + (c - 64) * 16;
      ptx::cp_async16(sbase + SaLayout::kOffQ + h * kSaRowBytes + ((c ^ (h & 7)) << 4), src, 16);
    }
  }
  if (ntiles > 0) issue_tile(0, 0);
  ptx::cp_async_commit();
  if (ntiles > 1) issue_tile(1, 1);
  ptx::cp_async_commit();
  ptx::cp_async_wait_group<1>();
  __syncthreads();

  // Q as A fragments of the 36 k-steps (576 = 36 x 16), kept in registers.
  uint32_t qf[36][4];
#pragma unroll
  for (int ks = 0; ks < 36; ++ks) {
    const int row = lane & 15, c = 2 * ks + (lane >> 4);
    ptx::ldmatrix_x4(qf[ks], sbase + SaLayout::kOffQ + row * kSaRowBytes + ((c ^ (row & 7)) << 4));
  }

  float o[8][4];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;  // running max (base-2 logits) of heads g and g+8
  float l0 = 0.f, l1 = 0.f;              // this thread's share of the running sums
  uint4* pfrag = reinterpret_cast<uint4*>(sm + SaLayout::kOffP);

#pragma unroll 1
  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kSaStages;
    ptx::cp_async_wait_group<1>();  // this thread's copies of tile i are done
    __syncthreads();                // ... everyone's; and tile i-1 is no longer read
    if (i + 2 < ntiles) issue_tile(i + 2, (i + 2) % kSaStages);
    ptx::cp_async_commit();
    const uint32_t stage = sbase + st * SaLayout::kStage;

    // S[16 heads x 8 keys] for keys 8w..8w+7; four accumulators cut the
    // dependent MMA chain to nine.
    float sacc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a) sacc[a][0] = sacc[a][1] = sacc[a][2] = sacc[a][3] = 0.f;
    {
      const uint32_t krow = stage + (8 * warp + (lane & 7)) * kSaRowBytes;
#pragma unroll
      for (int kk = 0; kk < 18; ++kk) {
        uint32_t b[4];
        const int c = 4 * kk + (lane >> 3);
        ptx::ldmatrix_x4(b, krow + ((c ^ (lane & 7)) << 4));
        ptx::mma_bf16_16816(sacc[(2 * kk) & 3], qf[2 * kk], b[0], b[1]);
        ptx::mma_bf16_16816(sacc[(2 * kk + 1) & 3], qf[2 * kk + 1], b[2], b[3]);
      }
    }
    const int key = i * kSaTile + 8 * warp + 2 * tig;
    const bool v0 = sidx[key] >= 0, v1 = sidx[key + 1] >= 0;
    float s[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] = ((sacc[0][e] + sacc[1][e]) + (sacc[2][e] + sacc[3][e])) * p.scale_log2;
    if (!v0) s[0] = s[2] = -INFINITY;
    if (!v1) s[1] = s[3] = -INFINITY;
    float x0 = fmaxf(s[0], s[1]), x1 = fmaxf(s[2], s[3]);
    x0 = fmaxf(x0, __shfl_xor_sync(0xFFFFFFFFu, x0, 1));
    x1 = fmaxf(x1, __shfl_xor_sync(0xFFFFFFFFu, x1, 1));
    x0 = fmaxf(x0, __shfl_xor_sync(0xFFFFFFFFu, x0, 2));
    x1 = fmaxf(x1, __shfl_xor_sync(0xFFFFFFFFu, x1, 2));
    if (tig == 0) {  // head-major: red[h * 8 + w]
      red[g * kSaWarps + warp] = x0;
      red[(g + 8) * kSaWarps + warp] = x1;
    }
    // Lazy reference maximum (base 2, per head, identical in every warp): it
    // only moves when a tile's maximum exceeds it by more than kSaSlack, so
    // p = 2^(s - m) stays <= 2^kSaSlack and most tiles need neither the
    // rescale of O and l nor a second barrier. P is first computed with the
    // current reference; if any head moves, every warp (all read the same
    // maxima) recomputes and rewrites it behind one more barrier.
    const float mu0 = m0 == -INFINITY ? 0.f : m0, mu1 = m1 == -INFINITY ? 0.f : m1;
    float p0 = exp2f(s[0] - mu0), p1 = exp2f(s[1] - mu0);
    float p2 = exp2f(s[2] - mu1), p3 = exp2f(s[3] - mu1);
    // P fragment of k-block w/2: even warps hold its keys 0..7 (a0, a1),
    // odd warps its keys 8..15 (a2, a3).
    uint2* pslot = reinterpret_cast<uint2*>(pfrag + (warp >> 1) * 32 + lane) + (warp & 1);
    *pslot = make_uint2(pack_bf16x2(p0, p1), pack_bf16x2(p2, p3));
    __syncthreads();
    float tm0, tm1;
    {
      const float4* r0 = reinterpret_cast<const float4*>(red + g * kSaWarps);
      const float4* r1 = reinterpret_cast<const float4*>(red + (g + 8) * kSaWarps);
      const float4 u0 = r0[0], u1 = r0[1], w0 = r1[0], w1 = r1[1];
      tm0 = fmaxf(fmaxf(fmaxf(u0.x, u0.y), fmaxf(u0.z, u0.w)), fmaxf(fmaxf(u1.x, u1.y), fmaxf(u1.z, u1.w)));
      tm1 = fmaxf(fmaxf(fmaxf(w0.x, w0.y), fmaxf(w0.z, w0.w)), fmaxf(fmaxf(w1.x, w1.y), fmaxf(w1.z, w1.w)));
    }
    const bool up0 = tm0 > m0 + kSaSlack, up1 = tm1 > m1 + kSaSlack;
    if (__any_sync(0xFFFFFFFFu, up0 || up1)) {  // uniform across the CTA
      const float mn0 = up0 ? tm0 : m0, mn1 = up1 ? tm1 : m1;
      const float nu0 = mn0 == -INFINITY ? 0.f : mn0, nu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float a0 = exp2f(m0 - nu0), a1 = exp2f(m1 - nu1);
      m0 = mn0;
      m1 = mn1;
      p0 = exp2f(s[0] - nu0);
      p1 = exp2f(s[1] - nu0);
      p2 = exp2f(s[2] - nu1);
      p3 = exp2f(s[3] - nu1);
      l0 *= a0;
      l1 *= a1;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        o[nb][0] *= a0;
        o[nb][1] *= a0;
        o[nb][2] *= a1;
        o[nb][3] *= a1;
      }
      *pslot = make_uint2(pack_bf16x2(p0, p1), pack_bf16x2(p2, p3));  // own slot only
      __syncthreads();  // the rewritten P is visible before any warp's P V
    }
    l0 += p0 + p1;
    l1 += p2 + p3;

#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      const uint4 af4 = pfrag[kb * 32 + lane];
      const uint32_t af[4] = {af4.x, af4.y, af4.z, af4.w};
      const int vkey = 16 * kb + (lane & 7) + ((lane >> 3) & 1) * 8;
      const uint32_t vrow = stage + vkey * kSaRowBytes;
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        const int c = 8 * warp + 2 * np + (lane >> 4);
        ptx::ldmatrix_x4_trans(b, vrow + ((c ^ (lane & 7)) << 4));
        ptx::mma_bf16_16816(o[2 * np], af, b[0], b[1]);
        ptx::mma_bf16_16816(o[2 * np + 1], af, b[2], b[3]);
      }
    }
  }
  ptx::cp_async_wait_all();
  __syncthreads();  // every warp is done with red and the ring

  // Sums over the whole split: quad, then warps.
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
  if (tig == 0) {
    red[warp * kSaHeads + g] = l0;
    red[warp * kSaHeads + g + 8] = l1;
  }
  __syncthreads();
  float L0 = 0.f, L1 = 0.f;
#pragma unroll
  for (int w = 0; w < kSaWarps; ++w) {
    L0 += red[w * kSaHeads + g];
    L1 += red[w * kSaHeads + g + 8];
  }
  const int col = 64 * warp + 2 * tig;  // value column of o[nb][0] is col + 8 nb

  if (p.splits == 1) {
    const float i0 = L0 > 0.f ? 1.f / L0 : 0.f, i1 = L1 > 0.f ? 1.f / L1 : 0.f;
    __nv_bfloat16* r0 = p.out + (t * kSaHeads + g) * kSaCkv + col;
    __nv_bfloat16* r1 = r0 + 8 * kSaCkv;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      *reinterpret_cast<uint32_t*>(r0 + 8 * nb) = pack_bf16x2(o[nb][0] * i0, o[nb][1] * i0);
      *reinterpret_cast<uint32_t*>(r1 + 8 * nb) = pack_bf16x2(o[nb][2] * i1, o[nb][3] * i1);
    }
    if (warp == 0 && tig == 0) {
      p.lse[t * kSaHeads + g] = L0 > 0.f ? m0 + log2f(L0) : -INFINITY;
      p.lse[t * kSaHeads + g + 8] = L1 > 0.f ? m1 + log2f(L1) : -INFINITY;
    }
    return;
  }

  // Split: publish the unnormalised partial and (max, sum) per head.
  {
    float* po = p.part_o + static_cast<int64_t>(blockIdx.x) * kSaHeads * kSaCkv + g * kSaCkv + col;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      *reinterpret_cast<float2*>(po + 8 * nb) = make_float2(o[nb][0], o[nb][1]);
      *reinterpret_cast<float2*>(po + 8 * kSaCkv + 8 * nb) = make_float2(o[nb][2], o[nb][3]);
    }
    if (warp == 0 && tig == 0) {
      float* pm = p.part_ml + static_cast<int64_t>(blockIdx.x) * kSaHeads * 2;
      *reinterpret_cast<float2*>(pm + 2 * g) = make_float2(m0, L0);
      *reinterpret_cast<float2*>(pm + 2 * (g + 8)) = make_float2(m1, L1);
    }
  }
  // One thread's acquire-release add after the barrier publishes the whole
  // CTA's partial and, for the last arriving split, acquires every other
  // split's (the barrier below extends that to all threads), instead of a
  // sequentially consistent fence in every thread.
  __syncthreads();
  if (tid == 0)
    misc[1] = ptx::atom_add_acq_rel_gpu(&p.counters[t], 1u) == static_cast<uint32_t>(p.splits - 1);
  __syncthreads();
  if (!misc[1]) return;
  // Last split of this token: every other split's partial is visible.
  if (tid == 0) p.counters[t] = 0u;
  const int S = p.splits;
  const int64_t first = t * S;
  float* wgt = reinterpret_cast<float*>(sm);                          // [S][16] weight of each partial
  float2* mls = reinterpret_cast<float2*>(sm + kSaMaxSplits * kSaHeads * 4);  // [S][16] (max, sum)
  // Every partial's (max, sum) in one round of loads (a loop over S in 16
  // threads would wait for each load in turn).
  for (int e = tid; e < S * kSaHeads; e += kSaThreads)
    mls[e] = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + first * kSaHeads + e);
  __syncthreads();
  if (tid < kSaHeads) {
    const int h = tid;
    float M = -INFINITY;
    for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, mls[s2 * kSaHeads + h].x);
    float L = 0.f;
    for (int s2 = 0; s2 < S; ++s2) {
      const float2 ml = mls[s2 * kSaHeads + h];
      const float e = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
      wgt[s2 * kSaHeads + h] = e;
      L += e * ml.y;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int s2 = 0; s2 < S; ++s2) wgt[s2 * kSaHeads + h] *= inv;
    p.lse[t * kSaHeads + h] = L > 0.f ? M + log2f(L) : -INFINITY;
  }
  // The partials (32 KB each) come in with cp.async, kSaCombineParts per
  // round, into the ring's stages 1-2 (plain loads from one SM keep too few
  // bytes in flight: ~18 GB/s). Thread tid owns float4 e = tid + 256 k
  // (k < 8) of the [16 heads x 128 float4] output, so every warp reads and
  // writes 512 contiguous bytes.
  float4 acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint32_t cbuf = sbase + SaLayout::kStage;
  const float4* cb = reinterpret_cast<const float4*>(sm + SaLayout::kStage);
  const uint8_t* parts = reinterpret_cast<const uint8_t*>(p.part_o + first * kSaHeads * kSaCkv);
#pragma unroll 1
  for (int s0 = 0; s0 < S; s0 += kSaCombineParts) {
    const int np = min(kSaCombineParts, S - s0);
    __syncthreads();  // the weights are visible; the previous round's buffer is read
    for (int c = tid; c < np * (kSaHeads * kSaCkv / 4); c += kSaThreads)
      ptx::cp_async16(cbuf + c * 16, parts + (static_cast<int64_t>(s0) * (kSaHeads * kSaCkv / 4) + c) * 16, 16u);
    ptx::cp_async_commit();
    ptx::cp_async_wait_all();
    __syncthreads();
    for (int q = 0; q < np; ++q) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = tid + kSaThreads * k;
        const float w = wgt[(s0 + q) * kSaHeads + (e >> 7)];
        const float4 v = cb[q * (kSaHeads * kSaCkv / 4) + e];
        acc[k].x += w * v.x;
        acc[k].y += w * v.y;
        acc[k].z += w * v.z;
        acc[k].w += w * v.w;
      }
    }
  }
  uint2* dst = reinterpret_cast<uint2*>(p.out + t * kSaHeads * kSaCkv);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    dst[tid + kSaThreads * k] = make_uint2(pack_bf16x2(acc[k].x, acc[k].y), pack_bf16x2(acc[k].z, acc[k].w));
}

}  // namespace dsa
