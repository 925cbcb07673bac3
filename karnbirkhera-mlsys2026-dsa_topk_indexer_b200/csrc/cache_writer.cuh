// Index-K cache writer: quantises new index-K vectors (128 values per token)
// to FP8 e4m3 with one fp32 scale per token and writes them into their slots
// of the paged cache the indexer reads. This is the producer side of the
// page format (64 tokens x 128 e4m3 bytes, then 64 fp32 scales; 8448 bytes
// a page), which the reference repository only consumes
// (solution/cuda/kernel.cu:22-25 and its dequantisation
// `f32(fp8) * scale`).
//
// Per token: amax = max |x_i| (fp32), scale = amax / 448 and inv = 448 / amax
// (IEEE fp32 divisions; 448 is the largest finite e4m3 value; both 1 when
// scale is not positive or inv not finite, e.g. an all-zero vector),
// q_i = e4m3(x_i * inv) rounded to nearest even, saturating. Inputs must be
// finite.
// Rows reach shared memory through a cp.async ring; eight lanes quantise a
// token (16 values each, one 16-byte store each), the first of them stores
// the scale. HBM-bound:
// per token 256 B (bf16) or 512 B (fp32) read, 8 B slot, 132 B written.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "indexer_kernel.cuh"

namespace dsa {

constexpr int kWriterWarps = 8;  // tokens per CTA

// Two fp32 values -> two e4m3 bytes (lo in bits 0..7), round to nearest even,
// saturating to +-448.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Rows are streamed through shared memory: a ring of kWriterStages chunks of
// kWriterChunk bytes of rows (+ their slots) filled with cp.async, so the
// loads in flight are bounded by shared memory rather than registers.
constexpr int kWriterStages = 3;
constexpr int kWriterChunk = 16384;

template <bool kBf16>
struct WriterGeom {
  static constexpr int kRowBytes = kBf16 ? 256 : 512;
  static constexpr int kTokens = kWriterChunk / kRowBytes;  // tokens per chunk
  static constexpr int kSlotOff = kWriterStages * kWriterChunk;
  static constexpr int kSmem = kSlotOff + kWriterStages * kTokens * 8;
};

template <bool kBf16>
__global__ void __launch_bounds__(32 * kWriterWarps)
    cache_write_kernel(const void* __restrict__ k, const int64_t* __restrict__ slots, uint8_t* __restrict__ cache,
                       int64_t num_tokens, int64_t num_pages) {
  using Geo = WriterGeom<kBf16>;
  extern __shared__ __align__(16) uint8_t wsm[];
  const uint32_t sbase = ptx::smem_addr(wsm);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nchunks = (num_tokens + Geo::kTokens - 1) / Geo::kTokens;
  const uint8_t* kb = static_cast<const uint8_t*>(k);
  // Chunk c of this CTA: global chunk blockIdx.x + c * gridDim.x.
  auto issue = [&](int64_t c, int stage) {
    const int64_t t0 = c * Geo::kTokens;
    const int64_t avail = num_tokens - t0;  // tokens of this chunk that exist
    const int64_t rows_bytes = (avail < Geo::kTokens ? avail : Geo::kTokens) * Geo::kRowBytes;
    for (int i = tid; i < kWriterChunk / 16; i += 32 * kWriterWarps) {
      const int64_t b = static_cast<int64_t>(i) * 16;
      ptx::cp_async16(sbase + stage * kWriterChunk + static_cast<uint32_t>(b),
                      kb + (b < rows_bytes ? t0 * Geo::kRowBytes + b : 0), b < rows_bytes ? 16u : 0u);
    }
    for (int i = tid; i < Geo::kTokens / 2; i += 32 * kWriterWarps) {
      const int64_t t = t0 + 2 * i;
      const uint32_t nb = t + 2 <= num_tokens ? 16u : (t < num_tokens ? 8u : 0u);
      ptx::cp_async16(sbase + Geo::kSlotOff + (stage * Geo::kTokens + 2 * i) * 8, nb ? slots + t : slots, nb);
    }
  };
  int64_t c_issue = blockIdx.x;
#pragma unroll
  for (int s = 0; s < kWriterStages - 1; ++s) {
    if (c_issue < nchunks) issue(c_issue, s);
    ptx::cp_async_commit();
    c_issue += gridDim.x;
  }
  int stage = 0;
#pragma unroll 1
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    // Refill the stage consumed last iteration, then wait for this one.
    if (c_issue < nchunks) issue(c_issue, (stage + kWriterStages - 1) % kWriterStages);
    ptx::cp_async_commit();
    c_issue += gridDim.x;
    ptx::cp_async_wait_group<kWriterStages - 1>();
    __syncthreads();
    const uint8_t* rows = wsm + stage * kWriterChunk;
    const int64_t* sl = reinterpret_cast<const int64_t*>(wsm + Geo::kSlotOff) + stage * Geo::kTokens;
    const int64_t t0 = c * Geo::kTokens;
    // Eight lanes per token (16 values each), four tokens per warp at once:
    // the token-wide work (max reduction, scale, address) is shared by 8
    // lanes instead of 32.
    const int sub = lane >> 3, l8 = lane & 7;
#pragma unroll 1
    for (int j0 = warp * 4; j0 < Geo::kTokens; j0 += kWriterWarps * 4) {
      const int j = j0 + sub;
      const int64_t slot = (t0 + j < num_tokens) ? sl[j] : -1;
      float v[16];
      if (kBf16) {
        const uint4* r = reinterpret_cast<const uint4*>(rows + j * Geo::kRowBytes) + 2 * l8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 raw = r[h];
          const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[e]);
            v[8 * h + 2 * e] = __low2float(b2);
            v[8 * h + 2 * e + 1] = __high2float(b2);
          }
        }
      } else {
        const float4* r = reinterpret_cast<const float4*>(rows + j * Geo::kRowBytes) + 4 * l8;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float4 raw = r[h];
          v[4 * h] = raw.x;
          v[4 * h + 1] = raw.y;
          v[4 * h + 2] = raw.z;
          v[4 * h + 3] = raw.w;
        }
      }
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
      for (int off = 4; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
      // One reciprocal per token; both quotients IEEE (bit-identical to the
      // CPU restatement). An all-zero vector, or one so small that either
      // quotient leaves the finite positive range, is stored with scale 1.
      float scale = __fdiv_rn(amax, 448.f);
      float inv = __fdiv_rn(448.f, amax);
      if (!(scale > 0.f) || !(inv < INFINITY)) scale = inv = 1.f;
      uint32_t q[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        q[e] = cvt_e4m3x2(__fmul_rn(v[4 * e], inv), __fmul_rn(v[4 * e + 1], inv)) |
               (cvt_e4m3x2(__fmul_rn(v[4 * e + 2], inv), __fmul_rn(v[4 * e + 3], inv)) << 16);
      if (slot < 0) continue;  // padding token (or past the end)
      const int64_t page = slot >> 6;
      if (page >= num_pages) {
        if (l8 == 0) atomicOr(&g_dsa_status, DSA_STATUS_BAD_PAGE);
        continue;
      }
      uint8_t* pg = cache + page * kPageBytes;
      const int off = static_cast<int>(slot & 63);
      reinterpret_cast<uint4*>(pg + off * 128)[l8] = make_uint4(q[0], q[1], q[2], q[3]);
      if (l8 == 0) reinterpret_cast<float*>(pg + kPageData)[off] = scale;
    }
    __syncthreads();  // the stage may be refilled next iteration
    stage = (stage + 1) % kWriterStages;
  }
  ptx::cp_async_wait_all();
}

}  // namespace dsa
