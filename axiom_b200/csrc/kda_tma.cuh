// TMA tile loads of [B, T, H, 128] bf16 tensors (q, k, v, g, dO) straight into
// the 8x8 core-matrix (CM) layout the tensor-core kernels use.
//
// The tensor map is 5-D, innermost first:
//   e  (8 elements of one 16-byte column group, contiguous)
//   r8 (8 rows of one row group, stride H*128*2 bytes)
//   cg (column groups of all heads, H*16 of them, stride 16 bytes)
//   rg (row groups, T/8 of them, stride 8*H*128*2 bytes)
//   b  (batch, stride T*H*128*2 bytes)
// and the box {8, 8, 16, 8, 1} at (0, 0, 16h, 8c, b) is the [64][128] tile of
// head h, chunk c: TMA writes it dim 0 fastest, i.e. core matrix (rg, cg) at
// ((rg * 16) + cg) * 128 bytes, rows 16 bytes apart inside -- the CM layout.
// Rows past T fall outside the rg extent and are zero-filled, which needs
// T % 8 == 0; other lengths use the cp.async staging.  The innermost
// coordinate is always 0, so every copy starts 16-byte aligned.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "kda_tc.cuh"

namespace kda {

// Encodes the tile map of a [B, T, H, 128] bf16 tensor at `base` (16-byte
// aligned).  Returns false (map unusable) when T % 8 != 0 or the driver's
// encoder is unavailable or rejects the map.
bool make_tile_map(CUtensorMap* map, const void* base, int B, int T, int H);

// Store map of a [B, T, H, 128] bf16 output: 4-D (channel, head, token, batch),
// box {64, 1, 64, 1} = 64 tokens x 64 channels of one head, SWIZZLE_128B: the
// shared source is 64 rows of 128 bytes whose 16-byte chunk j sits at position
// j ^ (row & 7).  Tokens past T are not written (any T).  Returns false when
// the encoder is unavailable or rejects the map.
bool make_out_map(CUtensorMap* map, const void* base, int B, int T, int H);

namespace tc {
// One [64][128] tile (16384 bytes) of head h, chunk c, batch b into `dst`
// (1024-byte aligned shared memory); completes 16384 transaction bytes on `mbar`.
// Issued by one thread.
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, int h, int c, int b,
                                         uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      :: "r"(smem_u32(dst)), "l"(map), "r"(0), "r"(0), "r"(16 * h), "r"(8 * c), "r"(b),
         "r"(smem_u32(mbar))
      : "memory");
}
// 64 tokens x 64 channels (8 KB, 1024-byte aligned shared memory, the
// make_out_map layout) to channels [d0, d0 + 64) of head h, tokens [t0, t0 + 64)
// of batch b.  Tracked by the issuing thread's bulk async-groups.
__device__ __forceinline__ void tma_out_store(const CUtensorMap* map, const void* src, int d0, int h,
                                              int t0, int b) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];"
      :: "l"(map), "r"(d0), "r"(h), "r"(t0), "r"(b), "r"(smem_u32(src))
      : "memory");
}
}  // namespace tc
}  // namespace kda
