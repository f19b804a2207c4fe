// Layout of the per-chunk factor block the tensor-core forward appends to its
// checkpoint (after the chunk-boundary states), one block per (batch, head,
// chunk).  It holds what the backward would otherwise recompute from q, k, g
// and beta; every tile is the shared-memory operand image (bf16 8 x 8 core
// matrices), so the backward moves each with one bulk copy.
#pragma once
#include <cstddef>
#include <cstdint>

namespace kda {

constexpr size_t FAC_T = 0;          // T = (I + diag(beta) Akk)^-1          bf16 CM [64][64]
constexpr size_t FAC_AQ = 8192;      // Aqk (inclusive lower)                bf16 CM [64][64]
constexpr size_t FAC_AK = 16384;     // Akk (strict lower)                   bf16 CM [64][64]
constexpr size_t FAC_W = 24576;      // W = T diag(beta) K Gam               bf16 CM [64][128]
constexpr size_t FAC_QG = 40960;     // Q Gam                                bf16 CM [64][128]
constexpr size_t FAC_KG = 57344;     // K Gam                                bf16 CM [64][128]
constexpr size_t FAC_KI = 73728;     // K Gam^-1 (fast-path chunks only)     bf16 CM [64][128]
constexpr size_t FAC_KL = 90112;     // lam K = K Gam^-1 Gam_C               bf16 CM [64][128]
constexpr size_t FAC_VT = 106496;    // v~ = U - W S_c                       bf16 CM [64][128]
constexpr size_t FAC_U = 122880;     // U = T diag(beta) V                   bf16 CM [64][128]
constexpr size_t FAC_GC = 139264;    // Gam_C                                fp32 [128]
constexpr size_t FAC_FLAG = 139776;  // u32 flags: FLAG_EXACT | FLAG_CHAIN
constexpr size_t FAC_GF_BYTES = 528; // Gam_C + flags, copied together
// Written only by the split forward's prep (the fused kernel leaves them): the
// chunk's state-chain operands, so that a state scan needs one MMA round trip
// per chunk, S' = Gam_C S + (lam K)^T U + NP S and dS = Gam_C dS' + NP^T dS' + Q~^T dO.
constexpr size_t FAC_NP = 140288;    // NP = -(lam K)^T W   (dk x dk)      bf16 CM [128][128]
constexpr size_t FAC_QT = 173056;    // Q~ = Q Gam - Aqk W                  bf16 CM [64][128]
constexpr size_t FAC_AU = 189440;    // Aqk U                               bf16 CM [64][128]
constexpr size_t FAC_UNIT = 205824;  // bytes per chunk-head (16-byte multiple)

constexpr uint32_t FLAG_EXACT = 1u;  // the chunk took the exact (strong-decay) score path
constexpr uint32_t FLAG_CHAIN = 2u;  // FAC_NP, FAC_QT and FAC_AU hold this chunk's values

static_assert(FAC_FLAG == FAC_GC + 512 && FAC_UNIT % 16 == 0 && FAC_GF_BYTES % 16 == 0 &&
                  FAC_QG == FAC_W + 16384 && FAC_KG == FAC_QG + 16384 && FAC_KL == FAC_KI + 16384 &&
                  FAC_NP == FAC_FLAG + 512 && FAC_QT == FAC_NP + 32768 && FAC_AU == FAC_QT + 16384 &&
                  FAC_UNIT == FAC_AU + 16384,
              "factor block layout");

}  // namespace kda
