// The tensor-core forward in two launches, for training (the checkpoint's
// factor block is where the two meet): bf16 inputs, dk = dv = 128, C = 64.
//
// fwd_prep -- persistent over all (batch, head, chunk) units: everything of a
//   chunk that does not depend on the state (the reference's chunked_cc body,
//   net/kda.py:669-687): G = cumsum(g) and the decay images Q Gam, K Gam,
//   K Gam^-1, lam K, Gam_C; the scores Aqk, Akk; T = (I + diag(beta) Akk)^-1;
//   W = T diag(beta) K Gam and U = T diag(beta) V.  It writes them to the
//   checkpoint's factor block (kda_ckpt_layout.h), the same block the backward
//   reads.  No unit waits on another, so the work spreads over every SM
//   whatever B * H is.
//
// fwd_scan -- the sequential part only (net/kda.py:689-702), one CTA per
//   (batch, head, column slice of the state): with S_s = S[:, slice] fp32 in
//   tensor memory, per chunk
//     W S_s, (Q Gam) S_s       (two M = 64 MMAs; S_s goes to the checkpoint)
//     v~_s = U_s - W S_s       (bf16, to the checkpoint)
//     O_s  = (Q Gam) S_s + Aqk v~_s ,  S_s <- Gam_C S_s + (lam K)^T v~_s
//   The columns of S never mix (W, Q Gam, Aqk and lam K act on the rows), so a
//   head's state splits into 128 / DVS independent slices: 2 to 8 CTAs walk one
//   head's chunks side by side when there are fewer heads than SMs.
//
// The fused kernel (kda_fwd_tc.cu) does both in one CTA per head; it stays the
// path without a checkpoint (inference), where there is no factor block to hand
// the work over in.
#include <cstdlib>

#include "kda_chunk.cuh"
#include "kda_ckpt_layout.h"
#include "kda_tma.cuh"

namespace kda {
namespace {

using namespace tc;
using namespace chunk;

__device__ int g_fwd_split_error = 0;

// ===========================================================================
// fwd_prep
// ===========================================================================
// shared-memory map (bytes)
constexpr int R_SQ = 0;                  // staging q   CM[64][128]
constexpr int R_SK = R_SQ + 16384;       // staging k
constexpr int R_SG = R_SK + 16384;       // staging g
constexpr int R_V = R_SG + 16384;        // v (operand) CM[64][128]
constexpr int R_A3 = R_V + 16384;        // [W ; Q Gam ; K Gam] CM[192][128]
constexpr int R_KI = R_A3 + 49152;       // K Gi CM[64][128] | T fp32 | G fp32 (slow, with TP)
constexpr int R_TP = R_KI + 16384;       // T diag(beta) CM[64][64] | G fp32 (slow)
constexpr int R_KL = R_TP + 16384;       // lam K CM[64][128]
constexpr int R_SB = R_KL + 16384;       // Aqk fp32 + Akk fp32 | Akk bf16 (first 8 KB)
constexpr int R_VT = R_SB + 32768;       // solve scratch | T, Aqk bf16 [64][64] | exact-path kbm
constexpr int R_BETA = R_VT + 16384;     // beta fp32[64]
constexpr int R_GC = R_BETA + 256;       // Gam_C fp32[128]
constexpr int R_BAR = R_GC + 512;        // mbarriers + tmem slot
constexpr int R_TRI = R_BAR + 128;       // [L ; U'] bf16 CM[128][64] (0/1, built once)
constexpr int R_GN = R_TRI + 16384;      // exp(-G_C) fp32[128] (G_C itself while staged)
constexpr int PREP_SMEM = R_GN + 512;

// Unit u = (b H + h) n_chunks + c: the kernels below also use u itself as the
// chunk-head's slot in the checkpoint (factor blocks, states), so this order
// and that addressing change together.
__device__ __forceinline__ void unit_coords(long long u, int n_chunks, int H, int& b, int& h, int& c) {
  const long long bh = u / n_chunks;
  c = static_cast<int>(u - bh * n_chunks);
  h = static_cast<int>(bh % H);
  b = static_cast<int>(bh / H);
}

template <typename Tc>
__global__ void __launch_bounds__(NT, 1)
fwd_prep_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
                const bf16* __restrict__ g, const bf16* __restrict__ beta,
                unsigned char* __restrict__ factors, int B, int T, int H, int* __restrict__ err,
                const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_v,
                int use_tma) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* beta_s = reinterpret_cast<float*>(sm + R_BETA);
  float* gamC = reinterpret_cast<float*>(sm + R_GC);
  float* gneg = reinterpret_cast<float*>(sm + R_GN);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + R_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + R_BAR + 8);
  uint64_t* mbar_in = reinterpret_cast<uint64_t*>(sm + R_BAR + 16);  // TMA: a unit's q, k, g, v

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;
  const int n_chunks = (T + C - 1) / C;
  const long long n_units = static_cast<long long>(B) * H * n_chunks;
  const size_t rstride = static_cast<size_t>(H) * DK;

  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_init(mbar_in, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  // staging of unit uu's q, k, g (qkg) or v: TMA tiles completing on mbar_in
  // (armed for all four tiles with the q, k, g issue), else cp.async
  auto stage = [&](long long uu, bool qkg) {
    int b_, h_, c_;
    unit_coords(uu, n_chunks, H, b_, h_, c_);
    if (!use_tma) {
      const size_t row0 = static_cast<size_t>(b_) * T + static_cast<size_t>(c_) * C;
      const int rv = min(C, T - c_ * C);
      if (qkg) {
        stage_tile(sm + R_SQ, q + h_ * DK + row0 * rstride, rv, rstride);
        stage_tile(sm + R_SK, k + h_ * DK + row0 * rstride, rv, rstride);
        stage_tile(sm + R_SG, g + h_ * DK + row0 * rstride, rv, rstride);
      } else {
        stage_tile(sm + R_V, v + h_ * DV + row0 * rstride, rv, rstride);
      }
      cp_async_commit();
      return;
    }
    if (tid != kIoThread) return;
    fence_async_smem();
    if (qkg) {
      mbar_expect_tx(mbar_in, 4 * 16384);
      tma_tile(sm + R_SQ, &tm_q, h_, c_, b_, mbar_in);
      tma_tile(sm + R_SK, &tm_k, h_, c_, b_, mbar_in);
      tma_tile(sm + R_SG, &tm_g, h_, c_, b_, mbar_in);
    } else {
      tma_tile(sm + R_V, &tm_v, h_, c_, b_, mbar_in);
    }
  };
  auto beta_load = [&](long long uu) -> unsigned short {
    int b_, h_, c_;
    unit_coords(uu, n_chunks, H, b_, h_, c_);
    const int rv = min(C, T - c_ * C);
    return ld_bf16_raw(beta + (static_cast<size_t>(b_) * T + static_cast<size_t>(c_) * C + tid) * H + h_,
                       tid < rv);
  };
  __syncthreads();  // mbar_in initialised
  const long long u0 = blockIdx.x;
  const bool any = u0 < n_units;
  if (any) {
    stage(u0, true);
    stage(u0, false);
  }
  unsigned short beta_nx = any ? beta_load(u0) : 0;
  bool in_pending = use_tma != 0 && any;
  uint32_t in_par = 0u, in_phase = 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t t_lane = static_cast<uint32_t>(32 * qw) << 16;
  const uint32_t T_D = tbase;  // cols [0, 256)
  uint32_t phase = 0;
  bool failed = false;
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };

  unsigned char* A3 = sm + R_A3;
  const uint32_t a3_addr = smem_u32(A3);
  // the cumulative-sum operand of the decay prep: [L ; U'] g = [G ; G_C - G]
  for (int i = tid; i < 128 * 8; i += NT) {
    const int row = i >> 3, c8 = 8 * (i & 7);
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const int j0 = c8 + e, j1 = c8 + e + 1;
      const bool b0 = row < 64 ? (j0 <= row) : (j0 > row - 64);
      const bool b1 = row < 64 ? (j1 <= row) : (j1 > row - 64);
      w[e >> 1] = (b0 ? 0x3F80u : 0u) | (b1 ? 0x3F800000u : 0u);
    }
    st16(sm + R_TRI, cm_off(row, c8, C), make_uint4(w[0], w[1], w[2], w[3]));
  }
  fence_async_smem();
  __syncthreads();

  for (long long u = u0; u < n_units; u += gridDim.x) {
    int b, h, c;
    unit_coords(u, n_chunks, H, b, h, c);
    const long long u_nx = u + gridDim.x;
    const bool has_nx = u_nx < n_units;
    cp_async_wait<0>();
    if (use_tma) {
      failed |= !mbar_wait(mbar_in, in_phase);
      in_phase ^= 1u;
      in_pending = false;
    }
    if (tid == kIoThread) bulk_wait_read();  // the previous unit's stores have left shared memory
    if (tid < C) beta_s[tid] = bf16_raw_to_float(beta_nx);
    if (has_nx) beta_nx = beta_load(u_nx);
    if (__syncthreads_or(failed)) break;
    float* Aq = reinterpret_cast<float*>(sm + R_SB);
    float* Akk = Aq + 4096;
    unsigned char* fu = factors + static_cast<size_t>(u) * FAC_UNIT;
    auto store_prep = [&](bool slow_chunk) {
      if (!slow_chunk) bulk_store(fu + FAC_KI, sm + R_KI, 16384);
      bulk_commit();
      bulk_store(fu + FAC_QG, A3 + cm_off(64, 0, DK), 2 * 16384);  // Q Gam, K Gam (adjacent)
      bulk_store(fu + FAC_KL, sm + R_KL, 16384);
      bulk_store(fu + FAC_GC, gamC, 512);
      bulk_commit();
      *reinterpret_cast<uint32_t*>(fu + FAC_FLAG) = (slow_chunk ? FLAG_EXACT : 0u) | FLAG_CHAIN;
    };
    // ---- decay prep: [G ; G_C - G] = [L ; U'] g on the tensor core
    if (tid == 0) {
      tc_fence_after();
      const uint32_t tri = smem_u32(sm + R_TRI), gt = smem_u32(sm + R_SG);
      const uint32_t idesc = idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_D, desc_kmajor(tri + ks * 256, C), desc_mnmajor(gt + ks * 4096, DK), idesc, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    const int R = 32 * qw + lane;
    bool strong = false;
    if (qw == 1) {  // warps 1, 5 hold row 63 (lane 31): G_C of their 64 channels
      for (int half = 0; half < 2; ++half) {
        float gv[32];
        tmem_ld32(T_D + t_lane + hh * 64 + 32 * half, gv);
        tmem_wait_ld();
        if (lane == 31) {
#pragma unroll
          for (int j = 0; j < 32; ++j) gneg[hh * 64 + 32 * half + j] = gv[j];
        }
      }
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = hh * 64 + 2 * lane + e;
        const float gc = gneg[d];
        gamC[d] = __expf(gc);
        gneg[d] = __expf(-gc);
        strong |= fabsf(gc) > kExpBudget;
      }
    }
    const bool slow = __syncthreads_or(strong) != 0;
    float* Gf = reinterpret_cast<float*>(sm + R_KI);  // exact path: G fp32 [64][128] across KI|TP
    for (int half = 0; half < 2; ++half) {
      const int c32 = hh * 64 + 32 * half;
      float gv[32];
      tmem_ld32(T_D + t_lane + c32, gv);
      tmem_wait_ld();
      if (R < 64) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint32_t off = cm_off(R, c32 + j, DK);
          float qv[8], kv[8], qg[8], kg[8];
          unpack_bf16x8(ld16(sm + R_SQ, off), qv);
          unpack_bf16x8(ld16(sm + R_SK, off), kv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float gam = __expf(gv[j + e]);
            qg[e] = qv[e] * gam;
            kg[e] = kv[e] * gam;
          }
          st16(A3, cm_off(64 + R, c32 + j, DK), pack_bf16x8(qg));
          st16(A3, cm_off(128 + R, c32 + j, DK), pack_bf16x8(kg));
          if (slow) {
            *reinterpret_cast<float4*>(Gf + gsw(R, c32 + j)) = make_float4(gv[j], gv[j + 1], gv[j + 2], gv[j + 3]);
            *reinterpret_cast<float4*>(Gf + gsw(R, c32 + j + 4)) =
                make_float4(gv[j + 4], gv[j + 5], gv[j + 6], gv[j + 7]);
          }
        }
      } else {
        const int r = R - 64;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint32_t off = cm_off(r, c32 + j, DK);
          float kv[8], kl[8], ki[8];
          unpack_bf16x8(ld16(sm + R_SK, off), kv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            kl[e] = kv[e] * __expf(slow ? fminf(gv[j + e], 0.f) : gv[j + e]);
            ki[e] = kl[e] * gneg[c32 + j + e];
          }
          st16(sm + R_KL, off, pack_bf16x8(kl));
          if (!slow) st16(sm + R_KI, off, pack_bf16x8(ki));
        }
      }
    }
    tc_fence_before();  // the TMEM reads above precede the score MMA's writes to T_D
    if (!slow) {
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint32_t idesc = idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int ks = 0; ks < DK / 16; ++ks)
          mma_bf16(T_D, desc_kmajor(a3_addr + 64 * 256 + ks * 256, DK),
                   desc_kmajor(smem_u32(sm + R_KI) + ks * 256, DK), idesc, ks > 0);
        mma_commit(mbar);
      }
      if (tid == kIoThread) store_prep(false);
      if (has_nx) {  // the next unit's q, k, g (staging is free)
        stage(u_nx, true);
        in_pending = use_tma != 0;
        in_par = in_phase;
      }
      failed |= !mma_wait();
      if (__syncthreads_or(failed)) break;
      scores_epilogue(T_D, Aq, Akk);
    } else {
      fence_async_smem();
      __syncthreads();
      if (tid == kIoThread) store_prep(true);
      const bool halves = __syncthreads_or(!halves_within_budget(Gf)) == 0;
      if (halves) {
        unsigned char *bd = A3, *bc = sm + R_VT;  // A3 rows 0..63 (W comes later), VT
        scores_halves_prep(sm + R_SQ, sm + R_SK, bd, bc, Gf);
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
          tc_fence_after();
          scores_halves_mma(T_D, smem_u32(sm + R_SQ), smem_u32(bd), smem_u32(bc));
          mma_commit(mbar);
        }
        failed |= !mma_wait();
        if (__syncthreads_or(failed)) break;
        scores_halves_epilogue(T_D, Aq, Akk);
      } else {
        unsigned char *kbm1 = A3 + 12288, *kbm2 = sm + R_VT, *kbm3 = A3;
        scores_exact_prep(sm + R_SQ, sm + R_SK, sm + R_SG, kbm1, kbm2, kbm3, Gf, Aq, Akk);
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
          tc_fence_after();
          scores_exact_mma(T_D, smem_u32(sm + R_SQ), smem_u32(kbm1), smem_u32(kbm2), smem_u32(kbm3));
          mma_commit(mbar);
        }
        failed |= !mma_wait();
        if (__syncthreads_or(failed)) break;
        scores_exact_epilogue(T_D, Aq, Akk);
      }
      __syncthreads();
      if (has_nx) {
        stage(u_nx, true);
        in_pending = use_tma != 0;
        in_par = in_phase;
      }
    }
    // ---- solve: T = (I + L)^-1
    {
      float* Tm = reinterpret_cast<float*>(sm + R_KI);
      if (tid == kIoThread) bulk_wait_read<1>();  // KI has been stored and may be overwritten
      __syncthreads();
      solve_T(Akk, beta_s, Tm, reinterpret_cast<float*>(sm + R_VT));
      const int r = 8 * (tid >> 5) + (tid & 7), c0 = 16 * ((tid >> 3) & 3);
      float tv[16], a[16], kk[16];
      ld_row16_sw64(Tm, r, c0, tv);
      ld_row16_sw64(Aq, r, c0, a);
      ld_row16_sw64(Akk, r, c0, kk);
      st16(sm + R_VT, cm_off(r, c0, C), pack_bf16x8(tv));            // T      (bf16)
      st16(sm + R_VT, cm_off(r, c0 + 8, C), pack_bf16x8(tv + 8));
      st16(sm + R_VT + 8192, cm_off(r, c0, C), pack_bf16x8(a));      // Aqk    (bf16)
      st16(sm + R_VT + 8192, cm_off(r, c0 + 8, C), pack_bf16x8(a + 8));
#pragma unroll
      for (int j = 0; j < 16; ++j) tv[j] *= beta_s[c0 + j];
      st16(sm + R_TP, cm_off(r, c0, C), pack_bf16x8(tv));            // T diag(beta)
      st16(sm + R_TP, cm_off(r, c0 + 8, C), pack_bf16x8(tv + 8));
      __syncthreads();
      st16(sm + R_SB, cm_off(r, c0, C), pack_bf16x8(kk));            // Akk bf16 over the fp32 Aqk
      st16(sm + R_SB, cm_off(r, c0 + 8, C), pack_bf16x8(kk + 8));
    }
    fence_async_smem();
    __syncthreads();
    if (tid == kIoThread) {  // T, Aqk (adjacent in VT) and Akk
      bulk_store(fu + FAC_T, sm + R_VT, 16384);
      bulk_store(fu + FAC_AK, sm + R_SB, 8192);
      bulk_commit();
    }
    // ---- P = Aqk T  (M = 64: row r at TMEM lane 32 (r / 16) + r % 16)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(64, 64, false, true);
      const uint32_t tb = smem_u32(sm + R_VT), aqb = smem_u32(sm + R_VT + 8192);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_D, desc_kmajor(aqb + ks * 256, C), desc_mnmajor(tb + ks * 2048, C), idesc, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // P diag(beta) -> rows 64..127 of the [T b ; P b] operand
      float vals[32];
      tmem_ld32(T_D + t_lane + hh * 32, vals);
      tmem_wait_ld();
      if (lane < 16) {
        const int r = 16 * qw + lane;
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] *= beta_s[hh * 32 + j];
#pragma unroll
        for (int j = 0; j < 32; j += 8) st16(sm + R_TP, cm_off(64 + r, hh * 32 + j, C), pack_bf16x8(vals + j));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- [T b ; P b] [K Gam | V] -> W, U (rows 0..63), Aqk W, Aqk U (rows 64..127)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 128, false, true);
      const uint32_t tp = smem_u32(sm + R_TP);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        const uint64_t ad = desc_kmajor(tp + ks * 256, C);
        mma_bf16(T_D, ad, desc_mnmajor(a3_addr + 128 * 256 + ks * 4096, DK), idesc, ks > 0);
        mma_bf16(T_D + 128, ad, desc_mnmajor(smem_u32(sm + R_V) + ks * 4096, DV), idesc, ks > 0);
      }
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (tid == kIoThread) bulk_wait_read<1>();  // Q Gam, K Gam have left A3 (E2 overwrites Q Gam)
    if (__syncthreads_or(failed)) break;
    if (has_nx) stage(u_nx, false);  // V has been consumed
    // ---- E2: W -> A3 rows 0..63, U -> the checkpoint; Q~ = Q Gam - Aqk W -> A3 rows
    // 64..127, Aqk U -> the checkpoint
    {
      const int R = 32 * qw + lane;
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float wv[32], uu[32];
        tmem_ld32(T_D + t_lane + c0, wv);
        tmem_ld32(T_D + t_lane + 128 + c0, uu);
        tmem_wait_ld();
        const size_t fo = R < 64 ? FAC_U : FAC_AU;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint32_t off = cm_off(R, c0 + j, DK);  // rows 64..127 of A3 hold Q Gam
          if (R < 64) {
            st16(A3, off, pack_bf16x8(wv + j));
          } else {
            float qg[8];
            unpack_bf16x8(ld16(A3, off), qg);
#pragma unroll
            for (int e = 0; e < 8; ++e) qg[e] -= wv[j + e];
            st16(A3, off, pack_bf16x8(qg));
          }
          *reinterpret_cast<uint4*>(fu + fo + cm_off(R & 63, c0 + j, DV)) = pack_bf16x8(uu + j);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {  // W, then Q~
      bulk_store(fu + FAC_W, A3, 16384);
      bulk_store(fu + FAC_QT, A3 + 16384, 16384);
      bulk_commit();
    }
    // ---- NP = -(lam K)^T W  (M = dk = 128, N = dk, K = C)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 128, true, true);
      const uint32_t kl = smem_u32(sm + R_KL);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_D, desc_mnmajor(kl + ks * 4096, DK), desc_mnmajor(a3_addr + ks * 4096, DK), idesc, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (tid == kIoThread) bulk_wait_read<1>();  // T, Aqk, Akk have left VT and SB
    if (__syncthreads_or(failed)) break;
    {  // row i of NP = TMEM lane i -> bf16 CM [128][128] in SB (32 KB)
      const int i = 32 * qw + lane;
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float pv[32];
        tmem_ld32(T_D + t_lane + c0, pv);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) pv[j] = -pv[j];
#pragma unroll
        for (int j = 0; j < 32; j += 8) st16(sm + R_SB, cm_off(i, c0 + j, DK), pack_bf16x8(pv + j));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {
      bulk_store(fu + FAC_NP, sm + R_SB, 32768);
      bulk_commit();
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  cp_async_wait<0>();
  if (in_pending) mbar_wait(mbar_in, in_par);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// ===========================================================================
// fwd_scan: the state chain only
// ===========================================================================
// S_{c+1} = Gam_C S_c + (lam K)^T U + NP S_c with NP = -(lam K)^T W (the prep's
// FAC_NP): one MMA round trip per chunk.  Chunk c's operands (NP, lam K, the
// slice of U, Gam_C) land in set (c - c_beg) % NSET, issued NSET - 1 chunks
// ahead.
template <int DVS>
struct ScanMap {
  static constexpr int NP = 0, KL = 32768, US = 49152;
  static constexpr int GC = US + 128 * DVS;
  static constexpr int SET = GC + 512;
  // operand sets in flight: loads are issued NSET - 1 chunks ahead (three sets
  // fit beside the state image up to 64 columns, two at 128)
  static constexpr int NSET = DVS == 128 ? 2 : 3;
  static constexpr int SB = NSET * SET;       // S_s bf16 CM[128][DVS] (the MMA operand and checkpoint image)
  static constexpr int BAR = SB + 256 * DVS;
  static constexpr int SMEM = BAR + 64;
  static constexpr uint32_t TX = 32768 + 16384 + 128 * DVS + 512;
  static constexpr int TCOLS = DVS <= 32 ? 32 : DVS;
};

// TMEM loads / stores of N columns (8, 16 or 32) of this warp's 32 lanes.
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, float* v) {
  if constexpr (N == 32) tmem_ld32(taddr, v);
  else if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld8(taddr, v);
}
template <int N>
__device__ __forceinline__ void tmem_stn(uint32_t taddr, const float* v);
template <>
__device__ __forceinline__ void tmem_stn<32>(uint32_t taddr, const float* v) { tmem_st32(taddr, v); }
template <>
__device__ __forceinline__ void tmem_stn<16>(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
         "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
         "r"(r[15])
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_stn<8>(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                  "r"(r[7])
               : "memory");
}

template <typename To>
__device__ __forceinline__ void store_cols(To* dst, const float* v, int n);
template <>
__device__ __forceinline__ void store_cols<float>(float* dst, const float* v, int n) {
  for (int j = 0; j < n; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}
template <>
__device__ __forceinline__ void store_cols<bf16>(bf16* dst, const float* v, int n) {
  for (int j = 0; j < n; j += 8) *reinterpret_cast<uint4*>(dst + j) = pack_bf16x8(v + j);
}

template <typename Tc, int DVS>
__global__ void __launch_bounds__(NT, 1)
fwd_scan_kernel(const unsigned char* __restrict__ factors, const float* __restrict__ s0,
                float* __restrict__ s_out, Tc* __restrict__ s_ckpt, int T, int H, const int* __restrict__ cs,
                int* __restrict__ err) {
  using M = ScanMap<DVS>;
  constexpr int NS = DV / DVS;     // slices per head
  constexpr int CW = DVS / 2;      // columns per thread (each warp: one lane quarter, one column half)
  constexpr int CB = CW < 32 ? CW : 32;  // columns per TMEM access
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + M::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + M::BAR + 8);
  uint64_t* mbar_ld = reinterpret_cast<uint64_t*>(sm + M::BAR + 16);  // [NSET]: one per operand set
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;
  const int n_chunks = (T + C - 1) / C;
  const int s = blockIdx.x % NS;
  const int bh = blockIdx.x / NS;
  const int h = bh % H;
  const int seq = cs ? longest_first(cs, gridDim.x / (H * NS), bh / H, n_chunks, reinterpret_cast<int*>(sm))
                     : bh / H;
  const int b = cs ? 0 : seq;
  const int c_beg = cs ? min(max(cs[seq], 0), n_chunks) : 0;
  const int c_end = cs ? min(max(cs[seq + 1], c_beg), n_chunks) : n_chunks;
  const size_t unit0 = (static_cast<size_t>(b) * H + h) * n_chunks;  // factor / checkpoint row
  const int col0 = s * DVS;           // this CTA's state columns [col0, col0 + DVS)
  const int cg0 = col0 / 8;           // ... as core-matrix columns

  if (tid == 0) {
    mbar_init(mbar, 1);
    for (int p = 0; p < M::NSET; ++p) mbar_init(mbar_ld + p, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, M::TCOLS);
    tmem_relinquish();
  }
  uint32_t ld_par = 0u, ld_pending = 0u;  // bit p: phase parity / loads in flight of set p
  auto issue = [&](int cc) {
    const int p = (cc - c_beg) % M::NSET;
    if (tid == kIoThread) {
      unsigned char* set = sm + p * M::SET;
      const unsigned char* fu = factors + (unit0 + cc) * FAC_UNIT;
      fence_async_smem();  // the set's generic reads (chunk cc - 2) precede the copies' writes
      mbar_expect_tx(mbar_ld + p, M::TX);
      bulk_load(set + M::NP, fu + FAC_NP, 32768, mbar_ld + p);
      bulk_load(set + M::KL, fu + FAC_KL, 16384, mbar_ld + p);
#pragma unroll 1
      for (int rg = 0; rg < 8; ++rg)
        bulk_load(set + M::US + rg * (16 * DVS), fu + FAC_U + (rg * 16 + cg0) * 128, 16 * DVS, mbar_ld + p);
      bulk_load(set + M::GC, fu + FAC_GC, 512, mbar_ld + p);
    }
    ld_pending |= 1u << p;
  };
  __syncthreads();  // barriers initialised
  for (int cc = c_beg; cc < min(c_end, c_beg + M::NSET - 1); ++cc) issue(cc);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tl = static_cast<uint32_t>(32 * qw) << 16;
  const uint32_t T_S = tbase;
  uint32_t phase = 0;
  bool failed = false;
  const int d = 32 * qw + lane;  // the state row this thread moves
  const int cw0 = hh * CW;       // its first column within the slice
  {  // S0 -> TMEM
    const size_t sb = ((static_cast<size_t>(seq) * H + h) * DK + d) * DV + col0 + cw0;
#pragma unroll
    for (int j = 0; j < CW; j += CB) {
      float vals[CB];
#pragma unroll
      for (int e = 0; e < CB; ++e) vals[e] = s0 ? s0[sb + j + e] : 0.f;
      tmem_stn<CB>(T_S + tl + cw0 + j, vals);
    }
    tmem_wait_st();
  }

  for (int c = c_beg; c < c_end; ++c) {
    const int p = (c - c_beg) % M::NSET;
    unsigned char* set = sm + p * M::SET;
    failed |= !mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
    ld_par ^= 1u << p;
    ld_pending &= ~(1u << p);
    if (tid == kIoThread) bulk_wait_read();  // the previous S_s image has been stored
    if (__syncthreads_or(failed)) break;
    // the set of chunk c + NSET - 1 was last read by chunk c - 1, which has completed
    if (c + M::NSET - 1 < c_end) issue(c + M::NSET - 1);
    // ---- S pass: S_s -> bf16 operand (+ checkpoint), S_s *= Gam_C
    Tc* ck = s_ckpt + (unit0 + c) * (DK * DV);
    {
      const float gcd = reinterpret_cast<const float*>(set + M::GC)[d];
#pragma unroll
      for (int j = 0; j < CW; j += CB) {
        float vals[CB];
        tmem_ldn<CB>(T_S + tl + cw0 + j, vals);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < CB; e += 8) st16(sm + M::SB, cm_off(d, cw0 + j + e, DVS), pack_bf16x8(vals + e));
        if (sizeof(Tc) == 4) store_cols<float>(reinterpret_cast<float*>(ck) + d * DV + col0 + cw0 + j, vals, CB);
#pragma unroll
        for (int e = 0; e < CB; ++e) vals[e] *= gcd;
        tmem_stn<CB>(T_S + tl + cw0 + j, vals);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {  // the slice of the bf16 state image (one bulk group per chunk, maybe empty)
      if (sizeof(Tc) == 2) {
        unsigned char* img = reinterpret_cast<unsigned char*>(ck);
#pragma unroll 1
        for (int rg = 0; rg < 16; ++rg)
          bulk_store(img + (rg * 16 + cg0) * 128, sm + M::SB + rg * (16 * DVS), 16 * DVS);
      }
      bulk_commit();
    }
    // ---- S_s += (lam K)^T U_s + NP S_s  (M = dk, N = DVS)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t id = idesc_bf16(128, DVS, true, true), id_np = idesc_bf16(128, DVS, false, true);
      const uint32_t kl = smem_u32(set + M::KL), us = smem_u32(set + M::US), np = smem_u32(set + M::NP);
      const uint32_t sb = smem_u32(sm + M::SB);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_S, desc_mnmajor(kl + ks * 4096, DK), desc_mnmajor(us + ks * (32 * DVS), DVS), id, 1u);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks)
        mma_bf16(T_S, desc_kmajor(np + ks * 256, DK), desc_mnmajor(sb + ks * (32 * DVS), DVS), id_np, 1u);
      mma_commit(mbar);
    }
    // every thread sees the commit itself; the next chunk's barrier (after its
    // load wait) is the first one that needs all threads, and it shares failures
    failed |= !mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
  }
  failed = __syncthreads_or(failed) != 0;
  if (!failed && s_out) {
    float* so = s_out + ((static_cast<size_t>(seq) * H + h) * DK + d) * DV + col0 + cw0;
#pragma unroll
    for (int j = 0; j < CW; j += CB) {
      float vals[CB];
      tmem_ldn<CB>(T_S + tl + cw0 + j, vals);
      tmem_wait_ld();
      store_cols<float>(so + j, vals, CB);
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  for (int p = 0; p < M::NSET; ++p)
    if ((ld_pending >> p) & 1u) mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, M::TCOLS);
}

// ===========================================================================
// fwd_out: the chunk outputs, chunk-parallel
// ===========================================================================
// With every chunk's entering state in the checkpoint, each unit is
// independent: [W ; Q~] S_c (one M = 128 MMA) gives W S_c and Q~ S_c, then
//   v~ = U - W S_c  (bf16, the backward's FAC_VT)     O = Q~ S_c + Aqk U.
// Persistent over the units; a unit's operands (S_c, [W ; Q~], U, Aqk U) land in
// set it & 1 while the previous unit runs.
constexpr int O_SC = 0, O_WQ = 32768, O_U = 65536, O_AU = 81920, O_SET = 98304;
constexpr int O_VT = 2 * O_SET;       // v~ bf16 CM [64][128] (stored to the checkpoint)
constexpr int O_BAR = O_VT + 16384;
constexpr int OUT_SMEM = O_BAR + 64;

template <typename To, typename Tc>
__global__ void __launch_bounds__(NT, 1)
fwd_out_kernel(unsigned char* __restrict__ factors, const Tc* __restrict__ s_ckpt, To* __restrict__ o, int B,
               int T, int H, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + O_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + O_BAR + 8);
  uint64_t* mbar_ld = reinterpret_cast<uint64_t*>(sm + O_BAR + 16);  // [2]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;
  const int n_chunks = (T + C - 1) / C;
  const long long n_units = static_cast<long long>(B) * H * n_chunks;
  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_init(mbar_ld, 1);
    mbar_init(mbar_ld + 1, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  uint32_t ld_par = 0u, ld_pending = 0u;
  // (fp32 checkpoint states are converted by all threads when the unit starts)
  auto issue = [&](long long uu, int p) {
    unsigned char* set = sm + p * O_SET;
    if (tid == kIoThread) {
      const unsigned char* fu = factors + static_cast<size_t>(uu) * FAC_UNIT;
      fence_async_smem();
      mbar_expect_tx(mbar_ld + p, 16384 * 4 + (sizeof(Tc) == 2 ? 32768 : 0));  // one arrival per phase
      if (sizeof(Tc) == 2)
        bulk_load(set + O_SC, s_ckpt + static_cast<size_t>(uu) * (DK * DV), 32768, mbar_ld + p);
      bulk_load(set + O_WQ, fu + FAC_W, 16384, mbar_ld + p);
      bulk_load(set + O_WQ + 16384, fu + FAC_QT, 16384, mbar_ld + p);
      bulk_load(set + O_U, fu + FAC_U, 16384, mbar_ld + p);
      bulk_load(set + O_AU, fu + FAC_AU, 16384, mbar_ld + p);
    }
    ld_pending |= 1u << p;
  };
  __syncthreads();
  const long long u0 = blockIdx.x;
  if (u0 < n_units) issue(u0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tl = static_cast<uint32_t>(32 * qw) << 16;
  uint32_t phase = 0;
  bool failed = false;
  int it = 0;
  for (long long u = u0; u < n_units; u += gridDim.x, ++it) {
    const int p = it & 1;
    unsigned char* set = sm + p * O_SET;
    int b, h, c;
    unit_coords(u, n_chunks, H, b, h, c);
    if (sizeof(Tc) == 4) {  // fp32 checkpoint states (row-major) -> bf16 CM operand
      const float* src = reinterpret_cast<const float*>(s_ckpt) + static_cast<size_t>(u) * (DK * DV);
      for (int i = tid; i < 128 * 16; i += NT) {
        const int r = i >> 4, cg = i & 15;
        const float4 x0 = *reinterpret_cast<const float4*>(src + r * 128 + cg * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(src + r * 128 + cg * 8 + 4);
        const float f[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        st16(set + O_SC, cm_off(r, cg * 8, DV), pack_bf16x8(f));
      }
      fence_async_smem();
    }
    failed |= !mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
    ld_par ^= 1u << p;
    ld_pending &= ~(1u << p);
    if (tid == kIoThread) bulk_wait_read();  // the previous unit's v~ has been stored
    if (__syncthreads_or(failed)) break;
    if (u + gridDim.x < n_units) issue(u + gridDim.x, p ^ 1);  // the other set's unit has completed
    if (tid == 0) {  // [W ; Q~] S_c
      tc_fence_after();
      const uint32_t id = idesc_bf16(128, 128, false, true);
      const uint32_t wq = smem_u32(set + O_WQ), sc = smem_u32(set + O_SC);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks)
        mma_bf16(tbase, desc_kmajor(wq + ks * 256, DK), desc_mnmajor(sc + ks * 4096, DV), id, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    if (__syncthreads_or(failed)) break;
    {
      const int R = 32 * qw + lane, r = R & 63, rv = min(C, T - c * C);
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float x[32];
        tmem_ld32(tbase + tl + c0, x);
        tmem_wait_ld();
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; j += 8) unpack_bf16x8(ld16(set + (R < 64 ? O_U : O_AU), cm_off(r, c0 + j, DV)), y + j);
        if (R < 64) {  // v~ = U - W S_c
#pragma unroll
          for (int j = 0; j < 32; ++j) y[j] -= x[j];
#pragma unroll
          for (int j = 0; j < 32; j += 8) st16(sm + O_VT, cm_off(r, c0 + j, DV), pack_bf16x8(y + j));
        } else if (r < rv) {  // O = Q~ S_c + Aqk U
#pragma unroll
          for (int j = 0; j < 32; ++j) y[j] += x[j];
          store_cols<To>(o + ((static_cast<size_t>(b) * T + static_cast<size_t>(c) * C + r) * H + h) * DV + c0, y, 32);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {
      bulk_store(factors + static_cast<size_t>(u) * FAC_UNIT + FAC_VT, sm + O_VT, 16384);
      bulk_commit();
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  for (int p = 0; p < 2; ++p)
    if ((ld_pending >> p) & 1u) mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

template <typename Tc, int DVS>
int launch_scan(const unsigned char* factors, const float* s0, float* s_out, void* s_ckpt, int B, int T, int H,
                const int* cs, int n_seqs, int* err, cudaStream_t st) {
  static std::atomic<bool> done[64];
  auto kern = fwd_scan_kernel<Tc, DVS>;
  int rc = ensure_smem(kern, ScanMap<DVS>::SMEM, done);
  if (rc != KDA_OK) return rc;
  const long long grid = static_cast<long long>(cs ? n_seqs : B) * H * (DV / DVS);
  if (grid > 0x7fffffffLL) return KDA_ERR_SHAPE;
  kern<<<static_cast<unsigned>(grid), NT, ScanMap<DVS>::SMEM, st>>>(factors, s0, s_out, static_cast<Tc*>(s_ckpt),
                                                                   T, H, cs, err);
  return launch_status();
}

template <typename To, typename Tc>
int launch_split(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* s0,
                 void* o, float* s_out, void* s_ckpt, int B, int T, int H, const int* cs, int n_seqs,
                 int slices, cudaStream_t st) {
  static std::atomic<bool> done[64];
  auto prep = fwd_prep_kernel<Tc>;
  int rc = ensure_smem(prep, PREP_SMEM, done);
  if (rc != KDA_OK) return rc;
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_fwd_split_error) != cudaSuccess) return KDA_ERR_LAUNCH;
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KDA_ERR_DEVICE;
  const size_t n = (static_cast<size_t>(T) + C - 1) / C;
  unsigned char* factors = static_cast<unsigned char*>(s_ckpt) + static_cast<size_t>(B) * H * n * DK * DV * sizeof(Tc);
  CUtensorMap tm[4] = {};
  const void* srcs[4] = {q, k, g, v};
  int use_tma = 1;
  for (int i = 0; i < 4 && use_tma; ++i) use_tma = make_tile_map(&tm[i], srcs[i], B, T, H) ? 1 : 0;
  const long long units = static_cast<long long>(B) * H * static_cast<long long>(n);
  const int grid = static_cast<int>(units < n_sm ? units : n_sm);
  prep<<<grid, NT, PREP_SMEM, st>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                                    static_cast<const bf16*>(v), static_cast<const bf16*>(g),
                                    static_cast<const bf16*>(beta), factors, B, T, H, err, tm[0], tm[1], tm[2],
                                    tm[3], use_tma);
  rc = launch_status();
  if (rc != KDA_OK) return rc;
  switch (slices) {
    case 1: rc = launch_scan<Tc, 128>(factors, s0, s_out, s_ckpt, B, T, H, cs, n_seqs, err, st); break;
    case 2: rc = launch_scan<Tc, 64>(factors, s0, s_out, s_ckpt, B, T, H, cs, n_seqs, err, st); break;
    case 4: rc = launch_scan<Tc, 32>(factors, s0, s_out, s_ckpt, B, T, H, cs, n_seqs, err, st); break;
    case 8: rc = launch_scan<Tc, 16>(factors, s0, s_out, s_ckpt, B, T, H, cs, n_seqs, err, st); break;
    default: return KDA_ERR_SHAPE;
  }
  if (rc != KDA_OK) return rc;
  static std::atomic<bool> done_out[64];
  auto out = fwd_out_kernel<To, Tc>;
  rc = ensure_smem(out, OUT_SMEM, done_out);
  if (rc != KDA_OK) return rc;
  out<<<grid, NT, OUT_SMEM, st>>>(factors, static_cast<const Tc*>(s_ckpt), static_cast<To*>(o), B, T, H, err);
  return launch_status();
}

}  // namespace

// The number of column slices per head for `heads` (sequence, head) pairs: the
// largest of 1, 2, 4 that keeps the scans' CTAs within one per SM, or the value
// of the environment variable KDA_SCAN_SLICES (1, 2, 4 or 8) when set.  Used by
// the forward's and the backward's state scans alike.  Measured (B200, T = 8192,
// fwd + bwd): at 16 pairs 1 / 2 / 4 / 8 slices take 0.94 / 0.84 / 0.82 / 0.86 ms,
// at 32 pairs 1.33 / 1.23 / 1.22 / 1.53 ms: past 4 slices every slice CTA still
// loads the whole chunk operands, and the chain per chunk no longer shortens.
int tc_scan_slices(long long heads, int n_sm) {
  const char* e = std::getenv("KDA_SCAN_SLICES");
  if (e) {
    const int v = std::atoi(e);
    if (v == 1 || v == 2 || v == 4 || v == 8) return v;
  }
  int s = 1;
  while (s < 4 && heads * s * 2 <= n_sm) s *= 2;
  return s;
}

int tc_fwd_split_slices(long long heads) {
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  return tc_scan_slices(heads, n_sm);
}

int tc_fwd_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                        const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H, int o_dt,
                        int ck_dt, const int* cs, int n_seqs, int slices, cudaStream_t st) {
  if (!s_ckpt) return KDA_ERR_NULL;  // the factor block is where the two kernels meet
  if (o_dt == KDA_BF16 && ck_dt == KDA_BF16)
    return launch_split<bf16, bf16>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, slices, st);
  if (o_dt == KDA_BF16 && ck_dt == KDA_F32)
    return launch_split<bf16, float>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, slices, st);
  if (o_dt == KDA_F32 && ck_dt == KDA_BF16)
    return launch_split<float, bf16>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, slices, st);
  if (o_dt == KDA_F32 && ck_dt == KDA_F32)
    return launch_split<float, float>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, slices, st);
  return KDA_ERR_DTYPE;
}

int tc_fwd_split_error_flag(int* value, bool clear, cudaStream_t st) {
  static const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(value, g_fwd_split_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (clear && cudaMemcpyToSymbolAsync(g_fwd_split_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) !=
                   cudaSuccess)
    return KDA_ERR_LAUNCH;
  return KDA_OK;
}

}  // namespace kda
