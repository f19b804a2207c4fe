// Tensor-core (tcgen05) chunked KDA forward for bf16 inputs, dk = dv = 128,
// chunk C = 64.  One CTA per (batch, head) walks the sequence chunk by chunk;
// the fp32 state S (128 x 128) lives in TMEM for the whole sequence.
//
// Per chunk (the reference's chunked_cc body, net/kda.py:669-702, with the
// products regrouped so that every tensor-core product is an M = 128 MMA):
//   G = cumsum(g), Gam = exp(G), Gi = exp(-G), lam = exp(G_C - G)
//   MMA_sc : [Q*Gam ; K*Gam] (K*Gi)^T          -> Aqk (rows 0-63), Akk (64-127)
//            (single anchor at the chunk start; valid while max|G_C| <= 80,
//             else the scores are evaluated exactly on the CUDA cores)
//   solve  : T = (I + L)^-1, L = strict(beta_r Akk) (fp32, blocked substitution)
//            P = Aqk T
//   MMA_wu : [T diag(beta) ; P diag(beta)] [K*Gam | V]
//            -> W = T(beta Gam K), U = T(beta V), Aqk W, Aqk U
//   Q~ = Gam*Q - Aqk W                       (so that O = Q~ S + Aqk U)
//   MMA_1  : [W ; Q~] S_bf16                 -> W S (rows 0-63), Q~ S (64-127)
//   v~ = U - W S ;  O = Q~ S + Aqk U
//   MMA_3  : S <- Gam_C * S + (lam K)^T v~   (accumulated in TMEM)
// The chunk-boundary state (bf16 or fp32) is written for the backward.
#include "kda_chunk.cuh"
#include "kda_ckpt_layout.h"
#include "kda_tma.cuh"

namespace kda {
namespace {

using namespace tc;
using namespace chunk;

// shared-memory map (bytes)
constexpr int OFF_SQ = 0;                       // staging q   CM[64][128]
constexpr int OFF_SK = OFF_SQ + 16384;          // staging k
constexpr int OFF_SG = OFF_SK + 16384;          // staging g
constexpr int OFF_V = OFF_SG + 16384;           // v (operand) CM[64][128]
constexpr int OFF_A3 = OFF_V + 16384;           // [W ; Q~ ; K*Gam] CM[192][128]
constexpr int OFF_KI = OFF_A3 + 49152;          // K*Gi CM[64][128]   | T fp32 | G fp32 (slow)
constexpr int OFF_TP = OFF_KI + 16384;          // [T b ; P b] CM[128][64]    | G fp32 (slow)
constexpr int OFF_KL = OFF_TP + 16384;          // lam*K CM[64][128]
constexpr int OFF_SB = OFF_KL + 16384;          // S bf16 CM[128][128] | Aqk fp32 + Akk fp32
constexpr int OFF_VT = OFF_SB + 32768;          // v~ CM[64][128]      | T, Aqk bf16 [64][64]
constexpr int OFF_BETA = OFF_VT + 16384;        // beta fp32[64]
constexpr int OFF_GC = OFF_BETA + 256;          // Gam_C fp32[128]
constexpr int OFF_BAR = OFF_GC + 512;           // mbarrier + tmem slot
constexpr int OFF_TRI = OFF_BAR + 128;          // [L ; U'] bf16 CM[128][64] (0/1, built once)
constexpr int OFF_GN = OFF_TRI + 16384;         // exp(-G_C) fp32[128] (G_C itself while staged)
constexpr int SMEM_BYTES = OFF_GN + 512;

// Issue the cp.async copies of one chunk's q, k, g (qkg = true) or v into CM tiles.
__device__ __forceinline__ void stage_chunk(unsigned char* sm, const bf16* q, const bf16* k,
                                            const bf16* g, const bf16* v, size_t row0, int rows_valid,
                                            int H, bool qkg) {
  const size_t rstride = static_cast<size_t>(H) * DK;  // elements between tokens
  if (qkg) {
    stage_tile(sm + OFF_SQ, q + row0 * rstride, rows_valid, rstride);
    stage_tile(sm + OFF_SK, k + row0 * rstride, rows_valid, rstride);
    stage_tile(sm + OFF_SG, g + row0 * rstride, rows_valid, rstride);
  } else {
    stage_tile(sm + OFF_V, v + row0 * rstride, rows_valid, rstride);
  }
  cp_async_commit();
}

template <typename To, typename Tc>
__global__ void __launch_bounds__(NT, 1)
fwd_tc_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
              const bf16* __restrict__ g, const bf16* __restrict__ beta,
              const float* __restrict__ s0, To* __restrict__ o, float* __restrict__ s_out,
              Tc* __restrict__ s_ckpt, unsigned char* __restrict__ factors, int T, int H,
              const int* __restrict__ cs, int* __restrict__ err, const __grid_constant__ CUtensorMap tm_q,
              const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_g,
              const __grid_constant__ CUtensorMap tm_v, int use_tma) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* beta_s = reinterpret_cast<float*>(sm + OFF_BETA);
  float* gamC = reinterpret_cast<float*>(sm + OFF_GC);
  float* gneg = reinterpret_cast<float*>(sm + OFF_GN);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  uint64_t* mbar_in = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 16);  // TMA: a chunk's q, k, g, v

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;  // TMEM lane quarter, column half
  // CTA (seq, h) walks the chunks [c_beg, c_end) of batch row b: the whole row,
  // or with packed sequences (cs: chunk offsets, B = 1) the sequence's range
  const int n_chunks = (T + C - 1) / C;
  const int h = blockIdx.x % H;
  const int seq = cs ? longest_first(cs, gridDim.x / H, blockIdx.x / H, n_chunks, reinterpret_cast<int*>(sm + OFF_SQ))
                     : blockIdx.x / H;
  const int b = cs ? 0 : seq;
  // (clamped: a malformed table cannot take a chunk outside the tensors)
  const int c_beg = cs ? min(max(cs[seq], 0), n_chunks) : 0;
  const int c_end = cs ? min(max(cs[seq + 1], c_beg), n_chunks) : n_chunks;
  const size_t tok0 = static_cast<size_t>(b) * T;   // first token row of batch row b
  const size_t head_off = static_cast<size_t>(h) * DK;
  const bf16* qh = q + head_off;
  const bf16* kh = k + head_off;
  const bf16* gh = g + head_off;
  const bf16* vh = v + static_cast<size_t>(h) * DV;

  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_init(mbar_in, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  // Staging of chunk cc's q, k, g (qkg) or v: TMA tiles completing on mbar_in
  // (armed for all four tiles with the q, k, g issue), else cp.async.
  auto stage = [&](int cc, bool qkg) {
    if (!use_tma) {
      stage_chunk(sm, qh, kh, gh, vh, tok0 + static_cast<size_t>(cc) * C, min(C, T - cc * C), H, qkg);
      return;
    }
    if (tid != kIoThread) return;
    fence_async_smem();
    if (qkg) {
      mbar_expect_tx(mbar_in, 4 * 16384);
      tma_tile(sm + OFF_SQ, &tm_q, h, cc, b, mbar_in);
      tma_tile(sm + OFF_SK, &tm_k, h, cc, b, mbar_in);
      tma_tile(sm + OFF_SG, &tm_g, h, cc, b, mbar_in);
    } else {
      tma_tile(sm + OFF_V, &tm_v, h, cc, b, mbar_in);
    }
  };
  __syncthreads();  // mbar_in initialised
  const bool any = c_beg < c_end;
  if (any) {
    stage(c_beg, true);
    stage(c_beg, false);
  }
  // raw bf16 beta of the chunk to come, loaded one chunk ahead
  const size_t t_beg = static_cast<size_t>(c_beg) * C;
  unsigned short beta_nx = ld_bf16_raw(beta + (tok0 + t_beg + tid) * H + h, any && tid < min(C, T - static_cast<int>(t_beg)));
  bool in_pending = use_tma != 0 && any;  // TMA loads issued and not yet waited, for chunk parity in_par
  uint32_t in_par = 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t t_lane = static_cast<uint32_t>(32 * qw) << 16;
  const uint32_t T_D = tbase;          // cols [0, 256): MMA results
  const uint32_t T_S = tbase + 256;    // cols [256, 384): the state
  const uint32_t T_P = tbase + 384;    // cols [384, 448): P = Aqk T
  uint32_t phase = 0;
  bool failed = false;

  // S0 -> TMEM (row d = lane, 64 columns per warp)
  {
    const int d = 32 * qw + lane;
    const size_t sb = ((static_cast<size_t>(seq) * H + h) * DK + d) * DV;
    for (int half = 0; half < 2; ++half) {
      float vals[32];
      const int c0 = hh * 64 + half * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) vals[j] = s0 ? s0[sb + c0 + j] : 0.f;
      tmem_st32(T_S + t_lane + c0, vals);
    }
    tmem_wait_st();
  }

  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };

  unsigned char* A3 = sm + OFF_A3;
  const uint32_t a3_addr = smem_u32(A3);
  // The cumulative-sum operand of the decay prep: rows 0..63 L[i][j] = (j <= i),
  // rows 64..127 U'[i][j] = (j > i - 64), so [L ; U'] g = [G ; G_C - G].
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
    st16(sm + OFF_TRI, cm_off(row, c8, C), make_uint4(w[0], w[1], w[2], w[3]));
  }
  fence_async_smem();
  __syncthreads();

  for (int c = c_beg; c < c_end; ++c) {
    const int t0 = c * C;
    const int rows_valid = min(C, T - t0);
    cp_async_wait<0>();
    if (use_tma) {
      failed |= !mbar_wait(mbar_in, static_cast<uint32_t>(c - c_beg) & 1u);
      in_pending = false;
    }
    if (tid == kIoThread) bulk_wait_read();  // the previous state image in SB has been stored
    if (tid < C) beta_s[tid] = bf16_raw_to_float(beta_nx);
    if (c + 1 < c_end)
      beta_nx = ld_bf16_raw(beta + (tok0 + t0 + C + tid) * H + h, tid < min(C, T - t0 - C));
    if (__syncthreads_or(failed)) break;

    // ---------------- prep: G, exponentials, operand tiles ----------------
    float* Aq = reinterpret_cast<float*>(sm + OFF_SB);
    float* Akk = Aq + 4096;
    // the factor block of this chunk-head in the checkpoint (null when not training)
    unsigned char* fu = factors ? factors + ((static_cast<size_t>(b) * H + h) * n_chunks + c) * FAC_UNIT
                                : nullptr;
    // prep's operand images (Q Gam, K Gam, K Gam^-1, lam K) and Gam_C go to the
    // checkpoint with bulk copies; their shared sources stay untouched until the
    // solve (KI) and E2 (Q Gam), before which the copies are waited for
    // (two bulk groups: K Gam^-1 alone, which the solve overwrites first, then the rest)
    auto store_prep = [&](bool slow_chunk) {
      if (!fu) return;
      if (!slow_chunk) bulk_store(fu + FAC_KI, sm + OFF_KI, 16384);
      bulk_commit();
      bulk_store(fu + FAC_QG, A3 + cm_off(64, 0, DK), 2 * 16384);  // Q Gam, K Gam (adjacent)
      bulk_store(fu + FAC_KL, sm + OFF_KL, 16384);
      bulk_store(fu + FAC_GC, gamC, 512);
      bulk_commit();
      *reinterpret_cast<uint32_t*>(fu + FAC_FLAG) = slow_chunk ? 1u : 0u;
    };
    {
      // ---- decay prep.  [G ; G_C - G] = [L ; U'] g on the tensor core (exact
      // sums of the bf16 log-decays in fp32), then each thread takes TMEM lane R
      // (token R % 64) and 64 channels: rows R < 64 give Q Gam, K Gam (Gam =
      // exp(G)); rows R >= 64 give lam K = K exp(G_C - G) and K Gam^-1 = lam K
      // exp(-G_C).  Row 63 of G is G_C, which decides the path (kExpBudget).
      if (tid == 0) {
        tc_fence_after();
        const uint32_t tri = smem_u32(sm + OFF_TRI), gt = smem_u32(sm + OFF_SG);
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
        for (int half = 0; half < 2; ++half) {  // whole-warp TMEM loads
          float gv[32];
          tmem_ld32(T_D + t_lane + hh * 64 + 32 * half, gv);
          tmem_wait_ld();
          if (lane == 31) {
#pragma unroll
            for (int j = 0; j < 32; ++j) gneg[hh * 64 + 32 * half + j] = gv[j];
          }
        }
        __syncwarp();  // then Gam_C and exp(-G_C), two channels per lane
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
      float* Gf = reinterpret_cast<float*>(sm + OFF_KI);  // exact path: G fp32 [64][128] across KI|TP
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
            unpack_bf16x8(ld16(sm + OFF_SQ, off), qv);
            unpack_bf16x8(ld16(sm + OFF_SK, off), kv);
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
            unpack_bf16x8(ld16(sm + OFF_SK, off), kv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              kl[e] = kv[e] * __expf(slow ? fminf(gv[j + e], 0.f) : gv[j + e]);
              ki[e] = kl[e] * gneg[c32 + j + e];
            }
            st16(sm + OFF_KL, off, pack_bf16x8(kl));
            if (!slow) st16(sm + OFF_KI, off, pack_bf16x8(ki));
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
                     desc_kmajor(smem_u32(sm + OFF_KI) + ks * 256, DK), idesc, ks > 0);
          mma_commit(mbar);
        }
        if (tid == kIoThread) store_prep(false);
        // prefetch the next chunk's q, k, g (staging is free)
        if (c + 1 < c_end) {
          stage(c + 1, true);
          in_pending = use_tma != 0;
          in_par = static_cast<uint32_t>(c + 1 - c_beg) & 1u;
        }
        failed |= !mma_wait();
        if (__syncthreads_or(failed)) break;
        scores_epilogue(T_D, Aq, Akk);
      } else {
        // past the single anchor's budget: two-half anchors on the tensor cores while
        // each half is within it, else exact scores (16-token block anchors, block
        // pairs on the tensor cores, pairs inside a block exact)
        fence_async_smem();
        __syncthreads();
        if (tid == kIoThread) store_prep(true);
        const bool halves = __syncthreads_or(!halves_within_budget(Gf)) == 0;
        if (halves) {
          unsigned char *bd = A3, *bc = sm + OFF_VT;  // A3 rows 0..63 (W comes later), VT
          scores_halves_prep(sm + OFF_SQ, sm + OFF_SK, bd, bc, Gf);
          tc_fence_before();
          __syncthreads();
          if (tid == 0) {
            tc_fence_after();
            scores_halves_mma(T_D, smem_u32(sm + OFF_SQ), smem_u32(bd), smem_u32(bc));
            mma_commit(mbar);
          }
          failed |= !mma_wait();
          if (__syncthreads_or(failed)) break;
          scores_halves_epilogue(T_D, Aq, Akk);
        } else {
          // kbm_1 (4 KB), kbm_2 (8 KB), kbm_3 (12 KB) in A3 rows 0..63 (W comes later) and VT
          unsigned char *kbm1 = A3 + 12288, *kbm2 = sm + OFF_VT, *kbm3 = A3;
          scores_exact_prep(sm + OFF_SQ, sm + OFF_SK, sm + OFF_SG, kbm1, kbm2, kbm3, Gf, Aq, Akk);
          tc_fence_before();
          __syncthreads();
          if (tid == 0) {
            tc_fence_after();
            scores_exact_mma(T_D, smem_u32(sm + OFF_SQ), smem_u32(kbm1), smem_u32(kbm2), smem_u32(kbm3));
            mma_commit(mbar);
          }
          failed |= !mma_wait();
          if (__syncthreads_or(failed)) break;
          scores_exact_epilogue(T_D, Aq, Akk);
        }
        __syncthreads();
        if (c + 1 < c_end) {
          stage(c + 1, true);
          in_pending = use_tma != 0;
          in_par = static_cast<uint32_t>(c + 1 - c_beg) & 1u;
        }
      }
    }
    // ---------------- solve: T = (I + L)^-1, then P = Aqk T on the tensor cores ----------------
    {
      float* Tm = reinterpret_cast<float*>(sm + OFF_KI);
      if (tid == kIoThread) bulk_wait_read<1>();  // KI has been stored and may be overwritten
      __syncthreads();
      solve_T(Akk, beta_s, Tm, reinterpret_cast<float*>(sm + OFF_VT));
      // eight consecutive threads take eight rows of one column block: conflict-free
      // swizzled fp32 reads and core-matrix bf16 writes
      const int r = 8 * (tid >> 5) + (tid & 7), c0 = 16 * ((tid >> 3) & 3);
      float v[16], a[16], kk[16];
      ld_row16_sw64(Tm, r, c0, v);
      ld_row16_sw64(Aq, r, c0, a);
      if (fu) ld_row16_sw64(Akk, r, c0, kk);
      st16(sm + OFF_VT, cm_off(r, c0, C), pack_bf16x8(v));            // T      (bf16, K x N)
      st16(sm + OFF_VT, cm_off(r, c0 + 8, C), pack_bf16x8(v + 8));
      st16(sm + OFF_VT + 8192, cm_off(r, c0, C), pack_bf16x8(a));     // Aqk    (bf16, M x K)
      st16(sm + OFF_VT + 8192, cm_off(r, c0 + 8, C), pack_bf16x8(a + 8));
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] *= beta_s[c0 + j];
      st16(sm + OFF_TP, cm_off(r, c0, C), pack_bf16x8(v));            // T diag(beta)
      st16(sm + OFF_TP, cm_off(r, c0 + 8, C), pack_bf16x8(v + 8));
      // Akk bf16 for the checkpoint, over the fp32 Aqk just read (SB's first 16 KB)
      __syncthreads();
      if (fu) {
        st16(sm + OFF_SB, cm_off(r, c0, C), pack_bf16x8(kk));
        st16(sm + OFF_SB, cm_off(r, c0 + 8, C), pack_bf16x8(kk + 8));
      }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == kIoThread && fu) {  // T, Aqk (adjacent in VT) and Akk into the checkpoint
      bulk_store(fu + FAC_T, sm + OFF_VT, 16384);
      bulk_store(fu + FAC_AK, sm + OFF_SB, 8192);
      bulk_commit();
    }
    if (tid == 0) {  // P = Aqk T   (M = 64: row r at lane 32(r/16) + r%16)
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(64, 64, false, true);
      const uint32_t tb = smem_u32(sm + OFF_VT), aqb = smem_u32(sm + OFF_VT + 8192);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_P, desc_kmajor(aqb + ks * 256, C), desc_mnmajor(tb + ks * 2048, C), idesc, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // P diag(beta) -> rows 64..127 of the [T b ; P b] operand
      float vals[32];
      tmem_ld32(T_P + t_lane + hh * 32, vals);
      tmem_wait_ld();
      if (lane < 16) {
        const int r = 16 * qw + lane;
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] *= beta_s[hh * 32 + j];
#pragma unroll
        for (int j = 0; j < 32; j += 8) st16(sm + OFF_TP, cm_off(64 + r, hh * 32 + j, C), pack_bf16x8(vals + j));
      }
    }
    fence_async_smem();
    __syncthreads();
    // ---------------- MMA_wu: [Tb ; Pb] [K*Gam | V] ----------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 128, false, true);
      const uint32_t tp = smem_u32(sm + OFF_TP);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        const uint64_t ad = desc_kmajor(tp + ks * 256, C);
        mma_bf16(T_D, ad, desc_mnmajor(a3_addr + 128 * 256 + ks * 4096, DK), idesc, ks > 0);
        mma_bf16(T_D + 128, ad, desc_mnmajor(smem_u32(sm + OFF_V) + ks * 4096, DV), idesc, ks > 0);
      }
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (tid == kIoThread) bulk_wait_read();  // Q Gam has been stored: E2 overwrites it with Q~
    if (__syncthreads_or(failed)) break;
    if (c + 1 < c_end) stage(c + 1, false);
    // ---------------- E2: W -> A3[0:64), Q~ = Gam Q - Aqk W -> A3[64:128) ----------------
    {
      const int R = 32 * qw + lane;
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float vals[32];
        tmem_ld32(T_D + t_lane + c0, vals);
        tmem_wait_ld();
        if (R < 64) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) st16(A3, cm_off(R, c0 + j, DK), pack_bf16x8(vals + j));
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float qg[8];
            const uint32_t off = cm_off(R, c0 + j, DK);  // rows 64..127 of A3 hold Gam*Q
            unpack_bf16x8(ld16(A3, off), qg);
#pragma unroll
            for (int e = 0; e < 8; ++e) qg[e] -= vals[j + e];
            st16(A3, off, pack_bf16x8(qg));
          }
        }
      }
    }
    // ---------------- S pass: S_c -> bf16 operand (+ checkpoint), S *= Gam_C ----------------
    // A bf16 checkpoint entry is the operand image itself, stored below with one
    // bulk copy; an fp32 checkpoint is written row-major here.
    Tc* ck_unit = s_ckpt ? s_ckpt + ((static_cast<size_t>(b) * H + h) * n_chunks + c) * (DK * DV) : nullptr;
    {
      const int d = 32 * qw + lane;
      const float gcd = gamC[d];
      Tc* ck = (sizeof(Tc) == 4 && ck_unit) ? ck_unit + d * DV : nullptr;
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float vals[32];
        tmem_ld32(T_S + t_lane + c0, vals);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 8) st16(sm + OFF_SB, cm_off(d, c0 + j, DV), pack_bf16x8(vals + j));
        if (ck) store_row32<Tc>(ck + c0, vals);
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] *= gcd;
        tmem_st32(T_S + t_lane + c0, vals);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------- MMA_1: [W ; Q~] S ----------------
    if (tid == kIoThread && ((sizeof(Tc) == 2 && ck_unit) || fu)) {
      if (sizeof(Tc) == 2 && ck_unit) bulk_store(ck_unit, sm + OFF_SB, DK * DV * 2);
      if (fu) bulk_store(fu + FAC_W, A3, 16384);  // W (E2 wrote it to A3 rows 0..63)
      bulk_commit();
    }
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 128, false, true);
      const uint32_t sb = smem_u32(sm + OFF_SB);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks)
        mma_bf16(T_D, desc_kmajor(a3_addr + ks * 256, DK), desc_mnmajor(sb + ks * 4096, DV), idesc, ks > 0);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    // ---------------- E3: v~ = U - W S -> bf16 ; O = Q~ S + Aqk U -> global ----------------
    {
      const int R = 32 * qw + lane;
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float ws[32], u[32];
        tmem_ld32(T_D + t_lane + c0, ws);
        tmem_ld32(T_D + t_lane + 128 + c0, u);
        tmem_wait_ld();
        if (R < 64) {
          if (fu) {  // U (bf16 image) into the checkpoint
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              *reinterpret_cast<uint4*>(fu + FAC_U + cm_off(R, c0 + j, DV)) = pack_bf16x8(u + j);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) u[j] -= ws[j];
#pragma unroll
          for (int j = 0; j < 32; j += 8) st16(sm + OFF_VT, cm_off(R, c0 + j, DV), pack_bf16x8(u + j));
        } else {
          const int r = R - 64;
          if (r < rows_valid) {
#pragma unroll
            for (int j = 0; j < 32; ++j) u[j] += ws[j];
            store_row32<To>(o + ((tok0 + t0 + r) * H + h) * DV + c0, u);
          }
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread && fu) {  // v~ (bf16 image) into the checkpoint
      bulk_store(fu + FAC_VT, sm + OFF_VT, 16384);
      bulk_commit();
    }
    // ---------------- MMA_3: S += (lam K)^T v~ ----------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16(128, 128, true, true);
      const uint32_t kl = smem_u32(sm + OFF_KL), vt = smem_u32(sm + OFF_VT);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_S, desc_mnmajor(kl + ks * 4096, DK), desc_mnmajor(vt + ks * 4096, DV), idesc, 1u);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
  }

  if (!failed && s_out) {
    const int d = 32 * qw + lane;
    float* so = s_out + ((static_cast<size_t>(seq) * H + h) * DK + d) * DV;
    for (int half = 0; half < 2; ++half) {
      const int c0 = hh * 64 + half * 32;
      float vals[32];
      tmem_ld32(T_S + t_lane + c0, vals);
      tmem_wait_ld();
      store_row32<float>(so + c0, vals);
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  cp_async_wait<0>();
  // an abandoned chunk may leave tile loads in flight: wait (bounded) for them
  if (in_pending) mbar_wait(mbar_in, in_par);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

__device__ int g_fwd_tc_error = 0;

template <typename To, typename Tc>
int launch_t(const void* q, const void* k, const void* v, const void* g, const void* beta,
             const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
             const int* cs, int n_seqs, cudaStream_t st) {
  static std::atomic<bool> done[64];
  auto kern = fwd_tc_kernel<To, Tc>;
  int rc = ensure_smem(kern, SMEM_BYTES, done);
  if (rc != KDA_OK) return rc;
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_fwd_tc_error) != cudaSuccess) return KDA_ERR_LAUNCH;
  unsigned char* factors = nullptr;
  if (s_ckpt) {  // the per-chunk factors follow the boundary states
    const size_t n = (static_cast<size_t>(T) + C - 1) / C;
    factors = static_cast<unsigned char*>(s_ckpt) + static_cast<size_t>(B) * H * n * DK * DV * sizeof(Tc);
  }
  // TMA tile maps of q, k, g, v; a length or map the encoder refuses falls back
  // to cp.async staging inside the kernel
  CUtensorMap tm[4] = {};
  const void* srcs[4] = {q, k, g, v};
  int use_tma = 1;
  for (int i = 0; i < 4 && use_tma; ++i) use_tma = make_tile_map(&tm[i], srcs[i], B, T, H) ? 1 : 0;
  kern<<<(cs ? n_seqs : B) * H, NT, SMEM_BYTES, st>>>(
      static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
      static_cast<const bf16*>(g), static_cast<const bf16*>(beta), s0, static_cast<To*>(o), s_out,
      static_cast<Tc*>(s_ckpt), factors, T, H, cs, err, tm[0], tm[1], tm[2], tm[3], use_tma);
  return launch_status();
}

}  // namespace

bool tc_fwd_supported(int dk, int dv, int C_, int in_dt) {
  return dk == DK && dv == DV && C_ == C && in_dt == KDA_BF16;
}

int tc_fwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
                  int o_dt, int ck_dt, const int* cs, int n_seqs, cudaStream_t st) {
  if (static_cast<long long>(cs ? n_seqs : B) * H > 0x7fffffffLL) return KDA_ERR_SHAPE;
  if (o_dt == KDA_BF16 && ck_dt == KDA_BF16) return launch_t<bf16, bf16>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, st);
  if (o_dt == KDA_BF16 && ck_dt == KDA_F32) return launch_t<bf16, float>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, st);
  if (o_dt == KDA_F32 && ck_dt == KDA_BF16) return launch_t<float, bf16>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, st);
  if (o_dt == KDA_F32 && ck_dt == KDA_F32) return launch_t<float, float>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, cs, n_seqs, st);
  return KDA_ERR_DTYPE;
}

int tc_fwd_error_flag(int* value, bool clear, cudaStream_t st) {
  static const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(value, g_fwd_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (clear && cudaMemcpyToSymbolAsync(g_fwd_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  return KDA_OK;
}

}  // namespace kda
