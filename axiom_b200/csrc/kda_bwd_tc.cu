// Tensor-core (tcgen05) backward of the chunked KDA core for bf16 inputs,
// dk = dv = 128, chunk C = 64.  The analytic adjoint is the reference's
// (net/kernels/kda_cc_fused_bwd.py:117-239), run as two kernels:
//
// bwd_seq  -- one CTA per (batch, head), chunks in reverse.  Recomputes the
//   chunk-local W, Gam*Q, lam*K and Aqk from the inputs and runs the state
//   cotangent recurrence with dS' (fp32) resident in TMEM:
//     dU^T = dS'^T (lam K)^T + dO^T Aqk                (the cotangent of U = v~)
//     dS   = Gam_C dS' + (Gam Q)^T dO - W^T dU
//   Before each chunk it stores that chunk's incoming dS' (bf16) for bwd_par.
//
// bwd_par  -- persistent over all (batch, head, chunk) units, no sequential
//   dependency.  Recomputes the chunk (scores, T, W, U, v~ = U - W S_c from
//   the forward's checkpoint S_c), then forms every gradient.  All large
//   products are M = 128 MMAs whose results come out transposed (TMEM lane =
//   key/value channel, column = chunk row), so the final reverse cumulative
//   sum that gives dg runs inside one thread per channel:
//     dU^T   = dS'^T (lam K)^T + dO^T Aqk
//     dKL^T  = dS' v~^T                      (cotangent of lam*K)
//     S [dO^T | dU^T]  -> (dO S^T)^T, (dU S^T)^T = -dW^T
//     Yw^T = dW^T T,  Yu^T = dU^T T          (transposed UT-solve adjoints)
//     dAqk = tril(dO v~^T),  dL = -strict(Yu U^T + Yw W^T)       (M = 64)
//     [dQG^T | dKG^T] += KI^T [dAqk ; beta dL]^T,  dKI^T = QG^T dAqk + KG^T beta dL
//   with QG = Gam Q, KG = Gam K, KI = K exp(-G), KL = lam K, then
//     dq = dQG Gam,  dk = dKG Gam + dKI Gi + dKL lam,  dv = beta Yu,
//     dG = dQG QG + dKG KG - dKI KI - dKL KL,  dg = revcumsum(dG) + dG_C,
//     dbeta = rowsum(Yu v) + rowsum(Yw KG) + rowsum(dL Akk).
// Chunks whose decay exceeds the single-anchor budget take the exact
// CUDA-core path for the score products and their adjoints.
#include "kda_chunk.cuh"
#include "kda_tma.cuh"
#include "kda_ckpt_layout.h"

namespace kda {
namespace {

using namespace tc;
using namespace chunk;

__device__ __forceinline__ uint32_t lane_off(int qw) { return static_cast<uint32_t>(32 * qw) << 16; }

// Backward workspace: one dS' (the state cotangent entering the chunk, bf16
// [128][128] as the CM operand image) per (batch, head, chunk) unit, written by
// bwd_seq and read by bwd_par, each with one bulk copy.
constexpr size_t WS_UNIT = 32768;

// ===========================================================================
// bwd_seq
// ===========================================================================
// Chunk c works on operand set p = c & 1 while chunk c-1's set is loaded: the
// forward's W, Q Gam, lam K, Aqk, Gam_C (bulk copies from the checkpoint) and
// dO (TMA tile, or cp.async).  W, Q Gam are adjacent, in the set and in the
// checkpoint.
constexpr int Q_SET = 73728;             // bytes per operand set
constexpr int Q_W = 0, Q_QG = 16384, Q_KL = 32768, Q_DO = 49152, Q_AQ = 65536;  // offsets in a set
constexpr int Q_TP = 2 * Q_SET;          // -dU^T bf16 [128][64]
constexpr int Q_SB = Q_TP + 16384;       // dS' bf16 [128][128] (also stored to the workspace)
constexpr int Q_BETA = Q_SB + 32768;
constexpr int Q_GC0 = Q_BETA + 256, Q_GC1 = Q_GC0 + 512;  // Gam_C per set
constexpr int Q_BAR = Q_GC1 + 512;
constexpr int SEQ_SMEM = Q_BAR + 64;

__global__ void __launch_bounds__(NT, 1)
bwd_seq_kernel(const bf16* __restrict__ beta, const bf16* __restrict__ dout,
               const unsigned char* __restrict__ factors, const float* __restrict__ dsT,
               float* __restrict__ ds0, bf16* __restrict__ dsw, int T, int H, const int* __restrict__ cs,
               int* __restrict__ err, const __grid_constant__ CUtensorMap tm_do, int use_tma) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* beta_s = reinterpret_cast<float*>(sm + Q_BETA);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + Q_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + Q_BAR + 8);
  uint64_t* mbar_ld = reinterpret_cast<uint64_t*>(sm + Q_BAR + 16);  // [2]: one per operand set
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;
  // CTA (seq, h) walks the chunks [c_beg, c_end) of batch row b in reverse: the
  // whole row, or with packed sequences (cs: chunk offsets, B = 1) the sequence's range
  const int n_chunks = (T + C - 1) / C;
  const int h = blockIdx.x % H;
  const int seq = cs ? longest_first(cs, gridDim.x / H, blockIdx.x / H, n_chunks, reinterpret_cast<int*>(sm))
                     : blockIdx.x / H;
  const int b = cs ? 0 : seq;
  const int c_beg = cs ? min(max(cs[seq], 0), n_chunks) : 0;  // clamped like the forward's
  const int c_end = cs ? min(max(cs[seq + 1], c_beg), n_chunks) : n_chunks;
  const size_t tok0 = static_cast<size_t>(b) * T;
  const size_t rstride = static_cast<size_t>(H) * DK;
  const bf16* doh = dout + static_cast<size_t>(h) * DV;
  const size_t unit = static_cast<size_t>(b) * H + h;   // checkpoint row
  const size_t sunit = static_cast<size_t>(seq) * H + h;  // state (dS_T, dS_0) row
  auto set_gc = [](int ps) { return ps ? Q_GC1 : Q_GC0; };
  uint32_t ld_par = 0u, ld_pending = 0u;  // bit ps: phase parity / loads in flight of set ps

  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_init(mbar_ld, 1);
    mbar_init(mbar_ld + 1, 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(tslot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Issues every load of chunk cc into its operand set (after the set's last
  // reader has finished); the beta of chunk cc goes to a register.
  unsigned short beta_nx = 0;  // raw bf16 of the next chunk's beta (prefetch)
  auto issue_chunk = [&](int cc) {
    const int ps = cc & 1, t0 = cc * C, rv = min(C, T - t0);
    unsigned char* set = sm + ps * Q_SET;
    if (!use_tma) {
      stage_tile(set + Q_DO, doh + (tok0 + t0) * rstride, rv, rstride);
      cp_async_commit();
    }
    if (tid == kIoThread) {
      const unsigned char* fu = factors + (unit * n_chunks + cc) * FAC_UNIT;
      fence_async_smem();
      mbar_expect_tx(mbar_ld + ps, 32768 + 16384 + 8192 + 512 + (use_tma ? 16384 : 0));
      bulk_load(set + Q_W, fu + FAC_W, 32768, mbar_ld + ps);  // W, Q Gam
      bulk_load(set + Q_KL, fu + FAC_KL, 16384, mbar_ld + ps);
      bulk_load(set + Q_AQ, fu + FAC_AQ, 8192, mbar_ld + ps);
      bulk_load(sm + set_gc(ps), fu + FAC_GC, 512, mbar_ld + ps);
      if (use_tma) tma_tile(set + Q_DO, &tm_do, h, cc, b, mbar_ld + ps);
    }
    ld_pending |= 1u << ps;
    beta_nx = ld_bf16_raw(beta + (tok0 + t0 + tid) * H + h, tid < rv);
  };
  if (c_beg < c_end) issue_chunk(c_end - 1);
  const uint32_t tbase = *tslot;
  const uint32_t T_DS = tbase, T_U = tbase + 384;
  const uint32_t tl = lane_off(qw);
  uint32_t phase = 0;
  bool failed = false;
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };
  {  // dS_T -> TMEM
    const int d = 32 * qw + lane;
    for (int half = 0; half < 2; ++half) {
      const int c0 = hh * 64 + half * 32;
      float vals[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) vals[j] = dsT ? dsT[(sunit * DK + d) * DV + c0 + j] : 0.f;
      tmem_st32(T_DS + tl + c0, vals);
    }
    tmem_wait_st();
  }

  for (int c = c_end - 1; c >= c_beg; --c) {
    const int p = c & 1;
    cp_async_wait<0>();
    failed |= !mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
    ld_par ^= 1u << p;
    ld_pending &= ~(1u << p);
    if (tid == kIoThread) bulk_wait_read();  // SB may be rewritten: the previous dS' image is stored
    if (tid < C) beta_s[tid] = bf16_raw_to_float(beta_nx);
    if (__syncthreads_or(failed)) break;
    const float* gamC = reinterpret_cast<const float*>(sm + set_gc(p));
    const uint32_t set = smem_u32(sm + p * Q_SET);
    if (c > c_beg) issue_chunk(c - 1);  // the other set was last read by chunk c + 1
    {  // dS' pass: bf16 operand (stored to the workspace below), then dS *= Gam_C
      const int d = 32 * qw + lane;
      const float gcd = gamC[d];
      for (int half = 0; half < 2; ++half) {
        const int c0 = hh * 64 + half * 32;
        float vals[32];
        tmem_ld32(T_DS + tl + c0, vals);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 8) st16(sm + Q_SB, cm_off(d, c0 + j, DV), pack_bf16x8(vals + j));
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] *= gcd;
        tmem_st32(T_DS + tl + c0, vals);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {  // the workspace entry of chunk c is the dS' operand image
      bulk_store(reinterpret_cast<unsigned char*>(dsw) + (unit * n_chunks + c) * WS_UNIT, sm + Q_SB,
                 WS_UNIT);
      bulk_commit();
    }
    // dU^T = dS'^T (lam K)^T + dO^T Aqk
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sb = smem_u32(sm + Q_SB), kl = set + Q_KL, dob = set + Q_DO, aqb = set + Q_AQ;
      const uint32_t id1 = idesc_bf16(128, 64, true, false), id2 = idesc_bf16(128, 64, true, true);
#pragma unroll 1
      for (int ks = 0; ks < DK / 16; ++ks)
        mma_bf16(T_U, desc_mnmajor(sb + ks * 4096, DV), desc_kmajor(kl + ks * 256, DK), id1, ks > 0);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_U, desc_mnmajor(dob + ks * 4096, DV), desc_mnmajor(aqb + ks * 2048, C), id2, 1u);
      mma_commit(mbar);
      // filler, independent of dU (runs under the -dU^T epilogue): dS += (Gam Q)^T dO
      const uint32_t qg = set + Q_QG, id3 = idesc_bf16(128, 128, true, true);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_DS, desc_mnmajor(qg + ks * 4096, DK), desc_mnmajor(dob + ks * 4096, DV), id3, 1u);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // -dU^T -> bf16 [j][c] (TP region)
      const int j = 32 * qw + lane;
      float vals[32];
      tmem_ld32(T_U + tl + hh * 32, vals);
      tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) vals[jj] = -vals[jj];
#pragma unroll
      for (int jj = 0; jj < 32; jj += 8) st16(sm + Q_TP, cm_off(j, hh * 32 + jj, C), pack_bf16x8(vals + jj));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // dS += W^T (-dU)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t dut = smem_u32(sm + Q_TP), w = set + Q_W;
      const uint32_t id2 = idesc_bf16(128, 128, true, false);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_DS, desc_mnmajor(w + ks * 4096, DK), desc_kmajor(dut + ks * 256, C), id2, 1u);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
  }
  if (!failed && ds0) {
    const int d = 32 * qw + lane;
    for (int half = 0; half < 2; ++half) {
      const int c0 = hh * 64 + half * 32;
      float vals[32];
      tmem_ld32(T_DS + tl + c0, vals);
      tmem_wait_ld();
      store_row32<float>(ds0 + (sunit * DK + d) * DV + c0, vals);
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  cp_async_wait<0>();
  // a chunk abandoned on a timeout may leave loads in flight: wait (bounded)
  for (int ps = 0; ps < 2; ++ps)
    if ((ld_pending >> ps) & 1u) mbar_wait(mbar_ld + ps, (ld_par >> ps) & 1u);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// ===========================================================================
// bwd_par
// ===========================================================================
// Regions by phase.  Prefetched one unit ahead (during the previous epilogue):
// A3 = [W ; Gam Q ; Gam K], KI, KL, V (U), TP (v~), TB, AQB, AKB, GF.  Loaded at
// unit start: SQ (dO), SK|SG (dS'), SB (S_c).  Epilogue tiles (channel-major,
// then the outputs in place): SQ (g^T -> dg), SK (v^T -> dv), SG (KI^T),
// SB (QG^T -> dq, KG^T -> dk).
constexpr int P_SQ = 0;                  // dO | raw q (exact path) | g^T -> dg
constexpr int P_SK = 16384;              // dS' (lo) | dW^T [128][64] | raw k (exact path) | v^T -> dv
constexpr int P_SG = 32768;              // dS' (hi) | raw g | KI^T [128][64]
constexpr int P_V = 49152;               // U bf16 [64][128] | raw v
constexpr int P_A3 = 65536;              // [W ; Gam Q ; Gam K] (the forward's images)
constexpr int P_KI = P_A3 + 49152;       // K Gi (the forward's image)
constexpr int P_KL = P_KI + 16384;       // lam K | dU^T [128][64] | [dAqk ; beta dL] [128][64]
constexpr int P_SB = P_KL + 16384;       // S_c bf16 [128][128] | Yw^T, Yu^T | QG^T -> dq, KG^T -> dk
constexpr int P_TP = P_SB + 32768;       // v~ bf16 [64][128] | G fp32 (exact path, with TB/AQB)
constexpr int P_TB = P_TP + 16384;       // T bf16 [64][64]
constexpr int P_AQB = P_TB + 8192;       // Aqk bf16
constexpr int P_AKB = P_AQB + 8192;      // Akk bf16
constexpr int P_BETA = P_AKB + 8192;     // beta fp32[64]
constexpr int P_GF = P_BETA + 256;       // [2][544]: Gam_C fp32[128] + exact-path flag, per unit parity
constexpr int P_DGC = P_GF + 2 * 544;    // dGam_C partial fp32[128]
constexpr int P_DB = P_DGC + 512;        // dbeta accum fp32[64]
constexpr int P_XCH = P_DB + 256;        // half-exchange fp32[2][2][128]
constexpr int P_BAR = P_XCH + 2048;
constexpr int P_MMA = P_BAR + 64;         // MMA issue table (MmaOp[N_MMA])
// Issue-table groups (first entry, count).  A group's critical MMAs are
// committed before its filler MMAs: the tensor core runs in issue order, so the
// filler (needed only later) executes while the threads work on the critical
// results, and the next group's commit implies it has completed.
constexpr int G_DU = 0, N_DU = 12;        // dU^T               | filler: dKL^T
constexpr int F_DU = 12, NF_DU = 8;
constexpr int G_SD = 20, N_SD = 8;        // (dU S_c^T)^T       | filler: Yu^T, (dO S_c^T)^T
constexpr int F_SD = 28, NF_SD = 12;
constexpr int G_YW = 40, N_YW = 4;        // Yw^T               | filler: dAqk
constexpr int F_YW = 44, NF_YW = 8;
constexpr int G_DL = 52, N_DL = 16;       // dL
constexpr int G_VII = 68, N_VII = 12;     // [dQG^T | dKG^T] +=, dKI^T
constexpr int N_MMA = 80;
constexpr int P_DBQ = P_MMA + N_MMA * 32;  // dbeta partials per channel quarter fp32[4][64]
constexpr int PAR_SMEM = P_DBQ + 1024;
// the checkpoint's adjacent tiles land with one bulk copy each: [T, Aqk, Akk] in
// TB, AQB, AKB; [Q Gam, K Gam] in A3 rows 64..191; [K Gi, lam K] in KI, KL
static_assert(P_AQB - P_TB == static_cast<int>(FAC_AQ) && P_AKB - P_TB == static_cast<int>(FAC_AK) &&
                  FAC_KG == FAC_QG + 16384 && P_KL - P_KI == static_cast<int>(FAC_KL - FAC_KI),
              "factor staging layout");

// Four channel-major [128][64] CM tiles (rows = channels, cols = tokens) become,
// each in place, two 8 KB halves (channels 0..63, 64..127) of 64 token rows of
// 128 bytes, 16-byte chunk j of row r at position j ^ (r & 7): the SWIZZLE_128B
// image of an output store box (make_out_map), and conflict-free for the
// transposing stmatrix writes.  Every warp loads its core matrices of all four
// tiles into registers, a barrier, then the transposed writes and a proxy fence
// (the tiles are read by TMA next); ends with a barrier.
__device__ __forceinline__ void transpose4_to_rows_inplace(const uint32_t (&tile)[4], int warp, int lane) {
  uint32_t f[4][4][4];
  __syncthreads();  // every tile complete
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * warp + 32 * k + (lane >> 3), row = lane & 7;
      ldmatrix_x4(f[t][k], tile[t] + (((j >> 3) * 8 + (j & 7)) << 7) + (row << 4));
    }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * warp + 32 * k + (lane >> 3), row = lane & 7;
      const int rg = j >> 3, c = 8 * (j & 7) + row;
      stmatrix_x4_trans(tile[t] + ((rg >> 3) << 13) + (c << 7) + (((rg & 7) ^ (c & 7)) << 4), f[t][k]);
    }
  fence_async_smem();
  __syncthreads();
}
// Token rows (transpose4_to_rows_inplace) -> global rows (row r at dst + r*rstride),
// 16 bytes per thread and store, rows >= rows_valid skipped: the path taken when
// the shared memory is not 1024-byte aligned (the swizzle of a TMA store box
// follows the absolute address).
__device__ __forceinline__ void store_rows(bf16* dst, const unsigned char* rows, int rows_valid,
                                           size_t rstride) {
  for (int i = threadIdx.x; i < 64 * 16; i += NT) {
    const int r = i >> 4, j = i & 15;
    if (r < rows_valid)
      *reinterpret_cast<uint4*>(dst + r * rstride + j * 8) =
          ld16(rows, ((j >> 3) << 13) + (r << 7) + (((j & 7) ^ (r & 7)) << 4));
  }
}

// fp32 checkpoint state (row-major) -> bf16 CM operand tile.
__device__ __forceinline__ void stage_ckpt_f32(unsigned char* dst, const float* src) {
  for (int i = threadIdx.x; i < 128 * 16; i += NT) {
    const int r = i >> 4, cg = i & 15;
    const float4 a = *reinterpret_cast<const float4*>(src + r * 128 + cg * 8);
    const float4 bb = *reinterpret_cast<const float4*>(src + r * 128 + cg * 8 + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w};
    st16(dst, cm_off(r, cg * 8, 128), pack_bf16x8(f));
  }
}

template <typename Tc>
__global__ void __launch_bounds__(NT, 1)
bwd_par_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
               const bf16* __restrict__ g, const bf16* __restrict__ beta,
               const Tc* __restrict__ s_ckpt, const unsigned char* __restrict__ factors,
               const bf16* __restrict__ dsw,
               const bf16* __restrict__ dout, bf16* __restrict__ dq, bf16* __restrict__ dk,
               bf16* __restrict__ dv, bf16* __restrict__ dg, bf16* __restrict__ dbeta, int B,
               int T, int H, int* __restrict__ err, const __grid_constant__ CUtensorMap tm_q,
               const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_g,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
               const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
               const __grid_constant__ CUtensorMap tm_dv, const __grid_constant__ CUtensorMap tm_dg,
               int use_tma) {
  extern __shared__ __align__(1024) unsigned char sm[];
  // dq, dk, dv, dg leave as TMA stores of 128-byte-swizzled boxes (issued by the
  // copy thread, drained before the next unit's loads reuse the tiles)
  const bool out_tma = use_tma && (smem_u32(sm) & 1023u) == 0u;
  float* beta_s = reinterpret_cast<float*>(sm + P_BETA);
  float* dgc = reinterpret_cast<float*>(sm + P_DGC);
  float* dbs = reinterpret_cast<float*>(sm + P_DB);
  float* dbq = reinterpret_cast<float*>(sm + P_DBQ);  // one writer per entry: summed in a fixed order
  float* xch = reinterpret_cast<float*>(sm + P_XCH);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + P_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + P_BAR + 8);
  uint64_t* mbar_fac = reinterpret_cast<uint64_t*>(sm + P_BAR + 16);   // T, Aqk, Akk bulk load
  uint64_t* mbar_late = reinterpret_cast<uint64_t*>(sm + P_BAR + 24);  // dO, dS' (first needed)
  uint64_t* mbar_sc = reinterpret_cast<uint64_t*>(sm + P_BAR + 40);    // S_c (needed from G_SD)
  uint64_t* mbar_rs = reinterpret_cast<uint64_t*>(sm + P_BAR + 32);    // restaged tiles (TMA)
  unsigned char* A3 = sm + P_A3;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qw = warp & 3, hh = warp >> 2;
  const int n_chunks = (T + C - 1) / C;
  const long long n_units = static_cast<long long>(B) * H * n_chunks;
  const size_t rstride = static_cast<size_t>(H) * DK;

  if (tid == 0) {
    mbar_init(mbar, 1);
    mbar_init(mbar_fac, 1);
    mbar_init(mbar_late, 1);
    mbar_init(mbar_sc, 1);
    mbar_init(mbar_rs, 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(tslot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // TMEM columns
  const uint32_t T_IV = tbase;            // [0,128): (dO S^T)^T, dKG^T
  const uint32_t T_UF = tbase + 128;      // [128,256): Yw^T, Yu^T
  const uint32_t T_SC = tbase + 256;      // [256,320): dAqk | dKI^T
  const uint32_t T_L = tbase + 320;       // [320,384): dL (negated)
  const uint32_t T_DU = tbase + 384;      // [384,448): dU^T
  const uint32_t T_KL = tbase + 448;      // [448,512): dKL^T
  const uint32_t tl = lane_off(qw);
  uint32_t phase = 0;
  bool failed = false;
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };
  const uint32_t a3 = smem_u32(A3);

  // The MMA issue table: every descriptor of the unit loop is fixed for the
  // kernel's lifetime.  Only thread 0 builds and reads it.
  MmaOp* tab = reinterpret_cast<MmaOp*>(sm + P_MMA);
  if (tid == 0) {
    const uint32_t tp = smem_u32(sm + P_TP), vb = smem_u32(sm + P_V), sb = smem_u32(sm + P_SB);
    const uint32_t dsp = smem_u32(sm + P_SK), kl = smem_u32(sm + P_KL), dob = smem_u32(sm + P_SQ);
    const uint32_t aqb = smem_u32(sm + P_AQB), tb = smem_u32(sm + P_TB), ki = smem_u32(sm + P_KI);
    int n = G_DU;
    // G_DU: dU^T = dS'^T (lam K)^T + dO^T Aqk | F_DU: dKL^T = dS' v~^T
    for (int ks = 0; ks < DK / 16; ++ks)
      mma_op(tab, n++, T_DU, desc_mnmajor(dsp + ks * 4096, DV), desc_kmajor(kl + ks * 256, DK),
             idesc_bf16(128, 64, true, false), ks > 0);
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_DU, desc_mnmajor(dob + ks * 4096, DV), desc_mnmajor(aqb + ks * 2048, C),
             idesc_bf16(128, 64, true, true), 1u);
    for (int ks = 0; ks < DV / 16; ++ks)
      mma_op(tab, n++, T_KL, desc_kmajor(dsp + ks * 256, DV), desc_kmajor(tp + ks * 256, DV),
             idesc_bf16(128, 64, false, false), ks > 0);
    // G_SD: (dU S_c^T)^T = S_c dU^T | F_SD: Yu^T = dU^T T, (dO S_c^T)^T = S_c dO^T
    for (int ks = 0; ks < DV / 16; ++ks)
      mma_op(tab, n++, T_IV + 64, desc_kmajor(sb + ks * 256, DV), desc_mnmajor(kl + ks * 2048, C),
             idesc_bf16(128, 64, false, true), ks > 0);
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_UF + 64, desc_kmajor(kl + ks * 256, C), desc_mnmajor(tb + ks * 2048, C),
             idesc_bf16(128, 64, false, true), ks > 0);
    for (int ks = 0; ks < DV / 16; ++ks)
      mma_op(tab, n++, T_IV, desc_kmajor(sb + ks * 256, DV), desc_kmajor(dob + ks * 256, DV),
             idesc_bf16(128, 64, false, false), ks > 0);
    // G_YW: Yw^T = dW^T T | F_YW: dAqk = dO v~^T   (M = 64)
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_UF, desc_kmajor(dsp + ks * 256, C), desc_mnmajor(tb + ks * 2048, C),
             idesc_bf16(128, 64, false, true), ks > 0);
    for (int ks = 0; ks < DV / 16; ++ks)
      mma_op(tab, n++, T_SC, desc_kmajor(dob + ks * 256, DV), desc_kmajor(tp + ks * 256, DV),
             idesc_bf16(64, 64, false, false), ks > 0);
    // G_DL: dL~ = Yu U^T + Yw W^T   (M = 64)
    for (int ks = 0; ks < DV / 16; ++ks)
      mma_op(tab, n++, T_L, desc_mnmajor(sb + 16384 + ks * 2048, C), desc_kmajor(vb + ks * 256, DV),
             idesc_bf16(64, 64, true, false), ks > 0);
    for (int ks = 0; ks < DK / 16; ++ks)
      mma_op(tab, n++, T_L, desc_mnmajor(sb + ks * 2048, C), desc_kmajor(a3 + ks * 256, DK),
             idesc_bf16(64, 64, true, false), 1u);
    // [dQG^T | dKG^T] += KI^T [dAqk ; beta dL]^T ;  dKI^T = QG^T dAqk + KG^T (beta dL)
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_IV, desc_mnmajor(ki + ks * 4096, DK), desc_kmajor(kl + ks * 256, C),
             idesc_bf16(128, 128, true, false), 1u);
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_SC, desc_mnmajor(a3 + 64 * 256 + ks * 4096, DK), desc_mnmajor(kl + ks * 2048, C),
             idesc_bf16(128, 64, true, true), ks > 0);
    for (int ks = 0; ks < C / 16; ++ks)
      mma_op(tab, n++, T_SC, desc_mnmajor(a3 + 128 * 256 + ks * 4096, DK),
             desc_mnmajor(kl + 8192 + ks * 2048, C), idesc_bf16(128, 64, true, true), 1u);
  }

  // A unit's inputs are the forward's operand images (T, Aqk, Akk; Q Gam, K Gam;
  // K Gi, lam K; Gam_C and the exact-path flag: bulk copies from the checkpoint)
  // and v (TMA tile when use_tma, else one cp.async group of all threads).  They
  // are issued one unit ahead, during the previous unit's epilogue, and complete
  // on mbar_fac.  Every asynchronous phase is waited before the CTA exits.
  int it = 0;                                      // units processed by this CTA
  bool fac_pending = false, late_pending = false, sc_pending = false, rs_pending = false;  // issued, not waited
  uint32_t fac_par = 0, late_par = 0, sc_par = 0, rs_par = 0;
  auto issue_inputs = [&](long long uu, unsigned short& beta_nx) {
    const int cc = static_cast<int>(uu % n_chunks);
    const long long bhn = uu / n_chunks;
    const int hn = static_cast<int>(bhn % H), bn = static_cast<int>(bhn / H);
    const int rv = min(C, T - cc * C);
    const size_t tk = static_cast<size_t>(bn) * T + static_cast<size_t>(cc) * C;
    if (tid == kIoThread) {
      const unsigned char* fu = factors + ((static_cast<size_t>(bn) * H + hn) * n_chunks + cc) * FAC_UNIT;
      const int gf = P_GF + 544 * ((uu == blockIdx.x ? it : it + 1) & 1);
      fence_async_smem();
      mbar_expect_tx(mbar_fac, 24576 + 32768 + 32768 + 3 * 16384 + FAC_GF_BYTES);
      bulk_load(sm + P_TB, fu + FAC_T, 24576, mbar_fac);                  // T, Aqk, Akk
      bulk_load(A3 + cm_off(64, 0, DK), fu + FAC_QG, 32768, mbar_fac);    // Q Gam, K Gam
      bulk_load(sm + P_KI, fu + FAC_KI, 32768, mbar_fac);                 // K Gi, lam K
      bulk_load(A3, fu + FAC_W, 16384, mbar_fac);                         // W
      bulk_load(sm + P_V, fu + FAC_U, 16384, mbar_fac);                   // U
      bulk_load(sm + P_TP, fu + FAC_VT, 16384, mbar_fac);                 // v~
      bulk_load(sm + gf, fu + FAC_GC, FAC_GF_BYTES, mbar_fac);            // Gam_C, flag
    }
    fac_pending = true;
    fac_par = static_cast<uint32_t>(uu == blockIdx.x ? it : it + 1) & 1u;
    beta_nx = ld_bf16_raw(beta + (tk + tid) * H + hn, tid < rv);
  };
  unsigned short beta_nx = 0;  // raw bf16 of the next unit's beta (prefetch)
  if (blockIdx.x < n_units) issue_inputs(blockIdx.x, beta_nx);

  for (long long u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int c = static_cast<int>(u % n_chunks);
    const long long bh = u / n_chunks;
    const int h = static_cast<int>(bh % H), b = static_cast<int>(bh / H);
    const int t0 = c * C, rows_valid = min(C, T - t0);
    const size_t tok0 = static_cast<size_t>(b) * T + t0;
    const size_t hoff = static_cast<size_t>(h) * DK;
    const size_t unit_sq = (static_cast<size_t>(b) * H + h) * n_chunks + c;  // chunk index
    const long long u_next = u + gridDim.x;
    bool prefetched = false;

    // dO, dS' and S_c (bf16 checkpoint: the operand image) land while T beta and
    // the W, U MMAs run
    if (!use_tma) {
      stage_tile(sm + P_SQ, dout + hoff + tok0 * rstride, rows_valid, rstride);
      cp_async_commit();
    }
    if (tid == kIoThread) {  // in the order they are needed: dO, dS' (dU group), then S_c
      if (out_tma) bulk_wait_read();  // the previous unit's output stores read SQ, SK, SB
      fence_async_smem();
      mbar_expect_tx(mbar_late, WS_UNIT + (use_tma ? 16384 : 0));
      if (use_tma) tma_tile(sm + P_SQ, &tm_do, h, c, b, mbar_late);
      bulk_load(sm + P_SK, reinterpret_cast<const unsigned char*>(dsw) + unit_sq * WS_UNIT, WS_UNIT, mbar_late);
      if constexpr (sizeof(Tc) == 2) {
        mbar_expect_tx(mbar_sc, DK * DV * 2);
        bulk_load(sm + P_SB, s_ckpt + unit_sq * (DK * DV), DK * DV * 2, mbar_sc);
      }
    }
    late_pending = true;
    late_par = static_cast<uint32_t>(it) & 1u;
    sc_pending = sizeof(Tc) == 2;
    sc_par = static_cast<uint32_t>(it) & 1u;
    if (tid < C) beta_s[tid] = bf16_raw_to_float(beta_nx);
    if (tid < 128) dgc[tid] = 0.f;
    if (tid < 64) dbs[tid] = 0.f;
    cp_async_wait<1>();
    failed |= !mbar_wait(mbar_fac, fac_par);
    fac_pending = false;
    if (__syncthreads_or(failed)) break;

    // ---- the forward's W, U and v~ are resident: straight to the adjoint ----
    const float* gamC = reinterpret_cast<const float*>(sm + P_GF + 544 * (it & 1));
    const bool slow = (reinterpret_cast<const uint32_t*>(gamC)[128] & 1u) != 0u;  // exact-path chunk (bit 0)
    if constexpr (sizeof(Tc) == 4) stage_ckpt_f32(sm + P_SB, s_ckpt + unit_sq * (DK * DV));
    cp_async_wait<0>();
    failed |= !mbar_wait(mbar_late, late_par);
    late_pending = false;
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(failed)) break;
    // dU^T = dS'^T (lam K)^T + dO^T Aqk ;  dKL^T = dS' v~^T
    if (tid == 0) {
      tc_fence_after();
      mma_run(tab, G_DU, N_DU);
      mma_commit(mbar);
      mma_run(tab, F_DU, NF_DU);
    }

    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // dU^T -> bf16 [j][c] (KL region)
      const int j = 32 * qw + lane;
      float vals[32];
      tmem_ld32(T_DU + tl + hh * 32, vals);
      tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; jj += 8) st16(sm + P_KL, cm_off(j, hh * 32 + jj, C), pack_bf16x8(vals + jj));
    }
    if constexpr (sizeof(Tc) == 2) {
      failed |= !mbar_wait(mbar_sc, sc_par);
      sc_pending = false;
    }
    fence_async_smem();
    tc_fence_before();
    if (__syncthreads_or(failed)) break;
    // S_c [dO^T | dU^T] -> (dO S^T)^T | (dU S^T)^T
    if (tid == 0) {
      tc_fence_after();
      mma_run(tab, G_SD, N_SD);
      mma_commit(mbar);
      mma_run(tab, F_SD, NF_SD);
    }
    {  // dGam_C partial sums: sum_j S_c[d][j] dS'[d][j]  (under the S_c MMAs; both only read);
       // eight consecutive threads read eight rows of one core matrix (conflict-free)
      const int d = tid & 127, j0 = (tid >> 7) * 64;
      float acc = 0.f;
      for (int j = j0; j < j0 + 64; j += 8) {
        float a[8], bb[8];
        unpack_bf16x8(ld16(sm + P_SB, cm_off(d, j, DV)), a);
        unpack_bf16x8(ld16(sm + P_SK, cm_off(d, j, DV)), bb);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc += a[e] * bb[e];
      }
      atomicAdd(&dgc[d], acc);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    // dS' is dead (its last reader, the dKL^T filler, is done): restage g
    // (for the epilogue) over its upper half
    if (use_tma) {
      if (tid == kIoThread) {
        fence_async_smem();
        mbar_expect_tx(mbar_rs, slow ? 4 * 16384 : 2 * 16384);  // + v (and q, k) below
        tma_tile(sm + P_SG, &tm_g, h, c, b, mbar_rs);
      }
      rs_pending = true;
      rs_par = static_cast<uint32_t>(it) & 1u;
    } else {
      stage_tile(sm + P_SG, g + hoff + tok0 * rstride, rows_valid, rstride);
      cp_async_commit();
    }
    {  // dW^T = -(dU S^T)^T -> bf16 [d][c] (SK region)
      const int d = 32 * qw + lane;
      float vals[32];
      tmem_ld32(T_IV + 64 + tl + hh * 32, vals);
      tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) vals[jj] = -vals[jj];
#pragma unroll
      for (int jj = 0; jj < 32; jj += 8) st16(sm + P_SK, cm_off(d, hh * 32 + jj, C), pack_bf16x8(vals + jj));
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // Yw^T = dW^T T,  Yu^T = dU^T T
    if (tid == 0) {
      tc_fence_after();
      mma_run(tab, G_YW, N_YW);
      mma_commit(mbar);
      mma_run(tab, F_YW, NF_YW);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // Yw^T, Yu^T -> bf16 (SB region); beta_c Yw^T -> TMEM [64,128)
      const int d = 32 * qw + lane;
      float yw[32], yu[32];
      tmem_ld32(T_UF + tl + hh * 32, yw);
      tmem_ld32(T_UF + 64 + tl + hh * 32, yu);
      tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; jj += 8) {
        st16(sm + P_SB, cm_off(d, hh * 32 + jj, C), pack_bf16x8(yw + jj));
        st16(sm + P_SB + 16384, cm_off(d, hh * 32 + jj, C), pack_bf16x8(yu + jj));
      }
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) yw[jj] *= beta_s[hh * 32 + jj];
      tmem_st32(T_IV + 64 + tl + hh * 32, yw);
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // dAqk = dO v~^T, dL~ = Yu U^T + Yw W^T   (M = 64)
    if (tid == 0) {
      tc_fence_after();
      mma_run(tab, G_DL, N_DL);
      mma_commit(mbar);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    // U, dO and dW^T are dead: restage v (and raw q, k for the exact path)
    if (use_tma) {
      if (tid == kIoThread) {
        fence_async_smem();
        tma_tile(sm + P_V, &tm_v, h, c, b, mbar_rs);
        if (slow) {
          tma_tile(sm + P_SQ, &tm_q, h, c, b, mbar_rs);
          tma_tile(sm + P_SK, &tm_k, h, c, b, mbar_rs);
        }
      }
    } else {
      stage_tile(sm + P_V, v + hoff + tok0 * rstride, rows_valid, rstride);
      if (slow) {
        stage_tile(sm + P_SQ, q + hoff + tok0 * rstride, rows_valid, rstride);
        stage_tile(sm + P_SK, k + hoff + tok0 * rstride, rows_valid, rstride);
      }
      cp_async_commit();
    }
    {  // [dAqk ; beta dL] -> bf16 [128][64] (KL region); dbeta += rowsum(dL * Akk)
      const int r = 16 * qw + lane;
      float da[32], dl[32];
      tmem_ld32(T_SC + tl + hh * 32, da);
      tmem_ld32(T_L + tl + hh * 32, dl);
      tmem_wait_ld();
      if (lane < 16) {
        const float br = beta_s[r];
        float part = 0.f;
        float akk[32];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 8) unpack_bf16x8(ld16(sm + P_AKB, cm_off(r, hh * 32 + jj, C)), akk + jj);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int i = hh * 32 + jj;
          da[jj] = (i <= r) ? da[jj] : 0.f;
          const float l = (i < r) ? -dl[jj] : 0.f;
          part += l * akk[jj];
          dl[jj] = br * l;
        }
#pragma unroll
        for (int jj = 0; jj < 32; jj += 8) {
          st16(sm + P_KL, cm_off(r, hh * 32 + jj, C), pack_bf16x8(da + jj));
          st16(sm + P_KL, cm_off(64 + r, hh * 32 + jj, C), pack_bf16x8(dl + jj));
        }
        atomicAdd(&dbs[r], part);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (!slow) {
      // [dQG^T | dKG^T] += KI^T [dAqk ; beta dL]^T ;  dKI^T = QG^T dAqk + KG^T (beta dL)
      if (tid == 0) {
        tc_fence_after();
        mma_run(tab, G_VII, N_VII);
        mma_commit(mbar);
      }
      // channel-major copies for the epilogue: QG, KG -> SB (Yw^T, Yu^T are dead; the
      // MMAs only read QG, KG)
      transpose_cm<64, 128>(smem_u32(sm + P_SB), a3 + 64 * 256, warp, lane, NT / 32);
      transpose_cm<64, 128>(smem_u32(sm + P_SB + 16384), a3 + 128 * 256, warp, lane, NT / 32);
      cp_async_wait<0>();
      if (use_tma) {
        failed |= !mbar_wait(mbar_rs, rs_par);
        rs_pending = false;
      }
      if (__syncthreads_or(failed)) break;
      transpose_cm<64, 128>(smem_u32(sm + P_SQ), smem_u32(sm + P_SG), warp, lane, NT / 32);  // g
      transpose_cm<64, 128>(smem_u32(sm + P_SK), smem_u32(sm + P_V), warp, lane, NT / 32);   // v
      failed |= !mma_wait();
      if (__syncthreads_or(failed)) break;
      transpose_cm<64, 128>(smem_u32(sm + P_SG), smem_u32(sm + P_KI), warp, lane, NT / 32);  // KI
      __syncthreads();
      // A3, KI, KL, V, TP, TB, AQB, AKB and the other Gam_C slot are free: stage the
      // next unit
      if (u_next < n_units) issue_inputs(u_next, beta_nx);
      prefetched = true;
    } else {
      cp_async_wait<0>();
      if (use_tma) {
        failed |= !mbar_wait(mbar_rs, rs_par);
        rs_pending = false;
      }
      if (__syncthreads_or(failed)) break;
    }
    // ---- final epilogue: thread = channel d (lane), columns c in [32 hh, 32 hh + 32) ----
    {
      const int d = 32 * qw + lane;
      const int cb = hh * 32;
      const float gC = gamC[d];
      float dG[32];
      float klsum = 0.f;
      const size_t gbase = hoff + tok0 * rstride + d;
      if (!slow) {
        // channel-major tiles: g (SQ), v (SK), QG (SB), KG (SB + 16 KB), KI (SG), each [128][64]
        float gm[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack_bf16x8(ld16(sm + P_SQ, cm_off(d, cb + 8 * j, C)), gm + 8 * j);
        float run = 0.f;
        if (hh) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float t8[8];
            unpack_bf16x8(ld16(sm + P_SQ, cm_off(d, 8 * j, C)), t8);
#pragma unroll
            for (int e = 0; e < 8; ++e) run += t8[e];
          }
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int c8 = cb + 8 * qq;
          float dqg[8], dkg[8], dki[8], dkl[8], yw[8], yu[8], qg[8], kg[8], ki[8], vv[8];
          float oq[8], ok[8], ov[8], tb[8];
          tmem_ld8(T_IV + tl + c8, dqg);
          tmem_ld8(T_IV + 64 + tl + c8, dkg);
          tmem_ld8(T_SC + tl + c8, dki);
          tmem_ld8(T_KL + tl + c8, dkl);
          tmem_ld8(T_UF + tl + c8, yw);
          tmem_ld8(T_UF + 64 + tl + c8, yu);
          unpack_bf16x8(ld16(sm + P_SB, cm_off(d, c8, C)), qg);
          unpack_bf16x8(ld16(sm + P_SB + 16384, cm_off(d, c8, C)), kg);
          unpack_bf16x8(ld16(sm + P_SG, cm_off(d, c8, C)), ki);
          unpack_bf16x8(ld16(sm + P_SK, cm_off(d, c8, C)), vv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int cc = c8 + i;
            run += gm[8 * qq + i];
            const float gam = __expf(run), gi = __expf(-run);
            const float s2 = dki[i] + gC * dkl[i];
            dG[8 * qq + i] = dqg[i] * qg[i] + dkg[i] * kg[i] - s2 * ki[i];
            klsum += gC * dkl[i] * ki[i];
            tb[i] = yw[i] * kg[i] + yu[i] * vv[i];  // dbeta partial of token cc, channel d
            oq[i] = dqg[i] * gam;
            ok[i] = dkg[i] * gam + s2 * gi;
            ov[i] = beta_s[cc] * yu[i];
          }
          {  // dbeta partials: sum over this warp's 32 channels, 4 warps per token
            const float sb = warp_colsum<8>(tb, lane);
            if (lane < 8) dbq[qw * 64 + c8 + lane] = sb;
          }
          if (use_tma) {  // channel-major, over the tiles just read (stored below)
            st16(sm + P_SB, cm_off(d, c8, C), pack_bf16x8(oq));
            st16(sm + P_SB + 16384, cm_off(d, c8, C), pack_bf16x8(ok));
            st16(sm + P_SK, cm_off(d, c8, C), pack_bf16x8(ov));
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int cc = c8 + i;
              if (cc < rows_valid) {
                dq[gbase + cc * rstride] = __float2bfloat16_rn(oq[i]);
                dk[gbase + cc * rstride] = __float2bfloat16_rn(ok[i]);
                dv[gbase + cc * rstride] = __float2bfloat16_rn(ov[i]);
              }
            }
          }
        }
      } else {
        const unsigned char* sgt = sm + P_SG;
        float pre = 0.f, gtot = 0.f;
        for (int cc = 0; cc < C; ++cc) {
          const float x = ldbf(sgt, cm_off(cc, d, DK));
          pre += (cc < cb) ? x : 0.f;
          gtot += x;
        }
        float* Gs = reinterpret_cast<float*>(sm + P_TP);  // exact path: G fp32 [64][128] (gsw layout)
        {
          float run2 = pre;
          for (int jj = 0; jj < 32; ++jj) {
            run2 += ldbf(sgt, cm_off(cb + jj, d, DK));
            Gs[gsw(cb + jj, d)] = run2;
          }
        }
        __syncthreads();
        // Score adjoints with 16-token block anchors (every exponent <= 0).  For
        // token r of block I and i of an earlier block: exp(G_r - G_i) =
        // exp(G_r - G_16I) exp(G_16I - G_i), so the row sums
        //   sum_{i<16I} dAqk[r][i] k_i exp(G_r - G_i)   (and beta dL with k)
        // are exp(G_r - G_16I) times MMAs over kbm_I = k exp(G_16I - G_i); the
        // column sums over later blocks use qa_J, ka_J = (q, k) exp(G_r - G_e)
        // with e = 16J + 15 and the factor exp(G_e - G_c).  Pairs inside one
        // block take exact exponentials below.  Operands: kbm_I (I = 1..3) in
        // SB, qa_J / ka_J (J = 0..2) in A3 (both free in a slow unit's epilogue);
        // sums in the free TMEM columns T_SC, T_L, T_DU.
        unsigned char* kbm = sm + P_SB;
        unsigned char* qa = A3;
        unsigned char* ka = A3 + 24576;
        auto kbm_off = [](int I) { return I == 1 ? 0 : (I == 2 ? 4096 : 12288); };  // 16I rows each
        auto qa_off = [](int J) { return J == 0 ? 0 : (J == 1 ? 12288 : 20480); };   // 48 - 16J rows each
        auto t_row = [&](int I) { return I == 1 ? T_SC : (I == 2 ? T_SC + 32 : T_L); };          // [dra | drk]
        auto t_col = [&](int J) { return J == 0 ? T_L + 32 : (J == 1 ? T_L + 48 : T_DU); };      // dca + dck
        for (int idx = tid; idx < 96 * 16; idx += NT) {
          // eight consecutive threads take the eight rows of one core matrix (conflict-free
          // 16-byte accesses); blocks I, J start on multiples of 8 rows
          const int pr = ((idx >> 7) << 3) + (idx & 7), d8 = ((idx >> 3) & 15) * 8;
          {  // kbm: (I, i) for i < 16 I
            const int I = pr < 16 ? 1 : (pr < 48 ? 2 : 3);
            const int i = pr - (I == 1 ? 0 : (I == 2 ? 16 : 48));
            float kv[8], o[8], ga[8], gb[8];
            unpack_bf16x8(ld16(sm + P_SK, cm_off(i, d8, DK)), kv);
            ld8g(Gs, 16 * I, d8, ga);
            ld8g(Gs, i, d8, gb);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = kv[e] * __expf(fminf(ga[e] - gb[e], 0.f));
            st16(kbm + kbm_off(I), cm_off(i, d8, DK), pack_bf16x8(o));
          }
          {  // qa, ka: (J, r) for r > 16 J + 15
            const int J = pr < 48 ? 0 : (pr < 80 ? 1 : 2);
            const int rr = pr - (J == 0 ? 0 : (J == 1 ? 48 : 80));
            const int r = 16 * (J + 1) + rr;
            float qv[8], kv[8], oq[8], ok[8], ga[8], gb[8];
            unpack_bf16x8(ld16(sm + P_SQ, cm_off(r, d8, DK)), qv);
            unpack_bf16x8(ld16(sm + P_SK, cm_off(r, d8, DK)), kv);
            ld8g(Gs, r, d8, ga);
            ld8g(Gs, 16 * J + 15, d8, gb);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float f = __expf(fminf(ga[e] - gb[e], 0.f));
              oq[e] = qv[e] * f;
              ok[e] = kv[e] * f;
            }
            st16(qa + qa_off(J), cm_off(rr, d8, DK), pack_bf16x8(oq));
            st16(ka + qa_off(J), cm_off(rr, d8, DK), pack_bf16x8(ok));
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
          tc_fence_after();
          const uint32_t kl = smem_u32(sm + P_KL), kb0 = smem_u32(kbm), qa0 = smem_u32(qa), ka0 = smem_u32(ka);
          const uint32_t idr = idesc_bf16(128, 16, true, false), idc = idesc_bf16(128, 16, true, true);
          for (int I = 1; I <= 3; ++I)
            for (int ks = 0; ks < I; ++ks) {
              const uint64_t Ad = desc_mnmajor(kb0 + kbm_off(I) + ks * 4096, DK);
              mma_bf16(t_row(I), Ad, desc_kmajor(kl + 2048 * I + ks * 256, C), idr, ks > 0);
              mma_bf16(t_row(I) + 16, Ad, desc_kmajor(kl + 8192 + 2048 * I + ks * 256, C), idr, ks > 0);
            }
          for (int J = 0; J <= 2; ++J)
            for (int Ip = J + 1; Ip <= 3; ++Ip) {
              const int ks = Ip - J - 1;
              mma_bf16(t_col(J), desc_mnmajor(qa0 + qa_off(J) + ks * 4096, DK),
                       desc_mnmajor(kl + 2048 * Ip + 256 * J, C), idc, ks > 0);
              mma_bf16(t_col(J), desc_mnmajor(ka0 + qa_off(J) + ks * 4096, DK),
                       desc_mnmajor(kl + 8192 + 2048 * Ip + 256 * J, C), idc, 1u);
            }
          mma_commit(mbar);
        }
        failed |= !mma_wait();
        if (__syncthreads_or(failed)) break;
        float* dGs = reinterpret_cast<float*>(sm + P_SB);  // dG fp32 [64][128] (kbm is dead now)
        float run = pre;
#pragma unroll 1
        for (int part = 0; part < 2; ++part) {
          const int c16 = cb + 16 * part;
          const int I = c16 >> 4;  // this part's 16-token block (warp-uniform)
          // score adjoints of this block's tokens: dra / drk (row sums with k over
          // earlier tokens) and dcc (column sums with q, k over later tokens)
          float dra[16], drk[16], dcc[16];
          {  // earlier / later blocks: the MMA sums times their anchor factors
            float offr[16], offk[16], offc[16];
            if (I >= 1) {
              tmem_ld16(t_row(I) + tl, offr);
              tmem_ld16(t_row(I) + 16 + tl, offk);
            }
            if (I <= 2) tmem_ld16(t_col(I) + tl, offc);
            tmem_wait_ld();
            const float g_s = Gs[gsw(c16, d)], g_e = Gs[gsw(c16 + 15, d)];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float gi = Gs[gsw(c16 + i, d)];
              const float ar = __expf(fminf(gi - g_s, 0.f)), bc = __expf(fminf(g_e - gi, 0.f));
              dra[i] = I >= 1 ? ar * offr[i] : 0.f;
              drk[i] = I >= 1 ? ar * offk[i] : 0.f;
              dcc[i] = I <= 2 ? bc * offc[i] : 0.f;
            }
          }
          {  // pairs inside the block (r >= i): exp(G_r - G_i) is the running product of
             // the per-token decays exp(g_t), t = i+1 .. r (each <= 1), shared by row r's
             // sums and column i's sum
            float kd[16], ad[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              kd[j] = ldbf(sm + P_SK, cm_off(c16 + j, d, DK));
              ad[j] = __expf(ldbf(sgt, cm_off(c16 + j, d, DK)));
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) {
              float kla[16], klb[16];  // dAqk[r][16I + i], (beta dL)[r][16I + i]
              unpack_bf16x8(ld16(sm + P_KL, cm_off(c16 + r, c16, C)), kla);
              unpack_bf16x8(ld16(sm + P_KL, cm_off(64 + c16 + r, c16, C)), klb);
              if (r >= 8) {
                unpack_bf16x8(ld16(sm + P_KL, cm_off(c16 + r, c16 + 8, C)), kla + 8);
                unpack_bf16x8(ld16(sm + P_KL, cm_off(64 + c16 + r, c16 + 8, C)), klb + 8);
              }
              const float qr = ldbf(sm + P_SQ, cm_off(c16 + r, d, DK)), kr = kd[r];
              float sa = 0.f, sk = 0.f, e = 1.f;
#pragma unroll
              for (int i = r; i >= 0; --i) {
                if (i < r) e *= ad[i + 1];
                const float ke = kd[i] * e;
                sa = fmaf(kla[i], ke, sa);
                sk = fmaf(klb[i], ke, sk);
                dcc[i] = fmaf(fmaf(kla[i], qr, klb[i] * kr), e, dcc[i]);
              }
              dra[r] += sa;
              drk[r] += sk;
            }
          }
          float dqg[16], dkg[16], dkl[16], yw[16], yu[16], tb[16];
          tmem_ld16(T_IV + tl + c16, dqg);
          tmem_ld16(T_IV + 64 + tl + c16, dkg);
          tmem_ld16(T_KL + tl + c16, dkl);
          tmem_ld16(T_UF + tl + c16, yw);
          tmem_ld16(T_UF + 64 + tl + c16, yu);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int cc = c16 + i;
            run += ldbf(sgt, cm_off(cc, d, DK));
            const float gam = __expf(run);
            const float qv = ldbf(sm + P_SQ, cm_off(cc, d, DK));
            const float kv = ldbf(sm + P_SK, cm_off(cc, d, DK));
            const float lam = __expf(fminf(gtot - run, 0.f));
            const float dqv = dqg[i] * gam + dra[i];
            const float dkv = dkg[i] * gam + dkl[i] * lam + drk[i] + dcc[i];
            dGs[cc * DK + d] = dqg[i] * qv * gam + dkg[i] * kv * gam - dkl[i] * kv * lam + dra[i] * qv +
                               drk[i] * kv - dcc[i] * kv;
            klsum += dkl[i] * kv * lam;
            const float vv = ldbf(sm + P_V, cm_off(cc, d, DV));
            tb[i] = yw[i] * kv * gam + yu[i] * vv;
            if (cc < rows_valid) {
              dq[gbase + cc * rstride] = __float2bfloat16_rn(dqv);
              dk[gbase + cc * rstride] = __float2bfloat16_rn(dkv);
              dv[gbase + cc * rstride] = __float2bfloat16_rn(beta_s[cc] * yu[i]);
            }
          }
          const float sb = warp_colsum<16>(tb, lane);
          if (lane < 16) dbq[qw * 64 + c16 + lane] = sb;
        }
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) dG[jj] = dGs[(cb + jj) * DK + d];
      }
      float gsum = 0.f;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) gsum += dG[jj];
      xch[(0 * 2 + hh) * 128 + d] = gsum;
      xch[(1 * 2 + hh) * 128 + d] = klsum;
      __syncthreads();  // xch
      const float dGC = xch[(1 * 2 + 0) * 128 + d] + xch[(1 * 2 + 1) * 128 + d] + gC * dgc[d];
      float acc = dGC + (hh == 0 ? xch[(0 * 2 + 1) * 128 + d] : 0.f);
      if (use_tma && !slow) {  // dg over g^T (consumed), channel-major
#pragma unroll
        for (int jj = 31; jj >= 0; --jj) {
          acc += dG[jj];
          dG[jj] = acc;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) st16(sm + P_SQ, cm_off(d, cb + 8 * j, C), pack_bf16x8(dG + 8 * j));
      } else {
#pragma unroll
        for (int jj = 31; jj >= 0; --jj) {
          acc += dG[jj];
          const int cc = cb + jj;
          if (cc < rows_valid) dg[gbase + cc * rstride] = __float2bfloat16_rn(acc);
        }
      }
    }
    if (use_tma && !slow) {
      // dq, dk, dv, dg: channel-major tiles -> token rows (swizzled, in place) ->
      // 16-byte stores
      const uint32_t tiles[4] = {smem_u32(sm + P_SB), smem_u32(sm + P_SB + 16384), smem_u32(sm + P_SK),
                                 smem_u32(sm + P_SQ)};
      transpose4_to_rows_inplace(tiles, warp, lane);
      if (out_tma) {
        if (tid == kIoThread) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            tma_out_store(&tm_dq, sm + P_SB + hf * 8192, 64 * hf, h, t0, b);
            tma_out_store(&tm_dk, sm + P_SB + 16384 + hf * 8192, 64 * hf, h, t0, b);
            tma_out_store(&tm_dv, sm + P_SK + hf * 8192, 64 * hf, h, t0, b);
            tma_out_store(&tm_dg, sm + P_SQ + hf * 8192, 64 * hf, h, t0, b);
          }
          bulk_commit();
        }
      } else {
        const size_t obase = hoff + tok0 * rstride;
        store_rows(dq + obase, sm + P_SB, rows_valid, rstride);
        store_rows(dk + obase, sm + P_SB + 16384, rows_valid, rstride);
        store_rows(dv + obase, sm + P_SK, rows_valid, rstride);
        store_rows(dg + obase, sm + P_SQ, rows_valid, rstride);
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid < rows_valid)
      dbeta[(tok0 + tid) * H + h] =
          __float2bfloat16_rn(dbs[tid] + dbq[tid] + dbq[64 + tid] + dbq[128 + tid] + dbq[192 + tid]);
    if (!prefetched && u_next < n_units) issue_inputs(u_next, beta_nx);
    ++it;
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  cp_async_wait<0>();
  // a unit abandoned on a timeout may leave bulk loads in flight: wait (bounded)
  // for them before the shared memory is released
  if (fac_pending) mbar_wait(mbar_fac, fac_par);
  if (late_pending) mbar_wait(mbar_late, late_par);
  if (sc_pending) mbar_wait(mbar_sc, sc_par);
  if (rs_pending) mbar_wait(mbar_rs, rs_par);
  if (tid == kIoThread) bulk_wait_all();  // output stores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// ===========================================================================
// bwd_seq, column-sliced (fewer (sequence, head) pairs than SMs)
// ===========================================================================
// The same reverse recurrence on a slice dS'_s = dS'[:, col0 + DVS) of the
// state cotangent: the columns never mix (lam K, Aqk, Gam Q and W act on the
// rows), so 2 to 8 CTAs walk one head's chunks side by side.  Per chunk, in the
// untransposed form (M = 64 for the chunk-row products):
//   dU_s  = (lam K) dS'_s + Aqk^T dO_s               (M = 64, N = DVS)
//   dS_s  = Gam_C dS'_s + (Gam Q)^T dO_s - W^T dU_s  (M = 128, N = DVS)
// and the slice of each chunk's dS' image goes to the workspace for bwd_par.
// When the forward's prep wrote the chain operands (FLAG_CHAIN: NP = -(lam K)^T W
// and Q~ = Q Gam - Aqk W), the two products fold into one MMA round trip,
//   dS_s  = Gam_C dS'_s + NP^T dS'_s + Q~^T dO_s.
template <int DVS>
struct SeqSliceMap {
  // per operand set: W, Q Gam, lam K, dO, Aqk, Gam_C (two sets in flight); with
  // the prep's chain operands (FLAG_CHAIN) a set is NP, Q~, dO, Gam_C and three
  // sets fit, so loads are issued two chunks ahead
  static constexpr int W = 0, QG = 16384, KL = 32768, DO = 49152, AQ = 65536, GC = 73728;
  static constexpr int SET = GC + 512;
  static constexpr int NP = 0, QT = 32768, CGC = 65536;
  static constexpr int CSET = CGC + 512;
  static constexpr int RING = 3 * CSET > 2 * SET ? 3 * CSET : 2 * SET;
  static constexpr int SB = RING;             // dS'_s bf16 CM[128][DVS]
  static constexpr int DU = SB + 256 * DVS;   // -dU_s bf16 CM[64][DVS]
  static constexpr int BAR = DU + 128 * DVS;
  static constexpr int SMEM = BAR + 64;
  static constexpr int TCOLS = 2 * DVS <= 32 ? 32 : (2 * DVS <= 64 ? 64 : 128);
};

template <int N>
__device__ __forceinline__ void tmem_ldn_s(uint32_t taddr, float* v) {
  if constexpr (N == 32) tmem_ld32(taddr, v);
  else if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld8(taddr, v);
}
template <int N>
__device__ __forceinline__ void tmem_stn_s(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  if constexpr (N == 32) {
    tmem_st32(taddr, v);
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
           "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
           "r"(r[15])
        : "memory");
  } else {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
                    "r"(r[6]), "r"(r[7])
                 : "memory");
  }
}

template <int DVS>
__global__ void __launch_bounds__(NT, 1)
bwd_seq_sliced_kernel(const bf16* __restrict__ dout, const unsigned char* __restrict__ factors,
                      const float* __restrict__ dsT, float* __restrict__ ds0, bf16* __restrict__ dsw, int T,
                      int H, const int* __restrict__ cs, int* __restrict__ err,
                      const __grid_constant__ CUtensorMap tm_do, int use_tma) {
  using M = SeqSliceMap<DVS>;
  constexpr int NS = DV / DVS;
  constexpr int CW = DVS / 2;              // columns per warp (one lane quarter, one column half)
  constexpr int CB = CW < 32 ? CW : 32;    // columns per TMEM access
  extern __shared__ __align__(1024) unsigned char sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + M::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + M::BAR + 8);
  uint64_t* mbar_ld = reinterpret_cast<uint64_t*>(sm + M::BAR + 16);  // [3]: one per operand set
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
  const size_t tok0 = static_cast<size_t>(b) * T;
  const size_t rstride = static_cast<size_t>(H) * DK;
  const bf16* doh = dout + static_cast<size_t>(h) * DV;
  const size_t unit = static_cast<size_t>(b) * H + h;      // checkpoint row
  const size_t sunit = static_cast<size_t>(seq) * H + h;   // state (dS_T, dS_0) row
  const int col0 = s * DVS, cg0 = col0 / 8;
  uint32_t ld_par = 0u, ld_pending = 0u;
  // every chunk of a checkpoint comes from one forward schedule: the last
  // chunk's flags decide the form for the whole walk
  const bool chain = c_beg < c_end &&
                     (*reinterpret_cast<const uint32_t*>(factors + (unit * n_chunks + c_end - 1) * FAC_UNIT +
                                                         FAC_FLAG) & FLAG_CHAIN) != 0u;
  // the operand ring: chunk cc (walked in reverse) uses set (c_end - 1 - cc) % nset
  const int nset = chain && use_tma ? 3 : 2;
  const int set_bytes = chain ? M::CSET : M::SET, gc_off = chain ? M::CGC : M::GC;
  auto set_of = [&](int cc) { return (c_end - 1 - cc) % nset; };

  if (tid == 0) {
    mbar_init(mbar, 1);
    for (int p = 0; p < 3; ++p) mbar_init(mbar_ld + p, 1);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(tslot, M::TCOLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  auto issue_chunk = [&](int cc) {
    const int ps = set_of(cc), t0 = cc * C, rv = min(C, T - t0);
    unsigned char* set = sm + ps * set_bytes;
    if (!use_tma) {
      stage_tile(set + M::DO, doh + (tok0 + t0) * rstride, rv, rstride);
      cp_async_commit();
    }
    if (tid == kIoThread) {
      const unsigned char* fu = factors + (unit * n_chunks + cc) * FAC_UNIT;
      fence_async_smem();
      if (chain) {
        mbar_expect_tx(mbar_ld + ps, 32768 + 16384 + 512 + (use_tma ? 16384 : 0));
        bulk_load(set + M::NP, fu + FAC_NP, 32768, mbar_ld + ps);
        bulk_load(set + M::QT, fu + FAC_QT, 16384, mbar_ld + ps);
      } else {
        mbar_expect_tx(mbar_ld + ps, 32768 + 16384 + 8192 + 512 + (use_tma ? 16384 : 0));
        bulk_load(set + M::W, fu + FAC_W, 32768, mbar_ld + ps);  // W, Q Gam
        bulk_load(set + M::KL, fu + FAC_KL, 16384, mbar_ld + ps);
        bulk_load(set + M::AQ, fu + FAC_AQ, 8192, mbar_ld + ps);
      }
      bulk_load(set + gc_off, fu + FAC_GC, 512, mbar_ld + ps);
      if (use_tma) tma_tile(set + M::DO, &tm_do, h, cc, b, mbar_ld + ps);
    }
    ld_pending |= 1u << ps;
  };
  for (int cc = c_end - 1; cc >= max(c_beg, c_end - (nset - 1)); --cc) issue_chunk(cc);
  const uint32_t tbase = *tslot;
  const uint32_t T_DS = tbase, T_U = tbase + DVS;
  const uint32_t tl = static_cast<uint32_t>(32 * qw) << 16;
  uint32_t phase = 0;
  bool failed = false;
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mbar, phase);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };
  const int d = 32 * qw + lane, cw0 = hh * CW;
  {  // dS_T -> TMEM (this slice)
#pragma unroll
    for (int j = 0; j < CW; j += CB) {
      float vals[CB];
#pragma unroll
      for (int e = 0; e < CB; ++e) vals[e] = dsT ? dsT[(sunit * DK + d) * DV + col0 + cw0 + j + e] : 0.f;
      tmem_stn_s<CB>(T_DS + tl + cw0 + j, vals);
    }
    tmem_wait_st();
  }

  for (int c = c_end - 1; c >= c_beg; --c) {
    const int p = set_of(c);
    cp_async_wait<0>();
    failed |= !mbar_wait(mbar_ld + p, (ld_par >> p) & 1u);
    ld_par ^= 1u << p;
    ld_pending &= ~(1u << p);
    if (tid == kIoThread) bulk_wait_read();  // SB may be rewritten: the previous dS' slice is stored
    if (__syncthreads_or(failed)) break;
    const unsigned char* setp = sm + p * set_bytes;
    const uint32_t set = smem_u32(setp);
    const float* gamC = reinterpret_cast<const float*>(setp + gc_off);
    // chunk c - nset + 1 goes into the set of chunk c + 1, which has completed
    if (c - (nset - 1) >= c_beg) issue_chunk(c - (nset - 1));
    {  // dS' pass: bf16 operand (stored to the workspace below), then dS *= Gam_C
      const float gcd = gamC[d];
#pragma unroll
      for (int j = 0; j < CW; j += CB) {
        float vals[CB];
        tmem_ldn_s<CB>(T_DS + tl + cw0 + j, vals);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < CB; e += 8) st16(sm + M::SB, cm_off(d, cw0 + j + e, DVS), pack_bf16x8(vals + e));
#pragma unroll
        for (int e = 0; e < CB; ++e) vals[e] *= gcd;
        tmem_stn_s<CB>(T_DS + tl + cw0 + j, vals);
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIoThread) {  // this slice of chunk c's dS' image
      unsigned char* img = reinterpret_cast<unsigned char*>(dsw) + (unit * n_chunks + c) * WS_UNIT;
#pragma unroll 1
      for (int rg = 0; rg < 16; ++rg)
        bulk_store(img + (rg * 16 + cg0) * 128, sm + M::SB + rg * (16 * DVS), 16 * DVS);
      bulk_commit();
    }
    if (chain) {  // dS_s += NP^T dS'_s + Q~^T dO_s: one round trip
      if (tid == 0) {
        tc_fence_after();
        const uint32_t sb = smem_u32(sm + M::SB), np = set + M::NP, qt = set + M::QT,
                       dob = set + M::DO + cg0 * 128;
        const uint32_t id = idesc_bf16(128, DVS, true, true);
#pragma unroll 1
        for (int ks = 0; ks < DK / 16; ++ks)
          mma_bf16(T_DS, desc_mnmajor(np + ks * 4096, DK), desc_mnmajor(sb + ks * (32 * DVS), DVS), id, 1u);
#pragma unroll 1
        for (int ks = 0; ks < C / 16; ++ks)
          mma_bf16(T_DS, desc_mnmajor(qt + ks * 4096, DK), desc_mnmajor(dob + ks * 4096, DV), id, 1u);
        mma_commit(mbar);
      }
      failed |= !mma_wait();  // the next chunk's barrier shares failures
      continue;
    }
    // dU_s = (lam K) dS'_s + Aqk^T dO_s  (M = 64); filler: dS_s += (Gam Q)^T dO_s
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sb = smem_u32(sm + M::SB), kl = set + M::KL, dob = set + M::DO + cg0 * 128,
                     aqb = set + M::AQ, qg = set + M::QG;
      const uint32_t id1 = idesc_bf16(64, DVS, false, true), id2 = idesc_bf16(64, DVS, true, true);
      const uint32_t id3 = idesc_bf16(128, DVS, true, true);
#pragma unroll 1
      for (int ks = 0; ks < DK / 16; ++ks)
        mma_bf16(T_U, desc_kmajor(kl + ks * 256, DK), desc_mnmajor(sb + ks * (32 * DVS), DVS), id1, ks > 0);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_U, desc_mnmajor(aqb + ks * 2048, C), desc_mnmajor(dob + ks * 4096, DV), id2, 1u);
      mma_commit(mbar);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_DS, desc_mnmajor(qg + ks * 4096, DK), desc_mnmajor(dob + ks * 4096, DV), id3, 1u);
    }
    failed |= !mma_wait();
    if (__syncthreads_or(failed)) break;
    {  // -dU_s -> bf16 CM[64][DVS] (M = 64 layout: row r at lane 32 (r / 16) + r % 16)
      const int r = 16 * qw + lane;
#pragma unroll
      for (int j = 0; j < CW; j += CB) {
        float vals[CB];
        tmem_ldn_s<CB>(T_U + tl + cw0 + j, vals);
        tmem_wait_ld();
        if (lane < 16) {
#pragma unroll
          for (int e = 0; e < CB; ++e) vals[e] = -vals[e];
#pragma unroll
          for (int e = 0; e < CB; e += 8) st16(sm + M::DU, cm_off(r, cw0 + j + e, DVS), pack_bf16x8(vals + e));
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // dS_s += W^T (-dU_s)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t du = smem_u32(sm + M::DU), w = set + M::W;
      const uint32_t id = idesc_bf16(128, DVS, true, true);
#pragma unroll 1
      for (int ks = 0; ks < C / 16; ++ks)
        mma_bf16(T_DS, desc_mnmajor(w + ks * 4096, DK), desc_mnmajor(du + ks * (32 * DVS), DVS), id, 1u);
      mma_commit(mbar);
    }
    failed |= !mma_wait();  // the next chunk's barrier shares failures
  }
  failed = __syncthreads_or(failed) != 0;
  if (!failed && ds0) {
#pragma unroll
    for (int j = 0; j < CW; j += CB) {
      float vals[CB];
      tmem_ldn_s<CB>(T_DS + tl + cw0 + j, vals);
      tmem_wait_ld();
      float* dst = ds0 + (sunit * DK + d) * DV + col0 + cw0 + j;
#pragma unroll
      for (int e = 0; e < CB; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(vals[e], vals[e + 1], vals[e + 2], vals[e + 3]);
    }
  }
  if (failed && tid == 0 && err) atomicExch(err, 1);
  cp_async_wait<0>();
  for (int ps = 0; ps < 3; ++ps)
    if ((ld_pending >> ps) & 1u) mbar_wait(mbar_ld + ps, (ld_par >> ps) & 1u);
  if (tid == kIoThread) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, M::TCOLS);
}

template <int DVS>
int launch_seq_sliced(const void* dout, const unsigned char* factors, const float* dsT, float* ds0, bf16* dsw,
                      int B, int T, int H, const int* cs, int n_seqs, int* err, const CUtensorMap& tm_do,
                      int use_tma, cudaStream_t st) {
  static std::atomic<bool> done[64];
  auto kern = bwd_seq_sliced_kernel<DVS>;
  int rc = ensure_smem(kern, SeqSliceMap<DVS>::SMEM, done);
  if (rc != KDA_OK) return rc;
  const long long grid = static_cast<long long>(cs ? n_seqs : B) * H * (DV / DVS);
  if (grid > 0x7fffffffLL) return KDA_ERR_SHAPE;
  kern<<<static_cast<unsigned>(grid), NT, SeqSliceMap<DVS>::SMEM, st>>>(
      static_cast<const bf16*>(dout), factors, dsT, ds0, dsw, T, H, cs, err, tm_do, use_tma);
  return launch_status();
}

__device__ int g_bwd_tc_error = 0;
}  // namespace
int tc_scan_slices(long long heads, int n_sm);  // kda_fwd_split.cu
namespace {

int sm_count() {
  static std::atomic<int> cached[64];  // 0 until looked up (threads may race to fill it: same value)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename Tc>
int launch_bwd(const void* q, const void* k, const void* v, const void* g, const void* beta,
               const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
               void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T, int H,
               const int* cs, int n_seqs, cudaStream_t st) {
  static std::atomic<bool> done_seq[64], done_par[64];
  int rc = ensure_smem(bwd_seq_kernel, SEQ_SMEM, done_seq);
  if (rc != KDA_OK) return rc;
  rc = ensure_smem(bwd_par_kernel<Tc>, PAR_SMEM, done_par);
  if (rc != KDA_OK) return rc;
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_bwd_tc_error) != cudaSuccess) return KDA_ERR_LAUNCH;
  bf16* dsw = static_cast<bf16*>(work);
  const size_t n = (static_cast<size_t>(T) + C - 1) / C;
  const unsigned char* factors =
      static_cast<const unsigned char*>(s_ckpt) + static_cast<size_t>(B) * H * n * DK * DV * sizeof(Tc);
  // TMA tile maps of the inputs; any length or map the encoder refuses falls back
  // to cp.async staging inside the kernels
  CUtensorMap tm[5] = {}, to[4] = {};
  const void* srcs[5] = {q, k, g, v, dout};
  const void* outs[4] = {dq, dk_, dv_, dg};
  int use_tma = 1;
  for (int i = 0; i < 5 && use_tma; ++i) use_tma = make_tile_map(&tm[i], srcs[i], B, T, H) ? 1 : 0;
  for (int i = 0; i < 4 && use_tma; ++i) use_tma = make_out_map(&to[i], outs[i], B, T, H) ? 1 : 0;
  // the reverse state chain per sequence (batch row, or packed sequence), split
  // into column slices while the (sequence, head) pairs fill at most half the
  // SMs; the chunks themselves are then independent units of one launch
  const long long heads = static_cast<long long>(cs ? n_seqs : B) * H;
  const int slices = tc_scan_slices(heads, sm_count());
  switch (slices) {
    case 2: rc = launch_seq_sliced<64>(dout, factors, dsT, ds0, dsw, B, T, H, cs, n_seqs, err, tm[4], use_tma, st); break;
    case 4: rc = launch_seq_sliced<32>(dout, factors, dsT, ds0, dsw, B, T, H, cs, n_seqs, err, tm[4], use_tma, st); break;
    case 8: rc = launch_seq_sliced<16>(dout, factors, dsT, ds0, dsw, B, T, H, cs, n_seqs, err, tm[4], use_tma, st); break;
    default:
      bwd_seq_kernel<<<(cs ? n_seqs : B) * H, NT, SEQ_SMEM, st>>>(
          static_cast<const bf16*>(beta), static_cast<const bf16*>(dout), factors, dsT, ds0, dsw, T, H, cs, err,
          tm[4], use_tma);
      rc = launch_status();
  }
  if (rc != KDA_OK) return rc;
  const long long units = static_cast<long long>(B) * H * ((T + C - 1) / C);
  const int grid = static_cast<int>(units < sm_count() ? units : sm_count());
  bwd_par_kernel<Tc><<<grid, NT, PAR_SMEM, st>>>(
      static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v),
      static_cast<const bf16*>(g), static_cast<const bf16*>(beta), static_cast<const Tc*>(s_ckpt),
      factors, dsw, static_cast<const bf16*>(dout), static_cast<bf16*>(dq), static_cast<bf16*>(dk_),
      static_cast<bf16*>(dv_), static_cast<bf16*>(dg), static_cast<bf16*>(dbeta), B, T, H, err,
      tm[0], tm[1], tm[2], tm[3], tm[4], to[0], to[1], to[2], to[3], use_tma);
  return launch_status();
}

}  // namespace

bool tc_bwd_supported(int dk, int dv, int C_, int in_dt, int do_dt) {
  return dk == DK && dv == DV && C_ == C && in_dt == KDA_BF16 && do_dt == KDA_BF16;
}

size_t tc_bwd_workspace_bytes(int B, int T, int H) {
  const size_t n = (static_cast<size_t>(T) + C - 1) / C;
  return static_cast<size_t>(B) * H * n * WS_UNIT;
}

int tc_bwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
                  void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T, int H,
                  int ck_dt, const int* cs, int n_seqs, cudaStream_t st) {
  if (ck_dt == KDA_BF16)
    return launch_bwd<bf16>(q, k, v, g, beta, s_ckpt, dout, dsT, dq, dk_, dv_, dg, dbeta, ds0, work, B, T, H,
                            cs, n_seqs, st);
  if (ck_dt == KDA_F32)
    return launch_bwd<float>(q, k, v, g, beta, s_ckpt, dout, dsT, dq, dk_, dv_, dg, dbeta, ds0, work, B, T, H,
                             cs, n_seqs, st);
  return KDA_ERR_DTYPE;
}

int tc_bwd_error_flag(int* value, bool clear, cudaStream_t st) {
  static const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(value, g_bwd_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (clear && cudaMemcpyToSymbolAsync(g_bwd_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  return KDA_OK;
}

}  // namespace kda
