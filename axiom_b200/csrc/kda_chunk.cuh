// Per-chunk building blocks shared by the tensor-core forward and backward
// kernels (bf16 operands, dk = dv = 128, chunk C = 64, 256 threads):
// staging of input tiles, the score epilogue, the exact CUDA-core score
// fallback and the blocked unit-triangular inverse T = (I + diag(beta) Akk)^-1.
#pragma once

#include "kda_common.cuh"
#include "kda_tc.cuh"

namespace kda {
namespace chunk {

using namespace tc;

constexpr int C = 64, DK = 128, DV = 128, NT = 256;
//: Largest per-channel decay summed over a chunk for which the single anchor
//: at the chunk start keeps exp(-G) representable; the reference's
//: COL_EXP_BUDGET (net/kernels/kda_cc_fused_persist.py:224).
constexpr float kExpBudget = 80.f;

// fp32 64x64 matrices with a 16-byte-chunk XOR swizzle (conflict-free row writes)
__device__ __forceinline__ int sw64(int r, int c) {
  return (r << 6) + ((((c >> 2) ^ (r & 15)) << 2) | (c & 3));
}

__device__ __forceinline__ uint4 ld16(const unsigned char* base, uint32_t off) {
  return *reinterpret_cast<const uint4*>(base + off);
}
__device__ __forceinline__ void st16(unsigned char* base, uint32_t off, uint4 v) {
  *reinterpret_cast<uint4*>(base + off) = v;
}
__device__ __forceinline__ float ldbf(const unsigned char* base, uint32_t off) {
  return __bfloat162float(*reinterpret_cast<const bf16*>(base + off));
}

template <typename To>
__device__ __forceinline__ void store_row32(To* dst, const float* v);
template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float* v) {
#pragma unroll
  for (int j = 0; j < 32; j += 4)
    *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}
template <>
__device__ __forceinline__ void store_row32<bf16>(bf16* dst, const float* v) {
#pragma unroll
  for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = pack_bf16x8(v + j);
}

// Thread -> 16-byte chunk mapping for CM tiles: 8 consecutive lanes cover the
// 8 rows of one core matrix (conflict-free in shared memory) and lanes l, l+8,
// l+16, l+24 cover 64 contiguous bytes of one row in global memory.
__device__ __forceinline__ void chunk_of(int i, int n_rg, int& r, int& cg) {
  const int cq = i & 7, cgl = (i >> 3) & 3, rest = i >> 5;
  r = 8 * (rest % n_rg) + cq;
  cg = 4 * (rest / n_rg) + cgl;
}

// cp.async a [64][128] bf16 tile whose row r starts at src + r*rstride into a
// CM tile (rows >= rows_valid are zero-filled).  Does not commit.
__device__ __forceinline__ void stage_tile(unsigned char* dst, const bf16* src, int rows_valid,
                                           size_t rstride) {
  for (int i = threadIdx.x; i < C * 16; i += NT) {
    int r, cg;
    chunk_of(i, 8, r, cg);
    const bool ok = r < rows_valid;
    const bf16* p = ok ? src + static_cast<size_t>(r) * rstride + cg * 8 : src;
    cp_async16(dst + cm_off(r, cg * 8, 128), p, ok);
  }
}

// Score epilogue (fast path).  TMEM holds [Q*Gam ; K*Gam] (K*Gi)^T at `t_scores`
// (128 lanes x 64 columns).  Writes Aqk (lower, inclusive) and Akk (strict)
// as swizzled fp32 64x64 matrices.
__device__ __forceinline__ void scores_epilogue(uint32_t t_scores, float* Aq, float* Akk) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qw = warp & 3, hh = warp >> 2;
  float vals[32];
  tmem_ld32(t_scores + (static_cast<uint32_t>(32 * qw) << 16) + hh * 32, vals);
  tmem_wait_ld();
  const int R = 32 * qw + lane;
  const int r = R & 63;
  const bool is_q = R < 64;
  float* dst = is_q ? Aq : Akk;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const int i0 = hh * 32 + j;
    float4 w4;
    w4.x = (is_q ? (i0 + 0 <= r) : (i0 + 0 < r)) ? vals[j + 0] : 0.f;
    w4.y = (is_q ? (i0 + 1 <= r) : (i0 + 1 < r)) ? vals[j + 1] : 0.f;
    w4.z = (is_q ? (i0 + 2 <= r) : (i0 + 2 < r)) ? vals[j + 2] : 0.f;
    w4.w = (is_q ? (i0 + 3 <= r) : (i0 + 3 < r)) ? vals[j + 3] : 0.f;
    *reinterpret_cast<float4*>(dst + sw64(r, i0)) = w4;
  }
}

// Packed sequences, longest first: the per-(sequence, head) kernels walk one
// sequence's chunks in order, so a long sequence scheduled late sets the
// kernel's end.  CTA rank r (blockIdx / H) takes the sequence with the r-th
// largest chunk count (ties by index) when there are at most NT sequences;
// else rank = sequence.  `scratch`: NT + 1 ints of shared memory, free on
// entry and on exit.  All threads call it.
__device__ __forceinline__ int longest_first(const int* cs, int n, int r, int n_chunks, int* scratch) {
  if (n > NT) return r;
  const int tid = threadIdx.x;
  if (tid < n) {
    const int c0 = min(max(cs[tid], 0), n_chunks);
    scratch[tid] = min(max(cs[tid + 1], c0), n_chunks) - c0;  // clamped like the ranges themselves
  }
  __syncthreads();
  if (tid < n) {
    const int len = scratch[tid];
    int rank = 0;
    for (int s2 = 0; s2 < n; ++s2) {
      const int l2 = scratch[s2];
      rank += (l2 > len) || (l2 == len && s2 < tid);
    }
    if (rank == r) scratch[NT] = tid;
  }
  __syncthreads();
  const int seq = scratch[NT];
  __syncthreads();
  return seq;
}

// G fp32 [64][128] of the exact path: the 16-byte chunks of row r are
// XOR-swizzled by (r & 7), so eight rows' same chunk lie in distinct banks.
__device__ __forceinline__ int gsw(int r, int d) {
  return r * DK + ((((d >> 2) ^ r) & 7) | ((d >> 2) & ~7)) * 4 + (d & 3);
}
__device__ __forceinline__ void ld8g(const float* G, int r, int d8, float* o) {  // G[r][d8 .. d8 + 8)
  const float4 x = *reinterpret_cast<const float4*>(G + gsw(r, d8));
  const float4 y = *reinterpret_cast<const float4*>(G + gsw(r, d8 + 4));
  o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w; o[4] = y.x; o[5] = y.y; o[6] = y.z; o[7] = y.w;
}

// One row r of a diagonal block for the exact scores (two channels per lane):
// v[VQ + i] = sum_c q_r k_i exp(G_r - G_i), v[VK + i] = the same with k_r (i < r),
// exp(G_r - G_i) as the running product of the decays a_t = exp(g_t).
template <int R, int VQ, int VK>
__device__ __forceinline__ void exact_diag_row(const float (&q0)[16], const float (&q1)[16], const float (&k0)[16],
                                               const float (&k1)[16], const float (&a0)[16], const float (&a1)[16],
                                               float (&v)[32]) {
  float e0 = 1.f, e1 = 1.f;
#pragma unroll
  for (int i = R; i >= 0; --i) {
    if (i < R) {
      e0 *= a0[i + 1];
      e1 *= a1[i + 1];
    }
    const float x0 = k0[i] * e0, x1 = k1[i] * e1;
    v[VQ + i] = fmaf(q0[R], x0, q1[R] * x1);
    if (i < R) v[VK + i] = fmaf(k0[R], x0, k1[R] * x1);
  }
}

// Rows RP and 15 - RP of diagonal block `blk`: 17 Aq and 15 Akk sums, 32 in
// all, which one batched warp reduction spreads one per lane; each lane adds
// its sum (this warp's 64 channels) into Aq / Akk.
template <int RP>
__device__ __forceinline__ void exact_diag_pair(const float (&q0)[16], const float (&q1)[16], const float (&k0)[16],
                                                const float (&k1)[16], const float (&a0)[16], const float (&a1)[16],
                                                int lane, int blk, float* Aq, float* Akk) {
  float v[32];
  exact_diag_row<RP, 0, 17>(q0, q1, k0, k1, a0, a1, v);
  exact_diag_row<15 - RP, RP + 1, 17 + RP>(q0, q1, k0, k1, a0, a1, v);
  const float sum = warp_colsum<32>(v, lane);  // lane j: entry j
  int r, i;
  float* dst;
  if (lane <= RP) {
    dst = Aq; r = RP; i = lane;
  } else if (lane < 17) {
    dst = Aq; r = 15 - RP; i = lane - RP - 1;
  } else if (lane < 17 + RP) {
    dst = Akk; r = RP; i = lane - 17;
  } else {
    dst = Akk; r = 15 - RP; i = lane - 17 - RP;
  }
  atomicAdd(dst + sw64(16 * blk + r, 16 * blk + i), sum);
}

// Exact scores for chunks whose summed decay is beyond the single anchor's
// budget: Aq[r][i] = sum_d q_r k_i exp(G_r - G_i) (i <= r) and Akk likewise
// with k_r (i < r).  With blocks of 16 tokens, for row r of block I and column
// i of block J < I
//   exp(G_r - G_i) = exp(G_r - G_{16I}) * exp(G_{16I} - G_i),
// both factors <= 1 (G is non-increasing), so the block pairs are tensor-core
// products [q a ; k a] kbm_I^T with a_r = exp(G_r - G_{16I}) and
// kbm_I[i] = k_i exp(G_{16I} - G_i) (i < 16 I), N = 16 I.  This part, on the
// CUDA cores, fills the pairs inside each block (exact, fp32) and writes those
// operands: q a -> sq, k a -> sk (in place, so [sq ; sk] is the 128-row A
// operand) and kbm_1..3 (bf16 CM [16 I][128]).  Inputs: raw q, k, g (sq, sk,
// sg; bf16 CM [64][128]) and G (fp32, gsw layout).
static __device__ __noinline__ void scores_exact_prep(unsigned char* sq, unsigned char* sk, const unsigned char* sg,
                                                  unsigned char* kbm1, unsigned char* kbm2, unsigned char* kbm3,
                                                  const float* Gf, float* Aq, float* Akk) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // zeros above the diagonal and in the diagonal blocks (accumulated below)
  for (int idx = tid; idx < C * C; idx += NT) {
    const int r = idx >> 6, i = idx & 63;
    if (i > r || (i >> 4) == (r >> 4)) {
      Aq[sw64(r, i)] = 0.f;
      Akk[sw64(r, i)] = 0.f;
    }
  }
  __syncthreads();
  {
    // Pairs inside a block: warp w takes block w / 2 and 64 channels (two per
    // lane); the two channel halves meet in a shared-memory add onto zero
    // (two addends: order-free).
    const int blk = warp >> 1, d0 = 64 * (warp & 1) + 2 * lane;
    float q0[16], q1[16], k0[16], k1[16], a0[16], a1[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const uint32_t off = cm_off(16 * blk + t, d0, DK);
      const float2 qv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sq + off));
      const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sk + off));
      const float2 gv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sg + off));
      q0[t] = qv.x; q1[t] = qv.y; k0[t] = kv.x; k1[t] = kv.y;
      a0[t] = __expf(gv.x); a1[t] = __expf(gv.y);
    }
    exact_diag_pair<0>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<1>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<2>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<3>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<4>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<5>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<6>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
    exact_diag_pair<7>(q0, q1, k0, k1, a0, a1, lane, blk, Aq, Akk);
  }
  __syncthreads();  // the raw q, k are read: replace them with the factored rows
  // Operands: eight consecutive threads take the eight rows of one core matrix
  // (conflict-free 16-byte accesses); warps are uniform in the block I.
  for (int idx = tid; idx < C * (DK / 8); idx += NT) {
    const int t = ((idx >> 7) << 3) + (idx & 7), d8 = ((idx >> 3) & 15) * 8, I = t >> 4;
    const uint32_t off = cm_off(t, d8, DK);
    float qv[8], kv[8], gt[8], ga[8], o1[8], o2[8];
    unpack_bf16x8(ld16(sq, off), qv);
    unpack_bf16x8(ld16(sk, off), kv);
    ld8g(Gf, t, d8, gt);
    ld8g(Gf, 16 * I, d8, ga);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float av = __expf(fminf(gt[e] - ga[e], 0.f));
      o1[e] = qv[e] * av;
      o2[e] = kv[e] * av;
    }
    st16(sq, off, pack_bf16x8(o1));
    st16(sk, off, pack_bf16x8(o2));
    for (int I2 = I + 1; I2 < 4; ++I2) {
      ld8g(Gf, 16 * I2, d8, ga);
#pragma unroll
      for (int e = 0; e < 8; ++e) o1[e] = kv[e] * __expf(fminf(ga[e] - gt[e], 0.f));
      st16(I2 == 1 ? kbm1 : (I2 == 2 ? kbm2 : kbm3), off, pack_bf16x8(o1));
    }
  }
  fence_async_smem();  // generic writes -> the tensor core's reads
}

// Scores for chunks whose summed decay passes the single anchor's budget while
// each 32-token half stays within it (per channel: -G_31 <= 80 and
// G_31 - G_63 <= 80).  Half J is anchored at A_0 = 0 (before the chunk) and
// A_1 = G_31 (before token 32):
//   pairs inside half J:           exp(G_r - G_i) = exp(G_r - A_J) exp(A_J - G_i)
//   r in half 1, i in half 0:      exp(G_r - G_31) exp(G_31 - G_i), both <= 1,
// so two tensor-core products give every pair with no exact exponentials:
// D_diag = [q a ; k a] bd^T (N = 64) and D_cross = [q a ; k a] bc^T (N = 32),
// a_r = exp(G_r - A_J(r)) <= 1, bd_i = k_i exp(A_J(i) - G_i) <= exp(80),
// bc_i = k_i exp(G_31 - G_i) <= 1 (i < 32).
__device__ __forceinline__ bool halves_within_budget(const float* Gf) {  // this thread's channel
  const int d = threadIdx.x;
  if (d >= DK) return true;
  const float g31 = Gf[gsw(31, d)], g63 = Gf[gsw(63, d)];
  return -g31 <= kExpBudget && g31 - g63 <= kExpBudget;
}

// Operands of the two-half scores: q a -> sq, k a -> sk (in place, the 128-row A
// operand), bd -> CM [64][128], bc -> CM [32][128].  Inputs: raw q, k (sq, sk)
// and G (fp32, gsw layout).
static __device__ __noinline__ void scores_halves_prep(unsigned char* sq, unsigned char* sk, unsigned char* bd,
                                                       unsigned char* bc, const float* Gf) {
  for (int idx = threadIdx.x; idx < C * (DK / 8); idx += NT) {
    // eight consecutive threads take the eight rows of one core matrix; warps are
    // uniform in the half
    const int t = ((idx >> 7) << 3) + (idx & 7), d8 = ((idx >> 3) & 15) * 8, J = t >> 5;
    const uint32_t off = cm_off(t, d8, DK);
    float qv[8], kv[8], gt[8], ga[8], o1[8], o2[8];
    unpack_bf16x8(ld16(sq, off), qv);
    unpack_bf16x8(ld16(sk, off), kv);
    ld8g(Gf, t, d8, gt);
    if (J) {
      ld8g(Gf, 31, d8, ga);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) ga[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float av = __expf(fminf(gt[e] - ga[e], 0.f));
      o1[e] = qv[e] * av;
      o2[e] = kv[e] * av;
    }
    st16(sq, off, pack_bf16x8(o1));
    st16(sk, off, pack_bf16x8(o2));
#pragma unroll
    for (int e = 0; e < 8; ++e) o1[e] = kv[e] * __expf(ga[e] - gt[e]);
    st16(bd, off, pack_bf16x8(o1));
    if (!J) {
      ld8g(Gf, 31, d8, ga);
#pragma unroll
      for (int e = 0; e < 8; ++e) o2[e] = kv[e] * __expf(fminf(ga[e] - gt[e], 0.f));
      st16(bc, off, pack_bf16x8(o2));
    }
  }
  fence_async_smem();  // generic writes -> the tensor core's reads
}

// Issue (one thread): D_diag -> columns [0, 64), D_cross -> [64, 96).
__device__ __forceinline__ void scores_halves_mma(uint32_t tmem, uint32_t a_qk, uint32_t bd, uint32_t bc) {
  const uint32_t id64 = idesc_bf16(128, 64, false, false), id32 = idesc_bf16(128, 32, false, false);
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks)
    mma_bf16(tmem, desc_kmajor(a_qk + ks * 256, DK), desc_kmajor(bd + ks * 256, DK), id64, ks > 0);
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks)
    mma_bf16(tmem + 64, desc_kmajor(a_qk + ks * 256, DK), desc_kmajor(bc + ks * 256, DK), id32, ks > 0);
}

// TMEM -> Aq (lanes 0..63) / Akk (lanes 64..127), masked (i <= r, i < r).  Warp w
// takes TMEM lanes 32 (w % 4) .. +31 (one half of the rows) and the columns of
// half w / 4: the same half comes from D_diag, half 0 under rows of half 1 from
// D_cross, half 1 above rows of half 0 is zero.
__device__ __forceinline__ void scores_halves_epilogue(uint32_t tmem, float* Aq, float* Akk) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qw = warp & 3, hh = warp >> 2;
  const int R = 32 * qw + lane, r = R & 63, Jr = qw & 1;
  const bool is_q = R < 64;
  float* dst = is_q ? Aq : Akk;
  const uint32_t tl = static_cast<uint32_t>(32 * qw) << 16;
  float vals[32];
  if (hh == Jr || hh == 0) {
    tmem_ld32(tmem + tl + (hh == Jr ? 32 * hh : 64), vals);
    tmem_wait_ld();
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) vals[j] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const int i0 = hh * 32 + j;
    float4 w4;
    w4.x = (is_q ? (i0 + 0 <= r) : (i0 + 0 < r)) ? vals[j + 0] : 0.f;
    w4.y = (is_q ? (i0 + 1 <= r) : (i0 + 1 < r)) ? vals[j + 1] : 0.f;
    w4.z = (is_q ? (i0 + 2 <= r) : (i0 + 2 < r)) ? vals[j + 2] : 0.f;
    w4.w = (is_q ? (i0 + 3 <= r) : (i0 + 3 < r)) ? vals[j + 3] : 0.f;
    *reinterpret_cast<float4*>(dst + sw64(r, i0)) = w4;
  }
  tc_fence_before();  // the TMEM reads precede later MMAs into these columns
}

// Column of kbm_I's products in the score TMEM block: I = 1, 2, 3 -> 0, 16, 48.
__device__ __forceinline__ int exact_col(int I) { return 8 * I * (I - 1); }

// Issue of the block-pair products (one thread): D[:, col(I) .. col(I) + 16 I)
// = [q a ; k a] kbm_I^T, K = dk.
__device__ __forceinline__ void scores_exact_mma(uint32_t tmem, uint32_t a_qk, uint32_t kbm1, uint32_t kbm2,
                                                 uint32_t kbm3) {
#pragma unroll
  for (int I = 1; I <= 3; ++I) {
    const uint32_t idesc = idesc_bf16(128, 16 * I, false, false), kb = I == 1 ? kbm1 : (I == 2 ? kbm2 : kbm3);
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks)
      mma_bf16(tmem + exact_col(I), desc_kmajor(a_qk + ks * 256, DK), desc_kmajor(kb + ks * 256, DK), idesc,
               ks > 0);
  }
}

// TMEM -> Aq (lanes 0..63) / Akk (lanes 64..127) for the block pairs I > J.
// Warp w reads TMEM lanes 32 (w % 4) .. +31 (rows of blocks 2 (w % 2) and
// 2 (w % 2) + 1) and the column blocks J of parity w / 4.
__device__ __forceinline__ void scores_exact_epilogue(uint32_t tmem, float* Aq, float* Akk) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qw = warp & 3, hh = warp >> 2;
  const int R = 32 * qw + lane, r = R & 63;
  float* dst = R < 64 ? Aq : Akk;
  const uint32_t tl = static_cast<uint32_t>(32 * qw) << 16;
  const int Ib = 2 * (qw & 1);  // rows of blocks Ib (lanes 0..15) and Ib + 1 (lanes 16..31)
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int I = Ib + s;
    for (int J = hh; J < I; J += 2) {  // warp-uniform
      float x[16];
      tmem_ld16(tmem + tl + exact_col(I) + 16 * J, x);
      tmem_wait_ld();
      if ((r >> 4) == I) {
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(dst + sw64(r, 16 * J + j)) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
      }
    }
  }
  tc_fence_before();  // the TMEM reads precede later MMAs into these columns
}


// One merge step of the recursive-doubling inverse: for every pair of BS x BS
// diagonal blocks already inverted (A^-1 above, B^-1 below), fill the block
// between them with -B^-1 diag(beta) C A^-1.  Each thread owns an RB x CB
// block of outputs; 256 threads cover the (64 / 2BS) blocks of BS x BS
// outputs.  The loops run over whole blocks (the strictly upper parts of A^-1
// and B^-1 are zero), four k-steps per iteration with float4 loads of the C /
// B^-1 rows, so the shared-memory loads issue ahead of the FMAs.  X = C A^-1
// goes through `xs` (32 * BS floats) so the step needs two barriers.
template <int BS, int RB, int CB>
__device__ __forceinline__ void solve_merge(const float* Akk, const float* beta_s, float* Tm,
                                            float* xs) {
  static_assert((C / (2 * BS)) * (BS / RB) * (BS / CB) == NT, "one output block per thread");
  const int tid = threadIdx.x;
  constexpr int NR = BS / RB, NC = BS / CB;
  const int blk = tid / (NR * NC), rem = tid % (NR * NC);
  const int r0 = (rem / NC) * RB, c0 = (rem % NC) * CB, o = 2 * BS * blk;
  float x[RB][CB];
#pragma unroll
  for (int i = 0; i < RB; ++i)
#pragma unroll
    for (int j = 0; j < CB; ++j) x[i][j] = 0.f;
#pragma unroll
  for (int p = 0; p < BS; p += 4) {
    float a[4][CB];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (CB == 2) {
        const float2 t2 = *reinterpret_cast<const float2*>(Tm + sw64(o + p + u, o + c0));
        a[u][0] = t2.x;
        a[u][CB - 1] = t2.y;
      } else {
        a[u][0] = Tm[sw64(o + p + u, o + c0)];
      }
    }
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const float4 cv = *reinterpret_cast<const float4*>(Akk + sw64(o + BS + r0 + i, o + p));
#pragma unroll
      for (int j = 0; j < CB; ++j)
        x[i][j] += cv.x * a[0][j] + cv.y * a[1][j] + cv.z * a[2][j] + cv.w * a[3][j];
    }
  }
  // X (scaled by beta) -> xs[blk][r][c], row-major BS x BS per block
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    const float bb = beta_s[o + BS + r0 + i];
#pragma unroll
    for (int j = 0; j < CB; ++j) xs[(blk * BS + r0 + i) * BS + c0 + j] = bb * x[i][j];
  }
  __syncthreads();
  float y[RB][CB];
#pragma unroll
  for (int i = 0; i < RB; ++i)
#pragma unroll
    for (int j = 0; j < CB; ++j) y[i][j] = 0.f;
#pragma unroll
  for (int m = 0; m < BS; m += 4) {
    float xv[4][CB];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < CB; ++j) xv[u][j] = xs[(blk * BS + m + u) * BS + c0 + j];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const float4 bv = *reinterpret_cast<const float4*>(Tm + sw64(o + BS + r0 + i, o + BS + m));
#pragma unroll
      for (int j = 0; j < CB; ++j)
        y[i][j] -= bv.x * xv[0][j] + bv.y * xv[1][j] + bv.z * xv[2][j] + bv.w * xv[3][j];
    }
  }
#pragma unroll
  for (int i = 0; i < RB; ++i)
#pragma unroll
    for (int j = 0; j < CB; ++j) Tm[sw64(o + BS + r0 + i, o + c0 + j)] = y[i][j];
  __syncthreads();
}

// T = (I + L)^-1 with L = diag(beta) Akk (strictly lower, 64 x 64) by
// recursive doubling: the eight 8 x 8 diagonal blocks are inverted by forward
// substitution, then blocks of 8, 16 and 32 are merged pairwise with
//   [A 0; C B]^-1 = [A^-1 0; -B^-1 C A^-1 B^-1]   (fp32 throughout).
// `xs` is 4 KB of scratch.  All threads take part; ends synced.
__device__ __forceinline__ void solve_T(const float* Akk, const float* beta_s, float* Tm,
                                        float* xs) {
  const int tid = threadIdx.x;
  for (int idx = tid; idx < C * C; idx += NT) Tm[idx] = 0.f;  // the swizzle is a permutation
  __syncthreads();
  if (tid < 64) {  // diagonal 8x8 blocks, one column per thread
    const int o = 8 * (tid >> 3), j = tid & 7;
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc += Akk[sw64(o + i, o + m)] * x[m];
      x[i] = ((i == j) ? 1.f : 0.f) - beta_s[o + i] * acc;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) Tm[sw64(o + i, o + j)] = x[i];
  }
  __syncthreads();
  solve_merge<8, 1, 1>(Akk, beta_s, Tm, xs);
  solve_merge<16, 2, 1>(Akk, beta_s, Tm, xs);
  solve_merge<32, 2, 2>(Akk, beta_s, Tm, xs);
}

// Write row r, columns c0..c0+15 of a fp32 swizzled 64x64 matrix M (times
// colscale[c] when given) as bf16 into a CM tile with 64 columns at row `dst_row`.
// 16 consecutive fp32 values of row r of a swizzled 64 x 64 matrix (sw64),
// columns c0..c0+15, read with explicit shared-memory vector loads.
__device__ __forceinline__ void ld_row16_sw64(const float* M, int r, int c0, float* v) {
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(M));
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const uint32_t a = base + 4u * static_cast<uint32_t>(sw64(r, c0 + j));
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[j]), "=f"(v[j + 1]), "=f"(v[j + 2]), "=f"(v[j + 3]) : "r"(a));
  }
}

__device__ __forceinline__ void row16_to_cm(unsigned char* dst, int dst_row, const float* M, int r,
                                            int c0, const float* colscale) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const float4 t4 = *reinterpret_cast<const float4*>(M + sw64(r, c0 + j));
    v[j] = t4.x; v[j + 1] = t4.y; v[j + 2] = t4.z; v[j + 3] = t4.w;
  }
  if (colscale) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= colscale[c0 + j];
  }
  st16(dst, cm_off(dst_row, c0, 64), pack_bf16x8(v));
  st16(dst, cm_off(dst_row, c0 + 8, 64), pack_bf16x8(v + 8));
}

}  // namespace chunk
}  // namespace kda
