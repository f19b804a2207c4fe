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

// Exact scores for chunks whose summed decay is beyond the single anchor's
// budget: Aq[r][i] = sum_d q_r k_i exp(G_r - G_i) (i <= r) and Akk likewise
// with k_r (i < r), from G (fp32 [64][128], row-major).  With blocks of 16
// tokens, for row r of block I and column i of block J < I
//   exp(G_r - G_i) = a_r * m_IJ * b_i,   a_r = exp(G_r - G_{16I}),
//   m_IJ = exp(G_{16I} - G_{16J+15}),   b_i = exp(G_{16J+15} - G_i),
// and each factor is <= 1 (G is non-increasing), so nothing overflows and the
// O(C^2 dk) part needs no exponentials; pairs inside one block take exact
// exponentials.  q (sq) and k (sk) are overwritten with q a and k b (bf16 CM),
// k a goes to `ka` (CM [64][128]) and m to `m` (fp32 [6][128]).
__device__ __forceinline__ void scores_exact(unsigned char* sq, unsigned char* sk, unsigned char* ka,
                                             float* m, const float* Gf, float* Aq, float* Akk) {
  const int tid = threadIdx.x;
  // zeros above the diagonal
  for (int idx = tid; idx < C * C; idx += NT) {
    const int r = idx >> 6, i = idx & 63;
    if (i > r) {
      Aq[sw64(r, i)] = 0.f;
      Akk[sw64(r, i)] = 0.f;
    }
  }
  // (1) pairs inside a 16-token block: exact exponentials on the raw q, k
  for (int p = tid; p < 4 * 136; p += NT) {
    const int blk = p / 136, t = p % 136;
    int rr = static_cast<int>((sqrtf(8.f * t + 1.f) - 1.f) * 0.5f);
    if ((rr + 1) * (rr + 2) / 2 <= t) ++rr;
    if (rr * (rr + 1) / 2 > t) --rr;
    const int ii = t - rr * (rr + 1) / 2;
    const int r = 16 * blk + rr, i = 16 * blk + ii;
    float a = 0.f, l = 0.f;
    for (int d8 = 0; d8 < DK; d8 += 8) {
      float qr[8], kr[8], ki8[8];
      unpack_bf16x8(ld16(sq, cm_off(r, d8, DK)), qr);
      unpack_bf16x8(ld16(sk, cm_off(r, d8, DK)), kr);
      unpack_bf16x8(ld16(sk, cm_off(i, d8, DK)), ki8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float ex = __expf(fminf(Gf[r * DK + d8 + e] - Gf[i * DK + d8 + e], 0.f));
        a += qr[e] * ki8[e] * ex;
        l += kr[e] * ki8[e] * ex;
      }
    }
    Aq[sw64(r, i)] = a;
    Akk[sw64(r, i)] = (i < r) ? l : 0.f;
  }
  __syncthreads();  // the raw q, k are read: replace them with the factored rows
  // (2) a_t, b_t per (token, channel): q a -> sq, k a -> ka, k b -> sk; m per block pair
  for (int idx = tid; idx < C * (DK / 8); idx += NT) {
    const int t = idx >> 4, d8 = (idx & 15) * 8, I = t >> 4;
    const uint32_t off = cm_off(t, d8, DK);
    float qv[8], kv[8], qa[8], kav[8], kb[8];
    unpack_bf16x8(ld16(sq, off), qv);
    unpack_bf16x8(ld16(sk, off), kv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float g = Gf[t * DK + d8 + e];
      const float av = __expf(fminf(g - Gf[16 * I * DK + d8 + e], 0.f));
      const float bv = __expf(fminf(Gf[(16 * I + 15) * DK + d8 + e] - g, 0.f));
      qa[e] = qv[e] * av;
      kav[e] = kv[e] * av;
      kb[e] = kv[e] * bv;
    }
    st16(sq, off, pack_bf16x8(qa));
    st16(ka, off, pack_bf16x8(kav));
    st16(sk, off, pack_bf16x8(kb));
  }
  for (int idx = tid; idx < 6 * DK; idx += NT) {
    const int p = idx / DK, d = idx % DK;
    const int I = p < 3 ? p + 1 : (p < 5 ? p - 1 : 3), J = p < 3 ? 0 : (p < 5 ? 1 : 2);
    m[idx] = __expf(fminf(Gf[16 * I * DK + d] - Gf[(16 * J + 15) * DK + d], 0.f));
  }
  __syncthreads();
  // (3) block pairs I > J: (1,0) (2,0) (3,0) (2,1) (3,1) (3,2), multiply-adds only
  for (int idx = tid; idx < 6 * 256; idx += NT) {
    const int p = idx >> 8, w = idx & 255;
    const int I = p < 3 ? p + 1 : (p < 5 ? p - 1 : 3), J = p < 3 ? 0 : (p < 5 ? 1 : 2);
    const int r = 16 * I + (w >> 4), i = 16 * J + (w & 15);
    const float* mp = m + p * DK;
    float a = 0.f, l = 0.f;
    for (int d8 = 0; d8 < DK; d8 += 8) {
      float qa[8], kav[8], kb[8];
      unpack_bf16x8(ld16(sq, cm_off(r, d8, DK)), qa);
      unpack_bf16x8(ld16(ka, cm_off(r, d8, DK)), kav);
      unpack_bf16x8(ld16(sk, cm_off(i, d8, DK)), kb);
      const float4 m0 = *reinterpret_cast<const float4*>(mp + d8);
      const float4 m1 = *reinterpret_cast<const float4*>(mp + d8 + 4);
      const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float kbm = kb[e] * mv[e];
        a += qa[e] * kbm;
        l += kav[e] * kbm;
      }
    }
    Aq[sw64(r, i)] = a;
    Akk[sw64(r, i)] = l;
  }
  fence_async_smem();  // sq, sk, ka are the next chunk's TMA destinations
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
