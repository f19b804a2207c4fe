// Per-chunk building blocks shared by the tensor-core forward and backward
// kernels (bf16 operands, dk = dv = 128, chunk C = 64, 256 threads):
// staging of input tiles, the decay prep (G = cumsum(g) and the scaled operand
// tiles), the score epilogue, the exact CUDA-core score fallback and the
// blocked unit-triangular inverse T = (I + diag(beta) Akk)^-1.
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

// cp.async a [64][128] bf16 tile whose row r starts at src + r*rstride into a
// CM tile (rows >= rows_valid are zero-filled).  Does not commit.
__device__ __forceinline__ void stage_tile(unsigned char* dst, const bf16* src, int rows_valid,
                                           size_t rstride) {
  for (int i = threadIdx.x; i < C * 16; i += NT) {
    const int r = i >> 4, cg = i & 15;
    const bool ok = r < rows_valid;
    const bf16* p = ok ? src + static_cast<size_t>(r) * rstride + cg * 8 : src;
    cp_async16(dst + cm_off(r, cg * 8, 128), p, ok);
  }
}

// cp.async a contiguous [128][128] bf16 matrix (row stride 128) into a CM tile.
__device__ __forceinline__ void stage_square(unsigned char* dst, const bf16* src) {
  for (int i = threadIdx.x; i < 128 * 16; i += NT) {
    const int r = i >> 4, cg = i & 15;
    cp_async16(dst + cm_off(r, cg * 8, 128), src + r * 128 + cg * 8, true);
  }
}

// Decay prep for one chunk.  Thread t owns channels 8(t&15).. and rows
// 4(t>>4)..+3.  Reads the staged q, k, g tiles and writes the bf16 operand
// tiles (CM, 128 columns):
//   qg = q*Gam, kg = k*Gam, ki = k*exp(-G) (fast path only), kl = k*exp(G_C - G)
// with G = cumsum(g) over the chunk, Gam = exp(G).  gamC[d] = exp(G_C[d]).
// Any of the destinations may be null.  Returns true ("slow") when some
// channel decays by more than kExpBudget over the chunk; the caller must then
// use the exact score path.  `part` is 8 KB of scratch.  G (fp32) is returned
// in registers for the caller.
__device__ __forceinline__ bool prep(const unsigned char* sq, const unsigned char* sk,
                                     const unsigned char* sg, unsigned char* qg_dst,
                                     unsigned char* kg_dst, unsigned char* ki_dst,
                                     unsigned char* kl_dst, float* part, float* gamC,
                                     float (&G)[4][8]) {
  const int tid = threadIdx.x, cg = tid & 15, rg4 = tid >> 4;
  float run[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) run[e] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float gv[8];
    unpack_bf16x8(ld16(sg, cm_off(4 * rg4 + i, 8 * cg, 128)), gv);
#pragma unroll
    for (int e = 0; e < 8; ++e) { run[e] += gv[e]; G[i][e] = run[e]; }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[(rg4 * 16 + cg) * 8 + e] = run[e];
  __syncthreads();
  float pre[8], tot[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) { pre[e] = 0.f; tot[e] = 0.f; }
  for (int p = 0; p < 16; ++p) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = part[(p * 16 + cg) * 8 + e];
      tot[e] += x;
      if (p < rg4) pre[e] += x;
    }
  }
  bool strong = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    strong |= fabsf(tot[e]) > kExpBudget;
#pragma unroll
    for (int i = 0; i < 4; ++i) G[i][e] += pre[e];
  }
  float gce[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) gce[e] = __expf(tot[e]);
  if (rg4 == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) gamC[8 * cg + e] = gce[e];
  }
  // one barrier publishes gamC, frees `part`, and decides the path CTA-wide
  const bool slow = __syncthreads_or(strong) != 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rg4 + i;
    const uint32_t off = cm_off(r, 8 * cg, 128);
    float qv[8], kv[8], qg[8], kg[8], ki[8], kl[8];
    unpack_bf16x8(ld16(sq, off), qv);
    unpack_bf16x8(ld16(sk, off), kv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float gam = __expf(G[i][e]);
      qg[e] = qv[e] * gam;
      kg[e] = kv[e] * gam;
      if (!slow) {
        const float gi = __expf(-G[i][e]);
        ki[e] = kv[e] * gi;
        kl[e] = kv[e] * (gi * gce[e]);
      } else {
        ki[e] = 0.f;
        kl[e] = kv[e] * __expf(fminf(tot[e] - G[i][e], 0.f));
      }
    }
    if (qg_dst) st16(qg_dst, off, pack_bf16x8(qg));
    if (kg_dst) st16(kg_dst, off, pack_bf16x8(kg));
    if (ki_dst && !slow) st16(ki_dst, off, pack_bf16x8(ki));
    if (kl_dst) st16(kl_dst, off, pack_bf16x8(kl));
  }
  return slow;
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

// Exact scores on the CUDA cores (strong-decay chunks): Aqk and Akk with the
// direct ratio exp(min(G_c - G_i, 0)).  Gf is G as fp32 [64][128].
__device__ __forceinline__ void scores_exact(const unsigned char* sq, const unsigned char* sk,
                                             const float* Gf, float* Aq, float* Akk) {
  for (int idx = threadIdx.x; idx < C * C; idx += NT) {
    const int r = idx >> 6, i = idx & 63;
    float a = 0.f, l = 0.f;
    if (i <= r) {
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
    }
    Aq[sw64(r, i)] = a;
    Akk[sw64(r, i)] = (i < r) ? l : 0.f;
  }
}

// Store G (registers of prep) as fp32 [64][128] for scores_exact.
__device__ __forceinline__ void store_G(float* Gf, const float (&G)[4][8]) {
  const int cg = threadIdx.x & 15, rg4 = threadIdx.x >> 4;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) Gf[(4 * rg4 + i) * DK + 8 * cg + e] = G[i][e];
}

// T = (I + L)^-1 with L = diag(beta) Akk (strictly lower, 64 x 64), by blocked
// forward substitution on 16 x 16 blocks.  All threads take part; ends synced.
__device__ __forceinline__ void solve_T(const float* Akk, const float* beta_s, float* Tm) {
  const int tid = threadIdx.x;
  for (int idx = tid; idx < C * C; idx += NT) Tm[idx] = 0.f;  // the swizzle is a permutation
  __syncthreads();
  if (tid < 64) {  // diagonal blocks, one column per thread
    const int bb = tid >> 4, j = tid & 15, o = 16 * bb;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc += Akk[sw64(o + i, o + m)] * x[m];
      x[i] = ((i == j) ? 1.f : 0.f) - beta_s[o + i] * acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) Tm[sw64(o + i, o + j)] = x[i];
  }
  __syncthreads();
  for (int dl = 1; dl < 4; ++dl) {  // off-diagonal blocks by distance from the diagonal
    const int nblk = 4 - dl;
    float xs[3];
    for (int e = tid, n = 0; e < nblk * 256; e += NT, ++n) {
      const int bj = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int bi = bj + dl;
      float acc = 0.f;
      for (int m = 16 * bj; m < 16 * bi; ++m) acc += Akk[sw64(16 * bi + r, m)] * Tm[sw64(m, 16 * bj + cc)];
      xs[n] = beta_s[16 * bi + r] * acc;
    }
    __syncthreads();
    for (int e = tid, n = 0; e < nblk * 256; e += NT, ++n) {
      const int bj = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      Tm[sw64(16 * (bj + dl) + r, 16 * bj + cc)] = xs[n];
    }
    __syncthreads();
    for (int e = tid, n = 0; e < nblk * 256; e += NT, ++n) {
      const int bj = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int bi = bj + dl;
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) acc -= Tm[sw64(16 * bi + r, 16 * bi + m)] * Tm[sw64(16 * bi + m, 16 * bj + cc)];
      xs[n] = acc;
    }
    __syncthreads();
    for (int e = tid, n = 0; e < nblk * 256; e += NT, ++n) {
      const int bj = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      Tm[sw64(16 * (bj + dl) + r, 16 * bj + cc)] = xs[n];
    }
    __syncthreads();
  }
}

// Write row r, columns c0..c0+15 of a fp32 swizzled 64x64 matrix M (times
// colscale[c] when given) as bf16 into a CM tile with 64 columns at row `dst_row`.
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
