// Recurrent single-token decode step of KDA (HBM-bandwidth bound).
//
// Math (net/kda.py:298-310 and :293):
//   r  = (alpha*k)^T S                      (dv)
//   S' = diag(alpha) S + beta k (v - r)^T   (dk x dv)
//   o  = S'^T q                             (dv)
// with alpha = exp(g).  One CTA owns one (sequence, head) state and passes
// over it exactly once: every thread keeps its rows x 4 columns of S in
// registers between the read and the write, so the state moves through HBM
// once in each direction (the algorithmic minimum).  Loads and stores are
// 128-bit and a warp covers whole 512-byte state rows, so every request is
// fully coalesced.
#include "kda_common.cuh"

namespace kda {
namespace {

constexpr int kDecodeThreads = 256;

template <int DK, int DV, typename Tin, typename To>
__global__ void __launch_bounds__(kDecodeThreads, 2)
decode_kernel(float* __restrict__ S, const Tin* __restrict__ q, const Tin* __restrict__ k,
              const Tin* __restrict__ v, const Tin* __restrict__ g,
              const Tin* __restrict__ beta, To* __restrict__ o) {
  constexpr int TPR = DV / 4;                 // threads per state row
  constexpr int RPP = kDecodeThreads / TPR;   // rows per pass
  constexpr int NR = DK / RPP;                // rows per thread
  static_assert(DK % RPP == 0, "dk must be a multiple of the rows per pass");

  __shared__ float s_ak[DK];   // alpha * k
  __shared__ float s_a[DK];    // alpha
  __shared__ float s_bk[DK];   // beta * k
  __shared__ float s_q[DK];
  __shared__ float s_red[RPP][DV];

  const int n = blockIdx.x;
  const int tid = threadIdx.x;
  const int col = (tid % TPR) * 4;
  const int row0 = tid / TPR;

  float4* Sn = reinterpret_cast<float4*>(S + static_cast<size_t>(n) * DK * DV);

  // Issue the whole state read first: NR independent 16-byte loads per thread.
  float4 s[NR];
#pragma unroll
  for (int m = 0; m < NR; ++m) s[m] = Sn[((row0 + m * RPP) * DV + col) / 4];

  const float b = ldf(beta + n);
  for (int d = tid; d < DK; d += kDecodeThreads) {
    const size_t off = static_cast<size_t>(n) * DK + d;
    const float a = __expf(ldf(g + off));
    const float kk = ldf(k + off);
    s_a[d] = a;
    s_ak[d] = a * kk;
    s_bk[d] = b * kk;
    s_q[d] = ldf(q + off);
  }
  __syncthreads();

  // r = (alpha*k)^T S : partial over this thread's rows, then across row groups.
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const float w = s_ak[row0 + m * RPP];
    r.x += w * s[m].x; r.y += w * s[m].y; r.z += w * s[m].z; r.w += w * s[m].w;
  }
  *reinterpret_cast<float4*>(&s_red[row0][col]) = r;
  __syncthreads();
  r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int p = 0; p < RPP; ++p) {
    const float4 t = *reinterpret_cast<const float4*>(&s_red[p][col]);
    r.x += t.x; r.y += t.y; r.z += t.z; r.w += t.w;
  }
  float4 u;  // v - r for this thread's columns
  {
    const size_t vo = static_cast<size_t>(n) * DV + col;
    u.x = ldf(v + vo + 0) - r.x; u.y = ldf(v + vo + 1) - r.y;
    u.z = ldf(v + vo + 2) - r.z; u.w = ldf(v + vo + 3) - r.w;
  }

  // S' = alpha S + (beta k) u^T, written back; o partial = sum_d q_d S'[d].
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const int d = row0 + m * RPP;
    const float a = s_a[d], bk = s_bk[d], qd = s_q[d];
    float4 t;
    t.x = a * s[m].x + bk * u.x; t.y = a * s[m].y + bk * u.y;
    t.z = a * s[m].z + bk * u.z; t.w = a * s[m].w + bk * u.w;
    Sn[(d * DV + col) / 4] = t;
    acc.x += qd * t.x; acc.y += qd * t.y; acc.z += qd * t.z; acc.w += qd * t.w;
  }
  __syncthreads();  // every thread has finished reading s_red for r
  *reinterpret_cast<float4*>(&s_red[row0][col]) = acc;
  __syncthreads();
  if (tid < TPR) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < RPP; ++p) {
      const float4 x = *reinterpret_cast<const float4*>(&s_red[p][col]);
      t.x += x.x; t.y += x.y; t.z += x.z; t.w += x.w;
    }
    To* on = o + static_cast<size_t>(n) * DV + col;
    stf(on + 0, t.x); stf(on + 1, t.y); stf(on + 2, t.z); stf(on + 3, t.w);
  }
}

template <int DK, int DV, typename Tin, typename To>
int launch(float* S, const void* q, const void* k, const void* v, const void* g,
           const void* beta, void* o, int N, cudaStream_t st) {
  decode_kernel<DK, DV, Tin, To><<<N, kDecodeThreads, 0, st>>>(
      S, static_cast<const Tin*>(q), static_cast<const Tin*>(k), static_cast<const Tin*>(v),
      static_cast<const Tin*>(g), static_cast<const Tin*>(beta), static_cast<To*>(o));
  return launch_status();
}

template <int DK, int DV>
int dispatch_types(float* S, const void* q, const void* k, const void* v, const void* g,
                   const void* beta, void* o, int N, int in_dt, int o_dt, cudaStream_t st) {
  if (in_dt == KDA_BF16 && o_dt == KDA_BF16) return launch<DK, DV, bf16, bf16>(S, q, k, v, g, beta, o, N, st);
  if (in_dt == KDA_BF16 && o_dt == KDA_F32) return launch<DK, DV, bf16, float>(S, q, k, v, g, beta, o, N, st);
  if (in_dt == KDA_F32 && o_dt == KDA_F32) return launch<DK, DV, float, float>(S, q, k, v, g, beta, o, N, st);
  if (in_dt == KDA_F32 && o_dt == KDA_BF16) return launch<DK, DV, float, bf16>(S, q, k, v, g, beta, o, N, st);
  return KDA_ERR_DTYPE;
}

}  // namespace

int decode_launch(float* S, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, void* o, int N, int dk, int dv, int in_dt, int o_dt,
                  cudaStream_t st) {
  if (N == 0) return KDA_OK;
  if (dk == 128 && dv == 128) return dispatch_types<128, 128>(S, q, k, v, g, beta, o, N, in_dt, o_dt, st);
  if (dk == 64 && dv == 128) return dispatch_types<64, 128>(S, q, k, v, g, beta, o, N, in_dt, o_dt, st);
  if (dk == 128 && dv == 64) return dispatch_types<128, 64>(S, q, k, v, g, beta, o, N, in_dt, o_dt, st);
  if (dk == 64 && dv == 64) return dispatch_types<64, 64>(S, q, k, v, g, beta, o, N, in_dt, o_dt, st);
  return KDA_ERR_SHAPE;
}

}  // namespace kda
