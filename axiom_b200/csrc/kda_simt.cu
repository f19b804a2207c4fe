// Exact-fp32 KDA chunked forward and backward on the CUDA cores.
//
// This is the library's general path: any dk, dv <= 128 (multiples of 8),
// chunk in {16, 32, 64}, fp32 or bf16 operands, all arithmetic in fp32 with
// the direct decay ratio exp(min(G_c - G_i, 0)).  It is the path for the
// fp32 parity configuration and for shapes the tensor-core kernels do not
// cover.  The per-chunk algebra is the reference's chunked_cc body
// (net/kda.py:669-702) and its analytic adjoint
// (net/kernels/kda_cc_fused_bwd.py:117-239), with g = log(alpha) as the input.
#include "kda_common.cuh"

namespace kda {
namespace {

constexpr int kFwdThreads = 256;
constexpr int kFwdSlice = 32;    // dv columns per forward CTA
constexpr int kBwdThreads = 512;

__device__ __forceinline__ size_t row_off(int b, int t, int h, int T, int H, int D) {
  return ((static_cast<size_t>(b) * T + t) * H + h) * D;
}

// ---------------------------------------------------------------------------
// forward: grid (dv slices, H, B); the state slice S[:, j0:j0+nj] in smem.
// ---------------------------------------------------------------------------
template <typename Tin, typename To, typename Tc>
__global__ void __launch_bounds__(kFwdThreads)
fwd_simt_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k, const Tin* __restrict__ v,
                const Tin* __restrict__ g, const Tin* __restrict__ beta,
                const float* __restrict__ s0, To* __restrict__ o, float* __restrict__ s_out,
                Tc* __restrict__ s_ckpt, int T, int H, int dk, int dv, int C,
                const int* __restrict__ cs) {
  const int j0 = blockIdx.x * kFwdSlice;
  const int nj = min(kFwdSlice, dv - j0);
  // (seq, h): batch row seq, or with packed sequences (cs: chunk offsets, B = 1)
  // the chunk range [cs[seq], cs[seq + 1]) of row 0
  const int h = blockIdx.y, seq = blockIdx.z;
  const int b = cs ? 0 : seq;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int ldk = dk + 1, ldc = C + 1, ldj = kFwdSlice;
  extern __shared__ float sm[];
  float* Qs = sm;                  // C x ldk : q, then Gamma*q
  float* Ks = Qs + C * ldk;        // C x ldk : k, then lambda*k
  float* Gs = Ks + C * ldk;        // C x ldk : g, then G = cumsum(g)
  float* Ws = Gs + C * ldk;        // C x ldk : Gamma*k*beta, then W
  float* Vs = Ws + C * ldk;        // C x ldj : v*beta, then U, then v~
  float* As = Vs + C * ldj;        // C x ldc : Aqk
  float* Ls = As + C * ldc;        // C x ldc : L
  float* Ss = Ls + C * ldc;        // dk x ldj: state slice
  float* Bs = Ss + dk * ldj;       // C
  float* gC = Bs + C;              // dk : Gamma_C

  const size_t sbase = (static_cast<size_t>(seq) * H + h) * dk * dv;
  for (int idx = tid; idx < dk * nj; idx += nt) {
    const int d = idx / nj, j = idx % nj;
    Ss[d * ldj + j] = s0 ? s0[sbase + static_cast<size_t>(d) * dv + j0 + j] : 0.f;
  }
  const int n_chunks = (T + C - 1) / C;
  const int c_beg = cs ? min(max(cs[seq], 0), n_chunks) : 0;  // clamped to the tensors
  const int c_end = cs ? min(max(cs[seq + 1], c_beg), n_chunks) : n_chunks;
  for (int c = c_beg; c < c_end; ++c) {
    const int t0 = c * C;
    __syncthreads();
    if (s_ckpt) {
      Tc* ck = s_ckpt + ((static_cast<size_t>(b) * H + h) * n_chunks + c) * dk * dv;
      for (int idx = tid; idx < dk * nj; idx += nt) {
        const int d = idx / nj, j = idx % nj;
        stf(ck + static_cast<size_t>(d) * dv + j0 + j, Ss[d * ldj + j]);
      }
    }
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk, t = t0 + r;
      const bool ok = t < T;
      const size_t off = row_off(b, t, h, T, H, dk) + d;
      Qs[r * ldk + d] = ok ? ldf(q + off) : 0.f;
      Ks[r * ldk + d] = ok ? ldf(k + off) : 0.f;
      Gs[r * ldk + d] = ok ? ldf(g + off) : 0.f;
    }
    for (int idx = tid; idx < C * nj; idx += nt) {
      const int r = idx / nj, j = idx % nj, t = t0 + r;
      Vs[r * ldj + j] = t < T ? ldf(v + row_off(b, t, h, T, H, dv) + j0 + j) : 0.f;
    }
    for (int r = tid; r < C; r += nt) {
      const int t = t0 + r;
      Bs[r] = t < T ? ldf(beta + (static_cast<size_t>(b) * T + t) * H + h) : 0.f;
    }
    __syncthreads();
    for (int d = tid; d < dk; d += nt) {  // G = cumsum over the chunk (net/kda.py:397-399)
      float acc = 0.f;
      for (int r = 0; r < C; ++r) { acc += Gs[r * ldk + d]; Gs[r * ldk + d] = acc; }
      gC[d] = expf(acc);
    }
    __syncthreads();
    // Aqk (lower, inclusive) and L = beta_r * Akk (strict), direct decay ratio.
    for (int idx = tid; idx < C * C; idx += nt) {
      const int r = idx / C, i = idx % C;
      float a = 0.f, l = 0.f;
      if (i <= r) {
        for (int d = 0; d < dk; ++d) {
          const float e = expf(fminf(Gs[r * ldk + d] - Gs[i * ldk + d], 0.f));
          const float ki = Ks[i * ldk + d] * e;
          a += Qs[r * ldk + d] * ki;
          l += Ks[r * ldk + d] * ki;
        }
      }
      As[r * ldc + i] = a;
      Ls[r * ldc + i] = (i < r) ? l * Bs[r] : 0.f;
    }
    __syncthreads();
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk;
      const float G = Gs[r * ldk + d];
      const float gam = expf(G);
      const float lam = expf(fminf(Gs[(C - 1) * ldk + d] - G, 0.f));
      const float kk = Ks[r * ldk + d];
      Ws[r * ldk + d] = gam * kk * Bs[r];
      Qs[r * ldk + d] *= gam;
      Ks[r * ldk + d] = lam * kk;
    }
    for (int idx = tid; idx < C * nj; idx += nt) {
      const int r = idx / nj, j = idx % nj;
      Vs[r * ldj + j] *= Bs[r];
    }
    __syncthreads();
    // (I + L) X = [Gamma k beta | v beta] by forward substitution, one column per thread.
    for (int col = tid; col < dk + nj; col += nt) {
      float* X = col < dk ? Ws + col : Vs + (col - dk);
      const int ld = col < dk ? ldk : ldj;
      for (int r = 1; r < C; ++r) {
        float acc = X[r * ld];
        for (int i = 0; i < r; ++i) acc -= Ls[r * ldc + i] * X[i * ld];
        X[r * ld] = acc;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < C * nj; idx += nt) {  // v~ = U - W S
      const int r = idx / nj, j = idx % nj;
      float acc = Vs[r * ldj + j];
      for (int d = 0; d < dk; ++d) acc -= Ws[r * ldk + d] * Ss[d * ldj + j];
      Vs[r * ldj + j] = acc;
    }
    __syncthreads();
    for (int idx = tid; idx < C * nj; idx += nt) {  // o = (Gamma q) S + Aqk v~
      const int r = idx / nj, j = idx % nj, t = t0 + r;
      float acc = 0.f;
      for (int d = 0; d < dk; ++d) acc += Qs[r * ldk + d] * Ss[d * ldj + j];
      for (int i = 0; i <= r; ++i) acc += As[r * ldc + i] * Vs[i * ldj + j];
      if (t < T) stf(o + row_off(b, t, h, T, H, dv) + j0 + j, acc);
    }
    __syncthreads();
    for (int idx = tid; idx < dk * nj; idx += nt) {  // S' = Gamma_C S + (lambda k)^T v~
      const int d = idx / nj, j = idx % nj;
      float acc = gC[d] * Ss[d * ldj + j];
      for (int r = 0; r < C; ++r) acc += Ks[r * ldk + d] * Vs[r * ldj + j];
      Ss[d * ldj + j] = acc;
    }
  }
  __syncthreads();
  if (s_out) {
    for (int idx = tid; idx < dk * nj; idx += nt) {
      const int d = idx / nj, j = idx % nj;
      s_out[sbase + static_cast<size_t>(d) * dv + j0 + j] = Ss[d * ldj + j];
    }
  }
}

// ---------------------------------------------------------------------------
// backward: grid (H, B); one CTA walks its chunks in reverse.  Large
// intermediates live in a per-CTA slice of the caller's workspace (they stay
// L2-resident); the adjoint follows net/kernels/kda_cc_fused_bwd.py:184-231.
// ---------------------------------------------------------------------------
struct BwdScratch {
  float *Q, *K, *G, *W, *X, *A, *L, *V, *U, *Vt, *Do, *dVt, *Sc, *dS, *dSn, *dQa, *dKa, *dGa,
      *Bs, *gC, *dgc, *dsum, *dBa;
};

__host__ __device__ inline size_t bwd_scratch_floats(int C, int dk, int dv) {
  const size_t cdk = static_cast<size_t>(C) * dk, cdv = static_cast<size_t>(C) * dv;
  return 8 * cdk + 2 * static_cast<size_t>(C) * C + 5 * cdv + 3 * static_cast<size_t>(dk) * dv +
         2 * C + 3 * dk + 64;
}

__device__ inline BwdScratch carve(float* base, int C, int dk, int dv) {
  BwdScratch s;
  const size_t cdk = static_cast<size_t>(C) * dk, cdv = static_cast<size_t>(C) * dv;
  float* p = base;
  s.Q = p; p += cdk; s.K = p; p += cdk; s.G = p; p += cdk; s.W = p; p += cdk; s.X = p; p += cdk;
  s.dQa = p; p += cdk; s.dKa = p; p += cdk; s.dGa = p; p += cdk;
  s.A = p; p += static_cast<size_t>(C) * C; s.L = p; p += static_cast<size_t>(C) * C;
  s.V = p; p += cdv; s.U = p; p += cdv; s.Vt = p; p += cdv; s.Do = p; p += cdv; s.dVt = p; p += cdv;
  s.Sc = p; p += static_cast<size_t>(dk) * dv; s.dS = p; p += static_cast<size_t>(dk) * dv;
  s.dSn = p; p += static_cast<size_t>(dk) * dv;
  s.Bs = p; p += C; s.dBa = p; p += C; s.gC = p; p += dk; s.dgc = p; p += dk; s.dsum = p;
  return s;
}

template <typename Tin, typename Td, typename Tc>
__global__ void __launch_bounds__(kBwdThreads)
bwd_simt_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k, const Tin* __restrict__ v,
                const Tin* __restrict__ g, const Tin* __restrict__ beta,
                const Tc* __restrict__ s_ckpt, const Td* __restrict__ dout,
                const float* __restrict__ dsT, Tin* __restrict__ dq, Tin* __restrict__ dkout,
                Tin* __restrict__ dvout, Tin* __restrict__ dg, Tin* __restrict__ dbeta,
                float* __restrict__ ds0, float* __restrict__ work, int T, int H, int dk, int dv,
                int C, int states_cm, const int* __restrict__ cs) {
  const int h = blockIdx.x, seq = blockIdx.y;
  const int b = cs ? 0 : seq;
  const int tid = threadIdx.x, nt = blockDim.x;
  const size_t unit = static_cast<size_t>(b) * H + h;     // checkpoint row
  const size_t sunit = static_cast<size_t>(seq) * H + h;  // state and scratch row
  BwdScratch s = carve(work + sunit * bwd_scratch_floats(C, dk, dv), C, dk, dv);
  const int n_chunks = (T + C - 1) / C;
  const int c_beg = cs ? min(max(cs[seq], 0), n_chunks) : 0;  // clamped to the tensors
  const int c_end = cs ? min(max(cs[seq + 1], c_beg), n_chunks) : n_chunks;
  const size_t sbase = sunit * dk * dv;
  for (int idx = tid; idx < dk * dv; idx += nt) s.dS[idx] = dsT ? dsT[sbase + idx] : 0.f;

  for (int c = c_end - 1; c >= c_beg; --c) {
    const int t0 = c * C;
    __syncthreads();
    // (1) loads
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk, t = t0 + r;
      const bool ok = t < T;
      const size_t off = row_off(b, t, h, T, H, dk) + d;
      s.Q[idx] = ok ? ldf(q + off) : 0.f;
      s.K[idx] = ok ? ldf(k + off) : 0.f;
      s.G[idx] = ok ? ldf(g + off) : 0.f;
      s.dQa[idx] = 0.f; s.dKa[idx] = 0.f; s.dGa[idx] = 0.f;
    }
    for (int idx = tid; idx < C * dv; idx += nt) {
      const int r = idx / dv, j = idx % dv, t = t0 + r;
      const bool ok = t < T;
      const size_t off = row_off(b, t, h, T, H, dv) + j;
      s.V[idx] = ok ? ldf(v + off) : 0.f;
      s.Do[idx] = ok ? ldf(dout + off) : 0.f;
    }
    for (int r = tid; r < C; r += nt) {
      const int t = t0 + r;
      s.Bs[r] = t < T ? ldf(beta + (static_cast<size_t>(b) * T + t) * H + h) : 0.f;
      s.dBa[r] = 0.f;
    }
    {
      const Tc* ck = s_ckpt + (unit * n_chunks + c) * dk * dv;
      // states_cm: the entry is an 8 x 8 core-matrix operand image (tensor-core forward)
      for (int idx = tid; idx < dk * dv; idx += nt) {
        const int r = idx / dv, j = idx % dv;
        const int e = states_cm ? (((r >> 3) * (dv >> 3) + (j >> 3)) << 6) + ((r & 7) << 3) + (j & 7) : idx;
        s.Sc[idx] = ldf(ck + e);
      }
    }
    __syncthreads();
    // (2) G = cumsum(g)
    for (int d = tid; d < dk; d += nt) {
      float acc = 0.f;
      for (int r = 0; r < C; ++r) { acc += s.G[r * dk + d]; s.G[r * dk + d] = acc; }
      s.gC[d] = expf(acc);
    }
    __syncthreads();
    // (3) scores and (4) right-hand sides
    for (int idx = tid; idx < C * C; idx += nt) {
      const int r = idx / C, i = idx % C;
      float a = 0.f, l = 0.f;
      if (i <= r) {
        for (int d = 0; d < dk; ++d) {
          const float e = expf(fminf(s.G[r * dk + d] - s.G[i * dk + d], 0.f));
          const float ki = s.K[i * dk + d] * e;
          a += s.Q[r * dk + d] * ki;
          l += s.K[r * dk + d] * ki;
        }
      }
      s.A[idx] = a;
      s.L[idx] = (i < r) ? l * s.Bs[r] : 0.f;
    }
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk;
      s.W[idx] = expf(s.G[idx]) * s.K[idx] * s.Bs[r];
    }
    for (int idx = tid; idx < C * dv; idx += nt) s.U[idx] = s.V[idx] * s.Bs[idx / dv];
    __syncthreads();
    // (5) forward substitution: W = (I+L)^{-1} Gamma k beta, U = (I+L)^{-1} v beta
    for (int col = tid; col < dk + dv; col += nt) {
      float* X = col < dk ? s.W + col : s.U + (col - dk);
      const int ld = col < dk ? dk : dv;
      for (int r = 1; r < C; ++r) {
        float acc = X[r * ld];
        for (int i = 0; i < r; ++i) acc -= s.L[r * C + i] * X[i * ld];
        X[r * ld] = acc;
      }
    }
    __syncthreads();
    // (6) v~ = U - W S
    for (int idx = tid; idx < C * dv; idx += nt) {
      const int r = idx / dv, j = idx % dv;
      float acc = s.U[idx];
      for (int d = 0; d < dk; ++d) acc -= s.W[r * dk + d] * s.Sc[d * dv + j];
      s.Vt[idx] = acc;
    }
    __syncthreads();
    // (7) dv~ = Y dS' + Aqk^T do  with Y = lambda k
    for (int idx = tid; idx < C * dv; idx += nt) {
      const int r = idx / dv, j = idx % dv;
      float acc = 0.f;
      for (int d = 0; d < dk; ++d) {
        const float lam = expf(fminf(s.G[(C - 1) * dk + d] - s.G[r * dk + d], 0.f));
        acc += lam * s.K[r * dk + d] * s.dS[d * dv + j];
      }
      for (int i = r; i < C; ++i) acc += s.A[i * C + r] * s.Do[i * dv + j];
      s.dVt[idx] = acc;
    }
    __syncthreads();
    // (8) dS_in = Gamma_C dS' + (Gamma q)^T do - W^T dv~ ; dgc = rowsum(S * dS')
    for (int idx = tid; idx < dk * dv; idx += nt) {
      const int d = idx / dv, j = idx % dv;
      float acc = s.gC[d] * s.dS[idx];
      for (int r = 0; r < C; ++r)
        acc += expf(s.G[r * dk + d]) * s.Q[r * dk + d] * s.Do[r * dv + j] -
               s.W[r * dk + d] * s.dVt[r * dv + j];
      s.dSn[idx] = acc;
    }
    for (int d = tid; d < dk; d += nt) {
      float acc = 0.f;
      for (int j = 0; j < dv; ++j) acc += s.Sc[d * dv + j] * s.dS[d * dv + j];
      s.dgc[d] = acc;
    }
    // (9) dY, dgq terms (row-owned), dz stored in X for the chunk-sum
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk;
      float dY = 0.f, dgq = 0.f;
      for (int j = 0; j < dv; ++j) {
        dY += s.Vt[r * dv + j] * s.dS[d * dv + j];
        dgq += s.Do[r * dv + j] * s.Sc[d * dv + j];
      }
      const float G = s.G[idx];
      const float lam = expf(fminf(s.G[(C - 1) * dk + d] - G, 0.f));
      const float gam = expf(G);
      const float kk = s.K[idx];
      const float dz = dY * kk * lam;
      s.X[idx] = dz;
      s.dKa[idx] += dY * lam;
      s.dGa[idx] += -dz + dgq * s.Q[idx] * gam;
      s.dQa[idx] += dgq * gam;
    }
    // (10) dAqk = tril(do v~^T) into A (Aqk is consumed)
    __syncthreads();
    for (int idx = tid; idx < C * C; idx += nt) {
      const int r = idx / C, i = idx % C;
      float acc = 0.f;
      if (i <= r)
        for (int j = 0; j < dv; ++j) acc += s.Do[r * dv + j] * s.Vt[i * dv + j];
      s.A[idx] = acc;
    }
    for (int d = tid; d < dk; d += nt) {
      float acc = 0.f;
      for (int r = 0; r < C; ++r) acc += s.X[r * dk + d];
      s.dsum[d] = acc;
    }
    __syncthreads();
    // (11) dW = -dv~ S^T into X
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk;
      float acc = 0.f;
      for (int j = 0; j < dv; ++j) acc += s.dVt[r * dv + j] * s.Sc[d * dv + j];
      s.X[idx] = -acc;
    }
    __syncthreads();
    // (12) (I+L)^T Y = [dW | dv~] by backward substitution: Yw in X, Yu in dVt
    for (int col = tid; col < dk + dv; col += nt) {
      float* Y = col < dk ? s.X + col : s.dVt + (col - dk);
      const int ld = col < dk ? dk : dv;
      for (int r = C - 2; r >= 0; --r) {
        float acc = Y[r * ld];
        for (int i = r + 1; i < C; ++i) acc -= s.L[i * C + r] * Y[i * ld];
        Y[r * ld] = acc;
      }
    }
    __syncthreads();
    // (13) dL = -strict(Yw W^T + Yu U^T) into L (L is consumed)
    for (int idx = tid; idx < C * C; idx += nt) {
      const int r = idx / C, i = idx % C;
      float acc = 0.f;
      if (i < r) {
        for (int d = 0; d < dk; ++d) acc += s.X[r * dk + d] * s.W[i * dk + d];
        for (int j = 0; j < dv; ++j) acc += s.dVt[r * dv + j] * s.U[i * dv + j];
      }
      s.L[idx] = -acc;
    }
    __syncthreads();  // (13) read Yw, Yu of every row; (14) overwrites them with dbeta terms
    // (14) Yw / Yu terms; dv = Yu beta
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk;
      const float yw = s.X[idx], gam = expf(s.G[idx]), kk = s.K[idx], bb = s.Bs[r];
      s.dKa[idx] += yw * gam * bb;
      s.dGa[idx] += yw * kk * bb * gam;
      s.X[idx] = yw * gam * kk;  // dbeta term (Yw is dead after this)
    }
    for (int idx = tid; idx < C * dv; idx += nt) {
      const int r = idx / dv, j = idx % dv, t = t0 + r;
      const float dvt = s.dVt[idx];
      if (t < T) stf(dvout + row_off(b, t, h, T, H, dv) + j, dvt * s.Bs[r]);
      s.dVt[idx] = dvt * s.V[idx];  // dbeta term (dV~ is dead after this)
    }
    __syncthreads();
    // (15) score adjoints (row side then column side), direct decay ratio
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk;
      const float Gr = s.G[idx];
      float dra = 0.f, drk = 0.f;
      for (int i = 0; i <= r; ++i) {
        const float ke = s.K[i * dk + d] * expf(fminf(Gr - s.G[i * dk + d], 0.f));
        dra += s.A[r * C + i] * ke;
        drk += s.L[r * C + i] * ke;
      }
      const float kk = s.K[idx], bb = s.Bs[r];
      s.dQa[idx] += dra;
      s.dKa[idx] += drk * bb;
      s.dGa[idx] += dra * s.Q[idx] + drk * kk * bb;
      s.X[idx] += drk * kk;
    }
    __syncthreads();
    // dbeta: each row's terms summed by one thread in a fixed order (deterministic)
    for (int r = tid; r < C; r += nt) {
      float acc = 0.f;
      for (int d = 0; d < dk; ++d) acc += s.X[r * dk + d];
      for (int j = 0; j < dv; ++j) acc += s.dVt[r * dv + j];
      s.dBa[r] = acc;
    }
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int i = idx / dk, d = idx % dk;
      const float Gi = s.G[idx];
      float dca = 0.f, dck = 0.f;
      for (int r = i; r < C; ++r) {
        const float e = expf(fminf(s.G[r * dk + d] - Gi, 0.f));
        dca += s.A[r * C + i] * s.Q[r * dk + d] * e;
        dck += s.L[r * C + i] * s.K[r * dk + d] * s.Bs[r] * e;
      }
      s.dKa[idx] += dca + dck;
      s.dGa[idx] -= (dca + dck) * s.K[idx];
    }
    __syncthreads();
    // (16) dg = reverse cumsum of dG + chunk-sum terms; (17) writes
    for (int d = tid; d < dk; d += nt) {
      float acc = s.dsum[d] + s.gC[d] * s.dgc[d];
      for (int r = C - 1; r >= 0; --r) {
        acc += s.dGa[r * dk + d];
        s.X[r * dk + d] = acc;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < C * dk; idx += nt) {
      const int r = idx / dk, d = idx % dk, t = t0 + r;
      if (t < T) {
        const size_t off = row_off(b, t, h, T, H, dk) + d;
        stf(dq + off, s.dQa[idx]);
        stf(dkout + off, s.dKa[idx]);
        stf(dg + off, s.X[idx]);
      }
    }
    for (int r = tid; r < C; r += nt) {
      const int t = t0 + r;
      if (t < T) stf(dbeta + (static_cast<size_t>(b) * T + t) * H + h, s.dBa[r]);
    }
    for (int idx = tid; idx < dk * dv; idx += nt) s.dS[idx] = s.dSn[idx];
  }
  __syncthreads();
  if (ds0)
    for (int idx = tid; idx < dk * dv; idx += nt) ds0[sbase + idx] = s.dS[idx];
}

template <typename Tin, typename To, typename Tc>
int fwd_launch_t(const void* q, const void* k, const void* v, const void* g, const void* beta,
                 const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
                 int dk, int dv, int C, const int* cs, int n_seqs, cudaStream_t st) {
  static std::atomic<bool> done[64];
  const int bytes = static_cast<int>(sizeof(float)) *
                    (4 * C * (dk + 1) + C * kFwdSlice + 2 * C * (C + 1) + dk * kFwdSlice + C + dk);
  auto kern = fwd_simt_kernel<Tin, To, Tc>;
  int rc = ensure_smem(kern, 227 * 1024, done);
  if (rc != KDA_OK) return rc;
  dim3 grid((dv + kFwdSlice - 1) / kFwdSlice, H, cs ? n_seqs : B);
  kern<<<grid, kFwdThreads, bytes, st>>>(
      static_cast<const Tin*>(q), static_cast<const Tin*>(k), static_cast<const Tin*>(v),
      static_cast<const Tin*>(g), static_cast<const Tin*>(beta), s0, static_cast<To*>(o), s_out,
      static_cast<Tc*>(s_ckpt), T, H, dk, dv, C, cs);
  return launch_status();
}

template <typename Tin, typename Td, typename Tc>
int bwd_launch_t(const void* q, const void* k, const void* v, const void* g, const void* beta,
                 const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
                 void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T, int H,
                 int dk, int dv, int C, int states_cm, const int* cs, int n_seqs, cudaStream_t st) {
  dim3 grid(H, cs ? n_seqs : B);
  bwd_simt_kernel<Tin, Td, Tc><<<grid, kBwdThreads, 0, st>>>(
      static_cast<const Tin*>(q), static_cast<const Tin*>(k), static_cast<const Tin*>(v),
      static_cast<const Tin*>(g), static_cast<const Tin*>(beta), static_cast<const Tc*>(s_ckpt),
      static_cast<const Td*>(dout), dsT, static_cast<Tin*>(dq), static_cast<Tin*>(dk_),
      static_cast<Tin*>(dv_), static_cast<Tin*>(dg), static_cast<Tin*>(dbeta), ds0,
      static_cast<float*>(work), T, H, dk, dv, C, states_cm, cs);
  return launch_status();
}

}  // namespace

size_t simt_bwd_workspace_bytes(int B, int H, int dk, int dv, int C) {
  return static_cast<size_t>(B) * H * bwd_scratch_floats(C, dk, dv) * sizeof(float);
}

int simt_fwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
                    int dk, int dv, int C, int in_dt, int o_dt, int ck_dt, const int* cs, int n_seqs,
                    cudaStream_t st) {
#define KDA_FWD_CASE(I, O, K, TI, TO, TK)                                                     \
  if (in_dt == I && o_dt == O && ck_dt == K)                                                 \
    return fwd_launch_t<TI, TO, TK>(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, dk, dv, C, cs, n_seqs, st);
  KDA_FWD_CASE(KDA_F32, KDA_F32, KDA_F32, float, float, float)
  KDA_FWD_CASE(KDA_F32, KDA_F32, KDA_BF16, float, float, bf16)
  KDA_FWD_CASE(KDA_F32, KDA_BF16, KDA_F32, float, bf16, float)
  KDA_FWD_CASE(KDA_F32, KDA_BF16, KDA_BF16, float, bf16, bf16)
  KDA_FWD_CASE(KDA_BF16, KDA_F32, KDA_F32, bf16, float, float)
  KDA_FWD_CASE(KDA_BF16, KDA_F32, KDA_BF16, bf16, float, bf16)
  KDA_FWD_CASE(KDA_BF16, KDA_BF16, KDA_F32, bf16, bf16, float)
  KDA_FWD_CASE(KDA_BF16, KDA_BF16, KDA_BF16, bf16, bf16, bf16)
#undef KDA_FWD_CASE
  return KDA_ERR_DTYPE;
}

int simt_bwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
                    void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T,
                    int H, int dk, int dv, int C, int in_dt, int do_dt, int ck_dt,
                    int states_cm, const int* cs, int n_seqs, cudaStream_t st) {
#define KDA_BWD_CASE(I, D, K, TI, TD, TK)                                                     \
  if (in_dt == I && do_dt == D && ck_dt == K)                                                \
    return bwd_launch_t<TI, TD, TK>(q, k, v, g, beta, s_ckpt, dout, dsT, dq, dk_, dv_, dg,   \
                                    dbeta, ds0, work, B, T, H, dk, dv, C, states_cm, cs, n_seqs, st);
  KDA_BWD_CASE(KDA_F32, KDA_F32, KDA_F32, float, float, float)
  KDA_BWD_CASE(KDA_F32, KDA_F32, KDA_BF16, float, float, bf16)
  KDA_BWD_CASE(KDA_F32, KDA_BF16, KDA_F32, float, bf16, float)
  KDA_BWD_CASE(KDA_F32, KDA_BF16, KDA_BF16, float, bf16, bf16)
  KDA_BWD_CASE(KDA_BF16, KDA_F32, KDA_F32, bf16, float, float)
  KDA_BWD_CASE(KDA_BF16, KDA_F32, KDA_BF16, bf16, float, bf16)
  KDA_BWD_CASE(KDA_BF16, KDA_BF16, KDA_F32, bf16, bf16, float)
  KDA_BWD_CASE(KDA_BF16, KDA_BF16, KDA_BF16, bf16, bf16, bf16)
#undef KDA_BWD_CASE
  return KDA_ERR_DTYPE;
}

}  // namespace kda
