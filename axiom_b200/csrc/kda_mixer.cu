// Per-token work around the KDA core (all HBM-bandwidth bound):
//
//   * prologue fwd/bwd: causal depthwise short conv + Swish + L2 norm (q, k),
//     conv + Swish (v), sigmoid(beta), decay gate  (net/shortconv.py:14-30,
//     net/kda.py:169-180, :194-203, net/norm.py:15-61);
//   * output gate fwd/bwd: sigmoid(gate) * headwise_rms_norm(o)
//     (net/kda.py:206-214, net/norm.py:70-73);
//   * fused decode step: recurrent_step without the projection GEMMs
//     (net/kda.py:277-295, net/shortconv.py:33-53).
//
// Prologue mapping: a warp owns a strip of 256 consecutive tokens of one head
// and one tensor (a block's warps share the head and tensor; blockIdx.z picks
// q, k, v or the gates), each lane 2 or 4 adjacent channels, so a row of the
// head (128 or 256 bytes) is one coalesced warp access and the L2 norm is a
// warp reduction.  The strip's rows stream through a per-warp shared-memory
// ring filled by cp.async (several batches in flight without holding
// registers); the conv window lives in registers, so every input is read once
// plus K-1 halo rows per strip (L2 hits).  The L2 norms of a batch of tokens
// are one column-sum reduction.  The backward sweeps each strip from its end
// (plus K-1 halo tokens whose conv cotangents its inputs need) to its start,
// so dx[t] = sum_i w[i] dc[t+i] is complete when t is reached; weight
// gradients are reduced per block in shared memory, then over blocks in a
// fixed order by a second kernel (deterministic).
#include <climits>
#include <type_traits>

#include "kda_common.cuh"
#include "kda_mixer.h"
#include "kda_tc.cuh"

namespace kda {
namespace {

constexpr int kStrip = 256;  // tokens per warp strip (a long sweep amortises the ring fill)
constexpr int kWarps = 8;    // warps per prologue forward block
constexpr int kBwdWarps = 4; // warps per backward block (more registers per thread)
constexpr int kPre = 8;      // tokens per forward batch
constexpr int kStages = 4;   // forward ring stages per warp (3 batches in flight)
constexpr int kBwStages = 6; // backward ring stages per warp
constexpr int kBw = 4;       // tokens per backward batch
constexpr float kL2Eps = 1e-12f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Sigmoid at the precision its consumer keeps: with FAST (results rounded to
// bf16) one tanh.approx, sigmoid(x) = (1 + tanh(x / 2)) / 2, whose absolute
// error (below 2^-11) is under bf16's resolution; else exp and reciprocal.
template <bool FAST>
__device__ __forceinline__ float sigm(float x) {
  if constexpr (FAST) return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
  else return sigmoidf_(x);
}
__device__ __forceinline__ float softplusf_(float x) { return fmaxf(x, 0.f) + log1pf(__expf(-fabsf(x))); }
// Softplus at the precision its consumer keeps: with FAST (bf16 results)
// log(1 + e^-|x|) through the fast logarithm; its error (absolute, below
// e^-|x| ulp-scale) is under bf16's resolution of the result.
template <bool FAST>
__device__ __forceinline__ float softp(float x) {
  if constexpr (FAST) return fmaxf(x, 0.f) + __logf(1.f + __expf(-fabsf(x)));
  else return softplusf_(x);
}

// Two fp32 lanes per instruction (sm_100 packed f32x2 arithmetic).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

// Swish x sigmoid(x) of two lanes.  FAST (bf16 consumers): with h = x / 2,
// x sigmoid(x) = h + h tanh(h), one tanh.approx per element (absolute error of
// the sigmoid factor below 2^-12, as in sigm<true>).
template <bool FAST>
__device__ __forceinline__ float2 swish2(float2 x) {
  if constexpr (FAST) {
    const float2 h = fmul2(x, f2(0.5f));
    return ffma2(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h);
  } else {
    return make_float2(x.x * sigmoidf_(x.x), x.y * sigmoidf_(x.y));
  }
}
// Swish and its derivative d/dx [x sigmoid(x)] = sigmoid(x) (1 + x (1 - sigmoid(x))).
template <bool FAST>
__device__ __forceinline__ void swish_grad2(float2 x, float2& s, float2& ds) {
  float2 sig;
  if constexpr (FAST) {
    const float2 h = fmul2(x, f2(0.5f));
    const float2 th = make_float2(tanh_approx(h.x), tanh_approx(h.y));
    s = ffma2(h, th, h);
    sig = ffma2(th, f2(0.5f), f2(0.5f));
  } else {
    sig = make_float2(sigmoidf_(x.x), sigmoidf_(x.y));
    s = fmul2(x, sig);
  }
  const float2 om = ffma2(sig, f2(-1.f), f2(1.f));
  ds = fmul2(sig, ffma2(x, om, f2(1.f)));
}

// CPL (2 or 4) consecutive elements <-> floats, one vector access
template <int CPL>
__device__ __forceinline__ void ldv(const float* p, float (&x)[CPL]) {
  if constexpr (CPL == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
  } else {
    const float2 t = *reinterpret_cast<const float2*>(p);
    x[0] = t.x; x[1] = t.y;
  }
}
template <int CPL>
__device__ __forceinline__ void ldv(const bf16* p, float (&x)[CPL]) {
  if constexpr (CPL == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
    x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
  } else {
    const uint32_t t = *reinterpret_cast<const uint32_t*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t);
    x[0] = __low2float(a); x[1] = __high2float(a);
  }
}
template <int CPL>
__device__ __forceinline__ void stv(float* p, const float (&x)[CPL]) {
  if constexpr (CPL == 4) *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  else *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
}
template <int CPL>
__device__ __forceinline__ void stv(bf16* p, const float (&x)[CPL]) {
  if constexpr (CPL == 4) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]), b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 t;
    t.x = *reinterpret_cast<const uint32_t*>(&a);
    t.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
  } else {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
    *reinterpret_cast<uint32_t*>(p) = *reinterpret_cast<const uint32_t*>(&a);
  }
}

// A row slice of CPL elements as loaded (packed bf16 pairs or floats), kept
// packed while in flight and converted at use.
template <typename T, int CPL> struct Raw;
template <> struct Raw<bf16, 4> { uint2 v; };
template <> struct Raw<bf16, 2> { uint32_t v; };
template <> struct Raw<float, 4> { float4 v; };
template <> struct Raw<float, 2> { float2 v; };
template <int CPL, typename T>
__device__ __forceinline__ Raw<T, CPL> ldr(const T* p) {
  Raw<T, CPL> r;
  r.v = *reinterpret_cast<const decltype(r.v)*>(p);
  return r;
}
template <int CPL, typename T>
__device__ __forceinline__ void cvt(const Raw<T, CPL>& r, float (&x)[CPL]) {
  if constexpr (std::is_same<T, float>::value) {
    const float* f = reinterpret_cast<const float*>(&r.v);
#pragma unroll
    for (int c = 0; c < CPL; ++c) x[c] = f[c];
  } else {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&r.v);
#pragma unroll
    for (int c = 0; c < CPL / 2; ++c) {
      x[2 * c] = __low2float(p[c]);
      x[2 * c + 1] = __high2float(p[c]);
    }
  }
}

// One stage of a warp's shared-memory ring: NROWS rows of RB bytes, row r
// copied from src(r) with cp.async (16 bytes per lane and copy), or
// zero-filled when src(r) is null.  Rows in flight cost no registers, so a
// warp keeps several batches of its strip in flight.
template <int RB, int NROWS, typename Src>
__device__ __forceinline__ void ring_fill(unsigned char* dst, int lane, const void* any_valid, Src src) {
  constexpr int CPR = RB / 16;
  constexpr int N = NROWS * CPR;
  static_assert(N % 32 == 0, "whole warp copies");
#pragma unroll
  for (int it = 0; it < N / 32; ++it) {
    const int j = lane + 32 * it;
    const int r = j / CPR, c = j % CPR;
    const unsigned char* p = static_cast<const unsigned char*>(src(r));
    tc::cp_async16(dst + r * RB + c * 16, p ? p + c * 16 : any_valid, p != nullptr);
  }
}

// The same for NROWS rows all in range, `stride` bytes apart (negative: rows
// descending): `first` is this lane's chunk of row 0 (the row's address plus
// lane_src_off), `dst` its chunk in the stage (the stage's shared address plus
// lane_dst_off).  Lane l copies chunk l % CPR of rows l / CPR + RSTEP i.
template <int RB, int NROWS>
__device__ __forceinline__ void ring_fill_rows(uint32_t dst, const unsigned char* first, long long stride) {
  constexpr int CPR = RB / 16, RSTEP = 32 / CPR;
  static_assert(32 % CPR == 0 && NROWS % RSTEP == 0, "whole warp copies");
#pragma unroll
  for (int i = 0; i < NROWS / RSTEP; ++i) tc::cp_async16_s(dst + i * RSTEP * RB, first + i * RSTEP * stride);
}
template <int RB>
__device__ __forceinline__ long long lane_src_off(int lane, long long stride) {
  return (lane / (RB / 16)) * stride + (lane % (RB / 16)) * 16;
}
template <int RB>
__device__ __forceinline__ uint32_t lane_dst_off(int lane) {
  return (lane / (RB / 16)) * RB + (lane % (RB / 16)) * 16;
}

// CPL elements of this lane from a staged row (lane l holds elements [l CPL, l CPL + CPL)).
template <int CPL, typename T>
__device__ __forceinline__ void ld_row(const unsigned char* row, int lane, float (&x)[CPL]) {
  Raw<T, CPL> r;
  r.v = *reinterpret_cast<const decltype(r.v)*>(row + lane * CPL * sizeof(T));
  cvt<CPL>(r, x);
}

struct ProArgs {
  const void* x[4];  // qp, kp, vp, z
  const void* beta_logit;
  const float* w[3];  // conv_q, conv_k, conv_v
  const float* b_gate;
  const float* A;
  float g_min;
  int gate_kind;
  const float* st_in;
  float* st_out;
  const int* cu;
  int n_seqs;
  const int* out_rows;  // packed: row of each sequence's first token in q, k, v, g (and their cotangents)
  void* y[4];  // q, k, v, g
  void* beta;
  // backward
  const void* dy[4];  // dq, dk, dv, dg
  const void* dbeta;
  void* dx[4];  // dqp, dkp, dvp, dz
  void* dbeta_logit;
  float* dst;   // dconv_state_in
  float* ws;    // per-block partial sums
  int ws_stride;
  int B, T, H, dk, dv, K;
  int spb;      // strips per batch row
  int n_strips;
  int roles;    // tensor of each blockIdx.z, 4 bits each
  int head_x;   // forward grid (heads, strip groups): the heads of one token range run together
};

// Element r (0..3) of a 4-pointer parameter array by selects: indexing the
// kernel-parameter array with a runtime index would copy it to local memory.
template <typename P>
__device__ __forceinline__ P pick(const P (&p)[4], int r) {
  return r == 0 ? p[0] : r == 1 ? p[1] : r == 2 ? p[2] : p[3];
}
template <typename P>
__device__ __forceinline__ P pick(const P (&p)[3], int r) {
  return r == 0 ? p[0] : r == 1 ? p[1] : p[2];
}

// Index of the packed sequence holding token t (cu_seqlens[i] <= t < cu_seqlens[i+1]).
__device__ __forceinline__ int seq_of(const int* cu, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu + mid) <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Row of packed token t in the outputs (and, backward, the output cotangents):
// t itself, or with out_rows the chunk-aligned row of its sequence, for tokens
// visited in increasing (UP) or decreasing order.  The sequence and its row
// shift change only at sequence boundaries, so a call is a compare, with a
// reload when a boundary is crossed (no search per token).
template <bool UP>
struct RowWalk {
  const int* cu;
  const int* rows;
  int n, s, edge, shift;
  __device__ void init(const ProArgs& a, int t) {
    cu = a.cu;
    rows = a.out_rows;
    n = a.n_seqs;
    s = seq_of(cu, n, t);
    set();
  }
  __device__ void set() {
    edge = UP ? __ldg(cu + s + 1) : __ldg(cu + s);  // first token of the next / this sequence
    shift = rows ? __ldg(rows + s) - __ldg(cu + s) : 0;
  }
  __device__ int operator()(int t) {
    if (UP) {
      while (t >= edge && s < n - 1) {
        ++s;
        set();
      }
    } else {
      while (t < edge && s > 0) {
        --s;
        set();
      }
    }
    return t + shift;
  }
};

// Zeroes this lane's channels of the pad rows of every sequence ending in
// (t0, t1]: the rows between its last token and the next sequence's first row.
template <int CPL, typename T>
__device__ void zero_pads(const ProArgs& a, T* base, int HD, int t0, int t1) {
  if (!a.out_rows) return;
  const float z[CPL] = {};
  for (int s = seq_of(a.cu, a.n_seqs, t0); s < a.n_seqs; ++s) {
    const int e = __ldg(a.cu + s + 1);
    if (e > t1) break;
    const int r1 = __ldg(a.out_rows + s + 1);
    for (int r = __ldg(a.out_rows + s) + e - __ldg(a.cu + s); r < r1; ++r)
      stv<CPL>(base + static_cast<size_t>(r) * HD, z);
  }
}

// fp32 conv-state column of (role, head) and row width
__device__ __forceinline__ int state_col(const ProArgs& a, int role) {
  return role == 0 ? 0 : role == 1 ? a.H * a.dk : 2 * a.H * a.dk;
}

// The input x[t] of a strip's sequence for token t (t may be negative: the
// conv state, or zero).  Rows are loaded only inside [0, T).
template <int CPL, typename Tin>
__device__ __forceinline__ void load_x(const ProArgs& a, const Tin* x, size_t row0, int HD, int ch, int b,
                                       int role, int t, float (&v)[CPL]) {
  if (t >= 0 && t < a.T) {
    ldv<CPL>(x + (row0 + t) * HD + ch, v);
  } else if (t < 0 && a.st_in && t >= -(a.K - 1)) {
    const int sw = a.H * (2 * a.dk + a.dv);
    ldv<CPL>(a.st_in + (static_cast<size_t>(b) * (a.K - 1) + t + a.K - 1) * sw + state_col(a, role) + ch, v);
  } else {
#pragma unroll
    for (int c = 0; c < CPL; ++c) v[c] = 0.f;
  }
}

// ---------------------------------------------------------------- forward ----

// Bytes of one warp's ring in the forward and backward kernels.
template <int CPL, typename Tin>
__host__ __device__ constexpr int fwd_ring_bytes() { return kStages * kPre * CPL * 32 * static_cast<int>(sizeof(Tin)); }
template <int CPL, typename Tin, typename Tout>
__host__ __device__ constexpr int bwd_ring_bytes() {
  return kBwStages * kBw * CPL * 32 * static_cast<int>(sizeof(Tin) + sizeof(Tout));
}

// q, k, v of one strip.  Batches of kPre tokens stream through the warp's
// ring (kStages - 1 batches in flight); a batch's L2 norms are one column-sum
// reduction (warp_colsum) instead of kPre serial ones.  A batch whose rows are
// all in the strip and in one packed sequence takes the plain path: rows
// copied by running offsets, outputs stored through a running pointer, no
// per-token test; the others (a strip's ragged end, a sequence start inside
// the batch) test every token.
template <int CPL, bool VARLEN, bool NORM, typename Tin, typename Tout>
__device__ void pro_fwd_conv(const ProArgs& a, int role, int b, int t0, int t1, int h, int lane,
                             unsigned char* ring) {
  constexpr bool FAST = std::is_same<Tout, bf16>::value;
  constexpr int D = CPL * 32, RB = D * static_cast<int>(sizeof(Tin)), STG = kPre * RB;
  const int HD = a.H * D;
  const int ch = h * D + lane * CPL;
  const size_t row0 = static_cast<size_t>(b) * a.T;
  const Tin* xb = static_cast<const Tin*>(pick(a.x, role));
  const Tin* xh = xb + row0 * HD + h * D;  // token t of this head at xh + t * HD
  Tout* const y = static_cast<Tout*>(pick(a.y, role)) + row0 * HD + ch;
  float wt[4][CPL];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < CPL; ++c) wt[i][c] = i < a.K ? pick(a.w, role)[i * HD + ch + c] : 0.f;
  int si = 0, lb = 0, nb = INT_MAX, shift = 0;  // shift: output row - token of this sequence
  if constexpr (VARLEN) {
    si = seq_of(a.cu, a.n_seqs, t0);
    lb = __ldg(a.cu + si);
    nb = si + 1 < a.n_seqs ? __ldg(a.cu + si + 1) : INT_MAX;
    shift = a.out_rows ? __ldg(a.out_rows + si) - lb : 0;
  }
  const int nbat = (t1 - t0 + kPre - 1) / kPre;
  const long long stride = static_cast<long long>(HD) * sizeof(Tin);
  const unsigned char* src = reinterpret_cast<const unsigned char*>(xh + static_cast<size_t>(t0) * HD) +
                             lane_src_off<RB>(lane, stride);  // this lane's chunk of the strip's first row
  const uint32_t dst = tc::smem_u32(ring) + lane_dst_off<RB>(lane);
  auto fill = [&](int bi) {
    const int tb = t0 + bi * kPre;
    if (tb + kPre <= t1) {
      ring_fill_rows<RB, kPre>(dst + (bi % kStages) * STG, src + static_cast<long long>(bi) * kPre * stride, stride);
    } else {
      ring_fill<RB, kPre>(ring + (bi % kStages) * STG, lane, xh, [&](int r) -> const void* {
        return tb + r < t1 ? xh + static_cast<size_t>(tb + r) * HD : nullptr;
      });
    }
  };
#pragma unroll
  for (int bi = 0; bi < kStages - 1; ++bi) {
    if (bi < nbat) fill(bi);
    tc::cp_async_commit();
  }
  float hw[3][CPL];  // x[t-1], x[t-2], x[t-3]
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = t0 - 1 - j;
    if (VARLEN && t < lb) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) hw[j][c] = 0.f;
    } else {
      load_x<CPL>(a, xb, row0, HD, ch, b, role, t, hw[j]);
    }
  }
  Tout* yp = y + static_cast<size_t>(t0 + shift) * HD;  // output row of the batch's first token
  // One batch; CHECK: tokens past t1 are skipped and a sequence may start inside.
  auto batch = [&](const unsigned char* st, int tb, auto check) {
    constexpr bool CHECK = decltype(check)::value;
    float s[kPre][CPL], ss[kPre];
    int sh[CHECK ? kPre : 1];
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      float xv[CPL];
      ld_row<CPL, Tin>(st + u * RB, lane, xv);
      if constexpr (CHECK && VARLEN) {
        if (tb + u == nb) {  // a packed sequence starts: the window restarts from zeros
#pragma unroll
          for (int j = 0; j < 3; ++j)
#pragma unroll
            for (int c = 0; c < CPL; ++c) hw[j][c] = 0.f;
          do {  // past the empty sequences that start at the same token
            ++si;
            nb = si + 1 < a.n_seqs ? __ldg(a.cu + si + 1) : INT_MAX;
          } while (tb + u == nb);
          shift = a.out_rows ? __ldg(a.out_rows + si) - __ldg(a.cu + si) : 0;
        }
      }
      if constexpr (CHECK) sh[u] = shift;
      float2 ss2 = f2(0.f);
#pragma unroll
      for (int c = 0; c < CPL; c += 2) {
        float2 cv = fmul2(make_float2(wt[0][c], wt[0][c + 1]), make_float2(xv[c], xv[c + 1]));
#pragma unroll
        for (int j = 0; j < 3; ++j)
          cv = ffma2(make_float2(wt[j + 1][c], wt[j + 1][c + 1]), make_float2(hw[j][c], hw[j][c + 1]), cv);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          hw[2][c + e] = hw[1][c + e];
          hw[1][c + e] = hw[0][c + e];
          hw[0][c + e] = xv[c + e];
        }
        const float2 s2 = swish2<FAST>(cv);
        s[u][c] = s2.x;
        s[u][c + 1] = s2.y;
        if constexpr (NORM) ss2 = ffma2(s2, s2, ss2);
      }
      ss[u] = ss2.x + ss2.y;
    }
    if constexpr (NORM) {  // q, k: x / (|x| + eps), the batch's norms in one reduction
      const float tot = warp_colsum<kPre>(ss, lane);  // lane l: token l % kPre
      const float inv_l = 1.f / (sqrtf(tot) + kL2Eps);  // each lane's token, once
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const float2 inv = f2(__shfl_sync(0xffffffffu, inv_l, u));
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          const float2 r = fmul2(make_float2(s[u][c], s[u][c + 1]), inv);
          s[u][c] = r.x;
          s[u][c + 1] = r.y;
        }
      }
    }
    if constexpr (CHECK) {
#pragma unroll
      for (int u = 0; u < kPre; ++u)
        if (tb + u < t1) stv<CPL>(y + static_cast<size_t>(tb + u + sh[u]) * HD, s[u]);
      yp = y + static_cast<size_t>(tb + kPre + shift) * HD;
    } else {
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        stv<CPL>(yp, s[u]);
        yp += HD;
      }
    }
  };
  for (int bi = 0; bi < nbat; ++bi) {
    tc::cp_async_wait<kStages - 2>();
    __syncwarp();
    if (bi + kStages - 1 < nbat) fill(bi + kStages - 1);
    tc::cp_async_commit();
    const unsigned char* st = ring + (bi % kStages) * STG;
    const int tb = t0 + bi * kPre;
    if (tb + kPre <= t1 && (!VARLEN || tb + kPre <= nb)) batch(st, tb, std::false_type{});
    else batch(st, tb, std::true_type{});
  }
  tc::cp_async_wait<0>();
  __syncwarp();
  if constexpr (VARLEN) zero_pads<CPL>(a, y, HD, t0, t1);
  if (a.st_out && t1 == a.T) {  // this strip ends the sequence: its last K-1 inputs
    const int sw = a.H * (2 * a.dk + a.dv);
    for (int j = 0; j < a.K - 1; ++j) {
      float v[CPL];
      load_x<CPL>(a, xb, row0, HD, ch, b, role, a.T - (a.K - 1) + j, v);
      stv<CPL>(a.st_out + (static_cast<size_t>(b) * (a.K - 1) + j) * sw + state_col(a, role) + ch, v);
    }
  }
}

// The decay gate of two channels, u = z + b: g_min sigmoid(e^A u)
// (KDA_GATE_SIGMOID_MIN) or -e^A softplus(u) (KDA_GATE_SOFTPLUS).  FAST (bf16
// results): sigmoid through one tanh.approx and softplus(u) = max(u, 0) +
// log(1 + e^-|u|) through ex2 / lg2, errors below bf16's resolution.
// c0, c1: (e^A / 2, g_min / 2) or (-e^A, -e^A ln 2) for FAST; (e^A, g_min) or (-e^A, -) else.
template <bool FAST, int KIND>
__device__ __forceinline__ float2 gate2(float2 u, float2 c0, float2 c1) {
  if constexpr (KIND == KDA_GATE_SIGMOID_MIN) {
    if constexpr (FAST) {
      const float2 h = fmul2(u, c0);
      return ffma2(make_float2(tanh_approx(h.x), tanh_approx(h.y)), c1, c1);
    } else {
      return make_float2(c1.x * sigmoidf_(c0.x * u.x), c1.x * sigmoidf_(c0.x * u.y));
    }
  } else {
    if constexpr (FAST) {
      constexpr float kLog2e = 1.4426950408889634f;
      const float2 l = make_float2(log2f(1.f + exp2f(-fabsf(u.x) * kLog2e)), log2f(1.f + exp2f(-fabsf(u.y) * kLog2e)));
      return ffma2(l, c1, fmul2(make_float2(fmaxf(u.x, 0.f), fmaxf(u.y, 0.f)), c0));
    } else {
      return make_float2(c0.x * softplusf_(u.x), c0.x * softplusf_(u.y));
    }
  }
}

template <bool FAST, int KIND>
__device__ __forceinline__ void gate_consts(float ea, float g_min, float2& c0, float2& c1) {
  constexpr float kLn2 = 0.6931471805599453f;
  if constexpr (KIND == KDA_GATE_SIGMOID_MIN) {
    c0 = f2(FAST ? 0.5f * ea : ea);
    c1 = f2(FAST ? 0.5f * g_min : g_min);
  } else {
    c0 = f2(-ea);
    c1 = f2(-ea * kLn2);
  }
}

template <int CPL, bool VARLEN, int KIND, typename Tin, typename Tout>
__device__ void pro_fwd_gate(const ProArgs& a, int b, int t0, int t1, int h, int lane, unsigned char* ring) {
  constexpr bool FAST = std::is_same<Tout, bf16>::value;
  constexpr int D = CPL * 32, RB = D * static_cast<int>(sizeof(Tin)), STG = kPre * RB;
  const int HD = a.H * D;
  const int ch = h * D + lane * CPL;
  const size_t row0 = static_cast<size_t>(b) * a.T;
  const Tin* zh = static_cast<const Tin*>(a.x[3]) + row0 * HD + h * D;
  Tout* const g = static_cast<Tout*>(a.y[3]) + row0 * HD + ch;
  float bias[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) bias[c] = a.b_gate ? a.b_gate[ch + c] : 0.f;
  float2 c0, c1;
  gate_consts<FAST, KIND>(__expf(a.A[h]), a.g_min, c0, c1);
  const int nbat = (t1 - t0 + kPre - 1) / kPre;
  const long long stride = static_cast<long long>(HD) * sizeof(Tin);
  const unsigned char* src = reinterpret_cast<const unsigned char*>(zh + static_cast<size_t>(t0) * HD) +
                             lane_src_off<RB>(lane, stride);
  const uint32_t dst = tc::smem_u32(ring) + lane_dst_off<RB>(lane);
  auto fill = [&](int bi) {
    const int tb = t0 + bi * kPre;
    if (tb + kPre <= t1) {
      ring_fill_rows<RB, kPre>(dst + (bi % kStages) * STG, src + static_cast<long long>(bi) * kPre * stride, stride);
    } else {
      ring_fill<RB, kPre>(ring + (bi % kStages) * STG, lane, zh, [&](int r) -> const void* {
        return tb + r < t1 ? zh + static_cast<size_t>(tb + r) * HD : nullptr;
      });
    }
  };
#pragma unroll
  for (int bi = 0; bi < kStages - 1; ++bi) {
    if (bi < nbat) fill(bi);
    tc::cp_async_commit();
  }
  const Tin* bl = static_cast<const Tin*>(a.beta_logit);
  Tout* beta = static_cast<Tout*>(a.beta);
  RowWalk<true> rwb, rwm;  // rows of this lane's beta tokens, of the gate rows
  if (VARLEN) {
    rwb.init(a, min(t0 + lane, a.T - 1));
    rwm.init(a, t0);
  }
  for (int t = t0 + lane; t < t1; t += 32) {  // beta while the first batches land
    const size_t i = (row0 + t) * a.H + h;
    const int r = VARLEN ? rwb(t) : t;
    stf(beta + (row0 + r) * a.H + h, sigmoidf_(ldf(bl + i)));
  }
  if (VARLEN && a.out_rows && lane == 0) {  // beta of the pad rows
    for (int s = seq_of(a.cu, a.n_seqs, t0); s < a.n_seqs; ++s) {
      const int e = __ldg(a.cu + s + 1);
      if (e > t1) break;
      const int r1 = __ldg(a.out_rows + s + 1);
      for (int r = __ldg(a.out_rows + s) + e - __ldg(a.cu + s); r < r1; ++r)
        stf(beta + static_cast<size_t>(r) * a.H + h, 0.f);
    }
  }
  for (int bi = 0; bi < nbat; ++bi) {
    tc::cp_async_wait<kStages - 2>();
    __syncwarp();
    if (bi + kStages - 1 < nbat) fill(bi + kStages - 1);
    tc::cp_async_commit();
    const unsigned char* st = ring + (bi % kStages) * STG;
    const int tb = t0 + bi * kPre;
    const int rb = VARLEN ? rwm(tb) : tb;  // output row of the batch's first token
    const bool plain = tb + kPre <= t1 && (!VARLEN || tb + kPre <= rwm.edge || rwm.s == a.n_seqs - 1);
    float o[kPre][CPL];
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      float zv[CPL];
      ld_row<CPL, Tin>(st + u * RB, lane, zv);
#pragma unroll
      for (int c = 0; c < CPL; c += 2) {
        const float2 r = gate2<FAST, KIND>(fadd2(make_float2(zv[c], zv[c + 1]), make_float2(bias[c], bias[c + 1])),
                                           c0, c1);
        o[u][c] = r.x;
        o[u][c + 1] = r.y;
      }
    }
    if (plain) {
      Tout* p = g + static_cast<size_t>(rb) * HD;
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        stv<CPL>(p, o[u]);
        p += HD;
      }
    } else {
#pragma unroll
      for (int u = 0; u < kPre; ++u)
        if (tb + u < t1) stv<CPL>(g + static_cast<size_t>(VARLEN ? rwm(tb + u) : tb + u) * HD, o[u]);
    }
  }
  tc::cp_async_wait<0>();
  __syncwarp();
  if constexpr (VARLEN) zero_pads<CPL>(a, g, HD, t0, t1);
}

// blockIdx.z selects the tensor: role = 4-bit field z of a.roles (0 q, 1 k,
// 2 v, 3 gates), so one launch covers the tensors of one width D = 32 CPL.
template <int CPL, bool VARLEN, typename Tin, typename Tout>
__global__ void __launch_bounds__(kWarps * 32) prologue_fwd_kernel(const ProArgs a) {
  extern __shared__ __align__(16) unsigned char pro_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = (a.head_x ? blockIdx.y : blockIdx.x) * kWarps + warp;
  if (s >= a.n_strips) return;
  unsigned char* ring = pro_smem + warp * fwd_ring_bytes<CPL, Tin>();
  const int h = a.head_x ? blockIdx.x : blockIdx.y, role = (a.roles >> (4 * blockIdx.z)) & 15;
  const int b = s / a.spb;
  const int t0 = (s % a.spb) * kStrip, t1 = min(t0 + kStrip, a.T);
  if (role < 2) pro_fwd_conv<CPL, VARLEN, true, Tin, Tout>(a, role, b, t0, t1, h, lane, ring);
  else if (role == 2) pro_fwd_conv<CPL, VARLEN, false, Tin, Tout>(a, role, b, t0, t1, h, lane, ring);
  else if (a.gate_kind == KDA_GATE_SIGMOID_MIN)
    pro_fwd_gate<CPL, VARLEN, KDA_GATE_SIGMOID_MIN, Tin, Tout>(a, b, t0, t1, h, lane, ring);
  else pro_fwd_gate<CPL, VARLEN, KDA_GATE_SOFTPLUS, Tin, Tout>(a, b, t0, t1, h, lane, ring);
}

// --------------------------------------------------------------- backward ----

// q, k, v of one strip, swept from its end (hi: the last token whose conv
// cotangent the strip's inputs need) down to its start, kBw tokens a batch:
// the window x[base - j], j < kBw + 3 (every tap of every token of the batch),
// and the conv cotangents of the three tokens above the batch live in
// registers.  A batch's cotangent rows and the input rows the window moves
// onto stream through the warp's shared-memory ring.  The L2-norm cotangent needs two sums per token; a batch's
// 2 kBw sums are one column-sum reduction.  Batches inside the strip and
// inside one packed sequence, taps included, take the plain path (no
// per-token tests); the strip's ends and sequence edges test every token.
template <int CPL, bool VARLEN, bool NORM, typename Tin, typename Tout>
__device__ void pro_bwd_conv(const ProArgs& a, int role, int b, int t0, int t1, int h, int lane,
                             float (&dw)[4][4], unsigned char* ring) {
  constexpr bool FAST = std::is_same<Tin, bf16>::value;  // the cotangents leave as Tin
  constexpr int D = CPL * 32, NX = kBw + 3;
  constexpr int RBX = D * static_cast<int>(sizeof(Tin)), RBY = D * static_cast<int>(sizeof(Tout));
  constexpr int STG = kBw * (RBX + RBY);
  const int HD = a.H * D;
  const int ch = h * D + lane * CPL;
  const size_t row0 = static_cast<size_t>(b) * a.T;
  const Tin* xb = static_cast<const Tin*>(pick(a.x, role));
  const Tin* xh = xb + row0 * HD + h * D;
  const Tout* dyh = static_cast<const Tout*>(pick(a.dy, role)) + row0 * HD + h * D;
  Tin* dx = static_cast<Tin*>(pick(a.dx, role)) + row0 * HD + ch;
  const int K = a.K;
  float wt[4][CPL];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < CPL; ++c) wt[i][c] = i < K ? pick(a.w, role)[i * HD + ch + c] : 0.f;
  const int hi = min(t1 + K - 1, a.T) - 1;
  const int lo = (t0 == 0 && a.dst && !a.cu) ? -(K - 1) : t0;
  const int nbat = (hi - lo) / kBw + 1;
  // stage bi: the input rows base - NX - u (the window's next rows), then the
  // cotangent rows base - u, u < kBw, base = hi - bi kBw
  const long long sx = static_cast<long long>(HD) * sizeof(Tin), sy = static_cast<long long>(HD) * sizeof(Tout);
  const unsigned char* xsrc = reinterpret_cast<const unsigned char*>(xh) + lane_src_off<RBX>(lane, -sx);
  const unsigned char* ysrc = reinterpret_cast<const unsigned char*>(dyh) + lane_src_off<RBY>(lane, -sy);
  const uint32_t dstx = tc::smem_u32(ring) + lane_dst_off<RBX>(lane);
  const uint32_t dsty = tc::smem_u32(ring) + kBw * RBX + lane_dst_off<RBY>(lane);
  const int ylo = max(lo, 0);
  RowWalk<false> rwf;  // rows of the cotangent tokens the fills walk down
  if (VARLEN) rwf.init(a, max(hi, 0));
  auto fill = [&](int bi) {
    const int base = hi - bi * kBw;
    const uint32_t so = (bi % kBwStages) * STG;
    unsigned char* st = ring + so;
    if (base - NX - kBw + 1 >= 0) {
      ring_fill_rows<RBX, kBw>(dstx + so, xsrc + (base - NX) * sx, -sx);
    } else {
      ring_fill<RBX, kBw>(st, lane, xh, [&](int r) -> const void* {
        const int t = base - NX - r;
        return t >= 0 ? xh + static_cast<size_t>(t) * HD : nullptr;
      });
    }
    int ry = base;  // cotangent row of token base
    bool yplain = base - kBw + 1 >= ylo;
    if (VARLEN && base >= 0) {
      ry = rwf(base);
      yplain = yplain && base - kBw + 1 >= rwf.edge;
    }
    if (yplain) {
      ring_fill_rows<RBY, kBw>(dsty + so, ysrc + ry * sy, -sy);
    } else {
      int rw[kBw];  // cotangent row of token base - u
#pragma unroll
      for (int u = 0; u < kBw; ++u) rw[u] = VARLEN && base - u >= 0 ? rwf(base - u) : base - u;
      ring_fill<RBY, kBw>(st + kBw * RBX, lane, dyh, [&](int r) -> const void* {
        const int t = base - r;
        const int row = r == 0 ? rw[0] : r == 1 ? rw[1] : r == 2 ? rw[2] : rw[3];
        return t >= 0 && t >= lo ? dyh + static_cast<size_t>(row) * HD : nullptr;
      });
    }
  };
#pragma unroll
  for (int bi = 0; bi < kBwStages - 1; ++bi) {
    if (bi < nbat) fill(bi);
    tc::cp_async_commit();
  }
  int si = 0, lb = INT_MIN, ub = INT_MAX;  // the packed sequence [lb, ub) of the current token
  if constexpr (VARLEN) {
    si = seq_of(a.cu, a.n_seqs, hi);
    lb = __ldg(a.cu + si);
    ub = si + 1 < a.n_seqs ? __ldg(a.cu + si + 1) : INT_MAX;
  }
  // The input rows in a ring of 8: a batch of phase P (its index's parity)
  // sees x[base - j] in R[(4 P + j) % 8], j < NX, and loads the rows the next
  // batch adds into the slots its own first kBw rows leave (and the spare), so
  // the window moves by renaming instead of copies.  Likewise the two batches'
  // conv cotangents alternate between DA and DB, each batch reading the other's
  // as the cotangents of the three tokens above it.
  constexpr bool RING = true;
  static_assert(NX + 1 == 8 && kBw == 4, "an 8-row ring, 4 rows a batch");
  float R[8][CPL], DA[kBw][CPL], DB[kBw][CPL];
#pragma unroll
  for (int j = 0; j < NX; ++j) load_x<CPL>(a, xb, row0, HD, ch, b, role, hi - j, R[j]);
#pragma unroll
  for (int c = 0; c < CPL; ++c) R[NX][c] = 0.f;
#pragma unroll
  for (int j = 0; j < kBw; ++j)
#pragma unroll
    for (int c = 0; c < CPL; ++c) DA[j][c] = DB[j][c] = 0.f;
  const int sw = a.H * (2 * a.dk + a.dv);
  // One batch; CHECK: tokens may lie outside [t0, t1) or below 0, and taps may
  // cross a packed sequence's edge: bit 4 u + i of cm (dm) says whether token u's
  // tap i below (above) it lies in its sequence.
  auto batch = [&](const unsigned char* st, int base, unsigned cm, unsigned dm, auto check,
                   auto phase, float (&dc)[kBw][CPL], const float (&dcp)[kBw][CPL]) {
    constexpr bool CHECK = decltype(check)::value;
    constexpr bool MASK = CHECK && VARLEN;
    constexpr int P4 = 4 * decltype(phase)::value;
#define X(j) R[(P4 + (j)) & 7]
    // dc[u] = swish'(c) dv and, for the norm, bq[u] = swish'(c) s: the conv
    // cotangent of token u is then dc c1 + bq c2 with two scalars per token.
    float sums[2 * kBw];
    [[maybe_unused]] float bq[NORM ? kBw : 1][CPL];
#pragma unroll
    for (int u = 0; u < kBw; ++u) {
      float dvr[CPL];
      ld_row<CPL, Tout>(st + kBw * RBX + u * RBY, lane, dvr);
      float2 ss2 = f2(0.f), sd2 = f2(0.f);
#pragma unroll
      for (int c = 0; c < CPL; c += 2) {
        float2 cv2;
        if constexpr (MASK) {
          cv2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if ((cm >> (4 * u + i)) & 1u)
              cv2 = ffma2(make_float2(wt[i][c], wt[i][c + 1]), make_float2(X(u + i)[c], X(u + i)[c + 1]), cv2);
        } else {
          cv2 = fmul2(make_float2(wt[0][c], wt[0][c + 1]), make_float2(X(u)[c], X(u)[c + 1]));
#pragma unroll
          for (int i = 1; i < 4; ++i)
            cv2 = ffma2(make_float2(wt[i][c], wt[i][c + 1]), make_float2(X(u + i)[c], X(u + i)[c + 1]), cv2);
        }
        float2 s2, ds2;
        swish_grad2<FAST>(cv2, s2, ds2);
        const float2 d2 = make_float2(dvr[c], dvr[c + 1]);
        const float2 a2 = fmul2(ds2, d2);
        dc[u][c] = a2.x;
        dc[u][c + 1] = a2.y;
        if constexpr (NORM) {
          const float2 b2 = fmul2(ds2, s2);
          bq[u][c] = b2.x;
          bq[u][c + 1] = b2.y;
          ss2 = ffma2(s2, s2, ss2);
          sd2 = ffma2(s2, d2, sd2);
        }
      }
      sums[u] = ss2.x + ss2.y;
      sums[kBw + u] = sd2.x + sd2.y;
    }
    if constexpr (NORM) {
      // cotangent of s / (n + eps), n = |s|, p = s . dv: (dv - s p / (n (n + eps))) / (n + eps),
      // zero at n = 0.  Lane u (< kBw) holds n^2 and, after one exchange, p of token u.
      const float tot = warp_colsum<2 * kBw>(sums, lane);  // lane l: sum l % (2 kBw)
      const float p = __shfl_xor_sync(0xffffffffu, tot, kBw);
      const float n = sqrtf(tot);
      const float inv = 1.f / (n + kL2Eps);
      const float c1 = n > 0.f ? inv : 0.f;
      const float c2 = n > 0.f ? -p / n * inv * inv : 0.f;
#pragma unroll
      for (int u = 0; u < kBw; ++u) {
        const float2 k1 = f2(__shfl_sync(0xffffffffu, c1, u)), k2 = f2(__shfl_sync(0xffffffffu, c2, u));
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          const float2 r = ffma2(make_float2(bq[u][c], bq[u][c + 1]), k2,
                                 fmul2(make_float2(dc[u][c], dc[u][c + 1]), k1));
          dc[u][c] = r.x;
          dc[u][c + 1] = r.y;
        }
      }
    }
    if (CHECK && base < kBw - 1) {  // the batch reaches below token 0 (the conv state's rows)
#pragma unroll
      for (int u = 0; u < kBw; ++u) {
        if (base - u < 0) {
#pragma unroll
          for (int c = 0; c < CPL; ++c) dc[u][c] = 0.f;
        }
      }
    }
    // dx[tau] = sum_i w[i] dc[tau + i] (same sequence); dw[i] += dc[tau] x[tau - i]
    Tin* dxp = CHECK ? dx : dx + static_cast<size_t>(base) * HD;  // plain: row of token base
#pragma unroll
    for (int u = 0; u < kBw; ++u) {
      const int tau = base - u;
      if (!CHECK || (tau >= lo && tau < t1)) {
        float o[CPL];
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          float2 acc = fmul2(make_float2(wt[0][c], wt[0][c + 1]), make_float2(dc[u][c], dc[u][c + 1]));
#pragma unroll
          for (int i = 1; i < 4; ++i) {
            const float2 d = i <= u ? make_float2(dc[u - i][c], dc[u - i][c + 1])
                                    : make_float2(dcp[kBw - i + u][c], dcp[kBw - i + u][c + 1]);
            if (!MASK || ((dm >> (4 * u + i)) & 1u)) acc = ffma2(make_float2(wt[i][c], wt[i][c + 1]), d, acc);
          }
          o[c] = acc.x;
          o[c + 1] = acc.y;
        }
        if (!CHECK || tau >= t0) {
          if constexpr (CHECK) {
            stv<CPL>(dx + static_cast<size_t>(tau) * HD, o);
          } else {
            stv<CPL>(dxp, o);
            dxp -= HD;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (!MASK || ((cm >> (4 * u + i)) & 1u)) {
#pragma unroll
              for (int c = 0; c < CPL; c += 2) {
                const float2 w2 = ffma2(make_float2(dc[u][c], dc[u][c + 1]), make_float2(X(u + i)[c], X(u + i)[c + 1]),
                                        make_float2(dw[i][c], dw[i][c + 1]));
                dw[i][c] = w2.x;
                dw[i][c + 1] = w2.y;
              }
            }
          }
        } else {  // tau < 0: cotangent of the conv state row
          stv<CPL>(a.dst + (static_cast<size_t>(b) * (K - 1) + tau + K - 1) * sw + state_col(a, role) + ch, o);
        }
      }
    }
    // the next batch's window: its rows NX - kBw .. NX - 1 come in over this
    // batch's first kBw (ring), or after the rows that stay move down (copies)
    if constexpr (!RING) {
#pragma unroll
      for (int j = 0; j < NX - kBw; ++j)
#pragma unroll
        for (int c = 0; c < CPL; ++c) R[j][c] = R[j + kBw][c];
    }
#pragma unroll
    for (int u = 0; u < kBw; ++u) {
      const int t = base - NX - u;
      float (&row)[CPL] = RING ? X(NX + u) : R[NX - kBw + u];
      if (!CHECK || t >= 0) ld_row<CPL, Tin>(st + u * RBX, lane, row);
      else load_x<CPL>(a, xb, row0, HD, ch, b, role, t, row);
    }
#undef X
  };
  for (int bi = 0; bi < nbat; ++bi) {
    tc::cp_async_wait<kBwStages - 2>();
    __syncwarp();
    if (bi + kBwStages - 1 < nbat) fill(bi + kBwStages - 1);
    tc::cp_async_commit();
    const unsigned char* st = ring + (bi % kBwStages) * STG;
    const int base = hi - bi * kBw;
    // plain: every token in [t0, t1), the window's next rows at or above 0, and
    // (packed) every tap of the batch inside the sequence [lb, ub) the walk is
    // in (that of the token above the batch), so the walk stays where it is
    const bool plain = base < t1 && base - kBw + 1 >= t0 && base - NX - kBw + 1 >= 0 &&
                       (!VARLEN || (base + 3 < ub && base - kBw + 1 - 3 >= lb));
    unsigned cm = 0u, dm = 0u;
    if (VARLEN && !plain) {  // walk down to each token's sequence; its taps inside it
#pragma unroll
      for (int u = 0; u < kBw; ++u) {
        const int tau = base - u;
        while (tau < lb && si > 0) {  // below lb lies the previous sequence
          ub = lb;
          --si;
          lb = __ldg(a.cu + si);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          cm |= static_cast<unsigned>(tau - i >= lb) << (4 * u + i);
          dm |= static_cast<unsigned>(tau + i < ub) << (4 * u + i);
        }
      }
    }
    using P0 = std::integral_constant<int, 0>;
    using P1 = std::integral_constant<int, 1>;
    if (RING && (bi & 1)) {
      if (plain) batch(st, base, cm, dm, std::false_type{}, P1{}, DB, DA);
      else batch(st, base, cm, dm, std::true_type{}, P1{}, DB, DA);
    } else {
      if (plain) batch(st, base, cm, dm, std::false_type{}, P0{}, DA, DB);
      else batch(st, base, cm, dm, std::true_type{}, P0{}, DA, DB);
      if constexpr (!RING) {
#pragma unroll
        for (int j = 0; j < kBw; ++j)
#pragma unroll
          for (int c = 0; c < CPL; ++c) DB[j][c] = DA[j][c];
      }
    }
  }
  tc::cp_async_wait<0>();
  __syncwarp();
}

// Cotangents of gate2 for two channels: dz (written) and the terms of dA
// (accumulated in dA2), dg the gate's cotangent.  SIGMOID_MIN: dz = dg g_min
// sig (1 - sig) e^A, dA += dz u; SOFTPLUS: dz = -dg e^A sigmoid(u), dA -= dg e^A softplus(u).
template <bool FAST, int KIND>
__device__ __forceinline__ float2 gate_grad2(float2 u, float2 dg, float ea, float g_min, float2& dA2) {
  if constexpr (KIND == KDA_GATE_SIGMOID_MIN) {
    float2 sg;
    if constexpr (FAST) {
      const float2 h = fmul2(u, f2(0.5f * ea));
      sg = ffma2(make_float2(tanh_approx(h.x), tanh_approx(h.y)), f2(0.5f), f2(0.5f));
    } else {
      sg = make_float2(sigmoidf_(ea * u.x), sigmoidf_(ea * u.y));
    }
    // dg g_min e^A sg (1 - sg)
    const float2 t = fmul2(fmul2(dg, f2(g_min * ea)), fmul2(sg, ffma2(sg, f2(-1.f), f2(1.f))));
    dA2 = ffma2(t, u, dA2);
    return t;
  } else {
    const float2 gn = fmul2(dg, f2(-ea));
    float2 sg, sp;
    if constexpr (FAST) {
      constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
      const float2 h = fmul2(u, f2(0.5f));
      sg = ffma2(make_float2(tanh_approx(h.x), tanh_approx(h.y)), f2(0.5f), f2(0.5f));
      const float2 l = make_float2(log2f(1.f + exp2f(-fabsf(u.x) * kLog2e)), log2f(1.f + exp2f(-fabsf(u.y) * kLog2e)));
      sp = ffma2(l, f2(kLn2), make_float2(fmaxf(u.x, 0.f), fmaxf(u.y, 0.f)));
    } else {
      sg = make_float2(sigmoidf_(u.x), sigmoidf_(u.y));
      sp = make_float2(softplusf_(u.x), softplusf_(u.y));
    }
    dA2 = ffma2(gn, sp, dA2);
    return fmul2(gn, sg);
  }
}

template <int CPL, bool VARLEN, int KIND, typename Tin, typename Tout>
__device__ void pro_bwd_gate(const ProArgs& a, int b, int t0, int t1, int h, int lane, float (&db)[4],
                             float& dA, unsigned char* ring) {
  constexpr bool FAST = std::is_same<Tin, bf16>::value;
  constexpr int D = CPL * 32;
  constexpr int RBX = D * static_cast<int>(sizeof(Tin)), RBY = D * static_cast<int>(sizeof(Tout));
  constexpr int STG = kBw * (RBX + RBY);
  const int HD = a.H * D;
  const int ch = h * D + lane * CPL;
  const size_t row0 = static_cast<size_t>(b) * a.T;
  const Tin* zh = static_cast<const Tin*>(a.x[3]) + row0 * HD + h * D;
  const Tout* dgh = static_cast<const Tout*>(a.dy[3]) + row0 * HD + h * D;
  Tin* dz = static_cast<Tin*>(a.dx[3]) + row0 * HD + ch;
  float bias[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) bias[c] = a.b_gate ? a.b_gate[ch + c] : 0.f;
  const float ea = __expf(a.A[h]);
  const int nbat = (t1 - t0 + kBw - 1) / kBw;
  const long long sx = static_cast<long long>(HD) * sizeof(Tin), sy = static_cast<long long>(HD) * sizeof(Tout);
  const unsigned char* xsrc = reinterpret_cast<const unsigned char*>(zh) + lane_src_off<RBX>(lane, sx);
  const unsigned char* ysrc = reinterpret_cast<const unsigned char*>(dgh) + lane_src_off<RBY>(lane, sy);
  const uint32_t dstx = tc::smem_u32(ring) + lane_dst_off<RBX>(lane);
  const uint32_t dsty = tc::smem_u32(ring) + kBw * RBX + lane_dst_off<RBY>(lane);
  RowWalk<true> rwf, rwb;  // rows of the cotangent tokens the fills walk up, of this lane's beta tokens
  if (VARLEN) {
    rwf.init(a, t0);
    rwb.init(a, min(t0 + lane, a.T - 1));
  }
  auto fill = [&](int bi) {
    const int tb = t0 + bi * kBw;
    const uint32_t so = (bi % kBwStages) * STG;
    unsigned char* st = ring + so;
    const bool full = tb + kBw <= t1;
    if (full) {
      ring_fill_rows<RBX, kBw>(dstx + so, xsrc + tb * sx, sx);
    } else {
      ring_fill<RBX, kBw>(st, lane, zh, [&](int r) -> const void* {
        return tb + r < t1 ? zh + static_cast<size_t>(tb + r) * HD : nullptr;
      });
    }
    const int ry = VARLEN ? rwf(tb) : tb;  // cotangent row of token tb
    if (full && (!VARLEN || tb + kBw <= rwf.edge || rwf.s == a.n_seqs - 1)) {
      ring_fill_rows<RBY, kBw>(dsty + so, ysrc + ry * sy, sy);
    } else {
      int rw[kBw];  // cotangent row of token tb + u
#pragma unroll
      for (int u = 0; u < kBw; ++u) rw[u] = VARLEN && tb + u < t1 ? rwf(tb + u) : tb + u;
      ring_fill<RBY, kBw>(st + kBw * RBX, lane, dgh, [&](int r) -> const void* {
        const int row = r == 0 ? rw[0] : r == 1 ? rw[1] : r == 2 ? rw[2] : rw[3];
        return tb + r < t1 ? dgh + static_cast<size_t>(row) * HD : nullptr;
      });
    }
  };
#pragma unroll
  for (int bi = 0; bi < kBwStages - 1; ++bi) {
    if (bi < nbat) fill(bi);
    tc::cp_async_commit();
  }
  const Tin* bl = static_cast<const Tin*>(a.beta_logit);
  const Tout* dbt = static_cast<const Tout*>(a.dbeta);
  Tin* dbl = static_cast<Tin*>(a.dbeta_logit);
  for (int t = t0 + lane; t < t1; t += 32) {  // beta while the first batches land
    const size_t i = (row0 + t) * a.H + h;
    const float s = sigmoidf_(ldf(bl + i));
    const int r = VARLEN ? rwb(t) : t;
    stf(dbl + i, ldf(dbt + (row0 + r) * a.H + h) * s * (1.f - s));
  }
  float2 dA2 = f2(0.f);
  for (int bi = 0; bi < nbat; ++bi) {
    tc::cp_async_wait<kBwStages - 2>();
    __syncwarp();
    if (bi + kBwStages - 1 < nbat) fill(bi + kBwStages - 1);
    tc::cp_async_commit();
    const unsigned char* st = ring + (bi % kBwStages) * STG;
    const int tb = t0 + bi * kBw;
    const bool full = tb + kBw <= t1;
    Tin* p = dz + static_cast<size_t>(tb) * HD;
#pragma unroll
    for (int u = 0; u < kBw; ++u) {
      if (full || tb + u < t1) {
        float o[CPL], zv[CPL], gv[CPL];
        ld_row<CPL, Tin>(st + u * RBX, lane, zv);
        ld_row<CPL, Tout>(st + kBw * RBX + u * RBY, lane, gv);
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          const float2 uu = fadd2(make_float2(zv[c], zv[c + 1]), make_float2(bias[c], bias[c + 1]));
          const float2 r = gate_grad2<FAST, KIND>(uu, make_float2(gv[c], gv[c + 1]), ea, a.g_min, dA2);
          o[c] = r.x;
          o[c + 1] = r.y;
          const float2 d2 = fadd2(make_float2(db[c], db[c + 1]), r);
          db[c] = d2.x;
          db[c + 1] = d2.y;
        }
        stv<CPL>(p, o);
      }
      p += HD;
    }
  }
  dA += dA2.x + dA2.y;
  tc::cp_async_wait<0>();
  __syncwarp();
}

// Partial-sum slab of one block group: [q taps K x H*dk | k taps | v taps K x H*dv | db H*dk | dA H]
__host__ __device__ inline int slab_off(int role, int H, int dk, int K) {
  return role == 0 ? 0 : role == 1 ? K * H * dk : role == 2 ? 2 * K * H * dk : -1;
}

template <int CPL, bool VARLEN, typename Tin, typename Tout>
__global__ void __launch_bounds__(kBwdWarps * 32) prologue_bwd_kernel(const ProArgs a) {
  __shared__ float red[kBwdWarps][4][128];
  extern __shared__ __align__(16) unsigned char pro_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* ring = pro_smem + warp * bwd_ring_bytes<CPL, Tin, Tout>();
  const int s = blockIdx.x * kBwdWarps + warp;
  const int h = blockIdx.y, role = (a.roles >> (4 * blockIdx.z)) & 15;
  constexpr int D = CPL * 32;
  float acc[4][4] = {};
  float dA = 0.f;
  if (s < a.n_strips) {
    const int b = s / a.spb;
    const int t0 = (s % a.spb) * kStrip, t1 = min(t0 + kStrip, a.T);
    if (role < 2) pro_bwd_conv<CPL, VARLEN, true, Tin, Tout>(a, role, b, t0, t1, h, lane, acc, ring);
    else if (role == 2) pro_bwd_conv<CPL, VARLEN, false, Tin, Tout>(a, role, b, t0, t1, h, lane, acc, ring);
    else if (a.gate_kind == KDA_GATE_SIGMOID_MIN)
      pro_bwd_gate<CPL, VARLEN, KDA_GATE_SIGMOID_MIN, Tin, Tout>(a, b, t0, t1, h, lane, acc[0], dA, ring);
    else pro_bwd_gate<CPL, VARLEN, KDA_GATE_SOFTPLUS, Tin, Tout>(a, b, t0, t1, h, lane, acc[0], dA, ring);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (c < CPL) red[warp][i][lane * CPL + c] = acc[i][c];
  dA = warp_sum(dA);
  if (role == 3 && lane == 0) red[warp][1][0] = dA;
  __syncthreads();
  float* slab = a.ws + static_cast<size_t>(blockIdx.x) * a.ws_stride;
  if (role < 3) {
    const int HD = a.H * D;
    for (int e = threadIdx.x; e < a.K * D; e += blockDim.x) {
      const int i = e / D, c = e % D;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kBwdWarps; ++w) sum += red[w][i][c];
      slab[slab_off(role, a.H, a.dk, a.K) + i * HD + h * D + c] = sum;
    }
  } else {
    const int db_off = 2 * a.K * a.H * a.dk + a.K * a.H * a.dv;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kBwdWarps; ++w) sum += red[w][0][c];
      slab[db_off + h * D + c] = sum;
    }
    if (threadIdx.x == 0) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kBwdWarps; ++w) sum += red[w][1][0];
      slab[db_off + a.H * a.dk + h] = sum;
    }
  }
}

// Sum the per-group slabs (fixed order) into the weight gradients.
__global__ void prologue_reduce_kernel(const float* __restrict__ ws, int groups, int stride, int H, int dk,
                                       int dv, int K, float* dwq, float* dwk, float* dwv, float* db,
                                       float* dA) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= stride) return;
  float sum = 0.f;
  for (int g = 0; g < groups; ++g) sum += ws[static_cast<size_t>(g) * stride + e];
  const int nq = K * H * dk, nv = K * H * dv;
  if (e < nq) dwq[e] = sum;
  else if (e < 2 * nq) dwk[e - nq] = sum;
  else if (e < 2 * nq + nv) dwv[e - 2 * nq] = sum;
  else if (e < 2 * nq + nv + H * dk) db[e - 2 * nq - nv] = sum;
  else dA[e - 2 * nq - nv - H * dk] = sum;
}

// ------------------------------------------------------------ output gate ----

// Rows of o (and do) for the packed rows r = t H + h of y: the same row, or with
// out_rows that of token t in the chunk-aligned layout (sequence s from row
// out_rows[s]).
struct RowMap {
  const int* cu;
  const int* out_rows;
  int n_seqs;
  int H;
};
__device__ __forceinline__ long long o_row(const RowMap& m, long long r) {
  if (!m.out_rows) return r;
  const int t = static_cast<int>(r / m.H), h = static_cast<int>(r % m.H);
  const int s = seq_of(m.cu, m.n_seqs, t);
  return static_cast<long long>(t + __ldg(m.out_rows + s) - __ldg(m.cu + s)) * m.H + h;
}

// Zeroes the pad rows of sequence blockIdx.x (row_elems elements per token row).
template <typename T>
__global__ void zero_pad_rows_kernel(T* __restrict__ x, RowMap m, int row_elems) {
  const int s = blockIdx.x;
  const long long r0 = __ldg(m.out_rows + s) + (__ldg(m.cu + s + 1) - __ldg(m.cu + s));
  const long long r1 = __ldg(m.out_rows + s + 1);
  for (long long i = r0 * row_elems + threadIdx.x; i < r1 * row_elems; i += blockDim.x) stf(x + i, 0.f);
}

template <int CPL, typename To, typename Tg, typename Ty>
__global__ void __launch_bounds__(256) gated_rms_fwd_kernel(const To* __restrict__ o, const Tg* __restrict__ gate,
                                                            Ty* __restrict__ y, long long rows, float eps,
                                                            const RowMap m) {
  constexpr int D = CPL * 32;
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
    const size_t off = static_cast<size_t>(r) * D + lane * CPL;
    float ov[CPL], gv[CPL];
    ldv<CPL>(o + static_cast<size_t>(o_row(m, r)) * D + lane * CPL, ov);
    ldv<CPL>(gate + off, gv);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) ss += ov[c] * ov[c];
    const float rr = 1.f / sqrtf(warp_sum(ss) / D + eps);
#pragma unroll
    for (int c = 0; c < CPL; ++c) ov[c] = sigmoidf_(gv[c]) * ov[c] * rr;
    stv<CPL>(y + off, ov);
  }
}

template <int CPL, typename To, typename Tg, typename Ty>
__global__ void __launch_bounds__(256) gated_rms_bwd_kernel(const To* __restrict__ o, const Tg* __restrict__ gate,
                                                            const Ty* __restrict__ dy, To* __restrict__ dout,
                                                            Tg* __restrict__ dgate, long long rows, float eps,
                                                            const RowMap m) {
  constexpr int D = CPL * 32;
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
    const size_t off = static_cast<size_t>(r) * D + lane * CPL;
    const size_t ooff = static_cast<size_t>(o_row(m, r)) * D + lane * CPL;
    float ov[CPL], gv[CPL], dv[CPL];
    ldv<CPL>(o + ooff, ov);
    ldv<CPL>(gate + off, gv);
    ldv<CPL>(dy + off, dv);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) ss += ov[c] * ov[c];
    const float rr = 1.f / sqrtf(warp_sum(ss) / D + eps);
    float dn[CPL], dg[CPL], m = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const float n = ov[c] * rr, s = sigmoidf_(gv[c]);
      dg[c] = dv[c] * n * s * (1.f - s);
      dn[c] = dv[c] * s;
      m += dn[c] * n;
    }
    m = warp_sum(m) / D;
#pragma unroll
    for (int c = 0; c < CPL; ++c) dn[c] = rr * (dn[c] - ov[c] * rr * m);
    stv<CPL>(dout + ooff, dn);
    stv<CPL>(dgate + off, dg);
  }
}

// ------------------------------------------------------------ fused decode ----

struct DecArgs {
  float* S;
  float* buf;
  const void* qp;
  const void* kp;
  const void* vp;
  const void* z;
  const void* beta_logit;
  const void* gate;
  const float* w[3];
  const float* b_gate;
  const float* A;
  float g_min;
  int gate_kind;
  float rms_eps;
  void* out;
  int* err;
  int H, K;
};

constexpr int kDecThreads = 256;

// One CTA per (sequence, head).  The state (DK x DV fp32) comes into shared
// memory with one bulk copy issued first, so it is in flight without holding
// registers (three CTAs per SM); meanwhile threads [0, DK) form q, k, g of
// channel d and threads [DK, DK + DV) v of channel d - DK from the projections
// and the conv buffer (shifted in place, each thread its own channel); then
// the delta-rule update of the decode step (r = (alpha k)^T S,
// S' = alpha S + beta k (v - r)^T, o = S'^T q) reads the rows from shared
// memory and writes S' to HBM.  The copy's wait is bounded: on a timeout the
// CTA raises `err`, waits (bounded) once more and returns.
template <int DK, int DV, typename Tin, typename To>
__global__ void __launch_bounds__(kDecThreads, 3) decode_fused_kernel(const DecArgs a) {
  static_assert(DK + DV <= kDecThreads, "one thread per q/k/g and per v channel");
  constexpr int TPR = DV / 4;
  constexpr int RPP = kDecThreads / TPR;
  constexpr int NR = DK / RPP;
  __shared__ float s_ak[DK], s_a[DK], s_bk[DK], s_q[DK], s_v[DV];
  __shared__ float s_red[RPP][DV];
  __shared__ float s_nrm[2][8];
  __shared__ float s_beta;
  __shared__ __align__(8) uint64_t s_mbar;
  extern __shared__ __align__(128) float s_state[];  // DK x DV
  const int n = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col = (tid % TPR) * 4, row0 = tid / TPR;
  float4* Sn = reinterpret_cast<float4*>(a.S + static_cast<size_t>(blockIdx.x) * DK * DV);
  if (tid == 0) {
    tc::mbar_init(&s_mbar, 1);
    tc::mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {
    tc::mbar_expect_tx(&s_mbar, DK * DV * 4);
    tc::bulk_load(s_state, Sn, DK * DV * 4, &s_mbar);
  }

  // ---- prologue of this token: conv step, Swish, gates ----
  const int HK = a.H * DK, HV = a.H * DV;
  const int sw = 2 * HK + HV;
  float* bufn = a.buf ? a.buf + static_cast<size_t>(n) * (a.K - 1) * sw : nullptr;
  // Every load of this token's prologue is issued before any store (the conv
  // rows are shifted in place only at the end), so the round trips overlap.
  auto load_taps = [&](const Tin* xp, int stride_x, int col_buf, int c, float (&bj)[3]) -> float {
#pragma unroll
    for (int j = 0; j < 3; ++j) bj[j] = j < a.K - 1 ? bufn[static_cast<size_t>(j) * sw + col_buf + c] : 0.f;
    return ldf(xp + static_cast<size_t>(n) * stride_x + c);
  };
  auto conv = [&](const float* w, int stride_x, int c, float xt, const float (&bj)[3]) -> float {
    float acc = w[c] * xt;  // w[0] x_t + sum_j w[K-1-j] buf[j]
#pragma unroll
    for (int j = 0; j < 3; ++j)
      if (j < a.K - 1) acc += w[(a.K - 1 - j) * stride_x + c] * bj[j];
    return acc;
  };
  auto shift = [&](int col_buf, int c, float xt, const float (&bj)[3]) {  // oldest row out, x_t in
#pragma unroll
    for (int j = 0; j < 3; ++j)
      if (j < a.K - 1) bufn[static_cast<size_t>(j) * sw + col_buf + c] = j + 1 < a.K - 1 ? bj[j + 1] : xt;
  };
  float qv = 0.f, kv = 0.f;
  if (tid < DK) {
    const int c = h * DK + tid;
    float bq[3], bk[3];
    const float xq = load_taps(static_cast<const Tin*>(a.qp), HK, 0, c, bq);
    const float xk = load_taps(static_cast<const Tin*>(a.kp), HK, HK, c, bk);
    const float u = ldf(static_cast<const Tin*>(a.z) + static_cast<size_t>(n) * HK + c) + (a.b_gate ? a.b_gate[c] : 0.f);
    const float cq = conv(a.w[0], HK, c, xq, bq);
    const float ck = conv(a.w[1], HK, c, xk, bk);
    qv = cq * sigmoidf_(cq);
    kv = ck * sigmoidf_(ck);
    const float ea = __expf(a.A[h]);
    const float g = a.gate_kind == KDA_GATE_SIGMOID_MIN ? a.g_min * sigmoidf_(ea * u) : -ea * softplusf_(u);
    s_a[tid] = __expf(g);
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      s_nrm[0][warp] = sq;
      s_nrm[1][warp] = sk;
    }
    shift(0, c, xq, bq);
    shift(HK, c, xk, bk);
  } else if (tid < DK + DV) {
    const int c = h * DV + tid - DK;
    float bv[3];
    const float xv = load_taps(static_cast<const Tin*>(a.vp), HV, 2 * HK, c, bv);
    const float cv = conv(a.w[2], HV, c, xv, bv);
    s_v[tid - DK] = cv * sigmoidf_(cv);
    shift(2 * HK, c, xv, bv);
  }
  if (tid == kDecThreads - 1)
    s_beta = sigmoidf_(ldf(static_cast<const Tin*>(a.beta_logit) + static_cast<size_t>(n) * a.H + h));
  __syncthreads();
  if (tid < DK) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int w = 0; w < DK / 32; ++w) {
      sq += s_nrm[0][w];
      sk += s_nrm[1][w];
    }
    const float q = qv / (sqrtf(sq) + kL2Eps), k = kv / (sqrtf(sk) + kL2Eps);
    s_q[tid] = q;
    s_ak[tid] = s_a[tid] * k;
    s_bk[tid] = s_beta * k;
  }
  __syncthreads();

  // ---- delta-rule update ----
  if (!__syncthreads_and(tc::mbar_wait(&s_mbar, 0))) {
    if (tid == 0 && a.err) atomicExch(a.err, 1);
    tc::mbar_wait(&s_mbar, 0);  // the copy may still land: wait (bounded) before leaving
    return;
  }
  auto srow = [&](int m) { return *reinterpret_cast<const float4*>(&s_state[(row0 + m * RPP) * DV + col]); };
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const float w = s_ak[row0 + m * RPP];
    const float4 sv = srow(m);
    r.x += w * sv.x; r.y += w * sv.y; r.z += w * sv.z; r.w += w * sv.w;
  }
  *reinterpret_cast<float4*>(&s_red[row0][col]) = r;
  __syncthreads();
  r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int p = 0; p < RPP; ++p) {
    const float4 t = *reinterpret_cast<const float4*>(&s_red[p][col]);
    r.x += t.x; r.y += t.y; r.z += t.z; r.w += t.w;
  }
  const float4 u = make_float4(s_v[col] - r.x, s_v[col + 1] - r.y, s_v[col + 2] - r.z, s_v[col + 3] - r.w);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const int d = row0 + m * RPP;
    const float al = s_a[d], bk = s_bk[d], qd = s_q[d];
    const float4 sv = srow(m);
    float4 t;
    t.x = al * sv.x + bk * u.x; t.y = al * sv.y + bk * u.y;
    t.z = al * sv.z + bk * u.z; t.w = al * sv.w + bk * u.w;
    Sn[(d * DV + col) / 4] = t;
    acc.x += qd * t.x; acc.y += qd * t.y; acc.z += qd * t.z; acc.w += qd * t.w;
  }
  __syncthreads();
  *reinterpret_cast<float4*>(&s_red[row0][col]) = acc;
  __syncthreads();
  if (tid < TPR) {  // one warp (DV = 128) or half a warp (DV = 64) holds o
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < RPP; ++p) {
      const float4 x = *reinterpret_cast<const float4*>(&s_red[p][col]);
      o[0] += x.x; o[1] += x.y; o[2] += x.z; o[3] += x.w;
    }
    if (a.gate) {  // sigmoid(gate) * o / sqrt(mean(o^2) + eps)
      float ss = o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3];
#pragma unroll
      for (int off = TPR / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(TPR == 32 ? 0xffffffffu : 0xffffu, ss, off);
      const float rr = 1.f / sqrtf(ss / DV + a.rms_eps);
      const Tin* gp = static_cast<const Tin*>(a.gate) + static_cast<size_t>(n) * HV + h * DV + col;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = sigmoidf_(ldf(gp + j)) * o[j] * rr;
    }
    To* on = static_cast<To*>(a.out) + static_cast<size_t>(blockIdx.x) * DV + col;
#pragma unroll
    for (int j = 0; j < 4; ++j) stf(on + j, o[j]);
  }
}

}  // namespace

__device__ int g_decode_fused_error = 0;  // set when a state copy's wait timed out

int decode_fused_error_flag(int* value, bool clear, cudaStream_t st) {
  static const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(value, g_decode_fused_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) !=
      cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (clear &&
      cudaMemcpyToSymbolAsync(g_decode_fused_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  return KDA_OK;
}

namespace {

template <int CPL, bool VARLEN, typename Tin, typename Tout>
int launch_prologue_v(ProArgs& a, int roles, int n_roles, bool bwd, cudaStream_t st) {
  a.roles = roles;
  const int w = bwd ? kBwdWarps : kWarps;
  const int groups = (a.n_strips + w - 1) / w;
  // forward: heads along x, so the blocks in flight read every head of the same
  // token rows (whole DRAM rows; measured 4 % faster); the backward, bound by its
  // arithmetic, keeps (strip groups, heads)
  a.head_x = !bwd && groups <= 65535;
  const dim3 grid(a.head_x ? a.H : groups, a.head_x ? groups : a.H, n_roles);
  static std::atomic<bool> done_f[64], done_b[64];
  if (bwd) {
    constexpr int smem = kBwdWarps * bwd_ring_bytes<CPL, Tin, Tout>();
    const int rc = ensure_smem(prologue_bwd_kernel<CPL, VARLEN, Tin, Tout>, smem, done_b);
    if (rc != KDA_OK) return rc;
    prologue_bwd_kernel<CPL, VARLEN, Tin, Tout><<<grid, w * 32, smem, st>>>(a);
  } else {
    constexpr int smem = kWarps * fwd_ring_bytes<CPL, Tin>();
    const int rc = ensure_smem(prologue_fwd_kernel<CPL, VARLEN, Tin, Tout>, smem, done_f);
    if (rc != KDA_OK) return rc;
    prologue_fwd_kernel<CPL, VARLEN, Tin, Tout><<<grid, w * 32, smem, st>>>(a);
  }
  return launch_status();
}

template <int CPL, typename Tin, typename Tout>
int launch_prologue_d(ProArgs& a, int roles, int n_roles, bool bwd, cudaStream_t st) {
  return a.cu ? launch_prologue_v<CPL, true, Tin, Tout>(a, roles, n_roles, bwd, st)
              : launch_prologue_v<CPL, false, Tin, Tout>(a, roles, n_roles, bwd, st);
}

// q, k and the gates have width dk, v has dv: one launch when they agree.
template <typename Tin, typename Tout>
int launch_prologue(ProArgs& a, bool bwd, cudaStream_t st) {
  auto launch = [&](int D, int roles, int n) {
    return D == 128 ? launch_prologue_d<4, Tin, Tout>(a, roles, n, bwd, st)
                    : launch_prologue_d<2, Tin, Tout>(a, roles, n, bwd, st);
  };
  if (a.dk == a.dv) return launch(a.dk, 0x3210, 4);
  const int rc = launch(a.dk, 0x310, 3);
  return rc != KDA_OK ? rc : launch(a.dv, 0x2, 1);
}

template <int CPL, typename To, typename Tg, typename Ty>
int launch_grms(const void* o, const void* gate, const void* dy, void* y, void* dout, void* dgate,
                long long rows, float eps, bool bwd, const RowMap& m, cudaStream_t st) {
  const long long want = (rows + 7) / 8;
  const int grid = static_cast<int>(want < 148LL * 16 ? want : 148LL * 16);
  if (bwd) {
    gated_rms_bwd_kernel<CPL, To, Tg, Ty><<<grid, 256, 0, st>>>(
        static_cast<const To*>(o), static_cast<const Tg*>(gate), static_cast<const Ty*>(dy),
        static_cast<To*>(dout), static_cast<Tg*>(dgate), rows, eps, m);
    if (m.out_rows && m.n_seqs > 0)  // do's pad rows: zero cotangents for the core
      zero_pad_rows_kernel<To><<<m.n_seqs, 256, 0, st>>>(static_cast<To*>(dout), m, m.H * CPL * 32);
  } else {
    gated_rms_fwd_kernel<CPL, To, Tg, Ty><<<grid, 256, 0, st>>>(
        static_cast<const To*>(o), static_cast<const Tg*>(gate), static_cast<Ty*>(y), rows, eps, m);
  }
  return launch_status();
}

template <int CPL>
int grms_types(const void* o, const void* gate, const void* dy, void* y, void* dout, void* dgate, long long rows,
               float eps, int odt, int gdt, int ydt, bool bwd, const RowMap& m, cudaStream_t st) {
  // o and y in either type; the gate logits in either type
#define KDA_GRMS(TO, TG, TY)                                                                               \
  if (odt == (std::is_same<TO, float>::value ? KDA_F32 : KDA_BF16) &&                                      \
      gdt == (std::is_same<TG, float>::value ? KDA_F32 : KDA_BF16) &&                                      \
      ydt == (std::is_same<TY, float>::value ? KDA_F32 : KDA_BF16))                                        \
    return launch_grms<CPL, TO, TG, TY>(o, gate, dy, y, dout, dgate, rows, eps, bwd, m, st);
  KDA_GRMS(float, float, float)
  KDA_GRMS(float, float, bf16)
  KDA_GRMS(float, bf16, float)
  KDA_GRMS(float, bf16, bf16)
  KDA_GRMS(bf16, float, float)
  KDA_GRMS(bf16, float, bf16)
  KDA_GRMS(bf16, bf16, float)
  KDA_GRMS(bf16, bf16, bf16)
#undef KDA_GRMS
  return KDA_ERR_DTYPE;
}

template <int DK, int DV, typename Tin, typename To>
int dec_launch(const DecArgs& a, int N, cudaStream_t st) {
  static std::atomic<bool> done[64];
  constexpr int smem = DK * DV * 4;
  const int rc = ensure_smem(decode_fused_kernel<DK, DV, Tin, To>, smem, done);
  if (rc != KDA_OK) return rc;
  decode_fused_kernel<DK, DV, Tin, To><<<N * a.H, kDecThreads, smem, st>>>(a);
  return launch_status();
}

template <int DK, int DV>
int dec_types(const DecArgs& a, int N, int in_dt, int o_dt, cudaStream_t st) {
  if (in_dt == KDA_BF16 && o_dt == KDA_BF16) return dec_launch<DK, DV, bf16, bf16>(a, N, st);
  if (in_dt == KDA_BF16 && o_dt == KDA_F32) return dec_launch<DK, DV, bf16, float>(a, N, st);
  if (in_dt == KDA_F32 && o_dt == KDA_F32) return dec_launch<DK, DV, float, float>(a, N, st);
  if (in_dt == KDA_F32 && o_dt == KDA_BF16) return dec_launch<DK, DV, float, bf16>(a, N, st);
  return KDA_ERR_DTYPE;
}

}  // namespace

// ------------------------------------------------------------- entry points ----

int prologue_launch(ProArgs& a, int in_dt, int out_dt, bool bwd, cudaStream_t st) {
  if (in_dt == KDA_BF16 && out_dt == KDA_BF16) return launch_prologue<bf16, bf16>(a, bwd, st);
  if (in_dt == KDA_BF16 && out_dt == KDA_F32) return launch_prologue<bf16, float>(a, bwd, st);
  if (in_dt == KDA_F32 && out_dt == KDA_F32) return launch_prologue<float, float>(a, bwd, st);
  if (in_dt == KDA_F32 && out_dt == KDA_BF16) return launch_prologue<float, bf16>(a, bwd, st);
  return KDA_ERR_DTYPE;
}

}  // namespace kda

namespace {

bool valid_dt(int d) { return d == KDA_F32 || d == KDA_BF16; }
bool d_ok(int d) { return d == 64 || d == 128; }

// Shared validation of the prologue's dimensions and pointers.
int prologue_check(const void* qp, const void* kp, const void* vp, const void* z, const void* bl,
                   const float* cq, const float* ck, const float* cv, const float* A, int kind,
                   const float* st_in, const float* st_out, const int* cu, int n_seqs, int B, int T, int H,
                   int dk, int dv, int K, int in_dt, int out_dt) {
  if (B < 0 || T < 0 || H < 0 || H > 65535 || K < 1 || K > 4 || !d_ok(dk) || !d_ok(dv)) return KDA_ERR_SHAPE;
  if (!valid_dt(in_dt) || !valid_dt(out_dt)) return KDA_ERR_DTYPE;
  if (kind != KDA_GATE_SIGMOID_MIN && kind != KDA_GATE_SOFTPLUS) return KDA_ERR_SHAPE;
  if (cu && (B != 1 || n_seqs < 1 || st_in || st_out)) return KDA_ERR_SHAPE;
  if (B == 0 || T == 0 || H == 0) return KDA_OK;
  if (!qp || !kp || !vp || !z || !bl || !cq || !ck || !cv || !A) return KDA_ERR_NULL;
  const void* al[] = {qp, kp, vp, z, st_in, st_out};
  for (const void* p : al)
    if (p && !kda::aligned16(p)) return KDA_ERR_ALIGN;
  const long long strips = static_cast<long long>(B) * ((T + kda::kStrip - 1) / kda::kStrip);
  if (strips > 0x7fffffffLL) return KDA_ERR_SHAPE;
  return KDA_OK;
}

kda::ProArgs base_args(const void* qp, const void* kp, const void* vp, const void* z, const void* bl,
                       const float* cq, const float* ck, const float* cv, const float* b_gate,
                       const float* A, float g_min, int kind, const float* st_in, const int* cu,
                       int n_seqs, const int* out_rows, int B, int T, int H, int dk, int dv, int K) {
  kda::ProArgs a{};
  a.x[0] = qp; a.x[1] = kp; a.x[2] = vp; a.x[3] = z;
  a.beta_logit = bl;
  a.w[0] = cq; a.w[1] = ck; a.w[2] = cv;
  a.b_gate = b_gate; a.A = A; a.g_min = g_min; a.gate_kind = kind;
  a.st_in = st_in; a.cu = cu; a.n_seqs = n_seqs; a.out_rows = out_rows;
  a.B = B; a.T = T; a.H = H; a.dk = dk; a.dv = dv; a.K = K;
  a.spb = (T + kda::kStrip - 1) / kda::kStrip;
  a.n_strips = B * a.spb;
  return a;
}

int ws_stride(int H, int dk, int dv, int K) { return 2 * K * H * dk + K * H * dv + H * dk + H; }
size_t ws_groups(int B, int T) {
  const size_t strips = static_cast<size_t>(B) * ((static_cast<size_t>(T) + kda::kStrip - 1) / kda::kStrip);
  return (strips + kda::kBwdWarps - 1) / kda::kBwdWarps;
}

}  // namespace

extern "C" {

int kda_prologue_fwd(const void* qp, const void* kp, const void* vp, const void* z, const void* beta_logit,
                     const float* conv_q, const float* conv_k, const float* conv_v, const float* b_gate,
                     const float* A, float g_min, int gate_kind, const float* conv_state_in,
                     float* conv_state_out, const int* cu_seqlens, int n_seqs, const int* out_rows, void* q,
                     void* k, void* v, void* g, void* beta, int B, int T, int H, int dk, int dv, int K,
                     int in_dtype, int out_dtype, kda_stream_t stream) {
  int rc = prologue_check(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, gate_kind, conv_state_in,
                          conv_state_out, cu_seqlens, n_seqs, B, T, H, dk, dv, K, in_dtype, out_dtype);
  if (rc == KDA_OK && out_rows && !cu_seqlens) rc = KDA_ERR_SHAPE;
  if (rc != KDA_OK || B == 0 || T == 0 || H == 0) return rc;
  if (!q || !k || !v || !g || !beta) return KDA_ERR_NULL;
  const void* al[] = {q, k, v, g};
  for (const void* p : al)
    if (!kda::aligned16(p)) return KDA_ERR_ALIGN;
  kda::ProArgs a = base_args(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, b_gate, A, g_min, gate_kind,
                             conv_state_in, cu_seqlens, n_seqs, out_rows, B, T, H, dk, dv, K);
  a.st_out = conv_state_out;
  a.y[0] = q; a.y[1] = k; a.y[2] = v; a.y[3] = g;
  a.beta = beta;
  return kda::prologue_launch(a, in_dtype, out_dtype, false, stream);
}

size_t kda_prologue_bwd_workspace_bytes(int B, int T, int H, int dk, int dv, int K) {
  if (B < 0 || T < 0 || H < 0 || K < 1 || K > 4 || !d_ok(dk) || !d_ok(dv)) return 0;
  return ws_groups(B, T) * static_cast<size_t>(ws_stride(H, dk, dv, K)) * sizeof(float);
}

int kda_prologue_bwd(const void* qp, const void* kp, const void* vp, const void* z, const void* beta_logit,
                     const float* conv_q, const float* conv_k, const float* conv_v, const float* b_gate,
                     const float* A, float g_min, int gate_kind, const float* conv_state_in,
                     const int* cu_seqlens, int n_seqs, const int* out_rows, const void* dq, const void* dk_,
                     const void* dv_,
                     const void* dg, const void* dbeta, void* dqp, void* dkp, void* dvp, void* dz,
                     void* dbeta_logit, float* dconv_q, float* dconv_k, float* dconv_v, float* db_gate,
                     float* dA, float* dconv_state_in, void* workspace, size_t workspace_bytes, int B, int T,
                     int H, int dk, int dv, int K, int in_dtype, int out_dtype, kda_stream_t stream) {
  int rc = prologue_check(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, A, gate_kind, conv_state_in,
                          dconv_state_in, cu_seqlens, n_seqs, B, T, H, dk, dv, K, in_dtype, out_dtype);
  if (rc == KDA_OK && out_rows && !cu_seqlens) rc = KDA_ERR_SHAPE;
  if (rc != KDA_OK) return rc;
  if (!dconv_q || !dconv_k || !dconv_v || !db_gate || !dA) return KDA_ERR_NULL;
  const size_t nq = static_cast<size_t>(K) * H * dk, nv = static_cast<size_t>(K) * H * dv;
  if (B == 0 || T == 0 || H == 0) {  // no tokens: zero gradients
    cudaError_t e = cudaMemsetAsync(dconv_q, 0, nq * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(dconv_k, 0, nq * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(dconv_v, 0, nv * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(db_gate, 0, static_cast<size_t>(H) * dk * 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(dA, 0, static_cast<size_t>(H) * 4, stream);
    if (e == cudaSuccess && dconv_state_in && B > 0 && K > 1)
      e = cudaMemsetAsync(dconv_state_in, 0, static_cast<size_t>(B) * (K - 1) * H * (2 * dk + dv) * 4, stream);
    return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
  }
  if (!dq || !dk_ || !dv_ || !dg || !dbeta || !dqp || !dkp || !dvp || !dz || !dbeta_logit) return KDA_ERR_NULL;
  const void* al[] = {dq, dk_, dv_, dg, dqp, dkp, dvp, dz, dconv_state_in};
  for (const void* p : al)
    if (p && !kda::aligned16(p)) return KDA_ERR_ALIGN;
  const size_t need = kda_prologue_bwd_workspace_bytes(B, T, H, dk, dv, K);
  if (!workspace || workspace_bytes < need) return KDA_ERR_WORKSPACE;
  kda::ProArgs a = base_args(qp, kp, vp, z, beta_logit, conv_q, conv_k, conv_v, b_gate, A, g_min, gate_kind,
                             conv_state_in, cu_seqlens, n_seqs, out_rows, B, T, H, dk, dv, K);
  a.dy[0] = dq; a.dy[1] = dk_; a.dy[2] = dv_; a.dy[3] = dg;
  a.dbeta = dbeta;
  a.dx[0] = dqp; a.dx[1] = dkp; a.dx[2] = dvp; a.dx[3] = dz;
  a.dbeta_logit = dbeta_logit;
  a.dst = K > 1 ? dconv_state_in : nullptr;
  a.ws = static_cast<float*>(workspace);
  a.ws_stride = ws_stride(H, dk, dv, K);
  if (dconv_state_in && K == 1) {
    // K = 1 has no conv state; nothing to write
  }
  rc = kda::prologue_launch(a, in_dtype, out_dtype, true, stream);
  if (rc != KDA_OK) return rc;
  const int groups = static_cast<int>(ws_groups(B, T));
  kda::prologue_reduce_kernel<<<(a.ws_stride + 255) / 256, 256, 0, stream>>>(
      a.ws, groups, a.ws_stride, H, dk, dv, K, dconv_q, dconv_k, dconv_v, db_gate, dA);
  return kda::launch_status();
}

int kda_gated_rmsnorm_fwd(const void* o, const void* gate, void* y, const int* cu_seqlens, const int* out_rows,
                          int n_seqs, int N, int H, int dv, float eps, int o_dtype, int gate_dtype, int y_dtype,
                          kda_stream_t stream) {
  if (N < 0 || H < 0 || !d_ok(dv)) return KDA_ERR_SHAPE;
  if (!valid_dt(o_dtype) || !valid_dt(gate_dtype) || !valid_dt(y_dtype)) return KDA_ERR_DTYPE;
  if (out_rows && (!cu_seqlens || n_seqs < 1)) return KDA_ERR_SHAPE;
  if (N == 0 || H == 0) return KDA_OK;
  if (!o || !gate || !y) return KDA_ERR_NULL;
  if (!kda::aligned16(o) || !kda::aligned16(gate) || !kda::aligned16(y)) return KDA_ERR_ALIGN;
  const long long rows = static_cast<long long>(N) * H;
  const kda::RowMap m{cu_seqlens, out_rows, n_seqs, H};
  return dv == 128 ? kda::grms_types<4>(o, gate, nullptr, y, nullptr, nullptr, rows, eps, o_dtype, gate_dtype,
                                        y_dtype, false, m, stream)
                   : kda::grms_types<2>(o, gate, nullptr, y, nullptr, nullptr, rows, eps, o_dtype, gate_dtype,
                                        y_dtype, false, m, stream);
}

int kda_gated_rmsnorm_bwd(const void* o, const void* gate, const void* dy, void* do_, void* dgate,
                          const int* cu_seqlens, const int* out_rows, int n_seqs, int N, int H, int dv, float eps,
                          int o_dtype, int gate_dtype, int y_dtype, kda_stream_t stream) {
  if (N < 0 || H < 0 || !d_ok(dv)) return KDA_ERR_SHAPE;
  if (!valid_dt(o_dtype) || !valid_dt(gate_dtype) || !valid_dt(y_dtype)) return KDA_ERR_DTYPE;
  if (out_rows && (!cu_seqlens || n_seqs < 1)) return KDA_ERR_SHAPE;
  if (N == 0 || H == 0) return KDA_OK;
  if (!o || !gate || !dy || !do_ || !dgate) return KDA_ERR_NULL;
  const void* al[] = {o, gate, dy, do_, dgate};
  for (const void* p : al)
    if (!kda::aligned16(p)) return KDA_ERR_ALIGN;
  const long long rows = static_cast<long long>(N) * H;
  const kda::RowMap m{cu_seqlens, out_rows, n_seqs, H};
  return dv == 128 ? kda::grms_types<4>(o, gate, dy, nullptr, do_, dgate, rows, eps, o_dtype, gate_dtype,
                                        y_dtype, true, m, stream)
                   : kda::grms_types<2>(o, gate, dy, nullptr, do_, dgate, rows, eps, o_dtype, gate_dtype,
                                        y_dtype, true, m, stream);
}

int kda_decode_fused(float* S, float* conv_buf, const void* qp, const void* kp, const void* vp, const void* z,
                     const void* beta_logit, const void* gate_logit, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* b_gate, const float* A, float g_min, int gate_kind,
                     float rms_eps, void* out, int N, int H, int dk, int dv, int K, int in_dtype, int out_dtype,
                     kda_stream_t stream) {
  if (N < 0 || H < 0 || H > 65535 || K < 1 || K > 4 || !d_ok(dk) || !d_ok(dv)) return KDA_ERR_SHAPE;
  if (!valid_dt(in_dtype) || !valid_dt(out_dtype)) return KDA_ERR_DTYPE;
  if (gate_kind != KDA_GATE_SIGMOID_MIN && gate_kind != KDA_GATE_SOFTPLUS) return KDA_ERR_SHAPE;
  if (N == 0 || H == 0) return KDA_OK;
  if (static_cast<long long>(N) * H > 0x7fffffffLL) return KDA_ERR_SHAPE;
  if (!S || !qp || !kp || !vp || !z || !beta_logit || !conv_q || !conv_k || !conv_v || !A || !out)
    return KDA_ERR_NULL;
  if (K > 1 && !conv_buf) return KDA_ERR_NULL;
  if (!kda::aligned16(S)) return KDA_ERR_ALIGN;
  kda::DecArgs a{};
  a.S = S; a.buf = K > 1 ? conv_buf : nullptr;
  a.qp = qp; a.kp = kp; a.vp = vp; a.z = z; a.beta_logit = beta_logit; a.gate = gate_logit;
  a.w[0] = conv_q; a.w[1] = conv_k; a.w[2] = conv_v;
  a.b_gate = b_gate; a.A = A; a.g_min = g_min; a.gate_kind = gate_kind; a.rms_eps = rms_eps;
  a.out = out; a.H = H; a.K = K;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&a.err), kda::g_decode_fused_error) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (dk == 128 && dv == 128) return kda::dec_types<128, 128>(a, N, in_dtype, out_dtype, stream);
  if (dk == 64 && dv == 128) return kda::dec_types<64, 128>(a, N, in_dtype, out_dtype, stream);
  if (dk == 128 && dv == 64) return kda::dec_types<128, 64>(a, N, in_dtype, out_dtype, stream);
  return kda::dec_types<64, 64>(a, N, in_dtype, out_dtype, stream);
}

}  // extern "C"
