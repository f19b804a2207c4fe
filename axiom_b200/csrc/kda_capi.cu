// extern "C" entry points of libkda_b200.so: argument validation (fail
// closed, before any launch) and dispatch to the kernels.
#include <cstdlib>
#include <cstring>

#include <cuda_runtime.h>

#include "kda_ckpt_layout.h"
#include "kda_common.cuh"

namespace kda {
int decode_launch(float* S, const void* q, const void* k, const void* v, const void* g,
                  const void* beta, void* o, int N, int dk, int dv, int in_dt, int o_dt,
                  cudaStream_t st);
size_t simt_bwd_workspace_bytes(int B, int H, int dk, int dv, int C);
int simt_fwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
                    int dk, int dv, int C, int in_dt, int o_dt, int ck_dt, const int* cs, int n_seqs,
                    cudaStream_t st);
bool tc_fwd_supported(int dk, int dv, int C_, int in_dt);
constexpr size_t kTcFactorBytes = FAC_UNIT;  // factor block per chunk-head (kda_ckpt_layout.h)
int tc_fwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H,
                  int o_dt, int ck_dt, const int* cs, int n_seqs, cudaStream_t st);
int tc_fwd_split_slices(long long heads);
int tc_fwd_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                        const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H, int o_dt,
                        int ck_dt, const int* cs, int n_seqs, int slices, cudaStream_t st);
bool tc_bwd_supported(int dk, int dv, int C_, int in_dt, int do_dt);
size_t tc_bwd_workspace_bytes(int B, int T, int H);
int tc_bwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
                  void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T, int H,
                  int ck_dt, const int* cs, int n_seqs, cudaStream_t st);
int simt_bwd_launch(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const void* s_ckpt, const void* dout, const float* dsT, void* dq, void* dk_,
                    void* dv_, void* dg, void* dbeta, float* ds0, void* work, int B, int T,
                    int H, int dk, int dv, int C, int in_dt, int do_dt, int ck_dt,
                    int states_cm, const int* cs, int n_seqs, cudaStream_t st);
}  // namespace kda

namespace {

bool valid_dtype(int d) { return d == KDA_F32 || d == KDA_BF16; }

// Schedule of the tensor-core forward when a checkpoint is written (training):
// "split" (chunk-parallel prep + column-sliced state scan, kda_fwd_split.cu) or
// "fused" (one CTA per (sequence, head), kda_fwd_tc.cu).  The fused kernel's time
// is one head's chain of chunks, whatever the head count up to one CTA per SM;
// the split schedule's grows with the units but spreads a head over 2 to 8 SMs.
// By default the split one runs while the heads fill at most half the SMs (its
// state scan then takes two or more slices per head), the fused one otherwise;
// the environment variable KDA_FWD_SCHEDULE ("split" or "fused") overrides it.
// Without a checkpoint the fused kernel runs (the split schedule hands its
// work over in the checkpoint).
bool use_split_forward(long long heads) {
  const char* e = std::getenv("KDA_FWD_SCHEDULE");
  if (e && std::strcmp(e, "fused") == 0) return false;
  if (e && std::strcmp(e, "split") == 0) return true;
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  return 2 * heads <= n_sm;
}

int check_dims(int B, int T, int H, int dk, int dv, int chunk) {
  if (B < 0 || T < 0 || H < 0) return KDA_ERR_SHAPE;
  if (dk < 8 || dk > 128 || dk % 8 || dv < 8 || dv > 128 || dv % 8) return KDA_ERR_SHAPE;
  if (chunk != 16 && chunk != 32 && chunk != 64) return KDA_ERR_SHAPE;
  if (static_cast<long long>(B) * H > 65535LL * 65535LL) return KDA_ERR_SHAPE;
  if (B > 65535 || H > 65535) return KDA_ERR_SHAPE;
  return KDA_OK;
}

}  // namespace

extern "C" {

int kda_version(void) { return 100; }

const char* kda_strerror(int status) {
  switch (status) {
    case KDA_OK: return "ok";
    case KDA_ERR_SHAPE: return "unsupported or inconsistent dimensions";
    case KDA_ERR_DTYPE: return "unsupported element type";
    case KDA_ERR_ALIGN: return "pointer not 16-byte aligned";
    case KDA_ERR_NULL: return "required pointer is NULL";
    case KDA_ERR_LAUNCH: return "CUDA launch failed";
    case KDA_ERR_WORKSPACE: return "workspace missing or too small";
    case KDA_ERR_DEVICE: return "no usable CUDA device";
    case KDA_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than kda_bwd_noalloc's fixed array (KDA_NOALLOC_SCRATCH_BYTES)";
    case KDA_ERR_TIMEOUT: return "a kernel's bounded wait gave up (device status)";
    default: return "unknown status";
  }
}

size_t kda_ckpt_bytes(int B, int T, int H, int dk, int dv, int chunk, int in_dtype,
                      int ckpt_dtype) {
  if (check_dims(B, T, H, dk, dv, chunk) != KDA_OK || !valid_dtype(in_dtype) ||
      !valid_dtype(ckpt_dtype))
    return 0;
  const size_t n = (static_cast<size_t>(T) + chunk - 1) / chunk;
  const size_t units = static_cast<size_t>(B) * H * n;
  size_t bytes = units * dk * dv * (ckpt_dtype == KDA_F32 ? 4 : 2);
  if (kda::tc_fwd_supported(dk, dv, chunk, in_dtype)) bytes += units * kda::kTcFactorBytes;
  return bytes;
}

}  // extern "C"

namespace {

int fwd_impl(const void* q, const void* k, const void* v, const void* g, const void* beta,
             const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H, int dk,
             int dv, int chunk, int in_dtype, int o_dtype, int ckpt_dtype, const int* cs, int n_seqs,
             kda_stream_t stream) {
  int rc = check_dims(B, T, H, dk, dv, chunk);
  if (rc != KDA_OK) return rc;
  if (!valid_dtype(in_dtype) || !valid_dtype(o_dtype) || !valid_dtype(ckpt_dtype))
    return KDA_ERR_DTYPE;
  if (B == 0 || H == 0) return KDA_OK;
  if (T == 0) {
    if (s_out) {
      const size_t bytes = static_cast<size_t>(B) * H * dk * dv * sizeof(float);
      cudaError_t e = s0 ? cudaMemcpyAsync(s_out, s0, bytes, cudaMemcpyDeviceToDevice, stream)
                         : cudaMemsetAsync(s_out, 0, bytes, stream);
      return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
    }
    return KDA_OK;
  }
  if (!q || !k || !v || !g || !beta || !o) return KDA_ERR_NULL;
  if (kda::tc_fwd_supported(dk, dv, chunk, in_dtype)) {
    if (!kda::aligned16(q) || !kda::aligned16(k) || !kda::aligned16(v) || !kda::aligned16(g) ||
        !kda::aligned16(o) || (s_ckpt && !kda::aligned16(s_ckpt)) || (s_out && !kda::aligned16(s_out)) ||
        (s0 && !kda::aligned16(s0)))
      return KDA_ERR_ALIGN;
    const long long heads = static_cast<long long>(cs ? n_seqs : B) * H;
    if (s_ckpt && use_split_forward(heads)) {
      const int slices = kda::tc_fwd_split_slices(heads);
      return kda::tc_fwd_split_launch(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, o_dtype, ckpt_dtype, cs,
                                      n_seqs, slices, stream);
    }
    return kda::tc_fwd_launch(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, o_dtype, ckpt_dtype, cs,
                              n_seqs, stream);
  }
  return kda::simt_fwd_launch(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, dk, dv, chunk,
                              in_dtype, o_dtype, ckpt_dtype, cs, n_seqs, stream);
}

size_t bwd_ws_impl(int B, int n_state_rows, int T, int H, int dk, int dv, int chunk, int in_dtype) {
  if (check_dims(B, T, H, dk, dv, chunk) != KDA_OK) return 0;
  size_t n = kda::simt_bwd_workspace_bytes(n_state_rows, H, dk, dv, chunk);
  if (kda::tc_bwd_supported(dk, dv, chunk, in_dtype, KDA_BF16)) {
    const size_t t = kda::tc_bwd_workspace_bytes(B, T, H);
    if (t > n) n = t;
  }
  return n;
}

int bwd_impl(const void* q, const void* k, const void* v, const void* g, const void* beta,
             const void* s_ckpt, const void* do_, const float* dsT, void* dq, void* dk_, void* dv_,
             void* dg, void* dbeta, float* ds0, void* workspace, size_t workspace_bytes, int B,
             int T, int H, int dk, int dv, int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
             const int* cs, int n_seqs, kda_stream_t stream) {
  int rc = check_dims(B, T, H, dk, dv, chunk);
  if (rc != KDA_OK) return rc;
  if (!valid_dtype(in_dtype) || !valid_dtype(do_dtype) || !valid_dtype(ckpt_dtype))
    return KDA_ERR_DTYPE;
  if (B == 0 || H == 0) return KDA_OK;
  if (T == 0) {
    if (ds0) {
      const size_t bytes = static_cast<size_t>(B) * H * dk * dv * sizeof(float);
      cudaError_t e = dsT ? cudaMemcpyAsync(ds0, dsT, bytes, cudaMemcpyDeviceToDevice, stream)
                          : cudaMemsetAsync(ds0, 0, bytes, stream);
      return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
    }
    return KDA_OK;
  }
  if (!q || !k || !v || !g || !beta || !s_ckpt || !do_ || !dq || !dk_ || !dv_ || !dg || !dbeta)
    return KDA_ERR_NULL;
  if (kda::tc_bwd_supported(dk, dv, chunk, in_dtype, do_dtype)) {
    const size_t need = kda::tc_bwd_workspace_bytes(B, T, H);
    if (!workspace || workspace_bytes < need) return KDA_ERR_WORKSPACE;
    const void* ptrs[] = {q, k, v, g, do_, dq, dk_, dv_, dg, s_ckpt, workspace};
    for (const void* p : ptrs)
      if (!kda::aligned16(p)) return KDA_ERR_ALIGN;
    return kda::tc_bwd_launch(q, k, v, g, beta, s_ckpt, do_, dsT, dq, dk_, dv_, dg, dbeta, ds0,
                              workspace, B, T, H, ckpt_dtype, cs, n_seqs, stream);
  }
  const size_t need = kda::simt_bwd_workspace_bytes(cs ? n_seqs : B, H, dk, dv, chunk);
  if (need && (!workspace || workspace_bytes < need)) return KDA_ERR_WORKSPACE;
  // a bf16 checkpoint written by the tensor-core forward holds operand images
  const int states_cm = kda::tc_fwd_supported(dk, dv, chunk, in_dtype) && ckpt_dtype == KDA_BF16;
  return kda::simt_bwd_launch(q, k, v, g, beta, s_ckpt, do_, dsT, dq, dk_, dv_, dg, dbeta, ds0,
                              workspace, B, T, H, dk, dv, chunk, in_dtype, do_dtype, ckpt_dtype,
                              states_cm, cs, n_seqs, stream);
}

// Packed sequences: row 0 of a B = 1 batch holds n_seqs chunk-aligned sequences.
int check_packing(const int* cs, int n_seqs, int T, int chunk) {
  if (n_seqs < 0 || n_seqs > 65535 * 256) return KDA_ERR_SHAPE;
  if (chunk <= 0 || T < 0 || T % chunk != 0) return KDA_ERR_SHAPE;
  if (n_seqs > 0 && !cs) return KDA_ERR_NULL;
  return KDA_OK;
}

}  // namespace

extern "C" {

int kda_fwd(const void* q, const void* k, const void* v, const void* g, const void* beta,
            const float* s0, void* o, float* s_out, void* s_ckpt, int B, int T, int H, int dk,
            int dv, int chunk, int in_dtype, int o_dtype, int ckpt_dtype, kda_stream_t stream) {
  return fwd_impl(q, k, v, g, beta, s0, o, s_out, s_ckpt, B, T, H, dk, dv, chunk, in_dtype, o_dtype,
                  ckpt_dtype, nullptr, 0, stream);
}

int kda_fwd_varlen(const void* q, const void* k, const void* v, const void* g, const void* beta,
                   const float* s0, void* o, float* s_out, void* s_ckpt, const int* chunk_offsets,
                   int n_seqs, int T, int H, int dk, int dv, int chunk, int in_dtype, int o_dtype,
                   int ckpt_dtype, kda_stream_t stream) {
  int rc = check_packing(chunk_offsets, n_seqs, T, chunk);
  if (rc != KDA_OK) return rc;
  rc = check_dims(1, T, H, dk, dv, chunk);
  if (rc != KDA_OK || n_seqs == 0 || H == 0) return rc;
  if (T == 0) {  // empty sequences: S_T = S0
    if (!s_out) return KDA_OK;
    const size_t bytes = static_cast<size_t>(n_seqs) * H * dk * dv * sizeof(float);
    cudaError_t e = s0 ? cudaMemcpyAsync(s_out, s0, bytes, cudaMemcpyDeviceToDevice, stream)
                       : cudaMemsetAsync(s_out, 0, bytes, stream);
    return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
  }
  return fwd_impl(q, k, v, g, beta, s0, o, s_out, s_ckpt, 1, T, H, dk, dv, chunk, in_dtype, o_dtype,
                  ckpt_dtype, chunk_offsets, n_seqs, stream);
}

size_t kda_bwd_workspace_bytes(int B, int T, int H, int dk, int dv, int chunk, int in_dtype) {
  return bwd_ws_impl(B, B, T, H, dk, dv, chunk, in_dtype);
}

size_t kda_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv, int chunk,
                                      int in_dtype) {
  if (n_seqs < 0) return 0;
  return bwd_ws_impl(1, n_seqs, T, H, dk, dv, chunk, in_dtype);
}

int kda_bwd(const void* q, const void* k, const void* v, const void* g, const void* beta,
            const void* s_ckpt, const void* do_, const float* dsT, void* dq, void* dk_, void* dv_,
            void* dg, void* dbeta, float* ds0, void* workspace, size_t workspace_bytes, int B,
            int T, int H, int dk, int dv, int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
            kda_stream_t stream) {
  return bwd_impl(q, k, v, g, beta, s_ckpt, do_, dsT, dq, dk_, dv_, dg, dbeta, ds0, workspace,
                  workspace_bytes, B, T, H, dk, dv, chunk, in_dtype, do_dtype, ckpt_dtype, nullptr, 0,
                  stream);
}

int kda_bwd_varlen(const void* q, const void* k, const void* v, const void* g, const void* beta,
                   const void* s_ckpt, const void* do_, const float* dsT, void* dq, void* dk_,
                   void* dv_, void* dg, void* dbeta, float* ds0, void* workspace,
                   size_t workspace_bytes, const int* chunk_offsets, int n_seqs, int T, int H,
                   int dk, int dv, int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
                   kda_stream_t stream) {
  int rc = check_packing(chunk_offsets, n_seqs, T, chunk);
  if (rc != KDA_OK) return rc;
  rc = check_dims(1, T, H, dk, dv, chunk);
  if (rc != KDA_OK || n_seqs == 0 || H == 0) return rc;
  if (T == 0) {  // empty sequences: dS0 = dS_T
    if (!ds0) return KDA_OK;
    const size_t bytes = static_cast<size_t>(n_seqs) * H * dk * dv * sizeof(float);
    cudaError_t e = dsT ? cudaMemcpyAsync(ds0, dsT, bytes, cudaMemcpyDeviceToDevice, stream)
                        : cudaMemsetAsync(ds0, 0, bytes, stream);
    return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
  }
  return bwd_impl(q, k, v, g, beta, s_ckpt, do_, dsT, dq, dk_, dv_, dg, dbeta, ds0, workspace,
                  workspace_bytes, 1, T, H, dk, dv, chunk, in_dtype, do_dtype, ckpt_dtype, chunk_offsets,
                  n_seqs, stream);
}

int kda_decode(float* S, const void* q, const void* k, const void* v, const void* g,
               const void* beta, void* o, int N, int dk, int dv, int in_dtype, int o_dtype,
               kda_stream_t stream) {
  if (N < 0) return KDA_ERR_SHAPE;
  if (!valid_dtype(in_dtype) || !valid_dtype(o_dtype)) return KDA_ERR_DTYPE;
  if (!((dk == 64 || dk == 128) && (dv == 64 || dv == 128))) return KDA_ERR_SHAPE;
  if (N == 0) return KDA_OK;
  if (!S || !q || !k || !v || !g || !beta || !o) return KDA_ERR_NULL;
  if (!kda::aligned16(S)) return KDA_ERR_ALIGN;
  return kda::decode_launch(S, q, k, v, g, beta, o, N, dk, dv, in_dtype, o_dtype, stream);
}

}  // extern "C"
