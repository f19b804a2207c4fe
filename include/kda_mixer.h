/*
 * kda_mixer.h -- C ABI of the per-token work around the KDA core: the fused
 * prologue that turns the layer's projections into the core's inputs, the
 * output gate, and a fused streaming decode step.  Same conventions as
 * kda_b200.h (status codes, element types, no allocation, no host sync,
 * work only on `stream`), whose types this header uses.
 *
 * Reference interfaces replaced (AXIOM, pure JAX):
 *   kda_prologue_fwd/bwd   short_conv + _postprocess + sigmoid(beta) + decay gate
 *                          net/shortconv.py:14-30, net/kda.py:169-180, :194-203,
 *                          net/norm.py:15-61 (and their jax.grad)
 *   kda_gated_rmsnorm_*    _output_gate up to the W_o GEMM: sigmoid(gate) *
 *                          headwise_rms_norm(o)  net/kda.py:206-214, net/norm.py:70-73
 *   kda_decode_fused       recurrent_step without the projection GEMMs
 *                          net/kda.py:277-295 (short_conv_step net/shortconv.py:33-53)
 *
 * Layouts (row-major): projections qp, kp, z : [B, T, H*dk]; vp : [B, T, H*dv];
 * beta_logit : [B, T, H].  Conv weights are fp32 [K, H*d], w[i] weighting the
 * input i steps back (the reference's conv_q / conv_k / conv_v).  A conv state
 * is fp32 [B, K-1, H*dk | H*dk | H*dv]: the q, k and v buffers of
 * KDAState (net/kda.py:54-60) side by side, oldest row first.
 */
#ifndef KDA_MIXER_H
#define KDA_MIXER_H

#include "kda_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* decay-gate forms */
enum {
  KDA_GATE_SIGMOID_MIN = 0, /* g = g_min * sigmoid(exp(A_h) * (z + b))  net/kda.py:173-180 */
  KDA_GATE_SOFTPLUS = 1     /* g = -exp(A_h) * softplus(z + b)   (A holds A_log)          */
};

/* Fused prologue, forward: per (token, head)
 *   q = l2_norm(swish(conv_q * qp)),  k = l2_norm(swish(conv_k * kp)),
 *   v = swish(conv_v * vp),  beta = sigmoid(beta_logit),  g = gate(z + b_gate, A)
 * with the causal depthwise conv of K taps (1 <= K <= 4) and l2_norm's
 * x / (|x| + 1e-12).
 *   b_gate         : [H*dk] fp32 or NULL (zero);  A : [H] fp32
 *   conv_state_in  : fp32 conv state or NULL (zeros): inputs before t = 0
 *   conv_state_out : fp32 conv state or NULL: the last K-1 inputs (the next
 *                    call's conv_state_in); must not overlap conv_state_in
 *   cu_seqlens     : device int32 [n_seqs + 1] or NULL: packed sequences (B must
 *                    be 1, conv states NULL); every sequence starts from zeros
 *   out_rows       : device int32 [n_seqs + 1] or NULL (needs cu_seqlens): the
 *                    outputs' row of each sequence's first token; token t of
 *                    sequence s goes to row t - cu_seqlens[s] + out_rows[s] and
 *                    the rows after a sequence's last token up to
 *                    out_rows[s + 1] are written as zeros -- with
 *                    out_rows = chunk * chunk_offsets this is the packed layout
 *                    of kda_fwd_varlen
 *   q, k, g : [B,T',H,dk];  v : [B,T',H,dv];  beta : [B,T',H]   (out_dtype;
 *   T' = T, or out_rows[n_seqs])
 * Supported: dk, dv in {64, 128}; inputs in_dtype, outputs out_dtype
 * (KDA_BF16 or KDA_F32); every tensor pointer 16-byte aligned except beta
 * and beta_logit. */
int kda_prologue_fwd(const void* qp, const void* kp, const void* vp, const void* z,
                     const void* beta_logit, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* b_gate, const float* A, float g_min,
                     int gate_kind, const float* conv_state_in, float* conv_state_out,
                     const int* cu_seqlens, int n_seqs, const int* out_rows, void* q, void* k,
                     void* v, void* g, void* beta, int B, int T, int H, int dk, int dv, int K,
                     int in_dtype, int out_dtype, kda_stream_t stream);

/* Scratch bytes kda_prologue_bwd needs (per-block partial sums of the weight
 * gradients, reduced in a fixed order: the result is deterministic). */
size_t kda_prologue_bwd_workspace_bytes(int B, int T, int H, int dk, int dv, int K);

/* Fused prologue, backward: the same inputs, the cotangents of the forward's
 * outputs (dq, dk_, dg [B,T',H,dk], dv_ [B,T',H,dv], dbeta [B,T',H], out_dtype,
 * rows as the forward's outputs), and produces
 *   dqp, dkp, dz [B,T,H*dk], dvp [B,T,H*dv], dbeta_logit [B,T,H]   (in_dtype)
 *   dconv_q, dconv_k [K,H*dk], dconv_v [K,H*dv], db_gate [H*dk], dA [H]   (fp32,
 *   overwritten), dconv_state_in (fp32 conv state, or NULL).
 * The L2 norm's cotangent is zero at a zero vector (net/norm.py:26-48). */
int kda_prologue_bwd(const void* qp, const void* kp, const void* vp, const void* z,
                     const void* beta_logit, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* b_gate, const float* A, float g_min,
                     int gate_kind, const float* conv_state_in, const int* cu_seqlens,
                     int n_seqs, const int* out_rows, const void* dq, const void* dk_, const void* dv_,
                     const void* dg, const void* dbeta, void* dqp, void* dkp, void* dvp,
                     void* dz, void* dbeta_logit, float* dconv_q, float* dconv_k,
                     float* dconv_v, float* db_gate, float* dA, float* dconv_state_in,
                     void* workspace, size_t workspace_bytes, int B, int T, int H, int dk,
                     int dv, int K, int in_dtype, int out_dtype, kda_stream_t stream);

/* Output gate, forward: y = sigmoid(gate) * o / sqrt(mean_dv(o^2) + eps) per
 * (row, head) for N rows: gate logits and y [N, H*dv], o [N', H, dv] with row
 * t of y at row t of o, or (cu_seqlens and out_rows as kda_prologue_fwd's,
 * else NULL) at the packed layout's row of token t.
 * Supported: dv in {64, 128}; o, gate, y 16-byte aligned. */
int kda_gated_rmsnorm_fwd(const void* o, const void* gate, void* y, const int* cu_seqlens,
                          const int* out_rows, int n_seqs, int N, int H, int dv, float eps,
                          int o_dtype, int gate_dtype, int y_dtype, kda_stream_t stream);

/* Output gate, backward: do_ (o_dtype, o's rows; with out_rows its pad rows
 * are written as zeros) and dgate (gate_dtype) from dy (y_dtype). */
int kda_gated_rmsnorm_bwd(const void* o, const void* gate, const void* dy, void* do_,
                          void* dgate, const int* cu_seqlens, const int* out_rows, int n_seqs,
                          int N, int H, int dv, float eps, int o_dtype, int gate_dtype,
                          int y_dtype, kda_stream_t stream);

/* One streaming decode token for N sequences, H heads (recurrent_step
 * without the projection GEMMs): ShortConv steps over conv_buf (updated in
 * place), Swish, L2 norm, gates, the delta-rule update of S (in place) and
 * o = S^T q; with gate_logit ([N, H*dv]) the output is the gated RMSNorm of
 * o (eps rms_eps), else o itself.
 *   S : [N, H, dk, dv] fp32;  conv_buf : fp32 conv state of N sequences (NULL
 *   only when K == 1);  qp, kp, z : [N, H*dk];  vp : [N, H*dv];
 *   beta_logit : [N, H];  out : [N, H, dv] (out_dtype).
 * Supported: dk, dv in {64, 128}; S 16-byte aligned. */
int kda_decode_fused(float* S, float* conv_buf, const void* qp, const void* kp, const void* vp,
                     const void* z, const void* beta_logit, const void* gate_logit,
                     const float* conv_q, const float* conv_k, const float* conv_v,
                     const float* b_gate, const float* A, float g_min, int gate_kind,
                     float rms_eps, void* out, int N, int H, int dk, int dv, int K,
                     int in_dtype, int out_dtype, kda_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_MIXER_H */
