/*
 * kda_b200.h -- C ABI of the B200 (sm_100a) Kimi Delta Attention core.
 *
 * The library replaces the reference's KDA core interval (AXIOM, pure
 * JAX/Pallas): the operand-form whole-sequence scan and its custom_vjp,
 *
 *   cc_scan(q, k, v, alpha, beta32, S, tile, chunk) -> (o, S_T)
 *       net/kernels/kda_cc_fused_persist.py:920-932   (custom_vjp entry)
 *   kernel(...)      forward launch   net/kernels/kda_cc_fused_persist.py:718-759
 *   kernel_bwd(...)  backward launch  net/kernels/kda_cc_fused_persist.py:1707-1763
 *   _delta_step + o = S^T q           net/kda.py:298-310, :293  (decode)
 *
 * Conventions
 *   - Tensors are dense row-major device buffers:
 *       q, k, g : [B, T, H, dk]     v, o : [B, T, H, dv]     beta : [B, T, H]
 *       S0, S_T : [B, H, dk, dv] fp32
 *     (the reference's per-batch (T, H*D) interval layout with B in front).
 *   - g is the per-channel log-decay (alpha = exp(g), g <= 0); the reference
 *     passes alpha and takes log(alpha) itself, so dg here is its dalpha*alpha.
 *   - beta is the write gate per (token, head); the reference's beta32 is
 *     this value replicated over 32 columns.
 *   - T need not be a multiple of the chunk: the ragged tail is computed as
 *     zero-padded rows (q = k = v = 0, beta = 0, g = 0), which leaves the state
 *     and every real row exactly as the padded reference computes them.
 *   - Every entry point allocates nothing, never synchronises the host, and
 *     only enqueues work on `stream` (NULL = legacy default stream).  Scratch
 *     memory comes from the caller (`workspace`), except for kda_bwd_noalloc,
 *     which uses a fixed array built into the library (see its comment); all
 *     other entry points are stateless and may be called from several host
 *     threads at once, each on its own stream (the only state the library
 *     keeps is a per-device cache of launch attributes, held in atomics).
 *   - Return value: KDA_OK (0) or a negative KDA_ERR_* code; invalid shapes,
 *     dtypes, alignment or null pointers are rejected before any launch
 *     (fail-closed, the reference's typed-error contract net/kda.py:759-763).
 */
#ifndef KDA_B200_H
#define KDA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kda_stream_t;

/* element types */
enum {
  KDA_F32 = 0,
  KDA_BF16 = 1
};

/* status codes */
enum {
  KDA_OK = 0,
  KDA_ERR_SHAPE = -1,   /* unsupported or inconsistent dimensions */
  KDA_ERR_DTYPE = -2,   /* unsupported element type combination */
  KDA_ERR_ALIGN = -3,   /* a pointer is not 16-byte aligned */
  KDA_ERR_NULL = -4,    /* a required pointer is NULL */
  KDA_ERR_LAUNCH = -5,  /* the CUDA launch itself failed */
  KDA_ERR_WORKSPACE = -6, /* workspace missing or too small */
  KDA_ERR_DEVICE = -7,  /* no sm_100 device / device query failed */
  KDA_ERR_SCRATCH_LIMIT = -8, /* problem needs more than kda_bwd_noalloc's fixed scratch */
  KDA_ERR_TIMEOUT = -9  /* a kernel's bounded wait gave up (see kda_device_status) */
};

/* Device-side status bits (kda_device_status). */
enum {
  KDA_STATUS_FWD = 1,           /* tensor-core kda_fwd / kda_fwd_varlen */
  KDA_STATUS_BWD = 2,           /* tensor-core kda_bwd / kda_bwd_varlen / kda_bwd_noalloc */
  KDA_STATUS_DECODE_FUSED = 4,  /* kda_decode_fused */
  KDA_STATUS_SELFTEST = 8       /* kda_selftest_wait_timeout */
};

/* Library version (major*10000 + minor*100 + patch). */
int kda_version(void);

/* Human-readable text of a status code. */
const char* kda_strerror(int status);

/* Bytes of the checkpoint the forward stores for the backward (its
 * residuals).  It starts with the chunk-boundary states, [B, H, n, dk, dv]
 * elements of ckpt_dtype with n = ceil(T / chunk), entry c being the state
 * entering chunk c (the reference's pass-A state chain,
 * net/kernels/kda_cc_fused_persist.py:1282-1370).  On the tensor-core path
 * (bf16 inputs, dk = dv = 128, chunk = 64) it continues with a per-chunk
 * block (201 KB per chunk-head) of what the backward would otherwise
 * recompute: T = (I + diag(beta) Akk)^-1, Aqk, Akk (bf16 64 x 64 each),
 * W, Q Gam, K Gam, K Gam^-1, lam K, v~ = U - W S, U = T diag(beta) V (bf16
 * 64 x 128 each), Gam_C (fp32 x 128) and flags, then the state-chain
 * operands the split training forward hands from its chunk-parallel part to
 * its state scan (-(lam K)^T W, Q Gam - Aqk W, Aqk U).  The checkpoint is
 * an opaque blob passed from kda_fwd to kda_bwd: on the tensor-core path with
 * a bf16 checkpoint each state is stored as the shared-memory operand image
 * the kernels copy in one bulk transfer (8 x 8 core matrices of 128 bytes,
 * core (i, j) at byte ((i * dv / 8) + j) * 128, row-major inside), otherwise
 * row-major. */
size_t kda_ckpt_bytes(int B, int T, int H, int dk, int dv, int chunk, int in_dtype,
                      int ckpt_dtype);

/* Chunked forward (replaces kernel / cc_scan's forward rule,
 * net/kernels/kda_cc_fused_persist.py:718-759).
 *   in_dtype   : dtype of q, k, v, g, beta (KDA_F32 or KDA_BF16)
 *   o_dtype    : dtype of o
 *   s0         : [B,H,dk,dv] fp32 initial state, or NULL for zeros
 *   s_out      : [B,H,dk,dv] fp32 final state, or NULL
 *   s_ckpt     : the checkpoint for the backward (kda_ckpt_bytes bytes),
 *                or NULL when not training.
 * Supported: 1 <= dk, dv <= 128 (multiples of 8), chunk in {16, 32, 64}.
 * bf16 inputs with dk = dv = 128, chunk = 64 take the tensor-core path: one
 * kernel with one CTA per (batch, head) or, when s_ckpt is given and the
 * (batch, head) pairs fill at most half the SMs, three launches (chunk-parallel
 * prep, state scan sliced by state columns, chunk-parallel outputs) that meet
 * in the checkpoint.  The environment variables KDA_FWD_SCHEDULE
 * (split | fused) and KDA_SCAN_SLICES (1, 2, 4, 8) override the choice; the
 * results agree within the bf16 tolerance either way. */
int kda_fwd(const void* q, const void* k, const void* v, const void* g,
            const void* beta, const float* s0, void* o, float* s_out,
            void* s_ckpt, int B, int T, int H, int dk, int dv, int chunk,
            int in_dtype, int o_dtype, int ckpt_dtype, kda_stream_t stream);

/* Bytes of caller-provided scratch kda_bwd needs for these dimensions. */
size_t kda_bwd_workspace_bytes(int B, int T, int H, int dk, int dv, int chunk,
                               int in_dtype);

/* Fused backward (replaces kernel_bwd / cc_scan's backward rule,
 * net/kernels/kda_cc_fused_persist.py:1707-1763 and reference_bwd_scan
 * :794-849).  Walks the chunks in reverse, recomputing each chunk from its
 * checkpointed boundary state (s_ckpt written by kda_fwd with the same
 * dimensions, dtypes and ckpt_dtype), and produces
 *   dq, dk : [B,T,H,dk]   dv : [B,T,H,dv]   dg : [B,T,H,dk]   dbeta : [B,T,H]
 * in in_dtype, and ds0 : [B,H,dk,dv] fp32 (may be NULL).
 *   do_    : [B,T,H,dv] upstream cotangent of o, in do_dtype
 *   dsT    : [B,H,dk,dv] fp32 cotangent of the final state, or NULL (zero). */
int kda_bwd(const void* q, const void* k, const void* v, const void* g,
            const void* beta, const void* s_ckpt, const void* do_,
            const float* dsT, void* dq, void* dk_, void* dv_, void* dg,
            void* dbeta, float* ds0, void* workspace, size_t workspace_bytes,
            int B, int T, int H, int dk, int dv, int chunk, int in_dtype,
            int do_dtype, int ckpt_dtype, kda_stream_t stream);

/* Packed (variable-length) sequences.  No counterpart in the reference, which
 * pads every sequence of a batch to one length (net/kda.py:824-830); the
 * mixer's packed batches (cu_seqlens) need it.  The tensors hold n_seqs
 * sequences one after another in a single batch row (B = 1) of T tokens,
 * every sequence starting on a chunk boundary: rows padding a sequence to the
 * next boundary are zero (q = k = v = g = 0, beta = 0), which leaves the
 * state unchanged, so the states and every real row are those of the
 * unpadded sequences.  kda_prologue_fwd with out_rows = chunk * chunk_offsets
 * writes this layout from packed projections.
 *   chunk_offsets : device int32 [n_seqs + 1], the first chunk of each
 *                   sequence: chunk_offsets[0] = 0, non-decreasing,
 *                   chunk_offsets[n_seqs] = T / chunk
 *   s0, s_out, dsT, ds0 : [n_seqs, H, dk, dv] fp32 (per sequence)
 *   s_ckpt        : kda_ckpt_bytes(1, T, H, ...) bytes
 * T must be a multiple of chunk; everything else as kda_fwd / kda_bwd. */
int kda_fwd_varlen(const void* q, const void* k, const void* v, const void* g,
                   const void* beta, const float* s0, void* o, float* s_out,
                   void* s_ckpt, const int* chunk_offsets, int n_seqs, int T, int H,
                   int dk, int dv, int chunk, int in_dtype, int o_dtype, int ckpt_dtype,
                   kda_stream_t stream);

size_t kda_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv,
                                      int chunk, int in_dtype);

int kda_bwd_varlen(const void* q, const void* k, const void* v, const void* g,
                   const void* beta, const void* s_ckpt, const void* do_,
                   const float* dsT, void* dq, void* dk_, void* dv_, void* dg,
                   void* dbeta, float* ds0, void* workspace, size_t workspace_bytes,
                   const int* chunk_offsets, int n_seqs, int T, int H, int dk, int dv,
                   int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
                   kda_stream_t stream);

/* Size of the fixed device scratch array used by kda_bwd_noalloc (32 MiB). */
#define KDA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* kda_bwd for callers that cannot allocate device memory.  No counterpart in
 * the reference (XLA hands its kernels scratch through its own allocator).
 * A framework's custom-call handler, a serving loop with a fixed memory
 * budget, or any code that must not call cudaMalloc (it would take memory the
 * framework has reserved, and it synchronises the device) cannot supply
 * kda_bwd's workspace; this entry point takes the same arguments minus the
 * workspace and uses a file-scope device array of KDA_NOALLOC_SCRATCH_BYTES
 * instead, which every GPU that loads the library holds until exit.  It
 * allocates nothing.  Problems whose kda_bwd_workspace_bytes exceeds the
 * array are rejected with KDA_ERR_SCRATCH_LIMIT.  The first call on a device
 * looks up the array's device address (make it before any stream capture) and
 * keeps it for the life of the process: it stays valid while the device's
 * primary context lives, so a caller that resets the device (cudaDeviceReset)
 * or otherwise destroys that context must not call this entry point again in
 * the same process.  All calls share the array: calls whose kernels overlap on
 * the GPU race and must be serialised; no scratch content needs clearing
 * between calls. */
int kda_bwd_noalloc(const void* q, const void* k, const void* v, const void* g,
                    const void* beta, const void* s_ckpt, const void* do_,
                    const float* dsT, void* dq, void* dk_, void* dv_, void* dg,
                    void* dbeta, float* ds0, int B, int T, int H, int dk, int dv,
                    int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
                    kda_stream_t stream);

/* One recurrent decode step for N independent (sequence, head) states
 * (replaces _delta_step + o = S^T q, net/kda.py:298-310, :293):
 *   S <- diag(alpha) S - beta k ((alpha*k)^T S) + beta k v^T ;  o = S^T q
 * with alpha = exp(g).  S : [N, dk, dv] fp32, updated in place;
 * q, k, g : [N, dk]; v : [N, dv]; beta : [N] (in_dtype); o : [N, dv].
 * Supported: dk, dv in {64, 128}. */
int kda_decode(float* S, const void* q, const void* k, const void* v,
               const void* g, const void* beta, void* o, int N, int dk, int dv,
               int in_dtype, int o_dtype, kda_stream_t stream);

/* Every wait of a kernel on its own copies or MMAs (an mbarrier) is bounded:
 * when one gives up, the CTA records it in a device flag, skips its remaining
 * work, waits (again bounded) for its copies in flight, frees its tensor
 * memory and returns, so the context stays usable.  This reads those flags
 * as KDA_STATUS_* bits into *flags (0: no wait gave up since the last clear)
 * and, with clear != 0, resets them.  Unlike the compute entry points it
 * synchronises `stream` (the flags are read after its work).  Returns KDA_OK,
 * or KDA_ERR_LAUNCH if a copy fails. */
int kda_device_status(int* flags, int clear, kda_stream_t stream);

/* Exercises the bounded wait the kernels share: one CTA waits on an mbarrier
 * that nothing completes, gives up after `polls` polls (each ~0.1 us after
 * the first 64) and sets KDA_STATUS_SELFTEST.  For tests of the failure path;
 * it faults nothing. */
int kda_selftest_wait_timeout(unsigned int polls, kda_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_B200_H */
