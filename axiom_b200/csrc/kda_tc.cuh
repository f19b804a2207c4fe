// sm_100a building blocks for the tensor-core KDA kernels: tcgen05 (TMEM
// allocation, MMA issue, commit, TMEM loads/stores), mbarriers with bounded
// waits, cp.async copies and shared-memory matrix descriptors.
//
// Operand layout ("CM layout"): a bf16 tile of R rows x Cc columns is stored
// as 8x8 core matrices (8 rows x 16 bytes, 128 contiguous bytes), core matrix
// (rg, cg) at byte ((rg * Cc/8) + cg) * 128.  With SWIZZLE_NONE descriptors
// the same buffer is a K-major operand (rows = M/N, SBO = row-group stride,
// LBO = 128) or an MN-major operand (rows = K, SBO = 128, LBO = row-group
// stride), so a tile is used transposed without moving it.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace kda {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (r, c) of a CM-layout tile with `cols` columns.
__device__ __forceinline__ uint32_t cm_off(int r, int c, int cols) {
  return static_cast<uint32_t>((((r >> 3) * (cols >> 3) + (c >> 3)) << 7) + ((r & 7) << 4) + ((c & 7) << 1));
}

// ---- shared-memory matrix descriptor (SWIZZLE_NONE, sm_100 version 1) -----
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  return d;         // base offset 0, lbo mode 0, layout SWIZZLE_NONE
}

// K-major view of a CM tile with `cols` columns (rows = M or N, cols = K).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr, int cols) {
  return sdesc(saddr, 128u, static_cast<uint32_t>(cols >> 3) << 7);
}
// MN-major view of a CM tile with `cols` columns (rows = K, cols = M or N).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr, int cols) {
  return sdesc(saddr, static_cast<uint32_t>(cols >> 3) << 7, 128u);
}

// Instruction descriptor: kind::f16, bf16 x bf16 -> fp32.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format F32
         | (1u << 7)                                 // A format BF16
         | (1u << 10)                                // B format BF16
         | (static_cast<uint32_t>(a_mn_major) << 15)
         | (static_cast<uint32_t>(b_mn_major) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)
         | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---- TMEM ------------------------------------------------------------------
// Whole-warp operations.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(slot_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// One MMA of a precomputed issue table (32 bytes, in shared memory).  A kernel
// builds its table once; every MMA group is then issued by the same short loop,
// which stays in the instruction cache (an unrolled issue block per group runs
// once per work unit, cold, and costs about twice the tensor time).
struct MmaOp {
  uint64_t a, b;      // shared-memory descriptors
  uint32_t d, id;     // TMEM accumulator address, instruction descriptor
  uint32_t acc, pad;  // accumulate into d (else overwrite)
};
__device__ __forceinline__ void mma_op(MmaOp* t, int i, uint32_t d, uint64_t a, uint64_t b,
                                       uint32_t id, uint32_t acc) {
  t[i].a = a;
  t[i].b = b;
  t[i].d = d;
  t[i].id = id;
  t[i].acc = acc;
  t[i].pad = 0;
}
// Issues table entries [i0, i0 + n); one thread.
__device__ __forceinline__ void mma_run(const MmaOp* t, int i0, int n) {
#pragma unroll 2
  for (int i = i0; i < i0 + n; ++i) {
    const MmaOp op = t[i];
    mma_bf16(op.d, op.a, op.b, op.id, op.acc);
  }
}

// Arrive on an mbarrier once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(mbar)) : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread i gets lane (base+i), cols [c, c+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 8 columns: thread i gets lane (base+i), cols [c, c+8).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
// 32 lanes x 16 columns: thread i gets lane (base+i), cols [c, c+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
         "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
         "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]),
         "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
         "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- 8x8 b16 matrix moves (warp-collective) ---------------------------------
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(saddr));
}
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t saddr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};"
               :: "r"(saddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]) : "memory");
}

// Transpose a CM tile of R x Cc bf16 into a CM tile of Cc x R (core matrix
// (rg, cg) -> (cg, rg), each 8x8 block transposed), four core matrices per
// warp instruction; all warps of the CTA (nwarps) take part.
template <int R, int Cc>
__device__ __forceinline__ void transpose_cm(uint32_t dst, uint32_t src, int warp, int lane, int nwarps) {
  constexpr int NCM = (R / 8) * (Cc / 8);
  for (int j0 = 4 * warp; j0 < NCM; j0 += 4 * nwarps) {
    const int j = j0 + (lane >> 3), row = lane & 7;
    const int rg = j / (Cc / 8), cg = j % (Cc / 8);
    uint32_t f[4];
    ldmatrix_x4(f, src + ((rg * (Cc / 8) + cg) << 7) + (row << 4));
    stmatrix_x4_trans(dst + ((cg * (R / 8) + rg) << 7) + (row << 4), f);
  }
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(mbar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and never blocks forever) if the phase does not
// complete within `limit` polls; the caller then aborts cleanly.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(mbar, parity)) return true;
    if (i > 64) __nanosleep(64);
  }
  return false;
}

// ---- cp.async (16-byte global -> shared) ------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t n = valid ? 16u : 0u;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
               :: "r"(smem_u32(smem)), "l"(gmem), "r"(n) : "memory");
}
// All 16 bytes in range; `smem` a shared-window address.
__device__ __forceinline__ void cp_async16_s(uint32_t smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// ---- bulk copies (cp.async.bulk, contiguous, no tensor map) --------------------
// Copies (bulk and TMA) are issued by this thread, lane 0 of warp 1, so that
// they never queue behind thread 0's MMA issue (and the other way round).  The
// bulk async-group waits are per thread and are made by it too.
constexpr int kIoThread = 32;
// Issued by one thread.  Both addresses 16-byte aligned, size a multiple of 16.
// Arms `mbar` for one arrival plus `bytes` transaction bytes.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(mbar)), "r"(bytes) : "memory");
}
// global -> shared; completes `bytes` transaction bytes on `mbar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(mbar)) : "memory");
}
// shared -> global, tracked by this thread's bulk async-groups.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               :: "l"(dst), "r"(smem_u32(src)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared source of every committed bulk store but the newest N may be overwritten.
template <int N = 0>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}
// Every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Raw bf16 load kept as 16 bits: the value is converted where it is consumed,
// so no instruction waits on the load right after issuing it (a prefetch).
__device__ __forceinline__ unsigned short ld_bf16_raw(const __nv_bfloat16* p, bool valid) {
  unsigned short v = 0;
  if (valid) v = *reinterpret_cast<const unsigned short*>(p);
  return v;
}
__device__ __forceinline__ float bf16_raw_to_float(unsigned short v) {
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
}

// ---- bf16 packing ---------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void unpack_bf16x8(uint4 u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                    pack_bf16(f[6], f[7]));
}

}  // namespace tc
}  // namespace kda
