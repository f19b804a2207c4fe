// kda_bwd_noalloc: the fused backward for callers that cannot allocate device
// memory themselves.
//
// kda_bwd needs scratch memory (one bf16 state cotangent per chunk on the
// tensor-core path, a per-(batch, head) working set on the fp32 path) and asks
// the caller for it.  Some callers cannot provide it: a framework's custom-call
// handler runs on memory the framework owns and accounts for (and that it has
// often reserved almost entirely up front), so a cudaMalloc issued from inside
// the handler either fails or silently takes memory the framework believes is
// free; cudaMalloc also synchronises the device, which stalls every other
// stream the framework is driving; and serving loops with a fixed memory
// budget must not allocate per call.  For those callers the scratch lives in
// a file-scope device array of fixed size, KDA_NOALLOC_SCRATCH_BYTES, that the
// CUDA runtime creates on every device the first time this library's kernels
// are loaded there, and keeps until the process exits.
//
// Contract:
// * Problems whose kda_bwd_workspace_bytes exceeds KDA_NOALLOC_SCRATCH_BYTES
//   are rejected with KDA_ERR_SCRATCH_LIMIT before anything is launched.
// * The first call on a device looks up the device address of the array
//   (cudaGetSymbolAddress, with that device current).  Make that first call
//   before any stream capture on the device.  The address is cached for the
//   life of the process and is valid for as long as the device's primary
//   context lives: after cudaDeviceReset (or anything else that destroys that
//   context) the cached address is stale, so such a process must not call this
//   entry point again.
// * Every call uses the same array.  Nothing in it needs to start at zero: the
//   backward writes every scratch byte it reads earlier in the same call, so the
//   leftovers of the previous call are harmless.  Two calls whose kernels
//   overlap on the GPU (different streams, or different host threads) race on
//   the array and produce wrong results; serialise them.
// * It allocates nothing (no cudaMalloc, no cudaFree, no allocating library
//   call) and otherwise behaves exactly like kda_bwd.
#include <mutex>

#include <cuda_runtime.h>

#include "kda_common.cuh"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[KDA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device (looked up once).
int scratch_on_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KDA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return KDA_ERR_DEVICE;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KDA_OK;
}

}  // namespace

extern "C" int kda_bwd_noalloc(const void* q, const void* k, const void* v, const void* g,
                               const void* beta, const void* s_ckpt, const void* do_,
                               const float* dsT, void* dq, void* dk_, void* dv_, void* dg,
                               void* dbeta, float* ds0, int B, int T, int H, int dk, int dv,
                               int chunk, int in_dtype, int do_dtype, int ckpt_dtype,
                               kda_stream_t stream) {
  const size_t need = kda_bwd_workspace_bytes(B, T, H, dk, dv, chunk, in_dtype);
  if (need > static_cast<size_t>(KDA_NOALLOC_SCRATCH_BYTES)) return KDA_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (B > 0 && H > 0 && T > 0) {
    const int rc = scratch_on_current_device(&scratch);
    if (rc != KDA_OK) return rc;
  }
  return kda_bwd(q, k, v, g, beta, s_ckpt, do_, dsT, dq, dk_, dv_, dg, dbeta, ds0, scratch,
                 KDA_NOALLOC_SCRATCH_BYTES, B, T, H, dk, dv, chunk, in_dtype, do_dtype,
                 ckpt_dtype, stream);
}
