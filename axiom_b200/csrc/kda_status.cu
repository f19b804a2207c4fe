// Device-side status of the kernels' bounded waits (kda_device_status) and a
// self-test of that path (kda_selftest_wait_timeout).  Each kernel family
// records a wait that gave up in its own device flag (atomicExch to 1); the
// accessors below read and optionally clear them on the caller's stream.
#include "kda_b200.h"
#include "kda_tc.cuh"

namespace kda {

int tc_fwd_error_flag(int* value, bool clear, cudaStream_t st);
int tc_fwd_split_error_flag(int* value, bool clear, cudaStream_t st);
int tc_bwd_error_flag(int* value, bool clear, cudaStream_t st);
int decode_fused_error_flag(int* value, bool clear, cudaStream_t st);

namespace {

__device__ int g_selftest_error = 0;

// One CTA waits on an mbarrier that nothing completes, with the same bounded
// wait the kernels use; it gives up after `polls` polls and sets the flag.
__global__ void selftest_wait_kernel(unsigned int polls) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  __syncthreads();
  const bool ok = tc::mbar_wait(&bar, 0u, polls);
  if (!ok && threadIdx.x == 0) atomicExch(&g_selftest_error, 1);
}

int selftest_error_flag(int* value, bool clear, cudaStream_t st) {
  static const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(value, g_selftest_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (clear && cudaMemcpyToSymbolAsync(g_selftest_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) !=
                   cudaSuccess)
    return KDA_ERR_LAUNCH;
  return KDA_OK;
}

}  // namespace
}  // namespace kda

extern "C" int kda_device_status(int* flags, int clear, kda_stream_t stream) {
  if (!flags) return KDA_ERR_NULL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int v[5] = {0, 0, 0, 0, 0};
  const bool c = clear != 0;
  int rc = kda::tc_fwd_error_flag(&v[0], c, st);
  if (rc == KDA_OK) rc = kda::tc_fwd_split_error_flag(&v[4], c, st);
  if (rc == KDA_OK) rc = kda::tc_bwd_error_flag(&v[1], c, st);
  if (rc == KDA_OK) rc = kda::decode_fused_error_flag(&v[2], c, st);
  if (rc == KDA_OK) rc = kda::selftest_error_flag(&v[3], c, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) rc = KDA_ERR_LAUNCH;
  if (rc != KDA_OK) return rc;
  *flags = ((v[0] || v[4]) ? KDA_STATUS_FWD : 0) | (v[1] ? KDA_STATUS_BWD : 0) | (v[2] ? KDA_STATUS_DECODE_FUSED : 0) |
           (v[3] ? KDA_STATUS_SELFTEST : 0);
  return KDA_OK;
}

extern "C" int kda_selftest_wait_timeout(unsigned int polls, kda_stream_t stream) {
  if (polls == 0) return KDA_ERR_SHAPE;
  kda::selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(polls);
  return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
