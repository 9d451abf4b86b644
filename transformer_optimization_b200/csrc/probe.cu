// Test probe of the bounded-wait path shared by every pipeline kernel of the
// library (mbar_wait_ns in common.cuh): one CTA starts a 4 KiB bulk copy
// into shared memory, then waits on an mbarrier that nothing ever completes.
// The wait gives up after `limit_ns`, records kDevTimeoutProbe in the device
// status word, and the thread then drains what it issued (waits for its own
// copy) before the CTA leaves, as the GEMM and attention kernels do when one
// of their waits runs out. Nothing faults and nothing hangs: the only
// incomplete barrier lives in this CTA's shared memory and dies with it.
#include "common.cuh"
#include "launch.h"

namespace tfb {

constexpr int kProbeBytes = 4096;

__global__ void __launch_bounds__(32) wait_timeout_probe_kernel(const void* __restrict__ src, uint64_t limit_ns,
                                                                int* status, int* out) {
  __shared__ __align__(128) uint8_t buf[kProbeBytes];
  __shared__ __align__(8) uint64_t bars[2];
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);  // completes when the copy lands
    mbar_init(&bars[1], 1);  // nothing arrives on this one
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], kProbeBytes);
    bulk_load_1d(buf, src, kProbeBytes, &bars[0]);
    const bool completed = mbar_wait_ns(&bars[1], 0, status, kDevTimeoutProbe, limit_ns);
    // drain with the ordinary bound and no early exit on the raised status
    const bool drained = mbar_wait(&bars[0], 0, nullptr, kDevTimeoutDrain);
    out[0] = completed ? 0 : 1;
    out[1] = drained ? 1 : 0;
    out[2] = drained ? static_cast<int>(buf[kProbeBytes - 1]) : -1;  // a byte of the landed copy
  }
  __syncwarp();
}

int wait_timeout_probe(const void* src, long long limit_ns, int* out, cudaStream_t stream) {
  if (src == nullptr || out == nullptr) return set_error(TF_ERR_SHAPE, "wait probe: null pointer");
  if (!aligned16(src)) return set_error(TF_ERR_ALIGN, "wait probe: src must be 16-byte aligned");
  if (limit_ns < 1000 || limit_ns > 2000000000ll)
    return set_error(TF_ERR_SHAPE, "wait probe: limit_ns=%lld (1000 .. 2e9)", limit_ns);
  int* status = device_status_ptr();
  if (status == nullptr) return last_error_code();
  cudaError_t e = launch_k(wait_timeout_probe_kernel, dim3(1), dim3(32), 0, stream, src,
                           static_cast<uint64_t>(limit_ns), status, out);
  if (e != cudaSuccess) return set_error(TF_ERR_LAUNCH, "wait probe launch: %s", cudaGetErrorString(e));
  return TF_OK;
}

}  // namespace tfb
