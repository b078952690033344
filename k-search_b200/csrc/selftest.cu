// Self-test of the bounded device waits (failure detection without a GPU
// fault). Every hand-off in the kernels of this library waits on an mbarrier
// through mbar_wait_for (kq_device.cuh), which gives up after a wall-clock
// limit, records the waiter's code in the device error word and lets the
// kernel run to completion instead of hanging. This entry runs that same wait
// on a barrier that nothing ever arrives at, with a caller-chosen (short)
// limit, so a test can make the wait run out and check the status that the
// host reads; the context stays usable afterwards.
#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

__global__ void wait_probe_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none ever comes
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait_for(&bar, 0, err, DEV_TIMEOUT_FULL, limit_ns);
}

}  // namespace
}  // namespace kq

using namespace kq;

extern "C" kq_status_t kq_selftest_wait_timeout(int64_t limit_ns, kq_stream_t stream) {
  if (limit_ns <= 0 || limit_ns > (int64_t)kWaitLimitNs)
    return fail(KQ_ERR_INVALID, "selftest: wait limit %lld ns outside (0, %llu]", (long long)limit_ns,
                (unsigned long long)kWaitLimitNs);
  int* err = device_error_word();
  if (!err) return fail(KQ_ERR_NOMEM, "device error word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  wait_probe_kernel<<<1, 32, 0, s>>>(err, (uint64_t)limit_ns);
  kq_status_t st = check_launch("wait probe");
  if (st) return st;
  if ((st = check_cuda(cudaStreamSynchronize(s), "wait probe sync"))) return st;
  int v = 0;
  if ((st = check_cuda(cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost), "wait probe error word"))) return st;
  if (v == DEV_TIMEOUT_FULL || v == DEV_TIMEOUT_EMPTY)
    return fail(KQ_ERR_TIMEOUT, "bounded device wait gave up after %lld ns (device error %d)", (long long)limit_ns, v);
  return KQ_OK;
}
