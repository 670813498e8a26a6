// Self-test of the failure path every TMA pipeline in this library shares: the
// bounded mbarrier wait (pk_common.cuh, mbar_wait_bounded) that gives up after
// a time limit and records PK_DEV_TIMEOUT in the caller's error word instead
// of hanging the GPU.  One CTA initialises an mbarrier for one arrival and
// waits on its first phase.  With `arrive` set, a thread arrives first and the
// wait returns at once; without it nothing ever arrives (no copy is issued, so
// none is in flight when the kernel returns), the wait runs out after
// `limit_ns`, the kernel raises PK_DEV_TIMEOUT and returns, and the context
// stays usable.
#include "pk_common.cuh"
#include "pk_internal.h"

namespace pk {
namespace {

__device__ __forceinline__ void arrive_once(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__global__ void selftest_wait_kernel(int32_t *error, int32_t arrive, uint64_t limit_ns,
                                     int64_t *waited_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (arrive) arrive_once(&bar);
    const uint64_t t0 = globaltimer_ns();
    const bool ok = mbar_wait_bounded(&bar, 0, limit_ns);
    *waited_ns = static_cast<int64_t>(globaltimer_ns() - t0);
    if (!ok) raise(error, PK_DEV_TIMEOUT);
}

}  // namespace

int launch_selftest_wait(int32_t *error, int32_t arrive, uint64_t limit_ns, int64_t *waited_ns,
                         cudaStream_t stream) {
    selftest_wait_kernel<<<1, 32, 0, stream>>>(error, arrive, limit_ns, waited_ns);
    return cuda_status(cudaGetLastError(), "selftest_wait_kernel");
}

}  // namespace pk
