// Self-test of the bounded device-wait path shared by the tensor-core and
// TMA kernels: one CTA waits on an mbarrier that nothing will complete, gives
// up after `limit_ns`, records MLKB_ERR_TIMEOUT in the device status word and
// returns normally, leaving the context usable. Nothing faults or hangs.
#include "common.cuh"
#include "tc_common.cuh"

namespace mlkb {
namespace {

__global__ void bounded_wait_kernel(uint64_t limit_ns, int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        abort = 0;
        tc::fence_barrier_init();
    }
    __syncthreads();
    // Phase 0 of a count-1 barrier that never receives an arrival.
    const bool ok = tc::mbar_wait(&bar, 0, &abort, limit_ns);
    if (__syncthreads_or(!ok) && threadIdx.x == 0 && status != nullptr) {
        atomicExch(status, MLKB_ERR_TIMEOUT);
    }
}

}  // namespace
}  // namespace mlkb

extern "C" int mlkb_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
    using namespace mlkb;
    if (limit_ns == 0 || limit_ns > 2000000000ull) {
        return setError(MLKB_ERR_INVALID, "selftest: limit must be in (0, 2 s]");
    }
    bounded_wait_kernel<<<1, 32, 0, asStream(stream)>>>(limit_ns, deviceStatusPtr());
    return checkLaunch("selftest launch");
}
