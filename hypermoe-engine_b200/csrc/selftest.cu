// selftest.cu -- exercises the bounded device-side wait that every kernel
// of this library uses for its mbarrier spins (sm100::mbar_wait_for): a
// wait on a barrier that nothing arrives on must give up after its limit,
// record HMOE_TIMEOUT in the workspace status word and let the kernel
// return, leaving the context usable.
#include "common.cuh"
#include "sm100.cuh"

namespace hmoe {
namespace {

__global__ void bounded_wait_kernel(DeviceStatus* st, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_mbarrier_init();
    }
    __syncthreads();
    // Nothing arrives on `bar`: phase 0 never completes.
    if (!sm100::mbar_wait_for(&bar, 0, limit_ns)) {
        if (threadIdx.x == 0) device_fail(st, HMOE_TIMEOUT);
    }
}

} // namespace
} // namespace hmoe

extern "C" hmoe_status hmoe_selftest_bounded_wait(void* workspace, uint32_t limit_us, void* stream) {
    using namespace hmoe;
    if (!workspace || limit_us == 0 || limit_us > 1000000) return HMOE_INVALID_ARGUMENT;
    bounded_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(static_cast<DeviceStatus*>(workspace),
                                                        static_cast<uint64_t>(limit_us) * 1000ull);
    return check_launch("hmoe bounded-wait self-test");
}
