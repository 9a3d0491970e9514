// Diagnostic of the device-side failure path shared by every kernel here.
//
// Every mbarrier wait in the library is bounded (mbar_wait: kWaitNs of
// %globaltimer); a wait that runs out raises LI_ERR_TIMEOUT on the
// translation unit's device flag, the kernel skips its remaining work,
// drains its copies and returns, and li_device_status() reports the flag.
// li_selftest_bounded_wait makes that happen on purpose, with nothing at
// fault: one CTA initialises an mbarrier that nothing will complete (one
// expected arrival that never comes) and waits on its first phase with the
// same wait, cut short to the caller's limit. The GPU stays usable: the
// kernel ends by itself once the limit has passed.
#include "li_common.cuh"

LI_DEFINE_TU_STATUS(selftest)

namespace li {
namespace {

__global__ void __launch_bounds__(32) bounded_wait_kernel(unsigned long long limit_ns, unsigned long long *elapsed_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        const unsigned long long t0 = global_ns();
        const bool done = mbar_wait_for(&bar, 0u, limit_ns);   // phase 0 never completes
        if (elapsed_ns) *elapsed_ns = done ? 0ull : global_ns() - t0;
    }
}

}  // namespace
}  // namespace li

extern "C" int li_selftest_bounded_wait(int limit_us, unsigned long long *elapsed_ns, void *stream) {
    if (limit_us < 1 || limit_us > 1000000) return LI_ERR_BAD_ARG;
    li::bounded_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(1000ull * (unsigned long long)limit_us, elapsed_ns);
    return li::launch_status();
}
