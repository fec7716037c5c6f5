// selftest.cu -- exercises the bounded-wait path of the device-side pipelines.
//
// kc_selftest_bounded_wait launches one CTA that initializes an mbarrier and
// waits on a phase nothing will ever complete.  The wait gives up after the
// given time, records KC_ERR_TIMEOUT in the device status word and the kernel
// returns normally, leaving the context usable; kc_get_device_status() then
// reports the timeout.  No fault, trap or unbounded spin is involved.
#include "kc_common.cuh"
#include "sm100.cuh"

namespace {

__global__ void bounded_wait_kernel(uint64_t timeout_ns, int* waited_out) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = sm100::globaltimer();
        const bool ok = sm100::mbar_wait(&bar, 0, timeout_ns);  // nothing ever arrives
        const uint64_t dt = sm100::globaltimer() - t0;
        *waited_out = ok ? -1 : (int)(dt / 1000000ull);           // milliseconds waited
        sm100::mbar_arrive(&bar);  // complete the phase so the barrier is left idle
    }
}

}  // namespace

KC_DEFINE_STATUS_READER(selftest)

extern "C" {

int kc_selftest_bounded_wait(uint64_t timeout_ns, int* waited_ms_device, cudaStream_t stream) {
    KC_REQUIRE(waited_ms_device, KC_ERR_INVALID_ARG, "null output");
    KC_REQUIRE(timeout_ns > 0 && timeout_ns <= 5000000000ull, KC_ERR_INVALID_ARG,
               "timeout must be in (0, 5 s]");
    bounded_wait_kernel<<<1, 32, 0, stream>>>(timeout_ns, waited_ms_device);
    return kc::check_launch("bounded_wait_kernel");
}

}  // extern "C"
