// selftest.cu -- exercises the bounded-wait path of the device-side pipelines,
// and a streaming-read floor for the small memory-bound launches.
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

// One pass of streaming 16-byte loads, four in flight per thread, laid out
// like gemv_int4_f32_vec's weight reads (256-thread CTAs; the CTA's threads
// cover consecutive 16-byte words, u = 0..3 strides of one CTA span apart).
__global__ void __launch_bounds__(256) stream_read_kernel(const uint4* __restrict__ src, size_t n16,
                                                          uint32_t sentinel, uint32_t* sink) {
    const size_t base = (size_t)blockIdx.x * 1024 + threadIdx.x;
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const size_t i = base + 256 * u;
        v[u] = i < n16 ? kc_ldg_stream(src + i) : make_uint4(0, 0, 0, 0);
    }
    uint32_t h = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) h ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    if (h == sentinel) *sink = h;
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

int kc_selftest_stream_read(const void* src, size_t bytes, uint32_t sentinel, uint32_t* sink_device,
                            cudaStream_t stream) {
    KC_REQUIRE(sink_device, KC_ERR_INVALID_ARG, "null sink");
    KC_REQUIRE(bytes == 0 || src, KC_ERR_INVALID_ARG, "null source");
    KC_REQUIRE(bytes % 16 == 0 && kc::aligned(src, 16), KC_ERR_ALIGNMENT,
               "source must be 16-byte aligned and a multiple of 16 bytes");
    const size_t n16 = bytes / 16;
    const size_t ctas = n16 == 0 ? 1 : (n16 + 1023) / 1024;
    KC_REQUIRE(ctas < (1ull << 31), KC_ERR_INVALID_ARG, "too many bytes");
    stream_read_kernel<<<(unsigned)ctas, 256, 0, stream>>>(static_cast<const uint4*>(src), n16, sentinel,
                                                           sink_device);
    return kc::check_launch("stream_read_kernel");
}

}  // extern "C"
