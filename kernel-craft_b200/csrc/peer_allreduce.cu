// peer_allreduce.cu -- bf16 sum all-reduce over NVLink peer memory, one
// process per GPU, for the row-parallel FP8 GEMM's partial outputs.
//
// Two-shot in one pass: rank r owns the r-th 1/R slice of the flat array.  Its
// threads load the slice from all R partial buffers (its own and R-1 peers',
// mapped with kc_ipc_open), add them in fp32 in rank order 0..R-1 (so every
// element is reduced once, by one rank, the same way on every run), round once
// to bf16 and store the result into all R output buffers.  Per GPU that moves
// (R-1)/R of the array in over NVLink and (R-1)/R out, concurrently -- the
// traffic of a reduce-scatter followed by an all-gather, without the ring's
// R-1 dependent steps or the intermediate bf16 roundings.
//
// The reduction kernel neither waits for its peers nor signals them: the
// caller orders "every rank's partial is complete" before the launch and
// "every rank's stores are complete" after it, with kc_peer_barrier (a
// one-warp flag exchange over the same peer mappings, bounded by a timeout)
// or a collective on the same stream.
//
// A barrier that gives up has not ordered anything, so what follows it reads
// or overwrites buffers a peer may still use.  It then records
// KC_ERR_TIMEOUT in this unit's status word (and in the caller's host-visible
// status slot, if one was given), and from then on every reduction of this
// process writes NaN instead of sums, until kc_get_device_status() reads and
// clears the word: a timeout cannot pass for a plausible result.
#include <algorithm>

#include "kc_common.cuh"

namespace {

__device__ int g_peer_status;   // KC_ERR_TIMEOUT when a peer barrier gave up

struct PeerPtrs {
    const uint4* in[KC_MAX_RANKS];
    uint4* out[KC_MAX_RANKS];
};

__device__ __forceinline__ void add8(float (&acc)[8], const uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(w[i] << 16);
        acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Vectors [begin, end) of 8 bf16; U vectors per thread per round so the
// 2*U*R loads of a round are in flight together.
template <int R>
__global__ void __launch_bounds__(256) peer_allreduce_bf16_kernel(const __grid_constant__ PeerPtrs p,
                                                                  long begin, long end) {
    constexpr int U = 2;
    const bool poison = *reinterpret_cast<volatile int*>(&g_peer_status) != 0;
    const long stride = (long)gridDim.x * blockDim.x * U;
    for (long base = begin + ((long)blockIdx.x * blockDim.x + threadIdx.x) * U; base < end;
         base += stride) {
        float acc[U][8];
        uint4 v[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < R; ++r)
                v[u][r] = (base + u < end) ? __ldcg(p.in[r] + base + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
#pragma unroll
            for (int r = 0; r < R; ++r) add8(acc[u], v[u][r]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (base + u >= end) break;
            const uint4 o = poison ? make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u)
                                   : make_uint4(bf16x2_rn(acc[u][0], acc[u][1]), bf16x2_rn(acc[u][2], acc[u][3]),
                                                bf16x2_rn(acc[u][4], acc[u][5]), bf16x2_rn(acc[u][6], acc[u][7]));
#pragma unroll
            for (int r = 0; r < R; ++r) __stcg(p.out[r] + base + u, o);
        }
    }
}

// NVLink SHARP form: `mc` is the multicast address of a buffer bound on every
// rank (one physical copy per GPU).  Vectors [begin, end) of 8 bf16 -- this
// rank's slice -- are read through the switch, which sums the R copies
// (multimem.ld_reduce, fp32 accumulation), and the sum is written back
// through the switch into every rank's copy (multimem.st).  Per GPU the
// switch reads (R-1)/R of the array and writes (R-1)/R of it, once each: the
// traffic of a single pass, against 2(R-1)/R for the peer form.  Only the
// reducing rank touches its slice, so the sum can be in place.
__global__ void __launch_bounds__(256) nvls_allreduce_bf16_kernel(uint4* mc, long begin, long end) {
    constexpr int U = 4;
    const bool poison = *reinterpret_cast<volatile int*>(&g_peer_status) != 0;
    const long stride = (long)gridDim.x * blockDim.x * U;
    for (long base = begin + (long)blockIdx.x * blockDim.x * U + threadIdx.x; base < end; base += stride) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long i = base + (long)u * blockDim.x;
            if (i < end)
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                             : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                             : "l"(mc + i)
                             : "memory");
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long i = base + (long)u * blockDim.x;
            if (i >= end) break;
            const uint4 o = poison ? make_uint4(0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u, 0x7FC07FC0u) : v[u];
            asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};"
                         ::"l"(mc + i), "r"(o.x), "r"(o.y), "r"(o.z), "r"(o.w)
                         : "memory");
        }
    }
    __threadfence_system();   // the stores before the barrier that follows the kernel
}

template <int R>
void launch_r(const PeerPtrs& p, long begin, long end, cudaStream_t stream) {
    const long vecs = end - begin;
    const long want = (vecs + 2 * 256 - 1) / (2 * 256);
    const int grid = (int)std::max(1L, std::min(want, (long)kc::sm_count() * 8));
    peer_allreduce_bf16_kernel<R><<<grid, 256, 0, stream>>>(p, begin, end);
}

// One warp: lane r publishes this rank's epoch into rank r's flag slot
// `rank` (release, system scope), then waits until every rank's epoch in
// this rank's own slots has reached `epoch` (acquire), at most timeout_ns.
// Every rank launches it on its own GPU, so the wait ends as soon as the
// slowest rank has arrived; no kernel on one GPU waits for another kernel on
// the same GPU.  Epochs are compared modulo 2^32 (as the difference of the
// unsigned values read as a signed number), so they may wrap.
__global__ void peer_barrier_kernel(const __grid_constant__ PeerPtrs p, int nranks, int rank,
                                    int epoch, uint64_t timeout_ns, int* status_slot) {
    const int lane = threadIdx.x;
    if (lane < nranks) {
        int* slot = reinterpret_cast<int*>(p.out[lane]) + rank;
        __threadfence_system();
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
        const int* mine = reinterpret_cast<const int*>(p.in[rank]) + lane;
        uint64_t t0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        while (true) {
            int v;
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int)((unsigned)v - (unsigned)epoch) >= 0) break;
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > timeout_ns) {
                atomicCAS(&g_peer_status, 0, KC_ERR_TIMEOUT);
                if (status_slot != nullptr) {
                    *reinterpret_cast<volatile int*>(status_slot) = KC_ERR_TIMEOUT;
                    __threadfence_system();
                }
                break;
            }
        }
    }
}

}  // namespace

namespace kc {
int read_device_status_peer(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_peer_status, sizeof(int)) != cudaSuccess) return KC_ERR_CUDA;
    if (clear && v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(int));
    }
    return v;
}
}  // namespace kc

extern "C" {

int kc_peer_barrier(int* const* flags, int nranks, int rank, int epoch, uint64_t timeout_ns,
                    int* status_host, cudaStream_t stream) {
    KC_REQUIRE(flags && nranks >= 1 && nranks <= KC_MAX_RANKS && rank >= 0 && rank < nranks,
               KC_ERR_INVALID_ARG, "rank %d of %d outside 0..%d", rank, nranks, KC_MAX_RANKS - 1);
    KC_REQUIRE(timeout_ns <= KC_PEER_BARRIER_MAX_TIMEOUT_NS, KC_ERR_INVALID_ARG,
               "timeout %llu ns above the maximum of %llu ns", (unsigned long long)timeout_ns,
               (unsigned long long)KC_PEER_BARRIER_MAX_TIMEOUT_NS);
    if (timeout_ns == 0) timeout_ns = KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS;
    int* status_dev = nullptr;
    if (status_host != nullptr) {
        // pinned host memory: the address the device writes through
        KC_REQUIRE(kc::aligned(status_host, 4), KC_ERR_ALIGNMENT, "status slot not 4-byte aligned");
        void* d = nullptr;
        const cudaError_t e = cudaHostGetDevicePointer(&d, status_host, 0);
        if (e != cudaSuccess) {
            cudaGetLastError();  // not sticky: keep it from surfacing at a later launch check
            return kc::set_error(KC_ERR_INVALID_ARG,
                                 "status slot must be pinned, mapped host memory (%s)",
                                 cudaGetErrorString(e));
        }
        status_dev = static_cast<int*>(d);
    }
    PeerPtrs p{};
    for (int r = 0; r < nranks; ++r) {
        KC_REQUIRE(flags[r] && kc::aligned(flags[r], 4), KC_ERR_ALIGNMENT,
                   "flag array of rank %d is null or misaligned", r);
        p.in[r] = reinterpret_cast<const uint4*>(flags[r]);
        p.out[r] = reinterpret_cast<uint4*>(flags[r]);
    }
    peer_barrier_kernel<<<1, 32, 0, stream>>>(p, nranks, rank, epoch, timeout_ns, status_dev);
    return kc::check_launch("peer_barrier");
}

int kc_allreduce_bf16_peer(const void* const* partials, void* const* outs, int nranks, int rank,
                           long count, cudaStream_t stream) {
    KC_REQUIRE(partials && outs && nranks >= 1 && nranks <= KC_MAX_RANKS && rank >= 0 &&
                   rank < nranks,
               KC_ERR_INVALID_ARG, "rank %d of %d outside 0..%d", rank, nranks, KC_MAX_RANKS - 1);
    KC_REQUIRE(count >= 0 && count % (8L * nranks) == 0, KC_ERR_INVALID_ARG,
               "count=%ld must be a multiple of 8 * nranks", count);
    if (count == 0) return KC_OK;
    PeerPtrs p{};
    for (int r = 0; r < nranks; ++r) {
        KC_REQUIRE(partials[r] && outs[r] && kc::aligned(partials[r], 16) && kc::aligned(outs[r], 16),
                   KC_ERR_ALIGNMENT, "buffer of rank %d is null or not 16-byte aligned", r);
        p.in[r] = static_cast<const uint4*>(partials[r]);
        p.out[r] = static_cast<uint4*>(outs[r]);
    }
    const long vecs = count / 8, slice = vecs / nranks;
    const long begin = slice * rank, end = begin + slice;
    switch (nranks) {
        case 1: launch_r<1>(p, begin, end, stream); break;
        case 2: launch_r<2>(p, begin, end, stream); break;
        case 3: launch_r<3>(p, begin, end, stream); break;
        case 4: launch_r<4>(p, begin, end, stream); break;
        case 5: launch_r<5>(p, begin, end, stream); break;
        case 6: launch_r<6>(p, begin, end, stream); break;
        case 7: launch_r<7>(p, begin, end, stream); break;
        default: launch_r<8>(p, begin, end, stream); break;
    }
    return kc::check_launch("peer_allreduce_bf16");
}

int kc_allreduce_bf16_nvls(void* mc, int nranks, int rank, long count, int max_ctas,
                           cudaStream_t stream) {
    KC_REQUIRE(mc && nranks >= 1 && nranks <= KC_MAX_RANKS && rank >= 0 && rank < nranks,
               KC_ERR_INVALID_ARG, "rank %d of %d outside 0..%d", rank, nranks, KC_MAX_RANKS - 1);
    KC_REQUIRE(kc::aligned(mc, 16), KC_ERR_ALIGNMENT, "multicast address not 16-byte aligned");
    KC_REQUIRE(count >= 0 && count % (8L * nranks) == 0, KC_ERR_INVALID_ARG,
               "count=%ld must be a multiple of 8 * nranks", count);
    KC_REQUIRE(max_ctas >= 0, KC_ERR_INVALID_ARG, "max_ctas=%d", max_ctas);
    if (count == 0) return KC_OK;
    const long slice = count / 8 / nranks;
    const long begin = slice * rank, end = begin + slice;
    long grid = (slice + 4 * 256 - 1) / (4 * 256);
    grid = std::min(grid, (long)kc::sm_count() * 4);
    if (max_ctas > 0) grid = std::min(grid, (long)max_ctas);
    nvls_allreduce_bf16_kernel<<<(unsigned)std::max(1L, grid), 256, 0, stream>>>(static_cast<uint4*>(mc),
                                                                                 begin, end);
    return kc::check_launch("nvls_allreduce_bf16");
}

}  // extern "C"
