// gemm_fp8.cu -- FP8 E4M3 W8A8 GEMM on the 5th-generation tensor cores (sm_100a).
//
// C[m, n] = bf16( (sum_k e4m3(A[m, k]) * e4m3(W[n, k])) * sa[m] * sw[n] )
// A: per-token quantized activations (codes [M, K], scales sa[M]), W: per-output-
// channel quantized weights (codes [N, K], scales sw[N]), both K-major as the
// reference's quantizer writes them (src/kernels/transformer/fp8_quant.cu);
// fp32 accumulation in TMEM; bf16 output, or fp32 when requested.
//
// One persistent CTA per SM walks 128 x 256 output tiles.  Warp roles:
//   warp 0  TMA producer: 128 x 128-byte A and 256 x 128-byte W boxes per k-step
//           into a 4-stage ring (128-byte swizzle), completion on "full" mbarriers;
//   warp 1  allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and one
//           lane issues tcgen05.mma kind::f8f6f4 (M 128, N 256, K 32) four times
//           per stage, releasing the stage with tcgen05.commit on its "empty"
//           mbarrier and a finished accumulator on "tmem_full";
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time from the warp's 32 TMEM
//           lanes, scale by sa[m] * sw[n], convert, store; then free the
//           accumulator ("tmem_empty") so the MMA of tile i+2 can start while
//           tile i+1 accumulates.
// No TMA multicast is used (the kernel also runs inside multi-GPU jobs).
#include <algorithm>

#include "kc_common.cuh"
#include "sm100.cuh"
#include "tensor_map.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 128;   // BK in bytes = e4m3 elements
constexpr int kStages = 4;
constexpr int kABytes = BM * BK;              // 16 KB
constexpr int kBBytes = BN * BK;              // 32 KB
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr uint32_t kTmemCols = 512;

// Row-parallel sum fused into the epilogue (RS kernels): every rank computes
// the partial product of its K shard for all tiles; output rows are owned in R
// equal blocks.  A rank walks the owners' blocks starting after its own, so
// its own block comes last: a tile of another owner is written (bf16) into
// that owner's receive slot over NVLink and announced with a flag; a tile of
// its own waits for the R - 1 flags of that tile, adds the received partials
// to its fp32 accumulator and writes the bf16 sum into every rank's output.
// Per GPU that sends (R-1)/R of the output as partials and (R-1)/R as sums,
// both under the MMAs of the following tiles.
// Tiles travel as four 128-row x 64-column pieces (two TMEM chunks each),
// each staged in shared memory and written with one TMA store per
// destination: 128-byte rows over NVLink instead of per-thread 16-byte stores.
struct RsParams {
    CUtensorMap out_map[KC_MAX_RANKS];   // every rank's output bf16 {N, M}, box {64, 128}
    CUtensorMap recv_map[KC_MAX_RANKS];  // every rank's receive slots bf16 {N, (R-1) M/R}, box {64, 128}
    __nv_bfloat16* recv[KC_MAX_RANKS];   // every rank's receive slots: (R - 1) x [M / R, N] bf16
    int* flags[KC_MAX_RANKS];            // every rank's flags: (R - 1) x tiles per owner block
    int nranks, rank, epoch;
    uint64_t timeout_ns;
    // in-switch form (MC kernels): partials and sums in one symmetric buffer
    CUtensorMap part_map;                // this rank's copy bf16 {N, M}, box {64, 128}
    __nv_bfloat16* part;                 // this rank's copy [M, N]
    uint8_t* mc_part;                    // its multicast address
};

struct alignas(64) Params {
    CUtensorMap amap;   // A codes {K, M}, box {128, 128}, 128-byte swizzle
    CUtensorMap wmap;   // W codes {K, N}, box {128, 256}, 128-byte swizzle
    const float* sa;
    const float* sw;
    void* out;          // bf16 or fp32 [M, ldc]
    int M, N, K, ldc;
    int out_f32;
    int tiles_m, tiles_n;
    RsParams rs;
};

// Linear tile L -> its output tile (m0, n0); for RS also the owner and the
// tile's index within the owner's block.
template <bool RS>
__device__ __forceinline__ void tile_coords(const Params& P, int L, int& m0, int& n0, int& owner, int& j) {
    if constexpr (!RS) {
        m0 = (L % P.tiles_m) * BM;
        n0 = (L / P.tiles_m) * BN;
        owner = 0;
        j = L;
    } else {
        const int R = P.rs.nranks, tmo = P.tiles_m / R, per = tmo * P.tiles_n;
        const int b = L / per;
        j = L - b * per;
        owner = (P.rs.rank + 1 + b) % R;
        m0 = (owner * tmo + j % tmo) * BM;
        n0 = (j / tmo) * BN;
    }
}

struct Smem {
    uint8_t a[kStages][kABytes];   // 1024-byte aligned (swizzle atoms)
    uint8_t b[kStages][kBBytes];
    uint8_t stage[2][BM * 64 * 2]; // fused-sum epilogue: a 128 x 64 bf16 piece, double-buffered
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// MC (with RS): every rank writes its partial tile into its own copy of a
// symmetric buffer and flags the tile's owner; the owner writes its own
// partial there too, then sums the R copies in the NVSwitch
// (multimem.ld_reduce, fp32 accumulation) and stores the bf16 sum into every
// copy (multimem.st).  Per GPU that moves the output once out and
// (1 + 1/R) times in, against 2(R - 1)/R each way for the peer form.
template <bool RS, bool MC = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_fp8_kernel(const __grid_constant__ Params P) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles
    const uint32_t raw = sm100::smem_u32(smem_raw);
    Smem& S = *reinterpret_cast<Smem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = P.tiles_m * P.tiles_n;
    const int kblocks = (P.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            sm100::mbar_init(&S.full[i], 1);
            sm100::mbar_init(&S.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            sm100::mbar_init(&S.tmem_full[i], 1);
            sm100::mbar_init(&S.tmem_empty[i], kEpiWarps);
        }
        sm100::mbar_init(&S.drain, 1);
        S.abort = 0;
        sm100::fence_barrier_init();
    }
    if (warp == 1) {
        sm100::tmem_alloc(&S.tmem_base, kTmemCols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort = &S.abort;

    if (warp == 0) {
        // ------------------------------ TMA producer -----------------------------
        if (lane == 0) {
            sm100::prefetch_tensormap(&P.amap);
            sm100::prefetch_tensormap(&P.wmap);
            uint32_t it = 0;   // loads issued; nothing more is issued after a failed wait
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                int m0, n0, owner, j;
                tile_coords<RS>(P, tile, m0, n0, owner, j);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!(ok = sm100::mbar_wait_or_abort(&S.empty[s], ph ^ 1u, abort))) break;
                    sm100::mbar_arrive_expect_tx(&S.full[s], kABytes + kBBytes);
                    sm100::tma_load_2d(S.a[s], &P.amap, kb * BK, m0, &S.full[s]);
                    sm100::tma_load_2d(S.b[s], &P.wmap, kb * BK, n0, &S.full[s]);
                }
            }
            // drain: the last copies land before the CTA may exit (bounded)
            for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0u; j < it; ++j)
                sm100::mbar_wait(&S.full[j % kStages], (j / kStages) & 1u, 200000000ull);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            const uint32_t idesc = sm100::umma_idesc(sm100::kFmtE4M3, sm100::kFmtE4M3, BM, BN);
            uint32_t it = 0, t = 0;
            bool ok = true;   // false once a wait gave up: no MMA is issued after that
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t) {
                const uint32_t acc = t & 1u;
                ok = sm100::mbar_wait_or_abort(&S.tmem_empty[acc], ((t >> 1) & 1u) ^ 1u, abort) && ok;
                sm100::tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    ok = sm100::mbar_wait_or_abort(&S.full[s], ph, abort) && ok;
                    sm100::tc_fence_after();
                    if (ok) {   // a stage the TMA never filled is not multiplied
                        const uint64_t adesc = sm100::umma_desc_sw128(sm100::smem_u32(S.a[s]));
                        const uint64_t bdesc = sm100::umma_desc_sw128(sm100::smem_u32(S.b[s]));
#pragma unroll
                        for (int j = 0; j < BK / 32; ++j)  // K = 32 per instruction (32 bytes)
                            sm100::umma_f8f6f4_ss(d, adesc + 2 * j, bdesc + 2 * j, idesc,
                                                  (kb | j) != 0 ? 1u : 0u);
                    }
                    // committed either way, so the barriers keep completing and
                    // every role unwinds
                    sm100::tc_commit(&S.empty[s]);  // stage free once these MMAs retire
                }
                sm100::tc_commit(&S.tmem_full[acc]);  // accumulator complete
            }
            // drain: every MMA this thread issued retires before TMEM is freed
            sm100::tc_commit(&S.drain);
            sm100::mbar_wait(&S.drain, 0, 200000000ull);
        }
    } else {
        // -------------------------------- epilogue --------------------------------
        const int q = warp & 3;                      // TMEM lane quarter of this warp
        const int et = threadIdx.x - 64;             // 0..127 over the epilogue warps
        // RS: the flag of the last partial tile, raised once that tile's stores
        // have landed -- after the next tile's stores are issued, or before
        // this thread waits for peers, or at the end; it is never held while
        // this CTA waits for another rank, so no wait can close a cycle
        int* pend_flag = nullptr;
        auto raise_pending = [&]() {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __threadfence_system();
            asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(pend_flag), "r"(P.rs.epoch) : "memory");
            pend_flag = nullptr;
        };
        uint32_t t = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t) {
            const uint32_t acc = t & 1u;
            int m0, n0, owner, j;
            tile_coords<RS>(P, tile, m0, n0, owner, j);
            const int m = m0 + q * 32 + lane;
            const float sam = (m < P.M) ? __ldg(P.sa + m) : 0.f;
            const bool waited = sm100::mbar_wait_or_abort(&S.tmem_full[acc], (t >> 1) & 1u, abort);
            sm100::tc_fence_after();
            const bool mine = !RS || owner == P.rs.rank;
            bool peers_ok = true;
            if constexpr (RS) {
                // a tile of this rank's block: wait for every peer's partial of it
                // (bounded; a peer that never delivers makes the tile NaN)
                if (mine) {
                    if (et == 0) {
                        if (pend_flag) {   // nothing of ours is held while we wait
                            sm100::bulk_wait_group0();
                            raise_pending();
                        }
                        const int per = (P.tiles_m / P.rs.nranks) * P.tiles_n;
                        const uint64_t t0 = sm100::globaltimer();
                        for (int sl = 0; sl < P.rs.nranks - 1 && peers_ok; ++sl) {
                            const int* f = P.rs.flags[P.rs.rank] + sl * per + j;
                            while (true) {
                                int v;
                                asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                                if ((int)((unsigned)v - (unsigned)P.rs.epoch) >= 0) break;
                                if (*abort || sm100::globaltimer() - t0 > P.rs.timeout_ns) {
                                    sm100::record_status(KC_ERR_TIMEOUT);
                                    *abort = 1;
                                    peers_ok = false;
                                    break;
                                }
                            }
                        }
                    }
                    sm100::named_sync(1, 128);
                    peers_ok = !*abort;
                }
            }
            // after a wait gave up anywhere in the CTA the accumulator is not a
            // result: the tile is written as NaN, so a timeout cannot pass for
            // plausible output (kc_get_device_status reports it as well)
            const bool poison = !waited || *abort || !peers_ok;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, r);
                sm100::tmem_wait_ld();
                const int nb = n0 + c * 32;
                if (!RS && (m >= P.M || nb >= P.N)) continue;   // RS tiles are always whole
                const float4* swv = reinterpret_cast<const float4*>(P.sw + nb);
                float v[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 s4 = (nb + 4 * i + 3 < P.N) ? __ldg(swv + i)
                                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                    v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) * sam * s4.x;
                    v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) * sam * s4.y;
                    v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) * sam * s4.z;
                    v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) * sam * s4.w;
                }
                if constexpr (RS) {
                    const int R = P.rs.nranks, rows = P.M / R;
                    if constexpr (MC) {
                        if (mine) {
                            // the owner's partial into its own copy; the switch sums
                            // the copies once the tile is complete (below)
                            if (poison)
#pragma unroll
                                for (int i = 0; i < 32; ++i) v[i] = __int_as_float(0x7FC00000);
                            uint4* o = reinterpret_cast<uint4*>(P.rs.part + (size_t)m * P.N + nb);
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                o[i] = make_uint4(bf16x2_bits(v[8 * i], v[8 * i + 1]), bf16x2_bits(v[8 * i + 2], v[8 * i + 3]),
                                                  bf16x2_bits(v[8 * i + 4], v[8 * i + 5]),
                                                  bf16x2_bits(v[8 * i + 6], v[8 * i + 7]));
                            continue;
                        }
                    } else if (mine) {
                        // the owner: add the peers' partials (slots in order)
                        for (int sl = 0; sl < R - 1; ++sl) {
                            const uint4* in = reinterpret_cast<const uint4*>(
                                P.rs.recv[P.rs.rank] + ((size_t)sl * rows + (m - P.rs.rank * rows)) * P.N + nb);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint4 w = __ldcg(in + i);
                                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    v[8 * i + 2 * e] += __uint_as_float(ww[e] << 16);
                                    v[8 * i + 2 * e + 1] += __uint_as_float(ww[e] & 0xFFFF0000u);
                                }
                            }
                        }
                    }
                    if (poison)
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __int_as_float(0x7FC00000);
                    // stage the chunk (the tile's row q * 32 + lane, this thread's
                    // TMEM lane: 64 bytes), then one TMA store per
                    // destination: the owner's receive slot for a partial, every
                    // rank's output for a sum
                    // chunks 2p and 2p + 1 fill the halves of buffer p & 1
                    const int buf = (c >> 1) & 1, half = c & 1;
                    if (half == 0) {
                        if (et == 0) sm100::bulk_wait_group_read1();   // this buffer's last stores read it
                        sm100::named_sync(1, 128);
                    }
                    uint4* st4 = reinterpret_cast<uint4*>(S.stage[buf] + (q * 32 + lane) * 128 + half * 64);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        st4[i] = make_uint4(bf16x2_bits(v[8 * i], v[8 * i + 1]), bf16x2_bits(v[8 * i + 2], v[8 * i + 3]),
                                            bf16x2_bits(v[8 * i + 4], v[8 * i + 5]),
                                            bf16x2_bits(v[8 * i + 6], v[8 * i + 7]));
                    if (half == 1) {
                        sm100::fence_proxy_async_smem();
                        sm100::named_sync(1, 128);
                        if (et == 0) {
                            const int x = nb - 32;
                            if (MC) {   // a partial, into this rank's own copy
                                sm100::tma_store_2d(&P.rs.part_map, S.stage[buf], x, m0);
                            } else if (!mine) {
                                const int sl = (P.rs.rank - owner - 1 + R) % R;
                                sm100::tma_store_2d(&P.rs.recv_map[owner], S.stage[buf], x, sl * rows + (m0 - owner * rows));
                            } else {
                                for (int d = 0; d < R; ++d)   // own copy first
                                    sm100::tma_store_2d(&P.rs.out_map[(P.rs.rank + d) % R], S.stage[buf], x, m0);
                            }
                            sm100::bulk_commit_group();
                        }
                    }
                    continue;
                }
                if (poison)
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __int_as_float(0x7FC00000);
                if (P.out_f32) {
                    float* o = reinterpret_cast<float*>(P.out) + (size_t)m * P.ldc + nb;
                    if (nb + 32 <= P.N) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            reinterpret_cast<float4*>(o)[i] =
                                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    } else {
                        for (int i = 0; i < 32 && nb + i < P.N; ++i) o[i] = v[i];
                    }
                } else {
                    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(P.out) + (size_t)m * P.ldc + nb;
                    if (nb + 32 <= P.N) {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            reinterpret_cast<uint4*>(o)[i] =
                                make_uint4(bf16x2_bits(v[8 * i], v[8 * i + 1]),
                                           bf16x2_bits(v[8 * i + 2], v[8 * i + 3]),
                                           bf16x2_bits(v[8 * i + 4], v[8 * i + 5]),
                                           bf16x2_bits(v[8 * i + 6], v[8 * i + 7]));
                    } else {
                        for (int i = 0; i < 32 && nb + i < P.N; ++i) o[i] = __float2bfloat16_rn(v[i]);
                    }
                }
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&S.tmem_empty[acc]);
            if constexpr (MC) {
                if (mine) {
                    // every copy of the tile is complete: the switch sums them and
                    // writes the sum into every copy (128 rows x 32 pieces of 16 B)
                    __threadfence_system();
                    sm100::named_sync(1, 128);
                    uint8_t* base = P.rs.mc_part + ((size_t)m0 * P.N + n0) * 2;
#pragma unroll 8
                    for (int i = et; i < BM * (BN / 8); i += 128) {
                        uint8_t* a = base + (size_t)(i >> 5) * P.N * 2 + (i & 31) * 16;
                        uint32_t w0, w1, w2, w3;
                        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                                     : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                                     : "l"(a)
                                     : "memory");
                        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};"
                                     ::"l"(a), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                                     : "memory");
                    }
                }
            }
            if constexpr (RS) {
                if (et == 0) {
                    // the previous partial tile's flag: its groups are all but this
                    // tile's BN / 64 newest
                    if (pend_flag) {
                        sm100::bulk_wait_group<BN / 64>();
                        raise_pending();
                    }
                    if (!mine) {
                        const int R = P.rs.nranks, per = (P.tiles_m / R) * P.tiles_n;
                        const int sl = (P.rs.rank - owner - 1 + R) % R;
                        pend_flag = P.rs.flags[owner] + sl * per + j;
                    }
                }
            }
        }
        if constexpr (RS) {   // the sums and the last flag, before the barrier after the kernel
            if (et == 0) {
                sm100::bulk_wait_group0();
                if (pend_flag) raise_pending();
                asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            __threadfence_system();
        }
    }

    // teardown: every MMA has been consumed by the epilogue before this barrier
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

KC_DEFINE_STATUS_READER(gemm_fp8)

extern "C" {

int kc_gemm_fp8_ctas(const int8_t* a_codes, const float* sa, const int8_t* w_codes, const float* sw,
                     void* out, int out_f32, int M, int N, int K, int ldc, int max_ctas,
                     cudaStream_t stream) {
    KC_REQUIRE(a_codes && sa && w_codes && sw && out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(M >= 0 && N >= 0 && K >= 0, KC_ERR_INVALID_ARG, "negative size");
    if (M == 0 || N == 0) return KC_OK;
    KC_REQUIRE(K > 0 && K % 16 == 0, KC_ERR_INVALID_ARG, "K=%d must be a positive multiple of 16", K);
    KC_REQUIRE(N % 8 == 0 && ldc >= N && ldc % 8 == 0, KC_ERR_INVALID_ARG,
               "N=%d and ldc=%d must be multiples of 8 with ldc >= N", N, ldc);
    KC_REQUIRE(kc::aligned(a_codes, 16) && kc::aligned(w_codes, 16) && kc::aligned(out, 16) &&
                   kc::aligned(sw, 16),
               KC_ERR_ALIGNMENT, "operands must be 16-byte aligned");
    Params P{};
    int st = kc::encode_2d(&P.amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_codes, (uint64_t)K, (uint64_t)M,
                           (uint64_t)K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = kc::encode_2d(&P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, (uint64_t)K, (uint64_t)N,
                       (uint64_t)K, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    P.sa = sa;
    P.sw = sw;
    P.out = out;
    P.M = M;
    P.N = N;
    P.K = K;
    P.ldc = ldc;
    P.out_f32 = out_f32 ? 1 : 0;
    P.tiles_m = (M + BM - 1) / BM;
    P.tiles_n = (N + BN - 1) / BN;
    const size_t smem = sizeof(Smem) + 1024;
    KC_CUDA_TRY(cudaFuncSetAttribute(gemm_fp8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "gemm_fp8 shared-memory attribute");
    const int tiles = P.tiles_m * P.tiles_n;
    const int ctas = max_ctas > 0 ? std::min(max_ctas, kc::sm_count()) : kc::sm_count();
    const int grid = std::min(tiles, ctas);
    gemm_fp8_kernel<false><<<grid, kThreads, smem, stream>>>(P);
    return kc::check_launch("gemm_fp8");
}

int kc_gemm_fp8_allreduce(const int8_t* a_codes_shard, const float* sa, const int8_t* w_codes_shard,
                          const float* sw, void* const* outs, void* const* recvs, int* const* flags,
                          int nranks, int rank, int epoch, int M, int N, int K_shard, uint64_t timeout_ns,
                          cudaStream_t stream) {
    KC_REQUIRE(a_codes_shard && sa && w_codes_shard && sw && outs && recvs && flags, KC_ERR_INVALID_ARG,
               "null pointer argument");
    KC_REQUIRE(nranks >= 2 && nranks <= KC_MAX_RANKS && rank >= 0 && rank < nranks, KC_ERR_INVALID_ARG,
               "rank %d of %d: 2..%d ranks", rank, nranks, KC_MAX_RANKS);
    KC_REQUIRE(M > 0 && M % (BM * nranks) == 0, KC_ERR_INVALID_ARG,
               "M=%d must be a positive multiple of %d x nranks", M, BM);
    KC_REQUIRE(N > 0 && N % BN == 0, KC_ERR_INVALID_ARG, "N=%d must be a positive multiple of %d", N, BN);
    KC_REQUIRE(K_shard > 0 && K_shard % 16 == 0, KC_ERR_INVALID_ARG,
               "K_shard=%d must be a positive multiple of 16", K_shard);
    KC_REQUIRE(timeout_ns <= KC_PEER_BARRIER_MAX_TIMEOUT_NS, KC_ERR_INVALID_ARG, "timeout above the maximum");
    KC_REQUIRE(kc::aligned(a_codes_shard, 16) && kc::aligned(w_codes_shard, 16) && kc::aligned(sw, 16),
               KC_ERR_ALIGNMENT, "operands must be 16-byte aligned");
    Params P{};
    for (int r = 0; r < nranks; ++r) {
        KC_REQUIRE(outs[r] && recvs[r] && flags[r] && kc::aligned(outs[r], 16) && kc::aligned(recvs[r], 16) &&
                       kc::aligned(flags[r], 4),
                   KC_ERR_ALIGNMENT, "buffers of rank %d null or misaligned", r);
        P.rs.recv[r] = static_cast<__nv_bfloat16*>(recvs[r]);
        P.rs.flags[r] = flags[r];
        int e = kc::encode_2d(&P.rs.out_map[r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, outs[r], (uint64_t)N,
                              (uint64_t)M, (uint64_t)N * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (e) return e;
        e = kc::encode_2d(&P.rs.recv_map[r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, recvs[r], (uint64_t)N,
                          (uint64_t)(nranks - 1) * (M / nranks), (uint64_t)N * 2, 64, BM,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
        if (e) return e;
    }
    P.rs.nranks = nranks;
    P.rs.rank = rank;
    P.rs.epoch = epoch;
    P.rs.timeout_ns = timeout_ns ? timeout_ns : KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS;
    int st = kc::encode_2d(&P.amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_codes_shard, (uint64_t)K_shard, (uint64_t)M,
                           (uint64_t)K_shard, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = kc::encode_2d(&P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes_shard, (uint64_t)K_shard, (uint64_t)N,
                       (uint64_t)K_shard, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    P.sa = sa;
    P.sw = sw;
    P.out = outs[rank];
    P.M = M;
    P.N = N;
    P.K = K_shard;
    P.ldc = N;
    P.out_f32 = 0;
    P.tiles_m = M / BM;
    P.tiles_n = N / BN;
    const size_t smem = sizeof(Smem) + 1024;
    KC_CUDA_TRY(cudaFuncSetAttribute(gemm_fp8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "gemm_fp8 shared-memory attribute");
    const int tiles = P.tiles_m * P.tiles_n;
    gemm_fp8_kernel<true><<<std::min(tiles, kc::sm_count()), kThreads, smem, stream>>>(P);
    return kc::check_launch("gemm_fp8_allreduce");
}

int kc_gemm_fp8(const int8_t* a_codes, const float* sa, const int8_t* w_codes, const float* sw,
                void* out, int out_f32, int M, int N, int K, int ldc, cudaStream_t stream) {
    return kc_gemm_fp8_ctas(a_codes, sa, w_codes, sw, out, out_f32, M, N, K, ldc, 0, stream);
}

int kc_gemm_fp8_allreduce_mc(const int8_t* a_codes_shard, const float* sa, const int8_t* w_codes_shard,
                             const float* sw, void* part, void* mc_part, int* const* flags, int nranks,
                             int rank, int epoch, int M, int N, int K_shard, uint64_t timeout_ns,
                             cudaStream_t stream) {
    KC_REQUIRE(a_codes_shard && sa && w_codes_shard && sw && part && mc_part && flags, KC_ERR_INVALID_ARG,
               "null pointer argument");
    KC_REQUIRE(nranks >= 2 && nranks <= KC_MAX_RANKS && rank >= 0 && rank < nranks, KC_ERR_INVALID_ARG,
               "rank %d of %d: 2..%d ranks", rank, nranks, KC_MAX_RANKS);
    KC_REQUIRE(M > 0 && M % (BM * nranks) == 0, KC_ERR_INVALID_ARG,
               "M=%d must be a positive multiple of %d x nranks", M, BM);
    KC_REQUIRE(N > 0 && N % BN == 0, KC_ERR_INVALID_ARG, "N=%d must be a positive multiple of %d", N, BN);
    KC_REQUIRE(K_shard > 0 && K_shard % 16 == 0, KC_ERR_INVALID_ARG,
               "K_shard=%d must be a positive multiple of 16", K_shard);
    KC_REQUIRE(timeout_ns <= KC_PEER_BARRIER_MAX_TIMEOUT_NS, KC_ERR_INVALID_ARG, "timeout above the maximum");
    KC_REQUIRE(kc::aligned(a_codes_shard, 16) && kc::aligned(w_codes_shard, 16) && kc::aligned(sw, 16) &&
                   kc::aligned(part, 16) && kc::aligned(mc_part, 16),
               KC_ERR_ALIGNMENT, "operands must be 16-byte aligned");
    Params P{};
    for (int r = 0; r < nranks; ++r) {
        KC_REQUIRE(flags[r] && kc::aligned(flags[r], 4), KC_ERR_ALIGNMENT, "flags of rank %d null or misaligned", r);
        P.rs.flags[r] = flags[r];
    }
    P.rs.nranks = nranks;
    P.rs.rank = rank;
    P.rs.epoch = epoch;
    P.rs.timeout_ns = timeout_ns ? timeout_ns : KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS;
    P.rs.part = static_cast<__nv_bfloat16*>(part);
    P.rs.mc_part = static_cast<uint8_t*>(mc_part);
    int st = kc::encode_2d(&P.rs.part_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, part, (uint64_t)N, (uint64_t)M,
                           (uint64_t)N * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = kc::encode_2d(&P.amap, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_codes_shard, (uint64_t)K_shard, (uint64_t)M,
                       (uint64_t)K_shard, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = kc::encode_2d(&P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes_shard, (uint64_t)K_shard, (uint64_t)N,
                       (uint64_t)K_shard, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    P.sa = sa;
    P.sw = sw;
    P.out = part;
    P.M = M;
    P.N = N;
    P.K = K_shard;
    P.ldc = N;
    P.out_f32 = 0;
    P.tiles_m = M / BM;
    P.tiles_n = N / BN;
    const size_t smem = sizeof(Smem) + 1024;
    KC_CUDA_TRY(cudaFuncSetAttribute(gemm_fp8_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "gemm_fp8 shared-memory attribute");
    const int tiles = P.tiles_m * P.tiles_n;
    gemm_fp8_kernel<true, true><<<std::min(tiles, kc::sm_count()), kThreads, smem, stream>>>(P);
    return kc::check_launch("gemm_fp8_allreduce_mc");
}

}  // extern "C"
