// gemm_w4a16.cu -- W4A16 GEMM (prefill) on the 5th-generation tensor cores (sm_100a).
//
// C[m, n] = sum_k x[m, k] * w[n, k],  w[n, k] = bf16_rne((u - 8) * s[n, k / gs])
// x bf16 [M, K] (K-major), packed u8 [N, K/2] (low nibble = even k), fp16 scales
// [N, K/gs], fp32 accumulation, bf16 (or fp32) C [M, N].  The dequantized weights
// are exactly the ones kc_dequantize_w4_bf16 produces (the reference dequant of
// packed ^ 0x88 with zero points 0, quant_int4.cu:99-104, rounded to bf16).
//
// The weights are the MMA's A operand and live in TMEM, the activations are the
// B operand in shared memory, so the accumulator holds C^T tiles
// (128 weight rows x 256 tokens):
//  * warp 0, TMA producer: per 64-k step a 256-token x 128-byte activation box
//    (128-byte swizzle, K-major) and a 128-row x 32-byte packed-weight box, into
//    a 4-stage ring;
//  * warps 2-9, converters, two per TMEM lane quarter taking alternate steps:
//    thread i of a quarter owns weight row i (= TMEM lane i); it turns its 64
//    nibbles into bf16 (u - 8) * s with one exact fma and one RNE and writes
//    them with tcgen05.st as 32 TMEM columns of a 4-stage A ring.  Two warps
//    per quarter overlap one warp's TMEM-store wait with the other's ALU work;
//  * warp 1: allocates TMEM (256 accumulator + 4 x 32 A columns) and one lane
//    issues tcgen05.mma kind::f16 (A from TMEM, B from shared memory; M 128,
//    N 256, K 16) four times per step, committing to the stage barriers;
//  * warps 10-13, epilogue: drain the accumulator with tcgen05.ld, release it to
//    the MMA as soon as the last load returns, convert to bf16 into a
//    shared-memory tile and write it with a TMA store that runs under the next
//    tile's main loop (fp32 output, or a pitch the TMA cannot address, falls
//    back to direct coalesced stores).  An optional activation (the
//    sigmoid-approximated GELU of the reference's MLP block) is applied to the
//    fp32 accumulator before the conversion.
// TMEM holds one accumulator only (256 + 128 A columns of 512), so the early
// release keeps the MMA idle per tile to the drain time.  Staging bf16 weights
// in shared memory instead would need ~160 B/clk of shared-memory bandwidth per
// SM at full MMA rate (above the ~128 B/clk available); this layout needs
// ~100.  No TMA multicast is used.
#include <algorithm>

#include "kc_common.cuh"
#include "sm100.cuh"
#include "tensor_map.cuh"

namespace {

constexpr int BW = 128;      // weight rows per tile (MMA M)
constexpr int BT = 256;      // tokens per tile (MMA N)
constexpr int BK = 64;       // k per stage
constexpr int kStages = 4;
constexpr int kXBytes = BT * BK * 2;      // 32 KB activations per stage
constexpr int kWBytes = BW * BK / 2;      // 4 KB packed weights per stage
constexpr int kConvWarps = 8;
constexpr int kEpiWarp0 = 2 + kConvWarps;            // warps 10..13
constexpr int kThreads = (kEpiWarp0 + 4) * 32;       // 448
constexpr int kStageBytes = BT * BW * 2;             // 64 KB bf16 output tile staging
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 0;           // accumulator columns [0, 256)
constexpr uint32_t kACol = 256;           // A ring columns [256, 384)

struct alignas(64) Params {
    CUtensorMap xmap;   // activations bf16 {K, M}, box {64, 256}, 128-byte swizzle
    CUtensorMap wmap;   // packed weights u8 {K/2, N}, box {32, 128}
    CUtensorMap omap[KC_MAX_RANKS];  // output bf16 {N_out, M} (pitch ldc), box {128, 256}, one
                                     // per destination buffer; valid if tma_out
    const __half* scales;
    const uint8_t* zeros;   // per-group zero points u8[N, K/gs]; null: 8 (symmetric GPTQ)
    void* out;
    uint8_t* mc_out;        // multicast address of every rank's bf16 output (pitch ldc), or null
    int M, N, K, gs, ldc, out_f32, tma_out;
    int act;       // KC_ACT_NONE or KC_ACT_GELU_QUICK, applied in the epilogue
    int ndst;      // destination buffers of each tile (1, or the ranks of an all-gather)
    int col_off;   // first output column of this launch's N rows in every destination
    int tiles_w, tiles_t;
    uint32_t magic;     // 0x3F800000 (1.0f), kept in a register
    uint32_t gs_recip;      // ceil(2^32 / gs): k / gs == umulhi(k, gs_recip) for k * gs < 2^32
};

// The reference MLP block's activation, x * sigmoid(1.702 x)
// (examples/python/transformer/tensor_parallel.py:162), in fp32: __expf of a
// large positive argument gives inf and the quotient -0, of a large negative
// one 0 and the quotient x.
__device__ __forceinline__ float activate(float v, int act) {
    return act == KC_ACT_GELU_QUICK ? __fdividef(v, 1.f + __expf(-1.702f * v)) : v;
}

struct Smem {
    uint8_t x[kStages][kXBytes];   // 1024-byte aligned (swizzle atoms)
    uint8_t w[kStages][kWBytes];
    uint8_t stage[kStageBytes];    // epilogue tile: [256 tokens][128 weight rows] bf16
    uint64_t full[kStages];        // activations + packed weights landed (tx)
    uint64_t empty[kStages];       // MMA (commit) and the stage's 4 converter warps done
    uint64_t afull[kStages];       // converters wrote the TMEM A stage
    uint64_t aempty[kStages];      // MMA done reading the TMEM A stage (commit)
    uint64_t dfull;                // accumulator complete (commit)
    uint64_t dempty;               // epilogue drained the accumulator (4 warps)
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

// (x & mask) | magic in one LOP3 (magic passed in a register so the compiler
// cannot fold it into a second immediate)
template <uint32_t kMask>
__device__ __forceinline__ float nib_float(uint32_t x, uint32_t magic) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "n"(kMask), "r"(magic));
    return __uint_as_float(r);
}

// Per-group constants of the exact dequantization.  A nibble u placed at bit p
// (8, 12 or 16) of 1.0f reads f = 1 + u * 2^(p-23); then
//   fma(f, s * 2^(23-p), -(2^(23-p) + 8) * s) = (u - 8) * s
// exactly: s is an fp16 value (11 significant bits), so s * 2^(23-p) and
// (2^(23-p) + 8) * s (at most 13 + 11 bits) are exact fp32 values, the fma
// forms the exact sum, and (u - 8) * s (at most 15 bits) rounds to itself.
// One rounding then remains, the RNE to bf16 -- the same value as
// bf16_rne(float(u - 8) * s).
struct GroupConst {
    float m8, a8, m12, a12, m16, a16;
    __device__ __forceinline__ explicit GroupConst(float s)
        : m8(s * 32768.0f), a8(s * -32776.0f), m12(s * 2048.0f), a12(s * -2056.0f),
          m16(s * 128.0f), a16(s * -136.0f) {}
};

// 8 nibbles of one packed word (k = 8i .. 8i+7, low nibble first) -> 4 bf16x2
__device__ __forceinline__ void dequant_word(uint32_t w, const GroupConst& g, uint32_t magic,
                                             uint32_t* out) {
    const uint32_t lo = w << 8, hi = w >> 12;   // nibbles 0,1 -> bits 8,12; 5,6,7 -> 8,12,16
    const float w0 = __fmaf_rn(nib_float<0x00000F00u>(lo, magic), g.m8, g.a8);
    const float w1 = __fmaf_rn(nib_float<0x0000F000u>(lo, magic), g.m12, g.a12);
    const float w2 = __fmaf_rn(nib_float<0x00000F00u>(w, magic), g.m8, g.a8);
    const float w3 = __fmaf_rn(nib_float<0x0000F000u>(w, magic), g.m12, g.a12);
    const float w4 = __fmaf_rn(nib_float<0x000F0000u>(w, magic), g.m16, g.a16);
    const float w5 = __fmaf_rn(nib_float<0x00000F00u>(hi, magic), g.m8, g.a8);
    const float w6 = __fmaf_rn(nib_float<0x0000F000u>(hi, magic), g.m12, g.a12);
    const float w7 = __fmaf_rn(nib_float<0x000F0000u>(hi, magic), g.m16, g.a16);
    out[0] = bf16x2_bits(w0, w1);
    out[1] = bf16x2_bits(w2, w3);
    out[2] = bf16x2_bits(w4, w5);
    out[3] = bf16x2_bits(w6, w7);
}

// The same with a zero point z (0..15) per group.  With (2^(23-p) + z) * s
// the constant of the window at bit 8 would need up to 16 + 11 bits, so the
// nibbles use windows at bits p = 11, 15 and 19 of 2.0f instead (bit 23, the
// exponent's lowest bit, stays clear): f = 2 + u * 2^(p-22), and
//   fma(f, s * 2^(22-p), -(2^(23-p) + z) * s) = (u - z) * s
// exactly, the constants having at most 13 + 11 bits (p = 11), 9 + 11 and
// 5 + 11.  Nibbles 0-2 reach the windows by w << 11, 3-5 by w >> 1, 6-7 by
// w >> 13.
struct GroupConstZ {
    float m11, a11, m15, a15, m19, a19;
    __device__ __forceinline__ GroupConstZ(float s, float z)
        : m11(s * 2048.0f), a11(s * -(4096.0f + z)), m15(s * 128.0f), a15(s * -(256.0f + z)),
          m19(s * 8.0f), a19(s * -(16.0f + z)) {}
};

__device__ __forceinline__ void dequant_word_z(uint32_t w, const GroupConstZ& g, uint32_t magic2,
                                               uint32_t* out) {
    const uint32_t lo = w << 11, mid = w >> 1, hi = w >> 13;
    const float w0 = __fmaf_rn(nib_float<0x00007800u>(lo, magic2), g.m11, g.a11);
    const float w1 = __fmaf_rn(nib_float<0x00078000u>(lo, magic2), g.m15, g.a15);
    const float w2 = __fmaf_rn(nib_float<0x00780000u>(lo, magic2), g.m19, g.a19);
    const float w3 = __fmaf_rn(nib_float<0x00007800u>(mid, magic2), g.m11, g.a11);
    const float w4 = __fmaf_rn(nib_float<0x00078000u>(mid, magic2), g.m15, g.a15);
    const float w5 = __fmaf_rn(nib_float<0x00780000u>(mid, magic2), g.m19, g.a19);
    const float w6 = __fmaf_rn(nib_float<0x00007800u>(hi, magic2), g.m11, g.a11);
    const float w7 = __fmaf_rn(nib_float<0x00078000u>(hi, magic2), g.m15, g.a15);
    out[0] = bf16x2_bits(w0, w1);
    out[1] = bf16x2_bits(w2, w3);
    out[2] = bf16x2_bits(w4, w5);
    out[3] = bf16x2_bits(w6, w7);
}

__global__ void __launch_bounds__(kThreads, 1) gemm_w4a16_kernel(const __grid_constant__ Params P) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = sm100::smem_u32(smem_raw);
    Smem& S = *reinterpret_cast<Smem*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = P.tiles_w * P.tiles_t;
    const int ksteps = P.K / BK;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            sm100::mbar_init(&S.full[i], 1);
            sm100::mbar_init(&S.empty[i], 1 + 4);
            sm100::mbar_init(&S.afull[i], 4);
            sm100::mbar_init(&S.aempty[i], 1);
        }
        sm100::mbar_init(&S.dfull, 1);
        sm100::mbar_init(&S.dempty, 4);
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
            sm100::prefetch_tensormap(&P.xmap);
            sm100::prefetch_tensormap(&P.wmap);
            uint32_t it = 0;   // loads issued; nothing more is issued after a failed wait
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
                const int n0 = (tile / P.tiles_t) * BW, m0 = (tile % P.tiles_t) * BT;
                for (int ks = 0; ks < ksteps; ++ks, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    if (!(ok = sm100::mbar_wait_or_abort(&S.empty[s], ph ^ 1u, abort))) break;
                    sm100::mbar_arrive_expect_tx(&S.full[s], kXBytes + kWBytes);
                    sm100::tma_load_2d(S.x[s], &P.xmap, ks * BK, m0, &S.full[s]);
                    sm100::tma_load_2d(S.w[s], &P.wmap, ks * (BK / 2), n0, &S.full[s]);
                }
            }
            for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0u; j < it; ++j)
                sm100::mbar_wait(&S.full[j % kStages], (j / kStages) & 1u, 200000000ull);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            const uint32_t idesc = sm100::umma_idesc(sm100::kFmtBF16, sm100::kFmtBF16, BW, BT);
            uint32_t it = 0, t = 0;
            bool ok = true;   // false once a wait gave up: no MMA is issued after that
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t) {
                ok = sm100::mbar_wait_or_abort(&S.dempty, (t & 1u) ^ 1u, abort) && ok;
                sm100::tc_fence_after();
                for (int ks = 0; ks < ksteps; ++ks, ++it) {
                    const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                    ok = sm100::mbar_wait_or_abort(&S.full[s], ph, abort) && ok;
                    ok = sm100::mbar_wait_or_abort(&S.afull[s], ph, abort) && ok;
                    sm100::tc_fence_after();
                    if (ok) {   // stages that were never filled are not multiplied
                        const uint64_t bdesc = sm100::umma_desc_sw128(sm100::smem_u32(S.x[s]));
                        const uint32_t a_tmem = tmem + kACol + s * (BK / 2);
#pragma unroll
                        for (int j = 0; j < BK / 16; ++j)  // K = 16 per instruction
                            sm100::umma_f16_ts(tmem + kAccCol, a_tmem + j * 8, bdesc + 2 * j, idesc,
                                               (ks | j) != 0 ? 1u : 0u);
                    }
                    // committed either way, so the barriers keep completing
                    sm100::tc_commit(&S.empty[s]);   // activations free
                    sm100::tc_commit(&S.aempty[s]);  // TMEM A stage free
                }
                sm100::tc_commit(&S.dfull);
            }
            sm100::tc_commit(&S.drain);
            sm100::mbar_wait(&S.drain, 0, 200000000ull);
        }
    } else if (warp < kEpiWarp0) {
        // -------------------------------- converters --------------------------------
        const int q = warp & 3;                 // TMEM lane quarter (warp % 4 rule)
        const uint32_t par = (uint32_t)(warp - 2) >> 2;  // this warp takes steps it % 2 == par
        const int row = q * 32 + lane;          // weight row within the tile
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        uint32_t it = 0;
        const uint32_t magic2 = P.magic + 0x00800000u;   // 2.0f for the zero-point windows
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int n0 = (tile / P.tiles_t) * BW;
            const int n = min(n0 + row, P.N - 1);
            const __half* srow = P.scales + (size_t)n * (P.K / P.gs);
            const uint8_t* zrow = P.zeros ? P.zeros + (size_t)n * (P.K / P.gs) : nullptr;
            for (int ks = 0; ks < ksteps; ++ks, ++it) {
                if ((it & 1u) != par) continue;
                const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                const uint32_t grp = __umulhi((uint32_t)(ks * BK), P.gs_recip);
                const float sc = __half2float(__ldg(srow + grp));
                sm100::mbar_wait_or_abort(&S.full[s], ph, abort);
                const uint32_t wa = sm100::smem_u32(S.w[s]) + row * (BK / 2);
                const uint4 p0 = lds128(wa), p1 = lds128(wa + 16);
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(&S.empty[s]);  // packed bytes consumed
                const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                uint32_t v[32];  // column c of the A stage holds k = 2c (low half), 2c + 1
                if (zrow == nullptr) {
                    const GroupConst gc(sc);
#pragma unroll
                    for (int i = 0; i < 8; ++i) dequant_word(words[i], gc, P.magic, v + 4 * i);
                } else {
                    const GroupConstZ gz(sc, (float)(__ldg(zrow + grp) & 15));
#pragma unroll
                    for (int i = 0; i < 8; ++i) dequant_word_z(words[i], gz, magic2, v + 4 * i);
                }
                sm100::mbar_wait_or_abort(&S.aempty[s], ph ^ 1u, abort);
                __syncwarp();
                sm100::tc_fence_after();
                const uint32_t col = tmem + kACol + s * (BK / 2) + lane_addr;
                uint32_t r0[16], r1[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) { r0[i] = v[i]; r1[i] = v[16 + i]; }
                sm100::tmem_st_32x32b_x16(col, r0);
                sm100::tmem_st_32x32b_x16(col + 16, r1);
                sm100::tmem_wait_st();
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(&S.afull[s]);
            }
        }
    } else {
        // -------------------------------- epilogue --------------------------------
        const int q = warp & 3;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        uint8_t* stage = S.stage;
        const bool store_lead = warp == kEpiWarp0 && lane == 0;   // issues the tile's stores
        uint32_t t = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t) {
            const int n0 = (tile / P.tiles_t) * BW, m0 = (tile % P.tiles_t) * BT;
            const int n = n0 + q * 32 + lane;
            const bool waited = sm100::mbar_wait_or_abort(&S.dfull, t & 1u, abort);
            sm100::tc_fence_after();
            // after a wait gave up anywhere in the CTA the accumulator is not a
            // result: the tile is written as NaN, so a timeout cannot pass for
            // plausible output (kc_get_device_status reports it as well)
            const float nan = __int_as_float(0x7FC00000);
            const bool poison = !waited || *abort;
            if (P.tma_out || P.mc_out) {
                // the previous tile's TMA stores have finished reading the staging tile
                // (multicast stores take their data from registers: nothing to wait for)
                if (store_lead && P.tma_out) sm100::bulk_wait_group_read0();
                sm100::named_sync(1, 128);
#pragma unroll 1
                for (int c = 0; c < BT / 64; ++c) {
                    uint32_t r[32], r2[32];
                    __syncwarp();
                    sm100::tmem_ld_32x32b_x32(tmem + kAccCol + lane_addr + c * 64, r);
                    sm100::tmem_ld_32x32b_x32(tmem + kAccCol + lane_addr + c * 64 + 32, r2);
                    sm100::tmem_wait_ld();
                    if (c == BT / 64 - 1) {  // accumulator drained: hand it back to the MMA
                        sm100::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) sm100::mbar_arrive(&S.dempty);
                    }
                    // row m of the tile holds its 128 weight rows: 256 bytes, of
                    // which this warp writes its 32 (64 bytes, one per lane)
                    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(stage) + c * 64 * BW + q * 32 + lane;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        o[i * BW] = __float2bfloat16_rn(poison ? nan : activate(__uint_as_float(r[i]), P.act));
                        o[(32 + i) * BW] =
                            __float2bfloat16_rn(poison ? nan : activate(__uint_as_float(r2[i]), P.act));
                    }
                }
                if (P.mc_out) {
                    // every rank's copy at once through the NVSwitch: each 16-byte
                    // piece of the tile leaves the SM once (multimem.st), the switch
                    // writes it into all copies.  Token row r of the tile is 256
                    // bytes (16 pieces); the 128 threads take pieces t, t + 128, ...
                    sm100::named_sync(1, 128);   // all four strips are in the staging tile
                    const int rows = min(BT, P.M - m0);
                    const uint32_t stage_u32 = sm100::smem_u32(stage);
                    const int t = threadIdx.x - kEpiWarp0 * 32;
                    uint8_t* dst = P.mc_out + ((size_t)m0 * P.ldc + P.col_off + n0) * 2;
#pragma unroll 4
                    for (int i = t; i < rows * 16; i += 128) {
                        const int r = i >> 4, v = i & 15;
                        const uint4 d = lds128(stage_u32 + r * (BW * 2) + v * 16);
                        asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};"
                                     ::"l"(dst + (size_t)r * P.ldc * 2 + v * 16), "r"(d.x), "r"(d.y),
                                       "r"(d.z), "r"(d.w)
                                     : "memory");
                    }
                } else {
                    sm100::fence_proxy_async_smem();
                    sm100::named_sync(1, 128);   // all four strips are in the staging tile
                    if (store_lead) {
                        // one 128-column box per destination: 256-byte rows, local
                        // buffer or every rank's over NVLink
                        for (int d = 0; d < P.ndst; ++d)
                            sm100::tma_store_2d(&P.omap[d], stage, P.col_off + n0, m0);
                        sm100::bulk_commit_group();
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BT / 32; ++c) {
                    uint32_t r[32];
                    __syncwarp();
                    sm100::tmem_ld_32x32b_x32(tmem + kAccCol + lane_addr + c * 32, r);
                    sm100::tmem_wait_ld();
                    const int mb = m0 + c * 32;
                    if (n < P.N) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (mb + i < P.M) {
                                const float f = poison ? nan : activate(__uint_as_float(r[i]), P.act);
                                if (P.out_f32)
                                    reinterpret_cast<float*>(P.out)[(size_t)(mb + i) * P.ldc + n] = f;
                                else
                                    reinterpret_cast<__nv_bfloat16*>(P.out)[(size_t)(mb + i) * P.ldc + n] =
                                        __float2bfloat16_rn(f);
                            }
                        }
                    }
                }
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(&S.dempty);
            }
        }
        if (store_lead) sm100::bulk_wait_group0();  // stores complete before the CTA exits
        if (P.mc_out) __threadfence_system();        // the multicast stores, before the barrier after
    }

    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

KC_DEFINE_STATUS_READER(gemm_w4a16)

namespace {

// Shared launcher: outs[0..ndst) each receive columns [col_off, col_off + N)
// of the product (bf16 through the TMA-store epilogue when tma_out), or, for a
// single destination, fp32 / unaligned output through direct stores.
int launch_gemm_w4a16(const uint16_t* x_bf16, const uint8_t* packed, const uint16_t* scales_f16,
                      const uint8_t* zeros, void* const* outs, int ndst, int col_off, int out_cols,
                      int out_f32, int M, int N, int K, int group_size, int ldc, int act,
                      cudaStream_t stream, void* mc_out = nullptr) {
    KC_REQUIRE(x_bf16 && packed && scales_f16 && outs && outs[0], KC_ERR_INVALID_ARG,
               "null pointer argument");
    KC_REQUIRE(act == KC_ACT_NONE || act == KC_ACT_GELU_QUICK, KC_ERR_INVALID_ARG,
               "unknown activation %d", act);
    KC_REQUIRE(M >= 0 && N >= 0 && K >= 0, KC_ERR_INVALID_ARG, "negative size");
    if (M == 0 || N == 0) return KC_OK;
    KC_REQUIRE(K > 0 && K % BK == 0, KC_ERR_INVALID_ARG, "K=%d must be a positive multiple of %d", K, BK);
    KC_REQUIRE(group_size > 0 && group_size % BK == 0 && K % group_size == 0, KC_ERR_INVALID_ARG,
               "group_size=%d must be a multiple of %d dividing K=%d", group_size, BK, K);
    KC_REQUIRE(ldc >= out_cols, KC_ERR_INVALID_ARG, "ldc=%d < output columns %d", ldc, out_cols);
    KC_REQUIRE((uint64_t)K * (uint64_t)group_size < (1ull << 32), KC_ERR_INVALID_ARG,
               "K * group_size must be below 2^32");
    KC_REQUIRE(kc::aligned(x_bf16, 16) && kc::aligned(packed, 16) && kc::aligned(scales_f16, 2) &&
                   kc::aligned(outs[0], 4),
               KC_ERR_ALIGNMENT, "x and packed must be 16-byte aligned");
    Params P{};
    int st = kc::encode_2d(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x_bf16, (uint64_t)K, (uint64_t)M,
                           (uint64_t)K * 2, BK, BT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = kc::encode_2d(&P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, (uint64_t)(K / 2), (uint64_t)N,
                       (uint64_t)(K / 2), BK / 2, BW, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    bool aligned = true;
    for (int d = 0; d < ndst; ++d) aligned = aligned && outs[d] && kc::aligned(outs[d], 16);
    P.tma_out = (!out_f32 && aligned && ldc % 8 == 0 && mc_out == nullptr) ? 1 : 0;
    P.mc_out = static_cast<uint8_t*>(mc_out);
    KC_REQUIRE(ndst == 1 || P.tma_out, KC_ERR_ALIGNMENT,
               "all-gather outputs must be bf16, 16-byte aligned, with a pitch divisible by 8");
    if (P.tma_out) {
        for (int d = 0; d < ndst; ++d) {
            st = kc::encode_2d(&P.omap[d], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, outs[d],
                               (uint64_t)out_cols, (uint64_t)M, (uint64_t)ldc * 2, BW, BT,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
            if (st) return st;
        }
    }
    P.ndst = ndst;
    P.col_off = col_off;
    P.scales = reinterpret_cast<const __half*>(scales_f16);
    P.zeros = zeros;
    P.out = outs[0];
    P.M = M;
    P.N = N;
    P.K = K;
    P.gs = group_size;
    P.ldc = ldc;
    P.out_f32 = out_f32 ? 1 : 0;
    P.act = act;
    P.tiles_w = (N + BW - 1) / BW;
    P.tiles_t = (M + BT - 1) / BT;
    P.magic = 0x3F800000u;
    P.gs_recip = (uint32_t)((0x100000000ull + (uint64_t)group_size - 1) / (uint64_t)group_size);
    const size_t smem = sizeof(Smem) + 1024;
    KC_CUDA_TRY(cudaFuncSetAttribute(gemm_w4a16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "gemm_w4a16 shared-memory attribute");
    const int tiles = P.tiles_w * P.tiles_t;
    gemm_w4a16_kernel<<<std::min(tiles, kc::sm_count()), kThreads, smem, stream>>>(P);
    return kc::check_launch("gemm_w4a16");
}

}  // namespace

extern "C" {

int kc_gemm_w4a16(const uint16_t* x_bf16, const uint8_t* packed, const uint16_t* scales_f16,
                  void* out, int out_f32, int M, int N, int K, int group_size, int ldc,
                  cudaStream_t stream) {
    void* outs[1] = {out};
    return launch_gemm_w4a16(x_bf16, packed, scales_f16, nullptr, outs, 1, 0, N, out_f32, M, N, K,
                             group_size, ldc, KC_ACT_NONE, stream);
}

int kc_gemm_w4a16_zp(const uint16_t* x_bf16, const uint8_t* packed, const uint16_t* scales_f16,
                     const uint8_t* zeros, void* out, int out_f32, int M, int N, int K,
                     int group_size, int ldc, int act, cudaStream_t stream) {
    KC_REQUIRE(zeros != nullptr, KC_ERR_INVALID_ARG, "null zero points");
    void* outs[1] = {out};
    return launch_gemm_w4a16(x_bf16, packed, scales_f16, zeros, outs, 1, 0, N, out_f32, M, N, K,
                             group_size, ldc, act, stream);
}

int kc_gemm_w4a16_act(const uint16_t* x_bf16, const uint8_t* packed, const uint16_t* scales_f16,
                      void* out, int out_f32, int M, int N, int K, int group_size, int ldc, int act,
                      cudaStream_t stream) {
    void* outs[1] = {out};
    return launch_gemm_w4a16(x_bf16, packed, scales_f16, nullptr, outs, 1, 0, N, out_f32, M, N, K,
                             group_size, ldc, act, stream);
}

int kc_gemm_w4a16_allgather_mc(const uint16_t* x_bf16, const uint8_t* packed_shard,
                               const uint16_t* scales_shard, void* mc_out, int nranks, int rank, int M,
                               int N_shard, int K, int group_size, cudaStream_t stream) {
    KC_REQUIRE(mc_out != nullptr && kc::aligned(mc_out, 16), KC_ERR_ALIGNMENT,
               "multicast output null or not 16-byte aligned");
    KC_REQUIRE(nranks >= 1 && nranks <= KC_MAX_RANKS && rank >= 0 && rank < nranks, KC_ERR_INVALID_ARG,
               "rank %d of %d outside 0..%d", rank, nranks, KC_MAX_RANKS - 1);
    KC_REQUIRE(N_shard >= 0 && N_shard % BW == 0, KC_ERR_INVALID_ARG,
               "N_shard=%d must be a multiple of %d", N_shard, BW);
    const long cols = (long)N_shard * nranks;
    KC_REQUIRE(cols < (1L << 31), KC_ERR_INVALID_ARG, "output too wide");
    // outs[0] only passes the launcher's checks; every store goes through mc_out
    void* outs[1] = {mc_out};
    return launch_gemm_w4a16(x_bf16, packed_shard, scales_shard, nullptr, outs, 1, rank * N_shard,
                             (int)cols, 0, M, N_shard, K, group_size, (int)cols, KC_ACT_NONE, stream,
                             mc_out);
}

int kc_gemm_w4a16_allgather(const uint16_t* x_bf16, const uint8_t* packed_shard,
                            const uint16_t* scales_shard, void* const* outs, int nranks, int rank,
                            int M, int N_shard, int K, int group_size, cudaStream_t stream) {
    KC_REQUIRE(outs != nullptr && nranks >= 1 && nranks <= KC_MAX_RANKS && rank >= 0 &&
                   rank < nranks,
               KC_ERR_INVALID_ARG, "rank %d of %d outside 0..%d", rank, nranks, KC_MAX_RANKS - 1);
    KC_REQUIRE(N_shard >= 0 && N_shard % BW == 0, KC_ERR_INVALID_ARG,
               "N_shard=%d must be a multiple of %d (a store box never crosses into a peer's columns)",
               N_shard, BW);
    const long cols = (long)N_shard * nranks;
    KC_REQUIRE(cols < (1L << 31), KC_ERR_INVALID_ARG, "output too wide");
    return launch_gemm_w4a16(x_bf16, packed_shard, scales_shard, nullptr, outs, nranks, rank * N_shard,
                             (int)cols, 0, M, N_shard, K, group_size, (int)cols, KC_ACT_NONE, stream);
}

}  // extern "C"
