// int4.cu -- INT4 weight dequantization and the W4 GEMV family for sm_100a.
//
// Weight format (both APIs): packed u8[N, K/2], row-major, two 4-bit values per
// byte, low nibble = even k (src/kernels/transformer/quant_int4.cu:6-13).
//
//  * Reference ABI (launch_dequantize_int4 / launch_gemv_int4): fp32 scales,
//    nibbles SIGN-extended (quant_int4.cu:34-48), zero points read UNSIGNED from
//    a packed buffer whose row stride is floor(K/gs/2) (quant_int4.cu:93-96).
//    The index arithmetic below is the reference's, so the dequantized weights
//    are bit-identical for every zeros buffer.
//  * GPTQ API (kc_*_w4*): fp16 scales, implicit zero-point 8,
//    w = (u - 8) * s with u the unsigned nibble.
//
// The W4A16 GEMV (M <= 16) streams the packed weights through shared memory
// with bulk async copies issued by a producer warp and runs the dot products
// on the tensor cores: consumer warps turn each 16-byte weight slice into bf16
// MMA fragments in registers and feed them straight into mma.sync m16n8k16,
// activations as the B operand.  The group scale is applied in fp32 to the
// per-chunk partial product, so the only roundings are fp32 accumulations.
// Dequantized weights never touch shared memory or TMEM: at M <= 16 the kernel
// is bound by HBM, and staging bf16 weights for a tcgen05 A operand (2 bytes
// written and read per weight) would cost more on-chip bandwidth than the
// 0.5 byte per weight streamed from HBM.
#include <algorithm>

#include "kc_common.cuh"
#include "sm100.cuh"

namespace {

// ---------------------------------------------------------------------------
// Reference-ABI helpers (quant_int4.cu:34-48, 93-96)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int sx4(uint32_t v) {  // v in 0..15
    return (int)((v ^ 8u)) - 8;
}

__device__ __forceinline__ int ref_zp(const uint8_t* zeros, int row, int cols, int gs, int g) {
    const int zc = cols / gs / 2;
    const uint8_t zb = zeros[(long)row * zc + g / 2];
    return (g % 2 == 0) ? (zb & 0x0F) : (zb >> 4);
}

// One thread per packed byte: the reference's own decomposition, kept for any
// shape the vector path cannot take (odd group sizes, unaligned pointers).
__global__ void dequant_int4_f32_bytes(const uint8_t* __restrict__ packed,
                                       const float* __restrict__ scales,
                                       const uint8_t* __restrict__ zeros,
                                       float* __restrict__ out, int rows, int cols, int gs) {
    const long nbytes = (long)rows * (cols / 2);
    const int sc = cols / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nbytes;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / (cols / 2));
        const int b = (int)(i - (long)r * (cols / 2));
        const int c0 = 2 * b, c1 = c0 + 1;
        const uint8_t p = packed[i];
        const int g0 = c0 / gs, g1 = c1 / gs;
        const float s0 = scales[(long)r * sc + g0];
        const float s1 = scales[(long)r * sc + g1];
        out[(long)r * cols + c0] = (float)(sx4(p & 15u) - ref_zp(zeros, r, cols, gs, g0)) * s0;
        if (c1 < cols)
            out[(long)r * cols + c1] = (float)(sx4(p >> 4) - ref_zp(zeros, r, cols, gs, g1)) * s1;
    }
}

// One thread per 16-byte chunk (32 weights, all in one group): 128-bit load,
// eight 128-bit stores.  Requires cols % 32 == 0, gs % 32 == 0, 16B alignment.
__global__ void dequant_int4_f32_vec(const uint8_t* __restrict__ packed,
                                     const float* __restrict__ scales,
                                     const uint8_t* __restrict__ zeros,
                                     float* __restrict__ out, int rows, int cols, int gs) {
    const int cpr = cols / 32;  // chunks per row
    const long nchunks = (long)rows * cpr;
    const int sc = cols / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / cpr);
        const int j = (int)(i - (long)r * cpr);
        const int g = (32 * j) / gs;
        const float s = scales[(long)r * sc + g];
        const int zp = ref_zp(zeros, r, cols, gs, g);
        const uint4 v = kc_ldg_stream(packed + i * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float4* dst = reinterpret_cast<float4*>(out + (long)r * cols + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = (float)(sx4((w[q] >> (4 * e)) & 15u) - zp) * s;
            dst[2 * q]     = make_float4(f[0], f[1], f[2], f[3]);
            dst[2 * q + 1] = make_float4(f[4], f[5], f[6], f[7]);
        }
    }
}

// fp32 GEMV, one warp per row.  VEC: 16-byte chunks, one group per chunk.
template <bool VEC>
__global__ void __launch_bounds__(256) gemv_int4_f32(const uint8_t* __restrict__ packed,
                                                     const float* __restrict__ scales,
                                                     const uint8_t* __restrict__ zeros,
                                                     const float* __restrict__ x,
                                                     float* __restrict__ y, int rows, int cols,
                                                     int gs) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int sc = cols / gs;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        float acc = 0.f;
        if (VEC) {
            const uint8_t* prow = packed + (long)r * (cols / 2);
            for (int j = lane; j < cols / 32; j += 32) {
                const int g = (32 * j) / gs;
                const float s = scales[(long)r * sc + g];
                const int zp = ref_zp(zeros, r, cols, gs, g);
                const uint4 v = kc_ldg_stream(prow + 16 * j);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                const float4* xv = reinterpret_cast<const float4*>(x + 32 * j);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 xa = __ldg(xv + 2 * q), xb = __ldg(xv + 2 * q + 1);
                    const float xe[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float wv = (float)(sx4((w[q] >> (4 * e)) & 15u) - zp) * s;
                        acc = fmaf(wv, xe[e], acc);
                    }
                }
            }
        } else {
            for (int b = lane; 2 * b < cols; b += 32) {
                const int c0 = 2 * b, c1 = c0 + 1;
                const uint8_t p = packed[(long)r * (cols / 2) + b];
                const int g0 = c0 / gs, g1 = c1 / gs;
                const float w0 = (float)(sx4(p & 15u) - ref_zp(zeros, r, cols, gs, g0)) *
                                 scales[(long)r * sc + g0];
                acc = fmaf(w0, x[c0], acc);
                if (c1 < cols) {
                    const float w1 = (float)(sx4(p >> 4) - ref_zp(zeros, r, cols, gs, g1)) *
                                     scales[(long)r * sc + g1];
                    acc = fmaf(w1, x[c1], acc);
                }
            }
        }
        acc = kc_warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

// ---------------------------------------------------------------------------
// GPTQ (implicit zero-point 8) helpers
// ---------------------------------------------------------------------------

// bf16 dequant, one thread per 16-byte chunk (32 weights of one group).
__global__ void dequant_w4_bf16_vec(const uint8_t* __restrict__ packed,
                                    const __half* __restrict__ scales,
                                    __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const int cpr = K / 32;
    const long nchunks = (long)N * cpr;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / cpr);
        const int j = (int)(i - (long)r * cpr);
        const float s = __half2float(scales[(long)r * sc + (32 * j) / gs]);
        const uint4 v = kc_ldg_stream(packed + i * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint4* dst = reinterpret_cast<uint4*>(out + (long)r * K + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float lo = (float)((int)((w[q] >> (8 * e)) & 15u) - 8) * s;
                const float hi = (float)((int)((w[q] >> (8 * e + 4)) & 15u) - 8) * s;
                __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                o[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

__global__ void dequant_w4_bf16_scalar(const uint8_t* __restrict__ packed,
                                       const __half* __restrict__ scales,
                                       __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const long n = (long)N * K;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / K);
        const int c = (int)(i - (long)r * K);
        const uint8_t p = packed[(long)r * (K / 2) + c / 2];
        const int u = (c & 1) ? (p >> 4) : (p & 15);
        const float w = (float)(u - 8) * __half2float(scales[(long)r * sc + c / gs]);
        out[i] = __float2bfloat16_rn(w);
    }
}

// ---------------------------------------------------------------------------
// W4A16 GEMV on the tensor cores
// ---------------------------------------------------------------------------
struct W4A16Prob {
    const uint8_t* packed;
    const __half* scales;
    const __nv_bfloat16* x;
    float* y;
    int N, K;
    int tile_begin;  // first 16-row tile of this problem in the flattened tile list
};

struct W4A16Params {
    W4A16Prob p[KC_W4A16_MAX_PROBLEMS];
    int count;
    int total_tiles;
    int M;
    int gs;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void mma_bf16_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Warp-specialized, TMA-fed W4A16 GEMV.
//
// One CTA per SM, persistent over 16-row tiles (problem-major order).  Warp 8
// is the producer: one lane streams each tile's packed rows into an 8-stage
// shared-memory ring with 1-D bulk async copies (16 rows x 1 KB per stage,
// completion counted on the stage's "full" mbarrier), so HBM always has
// ~140 KB per SM in flight regardless of what the consumers are doing.
// Warps 0-7 are consumers: a stage's 16 chunks of 128 k are split across
// them (chunk c -> warp c % 8); each lane (g = lane/4, t = lane%4) reads rows
// g and g+8, bytes [64c' + 16t, +16) of its chunk c' from shared memory,
// turns each 32-bit word into four bf16x2 MMA fragments (128 + u, exact),
// and issues mma.sync m16n8k16 against the activation fragment; a second MMA
// with the constant fragment -136 on the same activations turns the sum into
// sum (u - 8) x without a per-weight subtraction.  The group scale is applied
// in fp32 to the per-chunk partial product.  At the end of a tile the eight
// warps' partial sums are reduced through shared memory and y is written.
// Row stride in shared memory is 1 KB + 64 B so the LDS.128 reads of rows g
// and g+1 fall in different banks.
// ---------------------------------------------------------------------------
constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageRowBytes = 1024;                 // packed bytes per row per stage
constexpr int kRowPitch = kStageRowBytes + 64;
constexpr int kStages = 8;

template <int NT>
struct GemvSmem {
    uint8_t ring[kStages][16][kRowPitch];
    float red[2][kConsumerWarps][16][NT * 8 + 1];
    uint64_t full[kStages];
    uint64_t empty[kStages];
};

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(sm100::smem_u32(p)));
    return v;
}

// Four bf16x2 fragments (128 + u) for the nibble pairs (k0,k4) (k1,k5) (k2,k6)
// (k3,k7) of one 32-bit word: OR-ing a nibble into the mantissa of bf16 128.0
// (0x4300) gives exactly 128 + u.
__device__ __forceinline__ void w4_to_bf16x2_biased(uint32_t w, uint32_t o[4]) {
    const uint32_t mask = 0x000F000Fu, magic = 0x43004300u;
    o[0] = (w & mask) | magic;
    o[1] = ((w >> 4) & mask) | magic;
    o[2] = ((w >> 8) & mask) | magic;
    o[3] = ((w >> 12) & mask) | magic;
}

__device__ __forceinline__ const W4A16Prob& problem_of(const W4A16Params& P, int tile) {
    int pi = 0;
#pragma unroll 1
    while (pi + 1 < P.count && tile >= P.p[pi + 1].tile_begin) ++pi;
    return P.p[pi];
}

template <int NT>
__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_w4a16_tma(const __grid_constant__ W4A16Params P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GemvSmem<NT>& S = *reinterpret_cast<GemvSmem<NT>*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            sm100::mbar_init(&S.full[i], 1);
            sm100::mbar_init(&S.empty[i], kConsumerWarps);
        }
        sm100::fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        if (lane != 0) return;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < P.total_tiles && ok; tile += gridDim.x) {
            const W4A16Prob& pr = problem_of(P, tile);
            const int row0 = (tile - pr.tile_begin) * 16;
            const int rowbytes = pr.K >> 1;
            for (int off = 0; off < rowbytes && ok; off += kStageRowBytes, ++it) {
                const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
                if (!sm100::mbar_wait(&S.empty[s], ph ^ 1u)) { ok = false; break; }
                const uint32_t len = (uint32_t)min(kStageRowBytes, rowbytes - off);
                sm100::mbar_arrive_expect_tx(&S.full[s], 16u * len);
#pragma unroll 4
                for (int r = 0; r < 16; ++r) {
                    const int row = min(row0 + r, pr.N - 1);
                    sm100::bulk_g2s(&S.ring[s][r][0], pr.packed + (size_t)row * rowbytes + off, len,
                                    &S.full[s]);
                }
            }
        }
        // Drain: every copy this thread issued must land before the CTA exits.
        const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0u;
        for (uint32_t j = first; j < it; ++j)
            if (!sm100::mbar_wait(&S.full[j % kStages], (j / kStages) & 1u)) break;
        return;
    }

    // ------------------------------- consumers --------------------------------
    const int g = lane >> 2, t = lane & 3;
    const int M = P.M, gs = P.gs;
    const uint32_t neg136 = 0xC308C308u;  // bf16x2 (-136, -136)
    uint32_t it = 0;
    int rb = 0;  // reduction buffer parity
    bool ok = true;
    for (int tile = blockIdx.x; tile < P.total_tiles; tile += gridDim.x) {
        const W4A16Prob& pr = problem_of(P, tile);
        const int N = pr.N, K = pr.K;
        const int row0 = (tile - pr.tile_begin) * 16;
        const int rowbytes = K >> 1;
        const int ra = min(row0 + g, N - 1), rb8 = min(row0 + g + 8, N - 1);
        const __half* sa_row = pr.scales + (size_t)ra * (K / gs);
        const __half* sb_row = pr.scales + (size_t)rb8 * (K / gs);

        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

        for (int off = 0; off < rowbytes; off += kStageRowBytes, ++it) {
            const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
            const int nch = min(kStageRowBytes, rowbytes - off) >> 6;  // 64-byte chunks
            // this warp's chunks: warp, warp + 8 (at most two per stage)
            const int c0 = warp, c1 = warp + kConsumerWarps;
            const bool h0 = c0 < nch, h1 = c1 < nch;
            // scales and activations do not depend on the stage: fetch them first
            float sa[2] = {0.f, 0.f}, sb[2] = {0.f, 0.f};
            uint4 X[2][NT][4];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const bool has = q ? h1 : h0;
                const int c = q ? c1 : c0;
                const int k0 = (off + c * 64) * 2;  // first k of the chunk
                if (has) {
                    sa[q] = __half2float(sa_row[k0 / gs]);
                    sb[q] = __half2float(sb_row[k0 / gs]);
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int n = nt * 8 + g;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        X[q][nt][j] = (has && n < M)
                                          ? kc_ldg_keep(pr.x + (size_t)n * K + k0 + 32 * t + 8 * j)
                                          : make_uint4(0u, 0u, 0u, 0u);
                }
            }
            if (ok && !sm100::mbar_wait(&S.full[s], ph)) ok = false;
            uint4 WA[2], WB[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int c = q ? c1 : c0;
                const bool has = q ? h1 : h0;
                WA[q] = has ? lds128(&S.ring[s][g][c * 64 + 16 * t]) : make_uint4(0u, 0u, 0u, 0u);
                WB[q] = has ? lds128(&S.ring[s][g + 8][c * 64 + 16 * t]) : make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&S.empty[s]);

            float cm[2][NT][4], cc[2][NT][4];
#pragma unroll
            for (int q = 0; q < 2; ++q)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) cm[q][nt][e] = cc[q][nt][e] = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint32_t wa = j == 0 ? WA[q].x : j == 1 ? WA[q].y : j == 2 ? WA[q].z : WA[q].w;
                    const uint32_t wb = j == 0 ? WB[q].x : j == 1 ? WB[q].y : j == 2 ? WB[q].z : WB[q].w;
                    uint32_t A[4], B[4];
                    w4_to_bf16x2_biased(wa, A);
                    w4_to_bf16x2_biased(wb, B);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint32_t xlo = h ? X[q][nt][j].y : X[q][nt][j].x;
                            const uint32_t xhi = h ? X[q][nt][j].w : X[q][nt][j].z;
                            const uint32_t b0 = prmt(xlo, xhi, 0x5410u);
                            const uint32_t b1 = prmt(xlo, xhi, 0x7632u);
                            mma_bf16_16816(cm[q][nt], A[2 * h], B[2 * h], A[2 * h + 1], B[2 * h + 1],
                                           b0, b1);
                            mma_bf16_16816(cc[q][nt], neg136, neg136, neg136, neg136, b0, b1);
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 2; ++q)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    acc[nt][0] = fmaf(sa[q], cm[q][nt][0] + cc[q][nt][0], acc[nt][0]);
                    acc[nt][1] = fmaf(sa[q], cm[q][nt][1] + cc[q][nt][1], acc[nt][1]);
                    acc[nt][2] = fmaf(sb[q], cm[q][nt][2] + cc[q][nt][2], acc[nt][2]);
                    acc[nt][3] = fmaf(sb[q], cm[q][nt][3] + cc[q][nt][3], acc[nt][3]);
                }
        }
        // ---- cross-warp reduction of the tile (double-buffered: one barrier)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            S.red[rb][warp][g][nt * 8 + 2 * t]         = acc[nt][0];
            S.red[rb][warp][g][nt * 8 + 2 * t + 1]     = acc[nt][1];
            S.red[rb][warp][g + 8][nt * 8 + 2 * t]     = acc[nt][2];
            S.red[rb][warp][g + 8][nt * 8 + 2 * t + 1] = acc[nt][3];
        }
        sm100::named_sync(1, kConsumerWarps * 32);
        for (int i = threadIdx.x; i < 16 * M; i += kConsumerWarps * 32) {
            const int r = i & 15, n = i >> 4;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) v += S.red[rb][w][r][n];
            if (row0 + r < N) pr.y[(size_t)n * N + row0 + r] = v;
        }
        rb ^= 1;
    }
}

// CUDA-core fallback for shapes the tensor-core path cannot take (group sizes
// that are not a multiple of 128, unaligned pointers).  One warp per row.
__global__ void __launch_bounds__(256) gemv_w4a16_scalar(const __grid_constant__ W4A16Params P) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    int total_rows = 0;
    for (int i = 0; i < P.count; ++i) total_rows += P.p[i].N;
    for (int gr = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; gr < total_rows; gr += warps) {
        int pi = 0, r = gr;
        while (r >= P.p[pi].N) { r -= P.p[pi].N; ++pi; }
        const W4A16Prob& pr = P.p[pi];
        const int K = pr.K, sc = K / P.gs;
        float acc[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) acc[m] = 0.f;
        for (int c = lane; c < K; c += 32) {
            const uint8_t p = pr.packed[(size_t)r * (K / 2) + c / 2];
            const int u = (c & 1) ? (p >> 4) : (p & 15);
            const float w = (float)(u - 8) * __half2float(pr.scales[(size_t)r * sc + c / P.gs]);
#pragma unroll
            for (int m = 0; m < 16; ++m)
                if (m < P.M) acc[m] = fmaf(w, __bfloat162float(pr.x[(size_t)m * K + c]), acc[m]);
        }
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            if (m < P.M) {
                const float s = kc_warp_sum(acc[m]);
                if (lane == 0) pr.y[(size_t)m * pr.N + r] = s;
            }
        }
    }
}

int grid_for(long work_items, int threads) {
    const long cap = (long)kc::sm_count() * (2048 / threads);
    long g = work_items < cap ? work_items : cap;
    return g < 1 ? 1 : (int)g;
}

int check_ref_int4_args(const void* packed, const void* scales, const void* zeros, const void* out,
                        int rows, int cols, int gs) {
    KC_REQUIRE(packed && scales && zeros && out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(rows >= 0 && cols >= 0, KC_ERR_INVALID_ARG, "negative size rows=%d cols=%d", rows, cols);
    KC_REQUIRE(cols % 2 == 0, KC_ERR_INVALID_ARG, "cols=%d must be even", cols);
    KC_REQUIRE(gs > 0 && cols % gs == 0, KC_ERR_INVALID_ARG,
               "group_size=%d must be > 0 and divide cols=%d", gs, cols);
    return KC_OK;
}

// Opt a kernel into more than 48 KB of dynamic shared memory (once per device).
template <typename KernelT>
cudaError_t set_smem_once(KernelT kernel, size_t bytes) {
    static thread_local int done_dev = -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev == done_dev) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done_dev = dev;
    return e;
}

int launch_w4a16(const W4A16Params& P, cudaStream_t stream) {
    if (P.total_tiles == 0) return KC_OK;
    bool fast = (P.gs % 128 == 0);
    for (int i = 0; i < P.count && fast; ++i) {
        const W4A16Prob& p = P.p[i];
        fast = (p.K % 128 == 0) && kc::aligned(p.packed, 16) && kc::aligned(p.x, 16);
    }
    if (fast) {
        const int grid = (int)std::min<long>(P.total_tiles, kc::sm_count());
        if (P.M <= 8) {
            const size_t smem = sizeof(GemvSmem<1>);
            KC_CUDA_TRY(set_smem_once(gemv_w4a16_tma<1>, smem), "gemv smem attribute");
            gemv_w4a16_tma<1><<<grid, kGemvThreads, smem, stream>>>(P);
        } else {
            const size_t smem = sizeof(GemvSmem<2>);
            KC_CUDA_TRY(set_smem_once(gemv_w4a16_tma<2>, smem), "gemv smem attribute");
            gemv_w4a16_tma<2><<<grid, kGemvThreads, smem, stream>>>(P);
        }
    } else {
        long rows = 0;
        for (int i = 0; i < P.count; ++i) rows += P.p[i].N;
        gemv_w4a16_scalar<<<grid_for((rows + 7) / 8, 256), 256, 0, stream>>>(P);
    }
    return kc::check_launch("gemv_w4a16");
}

}  // namespace

KC_DEFINE_STATUS_READER(int4)

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int kc_dequantize_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                           float* out, int rows, int cols, int gs, cudaStream_t stream) {
    int st = check_ref_int4_args(packed, scales, zeros, out, rows, cols, gs);
    if (st) return st;
    if (rows == 0 || cols == 0) return KC_OK;
    const bool vec = (cols % 32 == 0) && (gs % 32 == 0) && kc::aligned(packed, 16) &&
                     kc::aligned(out, 16);
    if (vec) {
        const long n = (long)rows * (cols / 32);
        dequant_int4_f32_vec<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(
            packed, scales, zeros, out, rows, cols, gs);
    } else {
        const long n = (long)rows * (cols / 2);
        dequant_int4_f32_bytes<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(
            packed, scales, zeros, out, rows, cols, gs);
    }
    return kc::check_launch("dequantize_int4_f32");
}

int kc_gemv_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                     const float* x, float* y, int rows, int cols, int gs, cudaStream_t stream) {
    int st = check_ref_int4_args(packed, scales, zeros, y, rows, cols, gs);
    if (st) return st;
    KC_REQUIRE(x != nullptr, KC_ERR_INVALID_ARG, "null x");
    if (rows == 0) return KC_OK;
    const bool vec = (cols % 32 == 0) && (gs % 32 == 0) && kc::aligned(packed, 16) &&
                     kc::aligned(x, 16);
    const int grid = grid_for(((long)rows + 7) / 8, 256);
    if (vec)
        gemv_int4_f32<true><<<grid, 256, 0, stream>>>(packed, scales, zeros, x, y, rows, cols, gs);
    else
        gemv_int4_f32<false><<<grid, 256, 0, stream>>>(packed, scales, zeros, x, y, rows, cols, gs);
    return kc::check_launch("gemv_int4_f32");
}

void launch_dequantize_int4(const uint8_t* d_packed, const float* d_scales, const uint8_t* d_zeros,
                            float* d_output, int rows, int cols, int group_size,
                            cudaStream_t stream) {
    if (kc_dequantize_int4_f32(d_packed, d_scales, d_zeros, d_output, rows, cols, group_size,
                               stream) == KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_dequantize_int4 sync");
}

void launch_gemv_int4(const uint8_t* d_packed, const float* d_scales, const uint8_t* d_zeros,
                      const float* d_x, float* d_y, int rows, int cols, int group_size,
                      cudaStream_t stream) {
    if (kc_gemv_int4_f32(d_packed, d_scales, d_zeros, d_x, d_y, rows, cols, group_size, stream) ==
        KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_gemv_int4 sync");
}

int kc_dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16, uint16_t* out_bf16,
                          int N, int K, int gs, cudaStream_t stream) {
    KC_REQUIRE(packed && scales_f16 && out_bf16, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(N >= 0 && K >= 0 && K % 2 == 0, KC_ERR_INVALID_ARG, "bad shape N=%d K=%d", N, K);
    KC_REQUIRE(gs > 0 && K % gs == 0, KC_ERR_INVALID_ARG, "group_size=%d must divide K=%d", gs, K);
    if (N == 0 || K == 0) return KC_OK;
    const __half* s = reinterpret_cast<const __half*>(scales_f16);
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out_bf16);
    if (K % 32 == 0 && gs % 32 == 0 && kc::aligned(packed, 16) && kc::aligned(out_bf16, 16)) {
        const long n = (long)N * (K / 32);
        dequant_w4_bf16_vec<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, o, N, K, gs);
    } else {
        const long n = (long)N * K;
        dequant_w4_bf16_scalar<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, o, N, K, gs);
    }
    return kc::check_launch("dequantize_w4_bf16");
}

int kc_gemv_w4a16_grouped(const kc_w4a16_problem* problems, int count, int M, int gs,
                          cudaStream_t stream) {
    KC_REQUIRE(problems != nullptr, KC_ERR_INVALID_ARG, "null problem list");
    KC_REQUIRE(count >= 1 && count <= KC_W4A16_MAX_PROBLEMS, KC_ERR_INVALID_ARG,
               "count=%d outside 1..%d", count, KC_W4A16_MAX_PROBLEMS);
    KC_REQUIRE(M >= 1 && M <= 16, KC_ERR_INVALID_ARG, "M=%d outside 1..16", M);
    KC_REQUIRE(gs > 0 && gs % 2 == 0, KC_ERR_INVALID_ARG, "group_size=%d must be even and > 0", gs);
    W4A16Params P{};
    P.count = count;
    P.M = M;
    P.gs = gs;
    long tiles = 0;
    for (int i = 0; i < count; ++i) {
        const kc_w4a16_problem& q = problems[i];
        KC_REQUIRE(q.packed && q.scales_f16 && q.x_bf16 && q.y, KC_ERR_INVALID_ARG,
                   "problem %d has a null pointer", i);
        KC_REQUIRE(q.N >= 0 && q.K > 0 && q.K % 2 == 0 && q.K % gs == 0, KC_ERR_INVALID_ARG,
                   "problem %d: bad shape N=%d K=%d for group_size=%d", i, q.N, q.K, gs);
        P.p[i].packed = q.packed;
        P.p[i].scales = reinterpret_cast<const __half*>(q.scales_f16);
        P.p[i].x = reinterpret_cast<const __nv_bfloat16*>(q.x_bf16);
        P.p[i].y = q.y;
        P.p[i].N = q.N;
        P.p[i].K = q.K;
        P.p[i].tile_begin = (int)tiles;
        tiles += (q.N + 15) / 16;
    }
    KC_REQUIRE(tiles < (1L << 30), KC_ERR_INVALID_ARG, "too many rows");
    P.total_tiles = (int)tiles;
    return launch_w4a16(P, stream);
}

int kc_gemv_w4a16(const uint8_t* packed, const uint16_t* scales_f16, const uint16_t* x_bf16,
                  float* y, int M, int N, int K, int gs, cudaStream_t stream) {
    kc_w4a16_problem p{packed, scales_f16, x_bf16, y, N, K};
    return kc_gemv_w4a16_grouped(&p, 1, M, gs, stream);
}

}  // extern "C"
